// Batched GQA decode that allocates no device memory.
//
// Some callers cannot call cudaMalloc on the decode path: an engine that runs
// under a memory budget fixed at start-up, a host that forbids allocation
// once serving begins (allocation can synchronise the device and stall other
// streams), or code that must not fail half-way through a step because the
// allocator ran out. For them, coli_cuda_gqa_decode_noalloc runs the same
// three kernels as coli_cuda_gqa_decode_dev (prologue, split-KV attention,
// combine + gate) but keeps every intermediate — the normed/roped bf16 q and
// the per-split partial sums — in one fixed array in device memory that is
// part of the library image, so it never allocates and never frees.
//
// The array holds COLI_NOALLOC_SCRATCH_BYTES (8 MiB). Every GPU that loads the
// library holds it until the process exits. The host cannot pass the array's
// name to a kernel (in host code the name is a host-side stand-in, not a
// device address), so the first call on each device looks its device address
// up with cudaGetSymbolAddress while that device is current; that first call
// should therefore be made before any stream capture begins. All calls share
// the one array and it keeps the last call's contents: nothing in it has to
// start at zero (every element a call reads, the same call wrote first), and
// two calls that overlap on the GPU (different streams, no ordering between
// them) race on it.
//
// Included by backend.cu (one translation unit), after the backend state.

#define COLI_NOALLOC_SCRATCH_BYTES (8u << 20)

namespace {

__device__ __align__(256) uint8_t g_noalloc_scratch[COLI_NOALLOC_SCRATCH_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;
void *g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

// Device address of the fixed array on the current device (looked up once).
int noalloc_scratch_ptr(void **out)
{
    int dev = -1;
    CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return fail("device %d out of range", dev);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return 1;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Bytes of the fixed array one call needs for nq rows and ns splits.
size_t noalloc_bytes(int nq, int H, int KH, int hd, int ns)
{
    return align256((size_t)nq * H * hd * 2) + align256((size_t)nq * KH * ns * 8 * hd * 4) +
           align256((size_t)nq * KH * ns * 8 * 2 * 4);
}

}  // namespace

extern "C" int coli_cuda_gqa_decode_noalloc(int layer, int B, const void *qg, const void *k,
                                            const void *v, const int *pos_dev, void *ctx, int H,
                                            int KH, int hd, int rot, float eps, float theta,
                                            int dtype)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    KvLayer &L = G.kv[layer];
    if (!gqa_shape_ok(L, H, KH, hd)) return 0;
    if (!L.qnw) return fail("q/k norm weights of layer %d not set (coli_cuda_gqa_norm_weight)", layer);
    if (B < 1 || B > L.batch) return fail("batch %d beyond the cache's %d requests", B, L.batch);
    if (rot < 2 || rot > hd || (rot & 1)) return fail("bad rot %d", rot);
    if (dtype != 0 && dtype != 1) return fail("dtype must be 0 (fp32) or 1 (bf16)");

    // Fewer KV splits when the default plan would not fit the fixed array.
    int ns = gqa_pick_splits(B, KH, L.max_t, G.num_sms);
    while (ns > 1 && noalloc_bytes(B, H, KH, hd, ns) > COLI_NOALLOC_SCRATCH_BYTES) --ns;
    const size_t need = noalloc_bytes(B, H, KH, hd, ns);
    if (need > COLI_NOALLOC_SCRATCH_BYTES)
        return fail("coli_cuda_gqa_decode_noalloc: %d requests need %zu bytes of scratch, more than "
                    "the fixed %u bytes (at most %d requests per call)", B, need,
                    COLI_NOALLOC_SCRATCH_BYTES,
                    (int)(COLI_NOALLOC_SCRATCH_BYTES / noalloc_bytes(1, H, KH, hd, 1)));
    void *base = nullptr;
    if (!noalloc_scratch_ptr(&base)) return 0;
    uint8_t *p8 = static_cast<uint8_t *>(base);
    __nv_bfloat16 *q = reinterpret_cast<__nv_bfloat16 *>(p8);
    float *po = reinterpret_cast<float *>(p8 + align256((size_t)B * H * hd * 2));
    float *pml = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(po) +
                                           align256((size_t)B * KH * ns * 8 * hd * 4));

    GqaPrologueArgs pa{};
    pa.qg = qg; pa.k = k; pa.v = v; pa.qnw = L.qnw; pa.knw = L.knw; pa.pos = pos_dev; pa.creq = nullptr;
    pa.qout = q; pa.kcache = L.k; pa.vcache = L.v;
    pa.nq = B; pa.H = H; pa.KH = KH; pa.max_t = L.max_t; pa.rot = rot; pa.eps = eps; pa.theta = theta;
    CK(launch_gqa_prologue(pa, dtype, stream()));

    GqaSplitArgs sa{};
    sa.q = q; sa.pos = pos_dev; sa.creq = nullptr; sa.part_o = po; sa.part_ml = pml;
    sa.nq = B; sa.H = H; sa.KH = KH; sa.max_t = L.max_t; sa.n_splits = ns; sa.appended = 1;
    sa.chunk = gqa_chunk_for(L.max_t, ns);
    sa.scale_log2 = (1.f / sqrtf((float)hd)) * 1.4426950408889634f;
    CK(launch_gqa_split(L.tmK, L.tmV, sa, stream()));

    GqaCombineArgs ca{};
    ca.part_o = po; ca.part_ml = pml; ca.qg = qg; ca.ctx = ctx;
    ca.nq = B; ca.H = H; ca.KH = KH; ca.n_splits = ns;
    CK(launch_gqa_combine(ca, dtype, dtype, stream()));
    g_launches += 3;
    return 1;
}
