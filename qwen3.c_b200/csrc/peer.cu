// Head-sharded prefill with the all-gather fused into the output kernels.
// Included at the end of backend.cu (one translation unit).
//
// Each rank's layer output block goes, from the epilogue of the kernel that
// produces it (gqa_prefill_kernel, gdn_pf_out_kernel), straight into every
// rank's gathered buffer through peer pointers: plain 16-byte stores over
// NVLink / NVSwitch, so the transfer overlaps the math instead of following it
// as an NCCL all-gather would. The buffers are cudaMalloc'd per rank and
// mapped into the other ranks with CUDA IPC; a flag array per rank (also IPC
// mapped) carries the cross-rank barrier that ends a layer: every rank stores
// its epoch into every peer's slot (release, system scope) and waits, with a
// time limit, until all peers' epochs have reached it in its own array.
// No TMA and no cluster multicast touches peer memory.

namespace {

struct PeerFlags {
    uint32_t *f[PEER_MAX];   // rank r's flag array ([world] words) as mapped here
    int world, rank;
    uint32_t epoch;
};

__global__ void peer_barrier_kernel(PeerFlags a)
{
    const int r = threadIdx.x;
    if (r < a.world) {
        // announce this rank's epoch in rank r's array (slot = this rank)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.f[r] + a.rank), "r"(a.epoch) : "memory");
        // wait until rank r has announced the same epoch in this rank's array
        const uint32_t *mine = a.f[a.rank] + r;
        const uint64_t t0 = globaltimer_ns(), lim = wait_limit_ns();
        for (uint32_t i = 0;; ++i) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if ((int32_t)(v - a.epoch) >= 0) break;
            if ((i & 63) == 63 && globaltimer_ns() - t0 > lim) {
                raise_error(1);
                break;
            }
        }
    }
    __syncthreads();
}

int gather_desc(PeerGather *g, void *const *dst, int world, int rank)
{
    if (world < 1 || world > PEER_MAX || rank < 0 || rank >= world || !dst)
        return fail("bad peer gather (world %d, rank %d)", world, rank);
    memset(g, 0, sizeof(*g));
    for (int r = 0; r < world; ++r) {
        if (!dst[r]) return fail("peer gather target %d is null", r);
        if ((uintptr_t)dst[r] & 15) return fail("peer gather target %d is not 16-byte aligned", r);
        g->dst[r] = dst[r];
    }
    g->world = world;
    g->rank = rank;
    return 1;
}

}  // namespace

extern "C" {

int coli_cuda_ipc_alloc(size_t bytes, void **dptr, void *handle)
{
    READY();
    if (!dptr || !handle || bytes == 0) return fail("bad ipc_alloc arguments");
    if (!dev_alloc(dptr, bytes)) return 0;
    CK(cudaMemset(*dptr, 0, bytes));
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, *dptr));
    memcpy(handle, &h, sizeof(h));
    return 1;
}

int coli_cuda_ipc_free(void *dptr, size_t bytes)
{
    READY();
    dev_free(dptr, bytes);
    return 1;
}

int coli_cuda_ipc_open(const void *handle, void **dptr)
{
    READY();
    if (!handle || !dptr) return fail("bad ipc_open arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    CK(cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess));
    return 1;
}

int coli_cuda_ipc_close(void *dptr)
{
    READY();
    CK(cudaIpcCloseMemHandle(dptr));
    return 1;
}

int coli_cuda_peer_barrier(void *const *flags, int world, int rank, unsigned epoch)
{
    READY();
    if (world < 1 || world > PEER_MAX || rank < 0 || rank >= world || !flags)
        return fail("bad peer barrier (world %d, rank %d)", world, rank);
    PeerFlags a;
    memset(&a, 0, sizeof(a));
    for (int r = 0; r < world; ++r) {
        if (!flags[r]) return fail("peer flag array %d is null", r);
        a.f[r] = static_cast<uint32_t *>(flags[r]);
    }
    a.world = world; a.rank = rank; a.epoch = epoch;
    peer_barrier_kernel<<<1, 32, 0, stream()>>>(a);
    CK(cudaGetLastError());
    g_launches += 1;
    return 1;
}

int coli_cuda_gqa_prefill_heads_gather_dev(int layer, int req, int S, int pos_base, const void *qg,
                                           const void *k, const void *v, void *const *dst, int world,
                                           int rank, int H, int KH, int hd, int rot, float eps,
                                           float theta, int dtype, int h0, int nh)
{
    READY();
    PeerGather g;
    if (!gather_desc(&g, dst, world, rank)) return 0;
    if (!dtype) return fail("the gathered prefill output is bf16 (dtype 1)");
    return gqa_prefill_heads(layer, req, S, pos_base, qg, k, v, dst[rank], H, KH, hd, rot, eps, theta,
                             dtype, h0, nh, &g);
}

int coli_cuda_gdn_prefill_heads_gather_dev(int layer, int req, int S, const void *qkv, const void *z,
                                           const void *a, const void *b, void *const *dst, int world,
                                           int rank, int KH, int KD, int VH, int VD, float eps,
                                           int dtype, int kh0, int nkh)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (S < GDN_CHUNK_MIN_ROWS) return fail("head-sharded GDN prefill needs S >= %d", GDN_CHUNK_MIN_ROWS);
    PeerGather g;
    if (!gather_desc(&g, dst, world, rank)) return 0;
    if (!dtype) return fail("the gathered prefill output is bf16 (dtype 1)");
    return gdn_prefill_chunked(layer, req, S, qkv, z, a, b, dst[rank], KH, KD, VH, VD, eps, dtype, kh0,
                               nkh, nullptr, &g);
}

}  // extern "C"
