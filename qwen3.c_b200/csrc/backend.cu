// backend.cu — host side of the B200 token-mixer backend: the C ABI declared
// in include/backend_cuda.h, device-resident state (bf16 KV cache, fp32 GDN
// state and conv history), scratch, TMA descriptors and kernel launches.
//
// The library is one translation unit: the kernel sources are included below
// so device globals (the error word) need no relocatable device code.
//
// Reference counterpart: the token-mixer subset of c/backend_vulkan.c
// (KV mirror :1705-1743, GDN :1745-2157, GQA :2159-2348). The reference keeps
// one global device context `G` (c/backend_vulkan.c:69-278); so does this file.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>
#include <algorithm>

#include "../../include/backend_cuda.h"
#include "common.cuh"
#include "kernels.h"

#include "gdn_decode.cu"
#include "gqa_decode.cu"
#include "gqa_prefill.cu"
#include "gdn_prefill.cu"
#include "linear.cu"

namespace {

using namespace coli;

constexpr int MAX_LAYERS = 160;  // per-type layer slots, as the reference's VK_KV_LAYERS

// cuTensorMapEncodeTiled, fetched through the runtime's driver entry point so
// the library does not link libcuda directly.
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct KvLayer {
    __nv_bfloat16 *k = nullptr, *v = nullptr;
    int batch = 0, KH = 0, max_t = 0, hd = 0;
    CUtensorMap tmK, tmV;      // 16-row boxes (decode)
    CUtensorMap tmK64, tmV64;  // 128-row boxes (prefill key tiles)
    float *qnw = nullptr, *knw = nullptr;  // [hd] resident norm weights
};

struct GdnLayer {
    float *state = nullptr;  // [batch][VH][KD][VD]
    int batch = 0, VH = 0, KD = 0, VD = 0;
    float *hist = nullptr;   // [hbatch][conv_k-1][conv_dim]
    int hbatch = 0, conv_k = 0, conv_dim = 0;
    float *conv_w = nullptr;                         // [conv_dim][conv_k]
    float *A_log = nullptr, *dt_bias = nullptr, *gnorm = nullptr;
    int pVH = 0, pVD = 0;
};

// Grow-only device scratch slots (activations staging, partials, indices).
enum Slot { S_IN0, S_IN1, S_IN2, S_IN3, S_OUT, S_Q, S_PO, S_PML, S_POS, S_CREQ, S_P0, S_P1, S_P2,
            S_GQ, S_GK, S_GKT, S_GV, S_GL, S_GB, S_GW, S_GU, S_GM, S_GDT, S_GQH, S_GHS, S_GXS,
            S_XB, S_PQ, S_PK, S_PV, S_PCTX, S_PY2, S_LPART, S_PAR, S_PY, S_RX, S_RXO, S_RN, S_RNB, S_RP, S_LCNT, S_COUNT };

struct Global {
    int ready = 0;
    int device = -1;
    int num_sms = 148;
    cudaStream_t stream = nullptr;     // backend's own stream
    // host-buffer decode: the gate half of q|gate is uploaded on this stream
    // while the kernels run (created at the first such call)
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_gate = nullptr;
    cudaStream_t user_stream = nullptr;
    bool user_stream_set = false;
    KvLayer kv[MAX_LAYERS];
    GdnLayer gdn[MAX_LAYERS];
    void *slot[S_COUNT] = {};
    size_t slot_bytes[S_COUNT] = {};
    size_t bytes = 0, tensors = 0;
    float *ln_w[MAX_LAYERS] = {};      // per model layer: [in_ln(D) | post_ln(D)] (route tail)
    int ln_D[MAX_LAYERS] = {};
    char err[512] = "not initialised";
    EncodeTiledFn encode = nullptr;
};
Global G;

// ---------------------------------------------------------------- kernel timer
struct KTimer {
    bool on = false;
    std::vector<cudaEvent_t> ev[COLI_K_COUNT];  // start/stop pairs, pending
    std::vector<cudaEvent_t> pool;
};
KTimer KT;
long long g_launches = 0;

cudaEvent_t kt_event()
{
    if (!KT.pool.empty()) { cudaEvent_t e = KT.pool.back(); KT.pool.pop_back(); return e; }
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
}
void kt_mark(int k)  // call before and after the launch of kernel k
{
    if (!KT.on) return;
    cudaEvent_t e = kt_event();
    cudaEventRecord(e, G.user_stream_set ? G.user_stream : G.stream);
    KT.ev[k].push_back(e);
}

// The device error word as read by the last download(), valid until the next
// stream() use (any later launch or copy may raise it again).
int g_err_host = 0;
bool g_err_fresh = false;
// Pinned landing word for that read (a pageable destination is a staged,
// slower copy on every host-buffer call); null if it could not be allocated.
int *g_err_pin = nullptr;

cudaStream_t stream()
{
    g_err_fresh = false;
    return G.user_stream_set ? G.user_stream : G.stream;
}

int fail(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(G.err, sizeof(G.err), fmt, ap);
    va_end(ap);
    return 0;
}

// A CUDA error from a launch or copy: record it and, if it is sticky, mark
// the backend dead so every later call returns 0 (reference: G.ready = 0).
int cuda_fail(cudaError_t e, const char *what)
{
    fail("%s: %s", what, cudaGetErrorString(e));
    cudaError_t again = cudaPeekAtLastError();
    if (again != cudaSuccess && again == e && e != cudaErrorInvalidValue &&
        e != cudaErrorMemoryAllocation)
        G.ready = 0;
    if (e == cudaErrorIllegalAddress || e == cudaErrorLaunchFailure || e == cudaErrorIllegalInstruction ||
        e == cudaErrorMisalignedAddress || e == cudaErrorHardwareStackError)
        G.ready = 0;
    return 0;
}
#define CK(call)                                                   \
    do {                                                           \
        cudaError_t e_ = (call);                                   \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);        \
    } while (0)
#define READY()                                                    \
    do {                                                           \
        if (!G.ready) return fail("backend not ready: %s", G.err); \
    } while (0)

int g_fail_alloc_after = -1;   // test hook: allocations left before one is refused (-1 = off)

int dev_alloc(void **p, size_t bytes)
{
    if (g_fail_alloc_after == 0) {
        g_fail_alloc_after = -1;
        *p = nullptr;
        return fail("cudaMalloc(%zu): refused by the allocation-failure test hook", bytes);
    }
    if (g_fail_alloc_after > 0) --g_fail_alloc_after;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) { *p = nullptr; cudaGetLastError(); return fail("cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e)); }
    G.bytes += bytes;
    G.tensors += 1;
    return 1;
}
void dev_free(void *p, size_t bytes)
{
    if (!p) return;
    cudaFree(p);
    G.bytes -= bytes;
    G.tensors -= 1;
}

void *scratch(Slot s, size_t bytes)
{
    if (G.slot_bytes[s] >= bytes) return G.slot[s];
    if (G.slot[s]) {
        cudaStreamSynchronize(stream());
        dev_free(G.slot[s], G.slot_bytes[s]);
        G.slot[s] = nullptr;
        G.slot_bytes[s] = 0;
    }
    size_t want = bytes < 4096 ? 4096 : bytes;
    if (!dev_alloc(&G.slot[s], want)) return nullptr;
    G.slot_bytes[s] = want;
    return G.slot[s];
}

int check_layer(int layer) { return layer >= 0 && layer < MAX_LAYERS; }

int make_kv_tmap(CUtensorMap *m, void *base, int rows, int hd, int box_rows = 16)
{
    cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = G.encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 1;
}

// Roped bf16 q [S][H][hd] as a 3D map (d, head, row) with 64 x 1 x 128 boxes.
int make_q_tmap(CUtensorMap *m, void *base, int S, int H, int hd)
{
    cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)H, (cuuint64_t)S};
    cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)H * hd * 2};
    cuuint32_t box[3] = {64, 1, 128};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = G.encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled (q) failed (%d)", (int)r);
    return 1;
}

// Maps of the prefill kernel's TMA epilogue: gate = the second half of each
// head's 2 hd values in qg [S][Hin][2 hd], ctx [S][H][hd]; 64 x 1 x 128 boxes.
int make_pf_epi_maps(PfEpiMaps *em, const void *qg, void *ctx, int S, int H, int Hin, int hd)
{
    if (!make_q_tmap(&em->ctx, ctx, S, H, hd)) return 0;
    cuuint64_t dims[3] = {(cuuint64_t)(2 * hd), (cuuint64_t)Hin, (cuuint64_t)S};
    cuuint64_t strides[2] = {(cuuint64_t)2 * hd * 2, (cuuint64_t)Hin * 2 * hd * 2};
    cuuint32_t box[3] = {64, 1, 128};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = G.encode(&em->gate, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(qg), dims, strides,
                          box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled (gate) failed (%d)", (int)r);
    return 1;
}

// fp32 host -> device staging (optionally converted to bf16 by the kernels'
// templated loads; the host API keeps fp32 end to end for parity).
void *upload(Slot s, const void *host, size_t bytes)
{
    void *d = scratch(s, bytes);
    if (!d) return nullptr;
    if (cudaMemcpyAsync(d, host, bytes, cudaMemcpyHostToDevice, stream()) != cudaSuccess) {
        cuda_fail(cudaGetLastError(), "cudaMemcpyAsync H2D");
        return nullptr;
    }
    return d;
}

// The result and the device error word come back in one synchronisation.
int download(void *host, const void *dev, size_t bytes)
{
    cudaStream_t st = stream();
    CK(cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyFromSymbolAsync(g_err_pin ? g_err_pin : &g_err_host, g_dev_error, sizeof(int), 0,
                                 cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (g_err_pin) g_err_host = *g_err_pin;
    g_err_fresh = true;
    return 1;
}

int check_dev_error()
{
    int h = 0;
    if (g_err_fresh) {   // read by the download that just finished, nothing launched since
        h = g_err_host;
        g_err_fresh = false;
    } else {
        cudaStream_t st = stream();
        CK(cudaMemcpyFromSymbolAsync(&h, g_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
    }
    if (h) {
        G.ready = 0;
        return fail("device error word %d (%s)", h, h == 1 ? "pipeline wait timed out" : "kernel fault");
    }
    return 1;
}

__global__ void iota_kernel(int *pos, int *creq, int n, int base, int req)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) { pos[i] = base + i; creq[i] = req; }
}

__global__ void split_q_kernel(const float *q, __nv_bfloat16 *out, int n_heads_total, int hd)
{
    // roped q | gate rows -> bf16 q (first hd of every head)
    const int i = blockIdx.x, d = threadIdx.x;
    if (i < n_heads_total) out[(size_t)i * hd + d] = __float2bfloat16_rn(q[(size_t)i * 2 * hd + d]);
}

// ---------------------------------------------------------------- GQA core
// Runs split-KV attention + combine for nq query rows whose roped bf16 q is
// in S_Q, positions in pos_d, cache requests in creq_d (nullable).
int gqa_attend(KvLayer &L, int nq, int H, const int *pos_d, const int *creq_d, int tmax,
               const void *qg_gate, void *ctx, int in_bf16, int out_bf16, float scale,
               cudaEvent_t gate_ready = nullptr, const GqaPrologueArgs *fused = nullptr)
{
    const int ns = gqa_pick_splits(nq, L.KH, tmax, G.num_sms);
    const int chunk = gqa_chunk_for(tmax, ns);
    float *po = (float *)scratch(S_PO, (size_t)nq * L.KH * ns * 8 * 256 * 4);
    float *pml = (float *)scratch(S_PML, (size_t)nq * L.KH * ns * 8 * 2 * 4);
    if (!po || !pml) return 0;
    GqaSplitArgs sa{};
    sa.q = (const __nv_bfloat16 *)G.slot[S_Q];
    sa.pos = pos_d;
    sa.creq = creq_d;
    sa.part_o = po;
    sa.part_ml = pml;
    sa.nq = nq; sa.H = H; sa.KH = L.KH; sa.max_t = L.max_t; sa.n_splits = ns; sa.chunk = chunk;
    // batched decode appends one row per request; the S rows of one request
    // (creq given) append up to S rows ending at each query row's position
    sa.appended = creq_d ? nq : 1;
    sa.scale_log2 = scale * 1.4426950408889634f;
    if (fused) {   // the split kernel does the prologue's work (small-batch decode)
        sa.fuse = in_bf16 ? 1 : 2;
        sa.pro = *fused;
    }
    kt_mark(COLI_K_GQA_SPLIT);
    CK(launch_gqa_split(L.tmK, L.tmV, sa, stream()));
    kt_mark(COLI_K_GQA_SPLIT);
    GqaCombineArgs ca{};
    ca.part_o = po; ca.part_ml = pml; ca.qg = qg_gate; ca.ctx = ctx;
    ca.nq = nq; ca.H = H; ca.KH = L.KH; ca.n_splits = ns;
    if (gate_ready) CK(cudaStreamWaitEvent(stream(), gate_ready, 0));   // the gate reads come last
    kt_mark(COLI_K_GQA_COMBINE);
    CK(launch_gqa_combine(ca, in_bf16, out_bf16, stream()));
    kt_mark(COLI_K_GQA_COMBINE);
    g_launches += 2;
    return 1;
}

// A one-request cache may have been declared as plain rows (KH = 1, max_t =
// KH * max_t: what coli_vk_kv_ensure(layer, KH*max_t, hd, hd) passes, which
// names no head count). Row kh*max_t + pos is the same address under either
// split, so the first call that names (KH, max_t) with the same row count
// adopts that split; the tensor maps cover all rows and stay valid.
void kv_adopt_split(KvLayer &L, int KH, int max_t)
{
    if (L.k && L.batch == 1 && KH > 0 && max_t > 0 && L.KH != KH && (long long)L.KH * L.max_t == (long long)KH * max_t) {
        L.KH = KH;
        L.max_t = max_t;
    }
}

int gqa_shape_ok(KvLayer &L, int H, int KH, int hd)
{
    if (!L.k) return fail("KV cache of this layer not allocated (coli_cuda_kv_ensure)");
    if (hd != 256 || KH != L.KH || hd != L.hd || H != 8 * KH)
        return fail("unsupported GQA shape H=%d KH=%d hd=%d (needs hd=256, H=8*KH, cache KH=%d)", H, KH, hd, L.KH);
    return 1;
}

constexpr int PREFILL_MIN_ROWS = 64;
constexpr int GQA_FUSE_MAX_ROWS = 8;   // decode batches up to this size use the fused split kernel (1: -13 % per step; 16: no gain measured)
int gqa_prefill_rows(KvLayer &L, int req, int S, int pos_base, int H, const void *qg, void *ctx,
                     int in_bf16, int out_bf16, float scale);

// prologue + attention for nq rows (pos_d/creq_d on device)
int gqa_rows(int layer, int nq, const void *qg, const void *k, const void *v, const int *pos_d,
             const int *creq_d, int tmax, void *ctx, int H, int KH, int hd, int rot, float eps,
             float theta, int in_bf16, int out_bf16, int prefill_req = -1, int pos_base = 0,
             cudaEvent_t gate_ready = nullptr)
{
    KvLayer &L = G.kv[layer];
    if (!gqa_shape_ok(L, H, KH, hd)) return 0;
    if (!L.qnw) return fail("q/k norm weights of layer %d not set (coli_cuda_gqa_norm_weight)", layer);
    if (rot < 2 || rot > hd || (rot & 1)) return fail("bad rot %d", rot);
    if (tmax > L.max_t) return fail("position %d beyond max_t %d", tmax - 1, L.max_t);
    __nv_bfloat16 *q = (__nv_bfloat16 *)scratch(S_Q, (size_t)nq * H * hd * 2);
    if (!q) return 0;
    GqaPrologueArgs pa{};
    pa.qg = qg; pa.k = k; pa.v = v; pa.qnw = L.qnw; pa.knw = L.knw; pa.pos = pos_d; pa.creq = creq_d;
    pa.qout = q; pa.kcache = L.k; pa.vcache = L.v;
    pa.nq = nq; pa.H = H; pa.KH = KH; pa.max_t = L.max_t; pa.rot = rot; pa.eps = eps; pa.theta = theta;
    // Small-batch decode (one appended row per query row: a batch of
    // requests, or a single row of one request; 16-byte aligned operands):
    // the split kernel norms / ropes q and appends the k / v rows itself, one
    // launch and one dependent wait fewer on a latency-bound step.
    const uintptr_t al = (uintptr_t)qg | (uintptr_t)k | (uintptr_t)v | (uintptr_t)L.qnw | (uintptr_t)L.knw |
                         (uintptr_t)L.k | (uintptr_t)L.v;
    const bool fuse = (nq == 1 || (!creq_d && prefill_req < 0)) && nq <= GQA_FUSE_MAX_ROWS && (al & 15) == 0;
    if (!fuse) {
        CK(launch_gqa_prologue(pa, in_bf16, stream()));
        g_launches += 1;
    }
    if (prefill_req >= 0 && nq >= PREFILL_MIN_ROWS)
        return gqa_prefill_rows(L, prefill_req, nq, pos_base, H, qg, ctx, in_bf16, out_bf16,
                                1.f / sqrtf((float)hd));
    return gqa_attend(L, nq, H, pos_d, creq_d, tmax, qg, ctx, in_bf16, out_bf16, 1.f / sqrtf((float)hd),
                      gate_ready, fuse ? &pa : nullptr);
}

// Causal prefill of S rows of one request on the tensor cores; the roped bf16
// q is already in S_Q and the new K/V rows are in the cache.
int gqa_prefill_rows(KvLayer &L, int req, int S, int pos_base, int H, const void *qg, void *ctx,
                     int in_bf16, int out_bf16, float scale)
{
    CUtensorMap tq;
    if (!make_q_tmap(&tq, G.slot[S_Q], S, H, L.hd)) return 0;
    GqaPrefillArgs a{};
    a.qg = qg; a.ctx = ctx; a.S = S; a.H = H; a.KH = L.KH; a.max_t = L.max_t; a.req = req;
    a.pos_base = pos_base; a.n_qtiles = (S + 127) / 128; a.scale_log2 = scale * 1.4426950408889634f;
    PfEpiMaps em;
    const bool tma_epi = in_bf16 && out_bf16;
    if (tma_epi && !make_pf_epi_maps(&em, qg, ctx, S, H, H, L.hd)) return 0;
    kt_mark(COLI_K_GQA_PREFILL);
    CK(launch_gqa_prefill(tq, L.tmK64, L.tmV64, a, in_bf16, out_bf16, stream(), tma_epi ? &em : nullptr));
    kt_mark(COLI_K_GQA_PREFILL);
    g_launches += 1;
    return 1;
}

// ---------------------------------------------------------------- GDN helpers
int gdn_shape_ok(GdnLayer &L, int KH, int KD, int VH, int VD, int need_conv)
{
    if (!L.state) return fail("GDN state of this layer not allocated (coli_cuda_gdn_state_ensure)");
    if (KD != 128 || VD != 128 || VH != 2 * KH || VH != L.VH || KD != L.KD || VD != L.VD)
        return fail("unsupported GDN shape KH=%d KD=%d VH=%d VD=%d", KH, KD, VH, VD);
    if (need_conv) {
        if (!L.hist || !L.conv_w) return fail("GDN conv history/weights not set for this layer");
        if (L.conv_k != 4 || L.conv_dim != 2 * KH * KD + VH * VD) return fail("GDN conv geometry mismatch");
    }
    return 1;
}

int gdn_decode_run(int layer, int B, int req0, const void *qkv, const void *z, const void *a,
                   const void *b, void *y, int KH, int KD, int VH, int VD, float eps, int bf16,
                   const float *pdecay = nullptr, const float *pbeta = nullptr, const float *pgnorm = nullptr)
{
    GdnLayer &L = G.gdn[layer];
    if (!gdn_shape_ok(L, KH, KD, VH, VD, 1)) return 0;
    if (req0 < 0 || req0 + B > L.batch || req0 + B > L.hbatch) return fail("request range beyond the allocated batch");
    GdnDecodeArgs ga;
    memset(&ga, 0, sizeof(ga));
    ga.qkv = qkv; ga.z = z; ga.a = a; ga.b = b;
    ga.conv_w = L.conv_w; ga.A_log = L.A_log; ga.dt_bias = L.dt_bias; ga.gnorm = L.gnorm;
    ga.pdecay = pdecay; ga.pbeta = pbeta;
    if (pgnorm) ga.gnorm = pgnorm;
    // gates from a / b need the layer's A_log / dt_bias; engine-packed params
    // (decay | beta | gnorm) carry everything
    if ((!pdecay && !L.A_log) || (!pgnorm && !L.gnorm))
        return fail("GDN A_log/dt_bias/gnorm not set (coli_cuda_gdn_params)");
    ga.hist = L.hist + (size_t)req0 * 3 * L.conv_dim;
    ga.state = L.state + (size_t)req0 * VH * KD * VD;
    ga.y = y;
    ga.B = B; ga.KH = KH; ga.KD = KD; ga.VH = VH; ga.VD = VD; ga.eps = eps;
    kt_mark(COLI_K_GDN_DECODE);
    CK(launch_gdn_decode(ga, bf16, bf16, 0, stream()));
    kt_mark(COLI_K_GDN_DECODE);
    g_launches += 1;
    return 1;
}

int make_f32_3d(CUtensorMap *m, void *base, int d0, int d1, int d2, int box0, int box1)
{
    cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
    cuuint64_t strides[2] = {(cuuint64_t)d0 * 4, (cuuint64_t)d0 * d1 * 4};
    cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = G.encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled (fp32 3d) failed (%d)", (int)r);
    return 1;
}

// Chunk-parallel GDN prefill (gdn_prefill.cu) for S >= GDN_CHUNK_MIN_ROWS.
constexpr int GDN_CHUNK_MIN_ROWS = 64;
int gdn_prefill_chunked(int layer, int req, int S, const void *qkv, const void *z, const void *a,
                        const void *b, void *y, int KHin, int KD, int VHin, int VD, float eps,
                        int dtype, int kh0 = 0, int nkh = -1, const float *params = nullptr,
                        const PeerGather *gather = nullptr)
{
    GdnLayer &L = G.gdn[layer];
    if (nkh < 0) nkh = KHin;
    const int KH = nkh, VH = 2 * nkh;  // heads this call owns
    if (!L.state || L.VH != VH || L.KD != KD || L.VD != VD || KD != 128 || VD != 128 || VHin != 2 * KHin)
        return fail("GDN state/shape mismatch (state VH=%d, owned VH=%d)", L.VH, VH);
    if (kh0 < 0 || kh0 + nkh > KHin) return fail("bad K head range");
    if (!L.hist || !L.conv_w || L.conv_k != 4 || L.conv_dim != 2 * KHin * KD + VHin * VD)
        return fail("GDN conv history/weights not set for this layer");
    if (!params && (!L.A_log || L.pVH != VHin)) return fail("GDN A_log/dt_bias/gnorm not set for %d V heads", VHin);
    if (req < 0 || req >= L.batch || req >= L.hbatch) return fail("request out of range");
    const int nch = (S + 63) / 64;
    GdnPrefillArgs p;
    memset(&p, 0, sizeof(p));
    p.qkv = qkv; p.z = z; p.a = a; p.b = b;
    p.conv_w = L.conv_w; p.A_log = L.A_log; p.dt_bias = L.dt_bias; p.gnorm = L.gnorm;
    if (params) {   // rows [decay(VHin) | beta(VHin) | gnorm(VD)]; gnorm from the first row
        p.params = params; p.pstride = 2 * VHin + VD; p.gnorm = params + 2 * VHin;
    }
    p.hist = L.hist + (size_t)req * 3 * L.conv_dim;
    p.state = L.state + (size_t)req * VH * KD * VD;
    p.y = y;
    p.Qh = (float *)scratch(S_GQ, (size_t)KH * S * 128 * 4);
    p.Kh = (float *)scratch(S_GK, (size_t)KH * S * 128 * 4);
    p.KT = (float *)scratch(S_GKT, (size_t)KH * nch * 64 * 128 * 4);
    p.VT = (float *)scratch(S_GV, (size_t)VH * nch * 64 * 128 * 4);
    p.GL = (float *)scratch(S_GL, (size_t)VH * S * 4);
    p.BETA = (float *)scratch(S_GB, (size_t)VH * S * 4);
    p.W = (float *)scratch(S_GW, (size_t)nch * VH * 64 * 128 * 4);
    p.U = (float *)scratch(S_GU, (size_t)nch * VH * 64 * 128 * 4);
    p.M = (float *)scratch(S_GM, (size_t)nch * VH * 64 * 64 * 4);
    p.Dt = (float *)scratch(S_GDT, (size_t)nch * VH * 128 * 64 * 4);
    p.QH = (float *)scratch(S_GQH, (size_t)nch * VH * 64 * 128 * 4);
    // Few heads per GPU leave the sequential chunk walk latency bound: split it
    // into segments when the segment-map pass (4 CTAs per head and segment)
    // still fits one wave.
    int nseg = 1;
    const int maxseg = 1 + G.num_sms / (4 * VH);
    if (maxseg >= 3) nseg = std::min(maxseg, nch / 8);
    if (nseg < 3) nseg = 1;
    p.seglen = (nch + nseg - 1) / nseg;
    p.nseg = (nch + p.seglen - 1) / p.seglen;
    if (p.nseg > 1) {
        p.Hs = (float *)scratch(S_GHS, (size_t)p.nseg * VH * 128 * 128 * 4);
        p.XS = (float *)scratch(S_GXS, (size_t)(p.nseg - 1) * VH * 128 * 256 * 4);
        if (!p.Hs || !p.XS) return 0;
    }
    if (!p.Qh || !p.Kh || !p.KT || !p.VT || !p.GL || !p.BETA || !p.W || !p.U || !p.M || !p.Dt || !p.QH) return 0;
    p.S = S; p.KH = KH; p.VH = VH; p.eps = eps;
    p.kh0 = kh0; p.KHin = KHin; p.VHin = VHin;
    if (gather) {
        p.gather = *gather;
        p.gather.block = (long long)S * VH * VD;
    }
    GdnPrefillMaps m;
    if (!make_f32_3d(&m.Q, p.Qh, 128, S, KH, 32, 64) || !make_f32_3d(&m.K, p.Kh, 128, S, KH, 32, 64) ||
        !make_f32_3d(&m.V, p.VT, 64, 128, nch * VH, 32, 128) ||
        !make_f32_3d(&m.W, p.W, 128, 64, nch * VH, 32, 64) ||
        !make_f32_3d(&m.M, p.M, 64, 64, nch * VH, 32, 64) ||
        !make_f32_3d(&m.U, p.U, 128, 64, nch * VH, 32, 64) ||
        !make_f32_3d(&m.Dt, p.Dt, 64, 128, nch * VH, 32, 128) ||
        !make_f32_3d(&m.KT, p.KT, 64, 128, nch * KH, 32, 128))
        return 0;
    kt_mark(COLI_K_GDN_PREFILL);
    CK(launch_gdn_prefill(p, m, dtype, stream()));
    kt_mark(COLI_K_GDN_PREFILL);
    g_launches += 5 + (p.nseg > 1 ? 2 : 0);
    return 1;
}

}  // namespace

// =================================================================== C ABI
extern "C" {

int coli_cuda_init(int device)
{
    if (G.ready && G.device == device) return 1;
    if (G.ready) coli_cuda_shutdown();
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n <= device || device < 0) {
        cudaGetLastError();
        return fail("no CUDA device %d (%s)", device, e == cudaSuccess ? "count too small" : cudaGetErrorString(e));
    }
    CK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail("device %d is sm_%d%d; this backend is built for sm_100a only", device, prop.major, prop.minor);
    G.num_sms = prop.multiProcessorCount;
    CK(cudaStreamCreateWithFlags(&G.stream, cudaStreamNonBlocking));
    if (!g_err_pin && cudaHostAlloc((void **)&g_err_pin, sizeof(int), cudaHostAllocDefault) != cudaSuccess) {
        g_err_pin = nullptr;   // the pageable word serves
        cudaGetLastError();
    }
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (!fn || q != cudaDriverEntryPointSuccess) return fail("cuTensorMapEncodeTiled entry point not found");
    G.encode = (EncodeTiledFn)fn;
    int zero = 0;
    CK(cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(int)));
    G.device = device;
    G.ready = 1;
    snprintf(G.err, sizeof(G.err), "ok");
    return 1;
}

void coli_cuda_shutdown(void)
{
    if (G.device < 0) return;
    cudaSetDevice(G.device);
    cudaDeviceSynchronize();
    coli_cuda_kv_reset();
    for (int i = 0; i < MAX_LAYERS; ++i) {
        GdnLayer &L = G.gdn[i];
        dev_free(L.state, (size_t)L.batch * L.VH * L.KD * L.VD * 4);
        dev_free(L.hist, (size_t)L.hbatch * (L.conv_k - 1) * L.conv_dim * 4);
        dev_free(L.conv_w, (size_t)L.conv_dim * L.conv_k * 4);
        dev_free(L.A_log, (size_t)(2 * L.pVH + L.pVD) * 4);
        L = GdnLayer();
    }
    for (int i = 0; i < MAX_LAYERS; ++i) {
        dev_free(G.ln_w[i], (size_t)2 * G.ln_D[i] * 4);
        G.ln_w[i] = nullptr;
        G.ln_D[i] = 0;
    }
    for (int s = 0; s < S_COUNT; ++s) {
        dev_free(G.slot[s], G.slot_bytes[s]);
        G.slot[s] = nullptr;
        G.slot_bytes[s] = 0;
    }
    if (G.stream) cudaStreamDestroy(G.stream);
    G.stream = nullptr;
    if (G.copy_stream) {
        cudaStreamDestroy(G.copy_stream);
        cudaEventDestroy(G.ev_fork);
        cudaEventDestroy(G.ev_gate);
    }
    G.copy_stream = nullptr;
    G.ev_fork = G.ev_gate = nullptr;
    if (g_err_pin) cudaFreeHost(g_err_pin);
    g_err_pin = nullptr;
    G.user_stream_set = false;
    G.ready = 0;
    G.device = -1;
    snprintf(G.err, sizeof(G.err), "shut down");
}

int coli_cuda_ktimer_enable(int on)
{
    READY();
    KT.on = on != 0;
    return 1;
}

int coli_cuda_ktimer_read(int kernel, double *total_ms, int *launches)
{
    READY();
    if (kernel < 0 || kernel >= COLI_K_COUNT) return fail("bad kernel id %d", kernel);
    CK(cudaStreamSynchronize(stream()));
    double tot = 0.0;
    std::vector<cudaEvent_t> &v = KT.ev[kernel];
    const int n = (int)v.size() / 2;
    for (int i = 0; i < n; ++i) {
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, v[2 * i], v[2 * i + 1]));
        tot += ms;
    }
    for (cudaEvent_t e : v) KT.pool.push_back(e);
    v.clear();
    if (total_ms) *total_ms = tot;
    if (launches) *launches = n;
    return 1;
}

long long coli_cuda_launch_count(void) { return g_launches; }

int coli_cuda_available(void) { return G.ready; }
int coli_cuda_gdn_available(void) { return G.ready; }
int coli_cuda_gqa_available(void) { return G.ready; }
int coli_cuda_gqa_full_available(void) { return G.ready; }
int coli_cuda_gdn_full_available(void) { return G.ready; }

void coli_cuda_mem_info(size_t *used_bytes, size_t *tensor_count)
{
    if (used_bytes) *used_bytes = G.bytes;
    if (tensor_count) *tensor_count = G.tensors;
}

const char *coli_cuda_last_error(void) { return G.err; }

int coli_cuda_set_wait_limit(unsigned long long ns)
{
    READY();
    const unsigned long long v = ns ? ns : COLI_WAIT_NS;
    CK(cudaMemcpyToSymbol(g_wait_ns, &v, sizeof(v)));
    return 1;
}

void coli_cuda_debug_fail_alloc(int n) { g_fail_alloc_after = n; }

#ifdef COLI_SCAN_PROBE
// development builds only: the chunk-walk timing probe (see gdn_prefill.cu)
int coli_cuda_debug_scan_probe(long long *out, int n)
{
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpyFromSymbol(out, coli::g_scan_probe, sizeof(long long) * (size_t)(n < 8192 ? n : 8192)));
    return 1;
}
int coli_cuda_debug_lin_probe(unsigned long long *out, int n)
{
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpyFromSymbol(out, coli::g_lin_probe, sizeof(unsigned long long) * (size_t)(n < 8192 ? n : 8192)));
    return 1;
}
int coli_cuda_debug_prep_probe(long long *out)
{
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpyFromSymbol(out, coli::g_prep_probe, sizeof(long long) * 32));
    return 1;
}
#endif

int coli_cuda_sync(void)
{
    READY();
    CK(cudaStreamSynchronize(stream()));
    return check_dev_error();
}

void *coli_cuda_get_stream(void) { return (void *)stream(); }

int coli_cuda_set_stream(void *s)
{
    READY();
    G.user_stream = (cudaStream_t)s;
    G.user_stream_set = s != nullptr;
    return 1;
}

// ------------------------------------------------------------------ KV cache
int coli_cuda_kv_ensure(int layer, int batch, int KH, int max_t, int hd)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (batch < 1 || KH < 1 || max_t < 1 || hd != 256) return fail("bad KV geometry");
    KvLayer &L = G.kv[layer];
    if (L.k && L.batch == batch && L.KH == KH && L.max_t == max_t && L.hd == hd) return 1;
    if (L.k) {
        CK(cudaStreamSynchronize(stream()));
        size_t old = (size_t)L.batch * L.KH * L.max_t * L.hd * 2;
        dev_free(L.k, old);
        dev_free(L.v, old);
        L.k = L.v = nullptr;
    }
    size_t bytes = (size_t)batch * KH * max_t * hd * 2;
    if (!dev_alloc((void **)&L.k, bytes)) return 0;
    if (!dev_alloc((void **)&L.v, bytes)) { dev_free(L.k, bytes); L.k = nullptr; return 0; }
    CK(cudaMemsetAsync(L.k, 0, bytes, stream()));
    CK(cudaMemsetAsync(L.v, 0, bytes, stream()));
    L.batch = batch; L.KH = KH; L.max_t = max_t; L.hd = hd;
    if (!make_kv_tmap(&L.tmK, L.k, batch * KH * max_t, hd)) return 0;
    if (!make_kv_tmap(&L.tmV, L.v, batch * KH * max_t, hd)) return 0;
    if (!make_kv_tmap(&L.tmK64, L.k, batch * KH * max_t, hd, 128)) return 0;
    if (!make_kv_tmap(&L.tmV64, L.v, batch * KH * max_t, hd, 128)) return 0;
    return 1;
}

static int kv_rows_impl(int layer, int req, int row0, int n, const float *k, const float *v, int read)
{
    READY();
    if (!check_layer(layer) || !G.kv[layer].k) return fail("KV layer %d not allocated", layer);
    KvLayer &L = G.kv[layer];
    if (req < 0 || req >= L.batch || row0 < 0 || n < 0 || row0 + n > L.KH * L.max_t) return fail("KV row range out of bounds");
    if (n == 0) return 1;
    const size_t base = ((size_t)req * L.KH * L.max_t + row0) * L.hd;
    const size_t cnt = (size_t)n * L.hd;
    std::vector<__nv_bfloat16> tmp(cnt);
    for (int which = 0; which < 2; ++which) {
        __nv_bfloat16 *dst = (which ? L.v : L.k) + base;
        float *hp = const_cast<float *>(which ? v : k);
        if (!hp) continue;
        if (read) {
            CK(cudaMemcpyAsync(tmp.data(), dst, cnt * 2, cudaMemcpyDeviceToHost, stream()));
            CK(cudaStreamSynchronize(stream()));
            for (size_t i = 0; i < cnt; ++i) hp[i] = __bfloat162float(tmp[i]);
        } else {
            for (size_t i = 0; i < cnt; ++i) tmp[i] = __float2bfloat16_rn(hp[i]);
            CK(cudaMemcpyAsync(dst, tmp.data(), cnt * 2, cudaMemcpyHostToDevice, stream()));
            CK(cudaStreamSynchronize(stream()));
        }
    }
    return 1;
}

int coli_cuda_kv_row(int layer, int req, int row, const float *k, const float *v)
{
    return kv_rows_impl(layer, req, row, 1, k, v, 0);
}
int coli_cuda_kv_rows(int layer, int req, int row0, int n, const float *k, const float *v)
{
    return kv_rows_impl(layer, req, row0, n, k, v, 0);
}
int coli_cuda_kv_read(int layer, int req, int row0, int n, float *k, float *v)
{
    return kv_rows_impl(layer, req, row0, n, k, v, 1);
}

__global__ void rows_to_bf16_kernel(const void *src, __nv_bfloat16 *dst, size_t n, int bf16)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = bf16 ? static_cast<const __nv_bfloat16 *>(src)[i]
                      : __float2bfloat16_rn(static_cast<const float *>(src)[i]);
}

int coli_cuda_kv_rows_dev(int layer, int req, int row0, int n, const void *k, const void *v, int dtype)
{
    READY();
    if (!check_layer(layer) || !G.kv[layer].k) return fail("KV layer %d not allocated", layer);
    KvLayer &L = G.kv[layer];
    if (req < 0 || req >= L.batch || row0 < 0 || n < 0 || row0 + n > L.KH * L.max_t) return fail("KV row range out of bounds");
    if (n == 0) return 1;
    const size_t base = ((size_t)req * L.KH * L.max_t + row0) * L.hd;
    const size_t cnt = (size_t)n * L.hd;
    const int blocks = (int)((cnt + 255) / 256 < 4096 ? (cnt + 255) / 256 : 4096);
    if (k) { rows_to_bf16_kernel<<<blocks, 256, 0, stream()>>>(k, L.k + base, cnt, dtype); CK(cudaGetLastError()); }
    if (v) { rows_to_bf16_kernel<<<blocks, 256, 0, stream()>>>(v, L.v + base, cnt, dtype); CK(cudaGetLastError()); }
    g_launches += (k != nullptr) + (v != nullptr);
    return 1;
}

void coli_cuda_kv_reset(void)
{
    if (G.device >= 0) cudaStreamSynchronize(stream());
    for (int i = 0; i < MAX_LAYERS; ++i) {
        KvLayer &L = G.kv[i];
        size_t bytes = (size_t)L.batch * L.KH * L.max_t * L.hd * 2;
        dev_free(L.k, bytes);
        dev_free(L.v, bytes);
        dev_free(L.qnw, (size_t)2 * L.hd * 4);
        L = KvLayer();
    }
}

int coli_cuda_kv_device_ptr(int layer, void **k, void **v)
{
    READY();
    if (!check_layer(layer) || !G.kv[layer].k) return fail("KV layer %d not allocated", layer);
    if (k) *k = G.kv[layer].k;
    if (v) *v = G.kv[layer].v;
    return 1;
}

int coli_cuda_gqa_norm_weight(int layer, const float *qnw, const float *knw, int hd)
{
    READY();
    if (!check_layer(layer) || !G.kv[layer].k) return fail("KV layer %d not allocated", layer);
    KvLayer &L = G.kv[layer];
    if (hd != L.hd) return fail("norm weight length %d != hd %d", hd, L.hd);
    if (!L.qnw) {
        if (!dev_alloc((void **)&L.qnw, (size_t)2 * hd * 4)) return 0;
        L.knw = L.qnw + hd;
    }
    CK(cudaMemcpyAsync(L.qnw, qnw, (size_t)hd * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaMemcpyAsync(L.knw, knw, (size_t)hd * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaStreamSynchronize(stream()));
    return 1;
}

// ------------------------------------------------------------------ GQA
}  // extern "C"

// The attention core of coli_cuda_gqa / coli_cuda_gqa_project: S roped query
// rows (host fp32) of request 0 at positions T-S .. T-1; ctx [S][H][hd] into
// device memory, fp32 or bf16.
static int gqa_core(int layer, const float *q, void *ctx_d, int out_bf16, int S, int H, int KH, int hd,
                    int max_t, int st0, int T, float scale)
{
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    KvLayer &L = G.kv[layer];
    kv_adopt_split(L, KH, max_t);
    if (!gqa_shape_ok(L, H, KH, hd)) return 0;
    if (st0 != 0) return fail("st0 != 0 is not supported");
    if (max_t != L.max_t || S < 1 || T < S || T > L.max_t) return fail("bad S/T/max_t");
    const float *qd = (const float *)upload(S_IN0, q, (size_t)S * H * 2 * hd * 4);
    if (!qd) return 0;
    // all S query rows belong to request 0, at positions T-S .. T-1
    int *pos_d = (int *)scratch(S_POS, (size_t)S * 4);
    int *creq_d = (int *)scratch(S_CREQ, (size_t)S * 4);
    __nv_bfloat16 *qb = (__nv_bfloat16 *)scratch(S_Q, (size_t)S * H * hd * 2);
    if (!pos_d || !creq_d || !qb) return 0;
    iota_kernel<<<(S + 255) / 256, 256, 0, stream()>>>(pos_d, creq_d, S, T - S, 0);
    CK(cudaGetLastError());
    split_q_kernel<<<S * H, hd, 0, stream()>>>(qd, qb, S * H, hd);
    CK(cudaGetLastError());
    g_launches += 2;
    if (S >= PREFILL_MIN_ROWS) return gqa_prefill_rows(L, 0, S, T - S, H, qd, ctx_d, 0, out_bf16, scale);
    return gqa_attend(L, S, H, pos_d, creq_d, T, qd, ctx_d, 0, out_bf16, scale);
}

extern "C" {

int coli_cuda_gqa(int layer, const float *q, float *ctx, int S, int H, int KH, int hd, int max_t,
                  int st0, int T, float scale)
{
    READY();
    float *out = (float *)scratch(S_OUT, (size_t)(S > 0 ? S : 1) * H * hd * 4);
    if (!out) return 0;
    if (!gqa_core(layer, q, out, 0, S, H, KH, hd, max_t, st0, T, scale)) return 0;
    if (!download(ctx, out, (size_t)S * H * hd * 4)) return 0;
    return check_dev_error();
}

int coli_cuda_gqa_step(int layer, int req, int S, int pos_base, const float *qg, const float *k,
                       const float *v, float *ctx, int H, int KH, int hd, int rot, float eps,
                       float theta)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (S < 1 || pos_base < 0) return fail("bad S/pos_base");
    const void *qd = upload(S_IN0, qg, (size_t)S * H * 2 * hd * 4);
    const void *kd = upload(S_IN1, k, (size_t)S * KH * hd * 4);
    const void *vd = upload(S_IN2, v, (size_t)S * KH * hd * 4);
    float *out = (float *)scratch(S_OUT, (size_t)S * H * hd * 4);
    if (!qd || !kd || !vd || !out) return 0;
    if (!coli_cuda_gqa_step_dev(layer, req, S, pos_base, qd, kd, vd, out, H, KH, hd, rot, eps, theta, 0))
        return 0;
    if (!download(ctx, out, (size_t)S * H * hd * 4)) return 0;
    return check_dev_error();
}

int coli_cuda_gqa_step_dev(int layer, int req, int S, int pos_base, const void *qg, const void *k,
                           const void *v, void *ctx, int H, int KH, int hd, int rot, float eps,
                           float theta, int dtype)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    KvLayer &L = G.kv[layer];
    if (!L.k) return fail("KV layer %d not allocated", layer);
    if (req < 0 || req >= L.batch) return fail("request %d beyond batch %d", req, L.batch);
    if (S < 1 || pos_base < 0) return fail("bad S/pos_base");
    int *pos_d = (int *)scratch(S_POS, (size_t)S * 4);
    int *creq_d = (int *)scratch(S_CREQ, (size_t)S * 4);
    if (!pos_d || !creq_d) return 0;
    iota_kernel<<<(S + 255) / 256, 256, 0, stream()>>>(pos_d, creq_d, S, pos_base, req);
    CK(cudaGetLastError());
    g_launches += 1;
    return gqa_rows(layer, S, qg, k, v, pos_d, creq_d, pos_base + S, ctx, H, KH, hd, rot, eps, theta,
                    dtype, dtype, req, pos_base);
}

int coli_cuda_gqa_decode(int layer, int B, const float *qg, const float *k, const float *v,
                         const int *pos, float *ctx, int H, int KH, int hd, int rot, float eps,
                         float theta)
{
    READY();
    if (B < 1 || hd < 1) return fail("bad batch");
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (B > G.kv[layer].batch) return fail("batch %d beyond the cache's %d requests", B, G.kv[layer].batch);
    int tmax = 0;
    for (int b = 0; b < B; ++b) {
        if (pos[b] < 0) return fail("negative position");
        tmax = pos[b] + 1 > tmax ? pos[b] + 1 : tmax;
    }
    // q|gate rows: the q halves go up first with k, v and the positions; the
    // gate halves (needed only by the combine, at the end) follow on the copy
    // stream while the prologue and the split kernel run
    if (!G.copy_stream) {   // all three or none
        cudaStream_t cs = nullptr;
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        cudaError_t e = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&e0, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&e1, cudaEventDisableTiming);
        if (e != cudaSuccess) {
            if (e1) cudaEventDestroy(e1);
            if (e0) cudaEventDestroy(e0);
            if (cs) cudaStreamDestroy(cs);
            return cuda_fail(e, "copy stream");
        }
        G.copy_stream = cs; G.ev_fork = e0; G.ev_gate = e1;
    }
    const size_t half = (size_t)hd * 4, rows = (size_t)B * H;
    char *qd = (char *)scratch(S_IN0, rows * 2 * half);
    if (!qd) return 0;
    CK(cudaMemcpy2DAsync(qd, 2 * half, qg, 2 * half, half, rows, cudaMemcpyHostToDevice, stream()));
    const void *kd = upload(S_IN1, k, (size_t)B * KH * hd * 4);
    const void *vd = upload(S_IN2, v, (size_t)B * KH * hd * 4);
    const int *pd = (const int *)upload(S_POS, pos, (size_t)B * 4);
    float *out = (float *)scratch(S_OUT, (size_t)B * H * hd * 4);
    if (!kd || !vd || !pd || !out) return 0;
    // after the q/k/v copies, so that the two do not share the link
    CK(cudaEventRecord(G.ev_fork, stream()));
    CK(cudaStreamWaitEvent(G.copy_stream, G.ev_fork, 0));
    CK(cudaMemcpy2DAsync(qd + half, 2 * half, (const char *)qg + half, 2 * half, half, rows,
                         cudaMemcpyHostToDevice, G.copy_stream));
    CK(cudaEventRecord(G.ev_gate, G.copy_stream));
    if (!gqa_rows(layer, B, qd, kd, vd, pd, nullptr, tmax, out, H, KH, hd, rot, eps, theta, 0, 0, -1, 0,
                  G.ev_gate)) {
        // rejected before the combine: the backend stream still joins the
        // gate copy, so no later call frees or regrows its buffer under it
        cudaStreamWaitEvent(stream(), G.ev_gate, 0);
        return 0;
    }
    if (!download(ctx, out, (size_t)B * H * hd * 4)) return 0;
    return check_dev_error();
}

int coli_cuda_gqa_decode_dev(int layer, int B, const void *qg, const void *k, const void *v,
                             const int *pos_dev, void *ctx, int H, int KH, int hd, int rot,
                             float eps, float theta, int dtype)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    KvLayer &L = G.kv[layer];
    if (!L.k) return fail("KV layer %d not allocated", layer);
    if (B < 1 || B > L.batch) return fail("batch %d beyond the cache's %d requests", B, L.batch);
    // Positions live on the device; the split plan uses max_t as the bound.
    return gqa_rows(layer, B, qg, k, v, pos_dev, nullptr, L.max_t, ctx, H, KH, hd, rot, eps, theta,
                    dtype, dtype);
}

static int gqa_prefill_heads(int layer, int req, int S, int pos_base, const void *qg, const void *k,
                             const void *v, void *ctx, int H, int KH, int hd, int rot, float eps,
                             float theta, int dtype, int h0, int nh, const PeerGather *gather);

int coli_cuda_gqa_prefill_heads_dev(int layer, int req, int S, int pos_base, const void *qg,
                                    const void *k, const void *v, void *ctx, int H, int KH,
                                    int hd, int rot, float eps, float theta, int dtype, int h0,
                                    int nh)
{
    return gqa_prefill_heads(layer, req, S, pos_base, qg, k, v, ctx, H, KH, hd, rot, eps, theta, dtype,
                             h0, nh, nullptr);
}

static int gqa_prefill_heads(int layer, int req, int S, int pos_base, const void *qg, const void *k,
                             const void *v, void *ctx, int H, int KH, int hd, int rot, float eps,
                             float theta, int dtype, int h0, int nh, const PeerGather *gather)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    KvLayer &L = G.kv[layer];
    if (!L.k) return fail("KV layer %d not allocated", layer);
    if (!L.qnw) return fail("q/k norm weights of layer %d not set", layer);
    if (hd != 256 || H != 8 * KH) return fail("unsupported GQA shape H=%d KH=%d hd=%d", H, KH, hd);
    if (nh < 1 || h0 < 0 || h0 + nh > H) return fail("bad head range [%d, %d)", h0, h0 + nh);
    const int kh0 = h0 / 8, nkh = (h0 + nh - 1) / 8 + 1 - kh0;
    if (L.KH != nkh) return fail("cache holds %d KV heads; heads [%d, %d) need %d", L.KH, h0, h0 + nh, nkh);
    if (S < PREFILL_MIN_ROWS) return fail("head-sharded prefill needs S >= %d", PREFILL_MIN_ROWS);
    if (req < 0 || req >= L.batch || pos_base < 0 || pos_base + S > L.max_t) return fail("bad request / positions");
    if (rot < 2 || rot > hd || (rot & 1)) return fail("bad rot %d", rot);
    int *pos_d = (int *)scratch(S_POS, (size_t)S * 4);
    int *creq_d = (int *)scratch(S_CREQ, (size_t)S * 4);
    __nv_bfloat16 *q = (__nv_bfloat16 *)scratch(S_Q, (size_t)S * nh * hd * 2);
    if (!pos_d || !creq_d || !q) return 0;
    iota_kernel<<<(S + 255) / 256, 256, 0, stream()>>>(pos_d, creq_d, S, pos_base, req);
    CK(cudaGetLastError());
    GqaPrologueArgs pa{};
    pa.qg = qg; pa.k = k; pa.v = v; pa.qnw = L.qnw; pa.knw = L.knw; pa.pos = pos_d; pa.creq = creq_d;
    pa.qout = q; pa.kcache = L.k; pa.vcache = L.v;
    pa.nq = S; pa.H = nh; pa.KH = nkh; pa.max_t = L.max_t; pa.rot = rot; pa.eps = eps; pa.theta = theta;
    pa.h0 = h0; pa.kh0 = kh0; pa.Hin = H; pa.KHin = KH;
    CK(launch_gqa_prologue(pa, dtype, stream()));
    CUtensorMap tq;
    if (!make_q_tmap(&tq, q, S, nh, hd)) return 0;
    GqaPrefillArgs a{};
    a.qg = qg; a.ctx = ctx; a.S = S; a.H = nh; a.KH = nkh; a.max_t = L.max_t; a.req = req;
    a.pos_base = pos_base; a.n_qtiles = (S + 127) / 128;
    a.scale_log2 = (1.f / sqrtf((float)hd)) * 1.4426950408889634f;
    a.h0 = h0; a.kh0 = kh0; a.Hin = H;
    if (gather) {
        a.gather = *gather;
        a.gather.block = (long long)S * nh * hd;
    }
    PfEpiMaps em;
    const bool tma_epi = dtype && !gather;
    if (tma_epi && !make_pf_epi_maps(&em, qg, ctx, S, nh, H, hd)) return 0;
    kt_mark(COLI_K_GQA_PREFILL);
    CK(launch_gqa_prefill(tq, L.tmK64, L.tmV64, a, dtype, dtype, stream(), tma_epi ? &em : nullptr));
    kt_mark(COLI_K_GQA_PREFILL);
    g_launches += 3;
    return 1;
}

// ------------------------------------------------------------------ GDN state
int coli_cuda_gdn_state_ensure(int layer, int batch, int VH, int KD, int VD)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (batch < 1 || VH < 1 || KD < 1 || VD < 1) return fail("bad GDN state geometry");
    GdnLayer &L = G.gdn[layer];
    if (L.state && L.batch == batch && L.VH == VH && L.KD == KD && L.VD == VD) return 1;
    if (L.state) {
        CK(cudaStreamSynchronize(stream()));
        dev_free(L.state, (size_t)L.batch * L.VH * L.KD * L.VD * 4);
        L.state = nullptr;
    }
    size_t bytes = (size_t)batch * VH * KD * VD * 4;
    if (!dev_alloc((void **)&L.state, bytes)) return 0;
    CK(cudaMemsetAsync(L.state, 0, bytes, stream()));
    L.batch = batch; L.VH = VH; L.KD = KD; L.VD = VD;
    return 1;
}

int coli_cuda_gdn_conv_ensure(int layer, int batch, int conv_k, int conv_dim)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (batch < 1 || conv_k < 2 || conv_k > 16 || conv_dim < 1) return fail("bad conv geometry");
    GdnLayer &L = G.gdn[layer];
    if (L.hist && L.hbatch == batch && L.conv_k == conv_k && L.conv_dim == conv_dim) return 1;
    if (L.hist) {
        CK(cudaStreamSynchronize(stream()));
        dev_free(L.hist, (size_t)L.hbatch * (L.conv_k - 1) * L.conv_dim * 4);
        L.hist = nullptr;
    }
    if (L.conv_w && (L.conv_k != conv_k || L.conv_dim != conv_dim)) {
        dev_free(L.conv_w, (size_t)L.conv_dim * L.conv_k * 4);
        L.conv_w = nullptr;
    }
    size_t bytes = (size_t)batch * (conv_k - 1) * conv_dim * 4;
    if (!dev_alloc((void **)&L.hist, bytes)) return 0;
    CK(cudaMemsetAsync(L.hist, 0, bytes, stream()));
    L.hbatch = batch; L.conv_k = conv_k; L.conv_dim = conv_dim;
    return 1;
}

int coli_cuda_gdn_conv_weight(int layer, const float *cw, int conv_k, int conv_dim)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    GdnLayer &L = G.gdn[layer];
    if (!L.hist || L.conv_k != conv_k || L.conv_dim != conv_dim) return fail("conv_ensure first (geometry mismatch)");
    if (!L.conv_w && !dev_alloc((void **)&L.conv_w, (size_t)conv_dim * conv_k * 4)) return 0;
    CK(cudaMemcpyAsync(L.conv_w, cw, (size_t)conv_dim * conv_k * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaStreamSynchronize(stream()));
    return 1;
}

int coli_cuda_gdn_params(int layer, const float *A_log, const float *dt_bias, const float *gnorm,
                         int VH, int VD)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    GdnLayer &L = G.gdn[layer];
    if (L.A_log && (L.pVH != VH || L.pVD != VD)) {
        dev_free(L.A_log, (size_t)(2 * L.pVH + L.pVD) * 4);
        L.A_log = nullptr;
    }
    if (!L.A_log && !dev_alloc((void **)&L.A_log, (size_t)(2 * VH + VD) * 4)) return 0;
    L.dt_bias = L.A_log + VH;
    L.gnorm = L.A_log + 2 * VH;
    L.pVH = VH; L.pVD = VD;
    CK(cudaMemcpyAsync(L.A_log, A_log, (size_t)VH * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaMemcpyAsync(L.dt_bias, dt_bias, (size_t)VH * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaMemcpyAsync(L.gnorm, gnorm, (size_t)VD * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaStreamSynchronize(stream()));
    return 1;
}

void coli_cuda_gdn_reset(void)
{
    if (!G.ready) return;
    for (int i = 0; i < MAX_LAYERS; ++i) {
        GdnLayer &L = G.gdn[i];
        if (L.state) cudaMemsetAsync(L.state, 0, (size_t)L.batch * L.VH * L.KD * L.VD * 4, stream());
        if (L.hist) cudaMemsetAsync(L.hist, 0, (size_t)L.hbatch * (L.conv_k - 1) * L.conv_dim * 4, stream());
    }
    cudaStreamSynchronize(stream());
}

static int gdn_state_io(int layer, int req, float *h, int set)
{
    READY();
    if (!check_layer(layer) || !G.gdn[layer].state) return fail("GDN layer %d not allocated", layer);
    GdnLayer &L = G.gdn[layer];
    if (req < 0 || req >= L.batch) return fail("request out of range");
    const size_t n = (size_t)L.VH * L.KD * L.VD;
    float *d = L.state + (size_t)req * n;
    if (set) {
        CK(cudaMemcpyAsync(d, h, n * 4, cudaMemcpyHostToDevice, stream()));
        CK(cudaStreamSynchronize(stream()));
        return 1;
    }
    return download(h, d, n * 4);
}
int coli_cuda_gdn_state_get(int layer, int req, float *state) { return gdn_state_io(layer, req, state, 0); }
int coli_cuda_gdn_state_set(int layer, int req, const float *state)
{
    return gdn_state_io(layer, req, const_cast<float *>(state), 1);
}

static int gdn_conv_io(int layer, int req, float *ring, int set)
{
    READY();
    if (!check_layer(layer) || !G.gdn[layer].hist) return fail("GDN conv of layer %d not allocated", layer);
    GdnLayer &L = G.gdn[layer];
    if (req < 0 || req >= L.hbatch) return fail("request out of range");
    const size_t n = (size_t)(L.conv_k - 1) * L.conv_dim;
    float *d = L.hist + (size_t)req * n;
    if (set) {
        CK(cudaMemcpyAsync(d, ring + L.conv_dim, n * 4, cudaMemcpyHostToDevice, stream()));
        CK(cudaStreamSynchronize(stream()));
        return 1;
    }
    memset(ring, 0, (size_t)L.conv_dim * 4);
    return download(ring + L.conv_dim, d, n * 4);
}
int coli_cuda_gdn_conv_get(int layer, int req, float *ring) { return gdn_conv_io(layer, req, ring, 0); }
int coli_cuda_gdn_conv_set(int layer, int req, const float *ring)
{
    return gdn_conv_io(layer, req, const_cast<float *>(ring), 1);
}

// ------------------------------------------------------------------ GDN compute
}  // extern "C"

// The recurrence of coli_cuda_gdn / coli_cuda_gdn_project on pre-normalised
// host inputs; y [VH*VD] fp32 into device memory.
static int gdn_core(int layer, const float *qn, const float *kn, const float *v, const float *z,
                    const float *decay, const float *beta, const float *gnorm, float *y_d, int KH, int KD,
                    int VH, int VD, float eps)
{
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    GdnLayer &L = G.gdn[layer];
    if (!gdn_shape_ok(L, KH, KD, VH, VD, 0)) return 0;
    const int key_dim = KH * KD, stride = 2 * key_dim + VH * VD;
    float *in = (float *)scratch(S_IN0, (size_t)stride * 4);
    float *zd = (float *)upload(S_IN1, z, (size_t)VH * VD * 4);
    float *pd = (float *)scratch(S_P0, (size_t)(2 * VH + VD) * 4);
    if (!in || !zd || !pd) return 0;
    CK(cudaMemcpyAsync(in, qn, (size_t)key_dim * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaMemcpyAsync(in + key_dim, kn, (size_t)key_dim * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaMemcpyAsync(in + 2 * key_dim, v, (size_t)VH * VD * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaMemcpyAsync(pd, decay, (size_t)VH * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaMemcpyAsync(pd + VH, beta, (size_t)VH * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaMemcpyAsync(pd + 2 * VH, gnorm, (size_t)VD * 4, cudaMemcpyHostToDevice, stream()));
    GdnDecodeArgs ga;
    memset(&ga, 0, sizeof(ga));
    ga.qkv = in; ga.z = zd; ga.decay = pd; ga.beta = pd + VH; ga.gnorm = pd + 2 * VH;
    ga.state = L.state; ga.y = y_d;
    ga.B = 1; ga.KH = KH; ga.KD = KD; ga.VH = VH; ga.VD = VD; ga.in_stride = stride; ga.eps = eps;
    CK(launch_gdn_decode(ga, 0, 0, 1, stream()));
    g_launches += 1;
    return 1;
}

extern "C" {

int coli_cuda_gdn(int layer, const float *qn, const float *kn, const float *v, const float *z,
                  const float *decay, const float *beta, const float *gnorm, float *y, int KH,
                  int KD, int VH, int VD, float eps)
{
    READY();
    float *out = (float *)scratch(S_OUT, (size_t)VH * VD * 4);
    if (!out) return 0;
    if (!gdn_core(layer, qn, kn, v, z, decay, beta, gnorm, out, KH, KD, VH, VD, eps)) return 0;
    if (!download(y, out, (size_t)VH * VD * 4)) return 0;
    return check_dev_error();
}

int coli_cuda_gdn_decode(int layer, int B, const float *qkv, const float *z, const float *a,
                         const float *b, float *y, int KH, int KD, int VH, int VD, float eps)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (B < 1) return fail("bad batch");
    const int CD = 2 * KH * KD + VH * VD;
    const void *qd = upload(S_IN0, qkv, (size_t)B * CD * 4);
    const void *zd = upload(S_IN1, z, (size_t)B * VH * VD * 4);
    const void *ad = upload(S_IN2, a, (size_t)B * VH * 4);
    const void *bd = upload(S_IN3, b, (size_t)B * VH * 4);
    float *out = (float *)scratch(S_OUT, (size_t)B * VH * VD * 4);
    if (!qd || !zd || !ad || !bd || !out) return 0;
    if (!gdn_decode_run(layer, B, 0, qd, zd, ad, bd, out, KH, KD, VH, VD, eps, 0)) return 0;
    if (!download(y, out, (size_t)B * VH * VD * 4)) return 0;
    return check_dev_error();
}

int coli_cuda_gdn_decode_dev(int layer, int B, const void *qkv, const void *z, const void *a,
                             const void *b, void *y, int KH, int KD, int VH, int VD, float eps,
                             int dtype)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (B < 1) return fail("bad batch");
    return gdn_decode_run(layer, B, 0, qkv, z, a, b, y, KH, KD, VH, VD, eps, dtype);
}

int coli_cuda_gdn_prefill_dev(int layer, int req, int S, const void *qkv, const void *z,
                              const void *a, const void *b, void *y, int KH, int KD, int VH,
                              int VD, float eps, int dtype)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (S < 1) return fail("bad S");
    if (S >= GDN_CHUNK_MIN_ROWS)
        return gdn_prefill_chunked(layer, req, S, qkv, z, a, b, y, KH, KD, VH, VD, eps, dtype);
    // Short runs: sequential token steps through the fused decode kernel.
    const int CD = 2 * KH * KD + VH * VD;
    const size_t es = dtype ? 2 : 4;
    for (int s = 0; s < S; ++s) {
        if (!gdn_decode_run(layer, 1, req, (const char *)qkv + (size_t)s * CD * es,
                            (const char *)z + (size_t)s * VH * VD * es, (const char *)a + (size_t)s * VH * es,
                            (const char *)b + (size_t)s * VH * es, (char *)y + (size_t)s * VH * VD * es, KH,
                            KD, VH, VD, eps, dtype))
            return 0;
    }
    return 1;
}

int coli_cuda_gdn_prefill_heads_dev(int layer, int req, int S, const void *qkv, const void *z,
                                    const void *a, const void *b, void *y, int KH, int KD, int VH,
                                    int VD, float eps, int dtype, int kh0, int nkh)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (S < GDN_CHUNK_MIN_ROWS) return fail("head-sharded GDN prefill needs S >= %d", GDN_CHUNK_MIN_ROWS);
    return gdn_prefill_chunked(layer, req, S, qkv, z, a, b, y, KH, KD, VH, VD, eps, dtype, kh0, nkh);
}

int coli_cuda_gdn_prefill(int layer, int req, int S, const float *qkv, const float *z,
                          const float *a, const float *b, float *y, int KH, int KD, int VH, int VD,
                          float eps)
{
    READY();
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (S < 1) return fail("bad S");
    const int CD = 2 * KH * KD + VH * VD;
    const void *qd = upload(S_IN0, qkv, (size_t)S * CD * 4);
    const void *zd = upload(S_IN1, z, (size_t)S * VH * VD * 4);
    const void *ad = upload(S_IN2, a, (size_t)S * VH * 4);
    const void *bd = upload(S_IN3, b, (size_t)S * VH * 4);
    float *out = (float *)scratch(S_OUT, (size_t)S * VH * VD * 4);
    if (!qd || !zd || !ad || !bd || !out) return 0;
    if (!coli_cuda_gdn_prefill_dev(layer, req, S, qd, zd, ad, bd, out, KH, KD, VH, VD, eps, 0)) return 0;
    if (!download(y, out, (size_t)S * VH * VD * 4)) return 0;
    return check_dev_error();
}

}  // extern "C"

// Fixed-scratch decode entry point (no device allocation on its path).
#include "noalloc.cu"
#include "block.cu"
#include "container.cu"
#include "peer.cu"
