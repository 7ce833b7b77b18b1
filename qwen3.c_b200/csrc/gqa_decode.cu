// Gated GQA decode: split-KV flash-decode over the resident bf16 KV cache.
//
// Semantics follow the reference's attention() for query rows that sit at the
// end of the cache (c/qwen.c:598-663): per-head zero-centred RMSNorm of q and
// k, partial NeoX RoPE on the first `rot` dims, K/V append, causal softmax
// attention over rows 0..pos with scale 1/sqrt(hd), then ctx *= sigmoid(gate).
//
// Kernels
//   gqa_prologue_warp_kernel  q/k norm + RoPE; bf16 q to scratch; k/v rows
//                        appended to the cache (a warp per head vector, 1-4
//                        query rows per CTA, 16-byte accesses);
//                        gqa_prologue_kernel is the same arithmetic for
//                        inputs that are not 16-byte aligned (a CTA per
//                        head vector).
//   gqa_split_kernel     one CTA per (query row, KV head, KV split). Each warp
//                        streams 16-token K/V tiles through its own TMA ring
//                        (128B-swizzled boxes, mbarrier completion) and runs
//                        S^T = K Q^T and O^T += V^T P^T on bf16 mma.sync with
//                        all 8 query heads of the KV head in the N dimension,
//                        online softmax in registers (log2 domain), P^T
//                        formed from the score fragments with movmatrix. The
//                        warps' partial (max, sum, O) are merged in shared
//                        memory and one partial per CTA goes to scratch.
//                        For decode batches of up to 8 rows (FUSE != 0) it
//                        also does the prologue's work for itself: its 8
//                        heads' q normed and roped into shared memory, and
//                        the new k / v row appended by the CTA whose key
//                        range holds it, so no prologue launch precedes it.
//   gqa_combine_kernel   log-sum-exp merge of the split partials, the
//                        sigmoid output gate, ctx out.
// The dominant kernel is HBM bound: 2*hd*2 bytes of K+V per cached token per
// KV head.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace coli {

constexpr int GQA_HD = 256, GQA_GRP = 8, GQA_TILE = 16;
constexpr int GQA_TILE_BYTES = GQA_TILE * GQA_HD * 2;  // one K (or V) tile: 8 KiB

// ------------------------------------------------------------------ prologue
template <typename TI>
__global__ void __launch_bounds__(GQA_HD)
gqa_prologue_kernel(GqaPrologueArgs p)
{
    griddep_launch();    // the split kernel may start its cache loads now
    const int n = blockIdx.x, j = blockIdx.y, d = threadIdx.x;
    const int H = p.H, KH = p.KH;
    const int Hin = p.Hin ? p.Hin : H, KHin = p.KHin ? p.KHin : KH;
    const int pos = p.pos[n];
    const float *w;
    float x;
    if (j < H) {
        x = to_f32(static_cast<const TI *>(p.qg)[((size_t)n * Hin + p.h0 + j) * 2 * GQA_HD + d]);
        w = p.qnw;
    } else {
        x = to_f32(static_cast<const TI *>(p.k)[((size_t)n * KHin + p.kh0 + (j - H)) * GQA_HD + d]);
        w = p.knw;
    }
    // zero-centred RMSNorm, sum of squares in double (c/qwen.c:326-330)
    __shared__ double red[8];
    __shared__ float vec[GQA_HD];
    double s2 = (double)x * x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    if ((d & 31) == 0) red[d >> 5] = s2;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float r = 1.f / sqrtf((float)(tot / GQA_HD) + p.eps);
    float y = x * r * (1.f + w[d]);
    vec[d] = y;
    __syncthreads();
    // partial NeoX RoPE on dims [0, rot) (c/qwen.c:570-579)
    const int half = p.rot >> 1;
    if (d < p.rot) {
        const int jj = d < half ? d : d - half;
        const float inv = powf(p.theta, -2.0f * jj / p.rot);
        const float ang = (float)pos * inv;
        const float cs = cosf(ang), sn = sinf(ang);
        const float lo = vec[jj], hi = vec[jj + half];
        y = d < half ? lo * cs - hi * sn : hi * cs + lo * sn;
    }
    if (j < H) {
        p.qout[((size_t)n * H + j) * GQA_HD + d] = __float2bfloat16_rn(y);
    } else {
        const int kh = j - H;
        const int creq = p.creq ? p.creq[n] : n;
        const size_t row = ((size_t)creq * KH + kh) * p.max_t + pos;
        p.kcache[row * GQA_HD + d] = __float2bfloat16_rn(y);
        const float v = to_f32(static_cast<const TI *>(p.v)[((size_t)n * KHin + p.kh0 + kh) * GQA_HD + d]);
        p.vcache[row * GQA_HD + d] = __float2bfloat16_rn(v);
    }
}

// Same arithmetic with one warp per head vector and one CTA per one to four query rows:
// lane l owns dims [8l, 8l+8) (16-byte loads and stores), the sum of squares
// is reduced across lanes in double, and the row's RoPE angles (which all its heads
// share) are computed once per CTA into shared memory; each warp issues the
// loads of three head vectors before it reduces any of them. Needs 16-byte aligned
// row bases; the launcher falls back to the kernel above otherwise.
template <typename TI>
__device__ __forceinline__ void load8(const TI *src, float (&x)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16 *src, float (&x)[8])
{
    const uint4 u = *reinterpret_cast<const uint4 *>(src);
    const __nv_bfloat162 *b = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) { const float2 f = __bfloat1622float2(b[i]); x[2 * i] = f.x; x[2 * i + 1] = f.y; }
}
template <>
__device__ __forceinline__ void load8<float>(const float *src, float (&x)[8])
{
    const float4 a = reinterpret_cast<const float4 *>(src)[0], b = reinterpret_cast<const float4 *>(src)[1];
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
// eight raw input elements held packed until they are used
template <typename TI> struct Raw8;
template <> struct Raw8<__nv_bfloat16> {
    uint4 u;
    __device__ __forceinline__ void load(const __nv_bfloat16 *src) { u = *reinterpret_cast<const uint4 *>(src); }
    __device__ __forceinline__ void unpack(float (&x)[8]) const
    {
        const __nv_bfloat162 *b = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) { const float2 f = __bfloat1622float2(b[i]); x[2 * i] = f.x; x[2 * i + 1] = f.y; }
    }
};
template <> struct Raw8<float> {
    float4 a, b;
    __device__ __forceinline__ void load(const float *src)
    {
        a = reinterpret_cast<const float4 *>(src)[0]; b = reinterpret_cast<const float4 *>(src)[1];
    }
    __device__ __forceinline__ void unpack(float (&x)[8]) const
    {
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
};
__device__ __forceinline__ void store8(__nv_bfloat16 *dst, const float (&y)[8])
{
    uint4 u;
    __nv_bfloat162 *b = reinterpret_cast<__nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = __floats2bfloat162_rn(y[2 * i], y[2 * i + 1]);
    *reinterpret_cast<uint4 *>(dst) = u;
}

constexpr int GQA_PRO_ROWS = 4, GQA_PRO_WARPS = 8, GQA_PRO_U = 3;

// One head vector of q or k, one warp, lane = 8 consecutive dims (d0 = 8 lane):
// zero-centred RMSNorm (c/qwen.c:326-330; per-lane partial sums of squares in
// fp32, the cross-lane sum in double as the reference does), then partial
// NeoX RoPE on dims [0, rot) (c/qwen.c:570-579) with the row's angle table
// cs / sn [rot / 2]. The RoPE partner of dim d is d +- rot/2: when rot/2 is a
// multiple of 8 it sits in the same slot of lane +- rot/16, else it goes
// through vw, a 256-float scratch of this warp. Shared by the prologue kernel
// and the fused decode split kernel, so both produce the same bits.
__device__ __forceinline__ void gqa_norm_rope(float (&y)[8], const float (&x)[8], const float (&w)[8],
                                              float eps, int rot, const float *cs, const float *sn,
                                              float *vw, int lane)
{
    const int d0 = lane * 8, half = rot >> 1;
    float sl = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) sl = fmaf(x[i], x[i], sl);
    double s2 = sl;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    const float rs = 1.f / sqrtf((float)(s2 / GQA_HD) + eps);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = x[i] * rs * (1.f + w[i]);
    if ((half & 7) == 0) {
        const int hl = half >> 3;
        const int src_lane = lane < hl ? lane + hl : lane - hl;
        float q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = __shfl_sync(0xffffffffu, y[i], src_lane);
        if (d0 < rot) {
            const bool lo_half = d0 < half;
            const int jj0 = lo_half ? d0 : d0 - half;
            const float4 c0 = *reinterpret_cast<const float4 *>(&cs[jj0]);
            const float4 c1 = *reinterpret_cast<const float4 *>(&cs[jj0 + 4]);
            const float4 s0 = *reinterpret_cast<const float4 *>(&sn[jj0]);
            const float4 s1 = *reinterpret_cast<const float4 *>(&sn[jj0 + 4]);
            const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
                y[i] = lo_half ? y[i] * c[i] - q[i] * sv[i] : y[i] * c[i] + q[i] * sv[i];
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) vw[d0 + i] = y[i];
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int d = d0 + i;
            if (d < rot) {
                const int jj = d < half ? d : d - half;
                const float lo = vw[jj], hi = vw[jj + half];
                y[i] = d < half ? lo * cs[jj] - hi * sn[jj] : hi * cs[jj] + lo * sn[jj];
            }
        }
        __syncwarp();
    }
}

// RoPE angle table of position pos (c/qwen.c:570-579): entries [0, rot/2),
// threads tid0, tid0 + nthr, ...
__device__ __forceinline__ void gqa_rope_table(float *cs, float *sn, int pos, int rot, float theta, int tid0,
                                               int nthr)
{
    const int half = rot >> 1;
    for (int jj = tid0; jj < half; jj += nthr) {
        const float inv = powf(theta, -2.0f * jj / rot);
        const float ang = (float)pos * inv;
        cs[jj] = cosf(ang); sn[jj] = sinf(ang);
    }
}

template <typename TI>
__global__ void __launch_bounds__(GQA_PRO_WARPS * 32, 4)
gqa_prologue_warp_kernel(GqaPrologueArgs p, int rpc)
{
    __shared__ float cs_t[GQA_PRO_ROWS][GQA_HD / 2], sn_t[GQA_PRO_ROWS][GQA_HD / 2];
    __shared__ float vec[GQA_PRO_WARPS][GQA_HD];
    griddep_launch();    // the split kernel may start its cache loads now
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * rpc, rows = min(rpc, p.nq - n0);
    const int H = p.H, KH = p.KH, nv = H + KH;
    const int Hin = p.Hin ? p.Hin : H, KHin = p.KHin ? p.KHin : KH;
    // the input loads of up to U head vectors of this warp (and, for k
    // vectors with bf16 inputs, the v row appended beside them; fp32 v is
    // loaded where it is stored, to stay within 64 registers), issued before
    // any arithmetic
    Raw8<TI> raw[GQA_PRO_U], vraw[GQA_PRO_U];
    auto issue = [&](int b) {
        int r = b / nv, j = b - r * nv;
#pragma unroll
        for (int u = 0; u < GQA_PRO_U; ++u) {
            if (r < rows) {
                const int n = n0 + r;
                if (j < H) {
                    raw[u].load(static_cast<const TI *>(p.qg) + ((size_t)n * Hin + p.h0 + j) * 2 * GQA_HD + lane * 8);
                } else {
                    const size_t off = ((size_t)n * KHin + p.kh0 + (j - H)) * GQA_HD + lane * 8;
                    raw[u].load(static_cast<const TI *>(p.k) + off);
                    if constexpr (sizeof(TI) == 2) vraw[u].load(static_cast<const TI *>(p.v) + off);
                }
            }
            for (j += GQA_PRO_WARPS; j >= nv; j -= nv) ++r;
        }
    };
    // the first batch goes out before the RoPE table, whose barrier would
    // otherwise hold it back (one global-memory wait instead of two on the
    // decode path, where a CTA holds one row)
    issue(warp);
    // RoPE angles of these rows (c/qwen.c:570-579), shared by all their heads
    for (int r = 0; r < rows; ++r)
        gqa_rope_table(cs_t[r], sn_t[r], p.pos[n0 + r], p.rot, p.theta, threadIdx.x, blockDim.x);
    __syncthreads();
    const int d0 = lane * 8, total = rows * nv;
    float *vw = vec[warp];
    for (int b = warp; b < total; b += GQA_PRO_WARPS * GQA_PRO_U) {
        if (b != warp) issue(b);
        int r = b / nv, j = b - r * nv;
#pragma unroll
        for (int u = 0; u < GQA_PRO_U; ++u) {
            if (r >= rows) break;
            const int n = n0 + r;
            const bool isq = j < H;
            float w[8], x[8], y[8];
            load8<float>((isq ? p.qnw : p.knw) + d0, w);
            raw[u].unpack(x);
            gqa_norm_rope(y, x, w, p.eps, p.rot, cs_t[r], sn_t[r], vw, lane);
            if (isq) {
                store8(p.qout + ((size_t)n * H + j) * GQA_HD + d0, y);
            } else {
                const int kh = j - H;
                const int creq = p.creq ? p.creq[n] : n;
                const size_t row = ((size_t)creq * KH + kh) * p.max_t + p.pos[n];
                store8(p.kcache + row * GQA_HD + d0, y);
                float v[8];
                if constexpr (sizeof(TI) == 2) vraw[u].unpack(v);
                else load8<TI>(static_cast<const TI *>(p.v) + ((size_t)n * KHin + p.kh0 + kh) * GQA_HD + d0, v);
                store8(p.vcache + row * GQA_HD + d0, v);
            }
            for (j += GQA_PRO_WARPS; j >= nv; j -= nv) ++r;
        }
    }
}

// ------------------------------------------------------------------ split-KV
template <int WARPS, int STAGES, int FUSE>
__global__ void __launch_bounds__(WARPS * 32, 1)
gqa_split_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                 GqaSplitArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(16) __nv_bfloat16 qsm[GQA_GRP * GQA_HD];
    __shared__ __align__(8) uint64_t full[WARPS][STAGES];

    const int split = blockIdx.x, kh = blockIdx.y, n = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int KH = p.KH;

    if (lane == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&full[warp][s], 1);
        fence_mbar_init();
    }
    if (tid == 0) { tma_prefetch_desc(&tmK); tma_prefetch_desc(&tmV); }
    __syncthreads();

    const int T = p.pos[n] + 1;
    const int start = split * p.chunk;
    const int end = min(T, start + p.chunk);
    const int ntiles = end > start ? (end - start + GQA_TILE - 1) / GQA_TILE : 0;
    const int my_tiles = ntiles > warp ? (ntiles - warp + WARPS - 1) / WARPS : 0;
    const int creq = p.creq ? p.creq[n] : n;
    const int rowbase = (creq * KH + kh) * p.max_t;

    uint8_t *wbuf = smem + (size_t)warp * STAGES * 2 * GQA_TILE_BYTES;
    auto issue = [&](int it) {
        const int s = it % STAGES;
        const int row = rowbase + start + (warp + it * WARPS) * GQA_TILE;
        uint8_t *kb = wbuf + (size_t)s * 2 * GQA_TILE_BYTES;
        uint8_t *vb = kb + GQA_TILE_BYTES;
        mbar_expect_tx(&full[warp][s], 2 * GQA_TILE_BYTES);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            tma_load_2d(kb + c * 2048, &tmK, 64 * c, row, &full[warp][s]);
            tma_load_2d(vb + c * 2048, &tmV, 64 * c, row, &full[warp][s]);
        }
    };
    // Launched as a programmatic dependent of the prologue: the first tiles of
    // the ring stream in while the prologue still runs, except the tile that
    // holds the row the prologue appends (position T - 1), which is loaded
    // after the wait together with the prologue's roped q.
    uint32_t deferred = 0;
    if (lane == 0)
        for (int it = 0; it < STAGES && it < my_tiles; ++it) {
            if (start + (warp + it * WARPS) * GQA_TILE + GQA_TILE > T - p.appended) deferred |= 1u << it;
            else issue(it);
        }
    griddep_wait();      // the prologue's q and appended rows (or, fused, the inputs) are visible
    griddep_launch();    // the combine may launch; it waits for this grid to finish
    if constexpr (FUSE == 0) {
        if (lane == 0 && deferred) {
            fence_proxy_async();   // generic-proxy cache writes of the prologue before the async-proxy read
            for (int it = 0; it < STAGES; ++it)
                if (deferred >> it & 1u) issue(it);
        }
        // q of the 8 heads sharing this KV head (bf16, roped)
        const uint4 *src = reinterpret_cast<const uint4 *>(p.q + ((size_t)n * p.H + kh * GQA_GRP) * GQA_HD);
        uint4 *dst = reinterpret_cast<uint4 *>(qsm);
        for (int i = tid; i < GQA_GRP * GQA_HD / 8; i += WARPS * 32) dst[i] = src[i];
    } else {
        // The prologue's work for this CTA, from the raw inputs: norm and rope
        // the q of the 8 heads of this KV head into qsm (every split of the
        // request does this for itself), and, in the CTA whose key range
        // holds position T - 1, norm and rope k and append the k / v row
        // there before the tile that holds it is loaded.
        using TI = typename std::conditional<FUSE == 1, __nv_bfloat16, float>::type;
        __shared__ __align__(16) float cs[GQA_HD / 2], sn[GQA_HD / 2];
        __shared__ float vws[WARPS][GQA_HD];
        const GqaPrologueArgs &a = p.pro;
        if (ntiles > 0) {                      // uniform across the CTA
            gqa_rope_table(cs, sn, T - 1, a.rot, a.theta, tid, WARPS * 32);
            __syncthreads();
            for (int hh = warp; hh < GQA_GRP; hh += WARPS) {
                float x[8], w[8], y[8];
                load8<TI>(static_cast<const TI *>(a.qg) + ((size_t)n * a.H + kh * GQA_GRP + hh) * 2 * GQA_HD + lane * 8, x);
                load8<float>(a.qnw + lane * 8, w);
                gqa_norm_rope(y, x, w, a.eps, a.rot, cs, sn, vws[warp], lane);
                store8(qsm + hh * GQA_HD + lane * 8, y);
            }
            if (warp == WARPS - 1 && start <= T - 1 && T - 1 < end) {
                float x[8], w[8], y[8], v[8];
                const size_t in = ((size_t)n * a.KH + kh) * GQA_HD + lane * 8;
                load8<TI>(static_cast<const TI *>(a.k) + in, x);
                load8<TI>(static_cast<const TI *>(a.v) + in, v);
                load8<float>(a.knw + lane * 8, w);
                gqa_norm_rope(y, x, w, a.eps, a.rot, cs, sn, vws[warp], lane);
                const size_t row = ((size_t)creq * a.KH + kh) * a.max_t + (T - 1);
                store8(a.kcache + row * GQA_HD + lane * 8, y);
                store8(a.vcache + row * GQA_HD + lane * 8, v);
                fence_proxy_async_global();    // the row before the tile load below reads it
            }
        }
        __syncthreads();
        if (lane == 0 && deferred)
            for (int it = 0; it < STAGES; ++it)
                if (deferred >> it & 1u) issue(it);
    }
    __syncthreads();

    // Q^T as the B operand: b0 = (dim = 16kk + 2(lane&3) + {0,1}, head = lane>>2), b1 = dim + 8
    uint32_t qf[16][2];
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
        const __nv_bfloat16 *qrow = qsm + (lane >> 2) * GQA_HD + kk * 16 + (lane & 3) * 2;
        qf[kk][0] = *reinterpret_cast<const uint32_t *>(qrow);
        qf[kk][1] = *reinterpret_cast<const uint32_t *>(qrow + 8);
    }

    float acc[16][4];
#pragma unroll
    for (int mt = 0; mt < 16; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const float sl2 = p.scale_log2;
    const int r8 = lane & 7, mi = lane >> 3;

    for (int it = 0; it < my_tiles; ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[warp][s], (it / STAGES) & 1)) break;  // error raised; finish quietly
        const uint32_t kb = smem_u32(wbuf + (size_t)s * 2 * GQA_TILE_BYTES);
        const uint32_t vb = kb + GQA_TILE_BYTES;
        const int tok0 = start + (warp + it * WARPS) * GQA_TILE;
        const int valid = min(GQA_TILE, end - tok0);

        // S^T[16 tok x 8 heads] = K[16 x 256] . Q^T[256 x 8]
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
        {
            const int tok = (mi & 1) * 8 + r8;
#pragma unroll
            for (int kk = 0; kk < 16; ++kk) {
                const int chunk = (kk & 3) * 2 + (mi >> 1);
                const uint32_t addr = kb + (kk >> 2) * 2048 + tok * 128 + ((chunk ^ (tok & 7)) << 4);
                uint32_t a0, a1, a2, a3;
                ldsm_x4(addr, a0, a1, a2, a3);
                mma_bf16_16816(sc, a0, a1, a2, a3, qf[kk][0], qf[kk][1]);
            }
        }
        // online softmax per head (heads h0 = 2(lane&3), h1 = h0 + 1)
        const int ta = lane >> 2, tb = ta + 8;
        float x0 = ta < valid ? sc[0] * sl2 : -INFINITY;
        float x1 = ta < valid ? sc[1] * sl2 : -INFINITY;
        float x2 = tb < valid ? sc[2] * sl2 : -INFINITY;
        float x3 = tb < valid ? sc[3] * sl2 : -INFINITY;
        float t0 = fmaxf(x0, x2), t1 = fmaxf(x1, x3);
#pragma unroll
        for (int o = 4; o <= 16; o <<= 1) {
            t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, o));
            t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, o));
        }
        const float n0 = fmaxf(m0, t0), n1 = fmaxf(m1, t1);
        const float u0 = n0 == -INFINITY ? 0.f : n0, u1 = n1 == -INFINITY ? 0.f : n1;
        const float al0 = exp2f(m0 - u0), al1 = exp2f(m1 - u1);
        const float p0 = exp2f(x0 - u0), p1 = exp2f(x1 - u1);
        const float p2 = exp2f(x2 - u0), p3 = exp2f(x3 - u1);
        m0 = n0; m1 = n1;
        l0 = l0 * al0 + (p0 + p2);
        l1 = l1 * al1 + (p1 + p3);
#pragma unroll
        for (int mt = 0; mt < 16; ++mt) {
            acc[mt][0] *= al0; acc[mt][1] *= al1; acc[mt][2] *= al0; acc[mt][3] *= al1;
        }
        const uint32_t pb0 = movmatrix_t(pack_bf16(p0, p1));
        const uint32_t pb1 = movmatrix_t(pack_bf16(p2, p3));
        if (valid < GQA_TILE) {
            // rows past the end of the request are never weighted; clear them
            // so stale non-finite cache contents cannot leak through 0 * inf
            uint8_t *vgen = wbuf + (size_t)s * 2 * GQA_TILE_BYTES + GQA_TILE_BYTES;
            for (int i = lane; i < (GQA_TILE - valid) * 32; i += 32) {
                const int row = valid + (i >> 5), c = (i & 31) >> 3, ch = i & 7;
                *reinterpret_cast<uint4 *>(vgen + c * 2048 + row * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
        }
        // O^T[256 dims x 8 heads] += V^T[256 x 16 tok] . P^T[16 tok x 8 heads]
        {
            const int tok = (mi >> 1) * 8 + r8;
#pragma unroll
            for (int mt = 0; mt < 16; ++mt) {
                const int chunk = (mt & 3) * 2 + (mi & 1);
                const uint32_t addr = vb + (mt >> 2) * 2048 + tok * 128 + ((chunk ^ (tok & 7)) << 4);
                uint32_t a0, a1, a2, a3;
                ldsm_x4_t(addr, a0, a1, a2, a3);
                mma_bf16_16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
            }
        }
        __syncwarp();
        if (lane == 0 && it + STAGES < my_tiles) {
            fence_proxy_async();
            issue(it + STAGES);
        }
    }
#pragma unroll
    for (int o = 4; o <= 16; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }

    // ---- merge the warps' partials in shared memory (stage buffers reused)
    __syncthreads();
    float *Osm = reinterpret_cast<float *>(smem);               // [WARPS][8][256]
    float *MLsm = Osm + WARPS * GQA_GRP * GQA_HD;                // [WARPS][8][2]
    {
        float *O = Osm + warp * GQA_GRP * GQA_HD;
        const int h0 = (lane & 3) * 2, dr = lane >> 2;
#pragma unroll
        for (int mt = 0; mt < 16; ++mt) {
            O[h0 * GQA_HD + mt * 16 + dr] = acc[mt][0];
            O[(h0 + 1) * GQA_HD + mt * 16 + dr] = acc[mt][1];
            O[h0 * GQA_HD + mt * 16 + dr + 8] = acc[mt][2];
            O[(h0 + 1) * GQA_HD + mt * 16 + dr + 8] = acc[mt][3];
        }
        if (lane < 4) {
            MLsm[(warp * GQA_GRP + h0) * 2] = m0;
            MLsm[(warp * GQA_GRP + h0) * 2 + 1] = l0;
            MLsm[(warp * GQA_GRP + h0 + 1) * 2] = m1;
            MLsm[(warp * GQA_GRP + h0 + 1) * 2 + 1] = l1;
        }
    }
    __syncthreads();
    const size_t pidx = (((size_t)n * KH + kh) * p.n_splits + split) * GQA_GRP;
    for (int i = tid; i < GQA_GRP * GQA_HD; i += WARPS * 32) {
        const int h = i / GQA_HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < WARPS; ++w) M = fmaxf(M, MLsm[(w * GQA_GRP + h) * 2]);
        float o = 0.f, L = 0.f;
#pragma unroll
        for (int w = 0; w < WARPS; ++w) {
            const float mw = MLsm[(w * GQA_GRP + h) * 2];
            const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
            o += Osm[(w * GQA_GRP + h) * GQA_HD + (i % GQA_HD)] * f;
            L += MLsm[(w * GQA_GRP + h) * 2 + 1] * f;
        }
        p.part_o[pidx * GQA_HD + i] = o;
        if ((i % GQA_HD) == 0) {
            p.part_ml[(pidx + h) * 2] = M;
            p.part_ml[(pidx + h) * 2 + 1] = L;
        }
    }
}

// ------------------------------------------------------------------ combine
// One CTA per (request, query head), 256 threads. Warp w merges the splits
// w, w + 8, .. with a running maximum (lane = 8 head dims, all of a warp's
// loads independent of each other), then thread d merges the 8 warp partials
// of dim d from shared memory: the loads of one request's splits are spread
// over the warps instead of two serial passes of every thread over all splits
// (a single request at 32k context has 74 splits).
template <typename TI, typename TO>
__global__ void __launch_bounds__(GQA_HD)
gqa_combine_kernel(GqaCombineArgs p)
{
    constexpr int CW = GQA_HD / 32;      // warps
    __shared__ float sm_ml[CW][2];
    __shared__ __align__(16) float sm_o[CW][GQA_HD];
    const int n = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // The gate is a caller input, complete before the prologue (a plain
    // launch) started and so before this kernel could: it is read ahead of
    // the wait for the split partials.
    const float gate = to_f32(static_cast<const TI *>(p.qg)[((size_t)n * p.H + h) * 2 * GQA_HD + GQA_HD + tid]);
    griddep_wait();      // launched as a programmatic dependent of the split kernel
    const int kh = h / GQA_GRP, hl = h % GQA_GRP;
    const size_t base = ((size_t)n * p.KH + kh) * p.n_splits;
    float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = 0.f;
    constexpr int CU = 4;                // splits whose loads a warp issues together
    for (int s0 = warp; s0 < p.n_splits; s0 += CU * CW) {
        float2 ml[CU];
        float4 a[CU], b[CU];
#pragma unroll
        for (int u = 0; u < CU; ++u) {
            const int s = s0 + u * CW;
            ml[u] = make_float2(-INFINITY, 0.f);
            if (s < p.n_splits) {
                const size_t pi = (base + s) * GQA_GRP + hl;
                ml[u] = *reinterpret_cast<const float2 *>(p.part_ml + pi * 2);
                a[u] = *reinterpret_cast<const float4 *>(p.part_o + pi * GQA_HD + 8 * lane);
                b[u] = *reinterpret_cast<const float4 *>(p.part_o + pi * GQA_HD + 8 * lane + 4);
            }
        }
#pragma unroll
        for (int u = 0; u < CU; ++u) {
            if (ml[u].x == -INFINITY) continue;             // no keys for this row (or past the last split)
            const float mn = fmaxf(m, ml[u].x);
            const float fo = m == -INFINITY ? 0.f : exp2f(m - mn), fs = exp2f(ml[u].x - mn);
            const float x[8] = {a[u].x, a[u].y, a[u].z, a[u].w, b[u].x, b[u].y, b[u].z, b[u].w};
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = o[i] * fo + x[i] * fs;
            l = l * fo + ml[u].y * fs;
            m = mn;
        }
    }
    if (lane == 0) { sm_ml[warp][0] = m; sm_ml[warp][1] = l; }
    *reinterpret_cast<float4 *>(&sm_o[warp][8 * lane]) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4 *>(&sm_o[warp][8 * lane + 4]) = make_float4(o[4], o[5], o[6], o[7]);
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < CW; ++w) M = fmaxf(M, sm_ml[w][0]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < CW; ++w) {
        const float mw = sm_ml[w][0];
        const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
        O += sm_o[w][tid] * f;
        L += sm_ml[w][1] * f;
    }
    static_cast<TO *>(p.ctx)[((size_t)n * p.H + h) * GQA_HD + tid] = from_f32<TO>(O / L * sigmoidf_(gate));
}

// ------------------------------------------------------------------ launch
constexpr int SPLIT_WARPS = 4, SPLIT_STAGES = 3;

size_t gqa_split_smem_bytes()
{
    size_t ring = (size_t)SPLIT_WARPS * SPLIT_STAGES * 2 * GQA_TILE_BYTES;
    size_t merge = (size_t)SPLIT_WARPS * GQA_GRP * (GQA_HD + 2) * 4;
    return (ring > merge ? ring : merge) + 1024;
}

cudaError_t launch_gqa_prologue(const GqaPrologueArgs &a, int in_bf16, cudaStream_t st)
{
    const uintptr_t al = (uintptr_t)a.qg | (uintptr_t)a.k | (uintptr_t)a.v | (uintptr_t)a.qnw |
                         (uintptr_t)a.knw | (uintptr_t)a.qout | (uintptr_t)a.kcache | (uintptr_t)a.vcache;
    if ((al & 15) == 0) {
        // rows per CTA: 4 once there are enough rows to fill the GPU, else 1 (latency)
        const int rpc = a.nq >= 2048 ? GQA_PRO_ROWS : 1;
        const int blocks = (a.nq + rpc - 1) / rpc;
        if (in_bf16) gqa_prologue_warp_kernel<__nv_bfloat16><<<blocks, GQA_PRO_WARPS * 32, 0, st>>>(a, rpc);
        else gqa_prologue_warp_kernel<float><<<blocks, GQA_PRO_WARPS * 32, 0, st>>>(a, rpc);
        return cudaGetLastError();
    }
    dim3 grid(a.nq, a.H + a.KH);
    if (in_bf16) gqa_prologue_kernel<__nv_bfloat16><<<grid, GQA_HD, 0, st>>>(a);
    else gqa_prologue_kernel<float><<<grid, GQA_HD, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_gqa_split(const CUtensorMap &tk, const CUtensorMap &tv, const GqaSplitArgs &a,
                             cudaStream_t st)
{
    if (a.fuse < 0 || a.fuse > 2) return cudaErrorInvalidValue;
    auto kern = a.fuse == 0 ? gqa_split_kernel<SPLIT_WARPS, SPLIT_STAGES, 0>
              : a.fuse == 1 ? gqa_split_kernel<SPLIT_WARPS, SPLIT_STAGES, 1>
                            : gqa_split_kernel<SPLIT_WARPS, SPLIT_STAGES, 2>;
    const size_t smem = gqa_split_smem_bytes();
    static bool attr_done[3] = {false, false, false};
    if (!attr_done[a.fuse]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr_done[a.fuse] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_splits, a.KH, a.nq); cfg.blockDim = dim3(SPLIT_WARPS * 32);
    cfg.dynamicSmemBytes = smem; cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // a dependent of the prologue (or, fused, of the inputs' producer)
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr; cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tk, tv, a);
}

cudaError_t launch_gqa_combine(const GqaCombineArgs &a, int in_bf16, int out_bf16, cudaStream_t st)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nq, a.H); cfg.blockDim = dim3(GQA_HD); cfg.dynamicSmemBytes = 0; cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // a dependent of the split kernel
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr; cfg.numAttrs = 1;
    if (in_bf16 && out_bf16) return cudaLaunchKernelEx(&cfg, gqa_combine_kernel<__nv_bfloat16, __nv_bfloat16>, a);
    if (!in_bf16 && !out_bf16) return cudaLaunchKernelEx(&cfg, gqa_combine_kernel<float, float>, a);
    return cudaErrorInvalidValue;
}

int gqa_pick_splits(int nq, int KH, int tmax, int num_sms)
{
    const int tiles = (tmax + GQA_TILE - 1) / GQA_TILE;
    int best = 1;
    double best_eff = -1.0;
    for (int s = 1; s <= 256; ++s) {
        const int per = (tiles + s - 1) / s;        // tiles per CTA
        // keep every warp busy for >= 2 tiles, or >= 1 while the grid is far
        // below one wave (a single request at short context: latency bound)
        const bool small = (long)nq * KH * s * 2 <= num_sms;
        if (s > 1 && per < (small ? SPLIT_WARPS : 2 * SPLIT_WARPS)) break;
        const long ctas = (long)nq * KH * s;
        const long waves = (ctas + num_sms - 1) / num_sms;
        // wave-quantisation efficiency, with a mild preference for fewer splits
        const double eff = (double)ctas / (double)(waves * num_sms) - 0.002 * s;
        if (eff > best_eff + 1e-9) { best_eff = eff; best = s; }
    }
    return best;
}

int gqa_chunk_for(int tmax, int n_splits)
{
    const int tiles = (tmax + GQA_TILE - 1) / GQA_TILE;
    return ((tiles + n_splits - 1) / n_splits) * GQA_TILE;
}

}  // namespace coli
