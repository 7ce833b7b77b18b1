// GatedDeltaNet prefill: the reference's S sequential gdn_step calls
// (c/qwen.c:1376-1380) computed chunk-parallel, 64 tokens per chunk.
//
// Per V head h (K head h/2), token t: S_t = g_t S_{t-1} + k_t d_t^T with
// d_t = beta_t (v_t - g_t S_{t-1}^T k_t) and y_t = S_t^T q_t (c/qwen.c:748-767).
// Inside a chunk with initial state S0 and inclusive cumulative log decay G_i
// (gamma_i = exp(G_i)), the recurrence unrolls exactly to
//   (I + A) D = beta (V - diag(gamma) K S0),  A_ij = beta_i e^{G_i-G_j} k_i.k_j (j < i)
//   D = U - W S0,  U = T beta V,  W = T beta gamma K,  T = (I + A)^-1
//   Y = diag(gamma) Q S0 + M D,   M_ij = e^{G_i-G_j} q_i.k_j (j <= i)
//   S_end = gamma_C S0 + K^T (e^{G_C-G} D)
// (exact algebra on the reference recurrence; only the arithmetic precision
// differs). y is then gated: y * rsqrt(mean y^2 + eps) * gnorm * silu(z)
// (c/qwen.c:768-772). Rows past S in the last chunk behave as identity tokens
// (decay 1, beta 0, zero q/k/v: TMA zero-fills them), so they change nothing.
//
// Kernels
//   gdn_pf_prologue_kernel  per (token, K head): conv4 over the token and its
//                           3 predecessors (or the carried history) + SiLU,
//                           q/k L2 norm, gates -> Q, K, V (fp32, head-major),
//                           log-decay and beta per V head.
//   gdn_pf_hist_kernel      carries the last 3 pre-conv rows out as history.
//   gdn_pf_prep_kernel      per (chunk, V head), fully parallel: K K^T and
//                           Q K^T on tf32 mma.sync, T by forward substitution
//                           in fp32, then W, U and the decay-masked M.
//   gdn_pf_scan_kernel      per (V head, 32-column block of the state), a
//                           cluster of the 4 column blocks of a head; walks
//                           the chunks in order with the state slice in mma
//                           accumulators; the gated-RMSNorm statistic goes
//                           through distributed shared memory. Operands
//                           arrive by TMA (128B swizzle, no multicast), each
//                           with its own barrier, so the next chunk's loads
//                           overlap the current chunk's later phases.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace coli {

constexpr int PFG_C = 64, PFG_D = 128;

// ---------------------------------------------------------------- tf32 MMA
__device__ __forceinline__ uint32_t f2tf32(float x)
{
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
// D[16x8] += A[16x8] . B[8x8] in tf32 with fp32 accumulation.
__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7},"
        " {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Element (row, col) of an fp32 tile that TMA wrote as 32-column boxes of
// `rows` rows with the 128B swizzle (16B chunk index XOR row % 8).
__device__ __forceinline__ float sw_ld(const float *tile, int rows, int row, int col)
{
    const int region = col >> 5, c = col & 31;
    return tile[region * rows * 32 + row * 32 + (((c >> 2) ^ (row & 7)) << 2) + (c & 3)];
}

// Inclusive cumulative sum of the log decay of one chunk (one warp, 2 rows/lane).
__device__ __forceinline__ void chunk_cumsum(const float *gl, int t0, int S, int lane, float *dst)
{
    float g0 = 0.f, g1 = 0.f;
    const int i0 = 2 * lane;
    if (t0 + i0 < S) g0 = gl[t0 + i0];
    if (t0 + i0 + 1 < S) g1 = gl[t0 + i0 + 1];
    float sum = g0 + g1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, sum, o);
        if (lane >= o) sum += v;
    }
    const float excl = sum - (g0 + g1);
    dst[i0] = excl + g0;
    dst[i0 + 1] = excl + g0 + g1;
}

// ---------------------------------------------------------------- prologue
template <typename TI>
__global__ void __launch_bounds__(PFG_D)
gdn_pf_prologue_kernel(GdnPrefillArgs p)
{
    const int s = blockIdx.x, kh = blockIdx.y, t = threadIdx.x;
    const int S = p.S;
    const int KHin = p.KHin ? p.KHin : p.KH, VHin = p.VHin ? p.VHin : p.VH;
    const int kg = p.kh0 + kh;                    // K head in the input layout
    const int key_dim = KHin * PFG_D, CD = 2 * key_dim + VHin * PFG_D;
    const TI *x = static_cast<const TI *>(p.qkv);
    auto tap = [&](int ch, int j) -> float {  // pre-conv value of channel ch at token s-3+j
        const int ts = s - 3 + j;
        return ts >= 0 ? to_f32(x[(size_t)ts * CD + ch]) : p.hist[(size_t)(3 + ts) * CD + ch];
    };
    auto conv = [&](int ch) -> float {
        const float4 w = *reinterpret_cast<const float4 *>(p.conv_w + (size_t)ch * 4);
        float a = 0.f;
        a += w.x * tap(ch, 0); a += w.y * tap(ch, 1); a += w.z * tap(ch, 2); a += w.w * tap(ch, 3);
        return siluf_(a);
    };
    const float qc = conv(kg * PFG_D + t), kc = conv(key_dim + kg * PFG_D + t);
    __shared__ float red[2][4];
    float sq = qc * qc, sk = kc * kc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    if ((t & 31) == 0) { red[0][t >> 5] = sq; red[1][t >> 5] = sk; }
    __syncthreads();
    sq = (red[0][0] + red[0][1]) + (red[0][2] + red[0][3]);
    sk = (red[1][0] + red[1][1]) + (red[1][2] + red[1][3]);
    const float rq = 1.f / sqrtf(sq + p.eps) / sqrtf((float)PFG_D);
    const float rk = 1.f / sqrtf(sk + p.eps);
    p.Qh[((size_t)kh * S + s) * PFG_D + t] = qc * rq;
    p.Kh[((size_t)kh * S + s) * PFG_D + t] = kc * rk;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int vh = kh * 2 + j, vg = kg * 2 + j;  // local / input-layout V head
        p.Vh[((size_t)vh * S + s) * PFG_D + t] = conv(2 * key_dim + vg * PFG_D + t);
        if (t == 0) {
            const float av = to_f32(static_cast<const TI *>(p.a)[(size_t)s * VHin + vg]);
            const float bv = to_f32(static_cast<const TI *>(p.b)[(size_t)s * VHin + vg]);
            // log of the reference's decay exp(-exp(A_log) * softplus(a + dt_bias))
            p.GL[(size_t)vh * S + s] = -expf(p.A_log[vg]) * softplusf_(av + p.dt_bias[vg]);
            p.BETA[(size_t)vh * S + s] = sigmoidf_(bv);
        }
    }
}

// New conv history = the last 3 pre-conv rows of the owned channels. Needs
// S >= 3 (the host routes shorter runs through the token-by-token decode kernel).
template <typename TI>
__global__ void gdn_pf_hist_kernel(GdnPrefillArgs p)
{
    const int KHin = p.KHin ? p.KHin : p.KH, VHin = p.VHin ? p.VHin : p.VH;
    const int key_dim = KHin * PFG_D, CD = 2 * key_dim + VHin * PFG_D;
    const int q0 = p.kh0 * PFG_D, q1 = q0 + p.KH * PFG_D;
    const int v0 = 2 * key_dim + 2 * p.kh0 * PFG_D, v1 = v0 + 2 * p.KH * PFG_D;
    const TI *x = static_cast<const TI *>(p.qkv);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 3 * CD; i += gridDim.x * blockDim.x) {
        const int j = i / CD, ch = i - j * CD;
        const bool own = (ch >= q0 && ch < q1) || (ch >= key_dim + q0 && ch < key_dim + q1) ||
                         (ch >= v0 && ch < v1);
        if (own) p.hist[i] = to_f32(x[(size_t)(p.S - 3 + j) * CD + ch]);
    }
}

// ---------------------------------------------------------------- chunk prep
constexpr int PREP_LD = 68;  // padded row stride (floats) of A / T in shared memory

__global__ void __launch_bounds__(128)
gdn_pf_prep_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, GdnPrefillArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    float *base = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *sQV = base;                          // Q chunk, later V chunk [64 x 128] swizzled
    float *sK = sQV + PFG_C * PFG_D;            // K chunk
    float *sA = sK + PFG_C * PFG_D;             // [64][68] strictly lower A
    float *sT = sA + PFG_C * PREP_LD;           // [64][68] T = (I + A)^-1
    __shared__ float G[PFG_C], bet[PFG_C];
    __shared__ __align__(8) uint64_t bar_qk, bar_v;

    const int n = blockIdx.x, h = blockIdx.y, kh = h >> 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
    const int s0 = n * PFG_C;
    if (tid == 0) {
        mbar_init(&bar_qk, 1);
        mbar_init(&bar_v, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_expect_tx(&bar_qk, 2 * PFG_C * PFG_D * 4);
        for (int c = 0; c < 4; ++c) {
            tma_load_3d(sQV + c * PFG_C * 32, &tmQ, 32 * c, s0, kh, &bar_qk);
            tma_load_3d(sK + c * PFG_C * 32, &tmK, 32 * c, s0, kh, &bar_qk);
        }
    }
    if (warp == 0) {
        chunk_cumsum(p.GL + (size_t)h * p.S, s0, p.S, lane, G);
    } else if (warp == 1) {
        for (int i = lane; i < PFG_C; i += 32)
            bet[i] = (s0 + i < p.S) ? p.BETA[(size_t)h * p.S + s0 + i] : 0.f;
    }
    __syncthreads();
    mbar_wait(&bar_qk, 0);  // a time-out raises the device error word

    // K K^T and Q K^T for this warp's 16 rows, all 64 columns
    const int r0 = warp * 16;
    {
        float kk[8][4], qk[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) kk[nt][e] = qk[nt][e] = 0.f;
#pragma unroll 4
        for (int ks = 0; ks < PFG_D / 8; ++ks) {
            const int c0 = ks * 8 + tq, c1 = c0 + 4;
            const uint32_t ak0 = f2tf32(sw_ld(sK, PFG_C, r0 + g, c0)), ak1 = f2tf32(sw_ld(sK, PFG_C, r0 + g + 8, c0));
            const uint32_t ak2 = f2tf32(sw_ld(sK, PFG_C, r0 + g, c1)), ak3 = f2tf32(sw_ld(sK, PFG_C, r0 + g + 8, c1));
            const uint32_t aq0 = f2tf32(sw_ld(sQV, PFG_C, r0 + g, c0)), aq1 = f2tf32(sw_ld(sQV, PFG_C, r0 + g + 8, c0));
            const uint32_t aq2 = f2tf32(sw_ld(sQV, PFG_C, r0 + g, c1)), aq3 = f2tf32(sw_ld(sQV, PFG_C, r0 + g + 8, c1));
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const uint32_t b0 = f2tf32(sw_ld(sK, PFG_C, nt * 8 + g, c0));
                const uint32_t b1 = f2tf32(sw_ld(sK, PFG_C, nt * 8 + g, c1));
                mma_tf32(kk[nt], ak0, ak1, ak2, ak3, b0, b1);
                mma_tf32(qk[nt], aq0, aq1, aq2, aq3, b0, b1);
            }
        }
        float *Mg = p.M + ((size_t)n * p.VH + h) * PFG_C * PFG_C;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = r0 + g + ((e >> 1) << 3), j = nt * 8 + 2 * tq + (e & 1);
                const float dec = expf(G[i] - G[j]);
                sA[i * PREP_LD + j] = j < i ? bet[i] * dec * kk[nt][e] : 0.f;
                Mg[i * PFG_C + j] = j <= i ? dec * qk[nt][e] : 0.f;
            }
        }
    }
    __syncthreads();
    // V replaces Q in shared memory while T is solved
    if (tid == 0) {
        fence_proxy_async();
        mbar_expect_tx(&bar_v, PFG_C * PFG_D * 4);
        for (int c = 0; c < 4; ++c) tma_load_3d(sQV + c * PFG_C * 32, &tmV, 32 * c, s0, h, &bar_v);
    }
    // T = (I + A)^-1 by forward substitution, one column per thread
    if (tid < PFG_C) {
        const int c = tid;
        for (int i = 0; i < PFG_C; ++i) {
            // four independent partial sums shorten the dependent FMA chain
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            int j = c;
            for (; j + 3 < i; j += 4) {
                a0 += sA[i * PREP_LD + j] * sT[j * PREP_LD + c];
                a1 += sA[i * PREP_LD + j + 1] * sT[(j + 1) * PREP_LD + c];
                a2 += sA[i * PREP_LD + j + 2] * sT[(j + 2) * PREP_LD + c];
                a3 += sA[i * PREP_LD + j + 3] * sT[(j + 3) * PREP_LD + c];
            }
            for (; j < i; ++j) a0 += sA[i * PREP_LD + j] * sT[j * PREP_LD + c];
            const float acc = ((i == c) ? 1.f : 0.f) - ((a0 + a1) + (a2 + a3));
            sT[i * PREP_LD + c] = i < c ? 0.f : acc;
        }
    }
    __syncthreads();
    mbar_wait(&bar_v, 0);

    // W = T (beta gamma K), U = T (beta V) for this warp's 16 rows, 128 columns
    float *Wg = p.W + ((size_t)n * p.VH + h) * PFG_C * PFG_D;
    float *Ug = p.U + ((size_t)n * p.VH + h) * PFG_C * PFG_D;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
        float w[8][4], u[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) w[nt][e] = u[nt][e] = 0.f;
#pragma unroll 2
        for (int ks = 0; ks < PFG_C / 8; ++ks) {
            const int c0 = ks * 8 + tq, c1 = c0 + 4;
            const uint32_t a0 = f2tf32(sT[(r0 + g) * PREP_LD + c0]), a1 = f2tf32(sT[(r0 + g + 8) * PREP_LD + c0]);
            const uint32_t a2 = f2tf32(sT[(r0 + g) * PREP_LD + c1]), a3 = f2tf32(sT[(r0 + g + 8) * PREP_LD + c1]);
            const float bg0 = bet[c0] * expf(G[c0]), bg1 = bet[c1] * expf(G[c1]);
            const float bb0 = bet[c0], bb1 = bet[c1];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int col = half * 64 + nt * 8 + g;
                const uint32_t bk0 = f2tf32(bg0 * sw_ld(sK, PFG_C, c0, col));
                const uint32_t bk1 = f2tf32(bg1 * sw_ld(sK, PFG_C, c1, col));
                const uint32_t bv0 = f2tf32(bb0 * sw_ld(sQV, PFG_C, c0, col));
                const uint32_t bv1 = f2tf32(bb1 * sw_ld(sQV, PFG_C, c1, col));
                mma_tf32(w[nt], a0, a1, a2, a3, bk0, bk1);
                mma_tf32(u[nt], a0, a1, a2, a3, bv0, bv1);
            }
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int col = half * 64 + nt * 8 + 2 * tq;
            const int ra = r0 + g, rb = ra + 8;
            *reinterpret_cast<float2 *>(Wg + ra * PFG_D + col) = make_float2(w[nt][0], w[nt][1]);
            *reinterpret_cast<float2 *>(Wg + rb * PFG_D + col) = make_float2(w[nt][2], w[nt][3]);
            *reinterpret_cast<float2 *>(Ug + ra * PFG_D + col) = make_float2(u[nt][0], u[nt][1]);
            *reinterpret_cast<float2 *>(Ug + rb * PFG_D + col) = make_float2(u[nt][2], u[nt][3]);
        }
    }
}

// ---------------------------------------------------------------- chunk scan
constexpr int SCAN_CB = 32;   // state columns per CTA
constexpr int SCAN_LD = 40;   // padded row stride of the h / D operand tiles

template <typename TI, typename TO>
__global__ void __cluster_dims__(4, 1, 1) __launch_bounds__(128, 1)
gdn_pf_scan_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmU,
                   const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmM,
                   const __grid_constant__ CUtensorMap tmK, GdnPrefillArgs p)
{
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ uint8_t smem_raw[];
    float *base = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *sW = base;                         // [64 x 128] swizzled
    float *sQ = sW + PFG_C * PFG_D;           // [64 x 128]
    float *sK = sQ + PFG_C * PFG_D;           // [64 x 128]
    float *sM = sK + PFG_C * PFG_D;           // [64 x 64]
    float *sU = sM + PFG_C * PFG_C;           // [64 x 32]
    float *sH = sU + PFG_C * SCAN_CB;         // h as [dk 128][40]
    float *sD = sH + PFG_D * SCAN_LD;         // D as [token 64][40]
    float *sDt = sD + PFG_C * SCAN_LD;        // e^{G_C - G} D as [token 64][40]
    __shared__ float G[2][PFG_C];
    __shared__ float ss[2][PFG_C];
    __shared__ __align__(8) uint64_t bar_wu, bar_qm, bar_k;

    const int cblk = blockIdx.x & 3, h = blockIdx.x >> 2, kh = h >> 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
    const int S = p.S, nchunks = (S + PFG_C - 1) / PFG_C;
    const int VD = PFG_D, VH = p.VH;
    const int VHin = p.VHin ? p.VHin : VH, vg = 2 * p.kh0 + h;  // V head in the input layout

    auto load_wu = [&](int n) {
        mbar_expect_tx(&bar_wu, (PFG_C * PFG_D + PFG_C * SCAN_CB) * 4);
        for (int c = 0; c < 4; ++c) tma_load_3d(sW + c * PFG_C * 32, &tmW, 32 * c, 0, n * VH + h, &bar_wu);
        tma_load_3d(sU, &tmU, 32 * cblk, 0, n * VH + h, &bar_wu);
    };
    auto load_qm = [&](int n) {
        mbar_expect_tx(&bar_qm, (PFG_C * PFG_D + PFG_C * PFG_C) * 4);
        for (int c = 0; c < 4; ++c) tma_load_3d(sQ + c * PFG_C * 32, &tmQ, 32 * c, n * PFG_C, kh, &bar_qm);
        for (int c = 0; c < 2; ++c) tma_load_3d(sM + c * PFG_C * 32, &tmM, 32 * c, 0, n * VH + h, &bar_qm);
    };
    auto load_k = [&](int n) {
        mbar_expect_tx(&bar_k, PFG_C * PFG_D * 4);
        for (int c = 0; c < 4; ++c) tma_load_3d(sK + c * PFG_C * 32, &tmK, 32 * c, n * PFG_C, kh, &bar_k);
    };

    if (tid == 0) {
        mbar_init(&bar_wu, 1); mbar_init(&bar_qm, 1); mbar_init(&bar_k, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) { load_wu(0); load_qm(0); load_k(0); }
    if (warp == 0) chunk_cumsum(p.GL + (size_t)h * S, 0, S, lane, G[0]);

    // state slice: warp owns dk rows 32w..32w+31 (2 m-tiles) x 32 columns (4 n-tiles)
    float hs[2][4][4];
    float *state = p.state + (size_t)h * PFG_D * VD + cblk * SCAN_CB;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const int ra = warp * 32 + mt * 16 + g, col = nt * 8 + 2 * tq;
            const float2 x0 = *reinterpret_cast<const float2 *>(state + (size_t)ra * VD + col);
            const float2 x1 = *reinterpret_cast<const float2 *>(state + (size_t)(ra + 8) * VD + col);
            hs[mt][nt][0] = x0.x; hs[mt][nt][1] = x0.y; hs[mt][nt][2] = x1.x; hs[mt][nt][3] = x1.y;
            *reinterpret_cast<float2 *>(sH + ra * SCAN_LD + col) = x0;
            *reinterpret_cast<float2 *>(sH + (ra + 8) * SCAN_LD + col) = x1;
        }
    __syncthreads();

    const int r0 = warp * 16;  // this warp's token rows in phases (a) and (b)
    // A timed-out wait raises the device error word; the loop still runs to
    // the end so that every CTA of the cluster meets every cluster barrier.
    for (int n = 0; n < nchunks; ++n) {
        const int par = n & 1;
        const float *Gc = G[par];
        // ---- (a) D = U - W h   (accumulated as W h - U, negated below)
        mbar_wait(&bar_wu, par);
        float d[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const int col = nt * 8 + 2 * tq;
            d[nt][0] = -sw_ld(sU, PFG_C, r0 + g, col);     d[nt][1] = -sw_ld(sU, PFG_C, r0 + g, col + 1);
            d[nt][2] = -sw_ld(sU, PFG_C, r0 + g + 8, col); d[nt][3] = -sw_ld(sU, PFG_C, r0 + g + 8, col + 1);
        }
#pragma unroll 4
        for (int ks = 0; ks < PFG_D / 8; ++ks) {
            const int c0 = ks * 8 + tq, c1 = c0 + 4;
            const uint32_t a0 = f2tf32(sw_ld(sW, PFG_C, r0 + g, c0)), a1 = f2tf32(sw_ld(sW, PFG_C, r0 + g + 8, c0));
            const uint32_t a2 = f2tf32(sw_ld(sW, PFG_C, r0 + g, c1)), a3 = f2tf32(sw_ld(sW, PFG_C, r0 + g + 8, c1));
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const uint32_t b0 = f2tf32(sH[c0 * SCAN_LD + nt * 8 + g]);
                const uint32_t b1 = f2tf32(sH[c1 * SCAN_LD + nt * 8 + g]);
                mma_tf32(d[nt], a0, a1, a2, a3, b0, b1);
            }
        }
        {
            const float gC = Gc[PFG_C - 1];
            const float sa = expf(gC - Gc[r0 + g]), sb = expf(gC - Gc[r0 + g + 8]);
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const int col = nt * 8 + 2 * tq;
                const float D0 = -d[nt][0], D1 = -d[nt][1], D2 = -d[nt][2], D3 = -d[nt][3];
                *reinterpret_cast<float2 *>(sD + (r0 + g) * SCAN_LD + col) = make_float2(D0, D1);
                *reinterpret_cast<float2 *>(sD + (r0 + g + 8) * SCAN_LD + col) = make_float2(D2, D3);
                *reinterpret_cast<float2 *>(sDt + (r0 + g) * SCAN_LD + col) = make_float2(D0 * sa, D1 * sa);
                *reinterpret_cast<float2 *>(sDt + (r0 + g + 8) * SCAN_LD + col) = make_float2(D2 * sb, D3 * sb);
            }
        }
        __syncthreads();                                   // D complete; W/U free
        if (tid == 0 && n + 1 < nchunks) { fence_proxy_async(); load_wu(n + 1); }

        // ---- (b) Y = diag(gamma) Q h + M D
        mbar_wait(&bar_qm, par);
        float y[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) y[nt][0] = y[nt][1] = y[nt][2] = y[nt][3] = 0.f;
#pragma unroll 4
        for (int ks = 0; ks < PFG_D / 8; ++ks) {
            const int c0 = ks * 8 + tq, c1 = c0 + 4;
            const uint32_t a0 = f2tf32(sw_ld(sQ, PFG_C, r0 + g, c0)), a1 = f2tf32(sw_ld(sQ, PFG_C, r0 + g + 8, c0));
            const uint32_t a2 = f2tf32(sw_ld(sQ, PFG_C, r0 + g, c1)), a3 = f2tf32(sw_ld(sQ, PFG_C, r0 + g + 8, c1));
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const uint32_t b0 = f2tf32(sH[c0 * SCAN_LD + nt * 8 + g]);
                const uint32_t b1 = f2tf32(sH[c1 * SCAN_LD + nt * 8 + g]);
                mma_tf32(y[nt], a0, a1, a2, a3, b0, b1);
            }
        }
        {
            const float ga = expf(Gc[r0 + g]), gb = expf(Gc[r0 + g + 8]);
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) { y[nt][0] *= ga; y[nt][1] *= ga; y[nt][2] *= gb; y[nt][3] *= gb; }
        }
#pragma unroll 2
        for (int ks = 0; ks < PFG_C / 8; ++ks) {
            const int c0 = ks * 8 + tq, c1 = c0 + 4;
            const uint32_t a0 = f2tf32(sw_ld(sM, PFG_C, r0 + g, c0)), a1 = f2tf32(sw_ld(sM, PFG_C, r0 + g + 8, c0));
            const uint32_t a2 = f2tf32(sw_ld(sM, PFG_C, r0 + g, c1)), a3 = f2tf32(sw_ld(sM, PFG_C, r0 + g + 8, c1));
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const uint32_t b0 = f2tf32(sD[c0 * SCAN_LD + nt * 8 + g]);
                const uint32_t b1 = f2tf32(sD[c1 * SCAN_LD + nt * 8 + g]);
                mma_tf32(y[nt], a0, a1, a2, a3, b0, b1);
            }
        }
        // partial sum of squares of this CTA's 32 columns, per token row
        {
            float sa = 0.f, sb = 0.f;
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                sa += y[nt][0] * y[nt][0] + y[nt][1] * y[nt][1];
                sb += y[nt][2] * y[nt][2] + y[nt][3] * y[nt][3];
            }
            sa += __shfl_xor_sync(0xffffffffu, sa, 1); sa += __shfl_xor_sync(0xffffffffu, sa, 2);
            sb += __shfl_xor_sync(0xffffffffu, sb, 1); sb += __shfl_xor_sync(0xffffffffu, sb, 2);
            if (tq == 0) { ss[par][r0 + g] = sa; ss[par][r0 + g + 8] = sb; }
        }
        __syncthreads();                                   // Q/M and sH reads done
        if (tid == 0 && n + 1 < nchunks) { fence_proxy_async(); load_qm(n + 1); }
        asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");

        // ---- (c) h = gamma_C h + K^T (e^{G_C - G} D)
        mbar_wait(&bar_k, par);
        {
            const float gam = expf(Gc[PFG_C - 1]);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) hs[mt][nt][e] *= gam;
        }
#pragma unroll 2
        for (int ks = 0; ks < PFG_C / 8; ++ks) {
            const int c0 = ks * 8 + tq, c1 = c0 + 4;   // token index (k dimension)
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const int ra = warp * 32 + mt * 16 + g;  // dk row
                const uint32_t a0 = f2tf32(sw_ld(sK, PFG_C, c0, ra)), a1 = f2tf32(sw_ld(sK, PFG_C, c0, ra + 8));
                const uint32_t a2 = f2tf32(sw_ld(sK, PFG_C, c1, ra)), a3 = f2tf32(sw_ld(sK, PFG_C, c1, ra + 8));
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    const uint32_t b0 = f2tf32(sDt[c0 * SCAN_LD + nt * 8 + g]);
                    const uint32_t b1 = f2tf32(sDt[c1 * SCAN_LD + nt * 8 + g]);
                    mma_tf32(hs[mt][nt], a0, a1, a2, a3, b0, b1);
                }
            }
        }
        if (warp == 0 && n + 1 < nchunks) chunk_cumsum(p.GL + (size_t)h * S, (n + 1) * PFG_C, S, lane, G[par ^ 1]);
        __syncthreads();                                   // K, sDt reads done
        if (tid == 0 && n + 1 < nchunks) { fence_proxy_async(); load_k(n + 1); }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const int ra = warp * 32 + mt * 16 + g, col = nt * 8 + 2 * tq;
                *reinterpret_cast<float2 *>(sH + ra * SCAN_LD + col) = make_float2(hs[mt][nt][0], hs[mt][nt][1]);
                *reinterpret_cast<float2 *>(sH + (ra + 8) * SCAN_LD + col) = make_float2(hs[mt][nt][2], hs[mt][nt][3]);
            }

        // ---- gated RMSNorm over the head's 128 columns (4 CTAs) and output
        asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int i = r0 + g + 8 * half, t = n * PFG_C + i;
            float tot = 0.f;
#pragma unroll
            for (int r = 0; r < 4; ++r) tot += *cluster.map_shared_rank(&ss[par][i], r);
            const float rinv = 1.f / sqrtf(tot / VD + p.eps);
            if (t < S) {
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int col = cblk * SCAN_CB + nt * 8 + 2 * tq + e;
                        const float z = to_f32(static_cast<const TI *>(p.z)[(size_t)t * VHin * VD + vg * VD + col]);
                        const float out = y[nt][2 * half + e] * rinv * p.gnorm[col] * siluf_(z);
                        static_cast<TO *>(p.y)[(size_t)t * VH * VD + h * VD + col] = from_f32<TO>(out);
                    }
                }
            }
        }
        __syncthreads();                                   // sH rewritten for the next chunk
    }
    // final state back to HBM
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const int ra = warp * 32 + mt * 16 + g, col = nt * 8 + 2 * tq;
            *reinterpret_cast<float2 *>(state + (size_t)ra * VD + col) = make_float2(hs[mt][nt][0], hs[mt][nt][1]);
            *reinterpret_cast<float2 *>(state + (size_t)(ra + 8) * VD + col) = make_float2(hs[mt][nt][2], hs[mt][nt][3]);
        }
    cluster.sync();  // peers may still read this CTA's ss
}

// ---------------------------------------------------------------- launch
size_t gdn_prep_smem() { return (size_t)(2 * PFG_C * PFG_D + 2 * PFG_C * PREP_LD) * 4 + 1024; }
size_t gdn_scan_smem()
{
    return (size_t)(3 * PFG_C * PFG_D + PFG_C * PFG_C + PFG_C * SCAN_CB + PFG_D * SCAN_LD +
                    2 * PFG_C * SCAN_LD) * 4 + 1024;
}

cudaError_t launch_gdn_prefill(const GdnPrefillArgs &a, const GdnPrefillMaps &m, int bf16,
                               cudaStream_t st)
{
    if (a.S < 3) return cudaErrorInvalidValue;
    const int nchunks = (a.S + PFG_C - 1) / PFG_C;
    const int CD = 2 * (a.KHin ? a.KHin : a.KH) * PFG_D + (a.VHin ? a.VHin : a.VH) * PFG_D;
    cudaError_t e;
    if (bf16) gdn_pf_prologue_kernel<__nv_bfloat16><<<dim3(a.S, a.KH), PFG_D, 0, st>>>(a);
    else gdn_pf_prologue_kernel<float><<<dim3(a.S, a.KH), PFG_D, 0, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (bf16) gdn_pf_hist_kernel<__nv_bfloat16><<<(3 * CD + 255) / 256, 256, 0, st>>>(a);
    else gdn_pf_hist_kernel<float><<<(3 * CD + 255) / 256, 256, 0, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    e = cudaFuncSetAttribute(gdn_pf_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gdn_prep_smem());
    if (e != cudaSuccess) return e;
    gdn_pf_prep_kernel<<<dim3(nchunks, a.VH), 128, gdn_prep_smem(), st>>>(m.Q, m.K, m.V, a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    auto scan = [&](auto kern) -> cudaError_t {
        cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gdn_scan_smem());
        if (e2 != cudaSuccess) return e2;
        kern<<<a.VH * 4, 128, gdn_scan_smem(), st>>>(m.W, m.U, m.Q, m.M, m.K, a);
        return cudaGetLastError();
    };
    return bf16 ? scan(gdn_pf_scan_kernel<__nv_bfloat16, __nv_bfloat16>)
                : scan(gdn_pf_scan_kernel<float, float>);
}

}  // namespace coli
