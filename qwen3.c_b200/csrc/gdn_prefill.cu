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
//   gdn_pf_prologue_kernel  per (64-token run, K head): sliding conv4 (history
//                           carried in from the previous call) + SiLU,
//                           q/k L2 norm, gates -> Q, K (fp32, head-major),
//                           K^T and V^T per chunk (the B operands of W and U),
//                           log-decay and beta per V head.
//   gdn_pf_hist_kernel      carries the last 3 pre-conv rows out as history.
//   gdn_pf_prep_kernel      per (chunk, V head), fully parallel: K K^T and
//                           Q K^T on tcgen05 (kind::tf32), T by blocked
//                           forward substitution in fp32, then W and U on
//                           tcgen05, and the decay-masked M.
//   gdn_pf_scan_kernel      per (V head, 64-column block of the state, segment
//                           of chunks): walks the chunks in order with the
//                           state slice in TMEM, products on tcgen05
//                           (kind::tf32), producing D and diag(gamma) Q S0 of
//                           every chunk. Operands arrive by TMA (128B swizzle,
//                           no multicast). With several segments a first
//                           pass of the same kernel computes each segment's
//                           affine state map and gdn_pf_combine_kernel chains
//                           the segment start states.
//   gdn_pf_out_kernel       per (chunk, V head), fully parallel: Y = QH + M D,
//                           gated RMSNorm over the head's 128 columns, y.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace cg = cooperative_groups;

namespace coli {

constexpr int PFG_C = 64, PFG_D = 128;

// ---------------------------------------------------------------- tf32 MMA
// fp32 -> tf32, round to nearest with ties away from zero (the rounding of
// cvt.rna.tf32.f32): add half a tf32 ulp (bit 12) to the magnitude bits and
// clear the 13 low mantissa bits; a carry moves into the exponent as it
// should. Operands that reach the MMA straight from shared memory are rounded
// once where they are produced (tf32r), since the MMA itself would truncate.
__device__ __forceinline__ uint32_t f2tf32(float x) { return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u; }
__device__ __forceinline__ float tf32r(float x) { return __uint_as_float(f2tf32(x)); }
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

// ldmatrix on fp32 data: an 8-row x 16-byte block delivers to lane l the
// word at (row l/4, column l%4), which is exactly the tf32 m16n8k8 fragment
// element (g, tq); four such blocks make an A fragment, two a B fragment.
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t &r0, uint32_t &r1)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r0), "=r"(r1) : "r"(addr));
}
// A fragment (16 rows from row0, k columns 8ks..8ks+7) of a 64-row fp32 tile
// that TMA wrote as 128B-swizzled 32-column boxes.
__device__ __forceinline__ void lda_sw(uint32_t tile, int row0, int ks, int lane, uint32_t (&a)[4])
{
    const int mat = lane >> 3, row = row0 + ((mat & 1) << 3) + (lane & 7);
    const int chunk = ((ks & 3) << 1) + (mat >> 1);
    ldsm_x4(tile + (ks >> 2) * (PFG_C * 128) + row * 128 + ((chunk ^ (row & 7)) << 4), a[0], a[1], a[2], a[3]);
}
// B fragment (n rows n0..n0+7, k columns 8ks..) of a swizzled tile of `rows`
// rows whose rows are the n index (regions rows x 128 bytes).
__device__ __forceinline__ void ldb_sw_rows(uint32_t tile, int rows, int n0, int ks, int lane, uint32_t &b0,
                                            uint32_t &b1)
{
    const int mat = (lane >> 3) & 1, row = n0 + (lane & 7);
    const int chunk = ((ks & 3) << 1) + mat;
    ldsm_x2(tile + (ks >> 2) * (rows * 128) + row * 128 + ((chunk ^ (row & 7)) << 4), b0, b1);
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

// Log decay and beta of token s, V head vh (vg in the input layout): from the
// a / b projections as the reference's gdn_step does (decay = exp(-exp(A_log)
// * softplus(a + dt_bias)), beta = sigmoid(b), c/qwen.c:725-730), or given by
// the caller (params rows [decay | beta | ...]); a decay of exactly 0 is kept
// finite in the log domain.
template <typename TI>
__device__ __forceinline__ void gdn_gates(const GdnPrefillArgs &p, int s, int vh, int vg, int VHin, const TI *a,
                                          const TI *b)
{
    float gl, beta;
    if (p.params) {
        const float *pr = p.params + (size_t)s * p.pstride;
        gl = fmaxf(logf(pr[vg]), -1.0e4f);
        beta = pr[VHin + vg];
    } else {
        gl = -expf(p.A_log[vg]) * softplusf_(to_f32(a[(size_t)s * VHin + vg]) + p.dt_bias[vg]);
        beta = sigmoidf_(to_f32(b[(size_t)s * VHin + vg]));
    }
    p.GL[(size_t)vh * p.S + s] = gl;
    p.BETA[(size_t)vh * p.S + s] = beta;
}

// ---------------------------------------------------------------- prologue
// One CTA walks a run of PRO_T tokens of one K head; thread t owns channel t
// of q, k and of the head's two V heads, keeping the last three pre-conv
// values in registers, so every input row is read once.
constexpr int PRO_T = 64;

template <typename TI>
__global__ void __launch_bounds__(PFG_D)
gdn_pf_prologue_kernel(GdnPrefillArgs p)
{
    const int kh = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int S = p.S, s_begin = blockIdx.x * PRO_T, s_end = min(S, s_begin + PRO_T);
    const int KHin = p.KHin ? p.KHin : p.KH, VHin = p.VHin ? p.VHin : p.VH;
    const int kg = p.kh0 + kh;                    // K head in the input layout
    const int key_dim = KHin * PFG_D, CD = 2 * key_dim + VHin * PFG_D;
    const TI *x = static_cast<const TI *>(p.qkv);
    const int ch[4] = {kg * PFG_D + t, key_dim + kg * PFG_D + t, 2 * key_dim + (2 * kg) * PFG_D + t,
                       2 * key_dim + (2 * kg + 1) * PFG_D + t};
    float4 w[4];
    float h0[4], h1[4], h2[4];                     // values at tokens s-3, s-2, s-1
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        w[c] = *reinterpret_cast<const float4 *>(p.conv_w + (size_t)ch[c] * 4);
        auto tap = [&](int ts) -> float {
            return ts >= 0 ? to_f32(x[(size_t)ts * CD + ch[c]]) : p.hist[(size_t)(3 + ts) * CD + ch[c]];
        };
        h0[c] = tap(s_begin - 3); h1[c] = tap(s_begin - 2); h2[c] = tap(s_begin - 1);
    }
    __shared__ float red[2][2][4];
    // K of this chunk also goes out transposed ([dk][64 tokens], tokens past S
    // zero), the A operand of the scan's state update; 4 tokens per store.
    float *kt = p.KT + (((size_t)kh * gridDim.x + blockIdx.x) * PFG_D + t) * PFG_C;
    // V^T likewise, per V head ([dv][64 tokens], tf32-rounded: the B operand of U)
    float *vt0 = p.VT + (((size_t)(2 * kh) * gridDim.x + blockIdx.x) * PFG_D + t) * PFG_C;
    float *vt1 = vt0 + (size_t)gridDim.x * PFG_D * PFG_C;
    float xn[4];                                   // next token's inputs, loaded one token ahead
#pragma unroll
    for (int c = 0; c < 4; ++c) xn[c] = to_f32(x[(size_t)s_begin * CD + ch[c]]);
    for (int s4 = s_begin; s4 < s_end; s4 += 4) {
        float kb[4], vb[2][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int s = s4 + u;
            kb[u] = 0.f; vb[0][u] = 0.f; vb[1][u] = 0.f;
            if (s >= s_end) continue;              // uniform across the CTA
            const int par = s & 1;
            float xv[4], out[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) xv[c] = xn[c];
            if (s + 1 < s_end) {
#pragma unroll
                for (int c = 0; c < 4; ++c) xn[c] = to_f32(x[(size_t)(s + 1) * CD + ch[c]]);
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float a = 0.f;
                a += w[c].x * h0[c]; a += w[c].y * h1[c]; a += w[c].z * h2[c]; a += w[c].w * xv[c];
                out[c] = __fdividef(a, 1.f + __expf(-a));  // silu (fast exp / divide)
                h0[c] = h1[c]; h1[c] = h2[c]; h2[c] = xv[c];
            }
            float sq = out[0] * out[0], sk = out[1] * out[1];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                sq += __shfl_xor_sync(0xffffffffu, sq, o);
                sk += __shfl_xor_sync(0xffffffffu, sk, o);
            }
            if (lane == 0) { red[par][0][warp] = sq; red[par][1][warp] = sk; }
            __syncthreads();
            sq = (red[par][0][0] + red[par][0][1]) + (red[par][0][2] + red[par][0][3]);
            sk = (red[par][1][0] + red[par][1][1]) + (red[par][1][2] + red[par][1][3]);
            const float rq = 1.f / sqrtf(sq + p.eps) / sqrtf((float)PFG_D);
            const float rk = 1.f / sqrtf(sk + p.eps);
            const float kv = out[1] * rk;
            kb[u] = tf32r(kv);
            p.Qh[((size_t)kh * S + s) * PFG_D + t] = out[0] * rq;   // full fp32: split by the consumers
            p.Kh[((size_t)kh * S + s) * PFG_D + t] = kv;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int vh = kh * 2 + j, vg = kg * 2 + j;  // local / input-layout V head
                vb[j][u] = tf32r(out[2 + j]);
                if (t == j) gdn_gates(p, s, vh, vg, VHin, static_cast<const TI *>(p.a), static_cast<const TI *>(p.b));
            }
        }
        *reinterpret_cast<float4 *>(kt + (s4 - s_begin)) = make_float4(kb[0], kb[1], kb[2], kb[3]);
        *reinterpret_cast<float4 *>(vt0 + (s4 - s_begin)) = make_float4(vb[0][0], vb[0][1], vb[0][2], vb[0][3]);
        *reinterpret_cast<float4 *>(vt1 + (s4 - s_begin)) = make_float4(vb[1][0], vb[1][1], vb[1][2], vb[1][3]);
    }
    for (int i = (s_end - s_begin + 3) & ~3; i < PRO_T; i += 4) {
        *reinterpret_cast<float4 *>(kt + i) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4 *>(vt0 + i) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4 *>(vt1 + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// bf16 inputs: the same prologue with the CTA's whole input tile (64 tokens x
// the 512 channels of one K head: q, k and its two V heads) brought into
// shared memory with wide loads first, then 8 warps x 8 tokens; the q/k norm
// is a warp reduction (lane = 4 q, 4 k and 8 v channels), and K^T leaves
// through a shared-memory transpose as contiguous rows. V goes back into the
// token's own input row (1 KiB: 512 bf16 in, 256 fp32 out, word c stored at
// c ^ (token % 32) so that both the row writes and the column reads are
// conflict-free) and leaves as V^T rows after the token loop.
constexpr int PRT_CH = 512;                  // channels of one K head's q|k|v0|v1
constexpr int PRT_KT_LD = PRO_T + 1;
size_t gdn_prologue_tile_smem()
{
    return (size_t)PRO_T * PRT_CH * 2 + 3 * PRT_CH * 4 + PRT_CH * 16 + PFG_D * PRT_KT_LD * 4;
}
__global__ void __launch_bounds__(256, 2)   // two CTAs per SM: at most 128 registers
gdn_pf_prologue_tile_kernel(GdnPrefillArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    __nv_bfloat16 *sX = reinterpret_cast<__nv_bfloat16 *>(smem_raw);        // [64][512]
    float *sHalo = reinterpret_cast<float *>(sX + PRO_T * PRT_CH);          // [3][512] tokens s_begin-3..-1
    float4 *sW = reinterpret_cast<float4 *>(sHalo + 3 * PRT_CH);            // [512] conv taps
    float *sKT = reinterpret_cast<float *>(sW + PRT_CH);                    // [128][65]
    const int kh = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = p.S, s_begin = blockIdx.x * PRO_T, nrow = min(S, s_begin + PRO_T) - s_begin;
    const int KHin = p.KHin ? p.KHin : p.KH, VHin = p.VHin ? p.VHin : p.VH;
    const int kg = p.kh0 + kh;
    const int key_dim = KHin * PFG_D, CD = 2 * key_dim + VHin * PFG_D;
    const __nv_bfloat16 *x = static_cast<const __nv_bfloat16 *>(p.qkv);
    auto gch = [&](int lc) {                 // local channel -> input channel
        return lc < PFG_D ? kg * PFG_D + lc
             : lc < 2 * PFG_D ? key_dim + kg * PFG_D + (lc - PFG_D)
                              : 2 * key_dim + 2 * kg * PFG_D + (lc - 2 * PFG_D);
    };
    {   // the tile (64 rows x 64 16-byte pieces), the 3 halo rows and the conv
        // taps: every load in flight before the first store, so the CTA waits
        // on global memory once
        uint4 v[16];
        float hv[3 * PRT_CH / 256];
        float4 wv[PRT_CH / 256];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int e = tid + 256 * i, row = e >> 6, lc = (e & 63) * 8;
            v[i] = row < nrow ? *reinterpret_cast<const uint4 *>(x + (size_t)(s_begin + row) * CD + gch(lc))
                              : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int i = 0; i < 3 * PRT_CH / 256; ++i) {
            const int e = tid + 256 * i, j = e / PRT_CH, lc = e - j * PRT_CH, ts = s_begin - 3 + j;
            hv[i] = ts >= 0 ? __bfloat162float(x[(size_t)ts * CD + gch(lc)]) : p.hist[(size_t)j * CD + gch(lc)];
        }
#pragma unroll
        for (int i = 0; i < PRT_CH / 256; ++i)
            wv[i] = *reinterpret_cast<const float4 *>(p.conv_w + (size_t)gch(tid + 256 * i) * 4);
        // the decay / beta gates of the chunk's 64 tokens x 2 V heads, one per
        // thread (their loads overlap the tile's instead of stalling a warp
        // once per token inside the token loop)
        if (tid < 2 * PRO_T && (tid >> 1) < nrow)
            gdn_gates(p, s_begin + (tid >> 1), kh * 2 + (tid & 1), kg * 2 + (tid & 1), VHin,
                      static_cast<const __nv_bfloat16 *>(p.a), static_cast<const __nv_bfloat16 *>(p.b));
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int e = tid + 256 * i, row = e >> 6, lc = (e & 63) * 8;
            *reinterpret_cast<uint4 *>(sX + row * PRT_CH + lc) = v[i];
        }
#pragma unroll
        for (int i = 0; i < 3 * PRT_CH / 256; ++i) sHalo[tid + 256 * i] = hv[i];
#pragma unroll
        for (int i = 0; i < PRT_CH / 256; ++i) sW[tid + 256 * i] = wv[i];
    }
    __syncthreads();

    const int r0 = warp * (PRO_T / 8);
    auto xin = [&](int r, int lc) -> float {
        return r >= 0 ? __bfloat162float(sX[r * PRT_CH + lc]) : sHalo[(3 + r) * PRT_CH + lc];
    };
    float h0[16], h1[16], h2[16];            // values at tokens s-3, s-2, s-1 of this lane's channels
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int lc = j * 32 + lane;
        h0[j] = xin(r0 - 3, lc); h1[j] = xin(r0 - 2, lc); h2[j] = xin(r0 - 1, lc);
    }
    __syncthreads();                         // halo rows read before their owners overwrite them with V
    for (int rr = 0; rr < PRO_T / 8; ++rr) {
        const int r = r0 + rr, s = s_begin + r;
        if (r >= nrow) break;                // warp-uniform
        float out[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int lc = j * 32 + lane;
            const float4 w = sW[lc];
            const float xv = __bfloat162float(sX[r * PRT_CH + lc]);
            float a = 0.f;
            a += w.x * h0[j]; a += w.y * h1[j]; a += w.z * h2[j]; a += w.w * xv;
            out[j] = __fdividef(a, 1.f + __expf(-a));  // silu (fast exp / divide)
            h0[j] = h1[j]; h1[j] = h2[j]; h2[j] = xv;
        }
        float sq = 0.f, sk = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) { sq += out[j] * out[j]; sk += out[4 + j] * out[4 + j]; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
            sk += __shfl_xor_sync(0xffffffffu, sk, o);
        }
        const float rq = 1.f / sqrtf(sq + p.eps) / sqrtf((float)PFG_D);
        const float rk = 1.f / sqrtf(sk + p.eps);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = j * 32 + lane;
            const float kv = out[4 + j] * rk;
            p.Qh[((size_t)kh * S + s) * PFG_D + c] = out[j] * rq;   // full fp32: split by the consumers
            p.Kh[((size_t)kh * S + s) * PFG_D + c] = kv;
            sKT[c * PRT_KT_LD + r] = tf32r(kv);
        }
        __syncwarp();                        // every lane has read row r
        float *vrow = reinterpret_cast<float *>(sX + r * PRT_CH);
#pragma unroll
        for (int j = 0; j < 8; ++j) vrow[(j * 32 + lane) ^ (r & 31)] = out[8 + j];
    }
    __syncthreads();
    // K^T of the chunk ([dk][64 tokens], tokens past S zero), row-contiguous
    float *kt = p.KT + ((size_t)kh * gridDim.x + blockIdx.x) * PFG_D * PFG_C;
    for (int e = tid; e < PFG_D * (PFG_C / 4); e += 256) {
        const int d = e >> 4, t4 = (e & 15) * 4;
        float4 v;
        v.x = t4 < nrow ? sKT[d * PRT_KT_LD + t4] : 0.f;
        v.y = t4 + 1 < nrow ? sKT[d * PRT_KT_LD + t4 + 1] : 0.f;
        v.z = t4 + 2 < nrow ? sKT[d * PRT_KT_LD + t4 + 2] : 0.f;
        v.w = t4 + 3 < nrow ? sKT[d * PRT_KT_LD + t4 + 3] : 0.f;
        *reinterpret_cast<float4 *>(kt + d * PFG_C + t4) = v;
    }
    // V^T of the chunk per V head ([dv][64 tokens], tokens past S zero, tf32):
    // a warp writes 32 consecutive tokens of one row
    // (four consecutive tokens per thread: one 16-byte store each)
    float *vt = p.VT + ((size_t)(2 * kh) * gridDim.x + blockIdx.x) * PFG_D * PFG_C;
    for (int e = tid; e < 2 * PFG_D * (PFG_C / 4); e += 256) {
        const int c = e >> 4, t4 = (e & 15) * 4;   // c = local V channel (head c / 128)
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int t = t4 + u;
            const float *vrow = reinterpret_cast<const float *>(sX + t * PRT_CH);
            v[u] = t < nrow ? tf32r(vrow[c ^ (t & 31)]) : 0.f;
        }
        *reinterpret_cast<float4 *>(vt + (size_t)(c >> 7) * gridDim.x * PFG_D * PFG_C + (c & 127) * PFG_C + t4) =
            make_float4(v[0], v[1], v[2], v[3]);
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

// Byte offset of element (row r, k) in a K-major 128B-swizzled fp32 tile with
// `rows` rows per k-atom (32 fp32 of k per 128 B row, 8-row groups 1 KiB apart).
__device__ __forceinline__ uint32_t kmaj_off(int rows, int r, int k)
{
    return (uint32_t)((k >> 5) * rows * 128 + r * 128 + ((((k & 31) >> 2) ^ (r & 7)) << 4) + (k & 3) * 4);
}

// The four products run on tcgen05 (kind::tf32, M = 64, one issuing thread,
// accumulators in 256 TMEM columns): K K^T and Q K^T (N = 64, K = 128 dk),
// then W = (T diag(beta gamma)) K and U = (T diag(beta)) V (N = 128 dk/dv,
// K = 64 tokens) with K^T / V^T from the prologue as the K-major B operands
// and the scaled T written K-major by the threads. The M = 64 accumulator
// puts row 16 q + i in TMEM lane 32 q + i, so warp w reads rows 16 (w % 4)..
// through the 16x256b shape, which is the mma.sync fragment layout.
// Warps 0-3 own the K K^T / W rows, warps 4-7 the Q K^T / U rows.
#ifdef COLI_SCAN_PROBE
__device__ long long g_prep_probe[2 * 16];
#define PREP_PROBE(slot) do { if (tid == 0 && blockIdx.y == 0 && (blockIdx.x == 0 || blockIdx.x == 200)) \
    g_prep_probe[(blockIdx.x ? 16 : 0) + (slot)] = clock64(); } while (0)
#else
#define PREP_PROBE(slot) do { } while (0)
#endif
constexpr int PREP_THREADS = 512;   // 16 warps: the SIMT phases of the chain run on twice the threads
__global__ void __launch_bounds__(PREP_THREADS)
gdn_pf_prep_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKT,
                   GdnPrefillArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    float *base = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // [K; Q] of the chunk: 4 k-atoms of 128 rows (K rows 0-63, Q rows 64-127),
    // 128B-swizzled; later V^T | K^T [128 x 64] swizzled
    float *sKQ = base;
    float *sQV = base;                          // V^T, after the products
    float *sK = base + PFG_C * PFG_D;           // K^T, after the products
    float *sA = sK + PFG_C * PFG_D;             // [64][68] strictly lower A; later T diag(beta gamma), K-major
    float *sT = sA + PFG_C * PREP_LD;           // [64][68] T = (I + A)^-1; later T diag(beta), K-major
    float *sX = sT + PFG_C * PREP_LD;           // [3][16][16] block products
    __shared__ float G[PFG_C], bet[PFG_C], bgam[PFG_C];   // bgam = beta e^G
    __shared__ __align__(8) uint64_t bar_qk, bar_v, bar_mma;
    __shared__ uint32_t tmem_base;

    const int n = blockIdx.x, h = blockIdx.y, kh = h >> 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
    const int s0 = n * PFG_C;
    if (tid == 0) {
        mbar_init(&bar_qk, 1);
        mbar_init(&bar_v, 1);
        mbar_init(&bar_mma, 1);
        fence_mbar_init();
    }
    if (warp == 0) tc::alloc(&tmem_base, 256);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = tmem_base;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    if (tid == 0) {
        mbar_expect_tx(&bar_qk, 2 * PFG_C * PFG_D * 4);
        for (int c = 0; c < 4; ++c) {
            tma_load_3d(sKQ + c * 2 * PFG_C * 32, &tmK, 32 * c, s0, kh, &bar_qk);
            tma_load_3d(sKQ + c * 2 * PFG_C * 32 + PFG_C * 32, &tmQ, 32 * c, s0, kh, &bar_qk);
        }
    }
    if (warp == 0) {
        chunk_cumsum(p.GL + (size_t)h * p.S, s0, p.S, lane, G);
    } else if (warp == 1) {
        for (int i = lane; i < PFG_C; i += 32)
            bet[i] = (s0 + i < p.S) ? p.BETA[(size_t)h * p.S + s0 + i] : 0.f;
    }
    __syncthreads();
    if (tid < PFG_C) bgam[tid] = bet[tid] * expf(G[tid]);   // read after later barriers
    // Q and K arrive in full fp32. Q K^T becomes M, which carries the outputs
    // (for a fast-decaying head almost all of y_t is M_tt d_t), so it runs as
    // three tf32 products, hi.hi + lo.hi + hi.lo (the split-tf32 scheme; a
    // product of plain tf32 roundings misses the output tolerance there);
    // K K^T, which enters the T solve, likewise. The tensor core reads the
    // tf32 truncation of an fp32 operand, so the K and Q rows serve as the hi
    // parts as they are (hi = x with the 13 low mantissa bits cleared) and
    // lo = x - hi is exact in fp32: only the lo tiles are written, K_lo then
    // Q_lo, in the A / T area (free until these products complete). Both
    // products come out of K [K; Q]^T (M = 64, N = 128: K K^T in TMEM columns
    // 0-63, K Q^T = (Q K^T)^T in 64-127), which takes a third fewer MMA
    // issues than separate N = 64 products:
    //   K_h [K_h; Q_h]^T + K_l [K_h; Q_h]^T + K_h K_l^T (cols 0-63) + K_h Q_l^T (cols 64-127)
    float *sLo = sA;                            // [64 x 128] in 4 k-atoms of 64 rows (32 KiB over sA, sT)
    auto lo_of = [](float x) { return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); };
    // lo of the K (part 0) or Q (part 1) rows of the [K; Q] atoms into sLo
    auto lo_pass = [&](int part) {
        for (int i = tid; i < PFG_C * PFG_D / 4; i += PREP_THREADS) {
            const int atom = i >> 9, o = i & 511;          // 512 float4 per 64-row atom
            const float4 x = reinterpret_cast<const float4 *>(sKQ)[atom * 1024 + part * 512 + o];
            reinterpret_cast<float4 *>(sLo)[i] = make_float4(lo_of(x.x), lo_of(x.y), lo_of(x.z), lo_of(x.w));
        }
    };
    PREP_PROBE(0);
    mbar_wait(&bar_qk, 0);
    PREP_PROBE(1);
    lo_pass(0);
    fence_proxy_async();                        // generic-proxy writes visible to the tensor core
    tc::fence_before();
    __syncthreads();
    constexpr uint32_t IDP64 = tc::idesc_tf32(64, 64), IDP128 = tc::idesc_tf32(64, 128);
    const uint32_t aKQ = smem_u32(sKQ), aLo = smem_u32(sLo);
    if (tid == 0) {
        tc::fence_after();
#pragma unroll
        for (int ks = 0; ks < PFG_D / 8; ++ks) {
            const uint32_t okq = (ks >> 2) * (2 * PFG_C * 128) + (ks & 3) * 32;   // K rows / [K; Q] rows
            const uint32_t olo = (ks >> 2) * (PFG_C * 128) + (ks & 3) * 32;
            tc::mma_tf32(tbase, tc::desc_k_sw128(aKQ + okq), tc::desc_k_sw128(aKQ + okq), IDP128, ks > 0);
            tc::mma_tf32(tbase, tc::desc_k_sw128(aLo + olo), tc::desc_k_sw128(aKQ + okq), IDP128, 1);
            tc::mma_tf32(tbase, tc::desc_k_sw128(aKQ + okq), tc::desc_k_sw128(aLo + olo), IDP64, 1);
        }
        tc::commit(&bar_mma);
    }
    PREP_PROBE(2);
    mbar_wait(&bar_mma, 0);                     // K_lo has been read: Q_lo over it
    tc::fence_after();
    PREP_PROBE(3);
    lo_pass(1);
    fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    if (tid == 0) {
        tc::fence_after();
#pragma unroll
        for (int ks = 0; ks < PFG_D / 8; ++ks) {
            const uint32_t okq = (ks >> 2) * (2 * PFG_C * 128) + (ks & 3) * 32;
            const uint32_t olo = (ks >> 2) * (PFG_C * 128) + (ks & 3) * 32;
            tc::mma_tf32(tbase + 64, tc::desc_k_sw128(aKQ + okq), tc::desc_k_sw128(aLo + olo), IDP64, 1);
        }
        tc::commit(&bar_mma);
    }
    mbar_wait(&bar_mma, 1);   // a time-out raises the device error word
    PREP_PROBE(4);
    tc::fence_after();

    // this warp's 16 rows of K K^T (w % 8 < 4) or K Q^T (w % 8 >= 4), 32 of
    // the 64 columns (w / 8): the decay-masked A to shared memory, M to global
    const int r0 = (warp & 3) * 16, second = (warp >> 2) & 1, ch = warp >> 3;
    {
        float acc[16];
        tc::ld16x256_x4(tbase + lane_off + (second ? 64u : 0u) + 32u * ch, acc);
        tc::wait_ld();
        float *Mg = p.M + ((size_t)n * p.VH + h) * PFG_C * PFG_C;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                const int i = r0 + g + 8 * hr, j = ch * 32 + nt * 8 + 2 * tq;
                const float v0 = acc[4 * nt + 2 * hr], v1 = acc[4 * nt + 2 * hr + 1];
                if (second) {
                    // K Q^T: row = key token i, column = query token j, so
                    // M[j][i] = e^{G_j - G_i} q_j.k_i for i <= j
                    const float e0 = ex2_approx((G[j] - G[i]) * 1.4426950408889634f);
                    const float e1 = ex2_approx((G[j + 1] - G[i]) * 1.4426950408889634f);
                    Mg[j * PFG_C + i] = i <= j ? e0 * v0 : 0.f;
                    Mg[(j + 1) * PFG_C + i] = i <= j + 1 ? e1 * v1 : 0.f;
                } else {
                    const float d0 = ex2_approx((G[i] - G[j]) * 1.4426950408889634f);
                    const float d1 = ex2_approx((G[i] - G[j + 1]) * 1.4426950408889634f);
                    sA[i * PREP_LD + j] = j < i ? bet[i] * d0 * v0 : 0.f;
                    sA[i * PREP_LD + j + 1] = j + 1 < i ? bet[i] * d1 * v1 : 0.f;
                }
            }
        }
    }
    // T = (I + A)^-1, A strictly lower triangular, by 16x16 blocks. The
    // diagonal block of these 16 A rows right away, by the warp that wrote its
    // columns, by forward substitution (lane c < 16 = column c, kept in
    // registers; two partial sums shorten the dependent chain), while the
    // Q K^T warps store M.
    if (!second && ch == (r0 >> 5)) {
        __syncwarp();                              // this warp's A rows written
        if (lane < 16) {
            const int c = lane;
            float t[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                // t[j] = 0 for j < c, so the sum may run over every j < i
                float acc0 = (i == c) ? 1.f : 0.f, acc1 = 0.f;
#pragma unroll
                for (int j = 0; j + 1 < i; j += 2) {
                    acc0 -= sA[(r0 + i) * PREP_LD + r0 + j] * t[j];
                    acc1 -= sA[(r0 + i) * PREP_LD + r0 + j + 1] * t[j + 1];
                }
                if (i & 1) acc0 -= sA[(r0 + i) * PREP_LD + r0 + i - 1] * t[i - 1];
                t[i] = acc0 + acc1;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) sT[(r0 + i) * PREP_LD + r0 + c] = t[i];
        }
    }
    tc::fence_before();
    __syncthreads();
    // V^T replaces Q and K^T replaces K in shared memory while T is solved
    // (the product MMAs that read them have completed)
    if (tid == 0) {
        mbar_expect_tx(&bar_v, 2 * PFG_C * PFG_D * 4);
        const int nch = (p.S + PFG_C - 1) / PFG_C;
        for (int c = 0; c < 2; ++c) tma_load_3d(sQV + c * PFG_D * 32, &tmV, 32 * c, 0, h * nch + n, &bar_v);
        for (int c = 0; c < 2; ++c) tma_load_3d(sK + c * PFG_D * 32, &tmKT, 32 * c, 0, kh * nch + n, &bar_v);
    }
    PREP_PROBE(5);
    // The off-diagonal blocks: T_pq = -T_pp * sum_{r=q}^{p-1} A_pr T_rq one
    // block diagonal at a time. The blocks above the diagonal are never
    // written: the operand build below treats them as zero.
    {
        for (int dist = 1; dist < 4; ++dist) {
            const int nblk = 4 - dist;                 // blocks (p, p - dist), p = dist..3
            // X_p = sum_{r=q}^{p-1} A_pr T_rq; a thread owns 4 adjacent columns
            for (int e = tid; e < nblk * 64; e += PREP_THREADS) {
                const int bi = e >> 6, i = (e >> 2) & 15, j = (e & 3) * 4;
                const int pr = (dist + bi) * 16, q = bi * 16;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int k = q; k < pr; ++k) {
                    const float a = sA[(pr + i) * PREP_LD + k];
                    const float4 t = *reinterpret_cast<const float4 *>(sT + k * PREP_LD + q + j);
                    acc.x += a * t.x; acc.y += a * t.y; acc.z += a * t.z; acc.w += a * t.w;
                }
                *reinterpret_cast<float4 *>(sX + (bi << 8) + (i << 4) + j) = acc;
            }
            __syncthreads();
            // T_pq = -T_pp X_p
            for (int e = tid; e < nblk * 64; e += PREP_THREADS) {
                const int bi = e >> 6, i = (e >> 2) & 15, j = (e & 3) * 4;
                const int pr = (dist + bi) * 16, q = bi * 16;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const float a = sT[(pr + i) * PREP_LD + pr + k];
                    const float4 x = *reinterpret_cast<const float4 *>(sX + (bi << 8) + (k << 4) + j);
                    acc.x += a * x.x; acc.y += a * x.y; acc.z += a * x.z; acc.w += a * x.w;
                }
                *reinterpret_cast<float4 *>(sT + (pr + i) * PREP_LD + q + j) =
                    make_float4(-acc.x, -acc.y, -acc.z, -acc.w);
            }
            __syncthreads();
        }
    }
    __syncthreads();
    PREP_PROBE(6);
    // T diag(beta gamma) and T diag(beta) as K-major tf32 A operands, over A and T
    {
        const int i = tid >> 3, j0 = (tid & 7) * 8;   // row i, columns j0 .. j0 + 7 (one 16-block)
        float t[8];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const float4 v = (j0 >> 4) > (i >> 4) ? make_float4(0.f, 0.f, 0.f, 0.f)
                                                  : *reinterpret_cast<const float4 *>(sT + i * PREP_LD + j0 + 4 * q);
            t[4 * q] = v.x; t[4 * q + 1] = v.y; t[4 * q + 2] = v.z; t[4 * q + 3] = v.w;
        }
        __syncthreads();
        uint8_t *aw = reinterpret_cast<uint8_t *>(sA), *au = reinterpret_cast<uint8_t *>(sT);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int j = j0 + 4 * q;
            *reinterpret_cast<float4 *>(aw + kmaj_off(PFG_C, i, j)) =
                make_float4(tf32r(t[4 * q] * bgam[j]), tf32r(t[4 * q + 1] * bgam[j + 1]),
                            tf32r(t[4 * q + 2] * bgam[j + 2]), tf32r(t[4 * q + 3] * bgam[j + 3]));
            *reinterpret_cast<float4 *>(au + kmaj_off(PFG_C, i, j)) =
                make_float4(tf32r(t[4 * q] * bet[j]), tf32r(t[4 * q + 1] * bet[j + 1]),
                            tf32r(t[4 * q + 2] * bet[j + 2]), tf32r(t[4 * q + 3] * bet[j + 3]));
        }
        fence_proxy_async();
    }
    tc::fence_before();
    __syncthreads();
    if (tid == 0) {
        // W -> columns 0..127, U -> 128..255 (K^T / V^T rows are the B operands)
        const bool ok = mbar_wait(&bar_v, 0);
        tc::fence_after();
        if (ok) {
            constexpr uint32_t ID = tc::idesc_tf32(64, 128);
            const uint32_t aW = smem_u32(sA), aU = smem_u32(sT), aKT = smem_u32(sK), aVT = smem_u32(sQV);
#pragma unroll
            for (int ks = 0; ks < PFG_C / 8; ++ks) {
                const uint32_t oa = (ks >> 2) * (PFG_C * 128) + (ks & 3) * 32;
                const uint32_t ob = (ks >> 2) * (PFG_D * 128) + (ks & 3) * 32;
                tc::mma_tf32(tbase, tc::desc_k_sw128(aW + oa), tc::desc_k_sw128(aKT + ob), ID, ks > 0);
                tc::mma_tf32(tbase + 128, tc::desc_k_sw128(aU + oa), tc::desc_k_sw128(aVT + ob), ID, ks > 0);
            }
        }
        tc::commit(&bar_mma);
    }
    PREP_PROBE(7);
    mbar_wait(&bar_mma, 0);   // third completion
    PREP_PROBE(8);
    tc::fence_after();
    // this warp's 16 rows of W (w % 8 < 4) or U (w % 8 >= 4), 64 of the 128 columns (w / 8)
    float *Og = (second ? p.U : p.W) + ((size_t)n * p.VH + h) * PFG_C * PFG_D;
    {
        const int half = ch;
        float w[32];
        tc::ld16x256_x8(tbase + lane_off + (second ? 128u : 0u) + 64 * half, w);
        tc::wait_ld();
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int col = half * 64 + nt * 8 + 2 * tq;
            const int ra = r0 + g, rb = ra + 8;
            // W feeds the walk's tensor core as is: rounded to tf32 here
            const float x0 = second ? w[4 * nt] : tf32r(w[4 * nt]), x1 = second ? w[4 * nt + 1] : tf32r(w[4 * nt + 1]);
            const float x2 = second ? w[4 * nt + 2] : tf32r(w[4 * nt + 2]), x3 = second ? w[4 * nt + 3] : tf32r(w[4 * nt + 3]);
            *reinterpret_cast<float2 *>(Og + ra * PFG_D + col) = make_float2(x0, x1);
            *reinterpret_cast<float2 *>(Og + rb * PFG_D + col) = make_float2(x2, x3);
        }
    }
    tc::fence_before();
    __syncthreads();
    PREP_PROBE(9);
    if (warp == 0) {
        tc::fence_after();
        tc::dealloc(tbase, 256);
    }
}

// ---------------------------------------------------------------- chunk scan
// The sequential part, on the 5th-gen tensor core (tcgen05, kind::tf32). Per
// (V head, 64-column block of the state) the chunks are walked in order:
//   (a) P = [W; Q] h            M = 128 (64 W rows over 64 Q rows), N = 64, K = 128
//   (e) D = U - P_W: D^T to scratch, D' = e^{G_C-G} D to shared memory;
//       QH = diag(gamma) P_Q to scratch (transposed, like D, so that the
//       stores of a warp are contiguous)
//   (c) h = gamma_C h + K^T D'  M = 128 (dk), N = 64, K = 64 tokens
// The fp32 state h lives in TMEM (64 columns). The epilogue warps copy it, tf32
// rounded, into shared memory as the B operand of (a) and scale it by gamma_C
// in TMEM before (c) accumulates onto it. Every operand is a K-major
// 128B-swizzled tile: W, Q (2-stage ring) and K^T (written transposed per
// chunk by the prologue; one stage, reloaded as soon as (c) has read it)
// arrive by TMA, as does U, h^T and D'^T are written by the epilogue threads.
// gdn_pf_out_kernel then turns D and QH into the outputs, parallel over chunks.
//
// Segments. A tcgen05.mma costs about the same for N = 32 as for N = 64, and
// the recurrence walks every chunk, so with few heads per GPU the scan is
// latency bound. The chunks are then split into `nseg` segments walked in
// parallel. The state after a segment is affine in the state before it,
// S_end = Phi S_start + Psi, and Phi (U taken as 0, start I) and Psi (start 0)
// obey the very recurrence above, so the TRANS pass runs this kernel on the
// 128 x 256 matrix [Phi | Psi] of every segment but the last, without outputs;
// gdn_pf_combine_kernel chains the segment start states in fp32, and the
// replay pass then produces every segment's outputs from its start state.
// Warp roles: 0 = TMA producer, 1 = TMEM owner and MMA issuer, then 16
// epilogue warps, 4 per TMEM lane quarter (warp % 4) with 16 columns each;
// quarters 0/1 hold the W rows (tokens 0-31 / 32-63), quarters 2/3 the Q
// rows; for h, lane = dk row.
// State columns per CTA: 32 for a single walk over many heads (more CTAs),
// 64 for segmented walks (fewer CTAs per segment); 4 epilogue warps per TMEM
// lane quarter with NC / 4 columns each either way.
constexpr int SCAN_EPI = 512;                 // epilogue threads
constexpr int SCAN_THREADS = 64 + SCAN_EPI;
constexpr uint32_t SC_A_BYTES = 4 * 16384;    // [W; Q]: 4 k-atoms x (128 rows x 128 B)
constexpr uint32_t SC_K_BYTES = 2 * 16384;    // K^T: 2 k-atoms x (128 dk rows x 128 B)
template <int NC> struct ScanSmem {
    static constexpr uint32_t BH = 4 * NC * 128;          // h^T: 4 k-atoms x (NC rows x 128 B)
    static constexpr uint32_t BD = 2 * NC * 128;          // D'^T: 2 k-atoms x (NC rows x 128 B)
    static constexpr uint32_t U = (NC / 32) * PFG_C * 128; // U: 32-column boxes x 64 tokens
    static constexpr uint32_t TOTAL = 2 * SC_A_BYTES + SC_K_BYTES + BH + BD + U;
    static_assert(TOTAL + 1024 <= 232448, "scan shared memory");
};


// Timing probe of the chunk walk (development builds with -DCOLI_SCAN_PROBE
// only): clock64 at fixed points of every chunk of the first CTA.
#ifdef COLI_SCAN_PROBE
__device__ long long g_scan_probe[1024 * 8];
#define SCAN_PROBE(i, slot) do { if (!TRANS && blockIdx.x == 0 && (i) < 1024) g_scan_probe[(i) * 8 + (slot)] = clock64(); } while (0)
#else
#define SCAN_PROBE(i, slot) do { } while (0)
#endif

// Grid: blockIdx.x = (seg * VH + h) * NB + blk, NB = 128 / NC state blocks
// (replay) or 256 / NC blocks of [Phi | Psi] (TRANS, segments 0 .. nseg-2).
template <bool TRANS, int NC>
__global__ void __launch_bounds__(SCAN_THREADS, 1)
gdn_pf_scan_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmKT, const __grid_constant__ CUtensorMap tmU,
                   GdnPrefillArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sA = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sK = sA + 2 * SC_A_BYTES;
    uint8_t *sBh = sK + SC_K_BYTES;
    uint8_t *sBd = sBh + ScanSmem<NC>::BH;
    uint8_t *sU = sBd + ScanSmem<NC>::BD;
    __shared__ __align__(8) uint64_t a_full[2], a_empty[2], k_full, k_empty, u_full, u_empty;
    __shared__ __align__(8) uint64_t h_ready, hs_ready, a_done, d_ready, c_done;
    __shared__ uint32_t tmem_base;

    constexpr int EC = NC / 4, NB = (TRANS ? 256 : 128) / NC;
    const int VH = p.VH;
    const int blk = blockIdx.x % NB, h = (blockIdx.x / NB) % VH, seg = blockIdx.x / (NB * VH);
    const int kh = h >> 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = p.S, nch = (S + PFG_C - 1) / PFG_C;
    const int n0 = seg * p.seglen, n1 = min(nch, n0 + p.seglen), cnt = n1 - n0;
    // TRANS: the first half of the blocks is Phi (U taken as 0, no Q), the second Psi
    const bool phi = TRANS && blk < NB / 2;
    const int col = (TRANS ? blk % (NB / 2) : blk) * NC;  // first state column (of Phi / Psi in TRANS)
    const uint32_t a_bytes = TRANS ? SC_A_BYTES / 2 : SC_A_BYTES;

    if (tid == 0) {
        for (int s = 0; s < 2; ++s) { mbar_init(&a_full[s], 1); mbar_init(&a_empty[s], 1); }
        mbar_init(&k_full, 1); mbar_init(&k_empty, 1);
        mbar_init(&u_full, 1); mbar_init(&u_empty, SCAN_EPI / 64);  // one arrival per W-row warp
        // hand-off barriers count one arrival per epilogue warp (lane 0 after
        // a __syncwarp), not one per thread: 512 arrivals on one shared word
        // serialise and sat on the chain's critical path
        mbar_init(&h_ready, SCAN_EPI / 32); mbar_init(&hs_ready, SCAN_EPI / 32); mbar_init(&a_done, 1);
        mbar_init(&d_ready, SCAN_EPI / 64); mbar_init(&c_done, 1);
        fence_mbar_init();
    }
    if (warp == 1) tc::alloc(&tmem_base, 2 * NC);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tP = tmem_base, tH = tmem_base + NC;

    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < cnt; ++i) {
                const int n = n0 + i, s = i & 1;
                if (i >= 2) mbar_wait(&a_empty[s], ((i >> 1) + 1) & 1);
                uint8_t *a = sA + s * SC_A_BYTES;
                mbar_expect_tx(&a_full[s], a_bytes);
                for (int c = 0; c < 4; ++c) {
                    tma_load_3d(a + c * 16384, &tmW, 32 * c, 0, n * VH + h, &a_full[s]);
                    if (!TRANS) tma_load_3d(a + c * 16384 + 8192, &tmQ, 32 * c, n * PFG_C, kh, &a_full[s]);
                }
                if (i >= 1) mbar_wait(&k_empty, (i + 1) & 1);
                mbar_expect_tx(&k_full, SC_K_BYTES);
                for (int c = 0; c < 2; ++c) tma_load_3d(sK + c * 16384, &tmKT, 32 * c, 0, kh * nch + n, &k_full);
                if (!phi) {
                    if (i >= 1) mbar_wait(&u_empty, (i + 1) & 1);
                    mbar_expect_tx(&u_full, ScanSmem<NC>::U);
                    for (int c = 0; c < NC / 32; ++c)
                        tma_load_3d(sU + c * PFG_C * 128, &tmU, col + 32 * c, 0, n * VH + h, &u_full);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_tf32(128, NC);
            const uint32_t aA = smem_u32(sA), aK = smem_u32(sK), aBh = smem_u32(sBh), aBd = smem_u32(sBd);
            for (int i = 0; i < cnt; ++i) {
                const int s = i & 1;
                mbar_wait(&a_full[s], (i >> 1) & 1);
                SCAN_PROBE(i, 7);
                mbar_wait(&h_ready, i & 1);
                SCAN_PROBE(i, 0);
                tc::fence_after();
#pragma unroll
                for (int ks = 0; ks < PFG_D / 8; ++ks)
                    tc::mma_tf32(tP, tc::desc_k_sw128(aA + s * SC_A_BYTES + (ks >> 2) * 16384 + (ks & 3) * 32),
                                 tc::desc_k_sw128(aBh + (ks >> 2) * (NC * 128) + (ks & 3) * 32), idesc, ks > 0);
                tc::commit(&a_done);
                tc::commit(&a_empty[s]);
                mbar_wait(&k_full, i & 1);
                mbar_wait(&d_ready, i & 1);
                mbar_wait(&hs_ready, i & 1);
                SCAN_PROBE(i, 1);
                tc::fence_after();
#pragma unroll
                for (int ks = 0; ks < PFG_C / 8; ++ks)
                    tc::mma_tf32(tH, tc::desc_k_sw128(aK + (ks >> 2) * 16384 + (ks & 3) * 32),
                                 tc::desc_k_sw128(aBd + (ks >> 2) * (NC * 128) + (ks & 3) * 32), idesc, 1);
                tc::commit(&c_done);
                tc::commit(&k_empty);
            }
        }
    } else {
        const int q = warp & 3, half = q & 1, c0 = ((warp - 2) >> 2) * EC;  // lane quarter, first column
        const uint32_t lane_off = ((uint32_t)(q * 32) << 16) + c0;
        const int r = q * 32 + lane;               // dk row of h / TMEM lane
        const int t = half * 32 + lane;            // token within the chunk in (e)
        const int cl = col + c0;                   // this thread's first state column
        const float *gl = p.GL + (size_t)h * S;
        float gl_lo, gl_hi;
        {
            const int t0 = n0 * PFG_C + lane;
            gl_lo = t0 < S ? gl[t0] : 0.f;
            gl_hi = t0 + 32 < S ? gl[t0 + 32] : 0.f;
        }
        float hv[EC], pv[EC];
        // start state
        if (TRANS) {
#pragma unroll
            for (int j = 0; j < EC; ++j) hv[j] = (phi && r == cl + j) ? 1.f : 0.f;
        } else {
            const float *src = (p.nseg > 1 ? p.Hs + ((size_t)seg * VH + h) * PFG_D * PFG_D
                                           : p.state + (size_t)h * PFG_D * PFG_D) + (size_t)r * PFG_D + cl;
#pragma unroll
            for (int i = 0; i < EC / 4; ++i) {
                const float4 v = reinterpret_cast<const float4 *>(src)[i];
                hv[4 * i] = v.x; hv[4 * i + 1] = v.y; hv[4 * i + 2] = v.z; hv[4 * i + 3] = v.w;
            }
        }
        for (int i = 0; i < cnt; ++i) {
            const int n = n0 + i;
            // inclusive cumulative log decay of this chunk: G_t for this
            // thread's token, G_C for the whole chunk
            float slo = gl_lo, shi = gl_hi;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float a = __shfl_up_sync(0xffffffffu, slo, o), b = __shfl_up_sync(0xffffffffu, shi, o);
                if (lane >= o) { slo += a; shi += b; }
            }
            const float tot_lo = __shfl_sync(0xffffffffu, slo, 31);
            const float GC = tot_lo + __shfl_sync(0xffffffffu, shi, 31);
            const float Gt = half ? tot_lo + shi : slo;
            // decay factors of this chunk: gamma_C for h, e^{G_C-G_t} for D', gamma_t for QH
            const float gC = expf(GC), sc = q < 2 ? expf(GC - Gt) : expf(Gt);
            asm volatile("" ::"f"(gC), "f"(sc));   // keep them here, off the critical path
            if (i + 1 < cnt) {
                const int t0 = (n + 1) * PFG_C + lane;
                gl_lo = t0 < S ? gl[t0] : 0.f;
                gl_hi = t0 + 32 < S ? gl[t0 + 32] : 0.f;
            }
            // ---- h -> h^T (tf32) for (a); gamma_C h back into TMEM for (c)
            if (i > 0) {
                mbar_wait(&c_done, (i - 1) & 1);
                if (warp == 4 && lane == 0) SCAN_PROBE(i, 2);
                tc::fence_after();
                tc::ldn<EC>(tH + lane_off, hv);
                tc::wait_ld();
            }
#pragma unroll
            for (int j = 0; j < EC; ++j) *reinterpret_cast<float *>(sBh + kmaj_off(NC, c0 + j, r)) = tf32r(hv[j]);
            fence_proxy_async();                    // h^T visible to the tensor core
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&h_ready);   // (a) may start
            if (warp == 4 && lane == 0) SCAN_PROBE(i, 3);
#pragma unroll
            for (int j = 0; j < EC; ++j) hv[j] *= gC;
            tc::stn<EC>(tH + lane_off, hv);
            tc::wait_st();
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&hs_ready);  // gamma_C h in place for (c)
            if (warp == 4 && lane == 0) SCAN_PROBE(i, 4);
            // ---- P = [W; Q] h is in TMEM
            mbar_wait(&a_done, i & 1);
            if (warp == 4 && lane == 0) SCAN_PROBE(i, 5);
            tc::fence_after();
            if (q < 2 || !TRANS) {
                tc::ldn<EC>(tP + lane_off, pv);
                tc::wait_ld();
            }
            if (q < 2) {
                if (!phi) {                         // D = U - W h (U of this chunk by TMA)
                    mbar_wait(&u_full, i & 1);
                    const float *ur = reinterpret_cast<const float *>(sU + (c0 >> 5) * PFG_C * 128 + t * 128);
#pragma unroll
                    for (int k = 0; k < EC / 4; ++k) {
                        const float4 v = *reinterpret_cast<const float4 *>(ur + (((((c0 & 31) >> 2) + k) ^ (t & 7)) << 2));
                        pv[4 * k] = v.x - pv[4 * k]; pv[4 * k + 1] = v.y - pv[4 * k + 1];
                        pv[4 * k + 2] = v.z - pv[4 * k + 2]; pv[4 * k + 3] = v.w - pv[4 * k + 3];
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&u_empty);
                } else {
#pragma unroll
                    for (int j = 0; j < EC; ++j) pv[j] = -pv[j];
                }
#pragma unroll
                for (int j = 0; j < EC; ++j)
                    *reinterpret_cast<float *>(sBd + kmaj_off(NC, c0 + j, t)) = tf32r(pv[j] * sc);
                fence_proxy_async();                // D'^T visible to the tensor core
                tc::fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&d_ready);
                if (warp == 4 && lane == 0) SCAN_PROBE(i, 6);
                if (!TRANS) {  // D^T for the output kernel, off the critical path
                    float *dt = p.Dt + (((size_t)n * VH + h) * PFG_D + cl) * PFG_C + t;
#pragma unroll
                    for (int j = 0; j < EC; ++j) dt[j * PFG_C] = pv[j];
                }
            } else if (!TRANS) {                    // QH^T, same layout as D^T
                float *qh = p.QH + (((size_t)n * VH + h) * PFG_D + cl) * PFG_C + t;
#pragma unroll
                for (int j = 0; j < EC; ++j) qh[j * PFG_C] = pv[j] * sc;
            }
        }
        // the state after this segment: the request's state (last segment),
        // [Phi | Psi] of the segment (TRANS)
        if (cnt > 0) {
            mbar_wait(&c_done, (cnt - 1) & 1);
            tc::fence_after();
            tc::ldn<EC>(tH + lane_off, hv);
            tc::wait_ld();
        }
        float *dst = nullptr;
        if (TRANS) dst = p.XS + (((size_t)seg * VH + h) * PFG_D + r) * (2 * PFG_D) + blk * NC + c0;
        else if (seg == p.nseg - 1) dst = p.state + ((size_t)h * PFG_D + r) * PFG_D + cl;
        if (dst) {
#pragma unroll
            for (int k = 0; k < EC / 4; ++k)
                reinterpret_cast<float4 *>(dst)[k] = make_float4(hv[4 * k], hv[4 * k + 1], hv[4 * k + 2], hv[4 * k + 3]);
        }
        tc::fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc::fence_after();
        tc::dealloc(tmem_base, 2 * NC);
    }
}

// Segment start states, in fp32: Hs[0] = S0, Hs[s+1] = Phi_s Hs[s] + Psi_s.
// Columns are independent (Phi acts from the left), so a CTA owns 16 state
// columns of one head: grid (VH, 8), 256 threads, thread = 2 rows x 4
// columns. Phi_{s+1} is copied into shared memory (cp.async) while step s
// computes.
constexpr int CMB_LD = 132;   // Phi row stride in shared memory (floats)
constexpr int CMB_NC = 16;    // state columns per CTA
__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__global__ void __launch_bounds__(256)
gdn_pf_combine_kernel(GdnPrefillArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    float *sPhi = reinterpret_cast<float *>(smem_raw);          // [2][128][CMB_LD]
    float *sH = sPhi + 2 * PFG_D * CMB_LD;                      // [128][CMB_NC]
    const int h = blockIdx.x, cb = blockIdx.y * CMB_NC, VH = p.VH, tid = threadIdx.x;
    const int r0 = (tid >> 2) * 2, c0 = (tid & 3) * 4;          // 2 rows x 4 columns
    auto fetch_phi = [&](int s) {
        const float *X = p.XS + ((size_t)s * VH + h) * PFG_D * (2 * PFG_D);
        float *dst = sPhi + (s & 1) * PFG_D * CMB_LD;
        for (int i = tid; i < PFG_D * PFG_D / 4; i += 256) {
            const int row = i >> 5, k4 = (i & 31) * 4;
            cp_async16(dst + row * CMB_LD + k4, X + (size_t)row * (2 * PFG_D) + k4);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    fetch_phi(0);
    for (int i = 0; i < 2; ++i) {
        const float4 v = *reinterpret_cast<const float4 *>(p.state + ((size_t)h * PFG_D + r0 + i) * PFG_D + cb + c0);
        *reinterpret_cast<float4 *>(sH + (r0 + i) * CMB_NC + c0) = v;
        *reinterpret_cast<float4 *>(p.Hs + ((size_t)h * PFG_D + r0 + i) * PFG_D + cb + c0) = v;
    }
    for (int s = 0; s + 1 < p.nseg; ++s) {
        if (s + 2 < p.nseg) {
            fetch_phi(s + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();                                        // Phi_s and H_s in place
        const float *X = p.XS + ((size_t)s * VH + h) * PFG_D * (2 * PFG_D);
        const float *ph = sPhi + (s & 1) * PFG_D * CMB_LD;
        float acc[2][4];
        for (int i = 0; i < 2; ++i) {
            const float4 v = *reinterpret_cast<const float4 *>(X + (size_t)(r0 + i) * (2 * PFG_D) + PFG_D + cb + c0);
            acc[i][0] = v.x; acc[i][1] = v.y; acc[i][2] = v.z; acc[i][3] = v.w;   // Psi
        }
#pragma unroll 4
        for (int k = 0; k < PFG_D; k += 4) {
            float4 hk[4], pr[2];
#pragma unroll
            for (int e = 0; e < 4; ++e) hk[e] = *reinterpret_cast<const float4 *>(sH + (k + e) * CMB_NC + c0);
#pragma unroll
            for (int i = 0; i < 2; ++i) pr[i] = *reinterpret_cast<const float4 *>(ph + (r0 + i) * CMB_LD + k);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const float a[4] = {pr[i].x, pr[i].y, pr[i].z, pr[i].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    acc[i][0] += a[e] * hk[e].x; acc[i][1] += a[e] * hk[e].y;
                    acc[i][2] += a[e] * hk[e].z; acc[i][3] += a[e] * hk[e].w;
                }
            }
        }
        __syncthreads();                                        // every read of H_s done
        for (int i = 0; i < 2; ++i) {
            const float4 v = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
            *reinterpret_cast<float4 *>(sH + (r0 + i) * CMB_NC + c0) = v;
            *reinterpret_cast<float4 *>(p.Hs + (((size_t)(s + 1) * VH + h) * PFG_D + r0 + i) * PFG_D + cb + c0) = v;
        }
    }
}
size_t gdn_combine_smem() { return (size_t)(2 * PFG_D * CMB_LD + PFG_D * CMB_NC) * 4; }

// ---------------------------------------------------------------- outputs
// Parallel over (chunk, V head): Y = QH + M D, then the gated RMSNorm over the
// head's 128 columns (all in this CTA) and y = Y * rsqrt(mean Y^2 + eps) *
// gnorm * silu(z).
template <typename TI, typename TO>
__global__ void __launch_bounds__(256, 3)   // three CTAs per SM (48 KiB shared memory each): at most 80 registers
gdn_pf_out_kernel(const __grid_constant__ CUtensorMap tmM, const __grid_constant__ CUtensorMap tmDt,
                  GdnPrefillArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    float *base = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *sM = base;                    // [64 x 64] swizzled (2 boxes of 32 columns)
    float *sDT = sM + PFG_C * PFG_C;     // D^T [128 dv x 64 tokens] swizzled (2 boxes of 32 tokens)
    __shared__ __align__(8) uint64_t bar;
    const int n = blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
    const int VH = p.VH, VD = PFG_D, S = p.S;
    const int VHin = p.VHin ? p.VHin : VH, vg = 2 * p.kh0 + h;
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_expect_tx(&bar, (PFG_C * PFG_C + PFG_D * PFG_C) * 4);
        for (int c = 0; c < 2; ++c) tma_load_3d(sM + c * PFG_C * 32, &tmM, 32 * c, 0, n * VH + h, &bar);
        for (int c = 0; c < 2; ++c) tma_load_3d(sDT + c * PFG_D * 32, &tmDt, 32 * c, 0, n * VH + h, &bar);
    }
    // warp w: token rows 16 (w % 4).., value columns 64 (w / 4)..
    const int r0 = (warp & 3) * 16, cq = (warp >> 2) * 64;
    __shared__ float rsum[2][PFG_C];
    // Y starts from QH, read from QH^T straight into the fragment layout
    // (8 consecutive tokens of a column per 32-byte sector)
    float y[8][4];
    {
        const float *qt = p.QH + ((size_t)n * VH + h) * PFG_D * PFG_C;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int col = cq + nt * 8 + 2 * tq;
            y[nt][0] = qt[col * PFG_C + r0 + g];     y[nt][1] = qt[(col + 1) * PFG_C + r0 + g];
            y[nt][2] = qt[col * PFG_C + r0 + g + 8]; y[nt][3] = qt[(col + 1) * PFG_C + r0 + g + 8];
        }
    }
    __syncthreads();
    mbar_wait(&bar, 0);
    const uint32_t aM = smem_u32(sM), aD = smem_u32(sDT);
    // M D (M is causal: token columns past this warp's 16 rows are zero and
    // skipped). The diagonal 16 x 16 block runs in split tf32 (M and D arrive
    // in full fp32; each fragment is split into hi = tf32(x) and
    // lo = tf32(x - hi), and hi.hi + lo.hi + hi.lo is accumulated): there
    // M_tj carries the outputs of fast-decaying heads, whose rows the gated
    // norm rescales. Older tokens come in with decayed weights and take
    // plain tf32.
#pragma unroll
    for (int ks = 0; ks < PFG_C / 8; ++ks) {
        if (8 * ks > r0 + 15) break;               // warp-uniform: M is zero beyond the diagonal
        const bool diag = 8 * ks >= r0;
        uint32_t a[4], ah[4], al[4];
        lda_sw(aM, r0, ks, lane, a);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ah[i] = f2tf32(__uint_as_float(a[i]));
            al[i] = f2tf32(__uint_as_float(a[i]) - __uint_as_float(ah[i]));
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            uint32_t b0, b1;
            ldb_sw_rows(aD, PFG_D, cq + nt * 8, ks, lane, b0, b1);
            const uint32_t bh0 = f2tf32(__uint_as_float(b0)), bh1 = f2tf32(__uint_as_float(b1));
            if (diag) {
                const uint32_t bl0 = f2tf32(__uint_as_float(b0) - __uint_as_float(bh0));
                const uint32_t bl1 = f2tf32(__uint_as_float(b1) - __uint_as_float(bh1));
                mma_tf32(y[nt], al[0], al[1], al[2], al[3], bh0, bh1);
                mma_tf32(y[nt], ah[0], ah[1], ah[2], ah[3], bl0, bl1);
            }
            mma_tf32(y[nt], ah[0], ah[1], ah[2], ah[3], bh0, bh1);
        }
    }
    // the gate rows this thread stores at the end, loaded now so that their
    // latency overlaps the row statistics (item e = tid + 256 k: token e / 16,
    // 8 columns from 8 (e % 16)); not earlier, to keep the products' registers
    // within three CTAs per SM
    const TI *z = static_cast<const TI *>(p.z);
    constexpr int ZW = sizeof(TI) == 2 ? 1 : 2;          // 16-byte pieces per 8 gate values
    uint4 zpre[4][ZW];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int e = tid + 256 * k, tok = n * PFG_C + (e >> 4);
        const TI *zr = z + (size_t)tok * VHin * VD + vg * VD + (e & 15) * 8;
#pragma unroll
        for (int w = 0; w < ZW; ++w)
            zpre[k][w] = tok < S ? reinterpret_cast<const uint4 *>(zr)[w] : make_uint4(0u, 0u, 0u, 0u);
    }
    float sa = 0.f, sb = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
        sa += y[nt][0] * y[nt][0] + y[nt][1] * y[nt][1];
        sb += y[nt][2] * y[nt][2] + y[nt][3] * y[nt][3];
    }
    sa += __shfl_xor_sync(0xffffffffu, sa, 1); sa += __shfl_xor_sync(0xffffffffu, sa, 2);
    sb += __shfl_xor_sync(0xffffffffu, sb, 1); sb += __shfl_xor_sync(0xffffffffu, sb, 2);
    if (tq == 0) { rsum[warp >> 2][r0 + g] = sa; rsum[warp >> 2][r0 + g + 8] = sb; }
    __syncthreads();                     // row sums of both column halves; every warp is done with sM / sDT
    sa = rsum[0][r0 + g] + rsum[1][r0 + g];
    sb = rsum[0][r0 + g + 8] + rsum[1][r0 + g + 8];
    const float ra_ = 1.f / sqrtf(sa / VD + p.eps), rb_ = 1.f / sqrtf(sb / VD + p.eps);
    // normalised rows (times gnorm) to shared memory, then the gate and the
    // store row by row so that z loads and y stores are 16-byte vectors
    constexpr int YLD = PFG_D + 4;
    float *sY = sM;                      // [64][YLD] over the M / D^T tiles (33 KiB of 48)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
        const int col = cq + nt * 8 + 2 * tq;
        const float g0 = p.gnorm[col], g1 = p.gnorm[col + 1];
        *reinterpret_cast<float2 *>(sY + (r0 + g) * YLD + col) = make_float2(y[nt][0] * ra_ * g0, y[nt][1] * ra_ * g1);
        *reinterpret_cast<float2 *>(sY + (r0 + g + 8) * YLD + col) = make_float2(y[nt][2] * rb_ * g0, y[nt][3] * rb_ * g1);
    }
    __syncthreads();
    TO *out = static_cast<TO *>(p.y);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int e = tid + 256 * k;
        const int row = e >> 4, c8 = (e & 15) * 8, tok = n * PFG_C + row;
        if (tok >= S) continue;
        const size_t ooff = (size_t)tok * VH * VD + h * VD + c8;
        float zv[8], v[8];
        if constexpr (sizeof(TI) == 2) {
            const __nv_bfloat16 *zb = reinterpret_cast<const __nv_bfloat16 *>(&zpre[k][0]);
#pragma unroll
            for (int j = 0; j < 8; ++j) zv[j] = to_f32(zb[j]);
        } else {
            const float *zf = reinterpret_cast<const float *>(&zpre[k][0]);
#pragma unroll
            for (int j = 0; j < 8; ++j) zv[j] = zf[j];
        }
        const float4 y0 = *reinterpret_cast<const float4 *>(sY + row * YLD + c8);
        const float4 y1 = *reinterpret_cast<const float4 *>(sY + row * YLD + c8 + 4);
        v[0] = y0.x; v[1] = y0.y; v[2] = y0.z; v[3] = y0.w; v[4] = y1.x; v[5] = y1.y; v[6] = y1.z; v[7] = y1.w;
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] *= siluf_(zv[j]);
        const int ndst = p.gather.world ? p.gather.world : 1;
        for (int r = 0; r < ndst; ++r) {
            // the local output, or every rank's gathered buffer (this rank's block)
            TO *orow = p.gather.world ? static_cast<TO *>(p.gather.dst[r]) + (size_t)p.gather.rank * p.gather.block + ooff
                                      : out + ooff;
            if constexpr (sizeof(TO) == 2) {
                uint4 o;
                o.x = pack_bf16(v[0], v[1]); o.y = pack_bf16(v[2], v[3]); o.z = pack_bf16(v[4], v[5]); o.w = pack_bf16(v[6], v[7]);
                *reinterpret_cast<uint4 *>(orow) = o;
            } else {
                *reinterpret_cast<float4 *>(orow) = make_float4(v[0], v[1], v[2], v[3]);
                *reinterpret_cast<float4 *>(orow + 4) = make_float4(v[4], v[5], v[6], v[7]);
            }
        }
    }
    if (p.gather.world) __threadfence_system();   // peer stores visible before the cross-rank barrier
}

// ---------------------------------------------------------------- launch
size_t gdn_prep_smem() { return (size_t)(2 * PFG_C * PFG_D + 2 * PFG_C * PREP_LD + 3 * 256) * 4 + 1024; }
template <int NC> size_t gdn_scan_smem() { return (size_t)ScanSmem<NC>::TOTAL + 1024; }
size_t gdn_out_smem() { return (size_t)(PFG_C * PFG_C + PFG_D * PFG_C) * 4 + 1024; }

cudaError_t launch_gdn_prefill(const GdnPrefillArgs &a, const GdnPrefillMaps &m, int bf16,
                               cudaStream_t st)
{
    if (a.S < 3) return cudaErrorInvalidValue;
    const int nchunks = (a.S + PFG_C - 1) / PFG_C;
    const int CD = 2 * (a.KHin ? a.KHin : a.KH) * PFG_D + (a.VHin ? a.VHin : a.VH) * PFG_D;
    cudaError_t e;
    if (bf16) {
        e = cudaFuncSetAttribute(gdn_pf_prologue_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)gdn_prologue_tile_smem());
        if (e != cudaSuccess) return e;
        gdn_pf_prologue_tile_kernel<<<dim3((a.S + PRO_T - 1) / PRO_T, a.KH), 256, gdn_prologue_tile_smem(), st>>>(a);
    } else {
        gdn_pf_prologue_kernel<float><<<dim3((a.S + PRO_T - 1) / PRO_T, a.KH), PFG_D, 0, st>>>(a);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (bf16) gdn_pf_hist_kernel<__nv_bfloat16><<<(3 * CD + 255) / 256, 256, 0, st>>>(a);
    else gdn_pf_hist_kernel<float><<<(3 * CD + 255) / 256, 256, 0, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    e = cudaFuncSetAttribute(gdn_pf_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gdn_prep_smem());
    if (e != cudaSuccess) return e;
    gdn_pf_prep_kernel<<<dim3(nchunks, a.VH), PREP_THREADS, gdn_prep_smem(), st>>>(m.Q, m.K, m.V, m.KT, a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    auto scan = [&](auto kern, size_t smem, int grid) -> cudaError_t {
        cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e2 != cudaSuccess) return e2;
        kern<<<grid, SCAN_THREADS, smem, st>>>(m.W, m.Q, m.KT, m.U, a);
        return cudaGetLastError();
    };
    if (a.nseg > 1) {
        if ((e = scan(gdn_pf_scan_kernel<true, 64>, gdn_scan_smem<64>(), (a.nseg - 1) * a.VH * 4)) != cudaSuccess)
            return e;
        e = cudaFuncSetAttribute(gdn_pf_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gdn_combine_smem());
        if (e != cudaSuccess) return e;
        gdn_pf_combine_kernel<<<dim3(a.VH, PFG_D / CMB_NC), 256, gdn_combine_smem(), st>>>(a);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        e = scan(gdn_pf_scan_kernel<false, 64>, gdn_scan_smem<64>(), a.nseg * a.VH * 2);
    } else {
        e = scan(gdn_pf_scan_kernel<false, 32>, gdn_scan_smem<32>(), a.VH * 4);
    }
    if (e != cudaSuccess) return e;
    auto out = [&](auto kern) -> cudaError_t {
        cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gdn_out_smem());
        if (e2 != cudaSuccess) return e2;
        kern<<<dim3(nchunks, a.VH), 256, gdn_out_smem(), st>>>(m.M, m.Dt, a);
        return cudaGetLastError();
    };
    return bf16 ? out(gdn_pf_out_kernel<__nv_bfloat16, __nv_bfloat16>) : out(gdn_pf_out_kernel<float, float>);
}

}  // namespace coli
