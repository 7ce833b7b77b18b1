// Gated GQA causal prefill on the 5th-gen tensor cores (tcgen05 + TMEM + TMA).
//
// Same per-row semantics as the reference's attention() hot loop
// (c/qwen.c:638-663): query row s (position pos_base+s) attends to cache rows
// 0..pos_base+s of its KV head (h / 8) with scale 1/sqrt(256); ctx is gated by
// sigmoid(gate). The prologue (q/k norm, RoPE, K/V append) runs before this
// kernel (gqa_prologue_warp_kernel), so the new rows are already in the cache.
//
// One CTA = 128 query rows of one Q head, 128-key tiles. A tcgen05.mma costs
// about the same for N = 64 as for N = 128, so 128-key score tiles halve the
// instruction count of S per key; the shared memory that this takes is freed
// by holding Q in TMEM (the A operand of S) instead of shared memory.
// Warp roles (320 threads):
//   warp 0      TMA producers. Lane 0: Q (once, into the V buffer), then K
//               tiles into a 2-stage ring. Lane 1: V tiles into one buffer,
//               once Q has been moved into TMEM and each PV has read the last.
//   warp 1      MMA issuer (one thread) and TMEM owner: S = Q K^T (M=128,
//               N=128, K=256; A from TMEM), O += P V (M=128, N=256, K=128;
//               V read MN-major). S(j+1) is issued before PV(j).
//   warps 2..9  copy Q into TMEM, then the softmax: 16 query rows per warp read
//               with the 16x256b TMEM shape (a lane quad per row, so row max
//               and sum are quad shuffles), causal mask on the tile that
//               crosses the diagonal, online softmax in the log2 domain with
//               lazy rescaling (O is corrected in TMEM only when the running
//               max grows by more than 2^8), P written to shared memory in the
//               UMMA K-major layout. Epilogue, bf16: the gate tile arrives
//               by TMA in the second K buffer (issued by warp 0 once the last
//               S reading it is done), ctx = O / l * sigmoid(gate) is staged
//               as bf16 boxes in the first and written by TMA box stores.
//               Otherwise (fp32, peer gather): O / l staged as fp32 rows in
//               the K buffers, then a warp per row applies sigmoid(gate) with
//               16-byte coalesced gate loads and ctx stores (a thread-per-row
//               store pattern touches 32 rows per instruction and cost as
//               much as 40 KV tiles per CTA).
// TMEM (512 columns): scores 128 | O 256 | Q 128 (bf16 pairs).
// Shared memory: K 2 x 64 KiB, V (and Q staging) 64 KiB, P 32 KiB.
// Every wait is bounded (see mbar_wait); no cluster multicast.
#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace coli {

constexpr int PF_BM = 128, PF_BN = 128, PF_HD = 256;
constexpr int PF_Q_BYTES = PF_BM * PF_HD * 2;        // 64 KiB (staged in the V buffer)
constexpr int PF_KV_BYTES = PF_BN * PF_HD * 2;       // 64 KiB per K (or V) tile
constexpr int PF_P_BYTES = PF_BM * PF_BN * 2;        // 32 KiB
constexpr int PF_DATA = 3 * PF_KV_BYTES + PF_P_BYTES;  // 224 KiB
constexpr int PF_SOFTMAX = 256;                    // softmax / epilogue threads
constexpr int PF_THREADS = 64 + PF_SOFTMAX;
constexpr float PF_RESCALE_LOG2 = 8.0f;
static_assert(PF_Q_BYTES <= PF_KV_BYTES, "Q is staged in the V buffer");

struct PfBars {
    uint64_t q_full, q_tmem, k_full[2], k_empty[2], v_full, v_empty, s_full, s_free, p_full, pv_done, g_full;
    uint32_t tmem_base;
    float lsum[PF_BM];        // final row sums for the epilogue
};
constexpr int PF_SMEM = PF_DATA + (int)sizeof(PfBars);
static_assert(PF_SMEM <= 232448, "prefill shared memory exceeds the 227 KiB per-CTA limit");

// eight consecutive elements, 16-byte (bf16) or 2 x 16-byte (fp32) accesses
__device__ __forceinline__ void load8v(const __nv_bfloat16 *src, float (&x)[8])
{
    const uint4 u = *reinterpret_cast<const uint4 *>(src);
    const __nv_bfloat162 *b = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) { const float2 f = __bfloat1622float2(b[i]); x[2 * i] = f.x; x[2 * i + 1] = f.y; }
}
__device__ __forceinline__ void load8v(const float *src, float (&x)[8])
{
    const float4 a = reinterpret_cast<const float4 *>(src)[0], b = reinterpret_cast<const float4 *>(src)[1];
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
__device__ __forceinline__ void store8v(__nv_bfloat16 *dst, const float (&y)[8])
{
    uint4 u;
    __nv_bfloat162 *b = reinterpret_cast<__nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = __floats2bfloat162_rn(y[2 * i], y[2 * i + 1]);
    *reinterpret_cast<uint4 *>(dst) = u;
}
__device__ __forceinline__ void store8v(float *dst, const float (&y)[8])
{
    reinterpret_cast<float4 *>(dst)[0] = make_float4(y[0], y[1], y[2], y[3]);
    reinterpret_cast<float4 *>(dst)[1] = make_float4(y[4], y[5], y[6], y[7]);
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(PF_THREADS, 1)
gqa_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, GqaPrefillArgs p,
                   const __grid_constant__ PfEpiMaps em)
{
    // All shared memory is dynamic (no static __shared__), so the window
    // starts 1024-byte aligned as the 128B-swizzled TMA boxes and UMMA
    // descriptors need; checked below rather than padded (the budget is tight).
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sK = smem_raw;                     // [2][64 KiB]
    uint8_t *sV = sK + 2 * PF_KV_BYTES;         // 64 KiB: Q first, then V tiles
    uint8_t *sP = sV + PF_KV_BYTES;             // 32 KiB P tile (two 64-key atoms)
    PfBars &bars = *reinterpret_cast<PfBars *>(sP + PF_P_BYTES);
    if (smem_u32(smem_raw) & 1023) {  // uniform across the CTA: nothing has started yet
        if (threadIdx.x == 0) raise_error(2);
        return;
    }

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = p.H;
    const int h = blockIdx.x % H;
    const int qt = p.n_qtiles - 1 - (int)(blockIdx.x / H);  // heaviest tiles first
    const int kh = (p.h0 + h) / 8 - p.kh0;                  // KV head in this call's cache
    const int Hin = p.Hin ? p.Hin : H;
    const int q0 = qt * PF_BM;                              // first query row of the tile
    const int last_row = min(p.S, q0 + PF_BM) - 1;
    const int nt = (p.pos_base + last_row) / PF_BN + 1;     // KV tiles touched
    const int kvrow0 = (p.req * p.KH + kh) * p.max_t;

    if (threadIdx.x == 0) {
        mbar_init(&bars.q_full, 1);
        mbar_init(&bars.q_tmem, PF_SOFTMAX);
        for (int i = 0; i < 2; ++i) { mbar_init(&bars.k_full[i], 1); mbar_init(&bars.k_empty[i], 1); }
        mbar_init(&bars.v_full, 1); mbar_init(&bars.v_empty, 1);
        mbar_init(&bars.s_full, 1); mbar_init(&bars.s_free, PF_SOFTMAX);
        mbar_init(&bars.p_full, PF_SOFTMAX); mbar_init(&bars.pv_done, 1);
        mbar_init(&bars.g_full, 1);
        fence_mbar_init();
    }
    if (warp == 1) tc::alloc(&bars.tmem_base, 512);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = bars.tmem_base;
    const uint32_t tS = tbase, tO = tbase + 128, tQ = tbase + 384;   // S 128 | O 256 | Q 128 (bf16 pairs)

    if (warp == 0) {
        // ------------------------------------------------ TMA producers
        if (lane == 0) {
            tma_prefetch_desc(&tmQ); tma_prefetch_desc(&tmK);
            mbar_expect_tx(&bars.q_full, PF_Q_BYTES);
            for (int c = 0; c < 4; ++c) tma_load_3d(sV + c * (PF_BM * 128), &tmQ, 64 * c, h, q0, &bars.q_full);
            bool kok = true;
            for (int j = 0; j < nt; ++j) {
                const int s = j & 1;
                if (j >= 2 && !mbar_wait(&bars.k_empty[s], ((j >> 1) - 1) & 1)) { kok = false; break; }
                mbar_expect_tx(&bars.k_full[s], PF_KV_BYTES);
                for (int c = 0; c < 4; ++c)
                    tma_load_2d(sK + s * PF_KV_BYTES + c * (PF_BN * 128), &tmK, 64 * c,
                                kvrow0 + j * PF_BN, &bars.k_full[s]);
            }
            if (p.tma_epi && kok) {
                // the gate tile into the second K buffer as soon as the last S
                // that reads that buffer (odd tile j1) is done; it lands while
                // the last tiles' softmax and PV run
                const int j1 = (nt - 1) & 1 ? nt - 1 : nt - 2;
                if (j1 < 1 || mbar_wait(&bars.k_empty[1], (j1 >> 1) & 1)) {
                    tma_prefetch_desc(&em.gate);
                    mbar_expect_tx(&bars.g_full, PF_BM * PF_HD * 2);
                    for (int c = 0; c < 4; ++c)
                        tma_load_3d(sK + PF_KV_BYTES + c * (PF_BM * 128), &em.gate, PF_HD + 64 * c, p.h0 + h, q0,
                                    &bars.g_full);
                }
            }
        } else if (lane == 1) {
            tma_prefetch_desc(&tmV);
            // the V buffer holds Q until the softmax warps have moved it into TMEM
            if (mbar_wait(&bars.q_tmem, 0)) {
                for (int j = 0; j < nt; ++j) {
                    if (j >= 1 && !mbar_wait(&bars.v_empty, (j - 1) & 1)) break;
                    mbar_expect_tx(&bars.v_full, PF_KV_BYTES);
                    for (int c = 0; c < 4; ++c)
                        tma_load_2d(sV + c * (PF_BN * 128), &tmV, 64 * c, kvrow0 + j * PF_BN, &bars.v_full);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t ID_QK = tc::idesc_bf16(PF_BM, PF_BN, 0, 0);
            constexpr uint32_t ID_PV = tc::idesc_bf16(PF_BM, PF_HD, 0, 1);
            const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
            bool ok = mbar_wait(&bars.q_tmem, 0);       // Q copied into TMEM by the softmax warps
            auto issue_s = [&](int j) -> bool {
                const int s = j & 1;
                if (!mbar_wait(&bars.k_full[s], (j >> 1) & 1)) return false;
                if (j >= 1 && !mbar_wait(&bars.s_free, (j - 1) & 1)) return false;   // S(j-1) read out
                tc::fence_after();
#pragma unroll
                for (int kk = 0; kk < PF_HD / 16; ++kk) {
                    const uint32_t offk = (kk >> 2) * (PF_BN * 128) + (kk & 3) * 32;
                    tc::mma_bf16_ts(tS, tQ + kk * 8, tc::desc_k_sw128(aK + s * PF_KV_BYTES + offk), ID_QK,
                                    kk > 0 ? 1u : 0u);
                }
                tc::commit(&bars.s_full);
                tc::commit(&bars.k_empty[s]);
                return true;
            };
            auto issue_pv = [&](int i) -> bool {
                if (!mbar_wait(&bars.p_full, i & 1)) return false;
                if (!mbar_wait(&bars.v_full, i & 1)) return false;
                tc::fence_after();
#pragma unroll
                for (int kk = 0; kk < PF_BN / 16; ++kk) {
                    const uint64_t da = tc::desc_k_sw128(aP + (kk >> 2) * (PF_BM * 128) + (kk & 3) * 32);
                    const uint64_t db = tc::desc_mn_sw128(aV + kk * 16 * 128, PF_BN * 128, 1024);
                    tc::mma_bf16(tO, da, db, ID_PV, (i > 0 || kk > 0) ? 1u : 0u);
                }
                tc::commit(&bars.pv_done);
                tc::commit(&bars.v_empty);
                return true;
            };
            tc::fence_after();
            if (ok) ok = issue_s(0);
            for (int j = 0; ok && j < nt; ++j) {
                if (j + 1 < nt) ok = issue_s(j + 1);
                if (ok) ok = issue_pv(j);
            }
        }
    } else {
        // ------------------------------------------------ Q to TMEM, softmax, epilogue
        // Warp w (2..9) owns 16 query rows, 32 (w % 4) + 16 u with u = (w - 2) / 4,
        // through the 16x256b TMEM shape: thread (g = lane / 4, tq = lane % 4)
        // holds rows g and g + 8 of the 16 and columns 8j + 2tq, +1 of every
        // 8-column block, so the four threads of a row are one lane quad and
        // the row max and sum need two shuffles. Waits never break out of the
        // loop (a time-out raises the error word and the loop runs on).
        const int quarter = warp & 3, u = (warp - 2) >> 2;
        const int g = lane >> 2, tq = lane & 3;
        const int rbase = 32 * quarter + 16 * u;                // first TMEM lane (tile row) of the warp
        const uint32_t lane_off = (uint32_t)rbase << 16;
        const int row0 = rbase + g, row1 = row0 + 8;           // tile rows of this thread
        const int qpos0 = p.pos_base + q0 + row0, qpos1 = qpos0 + 8;
        const float sl2 = p.scale_log2;
        {   // Q tile (staged in the V buffer, 128B-swizzled 64-column boxes) into TMEM
            // as bf16 pairs: thread = tile row 32 quarter + lane, head dims 128 u ..
            mbar_wait(&bars.q_full, 0);
            const int row = 32 * quarter + lane;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float v[32];
#pragma unroll
                for (int c = 0; c < 8; ++c) {          // 16-byte chunk: 8 head dims = 4 columns
                    const int d = 128 * u + 64 * hh + 8 * c;
                    const uint4 w = *reinterpret_cast<const uint4 *>(
                        sV + (d >> 6) * (PF_BM * 128) + row * 128 + ((((d & 63) >> 3) ^ (row & 7)) << 4));
                    v[4 * c] = __uint_as_float(w.x); v[4 * c + 1] = __uint_as_float(w.y);
                    v[4 * c + 2] = __uint_as_float(w.z); v[4 * c + 3] = __uint_as_float(w.w);
                }
                tc::st32(tQ + 64 * u + 32 * hh + ((uint32_t)(32 * quarter) << 16), v);
            }
            tc::wait_st();
            tc::fence_before();
            mbar_arrive(&bars.q_tmem);                 // also frees the V buffer
        }
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
        for (int i = 0; i < nt; ++i) {
            mbar_wait(&bars.s_full, i & 1);
            tc::fence_after();
            float x[64];                               // two 64-key halves of the 16x256b.x8 shape
            {
                float xa[32], xb[32];
                tc::ld16x256_x8(tS + lane_off, xa);
                tc::ld16x256_x8(tS + 64 + lane_off, xb);
                tc::wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) { x[e] = xa[e]; x[32 + e] = xb[e]; }
            }
            tc::fence_before();
            mbar_arrive(&bars.s_free);
            // x[4j + 0/1]: row0, keys 8j + 2tq, +1 (j = 0..15 over the 128 keys);
            // x[4j + 2/3]: row1. Raw scores; the log2-domain scale is applied
            // inside the exponent (scale > 0, so the max commutes with it).
            const int key0 = i * PF_BN;
            if (key0 + PF_BN - 1 > qpos0) {                    // the tile crosses row0's diagonal
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int k = key0 + 8 * j + 2 * tq;
                    if (k > qpos0) x[4 * j] = -INFINITY;
                    if (k + 1 > qpos0) x[4 * j + 1] = -INFINITY;
                    if (k > qpos1) x[4 * j + 2] = -INFINITY;
                    if (k + 1 > qpos1) x[4 * j + 3] = -INFINITY;
                }
            }
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                mx0 = fmaxf(mx0, fmaxf(x[4 * j], x[4 * j + 1]));
                mx1 = fmaxf(mx1, fmaxf(x[4 * j + 2], x[4 * j + 3]));
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2)) * sl2;
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2)) * sl2;
            const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
            if (i == 0) {
                m0 = mn0; m1 = mn1;
            } else {
                const bool need0 = mn0 > m0 + PF_RESCALE_LOG2, need1 = mn1 > m1 + PF_RESCALE_LOG2;
                if (__any_sync(0xffffffffu, need0 || need1)) {
                    // O must be complete up to tile i-1 before it is rescaled
                    mbar_wait(&bars.pv_done, (i - 1) & 1);
                    tc::fence_after();
                    const float a0 = need0 ? exp2f(m0 - mn0) : 1.f, a1 = need1 ? exp2f(m1 - mn1) : 1.f;
#pragma unroll 1
                    for (int c = 0; c < PF_HD / 64; ++c) {
                        float o[32];
                        tc::ld16x256_x8(tO + 64 * c + lane_off, o);
                        tc::wait_ld();
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            o[4 * j] *= a0; o[4 * j + 1] *= a0; o[4 * j + 2] *= a1; o[4 * j + 3] *= a1;
                        }
                        tc::st16x256_x8(tO + 64 * c + lane_off, o);
                    }
                    tc::wait_st();
                    if (need0) { l0 *= a0; m0 = mn0; }
                    if (need1) { l1 *= a1; m1 = mn1; }
                }
            }
            const float mu0 = (m0 == -INFINITY) ? 0.f : m0, mu1 = (m1 == -INFINITY) ? 0.f : m1;
            uint32_t pk0[16], pk1[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float p00 = ex2_approx(fmaf(x[4 * j], sl2, -mu0)), p01 = ex2_approx(fmaf(x[4 * j + 1], sl2, -mu0));
                const float p10 = ex2_approx(fmaf(x[4 * j + 2], sl2, -mu1)), p11 = ex2_approx(fmaf(x[4 * j + 3], sl2, -mu1));
                l0 += p00 + p01;
                l1 += p10 + p11;
                pk0[j] = pack_bf16(p00, p01);
                pk1[j] = pack_bf16(p10, p11);
            }
            // the P buffer was last read by PV(i-1)
            if (i >= 1) mbar_wait(&bars.pv_done, (i - 1) & 1);
            // P row r, keys 8j..8j+7: atom j / 8 (64 keys), 16-byte chunk (j % 8) ^ (r & 7), pair tq at 4 tq
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int at = (j >> 3) * (PF_BM * 128);
                *reinterpret_cast<uint32_t *>(sP + at + row0 * 128 + (((j & 7) ^ (row0 & 7)) << 4) + 4 * tq) = pk0[j];
                *reinterpret_cast<uint32_t *>(sP + at + row1 * 128 + (((j & 7) ^ (row1 & 7)) << 4) + 4 * tq) = pk1[j];
            }
            fence_proxy_async();
            mbar_arrive(&bars.p_full);
        }
        // row sums: the quad's partial sums (same running max)
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        if (tq == 0) { bars.lsum[row0] = l0; bars.lsum[row1] = l1; }
        asm volatile("bar.sync 1, %0;" ::"n"(PF_SOFTMAX) : "memory");
        mbar_wait(&bars.pv_done, (nt - 1) & 1);
        tc::fence_after();
        if (p.tma_epi) {
            // TMA epilogue (bf16): thread = tile row 32 quarter + lane, O columns
            // 128 u ..; the gate tile (loaded by TMA into the second K buffer)
            // and the bf16 ctx tile (staged in the first) share the layout of
            // the 128B-swizzled 64 x 128 boxes, and one thread stores the tile
            // with four TMA box stores (rows past S are not written).
            const int row = 32 * quarter + lane;
            const uint32_t qoff = (uint32_t)(32 * quarter) << 16;
            const float inv_l = 1.f / bars.lsum[row];
            uint8_t *stage = sK;
            const uint8_t *gt = sK + PF_KV_BYTES;
            mbar_wait(&bars.g_full, 0);
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                float o[32];
                const int d0 = 128 * u + 32 * c;
                tc::ld32(tO + d0 + qoff, o);
                tc::wait_ld();
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int chunk = ((d0 & 63) >> 3) + k;
                    const uint32_t off = (d0 >> 6) * (PF_BM * 128) + row * 128 + ((chunk ^ (row & 7)) << 4);
                    float gv[8];
                    load8v(reinterpret_cast<const __nv_bfloat16 *>(gt + off), gv);
                    float y[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) y[e] = o[8 * k + e] * inv_l * sigmoidf_(gv[e]);
                    store8v(reinterpret_cast<__nv_bfloat16 *>(stage + off), y);
                }
            }
            fence_proxy_async();                   // the staged tile visible to the TMA
            asm volatile("bar.sync 1, %0;" ::"n"(PF_SOFTMAX) : "memory");
            if (warp == 2 && lane == 0) {
                for (int c = 0; c < 4; ++c) tma_store_3d(&em.ctx, stage + c * (PF_BM * 128), 64 * c, h, q0);
                tma_store_commit_wait();
            }
        } else {
            // epilogue, part 1: O / l through the 32x32b shape (thread = tile row
            // 32 quarter + lane, O columns 128 u ..) into fp32 staging rows in the
            // K buffers, which the last PV has finished with. 16-byte chunk c of
            // row r sits at chunk c ^ (r & 7): a warp's 32 rows spread over all banks.
            const int row = 32 * quarter + lane;
            const uint32_t qoff = (uint32_t)(32 * quarter) << 16;
            const float inv_l = 1.f / bars.lsum[row];
            float *stage = reinterpret_cast<float *>(sK);
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                float o[32];
                const int d0 = 128 * u + 32 * c;
                tc::ld32(tO + d0 + qoff, o);
                tc::wait_ld();
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int ch = (d0 >> 2) + e;
                    *reinterpret_cast<float4 *>(stage + row * PF_HD + ((ch ^ (row & 7)) << 2)) =
                        make_float4(o[4 * e] * inv_l, o[4 * e + 1] * inv_l, o[4 * e + 2] * inv_l, o[4 * e + 3] * inv_l);
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(PF_SOFTMAX) : "memory");
            // part 2: a warp per row, lane = 8 head dims: coalesced gate loads and
            // ctx stores, ctx = O / l * sigmoid(gate)
            const int w = warp - 2;
#pragma unroll 1
            for (int r = w; r < PF_BM; r += PF_SOFTMAX / 32) {
                const int srow = q0 + r;
                if (srow >= p.S) break;
                const float4 a0 = *reinterpret_cast<const float4 *>(stage + r * PF_HD + (((2 * lane) ^ (r & 7)) << 2));
                const float4 a1 = *reinterpret_cast<const float4 *>(stage + r * PF_HD + (((2 * lane + 1) ^ (r & 7)) << 2));
                const float o[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const TI *gate = static_cast<const TI *>(p.qg) + ((size_t)srow * Hin + p.h0 + h) * 2 * PF_HD + PF_HD + 8 * lane;
                const size_t off = ((size_t)srow * H + h) * PF_HD + 8 * lane;
                float gv[8], y[8];
                load8v(gate, gv);
#pragma unroll
                for (int e = 0; e < 8; ++e) y[e] = o[e] * sigmoidf_(gv[e]);
                if (p.gather.world == 0) {
                    store8v(static_cast<TO *>(p.ctx) + off, y);
                } else {   // every rank's gathered buffer, this rank's block (peer stores over NVLink)
                    const size_t boff = (size_t)p.gather.rank * p.gather.block + off;
                    for (int rk = 0; rk < p.gather.world; ++rk) store8v(static_cast<TO *>(p.gather.dst[rk]) + boff, y);
                }
            }
            if (p.gather.world) __threadfence_system();   // peer stores visible before the cross-rank barrier
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after();
        tc::dealloc(tbase, 512);
    }
}

cudaError_t launch_gqa_prefill(const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv,
                               const GqaPrefillArgs &a, int in_bf16, int out_bf16, cudaStream_t st,
                               const PfEpiMaps *em)
{
    // the epilogue reads the gate and writes ctx with 16-byte vectors
    if (((uintptr_t)a.qg | (uintptr_t)a.ctx) & 15) return cudaErrorMisalignedAddress;
    dim3 grid(a.n_qtiles * a.H), block(PF_THREADS);
    GqaPrefillArgs args = a;
    PfEpiMaps maps;
    memset(&maps, 0, sizeof(maps));
    args.tma_epi = (em && in_bf16 && out_bf16 && a.gather.world == 0) ? 1 : 0;
    if (args.tma_epi) maps = *em;
    auto run = [&](auto kern) -> cudaError_t {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
        if (e != cudaSuccess) return e;
        kern<<<grid, block, PF_SMEM, st>>>(tq, tk, tv, args, maps);
        return cudaGetLastError();
    };
    if (in_bf16 && out_bf16) return run(gqa_prefill_kernel<__nv_bfloat16, __nv_bfloat16>);
    if (!in_bf16 && !out_bf16) return run(gqa_prefill_kernel<float, float>);
    return cudaErrorInvalidValue;
}

}  // namespace coli
