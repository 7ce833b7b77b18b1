// Gated GQA causal prefill on the 5th-gen tensor cores (tcgen05 + TMEM + TMA).
//
// Same per-row semantics as the reference's attention() hot loop
// (c/qwen.c:638-663): query row s (position pos_base+s) attends to cache rows
// 0..pos_base+s of its KV head (h / 8) with scale 1/sqrt(256); ctx is gated by
// sigmoid(gate). The prologue (q/k norm, RoPE, K/V append) runs before this
// kernel (gqa_prologue_kernel), so the new rows are already in the cache.
//
// One CTA = 128 query rows of one Q head. Warp roles (576 threads):
//   warp 0      TMA producers (lane 0: Q once, then K; lane 1: V): 64-key
//               tiles into separate 2-stage K and V rings (128B swizzle).
//   warp 1      MMA issuer (one thread) and TMEM owner: S = Q K^T into one of
//               two TMEM score buffers (M=128, N=64, K=256), then
//               O += P V (M=128, N=256, K=64) with V read MN-major.
//   warps 2..17 softmax: four threads per query row (TMEM lane), scores read
//               with tcgen05.ld, causal mask, online softmax in the log2
//               domain with lazy rescaling (O is corrected in TMEM only when
//               the running max grows by more than 2^8), P written to shared
//               memory in the UMMA K-major layout; final epilogue O / l *
//               sigmoid(gate).
// TMEM: 2 x 64 columns of scores + 256 columns of O (512 allocated).
// Every wait is bounded (see mbar_wait); no cluster multicast.
#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace coli {

constexpr int PF_BM = 128, PF_BN = 64, PF_HD = 256;
constexpr int PF_Q_BYTES = PF_BM * PF_HD * 2;        // 64 KiB
constexpr int PF_KV_BYTES = PF_BN * PF_HD * 2;       // 32 KiB per K (or V) tile
constexpr int PF_P_BYTES = PF_BM * PF_BN * 2;        // 16 KiB
constexpr int PF_DATA = PF_Q_BYTES + 4 * PF_KV_BYTES + PF_P_BYTES;  // 208 KiB
constexpr int PF_THREADS = 576;
constexpr float PF_RESCALE_LOG2 = 8.0f;


struct PfBars {
    uint64_t q_full, k_full[2], v_full[2], k_empty[2], v_empty[2], s_full[2], s_free[2], p_full[2], pv_done[2];
    uint32_t tmem_base;
    // per-tile row max of each half (double-buffered by tile parity); after
    // the loop the buffer the last tile did not use carries the row sums
    float mx[2][4][PF_BM];
};
constexpr int PF_SMEM = PF_DATA + (int)sizeof(PfBars);
static_assert(PF_SMEM <= 232448, "prefill shared memory exceeds the 227 KiB per-CTA limit");

template <typename TI, typename TO>
__global__ void __launch_bounds__(PF_THREADS, 1)
gqa_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, GqaPrefillArgs p)
{
    // All shared memory is dynamic (no static __shared__), so the window
    // starts 1024-byte aligned as the 128B-swizzled TMA boxes and UMMA
    // descriptors need; checked below rather than padded (the budget is tight).
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw;
    uint8_t *sQ = smem;
    uint8_t *sK = sQ + PF_Q_BYTES;              // [2][32 KiB]
    uint8_t *sV = sK + 2 * PF_KV_BYTES;         // [2][32 KiB]
    uint8_t *sP = sV + 2 * PF_KV_BYTES;         // 16 KiB P tile
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
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars.k_full[i], 1);
            mbar_init(&bars.v_full[i], 1);
            mbar_init(&bars.k_empty[i], 1);
            mbar_init(&bars.v_empty[i], 1);
            mbar_init(&bars.s_full[i], 1);
            mbar_init(&bars.s_free[i], 512);
            mbar_init(&bars.p_full[i], 512);
            mbar_init(&bars.pv_done[i], 1);
        }
        fence_mbar_init();
    }
    if (warp == 1) tc::alloc(&bars.tmem_base, 512);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = bars.tmem_base;
    const uint32_t tS0 = tbase, tO = tbase + 128;

    if (warp == 0) {
        // ------------------------------------------------ TMA producers
        // Lane 0 streams K (a stage frees as soon as its S MMA completes),
        // lane 1 streams V (freed after its PV MMA), so the next K tile is in
        // flight while the current tile's softmax and PV still run.
        if (lane == 0) {
            tma_prefetch_desc(&tmQ); tma_prefetch_desc(&tmK);
            mbar_expect_tx(&bars.q_full, PF_Q_BYTES);
            for (int c = 0; c < 4; ++c) tma_load_3d(sQ + c * (PF_BM * 128), &tmQ, 64 * c, h, q0, &bars.q_full);
            for (int j = 0; j < nt; ++j) {
                const int s = j & 1;
                if (j >= 2 && !mbar_wait(&bars.k_empty[s], ((j >> 1) - 1) & 1)) break;
                mbar_expect_tx(&bars.k_full[s], PF_KV_BYTES);
                for (int c = 0; c < 4; ++c)
                    tma_load_2d(sK + s * PF_KV_BYTES + c * (PF_BN * 128), &tmK, 64 * c,
                                kvrow0 + j * PF_BN, &bars.k_full[s]);
            }
        } else if (lane == 1) {
            tma_prefetch_desc(&tmV);
            for (int j = 0; j < nt; ++j) {
                const int s = j & 1;
                if (j >= 2 && !mbar_wait(&bars.v_empty[s], ((j >> 1) - 1) & 1)) break;
                mbar_expect_tx(&bars.v_full[s], PF_KV_BYTES);
                for (int c = 0; c < 4; ++c)
                    tma_load_2d(sV + s * PF_KV_BYTES + c * (PF_BN * 128), &tmV, 64 * c,
                                kvrow0 + j * PF_BN, &bars.v_full[s]);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t ID_QK = tc::idesc_bf16(PF_BM, PF_BN, 0, 0);
            constexpr uint32_t ID_PV = tc::idesc_bf16(PF_BM, PF_HD, 0, 1);
            const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
            bool ok = mbar_wait(&bars.q_full, 0);
            auto issue_pv = [&](int i) -> bool {
                const int b = i & 1;
                if (!mbar_wait(&bars.p_full[b], (i >> 1) & 1)) return false;
                if (!mbar_wait(&bars.v_full[b], (i >> 1) & 1)) return false;
                tc::fence_after();
#pragma unroll
                for (int kk = 0; kk < PF_BN / 16; ++kk) {
                    const uint64_t da = tc::desc_k_sw128(aP + kk * 32);
                    const uint64_t db = tc::desc_mn_sw128(aV + b * PF_KV_BYTES + kk * 16 * 128,
                                                          PF_BN * 128, 1024);
                    tc::mma_bf16(tO, da, db, ID_PV, (i > 0 || kk > 0) ? 1u : 0u);
                }
                tc::commit(&bars.pv_done[b]);
                tc::commit(&bars.v_empty[b]);
                return true;
            };
            for (int j = 0; ok && j < nt; ++j) {
                const int s = j & 1;
                if (!mbar_wait(&bars.k_full[s], (j >> 1) & 1)) { ok = false; break; }
                if (j >= 2 && !mbar_wait(&bars.s_free[s], ((j >> 1) - 1) & 1)) { ok = false; break; }
                tc::fence_after();
#pragma unroll
                for (int kk = 0; kk < PF_HD / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * (PF_BM * 128) + (kk & 3) * 32;
                    const uint32_t offk = (kk >> 2) * (PF_BN * 128) + (kk & 3) * 32;
                    tc::mma_bf16(tS0 + s * PF_BN, tc::desc_k_sw128(aQ + off),
                                 tc::desc_k_sw128(aK + s * PF_KV_BYTES + offk), ID_QK, kk > 0 ? 1u : 0u);
                }
                tc::commit(&bars.s_full[s]);
                tc::commit(&bars.k_empty[s]);
                if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
            }
            if (ok) issue_pv(nt - 1);
        }
    } else {
        // ------------------------------------------------ softmax + epilogue
        // Four threads per query row: warp w (2..17) takes score columns
        // 16q..16q+15 and O columns 64q..64q+63 with q = (w-2)/4, of TMEM lanes
        // 32(w%4).. Row maxima are exchanged through shared memory under a
        // named barrier of the 512 softmax threads. Waits never break out of
        // the loop (a time-out raises the error word and the loop runs on), so
        // every thread meets every named barrier.
        const int qr = (warp - 2) >> 2;
        const int row = 32 * (warp & 3) + lane;            // TMEM lane == query row in tile
        const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
        const int srow = q0 + row;                         // query row index in [0, S)
        const int qpos = p.pos_base + srow;
        const float sl2 = p.scale_log2;
        float m = -INFINITY, l = 0.f;
        for (int i = 0; i < nt; ++i) {
            const int b = i & 1;
            mbar_wait(&bars.s_full[b], (i >> 1) & 1);
            tc::fence_after();
            float x[16];
            tc::ld16(tS0 + b * PF_BN + 16 * qr + lane_off, x);
            tc::wait_ld();
            tc::fence_before();
            mbar_arrive(&bars.s_free[b]);
            // Raw scores; the log2-domain scale is applied inside the exponent
            // (scale > 0, so the max commutes with it).
            const int key0 = i * PF_BN + 16 * qr;
            float mx = -INFINITY;
            if (key0 + 15 <= qpos) {                       // tile fully visible to this row
#pragma unroll
                for (int c = 0; c < 16; ++c) mx = fmaxf(mx, x[c]);
            } else {
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    x[c] = (key0 + c <= qpos) ? x[c] : -INFINITY;
                    mx = fmaxf(mx, x[c]);
                }
            }
            mx *= sl2;
            bars.mx[b][qr][row] = mx;
            asm volatile("bar.sync 1, 512;" ::: "memory");
            mx = fmaxf(fmaxf(bars.mx[b][0][row], bars.mx[b][1][row]),
                       fmaxf(bars.mx[b][2][row], bars.mx[b][3][row]));
            const float mnew = fmaxf(m, mx);
            if (i == 0) {
                m = mnew;
            } else {
                const bool need = mnew > m + PF_RESCALE_LOG2;
                if (__any_sync(0xffffffffu, need)) {
                    // O must be complete up to tile i-1 before it is rescaled
                    mbar_wait(&bars.pv_done[(i - 1) & 1], ((i - 1) >> 1) & 1);
                    tc::fence_after();
                    const float alpha = need ? exp2f(m - mnew) : 1.f;
#pragma unroll 1
                    for (int c = 0; c < 2; ++c) {
                        float o[32];
                        const uint32_t col = tO + 64 * qr + 32 * c + lane_off;
                        tc::ld32(col, o);
                        tc::wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] *= alpha;
                        tc::st32(col, o);
                    }
                    tc::wait_st();
                    if (need) { l *= alpha; m = mnew; }
                }
            }
            const float mu = (m == -INFINITY) ? 0.f : m;
            float rs = 0.f;
            uint32_t pk[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float p0 = ex2_approx(fmaf(x[2 * c], sl2, -mu)), p1 = ex2_approx(fmaf(x[2 * c + 1], sl2, -mu));
                rs += p0 + p1;
                pk[c] = pack_bf16(p0, p1);
            }
            l += rs;
            // the single P buffer was last read by PV(i-1)
            if (i >= 1) mbar_wait(&bars.pv_done[(i - 1) & 1], ((i - 1) >> 1) & 1);
            uint8_t *prow = sP + row * 128;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int ch = 2 * qr + q;
                *reinterpret_cast<uint4 *>(prow + ((ch ^ (row & 7)) << 4)) =
                    make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
            }
            fence_proxy_async();
            mbar_arrive(&bars.p_full[b]);
        }
        // row sum = the four partial sums (same running max); the buffer the
        // last tile did not use carries them
        bars.mx[nt & 1][qr][row] = l;
        asm volatile("bar.sync 1, 512;" ::: "memory");
        l = (bars.mx[nt & 1][0][row] + bars.mx[nt & 1][1][row]) +
            (bars.mx[nt & 1][2][row] + bars.mx[nt & 1][3][row]);
        mbar_wait(&bars.pv_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1);
        tc::fence_after();
        {
            const float inv_l = 1.f / l;
            const bool valid = srow < p.S;
            const TI *gate = static_cast<const TI *>(p.qg) + ((size_t)srow * Hin + p.h0 + h) * 2 * PF_HD + PF_HD;
            TO *out = static_cast<TO *>(p.ctx) + ((size_t)srow * H + h) * PF_HD;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                float o[32];
                const int d0 = 64 * qr + 32 * c;
                tc::ld32(tO + d0 + lane_off, o);
                tc::wait_ld();
                if (valid) {
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        out[d0 + e] = from_f32<TO>(o[e] * inv_l * sigmoidf_(to_f32(gate[d0 + e])));
                }
            }
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
                               const GqaPrefillArgs &a, int in_bf16, int out_bf16, cudaStream_t st)
{
    dim3 grid(a.n_qtiles * a.H), block(PF_THREADS);
    auto run = [&](auto kern) -> cudaError_t {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
        if (e != cudaSuccess) return e;
        kern<<<grid, block, PF_SMEM, st>>>(tq, tk, tv, a);
        return cudaGetLastError();
    };
    if (in_bf16 && out_bf16) return run(gqa_prefill_kernel<__nv_bfloat16, __nv_bfloat16>);
    if (!in_bf16 && !out_bf16) return run(gqa_prefill_kernel<float, float>);
    return cudaErrorInvalidValue;
}

}  // namespace coli
