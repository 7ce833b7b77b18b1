// Dense projections on the 5th-gen tensor core: y[s][o] = sum_i x[s][i] W[o][i]
// (the reference's matmul(), c/qwen.c:178-189, with W [O][I] row-major as the
// engine stores it). bf16 W and x, fp32 accumulation in TMEM.
//
// One CTA = 128 output features x BN tokens (BN = 16..256 by S, so decode with
// a handful of tokens is a weight-streaming pass), K walked in 64-element
// (128 B) steps through a TMA ring of 4 (BN = 256) to 12 (BN = 16) stages. W is the M operand (K-major rows),
// x the N operand (K-major rows); both 128B-swizzled. When the output tiles
// cannot fill the GPU (decode), K is split over blockIdx.z and the partial sums
// are added in split order (deterministic): for up to 16 tokens by the last
// split of each output tile to arrive (an atomic counter per tile), with no
// second launch; for more tokens by linear_reduce_kernel.
// For up to 16 tokens and at most 8 splits the splits of a tile run as one
// thread-block cluster instead: each leaves its partial in its own shared
// memory and the first adds them in split order through distributed shared
// memory (no global partials, counters or fences on the tail).
// Warp roles: 0 = TMA producer, 1 = TMEM owner + MMA issuer, 2..5 = epilogue
// (TMEM lane = output feature; stores are contiguous along o for each token).
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace coli {

#ifndef LIN_DEC_STAGES
#define LIN_DEC_STAGES 6    // ring stages of the decode (BN = 16) kernel: two CTAs fit an SM
#endif
#ifndef LIN_MAX_CLUSTER
#define LIN_MAX_CLUSTER 8   // most K splits reduced in a cluster (portable cluster size)
#endif
constexpr int LN_BM = 128, LN_BK = 64;
constexpr int LN_A_BYTES = LN_BM * LN_BK * 2;   // 16 KiB

template <int BN> struct LinSmem {
    static constexpr int B_BYTES = BN * LN_BK * 2;
    static constexpr int STAGE = LN_A_BYTES + B_BYTES;
    // as many ring stages as ~220 KiB holds (at most 12): a weight-streaming
    // decode pass needs many bytes in flight per SM to cover HBM latency
    static constexpr int STAGES_FIT = (220 * 1024) / STAGE;
    static constexpr int STAGES_MAX = BN == 16 ? LIN_DEC_STAGES : 12;
    static constexpr int STAGES = STAGES_FIT > STAGES_MAX ? STAGES_MAX : (STAGES_FIT < 2 ? 2 : STAGES_FIT);
    static constexpr int TOTAL = STAGES * STAGE + 1024;
    static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
};

// The weights of one launch: w[i] covers output tiles [tile_end[i-1], tile_end[i])
// of blockIdx.x, has O[i] outputs into y[i], and its split-K partials start
// part_off[i] floats into LinearArgs::part.
struct LinWeights {
    CUtensorMap w[LIN_MAXW];
    int tile_end[LIN_MAXW], O[LIN_MAXW];
    void *y[LIN_MAXW];
    size_t part_off[LIN_MAXW];
    int nw;
};

// Timing probe (development builds with -DCOLI_SCAN_PROBE only): globaltimer
// at fixed points of every CTA of the decode kernel.
#ifdef COLI_SCAN_PROBE
__device__ unsigned long long g_lin_probe[1024 * 8];
#define LIN_PROBE(slot) do { if (BN == 16) { const int c_ = blockIdx.x + gridDim.x * blockIdx.z; \
    if (c_ < 1024) g_lin_probe[c_ * 8 + (slot)] = globaltimer_ns(); } } while (0)
#else
#define LIN_PROBE(slot) do { } while (0)
#endif

template <int BN>
__global__ void __launch_bounds__(192, 1)
linear_kernel(const __grid_constant__ LinWeights lw, const __grid_constant__ CUtensorMap tmX, LinearArgs a)
{
    constexpr int LN_STAGES = LinSmem<BN>::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full[LN_STAGES], empty[LN_STAGES], done;
    __shared__ uint32_t tmem_base;
    __shared__ int last_split;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int wi = 0;                                // this CTA's weight
    while (wi + 1 < lw.nw && (int)blockIdx.x >= lw.tile_end[wi]) ++wi;
    const CUtensorMap *tmW = &lw.w[wi];
    const int O = lw.O[wi];
    void *const yout = lw.y[wi];
    float *const part = a.part ? a.part + lw.part_off[wi] : nullptr;
    const int o0 = ((int)blockIdx.x - (wi ? lw.tile_end[wi - 1] : 0)) * LN_BM, s0 = blockIdx.y * BN, z = blockIdx.z;
    const int nk = (a.I + LN_BK - 1) / LN_BK;
    const int k0 = z * a.kchunks, k1 = min(nk, k0 + a.kchunks), cnt = max(0, k1 - k0);
    const bool clus = BN <= 64 && a.cluster && gridDim.z > 1;   // uniform across the cluster

    if (threadIdx.x == 0) {
        for (int i = 0; i < LN_STAGES; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        mbar_init(&done, 1);
        fence_mbar_init();
    }
    if (warp == 1) tc::alloc(&tmem_base, LinSmem<BN>::TMEM_COLS);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tD = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            LIN_PROBE(0);
            tma_prefetch_desc(tmW); tma_prefetch_desc(&tmX);
            // the weights do not depend on the previous kernel: the first ring's
            // worth streams in while that kernel finishes (programmatic launch)
            const int pre = min(cnt, LN_STAGES);
            for (int i = 0; i < pre; ++i) {
                mbar_expect_tx(&full[i], LinSmem<BN>::STAGE);
                tma_load_2d(sm + i * LinSmem<BN>::STAGE, tmW, (k0 + i) * LN_BK, o0, &full[i]);
            }
            griddep_wait();
            LIN_PROBE(1);
            for (int i = 0; i < pre; ++i)
                tma_load_2d(sm + i * LinSmem<BN>::STAGE + LN_A_BYTES, &tmX, (k0 + i) * LN_BK, s0, &full[i]);
            for (int i = pre; i < cnt; ++i) {
                const int st = i % LN_STAGES;
                mbar_wait(&empty[st], ((i / LN_STAGES) + 1) & 1);
                uint8_t *sA = sm + st * LinSmem<BN>::STAGE, *sB = sA + LN_A_BYTES;
                mbar_expect_tx(&full[st], LinSmem<BN>::STAGE);
                tma_load_2d(sA, tmW, (k0 + i) * LN_BK, o0, &full[st]);
                tma_load_2d(sB, &tmX, (k0 + i) * LN_BK, s0, &full[st]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_bf16(LN_BM, BN, 0, 0);
            const uint32_t base = smem_u32(sm);
            for (int i = 0; i < cnt; ++i) {
                const int st = i % LN_STAGES;
                mbar_wait(&full[st], (i / LN_STAGES) & 1);
                tc::fence_after();
                const uint32_t aA = base + st * LinSmem<BN>::STAGE, aB = aA + LN_A_BYTES;
#pragma unroll
                for (int kk = 0; kk < LN_BK / 16; ++kk)
                    tc::mma_bf16(tD, tc::desc_k_sw128(aA + kk * 32), tc::desc_k_sw128(aB + kk * 32), idesc,
                                 (i > 0 || kk > 0) ? 1u : 0u);
                tc::commit(&empty[st]);
            }
            tc::commit(&done);
        }
    } else {
        const int q = warp & 3, o = o0 + q * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        griddep_wait();                       // y / partials / counters may still be in use
        if (cnt > 0) {
            mbar_wait(&done, 0);
            tc::fence_after();
        }
        if (threadIdx.x == 64) LIN_PROBE(2);
        griddep_launch();
        for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
            if (cnt > 0) {
                tc::ld16(tD + lane_off + c0, v);
                tc::wait_ld();
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0.f;
            }
            if (clus) {   // [BN tokens][128 outputs] over the first ring stages (every MMA has completed)
                float *red = reinterpret_cast<float *>(sm);
#pragma unroll
                for (int j = 0; j < 16; ++j) red[(c0 + j) * LN_BM + q * 32 + lane] = v[j];
                continue;
            }
            if (o < O) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int s = s0 + c0 + j;
                    if (s >= a.S) break;
                    const size_t idx = (size_t)s * O + o;
                    if (part) part[(size_t)z * a.S * O + idx] = v[j];
                    else if (a.y_bf16) static_cast<__nv_bfloat16 *>(yout)[idx] = __float2bfloat16_rn(v[j]);
                    else static_cast<float *>(yout)[idx] = v[j];
                }
            }
        }
        tc::fence_before();
        if (BN == 16 && part && a.tile_cnt && !clus) {
            // split-K: the last split of this output tile to arrive adds the
            // partials in split order (the same sum as linear_reduce_kernel)
            __threadfence();
            asm volatile("bar.sync 2, 128;" ::: "memory");
            const int tile = blockIdx.x + gridDim.x * blockIdx.y;
            if (threadIdx.x == 64) {
                LIN_PROBE(3);
                last_split = atomicAdd(&a.tile_cnt[tile], 1) == (int)gridDim.z - 1;
            }
            asm volatile("bar.sync 2, 128;" ::: "memory");
            if (last_split) {
                __threadfence();
                const size_t n = (size_t)a.S * O;
                if (o < O) {
                    // up to 16 token rows: each split's loads go out together
                    const int rows = min(a.S - s0, min(BN, 16));
                    float acc[16];
#pragma unroll
                    for (int r = 0; r < 16; ++r) acc[r] = 0.f;
                    for (int zz = 0; zz < (int)gridDim.z; ++zz) {
                        const float *pz = part + zz * n + (size_t)s0 * O + o;
#pragma unroll
                        for (int r = 0; r < 16; ++r)
                            if (r < rows) acc[r] += __ldcg(pz + (size_t)r * O);
                    }
#pragma unroll
                    for (int r = 0; r < 16; ++r) {
                        if (r >= rows) break;
                        const size_t idx = (size_t)(s0 + r) * O + o;
                        if (a.y_bf16) static_cast<__nv_bfloat16 *>(yout)[idx] = __float2bfloat16_rn(acc[r]);
                        else static_cast<float *>(yout)[idx] = acc[r];
                    }
                }
                if (threadIdx.x == 64) {
                    a.tile_cnt[tile] = 0;
                    LIN_PROBE(4);
                }
            }
        }
    }
    if (clus) {
        namespace cg = cooperative_groups;
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();                                 // every split's partial in its shared memory
        if (z == 0 && warp >= 2) {
            const int q = warp & 3, ol = q * 32 + lane, o = o0 + ol;
            if (threadIdx.x == 64) LIN_PROBE(3);
            for (int c0 = 0; c0 < BN && o < O; c0 += 16) {   // 16 token rows at a time
                const int rows = min(a.S - s0 - c0, 16);
                if (rows <= 0) break;
                float acc[16];
#pragma unroll
                for (int r = 0; r < 16; ++r) acc[r] = 0.f;
                for (int zz = 0; zz < (int)gridDim.z; ++zz) {
                    const float *pr = cl.map_shared_rank(reinterpret_cast<const float *>(sm), zz) + c0 * LN_BM + ol;
#pragma unroll
                    for (int r = 0; r < 16; ++r)
                        if (r < rows) acc[r] += pr[r * LN_BM];
                }
#pragma unroll
                for (int r = 0; r < 16; ++r) {
                    if (r >= rows) break;
                    const size_t idx = (size_t)(s0 + c0 + r) * O + o;
                    if (a.y_bf16) static_cast<__nv_bfloat16 *>(yout)[idx] = __float2bfloat16_rn(acc[r]);
                    else static_cast<float *>(yout)[idx] = acc[r];
                }
            }
            if (threadIdx.x == 64) LIN_PROBE(4);
        }
        cl.sync();                                 // the peers' shared memory stays until it has been read
    }
    __syncthreads();
    if (warp == 1) {
        tc::fence_after();
        tc::dealloc(tmem_base, LinSmem<BN>::TMEM_COLS);
    }
}

// Persistent variant for large token counts (BN = 128 / 256, no K split): one
// CTA per SM walks the output tiles (tile t = blockIdx.x + k gridDim.x, output
// features fastest) with two TMEM accumulators, so the epilogue of tile j
// overlaps the MMAs of tile j + 1 and the TMA ring never drains between tiles.
template <int BN>
__global__ void __launch_bounds__(192, 1)
linear_persistent_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                         LinearArgs a)
{
    constexpr int ST = LinSmem<BN>::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full[ST], empty[ST], tfull[2], tempty[2];
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntx = (a.O + LN_BM - 1) / LN_BM, nty = (a.S + BN - 1) / BN, ntiles = ntx * nty;
    const int nk = (a.I + LN_BK - 1) / LN_BK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < ST; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], 128); }
        fence_mbar_init();
    }
    if (warp == 1) tc::alloc(&tmem_base, 2 * BN);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tD = tmem_base;
    griddep_wait();

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmW); tma_prefetch_desc(&tmX);
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
                const int o0 = (t % ntx) * LN_BM, s0 = (t / ntx) * BN;
                for (int k = 0; k < nk; ++k, ++it) {
                    const int st = it % ST;
                    if (it >= ST && !mbar_wait(&empty[st], ((it / ST) + 1) & 1)) { ok = false; break; }
                    uint8_t *sA = sm + st * LinSmem<BN>::STAGE, *sB = sA + LN_A_BYTES;
                    mbar_expect_tx(&full[st], LinSmem<BN>::STAGE);
                    tma_load_2d(sA, &tmW, k * LN_BK, o0, &full[st]);
                    tma_load_2d(sB, &tmX, k * LN_BK, s0, &full[st]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_bf16(LN_BM, BN, 0, 0);
            const uint32_t base = smem_u32(sm);
            int it = 0, j = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++j) {
                const int acc = j & 1;
                if (j >= 2 && !mbar_wait(&tempty[acc], ((j >> 1) + 1) & 1)) break;   // epilogue drained it
                tc::fence_after();
                const uint32_t d = tD + acc * BN;
                for (int k = 0; k < nk; ++k, ++it) {
                    const int st = it % ST;
                    if (!mbar_wait(&full[st], (it / ST) & 1)) { ok = false; break; }
                    tc::fence_after();
                    const uint32_t aA = base + st * LinSmem<BN>::STAGE, aB = aA + LN_A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < LN_BK / 16; ++kk)
                        tc::mma_bf16(d, tc::desc_k_sw128(aA + kk * 32), tc::desc_k_sw128(aB + kk * 32), idesc,
                                     (k > 0 || kk > 0) ? 1u : 0u);
                    tc::commit(&empty[st]);
                }
                tc::commit(&tfull[acc]);
            }
        }
    } else {
        const int q = warp & 3;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        int j = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++j) {
            const int acc = j & 1;
            const int o = (t % ntx) * LN_BM + q * 32 + lane, s0 = (t / ntx) * BN;
            if (!mbar_wait(&tfull[acc], (j >> 1) & 1)) break;
            tc::fence_after();
            const uint32_t d = tD + acc * BN + lane_off;
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float v[16];
                tc::ld16(d + c0, v);
                tc::wait_ld();
                if (o < a.O) {
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int s = s0 + c0 + jj;
                        if (s >= a.S) break;
                        const size_t idx = (size_t)s * a.O + o;
                        if (a.y_bf16) static_cast<__nv_bfloat16 *>(a.y)[idx] = __float2bfloat16_rn(v[jj]);
                        else static_cast<float *>(a.y)[idx] = v[jj];
                    }
                }
            }
            tc::fence_before();
            mbar_arrive(&tempty[acc]);
        }
        griddep_launch();
    }
    __syncthreads();
    if (warp == 1) {
        tc::fence_after();
        tc::dealloc(tmem_base, 2 * BN);
    }
}

// y = sum over splits of the partials, in split order.
__global__ void linear_reduce_kernel(LinearArgs a, int splits)
{
    const size_t n = (size_t)a.S * a.O;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float acc = 0.f;
        for (int z = 0; z < splits; ++z) acc += a.part[(size_t)z * n + i];
        if (a.y_bf16) static_cast<__nv_bfloat16 *>(a.y)[i] = __float2bfloat16_rn(acc);
        else static_cast<float *>(a.y)[i] = acc;
    }
}

// fp32 -> bf16, n elements (n a multiple of 4 is not required).
__global__ void f32_to_bf16_kernel(const float *x, __nv_bfloat16 *y, size_t n)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __float2bfloat16_rn(x[i]);
}

cudaError_t launch_f32_to_bf16(const float *x, __nv_bfloat16 *y, size_t n, cudaStream_t st)
{
    const int blocks = (int)std::min<size_t>((n + 255) / 256, 4096);
    f32_to_bf16_kernel<<<blocks, 256, 0, st>>>(x, y, n);
    return cudaGetLastError();
}

int linear_pick_bn(int S)
{
    return S <= 16 ? 16 : S <= 32 ? 32 : S <= 64 ? 64 : S <= 128 ? 128 : 256;
}

cudaError_t launch_linear(const CUtensorMap &tmW, const CUtensorMap &tmX, LinearArgs a, int bn, int splits,
                          cudaStream_t st, int *launches)
{
    static_assert(64 * LN_BM * 4 <= 2 * LinSmem<64>::STAGE, "cluster partials fit the first two ring stages");
    if (launches) *launches = 1;
    const int nk = (a.I + LN_BK - 1) / LN_BK;
    a.kchunks = (nk + splits - 1) / splits;
    splits = (nk + a.kchunks - 1) / a.kchunks;   // no split without K chunks
    if (splits == 1) { a.part = nullptr; a.tile_cnt = nullptr; }
    // clusters of up to 8 CTAs at two CTAs per SM (BN = 16); the larger tiles
    // hold one CTA per SM, where 8-CTA clusters no longer fit one wave
    a.cluster = bn <= 64 && splits > 1 && splits <= (bn == 16 ? LIN_MAX_CLUSTER : 4);
    dim3 grid((a.O + LN_BM - 1) / LN_BM, (a.S + bn - 1) / bn, splits);
    // the shared-memory opt-in, once per instantiation and device
    static bool attr_set[16][7] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    bool *set = attr_set[dev & 15];
    LinWeights lw;
    memset(&lw, 0, sizeof(lw));
    lw.w[0] = tmW; lw.tile_end[0] = grid.x; lw.O[0] = a.O; lw.y[0] = a.y; lw.nw = 1;
    auto run = [&](auto kern, int smem, int which, const auto &wts) -> cudaError_t {
        if (!set[which] || dev >= 16) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return e;
            set[which] = true;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = grid; cfg.blockDim = dim3(192); cfg.dynamicSmemBytes = smem; cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr; cfg.numAttrs = 1;
        if (a.cluster) {
            attr[1].id = cudaLaunchAttributeClusterDimension;
            attr[1].val.clusterDim.x = 1; attr[1].val.clusterDim.y = 1; attr[1].val.clusterDim.z = grid.z;
            cfg.numAttrs = 2;
        }
        return cudaLaunchKernelEx(&cfg, kern, wts, tmX, a);
    };
    cudaError_t e;
    if (splits == 1 && bn >= 128) {
        // persistent: one CTA per SM over all output tiles
        const int tiles = grid.x * grid.y;
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        grid = dim3(std::min(tiles, std::max(sms, 1)), 1, 1);
        if (bn == 128) return run(linear_persistent_kernel<128>, LinSmem<128>::TOTAL, 5, tmW);
        return run(linear_persistent_kernel<256>, LinSmem<256>::TOTAL, 6, tmW);
    }
    switch (bn) {
    case 16: e = run(linear_kernel<16>, LinSmem<16>::TOTAL, 0, lw); break;
    case 32: e = run(linear_kernel<32>, LinSmem<32>::TOTAL, 1, lw); break;
    case 64: e = run(linear_kernel<64>, LinSmem<64>::TOTAL, 2, lw); break;
    case 128: e = run(linear_kernel<128>, LinSmem<128>::TOTAL, 3, lw); break;
    case 256: e = run(linear_kernel<256>, LinSmem<256>::TOTAL, 4, lw); break;
    default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess || splits == 1 || a.cluster || (bn == 16 && a.tile_cnt)) return e;
    if (launches) *launches = 2;
    const size_t n = (size_t)a.S * a.O;
    linear_reduce_kernel<<<(int)std::min<size_t>((n + 255) / 256, 4096), 256, 0, st>>>(a, splits);
    return cudaGetLastError();
}

cudaError_t launch_linear_multi(const CUtensorMap *const *tmW, const int *O, void *const *y, int nw,
                                const CUtensorMap &tmX, LinearArgs a, int splits, cudaStream_t st)
{
    if (nw < 1 || nw > LIN_MAXW || a.S > 16) return cudaErrorInvalidValue;
    const int nk = (a.I + LN_BK - 1) / LN_BK;
    a.kchunks = (nk + splits - 1) / splits;
    splits = (nk + a.kchunks - 1) / a.kchunks;
    if (splits == 1) { a.part = nullptr; a.tile_cnt = nullptr; }
    a.cluster = splits > 1 && splits <= LIN_MAX_CLUSTER;
    if (splits > 1 && !a.cluster && (!a.part || !a.tile_cnt)) return cudaErrorInvalidValue;
    LinWeights lw;
    memset(&lw, 0, sizeof(lw));
    int tiles = 0;
    size_t off = 0;
    for (int i = 0; i < nw; ++i) {
        lw.w[i] = *tmW[i];
        tiles += (O[i] + LN_BM - 1) / LN_BM;
        lw.tile_end[i] = tiles; lw.O[i] = O[i]; lw.y[i] = y[i]; lw.part_off[i] = off;
        off += (size_t)splits * a.S * O[i];
    }
    lw.nw = nw;
    static bool attr_set[16] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 16 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(linear_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             LinSmem<16>::TOTAL);
        if (e != cudaSuccess) return e;
        if (dev < 16) attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, 1, splits); cfg.blockDim = dim3(192);
    cfg.dynamicSmemBytes = LinSmem<16>::TOTAL; cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr; cfg.numAttrs = 1;
    if (a.cluster) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 1; attr[1].val.clusterDim.y = 1; attr[1].val.clusterDim.z = splits;
        cfg.numAttrs = 2;
    }
    return cudaLaunchKernelEx(&cfg, linear_kernel<16>, lw, tmX, a);
}

}  // namespace coli

namespace coli {
// ---------------------------------------------------------------- norm / residual tail
// Zero-centred RMSNorm of one row (c/qwen.c:326-330: x * rsqrt(mean x^2 + eps)
// * (1 + w)), one CTA of 256 threads per row; with `delta` the row is first
// resid + delta (the residual add of the route tail), written to `sum_out`.
// The normed row goes out in fp32 (optional) and bf16 (the next projection's
// input).
__global__ void __launch_bounds__(256)
rmsnorm_zc_rows_kernel(const float *x, const float *delta, const float *w, float *sum_out, float *nrm_out,
                       __nv_bfloat16 *nrm_bf16, int D, float eps)
{
    const size_t row = blockIdx.x;
    const float *xr = x + row * D;
    const float *dr = delta ? delta + row * D : nullptr;
    __shared__ float red[8];
    float ss = 0.f;
    for (int i = threadIdx.x; i < D; i += 256) {
        float v = xr[i];
        if (dr) {
            v += dr[i];
            sum_out[row * D + i] = v;
        }
        ss += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    const float r = 1.f / sqrtf(tot / D + eps);
    for (int i = threadIdx.x; i < D; i += 256) {
        const float v = dr ? sum_out[row * D + i] : xr[i];
        const float o = v * r * (1.f + w[i]);
        if (nrm_out) nrm_out[row * D + i] = o;
        if (nrm_bf16) nrm_bf16[row * D + i] = __float2bfloat16_rn(o);
    }
}

cudaError_t launch_rmsnorm_zc_rows(const float *x, const float *delta, const float *w, float *sum_out,
                                   float *nrm_out, __nv_bfloat16 *nrm_bf16, int S, int D, float eps,
                                   cudaStream_t st)
{
    rmsnorm_zc_rows_kernel<<<S, 256, 0, st>>>(x, delta, w, sum_out, nrm_out, nrm_bf16, D, eps);
    return cudaGetLastError();
}
}  // namespace coli
