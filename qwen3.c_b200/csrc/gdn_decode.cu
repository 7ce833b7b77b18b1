// GatedDeltaNet decode step: one token per request, fused end to end.
//
// Follows the reference's gdn_step() arithmetic after the projections
// (c/qwen.c:697-773): conv4 ring + SiLU, per-K-head L2 norm (eps on the sum,
// q scaled by 1/sqrt(KD)), beta = sigmoid(b), decay = exp(-exp(A_log) *
// softplus(a + dt_bias)), then per V head on the 128x128 fp32 state:
//   S *= decay;  m = S^T k;  delta = (v - m) * beta;  S += k delta^T;
//   y = S^T q;   y = y * rsqrt(mean(y^2) + eps) * gnorm * silu(z).
//
// Work decomposition (bandwidth bound: the 64 KiB state per V head is read and
// written once). A thread-block cluster of 8 CTAs serves one (request, K head):
// 2 V heads x 4 column blocks of 32 state columns. Each CTA streams its
// 128x32 fp32 state slice through registers (8 float4 per thread, issued
// before the prologue so the loads overlap it). The cluster barrier orders the
// q/k conv-history reads of all 8 CTAs before the one CTA that owns those
// channels shifts the history, and the per-row RMSNorm statistic of a V head
// is exchanged through distributed shared memory.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace coli {

constexpr int GDN_KD = 128, GDN_VD = 128, GDN_CB = 32, GDN_THREADS = 128;

template <typename TI, typename TO, bool PRENORM>
__global__ void __cluster_dims__(8, 1, 1) __launch_bounds__(GDN_THREADS)
gdn_decode_kernel(GdnDecodeArgs p)
{
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = blockIdx.x & 7;
    const int cid = blockIdx.x >> 3;
    const int KH = p.KH, VH = p.VH;
    const int b = cid / KH, kh = cid - b * KH;
    const int vh = kh * 2 + (rank >> 2), cblk = rank & 3;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int key_dim = KH * GDN_KD, CD = 2 * key_dim + VH * GDN_VD;

    __shared__ __align__(16) float qs[GDN_KD], ks[GDN_KD], vs[GDN_CB], zs[GDN_CB];
    __shared__ __align__(16) float red[4][GDN_CB];
    __shared__ float nrm[2][4];
    __shared__ double ss_sh;

    // ---- issue the state loads first (128 rows x 32 cols, 8 float4 / thread)
    float *Sbase = p.state + ((size_t)b * VH + vh) * GDN_KD * GDN_VD + cblk * GDN_CB;
    const int c4 = lane & 7, rs = lane >> 3;
    float4 S[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = warp * 4 + rs + 16 * i;
        S[i] = __ldcs(reinterpret_cast<const float4 *>(Sbase + (size_t)r * GDN_VD + 4 * c4));
    }

    float decay, beta;
    if constexpr (!PRENORM) {
        // ---- conv4 + SiLU for this K head's q and k channels (thread t = channel t)
        const TI *x = static_cast<const TI *>(p.qkv) + (size_t)b * CD;
        float *hist = p.hist + (size_t)b * 3 * CD;
        const int cq = kh * GDN_KD + t, ck = key_dim + kh * GDN_KD + t;
        float hq0 = hist[cq], hq1 = hist[CD + cq], hq2 = hist[2 * CD + cq], xq = to_f32(x[cq]);
        float hk0 = hist[ck], hk1 = hist[CD + ck], hk2 = hist[2 * CD + ck], xk = to_f32(x[ck]);
        const float4 wq = *reinterpret_cast<const float4 *>(p.conv_w + (size_t)cq * 4);
        const float4 wk = *reinterpret_cast<const float4 *>(p.conv_w + (size_t)ck * 4);
        float aq = 0.f, ak = 0.f;
        aq += wq.x * hq0; aq += wq.y * hq1; aq += wq.z * hq2; aq += wq.w * xq;
        ak += wk.x * hk0; ak += wk.y * hk1; ak += wk.z * hk2; ak += wk.w * xk;
        const float qc = siluf_(aq), kc = siluf_(ak);
        // ---- v channels of this CTA's 32 columns; this CTA owns their history
        float vh1 = 0.f, vh2 = 0.f, vxv = 0.f;
        if (t < GDN_CB) {
            const int cv = 2 * key_dim + vh * GDN_VD + cblk * GDN_CB + t;
            const float h0 = hist[cv], h1 = hist[CD + cv], h2 = hist[2 * CD + cv];
            const float xv = to_f32(x[cv]);
            const float4 wv = *reinterpret_cast<const float4 *>(p.conv_w + (size_t)cv * 4);
            float av = 0.f;
            av += wv.x * h0; av += wv.y * h1; av += wv.z * h2; av += wv.w * xv;
            vs[t] = siluf_(av);
            vh1 = h1; vh2 = h2; vxv = xv;
            zs[t] = siluf_(to_f32(static_cast<const TI *>(p.z)[(size_t)b * VH * GDN_VD + vh * GDN_VD + cblk * GDN_CB + t]));
        }
        // ---- L2 norms over the 128 channels of the K head
        float sq = qc * qc, sk = kc * kc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
            sk += __shfl_xor_sync(0xffffffffu, sk, o);
        }
        if (lane == 0) { nrm[0][warp] = sq; nrm[1][warp] = sk; }
        __syncthreads();
        sq = (nrm[0][0] + nrm[0][1]) + (nrm[0][2] + nrm[0][3]);
        sk = (nrm[1][0] + nrm[1][1]) + (nrm[1][2] + nrm[1][3]);
        const float rq = 1.f / sqrtf(sq + p.eps) / sqrtf((float)GDN_KD);
        const float rk = 1.f / sqrtf(sk + p.eps);
        qs[t] = qc * rq;
        ks[t] = kc * rk;
        if (p.pdecay) {
            beta = p.pbeta[(size_t)b * VH + vh];
            decay = p.pdecay[(size_t)b * VH + vh];
        } else {
            const float av = to_f32(static_cast<const TI *>(p.a)[(size_t)b * VH + vh]);
            const float bv = to_f32(static_cast<const TI *>(p.b)[(size_t)b * VH + vh]);
            beta = sigmoidf_(bv);
            decay = expf(-expf(p.A_log[vh]) * softplusf_(av + p.dt_bias[vh]));
        }
        // All CTAs of the cluster have read (and used) the old q/k history:
        // the owner (rank 0) may now shift it. The history stores are issued
        // only after this barrier, so the arrive does not wait on them.
        cluster_arrive_relaxed();
        cluster_wait();
        if (t < GDN_CB) {
            const int cv = 2 * key_dim + vh * GDN_VD + cblk * GDN_CB + t;
            hist[cv] = vh1; hist[CD + cv] = vh2; hist[2 * CD + cv] = vxv;
        }
        if (rank == 0) {
            hist[cq] = hq1; hist[CD + cq] = hq2; hist[2 * CD + cq] = xq;
            hist[ck] = hk1; hist[CD + ck] = hk2; hist[2 * CD + ck] = xk;
        }
    } else {
        // Pre-normalised inputs (the reference's coli_vk_gdn contract).
        qs[t] = to_f32(static_cast<const TI *>(p.qkv)[(size_t)b * p.in_stride + kh * GDN_KD + t]);
        ks[t] = to_f32(static_cast<const TI *>(p.qkv)[(size_t)b * p.in_stride + key_dim + kh * GDN_KD + t]);
        if (t < GDN_CB) {
            vs[t] = to_f32(static_cast<const TI *>(p.qkv)[(size_t)b * p.in_stride + 2 * key_dim + vh * GDN_VD +
                                 cblk * GDN_CB + t]);
            zs[t] = siluf_(to_f32(static_cast<const TI *>(p.z)[(size_t)b * VH * GDN_VD + vh * GDN_VD + cblk * GDN_CB + t]));
        }
        decay = p.decay[(size_t)b * VH + vh];
        beta = p.beta[(size_t)b * VH + vh];
    }
    __syncthreads();

    // ---- S *= decay; m = S^T k
    float4 mp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float kk = ks[warp * 4 + rs + 16 * i];
        S[i].x *= decay; S[i].y *= decay; S[i].z *= decay; S[i].w *= decay;
        mp.x += S[i].x * kk; mp.y += S[i].y * kk; mp.z += S[i].z * kk; mp.w += S[i].w * kk;
    }
#pragma unroll
    for (int o = 8; o <= 16; o <<= 1) {
        mp.x += __shfl_xor_sync(0xffffffffu, mp.x, o);
        mp.y += __shfl_xor_sync(0xffffffffu, mp.y, o);
        mp.z += __shfl_xor_sync(0xffffffffu, mp.z, o);
        mp.w += __shfl_xor_sync(0xffffffffu, mp.w, o);
    }
    if (rs == 0) *reinterpret_cast<float4 *>(&red[warp][4 * c4]) = mp;
    __syncthreads();
    float4 dl;
    {
        const float4 r0 = *reinterpret_cast<const float4 *>(&red[0][4 * c4]);
        const float4 r1 = *reinterpret_cast<const float4 *>(&red[1][4 * c4]);
        const float4 r2 = *reinterpret_cast<const float4 *>(&red[2][4 * c4]);
        const float4 r3 = *reinterpret_cast<const float4 *>(&red[3][4 * c4]);
        const float4 v4 = *reinterpret_cast<const float4 *>(&vs[4 * c4]);
        dl.x = (v4.x - ((r0.x + r1.x) + (r2.x + r3.x))) * beta;
        dl.y = (v4.y - ((r0.y + r1.y) + (r2.y + r3.y))) * beta;
        dl.z = (v4.z - ((r0.z + r1.z) + (r2.z + r3.z))) * beta;
        dl.w = (v4.w - ((r0.w + r1.w) + (r2.w + r3.w))) * beta;
    }
    // ---- S += k delta^T; y = S^T q; write the state back
    float4 yp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = warp * 4 + rs + 16 * i;
        const float kk = ks[r], qq = qs[r];
        S[i].x += kk * dl.x; S[i].y += kk * dl.y; S[i].z += kk * dl.z; S[i].w += kk * dl.w;
        yp.x += S[i].x * qq; yp.y += S[i].y * qq; yp.z += S[i].z * qq; yp.w += S[i].w * qq;
    }
#pragma unroll
    for (int o = 8; o <= 16; o <<= 1) {
        yp.x += __shfl_xor_sync(0xffffffffu, yp.x, o);
        yp.y += __shfl_xor_sync(0xffffffffu, yp.y, o);
        yp.z += __shfl_xor_sync(0xffffffffu, yp.z, o);
        yp.w += __shfl_xor_sync(0xffffffffu, yp.w, o);
    }
    __syncthreads();  // everyone has consumed red[] (m); reuse it for y
    if (rs == 0) *reinterpret_cast<float4 *>(&red[warp][4 * c4]) = yp;
    __syncthreads();
    float yv = 0.f;
    if (t < GDN_CB) {
        yv = (red[0][t] + red[1][t]) + (red[2][t] + red[3][t]);
        double s2 = (double)yv * yv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        if (t == 0) ss_sh = s2;
    }
    // ---- gated RMSNorm over the V head's 128 columns (4 CTAs of the cluster).
    // Publish the statistic, then stream the state back while peers arrive.
    cluster_arrive_release();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = warp * 4 + rs + 16 * i;
        __stcs(reinterpret_cast<float4 *>(Sbase + (size_t)r * GDN_VD + 4 * c4), S[i]);
    }
    cluster_wait();
    if (t < GDN_CB) {
        const int first = rank & 4;
        double tot = 0.0;
#pragma unroll
        for (int j = 0; j < 4; ++j) tot += *cluster.map_shared_rank(&ss_sh, first + j);
        const float r = 1.f / sqrtf((float)(tot / GDN_VD) + p.eps);
        const int col = cblk * GDN_CB + t;
        const float out = yv * r * p.gnorm[col] * zs[t];
        static_cast<TO *>(p.y)[(size_t)b * VH * GDN_VD + vh * GDN_VD + col] = from_f32<TO>(out);
    }
    // keep shared memory alive until every peer has read (and used) it
    cluster_arrive_relaxed();
    cluster_wait();
}

template <typename TI, typename TO, bool PRENORM>
static cudaError_t launch_gdn_decode_t(const GdnDecodeArgs &a, cudaStream_t st)
{
    dim3 grid(a.B * a.KH * 8), block(GDN_THREADS);
    gdn_decode_kernel<TI, TO, PRENORM><<<grid, block, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_gdn_decode(const GdnDecodeArgs &a, int in_bf16, int out_bf16, int prenorm,
                              cudaStream_t st)
{
    if (a.KD != GDN_KD || a.VD != GDN_VD || a.VH != 2 * a.KH || a.B <= 0) return cudaErrorInvalidValue;
    if (prenorm) {
        if (in_bf16 || out_bf16) return cudaErrorInvalidValue;
        return launch_gdn_decode_t<float, float, true>(a, st);
    }
    if (in_bf16 && out_bf16) return launch_gdn_decode_t<__nv_bfloat16, __nv_bfloat16, false>(a, st);
    if (!in_bf16 && !out_bf16) return launch_gdn_decode_t<float, float, false>(a, st);
    return cudaErrorInvalidValue;
}

}  // namespace coli
