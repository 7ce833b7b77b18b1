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
// written once). One CTA of 256 threads owns the whole 128x128 fp32 state of
// one (request, V head): lane l of every warp owns columns 4l..4l+3 and warp w
// rows w, w+8, .., so each state load / store of a warp is one contiguous
// 512-byte row, and all 16 float4 loads per thread are issued before the
// prologue. Reductions over rows (S^T k, S^T q) go through shared memory;
// the gated RMSNorm statistic is local to the CTA. The two V heads of a K
// head form a cluster of 2 CTAs: both read the old q/k conv history, one
// relaxed cluster barrier orders those reads before rank 0 shifts it (each
// CTA shifts its own v channels). Compared with the earlier 8-CTA cluster
// per (request, K head) over 32-column slices, a CTA moves 4x the state per
// fixed cost (input loads, conv, norms, barrier) and needs no distributed
// shared memory.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace coli {

constexpr int GDN_KD = 128, GDN_VD = 128, GDN_THREADS = 256, GDN_ROWS = 16;   // rows per thread

template <typename TI, typename TO, bool PRENORM>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GDN_THREADS, 2)
gdn_decode_kernel(GdnDecodeArgs p)
{
    const int rank = blockIdx.x & 1;
    const int cid = blockIdx.x >> 1;
    const int KH = p.KH, VH = p.VH;
    const int b = cid / KH, kh = cid - b * KH;
    const int vh = kh * 2 + rank;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int key_dim = KH * GDN_KD, CD = 2 * key_dim + VH * GDN_VD;

    __shared__ __align__(16) float qs[GDN_KD], ks[GDN_KD], vs[GDN_VD], zs[GDN_VD];
    __shared__ __align__(16) float red[8][GDN_VD];
    __shared__ float nrm[8];
    __shared__ double ssd[4];

    // ---- issue the state loads first: rows warp + 8 i, columns 4 lane ..
    float *Sbase = p.state + ((size_t)b * VH + vh) * GDN_KD * GDN_VD + 4 * lane;
    float4 S[GDN_ROWS];
#pragma unroll
    for (int i = 0; i < GDN_ROWS; ++i)
        S[i] = __ldcs(reinterpret_cast<const float4 *>(Sbase + (size_t)(warp + 8 * i) * GDN_VD));

    float decay, beta;
    if constexpr (!PRENORM) {
        // ---- conv4 + SiLU: thread t = q channel t (t < 128) or k channel t - 128,
        // and for t < 128 also v channel t of this V head
        const TI *x = static_cast<const TI *>(p.qkv) + (size_t)b * CD;
        float *hist = p.hist + (size_t)b * 3 * CD;
        const int c = t < GDN_KD ? kh * GDN_KD + t : key_dim + kh * GDN_KD + (t - GDN_KD);
        const float h0 = hist[c], h1 = hist[CD + c], h2 = hist[2 * CD + c], xc = to_f32(x[c]);
        const float4 w = *reinterpret_cast<const float4 *>(p.conv_w + (size_t)c * 4);
        float a = 0.f;
        a += w.x * h0; a += w.y * h1; a += w.z * h2; a += w.w * xc;
        const float qk = siluf_(a);
        float vh1 = 0.f, vh2 = 0.f, vxv = 0.f;
        const int cv = 2 * key_dim + vh * GDN_VD + t;
        if (t < GDN_VD) {
            const float g0 = hist[cv], g1 = hist[CD + cv], g2 = hist[2 * CD + cv];
            const float xv = to_f32(x[cv]);
            const float4 wv = *reinterpret_cast<const float4 *>(p.conv_w + (size_t)cv * 4);
            float av = 0.f;
            av += wv.x * g0; av += wv.y * g1; av += wv.z * g2; av += wv.w * xv;
            vs[t] = siluf_(av);
            vh1 = g1; vh2 = g2; vxv = xv;
            zs[t] = siluf_(to_f32(static_cast<const TI *>(p.z)[(size_t)b * VH * GDN_VD + vh * GDN_VD + t]));
        }
        // ---- L2 norms over the 128 q (warps 0-3) and 128 k (warps 4-7) channels
        float sq = qk * qk;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) nrm[warp] = sq;
        if (p.pdecay) {
            beta = p.pbeta[(size_t)b * VH + vh];
            decay = p.pdecay[(size_t)b * VH + vh];
        } else {
            const float av = to_f32(static_cast<const TI *>(p.a)[(size_t)b * VH + vh]);
            const float bv = to_f32(static_cast<const TI *>(p.b)[(size_t)b * VH + vh]);
            beta = sigmoidf_(bv);
            decay = expf(-expf(p.A_log[vh]) * softplusf_(av + p.dt_bias[vh]));
        }
        __syncthreads();
        if (t < GDN_KD) {
            const float s2 = (nrm[0] + nrm[1]) + (nrm[2] + nrm[3]);
            qs[t] = qk * (1.f / sqrtf(s2 + p.eps) / sqrtf((float)GDN_KD));
        } else {
            const float s2 = (nrm[4] + nrm[5]) + (nrm[6] + nrm[7]);
            ks[t - GDN_KD] = qk * (1.f / sqrtf(s2 + p.eps));
        }
        // Both CTAs of the cluster have read the old q/k history: rank 0 may
        // now shift it. The stores come after the barrier, so the arrive does
        // not wait on them.
        cluster_arrive_relaxed();
        cluster_wait();
        if (t < GDN_VD) { hist[cv] = vh1; hist[CD + cv] = vh2; hist[2 * CD + cv] = vxv; }
        if (rank == 0) { hist[c] = h1; hist[CD + c] = h2; hist[2 * CD + c] = xc; }
    } else {
        // Pre-normalised inputs (the reference's coli_vk_gdn contract).
        const TI *in = static_cast<const TI *>(p.qkv) + (size_t)b * p.in_stride;
        if (t < GDN_KD) qs[t] = to_f32(in[kh * GDN_KD + t]);
        else ks[t - GDN_KD] = to_f32(in[key_dim + kh * GDN_KD + (t - GDN_KD)]);
        if (t < GDN_VD) {
            vs[t] = to_f32(in[2 * key_dim + vh * GDN_VD + t]);
            zs[t] = siluf_(to_f32(static_cast<const TI *>(p.z)[(size_t)b * VH * GDN_VD + vh * GDN_VD + t]));
        }
        decay = p.decay[(size_t)b * VH + vh];
        beta = p.beta[(size_t)b * VH + vh];
        cluster_arrive_relaxed();   // the cluster barrier every CTA takes part in
        cluster_wait();
    }
    __syncthreads();

    // ---- S *= decay; m = S^T k (this thread's 16 rows, 4 columns)
    float4 mp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < GDN_ROWS; ++i) {
        const float kk = ks[warp + 8 * i];
        S[i].x *= decay; S[i].y *= decay; S[i].z *= decay; S[i].w *= decay;
        mp.x += S[i].x * kk; mp.y += S[i].y * kk; mp.z += S[i].z * kk; mp.w += S[i].w * kk;
    }
    *reinterpret_cast<float4 *>(&red[warp][4 * lane]) = mp;
    __syncthreads();
    float4 dl = *reinterpret_cast<const float4 *>(&vs[4 * lane]);
    {
        float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const float4 r = *reinterpret_cast<const float4 *>(&red[w][4 * lane]);
            m.x += r.x; m.y += r.y; m.z += r.z; m.w += r.w;
        }
        dl.x = (dl.x - m.x) * beta; dl.y = (dl.y - m.y) * beta;
        dl.z = (dl.z - m.z) * beta; dl.w = (dl.w - m.w) * beta;
    }
    // ---- S += k delta^T; y = S^T q; the state goes back as soon as it is final
    float4 yp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < GDN_ROWS; ++i) {
        const int r = warp + 8 * i;
        const float kk = ks[r], qq = qs[r];
        S[i].x += kk * dl.x; S[i].y += kk * dl.y; S[i].z += kk * dl.z; S[i].w += kk * dl.w;
        yp.x += S[i].x * qq; yp.y += S[i].y * qq; yp.z += S[i].z * qq; yp.w += S[i].w * qq;
        __stcs(reinterpret_cast<float4 *>(Sbase + (size_t)r * GDN_VD), S[i]);
    }
    __syncthreads();  // every thread has read red[] (m); reuse it for y
    *reinterpret_cast<float4 *>(&red[warp][4 * lane]) = yp;
    __syncthreads();
    // ---- gated RMSNorm over the V head's 128 columns (thread t < 128 = column t),
    // mean square in double as the reference (c/qwen.c:768-772)
    float yv = 0.f;
    if (t < GDN_VD) {
#pragma unroll
        for (int w = 0; w < 8; ++w) yv += red[w][t];
        double s2 = (double)yv * yv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        if (lane == 0) ssd[warp] = s2;
    }
    __syncthreads();
    if (t < GDN_VD) {
        const double tot = (ssd[0] + ssd[1]) + (ssd[2] + ssd[3]);
        const float r = 1.f / sqrtf((float)(tot / GDN_VD) + p.eps);
        const float out = yv * r * p.gnorm[t] * zs[t];
        static_cast<TO *>(p.y)[(size_t)b * VH * GDN_VD + vh * GDN_VD + t] = from_f32<TO>(out);
    }
}

template <typename TI, typename TO, bool PRENORM>
static cudaError_t launch_gdn_decode_t(const GdnDecodeArgs &a, cudaStream_t st)
{
    dim3 grid(a.B * a.KH * 2), block(GDN_THREADS);
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
