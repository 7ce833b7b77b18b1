// Launch interfaces between the host backend (backend.cu) and the kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace coli {

// ---------------------------------------------------------------- GDN decode
struct GdnDecodeArgs {
    const void *qkv;      // [B][CD] pre-conv (fused) or [B][in_stride] = qn|kn|v (prenorm)
    const void *z;        // [B][VH*VD]
    const void *a, *b;    // [B][VH] (fused)
    const float *decay, *beta;  // [B][VH] (prenorm)
    const float *pdecay, *pbeta;  // [B][VH] given decay / beta (fused; nullptr = from a, b)
    const float *conv_w;  // [CD][4]
    const float *A_log, *dt_bias, *gnorm;
    float *hist;          // [B][3][CD] conv history (fused)
    float *state;         // [B][VH][KD][VD]
    void *y;              // [B][VH*VD]
    int B, KH, KD, VH, VD, in_stride;
    float eps;
};
cudaError_t launch_gdn_decode(const GdnDecodeArgs &a, int in_bf16, int out_bf16, int prenorm,
                              cudaStream_t st);

// ---------------------------------------------------------------- GQA decode
// Output of a head-sharded prefill written straight into every rank's
// gathered buffer (rank-major [world][rows][cols], the all-gather layout)
// through peer (NVLink) pointers, so the transfer overlaps the kernel instead
// of following it. dst[r] is rank r's buffer as mapped in this process.
constexpr int PEER_MAX = 8;
struct PeerGather {
    void *dst[PEER_MAX];
    int world, rank;      // world 0 = write the local output as usual
    long long block;      // elements of one rank's block (rows x cols)
};

struct GqaPrologueArgs {
    const void *qg;       // [nq][H][2*hd] raw q | gate
    const void *k, *v;    // [nq][KH][hd] raw
    const float *qnw, *knw;
    const int *pos;       // [nq] position of each query row (sees rows 0..pos)
    const int *creq;      // [nq] cache request of each query row (nullptr = identity)
    __nv_bfloat16 *qout;  // [nq][H][hd] normed + roped q
    __nv_bfloat16 *kcache, *vcache;  // [reqs][KH][max_t][hd]
    int nq, H, KH, max_t, rot;
    float eps, theta;
    // head-sharded prefill: this call computes query heads [h0, h0+H) and KV
    // heads [kh0, kh0+KH) of inputs laid out with Hin / KHin heads (0 = H / KH)
    int h0, kh0, Hin, KHin;
};
struct GqaSplitArgs {
    const __nv_bfloat16 *q;  // [nq][H][hd] roped
    const int *pos, *creq;
    float *part_o;           // [nq][KH][n_splits][8][hd]
    float *part_ml;          // [nq][KH][n_splits][8][2]
    int nq, H, KH, max_t, n_splits, chunk;
    int appended;            // rows pos-appended+1 .. pos of each query row may be written by the
                             // kernel just before (the prologue): loaded only after the grid dependency
    float scale_log2;
    // Small-batch decode (no cache request map, one appended row per query
    // row): fuse = 1 (bf16 inputs) or 2 (fp32) makes the split kernel do the
    // prologue's work itself from `pro` -- each CTA norms and ropes the q of
    // its 8 heads, and the CTA whose key range holds position pos appends
    // that row -- and q above is unused; 0 = q from gqa_prologue_warp_kernel.
    int fuse;
    GqaPrologueArgs pro;
};
struct GqaCombineArgs {
    const float *part_o, *part_ml;
    const void *qg;          // gate source [nq][H][2*hd]
    void *ctx;               // [nq][H][hd]
    int nq, H, KH, n_splits;
};
cudaError_t launch_gqa_prologue(const GqaPrologueArgs &a, int in_bf16, cudaStream_t st);
cudaError_t launch_gqa_split(const CUtensorMap &tk, const CUtensorMap &tv, const GqaSplitArgs &a,
                             cudaStream_t st);
cudaError_t launch_gqa_combine(const GqaCombineArgs &a, int in_bf16, int out_bf16, cudaStream_t st);
size_t gqa_split_smem_bytes();
int gqa_pick_splits(int nq, int KH, int tmax, int num_sms);
int gqa_chunk_for(int tmax, int n_splits);

}  // namespace coli

namespace coli {
// ---------------------------------------------------------------- GQA prefill
struct GqaPrefillArgs {
    const void *qg;   // [S][H][2*hd] raw q | gate (gate read in the epilogue)
    void *ctx;        // [S][H][hd]
    int S, H, KH, max_t, req, pos_base, n_qtiles;
    float scale_log2;
    int h0, kh0, Hin;  // head-sharded prefill (see GqaPrologueArgs); 0 = unsharded
    PeerGather gather; // world > 0: ctx goes to every rank's gathered buffer instead
    int tma_epi;       // 1: gate tile loaded and ctx tile stored by TMA (bf16, no gather)
};
// Tensor maps of the TMA epilogue: the gate half of qg ([S][Hin][2 hd], boxes
// of 64 x 1 x 128 at x = hd + 64 c) and ctx ([S][H][hd], same boxes).
struct PfEpiMaps {
    CUtensorMap gate, ctx;
};
cudaError_t launch_gqa_prefill(const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv,
                               const GqaPrefillArgs &a, int in_bf16, int out_bf16, cudaStream_t st,
                               const PfEpiMaps *em = nullptr);
}  // namespace coli

namespace coli {
// ---------------------------------------------------------------- GDN prefill
struct GdnPrefillArgs {
    PeerGather gather;                    // world > 0: y goes to every rank's gathered buffer instead
    const void *qkv, *z, *a, *b;          // [S][CD], [S][VH*VD], [S][VH], [S][VH]
    const float *conv_w, *A_log, *dt_bias, *gnorm;
    float *hist;                          // [3][CD] of the request (read, then rewritten)
    float *state;                         // [VH][KD][VD] of the request (in/out)
    void *y;                              // [S][VH*VD]
    float *Qh, *Kh;                       // scratch [KH][S][128]
    float *KT;                            // scratch [KH][nchunks][128][64] (K^T per chunk)
    float *VT;                            // scratch [VH][nchunks][128][64] (V^T per chunk, tf32)
    float *GL, *BETA;                     // scratch [VH][S]
    float *W, *U;                         // scratch [nchunks][VH][64][128]
    float *M;                             // scratch [nchunks][VH][64][64]
    float *Dt;                            // scratch [nchunks][VH][128][64] (D transposed)
    float *QH;                            // scratch [nchunks][VH][128][64] (diag(gamma) Q S0, transposed)
    float *Hs;                            // scratch [nseg][VH][128][128] segment start states
    float *XS;                            // scratch [nseg-1][VH][128][256] segment maps [Phi | Psi]
    int nseg, seglen;                     // chunk segments walked in parallel (1 = one walk)
    const float *params;                  // [S][pstride] = decay | beta (per input V head) | ..., or nullptr (from a, b)
    int pstride;
    int S, KH, VH;
    float eps;
    // head-sharded prefill: this call owns K heads [kh0, kh0+KH) (V heads
    // [2*kh0, 2*kh0+2*KH)) of inputs laid out with KHin / VHin heads (0 = KH / VH);
    // state, y and scratch hold only the owned heads
    int kh0, KHin, VHin;
};
struct GdnPrefillMaps {
    CUtensorMap Q, K, V, W, U, M, Dt, KT;
};
cudaError_t launch_gdn_prefill(const GdnPrefillArgs &a, const GdnPrefillMaps &m, int bf16,
                               cudaStream_t st);
}  // namespace coli

namespace coli {
// ---------------------------------------------------------------- dense projections
struct LinearArgs {
    void *y;              // [S][O] fp32 or bf16 (y_bf16)
    float *part;          // split-K partials [splits][S][O] (nullptr = no split)
    int S, I, O;
    int kchunks;          // 64-element K chunks per split (set by launch_linear)
    int y_bf16;
    int *tile_cnt;        // split-K arrival counters, one per output tile, zero between
                          // launches (nullptr = a separate reduce kernel adds the splits)
    int cluster;          // set by the launchers: the K splits of a tile form one thread-block
                          // cluster and are added through distributed shared memory
};
cudaError_t launch_linear(const CUtensorMap &tmW, const CUtensorMap &tmX, LinearArgs a, int bn, int splits,
                          cudaStream_t st, int *launches = nullptr);
// Up to LIN_MAXW projections of the same x ([S][I], S <= 16) in one launch:
// weight w has O[w] outputs into y[w]; the output tiles of all weights share
// the grid (and the split-K plan, with the reduction in the kernel).
constexpr int LIN_MAXW = 4;
cudaError_t launch_linear_multi(const CUtensorMap *const *tmW, const int *O, void *const *y, int nw,
                                const CUtensorMap &tmX, LinearArgs a, int splits, cudaStream_t st);
cudaError_t launch_f32_to_bf16(const float *x, __nv_bfloat16 *y, size_t n, cudaStream_t st);
int linear_pick_bn(int S);
cudaError_t launch_rmsnorm_zc_rows(const float *x, const float *delta, const float *w, float *sum_out,
                                   float *nrm_out, __nv_bfloat16 *nrm_bf16, int S, int D, float eps,
                                   cudaStream_t st);
}  // namespace coli
