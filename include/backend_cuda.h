/*
 * backend_cuda.h — B200 (sm_100a) CUDA backend for the qwen3.c token mixers.
 *
 * Plays the role c/backend_vulkan.h plays for c/qwen.c, for the token-mixing
 * hot path only: the gated GQA full-attention layers and the GatedDeltaNet
 * linear-attention layers, decode and prefill. Each declaration names the
 * reference interface it replaces (file:line in the reference project).
 *
 * Conventions (as in the reference backend):
 *   - Every int-returning call returns 1 on success and 0 on failure; the
 *     reason is in coli_cuda_last_error(). There is NO CPU fallback inside the
 *     backend: a 0 is the caller's signal, exactly like a coli_vk_* 0
 *     (c/qwen.c:592, 635, 691, 745). A device-side failure marks the backend
 *     not ready and every later call returns 0 (c/backend_vulkan.c:1836).
 *   - Host-pointer entry points take fp32 row-major arrays the caller owns and
 *     copy them in and out per call (synchronous). *_dev entry points take
 *     device pointers, run asynchronously on the backend stream and never
 *     copy; their `dtype` is 0 for fp32 or 1 for bf16 activations.
 *   - State is device-resident and keyed by a per-type layer index (`layer`
 *     counts full-attention layers for KV, GDN layers for GDN state, like the
 *     reference's kvi / gi), plus a request index `req` for batched decode.
 *     KV cache: bf16 [batch][KH][max_t][hd]. GDN state: fp32
 *     [batch][VH][KD][VD] (the reference's [VH][KD][VD] per request). Conv
 *     history: fp32 [batch][conv_k-1][conv_dim] (the reference ring's slots
 *     1..conv_k-1; slot 0 is dead state, always overwritten before use).
 *   - Single host thread; calls are not reentrant (c/backend_vulkan.c:1838).
 *   - Shapes: hd = 256 with H/KH = 8 for GQA; KD = VD = 128, VH = 2*KH and
 *     conv_k = 4 for GDN (the Qwen3.5/3.6-MoE token mixers). Other shapes
 *     return 0 with an error.
 */
#ifndef COLI_BACKEND_CUDA_H
#define COLI_BACKEND_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- lifecycle: replaces coli_vk_init / coli_vk_shutdown / coli_vk_available
 * (c/backend_vulkan.h:37-39) and coli_vk_mem_info (:40). */
int  coli_cuda_init(int device);
void coli_cuda_shutdown(void);
int  coli_cuda_available(void);
void coli_cuda_mem_info(size_t *used_bytes, size_t *tensor_count);
/* New: the reason for the last 0 return (never NULL). */
const char *coli_cuda_last_error(void);
/* New: the time limit of every device-side wait (mbarrier waits in the
 * kernels, the cross-rank barrier) in nanoseconds; 0 restores the default
 * 2 s. On time-out a kernel raises the device error word and returns, the
 * next synchronising call returns 0 with "pipeline wait timed out" and the
 * backend is marked not ready (c/backend_vulkan.c:1836: a lost device), until
 * coli_cuda_init is called again. */
int  coli_cuda_set_wait_limit(unsigned long long ns);
/* New, a failure-injection hook for tests: after n more successful device
 * allocations the next one is refused as if cudaMalloc had failed (the call
 * that needed it returns 0; the backend stays usable). n < 0 disables. */
void coli_cuda_debug_fail_alloc(int n);
/* New: wait for queued *_dev work and check the device error word. */
int  coli_cuda_sync(void);
/* New: the cudaStream_t the backend launches on; set it to run inside a
 * caller's stream (or a CUDA graph capture). NULL restores the default. */
void *coli_cuda_get_stream(void);
int  coli_cuda_set_stream(void *stream);

/* ---- New: per-kernel device timing (CUDA events recorded on the launching
 * stream around every launch of the named kernel while enabled) and a count
 * of every kernel this library launched. Replaces the reference's wall-clock
 * and Vulkan timestamp profiling (c/qwen.c:163, c/backend_vulkan.c:1130-1213).
 * Kernel ids: 0 GQA split-KV decode, 1 GDN decode, 2 GQA prefill,
 * 3 GDN chunked prefill, 4 GQA combine. ktimer_read synchronises, sums the
 * recorded intervals and clears them. */
enum { COLI_K_GQA_SPLIT = 0, COLI_K_GDN_DECODE = 1, COLI_K_GQA_PREFILL = 2,
       COLI_K_GDN_PREFILL = 3, COLI_K_GQA_COMBINE = 4, COLI_K_COUNT = 5 };
int  coli_cuda_ktimer_enable(int on);
int  coli_cuda_ktimer_read(int kernel, double *total_ms, int *launches);
long long coli_cuda_launch_count(void);

/* ---- capability probes: coli_vk_gdn_available (c/backend_vulkan.h:151),
 * coli_vk_gqa_available (:162), coli_vk_gqa_full_available (:173),
 * coli_vk_gdn_full_available (:265). */
int  coli_cuda_gdn_available(void);
int  coli_cuda_gqa_available(void);
int  coli_cuda_gqa_full_available(void);
int  coli_cuda_gdn_full_available(void);

/* ---- KV cache: coli_vk_kv_ensure / coli_vk_kv_row / coli_vk_kv_reset
 * (c/backend_vulkan.h:114-116, impl c/backend_vulkan.c:1705-1743) with a
 * request dimension. `row` = kh*max_t + pos, as in the reference. Host rows
 * are fp32 and stored as bf16. kv_ensure zero-fills a new cache; calling it
 * again with the same geometry keeps the contents. kv_reset drops all layers.
 * A one-request cache may be declared as rows, KH = 1 and max_t = KH*max_t
 * (all coli_vk_kv_ensure knows); the first attention call naming (KH, max_t)
 * with the same row count adopts that split, rows keep their addresses. */
int  coli_cuda_kv_ensure(int layer, int batch, int KH, int max_t, int hd);
int  coli_cuda_kv_row(int layer, int req, int row, const float *k, const float *v);
/* New: n consecutive rows starting at row0 (bulk upload / read-back). */
int  coli_cuda_kv_rows(int layer, int req, int row0, int n, const float *k, const float *v);
int  coli_cuda_kv_read(int layer, int req, int row0, int n, float *k, float *v);
void coli_cuda_kv_reset(void);
/* New: n rows from device memory (dtype 0 fp32 / 1 bf16), e.g. rows an
 * engine-side prefill produced on the GPU. Asynchronous on the backend stream. */
int  coli_cuda_kv_rows_dev(int layer, int req, int row0, int n, const void *k, const void *v,
                           int dtype);
/* New: device base pointers of a layer's bf16 K and V caches. */
int  coli_cuda_kv_device_ptr(int layer, void **k, void **v);
/* Resident q_norm / k_norm weights [hd] of a full layer:
 * coli_vk_gqa_norm_weight (c/backend_vulkan.h:172). */
int  coli_cuda_gqa_norm_weight(int layer, const float *qnw, const float *knw, int hd);

/* ---- GQA attention core: coli_vk_gqa (c/backend_vulkan.h:163-164,
 * c/backend_vulkan.c:2167-2199). q [S][H][2*hd] holds roped q | gate per
 * head; query row s sees cache rows 0..T-S+s of request 0; ctx [S][H][hd]
 * = softmax(q k^T * scale) v * sigmoid(gate). st0 must be 0 (the only value
 * the engine passes, c/qwen.c:623, 629). */
int  coli_cuda_gqa(int layer, const float *q, float *ctx, int S, int H, int KH, int hd,
                   int max_t, int st0, int T, float scale);

/* ---- GQA block minus projections for S tokens of one request at
 * pos_base..pos_base+S-1: the body of attention() between the projections
 * and o_proj (c/qwen.c:598-663): q/k zero-centred RMSNorm with the resident
 * norm weights, partial RoPE (rot dims, theta), K/V append, causal attention
 * with scale 1/sqrt(hd), sigmoid output gate. qg [S][H][2*hd] raw q|gate,
 * k/v [S][KH][hd] raw, ctx [S][H][hd]. The device part of
 * coli_vk_gqa_full (c/backend_vulkan.h:174-177). */
int  coli_cuda_gqa_step(int layer, int req, int S, int pos_base, const float *qg, const float *k,
                        const float *v, float *ctx, int H, int KH, int hd, int rot, float eps,
                        float theta);
int  coli_cuda_gqa_step_dev(int layer, int req, int S, int pos_base, const void *qg, const void *k,
                            const void *v, void *ctx, int H, int KH, int hd, int rot, float eps,
                            float theta, int dtype);

/* ---- New (no reference counterpart: the reference is single-device):
 * head-sharded causal prefill for one rank of a multi-GPU prefill. Computes
 * query heads [h0, h0+nh) of inputs laid out with all H / KH heads (qg
 * [S][H][2*hd], k/v [S][KH][hd]); the layer's cache holds only the KV heads
 * those query heads read (h0/8 .. (h0+nh-1)/8), and ctx is [S][nh][hd]. The
 * per-rank ctx blocks are then all-gathered by the caller. S >= 64. */
int  coli_cuda_gqa_prefill_heads_dev(int layer, int req, int S, int pos_base, const void *qg,
                                     const void *k, const void *v, void *ctx, int H, int KH,
                                     int hd, int rot, float eps, float theta, int dtype, int h0,
                                     int nh);

/* ---- New: batched GQA decode, one new token for each request b < B at its
 * own position pos[b] (requests 0..B-1 of the layer's cache). Same per-row
 * semantics as coli_cuda_gqa_step with S = 1. The _dev form takes pos on the
 * device (int32 [B]). The host form returns when ctx is written; inside, the
 * gate halves of qg travel on a second, backend-owned copy stream while the
 * attention runs (pinned host buffers make all its copies asynchronous). */
int  coli_cuda_gqa_decode(int layer, int B, const float *qg, const float *k, const float *v,
                          const int *pos, float *ctx, int H, int KH, int hd, int rot, float eps,
                          float theta);
int  coli_cuda_gqa_decode_dev(int layer, int B, const void *qg, const void *k, const void *v,
                              const int *pos_dev, void *ctx, int H, int KH, int hd, int rot,
                              float eps, float theta, int dtype);

/* ---- No counterpart in the reference. Batched GQA decode that allocates no
 * device memory, for callers that cannot call cudaMalloc while serving (a
 * memory budget fixed at start-up, or no allocation allowed once decoding
 * runs). Same arguments and results as coli_cuda_gqa_decode_dev (device
 * pointers, pos on the device, dtype 0 fp32 / 1 bf16). Its intermediates live
 * in one fixed 8 MiB device array inside the library, which every GPU that
 * loads the library holds until exit; a call whose batch does not fit returns
 * 0 with the limit in the error message (about 340 requests). The first call
 * on a device looks up that array's device address, so make it before any
 * stream capture. All calls share the array: calls that overlap on the GPU
 * race. */
int  coli_cuda_gqa_decode_noalloc(int layer, int B, const void *qg, const void *k, const void *v,
                                  const int *pos_dev, void *ctx, int H, int KH, int hd, int rot,
                                  float eps, float theta, int dtype);

/* ---- GatedDeltaNet state: coli_vk_gdn_state_ensure / coli_vk_gdn_reset
 * (c/backend_vulkan.h:152-153), coli_vk_gdn_conv_ensure / _weight (:266-267),
 * coli_vk_gdn_ba_weight (:206) for the per-layer A_log, dt_bias, gnorm.
 * gdn_reset zeroes every state and conv history in place. */
int  coli_cuda_gdn_state_ensure(int layer, int batch, int VH, int KD, int VD);
int  coli_cuda_gdn_conv_ensure(int layer, int batch, int conv_k, int conv_dim);
int  coli_cuda_gdn_conv_weight(int layer, const float *cw, int conv_k, int conv_dim);
int  coli_cuda_gdn_params(int layer, const float *A_log, const float *dt_bias, const float *gnorm,
                          int VH, int VD);
void coli_cuda_gdn_reset(void);
/* New (state parity / checkpoint): one request's state [VH][KD][VD] and conv
 * ring [conv_k][conv_dim] in the reference's layout (slot conv_k-1 newest;
 * get writes zeros to the dead slot 0, set ignores it). */
int  coli_cuda_gdn_state_get(int layer, int req, float *state);
int  coli_cuda_gdn_state_set(int layer, int req, const float *state);
int  coli_cuda_gdn_conv_get(int layer, int req, float *ring);
int  coli_cuda_gdn_conv_set(int layer, int req, const float *ring);

/* ---- GDN recurrence on pre-normalised inputs: coli_vk_gdn
 * (c/backend_vulkan.h:154-156). Request 0; qn/kn [KH*KD] (q already scaled
 * by 1/sqrt(KD)), v/z [VH*VD], decay/beta [VH], gnorm [VD] -> y [VH*VD]. */
int  coli_cuda_gdn(int layer, const float *qn, const float *kn, const float *v, const float *z,
                   const float *decay, const float *beta, const float *gnorm, float *y,
                   int KH, int KD, int VH, int VD, float eps);

/* ---- GDN decode, fused conv4 + SiLU + L2 norm + gates + recurrence + gated
 * RMSNorm, one token for each request b < B: gdn_step() after the
 * projections (c/qwen.c:697-773); the device part of coli_vk_gdn_full
 * (c/backend_vulkan.h:268-270). qkv [B][conv_dim] pre-conv (q|k|v),
 * z [B][VH*VD], a/b [B][VH] -> y [B][VH*VD] (the out_proj input). */
int  coli_cuda_gdn_decode(int layer, int B, const float *qkv, const float *z, const float *a,
                          const float *b, float *y, int KH, int KD, int VH, int VD, float eps);
int  coli_cuda_gdn_decode_dev(int layer, int B, const void *qkv, const void *z, const void *a,
                              const void *b, void *y, int KH, int KD, int VH, int VD, float eps,
                              int dtype);

/* ---- GDN prefill of S tokens of one request, carrying the conv history and
 * state in and out: the reference's S sequential gdn_step calls
 * (c/qwen.c:1376-1380) and the device part of coli_vk_gdn_full_seq
 * (c/backend_vulkan.h:274-278). Row layouts as in coli_cuda_gdn_decode. */
int  coli_cuda_gdn_prefill(int layer, int req, int S, const float *qkv, const float *z,
                           const float *a, const float *b, float *y, int KH, int KD, int VH, int VD,
                           float eps);
int  coli_cuda_gdn_prefill_dev(int layer, int req, int S, const void *qkv, const void *z,
                               const void *a, const void *b, void *y, int KH, int KD, int VH,
                               int VD, float eps, int dtype);

/* ---- New (no reference counterpart): head-sharded GDN prefill for one rank.
 * Owns K heads [kh0, kh0+nkh) and their V heads [2*kh0, 2*kh0+2*nkh) of
 * inputs laid out with all KH / VH heads; the layer's state holds only the
 * owned V heads (state_ensure with VH = 2*nkh), its conv history is the full
 * width (only owned channels are read and advanced) and its params are the
 * full VH arrays. y is [S][2*nkh*VD]. S >= 64. */
int  coli_cuda_gdn_prefill_heads_dev(int layer, int req, int S, const void *qkv, const void *z,
                                     const void *a, const void *b, void *y, int KH, int KD,
                                     int VH, int VD, float eps, int dtype, int kh0, int nkh);

/* ---- New: head-sharded prefill with the all-gather fused into the output
 * kernels (no reference counterpart: the reference runs on one device). The
 * caller's per-layer NCCL all-gather of the rank outputs (rank-major
 * [world][S][cols], cols = nh*hd or 2*nkh*VD) is replaced by the kernels'
 * epilogues storing this rank's block into every rank's gathered buffer
 * through peer pointers (NVLink); dst[r] is rank r's buffer as mapped in
 * this process (dst[rank] is the local one), world <= 8, bf16 only.
 * A layer ends with coli_cuda_peer_barrier on every rank before any rank
 * reads the gathered output.
 *   coli_cuda_ipc_alloc   cudaMalloc + zero + IPC handle (64 bytes) of a buffer
 *   coli_cuda_ipc_open    map a peer's buffer from its handle (_close unmaps)
 *   coli_cuda_peer_barrier  flags[r] = rank r's [world] uint32 flag array
 *                         (IPC mapped); epoch increases by one per call; a
 *                         wait longer than ~2 s sets the device error word. */
int  coli_cuda_ipc_alloc(size_t bytes, void **dptr, void *handle);
int  coli_cuda_ipc_free(void *dptr, size_t bytes);
int  coli_cuda_ipc_open(const void *handle, void **dptr);
int  coli_cuda_ipc_close(void *dptr);
int  coli_cuda_peer_barrier(void *const *flags, int world, int rank, unsigned epoch);
int  coli_cuda_gqa_prefill_heads_gather_dev(int layer, int req, int S, int pos_base, const void *qg,
                                            const void *k, const void *v, void *const *dst,
                                            int world, int rank, int H, int KH, int hd, int rot,
                                            float eps, float theta, int dtype, int h0, int nh);
int  coli_cuda_gdn_prefill_heads_gather_dev(int layer, int req, int S, const void *qkv,
                                            const void *z, const void *a, const void *b,
                                            void *const *dst, int world, int rank, int KH, int KD,
                                            int VH, int VD, float eps, int dtype, int kh0, int nkh);

/* ==== Block level: projections + mixer + out-projection ====
 * Resident dense weights, W [O][I] row-major as the engine stores it, held on
 * the device in bf16. Replaces coli_vk_tensor_ensure / _free / _bytes
 * (c/backend_vulkan.h:105, 143-144): fmt 0 = f32 weights, fmt 1 = int8 with
 * one scale per output row (dequantised to bf16 on upload); other formats
 * return 0 (caller keeps its own path). An existing handle of the same shape
 * is kept as is. I must be a multiple of 8. */
typedef struct ColiCudaTensor ColiCudaTensor;
int    coli_cuda_tensor_ensure(ColiCudaTensor **tensor, const void *weights, const float *scales,
                               int fmt, int I, int O, int grp);
void   coli_cuda_tensor_free(ColiCudaTensor *t);
size_t coli_cuda_tensor_bytes(const ColiCudaTensor *t);

/* y[S][O] = x[S][I] W^T (c/qwen.c:178-189 matmul; coli_vk_matmul,
 * c/backend_vulkan.h:56): uploads the tensor on first use. */
int  coli_cuda_matmul(ColiCudaTensor **tensor, float *y, const float *x, const void *w,
                      const float *scales, int fmt, int S, int I, int O, int gs);

/* Device-pointer form: x bf16 [S][I] (16-byte aligned), y [S][O] fp32
 * (y_bf16 = 0) or bf16 (1), asynchronous on the backend stream. */
int  coli_cuda_matmul_dev(const ColiCudaTensor *tensor, const void *x, int S, void *y, int y_bf16);

/* Up to 4 projections of the same x in one launch when S <= 16 (the output
 * tiles of all weights share the grid and the split-K plan; a decode step's
 * q|gate / k / v, or qkv / z / a / b, as the block calls issue them); larger
 * S runs them one by one. Same argument rules as coli_cuda_matmul_dev; the
 * weights need the same input width. */
int  coli_cuda_matmul_multi_dev(const ColiCudaTensor *const *tensors, int n, const void *x, int S,
                                void *const *y, int y_bf16);

/* Attention + resident o_proj in one call, ctx staying on the device:
 * coli_vk_gqa_project (c/backend_vulkan.h:165-170; called at c/qwen.c:623).
 * Same q / cache contract as coli_cuda_gqa; out [S][Dout] fp32 host. */
int  coli_cuda_gqa_project(int layer, const float *q, ColiCudaTensor *ot, float *out, int S, int H,
                           int KH, int hd, int max_t, int st0, int T, float scale, int Dout);
/* Delta rule + gated RMSNorm + resident out_proj in one call, y staying on
 * the device: coli_vk_gdn_project (c/backend_vulkan.h:256-260; called at
 * c/qwen.c:734). Same inputs as coli_cuda_gdn; out [Dout] fp32 host. */
int  coli_cuda_gdn_project(int layer, const float *qn, const float *kn, const float *v,
                           const float *z, const float *decay, const float *beta,
                           const float *gnorm, ColiCudaTensor *ot, float *out, int KH, int KD,
                           int VH, int VD, float eps, int Dout);

/* Whole gated-GQA block for S rows of request 0 (coli_vk_gqa_full,
 * c/backend_vulkan.h:173-177; CPU c/qwen.c:595-665): q|gate, k, v
 * projections -> q/k norm + RoPE + KV append -> causal attention -> gate ->
 * o_proj. Needs coli_cuda_kv_ensure + coli_cuda_gqa_norm_weight. x [S][D],
 * out [S][Dout] fp32 host. */
int  coli_cuda_gqa_full(int layer, const float *x, int D, ColiCudaTensor *gq_t,
                        ColiCudaTensor *gk_t, ColiCudaTensor *gv_t, ColiCudaTensor *out_t,
                        float *out, int S, int H, int KH, int hd, int rot, int pos_base,
                        int max_t, float eps, float theta, int Dout);

/* Whole GatedDeltaNet block for one token of request 0 (coli_vk_gdn_full,
 * c/backend_vulkan.h:266-272; CPU c/qwen.c:697-773): in_proj_qkv / in_proj_z
 * -> conv4 (+ history) -> q/k norm -> delta rule -> gated RMSNorm ->
 * out_proj. params = [decay(VH) | beta(VH) | gnorm(VD)] as the engine packs
 * them (c/qwen.c:681-686). Needs coli_cuda_gdn_state_ensure,
 * coli_cuda_gdn_conv_ensure and coli_cuda_gdn_conv_weight. */
int  coli_cuda_gdn_full(int layer, const float *x, int D, ColiCudaTensor *gqkv_t,
                        ColiCudaTensor *gz_t, const float *params, ColiCudaTensor *out_t,
                        float *out, int KH, int KD, int VH, int VD, int conv_dim, int conv_k,
                        float eps, int Dout);
/* S tokens of the same block (coli_vk_gdn_full_seq, c/backend_vulkan.h:276-281):
 * params [S][2*VH+VD], out [S][Dout]; S >= 64 runs the chunk-parallel prefill,
 * shorter runs step token by token. */
int  coli_cuda_gdn_full_seq(int layer, const float *x, int S, int D, ColiCudaTensor *gqkv_t,
                            ColiCudaTensor *gz_t, const float *params, ColiCudaTensor *out_t,
                            float *out, int KH, int KD, int VH, int VD, int conv_dim,
                            int conv_k, float eps, int Dout);
/* The same block with the tiny a / b projections on the device as well
 * (c/qwen.c:709-711; the engine keeps them on the host and passes params,
 * c/qwen.c:681-686): ga_t / gb_t are in_proj_a / in_proj_b [VH][D], run in
 * one launch with in_proj_qkv / in_proj_z (S <= 16), and the gates come from
 * the layer's A_log / dt_bias / gnorm (coli_cuda_gdn_params; c/qwen.c:722-727).
 * S >= 64 runs the chunk-parallel prefill. No counterpart in the Vulkan ABI. */
int  coli_cuda_gdn_full_ab(int layer, const float *x, int S, int D, ColiCudaTensor *gqkv_t,
                           ColiCudaTensor *gz_t, ColiCudaTensor *ga_t, ColiCudaTensor *gb_t,
                           ColiCudaTensor *out_t, float *out, int KH, int KD, int VH, int VD,
                           int conv_dim, int conv_k, float eps, int Dout);

/* Route tail (the fused residual + post_ln + router epilogue):
 * coli_vk_layer_norm_weight / coli_vk_moe_route_available /
 * coli_vk_gqa_full_route / coli_vk_gdn_full_route (c/backend_vulkan.h:180-198).
 * layer_norm_weight uploads one model layer's in_ln and post_ln (D floats each).
 * gqa_full_route: x = rmsnorm_zc(resid, in_ln) on the device, the GQA block,
 * then resid_out = resid + delta, nrm_out = rmsnorm_zc(resid_out, post_ln)
 * (c/qwen.c:326-330) and pr_out = nrm_out router^T [S][E]; gdn_full_route
 * takes x_in already normed (the caller computes b/a from it) for one token.
 * Dout must equal D. */
int  coli_cuda_moe_route_available(void);
int  coli_cuda_layer_norm_weight(int layer, const float *in_ln, const float *post_ln, int D);
int  coli_cuda_gqa_full_route(int layer, const float *resid, int D,
                              ColiCudaTensor *gq_t, ColiCudaTensor *gk_t, ColiCudaTensor *gv_t,
                              ColiCudaTensor *out_t, ColiCudaTensor *router, int ln_layer,
                              float *resid_out, float *nrm_out, float *pr_out,
                              int S, int H, int KH, int hd, int rot, int pos_base, int max_t,
                              float eps, float theta, int Dout, int E);
int  coli_cuda_gdn_full_route(int layer, const float *x_in, const float *resid, int D,
                              ColiCudaTensor *gqkv_t, ColiCudaTensor *gz_t, const float *params,
                              ColiCudaTensor *out_t, ColiCudaTensor *router, int ln_layer,
                              float *resid_out, float *nrm_out, float *pr_out,
                              int KH, int KD, int VH, int VD, int conv_dim, int conv_k,
                              float eps, int Dout, int E);

/* ==== Snapshot loader (safetensors) ====
 * The reference's shard index (c/st.h:248-479) and the mixer part of
 * model_init (c/qwen.c:433-485): st_open indexes every *.safetensors file of
 * a snapshot directory (name order) and returns a handle (-1 on a missing or
 * malformed file; offsets, shapes and byte spans are checked before any
 * read). st_info gives shape / ndim / dtype (0 BF16, 1 F16, 2 F32, 3 I8/U8)
 * of a named tensor; st_read_f32 converts a float tensor into out (at most
 * cap elements; returns the element count, -1 on error); st_dense uploads a
 * 2-D [O][I] weight as a resident dense tensor (BF16 sources exactly). The
 * st_open / st_info / st_read_f32 / st_close calls need no device. */
int       coli_cuda_st_open(const char *snap_dir);
void      coli_cuda_st_close(int handle);
int       coli_cuda_st_info(int handle, const char *name, long long *shape, int *ndim, int *dtype);
long long coli_cuda_st_read_f32(int handle, const char *name, float *out, long long cap);
int       coli_cuda_st_dense(int handle, const char *name, ColiCudaTensor **tensor);

#ifdef __cplusplus
}
#endif

#endif /* COLI_BACKEND_CUDA_H */
