/*
 * CPU oracle for the qwen3.c token-mixing hot path — TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C and fp32 with the same operation order, the
 * reference engine's CPU arithmetic for the two token mixers:
 *   - gated GQA attention (qwen.c `attention()`, c/qwen.c:581-666) minus the
 *     dense projections: per-head zero-centred q/k RMSNorm, partial NeoX RoPE,
 *     KV append, causal softmax attention and the sigmoid output gate;
 *   - GatedDeltaNet (qwen.c `gdn_step()`, c/qwen.c:669-776) minus the dense
 *     projections: conv4 ring + SiLU, q/k L2-norm, decay/beta gates, the
 *     delta-rule recurrence and the gated RMSNorm.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs load
 * it, as the checker or as the timed CPU baseline. The CUDA backend never
 * links or calls it.
 *
 * Parity of this restatement with the reference itself is pinned by
 * tests/test_oracle_golden.py against fixtures produced by the reference's own
 * functions (oracle/ref_harness.c compiles c/qwen.c unmodified).
 *
 * Dims are runtime parameters (as in the reference's Cfg), so the oracle runs
 * any head geometry. Requests are processed one after another, because the
 * reference engine is single-sequence (one KV cache, one GDN state set).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* c/qwen.c:172-175 */
static inline float orc_sigmoid(float x) { return 1.f / (1.f + expf(-x)); }
static inline float orc_silu(float x) { return x / (1.f + expf(-x)); }
static inline float orc_softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }

/* Zero-centred RMSNorm, c/qwen.c:326-330: x * rsqrt(mean(x^2)+eps) * (1+w),
 * with the sum of squares in double. In-place safe. */
static void orc_rmsnorm_zc(float *out, const float *x, const float *w, int n, float eps)
{
    double acc = 0;
    for (int i = 0; i < n; i++) acc += (double)x[i] * x[i];
    float r = 1.f / sqrtf((float)(acc / n) + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * r * (1.f + w[i]);
}

/* Half-split (NeoX) rotation of dims j and j+rot/2 for j < rot/2,
 * c/qwen.c:570-579. Dims >= rot are untouched. */
static void orc_rope_partial(float *x, int pos, int rot, float theta)
{
    int half = rot / 2;
    for (int j = 0; j < half; j++) {
        float inv = powf(theta, -2.0f * j / rot);
        float ang = (float)pos * inv;
        float cs = cosf(ang), sn = sinf(ang);
        float a = x[j], b = x[j + half];
        x[j] = a * cs - b * sn;
        x[j + half] = b * cs + a * sn;
    }
}

/* Max-subtracted softmax, c/qwen.c:332-336. */
static void orc_softmax(float *x, int n)
{
    float mx = -1e30f;
    for (int i = 0; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

/*
 * GQA prologue for S new tokens at positions pos_base..pos_base+S-1
 * (c/qwen.c:598-611): q heads of qg [S][H][2*hd] (q | gate per head) are
 * normed and roped in place; k heads [S][KH][hd] are normed + roped and, with
 * the raw v, written to the cache rows Kc/Vc [KH][max_t][hd].
 */
void orc_gqa_prologue(float *qg, float *k, const float *v, const float *qnw, const float *knw,
                      int S, int H, int KH, int hd, int rot, float theta, float eps,
                      int pos_base, float *Kc, float *Vc, int max_t)
{
    for (int s = 0; s < S; s++) {
        int pos = pos_base + s;
        for (int h = 0; h < H; h++) {
            float *qh = qg + ((int64_t)s * H + h) * 2 * hd;
            orc_rmsnorm_zc(qh, qh, qnw, hd, eps);
            orc_rope_partial(qh, pos, rot, theta);
        }
        for (int h = 0; h < KH; h++) {
            float *kh = k + ((int64_t)s * KH + h) * hd;
            orc_rmsnorm_zc(kh, kh, knw, hd, eps);
            orc_rope_partial(kh, pos, rot, theta);
            memcpy(Kc + ((int64_t)h * max_t + pos) * hd, kh, hd * sizeof(float));
            memcpy(Vc + ((int64_t)h * max_t + pos) * hd, v + ((int64_t)s * KH + h) * hd,
                   hd * sizeof(float));
        }
    }
}

/*
 * Causal attention core with the sigmoid output gate (c/qwen.c:617-663).
 * qg [S][H][2*hd] holds roped q | gate; query row s sits at position
 * pos_base+s and sees cache rows 0..pos_base+s. ctx [S][H][hd].
 * Q head h reads KV head h / (H/KH). scale = 1/sqrt(hd) in the reference.
 */
void orc_gqa_attend(const float *qg, const float *Kc, const float *Vc, float *ctx,
                    int S, int H, int KH, int hd, int max_t, int pos_base, float scale)
{
    int grp = H / KH;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < H; h++) {
        for (int s = 0; s < S; s++) {
            int qpos = pos_base + s, kh = h / grp;
            float *sc = malloc((size_t)(qpos + 1) * sizeof(float));
            const float *qv = qg + ((int64_t)s * H + h) * 2 * hd;
            for (int t = 0; t <= qpos; t++) {
                const float *kr = Kc + ((int64_t)kh * max_t + t) * hd;
                float acc = 0;
                for (int d = 0; d < hd; d++) acc += qv[d] * kr[d];
                sc[t] = acc * scale;
            }
            orc_softmax(sc, qpos + 1);
            float *cx = ctx + ((int64_t)s * H + h) * hd;
            for (int d = 0; d < hd; d++) cx[d] = 0;
            for (int t = 0; t <= qpos; t++) {
                const float *vr = Vc + ((int64_t)kh * max_t + t) * hd;
                float p = sc[t];
                for (int d = 0; d < hd; d++) cx[d] += p * vr[d];
            }
            const float *gate = qv + hd;
            for (int d = 0; d < hd; d++) cx[d] *= orc_sigmoid(gate[d]);
            free(sc);
        }
    }
}

/*
 * One GatedDeltaNet token for one request, from the post-projection inputs
 * (c/qwen.c:697-773):
 *   qkv [CD] pre-conv (q | k | v channel order), z [VH*VD], a, b [VH];
 *   conv_w [CD][K], A_log, dt_bias [VH], gnorm [VD];
 *   ring [K][CD] (slot K-1 newest) and state [VH][KD][VD] updated in place;
 *   y [VH*VD] = gated-RMSNorm output (the out_proj input).
 * CD = 2*KH*KD + VH*VD.
 */
void orc_gdn_step(const float *qkv, const float *z, const float *a, const float *b,
                  const float *conv_w, const float *A_log, const float *dt_bias,
                  const float *gnorm, float *ring, float *state, float *y,
                  int KH, int KD, int VH, int VD, int K, float eps)
{
    int key_dim = KH * KD, CD = 2 * key_dim + VH * VD;
    float *cv = malloc((size_t)CD * sizeof(float));
    /* ring shift + append + depthwise conv + SiLU (c/qwen.c:697-707) */
    memmove(ring, ring + CD, (size_t)(K - 1) * CD * sizeof(float));
    memcpy(ring + (size_t)(K - 1) * CD, qkv, (size_t)CD * sizeof(float));
    for (int ch = 0; ch < CD; ch++) {
        const float *w = conv_w + (int64_t)ch * K;
        float acc = 0;
        for (int j = 0; j < K; j++) acc += w[j] * ring[(size_t)j * CD + ch];
        cv[ch] = orc_silu(acc);
    }
    /* per K head L2 norm with eps on the sum; q also scaled by 1/sqrt(KD)
     * (c/qwen.c:712-720) */
    float *qn = malloc((size_t)key_dim * sizeof(float)), *kn = malloc((size_t)key_dim * sizeof(float));
    for (int h = 0; h < KH; h++) {
        const float *qs = cv + h * KD, *ks = cv + key_dim + h * KD;
        float sq = 0, sk = 0;
        for (int d = 0; d < KD; d++) { sq += qs[d] * qs[d]; sk += ks[d] * ks[d]; }
        float rq = 1.f / sqrtf(sq + eps) / sqrtf((float)KD), rk = 1.f / sqrtf(sk + eps);
        for (int d = 0; d < KD; d++) { qn[h * KD + d] = qs[d] * rq; kn[h * KD + d] = ks[d] * rk; }
    }
    /* gates (c/qwen.c:722-727) then the recurrence (c/qwen.c:748-773) */
    int grp = VH / KH;
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < VH; h++) {
        float beta = orc_sigmoid(b[h]);
        float decay = expf(-expf(A_log[h]) * orc_softplus(a[h] + dt_bias[h]));
        int src = h / grp;
        const float *qh = qn + src * KD, *kh = kn + src * KD, *vh = cv + 2 * key_dim + h * VD;
        float *Sh = state + (size_t)h * KD * VD;
        float *mem = calloc((size_t)VD, sizeof(float));
        float *dl = malloc((size_t)VD * sizeof(float));
        for (int kd = 0; kd < KD; kd++) {
            float *row = Sh + (size_t)kd * VD;
            float kk = kh[kd];
            for (int vd = 0; vd < VD; vd++) { row[vd] *= decay; mem[vd] += row[vd] * kk; }
        }
        for (int vd = 0; vd < VD; vd++) dl[vd] = (vh[vd] - mem[vd]) * beta;
        float *yh = y + (size_t)h * VD;
        for (int vd = 0; vd < VD; vd++) yh[vd] = 0;
        for (int kd = 0; kd < KD; kd++) {
            float *row = Sh + (size_t)kd * VD;
            float kk = kh[kd], qq = qh[kd];
            for (int vd = 0; vd < VD; vd++) { row[vd] += kk * dl[vd]; yh[vd] += row[vd] * qq; }
        }
        const float *zh = z + (size_t)h * VD;
        double ms = 0;
        for (int vd = 0; vd < VD; vd++) ms += (double)yh[vd] * yh[vd];
        float r = 1.f / sqrtf((float)(ms / VD) + eps);
        for (int vd = 0; vd < VD; vd++) yh[vd] = yh[vd] * r * gnorm[vd] * orc_silu(zh[vd]);
        free(mem); free(dl);
    }
    free(cv); free(qn); free(kn);
}

/*
 * The recurrence + gated RMSNorm alone, on pre-normalised inputs
 * (c/qwen.c:748-773; the contract of the reference's coli_vk_gdn):
 * qn/kn [KH*KD], v/z [VH*VD], decay/beta [VH], gnorm [VD] -> y [VH*VD].
 */
void orc_gdn_recur(const float *qn, const float *kn, const float *v, const float *z,
                   const float *decay, const float *beta, const float *gnorm, float *state,
                   float *y, int KH, int KD, int VH, int VD, float eps)
{
    int grp = VH / KH;
    for (int h = 0; h < VH; h++) {
        int src = h / grp;
        const float *qh = qn + src * KD, *kh = kn + src * KD, *vh = v + h * VD;
        float *Sh = state + (size_t)h * KD * VD;
        float *mem = calloc((size_t)VD, sizeof(float));
        float *dl = malloc((size_t)VD * sizeof(float));
        for (int kd = 0; kd < KD; kd++) {
            float *row = Sh + (size_t)kd * VD;
            float kk = kh[kd];
            for (int vd = 0; vd < VD; vd++) { row[vd] *= decay[h]; mem[vd] += row[vd] * kk; }
        }
        for (int vd = 0; vd < VD; vd++) dl[vd] = (vh[vd] - mem[vd]) * beta[h];
        float *yh = y + (size_t)h * VD;
        for (int vd = 0; vd < VD; vd++) yh[vd] = 0;
        for (int kd = 0; kd < KD; kd++) {
            float *row = Sh + (size_t)kd * VD;
            float kk = kh[kd], qq = qh[kd];
            for (int vd = 0; vd < VD; vd++) { row[vd] += kk * dl[vd]; yh[vd] += row[vd] * qq; }
        }
        const float *zh = z + (size_t)h * VD;
        double ms = 0;
        for (int vd = 0; vd < VD; vd++) ms += (double)yh[vd] * yh[vd];
        float r = 1.f / sqrtf((float)(ms / VD) + eps);
        for (int vd = 0; vd < VD; vd++) yh[vd] = yh[vd] * r * gnorm[vd] * orc_silu(zh[vd]);
        free(mem); free(dl);
    }
}

/*
 * S GatedDeltaNet tokens in sequence for one request: the reference prefill
 * is exactly S gdn_step calls (c/qwen.c:1378-1379). Row strides: qkv CD,
 * z VH*VD, a/b VH, y VH*VD.
 */
void orc_gdn_seq(const float *qkv, const float *z, const float *a, const float *b,
                 const float *conv_w, const float *A_log, const float *dt_bias,
                 const float *gnorm, float *ring, float *state, float *y,
                 int S, int KH, int KD, int VH, int VD, int K, float eps)
{
    int CD = 2 * KH * KD + VH * VD, VDim = VH * VD;
    for (int s = 0; s < S; s++)
        orc_gdn_step(qkv + (int64_t)s * CD, z + (int64_t)s * VDim, a + (int64_t)s * VH,
                     b + (int64_t)s * VH, conv_w, A_log, dt_bias, gnorm, ring, state,
                     y + (int64_t)s * VDim, KH, KD, VH, VD, K, eps);
}

/* Threads the OpenMP loops may use (1 when built without -fopenmp). */
int orc_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
