/*
 * Harness around the UNMODIFIED reference engine — TEST INFRASTRUCTURE ONLY.
 *
 * This translation unit includes the reference's c/qwen.c as-is (found on the
 * include path given by oracle/Makefile; nothing is copied into this
 * repository) with its `main` renamed, and exports C entry points that drive
 * the reference's own static functions on caller-provided weights and state:
 *   ref_attention -> attention()  c/qwen.c:581-666 (gated GQA block)
 *   ref_gdn_step  -> gdn_step()   c/qwen.c:669-776 (GatedDeltaNet block)
 *   ref_matmul    -> matmul()     c/qwen.c:177-189 (the projections)
 * The build writes oracle/_ref/libqwenref.so. tests/golden/make_golden.py uses
 * it to generate the committed golden fixtures that pin oracle/oracle.c, and
 * bench.py --impl reference times it as the reference CPU baseline.
 */
/* qwen.c needs struct rusage; the stock Linux build lacks this include. */
#define _GNU_SOURCE
#include <sys/resource.h>
#define main qwen_ref_main
#include "qwen.c"
#undef main
#ifdef _OPENMP
#include <omp.h>
#endif

static void ref_fill_cfg(Cfg *c, int hidden)
{
    memset(c, 0, sizeof(*c));
    c->hidden = hidden;
    c->n_layers = 1;
}

/*
 * One gated GQA block call: out[S][hidden] = attention(x[S][hidden]) with
 * W_q [H*2*hd][hidden], W_k/W_v [KH*hd][hidden], W_o [hidden][H*hd],
 * qn/kn [hd]. Kc/Vc [KH][max_t][hd] are the caller's fp32 cache (rows
 * < pos_base must already hold roped k / raw v); new rows are written.
 */
void ref_attention(const float *x, float *out, int S, int pos_base, int hidden,
                   int H, int KH, int hd, float partial_rotary, float theta, float eps,
                   float *Wq, float *Wk, float *Wv, float *Wo, float *qn, float *kn,
                   float *Kc, float *Vc, int max_t)
{
    Model m;
    Layer l;
    memset(&m, 0, sizeof(m));
    memset(&l, 0, sizeof(l));
    ref_fill_cfg(&m.c, hidden);
    m.c.n_heads = H;
    m.c.n_kv_heads = KH;
    m.c.head_dim = hd;
    m.c.rot = (int)(hd * partial_rotary); /* c/qwen.c:358-359 */
    m.c.theta = theta;
    m.c.eps = eps;
    float *Kp[1] = {Kc}, *Vp[1] = {Vc};
    m.K = Kp;
    m.V = Vp;
    m.max_t = max_t;
    l.q = Wq; l.k = Wk; l.v = Wv; l.o = Wo; l.qn = qn; l.kn = kn;
    attention(&m, &l, 0, x, S, pos_base, out);
}

/*
 * S GatedDeltaNet tokens through gdn_step(): x [S][hidden] -> out
 * [S][hidden]. Weights: Wqkv [CD][hidden], Wz [VH*VD][hidden],
 * Wa/Wb [VH][hidden], conv [CD][K], A_log/dt_bias [VH], gnorm [VD],
 * Wout [hidden][VH*VD]. state [VH][KD][VD] and ring [K][CD] update in place.
 */
void ref_gdn_steps(const float *x, float *out, int S, int hidden,
                   int KH, int KD, int VH, int VD, int K, float eps,
                   float *Wqkv, float *Wz, float *Wa, float *Wb, float *conv,
                   float *A_log, float *dt_bias, float *gnorm, float *Wout,
                   float *state, float *ring)
{
    Model m;
    Layer l;
    memset(&m, 0, sizeof(m));
    memset(&l, 0, sizeof(l));
    ref_fill_cfg(&m.c, hidden);
    m.c.eps = eps;
    m.c.gdn_kh = KH; m.c.gdn_kd = KD; m.c.gdn_vh = VH; m.c.gdn_vd = VD; m.c.conv_k = K;
    m.c.key_dim = KH * KD;                    /* c/qwen.c:367-369 */
    m.c.value_dim = VH * VD;
    m.c.conv_dim = 2 * m.c.key_dim + m.c.value_dim;
    float *Sp[1] = {state}, *Rp[1] = {ring};
    m.gdnS = Sp;
    m.convst = Rp;
    l.qkv = Wqkv; l.z = Wz; l.a = Wa; l.b = Wb; l.conv = conv;
    l.alog = A_log; l.dtb = dt_bias; l.gnorm = gnorm; l.outp = Wout;
    for (int s = 0; s < S; s++)
        gdn_step(&m, &l, 0, x + (int64_t)s * hidden, out + (int64_t)s * hidden);
}

/* y[S][O] = x[S][I] . W[O][I]^T with the reference's own loop. */
void ref_matmul(float *y, const float *x, const float *W, int S, int I, int O)
{
    matmul(y, x, W, S, I, O);
}

int ref_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
