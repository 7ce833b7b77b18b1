// Block-level entry points: the mixer with its projections, the role of
// coli_vk_gqa_full / coli_vk_gdn_full / coli_vk_gdn_full_seq
// (c/backend_vulkan.h:173-185, 266-283) and of the resident dense tensors
// they take (coli_vk_tensor_ensure, c/backend_vulkan.h:105). Included at the
// end of backend.cu (one translation unit).
//
// Weights are held in bf16 ([O][I], the engine's row-major layout), uploaded
// once; activations between the steps stay on the device (bf16, except the
// GDN block's qkv / z, kept fp32 for the recurrence), only x goes
// up and the block output comes back, as in the Vulkan backend's single
// submit. The projections run on linear_kernel (tcgen05); the mixer steps are
// the same kernels as the *_dev entry points.

struct ColiCudaTensor {
    __nv_bfloat16 *w = nullptr;   // [O][I]
    int I = 0, O = 0;
    CUtensorMap tm;               // 64 x 128 boxes, 128B swizzle
};

namespace {

int make_bf16_2d(CUtensorMap *m, const void *base, int inner, int outer, int box_inner, int box_outer)
{
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = G.encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled (bf16 2d) failed (%d)", (int)r);
    return 1;
}

// y[S][O] = x[S][I] W^T on the device (x bf16, y fp32 or bf16).
// K splits of a projection whose output tiles cannot fill the GPU: the
// 16-token decode kernel holds two CTAs per SM, so it targets 7/8 of two per
// SM (clusters placed near the full count spilled into a second wave), at
// most 8 splits (one thread-block cluster reduces them); the larger tiles hold
// one CTA per SM.
int linear_splits(int tiles, int nk, int bn)
{
    const int slots = bn == 16 ? 2 * G.num_sms * 7 / 8 : G.num_sms;
    if (2 * tiles > slots) return 1;
    int s = std::max(1, std::min(slots / tiles, nk / 4));
    if (bn == 16) s = std::min(s, 8);
    return s;
}
int linear_dev(const ColiCudaTensor *t, const __nv_bfloat16 *x, int S, void *y, int y_bf16)
{
    if (!t || !t->w) return fail("dense tensor not uploaded");
    const int bn = linear_pick_bn(S);
    CUtensorMap tx;
    if (!make_bf16_2d(&tx, x, t->I, S, 64, bn)) return 0;
    const int tiles = ((t->O + 127) / 128) * ((S + bn - 1) / bn), nk = (t->I + 63) / 64;
    const int splits = linear_splits(tiles, nk, bn);
    LinearArgs la;
    memset(&la, 0, sizeof(la));
    la.y = y; la.S = S; la.I = t->I; la.O = t->O; la.y_bf16 = y_bf16;
    if (splits > 1) {
        la.part = (float *)scratch(S_LPART, (size_t)splits * S * t->O * 4);
        if (!la.part) return 0;
        // per-tile arrival counters (used when bn == 16): zeroed when the slot is (re)allocated, and
        // the last split of each tile puts its counter back to zero
        const size_t need = (size_t)tiles * sizeof(int);
        if (G.slot_bytes[S_LCNT] < need) {
            if (!scratch(S_LCNT, need)) return 0;
            CK(cudaMemsetAsync(G.slot[S_LCNT], 0, G.slot_bytes[S_LCNT], stream()));
        }
        la.tile_cnt = (int *)G.slot[S_LCNT];
    }
    int nl = 1;
    CK(launch_linear(t->tm, tx, la, bn, splits, stream(), &nl));
    g_launches += nl;
    return 1;
}

// Several projections of the same x (S <= 16 rows: decode) in one launch;
// larger S runs them one by one (each already fills the GPU).
int linear_dev_multi(const ColiCudaTensor *const *t, int nw, const __nv_bfloat16 *x, int S, void *const *y,
                     int y_bf16)
{
    if (S > 16 || nw > LIN_MAXW) {
        for (int i = 0; i < nw; ++i)
            if (!linear_dev(t[i], x, S, y[i], y_bf16)) return 0;
        return 1;
    }
    const CUtensorMap *maps[LIN_MAXW];
    int O[LIN_MAXW];
    int tiles = 0, Osum = 0;
    for (int i = 0; i < nw; ++i) {
        if (!t[i] || !t[i]->w) return fail("dense tensor not uploaded");
        if (t[i]->I != t[0]->I) return fail("projections of one launch need the same input width");
        maps[i] = &t[i]->tm; O[i] = t[i]->O;
        tiles += (O[i] + 127) / 128; Osum += O[i];
    }
    CUtensorMap tx;
    if (!make_bf16_2d(&tx, x, t[0]->I, S, 64, 16)) return 0;
    const int nk = (t[0]->I + 63) / 64;
    const int splits = linear_splits(tiles, nk, 16);
    LinearArgs la;
    memset(&la, 0, sizeof(la));
    la.S = S; la.I = t[0]->I; la.O = Osum; la.y_bf16 = y_bf16;
    if (splits > 1) {
        la.part = (float *)scratch(S_LPART, (size_t)splits * S * Osum * 4);
        if (!la.part) return 0;
        const size_t need = (size_t)tiles * sizeof(int);
        if (G.slot_bytes[S_LCNT] < need) {
            if (!scratch(S_LCNT, need)) return 0;
            CK(cudaMemsetAsync(G.slot[S_LCNT], 0, G.slot_bytes[S_LCNT], stream()));
        }
        la.tile_cnt = (int *)G.slot[S_LCNT];
    }
    CK(launch_linear_multi(maps, O, y, nw, tx, la, splits, stream()));
    g_launches += 1;
    return 1;
}

// Host fp32 [n] -> device bf16 (through an fp32 staging slot).
const __nv_bfloat16 *upload_bf16(const float *x, size_t n)
{
    const float *xd = (const float *)upload(S_IN0, x, n * 4);
    __nv_bfloat16 *xb = (__nv_bfloat16 *)scratch(S_XB, n * 2);
    if (!xd || !xb) return nullptr;
    if (launch_f32_to_bf16(xd, xb, n, stream()) != cudaSuccess) {
        cuda_fail(cudaGetLastError(), "f32_to_bf16");
        return nullptr;
    }
    g_launches += 1;
    return xb;
}

int tensor_shape(const ColiCudaTensor *t, int I, int O, const char *what)
{
    if (!t || !t->w) return fail("%s tensor not uploaded", what);
    if (t->I != I || t->O != O) return fail("%s tensor is %dx%d, expected %dx%d", what, t->O, t->I, O, I);
    return 1;
}

}  // namespace

extern "C" {

int coli_cuda_tensor_ensure(ColiCudaTensor **tensor, const void *weights, const float *scales, int fmt, int I,
                            int O, int grp)
{
    READY();
    (void)grp;
    if (!tensor) return fail("null tensor handle");
    if (*tensor && (*tensor)->I == I && (*tensor)->O == O) return 1;   // resident already
    if (fmt != 0 && fmt != 1) return fail("dense format %d not supported (0 = f32, 1 = int8 per-row scale)", fmt);
    if (fmt == 1 && !scales) return fail("int8 weights need per-row scales");
    if (I < 8 || I % 8 || O < 1 || !weights) return fail("bad dense shape %dx%d (I must be a multiple of 8)", O, I);
    ColiCudaTensor *t = *tensor ? *tensor : new ColiCudaTensor();
    if (t->w) { dev_free(t->w, (size_t)t->I * t->O * 2); t->w = nullptr; }
    std::vector<__nv_bfloat16> h((size_t)I * O);
    for (int o = 0; o < O; ++o) {
        for (int i = 0; i < I; ++i) {
            const size_t k = (size_t)o * I + i;
            const float v = fmt == 0 ? static_cast<const float *>(weights)[k]
                                     : (float)static_cast<const int8_t *>(weights)[k] * scales[o];
            h[k] = __float2bfloat16_rn(v);
        }
    }
    void *d = nullptr;
    if (!dev_alloc(&d, h.size() * 2)) { if (!*tensor) delete t; return 0; }
    t->w = (__nv_bfloat16 *)d;
    t->I = I; t->O = O;
    if (cudaMemcpyAsync(t->w, h.data(), h.size() * 2, cudaMemcpyHostToDevice, stream()) != cudaSuccess ||
        cudaStreamSynchronize(stream()) != cudaSuccess) {
        cuda_fail(cudaGetLastError(), "tensor upload");
        return 0;
    }
    if (!make_bf16_2d(&t->tm, t->w, I, O, 64, 128)) return 0;
    *tensor = t;
    return 1;
}

void coli_cuda_tensor_free(ColiCudaTensor *t)
{
    if (!t) return;
    if (t->w) dev_free(t->w, (size_t)t->I * t->O * 2);
    delete t;
}

size_t coli_cuda_tensor_bytes(const ColiCudaTensor *t) { return t && t->w ? (size_t)t->I * t->O * 2 : 0; }

int coli_cuda_matmul(ColiCudaTensor **tensor, float *y, const float *x, const void *w, const float *scales, int fmt,
                     int S, int I, int O, int gs)
{
    READY();
    if (S < 1) return fail("bad S");
    if (!coli_cuda_tensor_ensure(tensor, w, scales, fmt, I, O, gs)) return 0;
    const __nv_bfloat16 *xb = upload_bf16(x, (size_t)S * I);
    float *yd = (float *)scratch(S_OUT, (size_t)S * O * 4);
    if (!xb || !yd) return 0;
    if (!linear_dev(*tensor, xb, S, yd, 0)) return 0;
    if (!download(y, yd, (size_t)S * O * 4)) return 0;
    return check_dev_error();
}

int coli_cuda_matmul_dev(const ColiCudaTensor *tensor, const void *x, int S, void *y, int y_bf16)
{
    READY();
    if (S < 1 || !x || !y) return fail("bad matmul_dev arguments");
    if (reinterpret_cast<uintptr_t>(x) & 15) return fail("x must be 16-byte aligned");
    return linear_dev(tensor, static_cast<const __nv_bfloat16 *>(x), S, y, y_bf16);
}

int coli_cuda_matmul_multi_dev(const ColiCudaTensor *const *tensors, int n, const void *x, int S,
                               void *const *y, int y_bf16)
{
    READY();
    if (n < 1 || n > LIN_MAXW || S < 1 || !tensors || !x || !y) return fail("bad matmul_multi_dev arguments");
    if (reinterpret_cast<uintptr_t>(x) & 15) return fail("x must be 16-byte aligned");
    for (int i = 0; i < n; ++i)
        if (!y[i]) return fail("matmul_multi_dev: output %d missing", i);
    return linear_dev_multi(tensors, n, static_cast<const __nv_bfloat16 *>(x), S, y, y_bf16);
}

}  // extern "C"

namespace {

// The GQA block on device data: x bf16 [S][D] -> out fp32 [S][Dout].
int gqa_block_dev(int layer, const __nv_bfloat16 *xb, int D, ColiCudaTensor *gq_t, ColiCudaTensor *gk_t,
                  ColiCudaTensor *gv_t, ColiCudaTensor *out_t, float *od, int S, int H, int KH, int hd, int rot,
                  int pos_base, int max_t, float eps, float theta, int Dout)
{
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (S < 1 || pos_base < 0) return fail("bad S/pos_base");
    KvLayer &L = G.kv[layer];
    if (!L.k) return fail("KV layer %d not allocated", layer);
    kv_adopt_split(L, KH, max_t);
    if (max_t > L.max_t || pos_base + S > L.max_t) return fail("positions beyond the cache (max_t %d)", L.max_t);
    if (!tensor_shape(gq_t, D, H * 2 * hd, "q|gate") || !tensor_shape(gk_t, D, KH * hd, "k") ||
        !tensor_shape(gv_t, D, KH * hd, "v") || !tensor_shape(out_t, H * hd, Dout, "o_proj"))
        return 0;
    auto *qg = (__nv_bfloat16 *)scratch(S_PQ, (size_t)S * H * 2 * hd * 2);
    auto *k = (__nv_bfloat16 *)scratch(S_PK, (size_t)S * KH * hd * 2);
    auto *v = (__nv_bfloat16 *)scratch(S_PV, (size_t)S * KH * hd * 2);
    auto *ctx = (__nv_bfloat16 *)scratch(S_PCTX, (size_t)S * H * hd * 2);
    if (!qg || !k || !v || !ctx) return 0;
    {
        const ColiCudaTensor *ts[3] = {gq_t, gk_t, gv_t};
        void *ys[3] = {qg, k, v};
        if (!linear_dev_multi(ts, 3, xb, S, ys, 1)) return 0;
    }
    if (!coli_cuda_gqa_step_dev(layer, 0, S, pos_base, qg, k, v, ctx, H, KH, hd, rot, eps, theta, 1)) return 0;
    return linear_dev(out_t, ctx, S, od, 0);
}

// The GDN block on device data (request 0): x bf16 [S][D] -> out fp32
// [S][Dout]. The gates come either from params rows on the device
// [S][2*VH+VD] (decay | beta | gnorm, the engine's packing), or, with ga_t /
// gb_t given (pd unused), from the a / b projections run on the device in the
// same launch as in_proj_qkv / in_proj_z (c/qwen.c:709-711) and turned into
// decay / beta inside the mixer kernels with the layer's A_log / dt_bias /
// gnorm (c/qwen.c:722-727).
int gdn_block_dev(int layer, const __nv_bfloat16 *xb, int S, int D, ColiCudaTensor *gqkv_t, ColiCudaTensor *gz_t,
                  const float *pd, ColiCudaTensor *out_t, float *od, int KH, int KD, int VH, int VD, int conv_dim,
                  int conv_k, float eps, int Dout, ColiCudaTensor *ga_t = nullptr, ColiCudaTensor *gb_t = nullptr)
{
    if (!check_layer(layer)) return fail("layer %d out of range", layer);
    if (S < 1) return fail("bad S");
    if (conv_k != 4 || conv_dim != 2 * KH * KD + VH * VD) return fail("conv shape %d x %d not supported", conv_k, conv_dim);
    if (!tensor_shape(gqkv_t, D, conv_dim, "in_proj_qkv") || !tensor_shape(gz_t, D, VH * VD, "in_proj_z") ||
        !tensor_shape(out_t, VH * VD, Dout, "out_proj"))
        return 0;
    const bool dev_ab = ga_t && gb_t;
    if (dev_ab) {
        if (!tensor_shape(ga_t, D, VH, "in_proj_a") || !tensor_shape(gb_t, D, VH, "in_proj_b")) return 0;
        const GdnLayer &L = G.gdn[layer];
        if (!L.A_log || !L.gnorm || L.pVH != VH || L.pVD != VD)
            return fail("GDN A_log/dt_bias/gnorm not set for %d x %d", VH, VD);
        pd = nullptr;
    } else if (!pd) {
        return fail("GDN params rows or a / b projections required");
    }
    // The projections leave qkv and z in fp32: the recurrence is sensitive to
    // the rounding of q and k (for a fast-decaying head y_t is nearly
    // (q_t . k_t) d_t, and the gated norm rescales a small row back to unit
    // size), so they are not rounded to bf16 between the GEMM and the mixer.
    const int ps = 2 * VH + VD;
    auto *qkv = (float *)scratch(S_PQ, (size_t)S * conv_dim * 4);
    auto *z = (float *)scratch(S_PK, (size_t)S * VH * VD * 4);
    auto *yf = (float *)scratch(S_PY2, (size_t)S * VH * VD * 4);
    auto *y = (__nv_bfloat16 *)scratch(S_PCTX, (size_t)S * VH * VD * 2);
    auto *ab = dev_ab ? (float *)scratch(S_PV, (size_t)S * 2 * VH * 4) : nullptr;   // a [S][VH] | b [S][VH]
    if (!qkv || !z || !yf || !y || (dev_ab && !ab)) return 0;
    float *a = dev_ab ? ab : nullptr, *b = dev_ab ? ab + (size_t)S * VH : nullptr;
    {
        const ColiCudaTensor *ts[4] = {gqkv_t, gz_t, ga_t, gb_t};
        void *ys[4] = {qkv, z, a, b};
        if (!linear_dev_multi(ts, dev_ab ? 4 : 2, xb, S, ys, 0)) return 0;
    }
    if (S >= GDN_CHUNK_MIN_ROWS) {
        if (!gdn_prefill_chunked(layer, 0, S, qkv, z, a, b, yf, KH, KD, VH, VD, eps, 0, 0, -1, pd))
            return 0;
    } else {
        for (int s = 0; s < S; ++s) {
            const float *pr = pd ? pd + (size_t)s * ps : nullptr;
            if (!gdn_decode_run(layer, 1, 0, qkv + (size_t)s * conv_dim, z + (size_t)s * VH * VD,
                                a ? a + (size_t)s * VH : nullptr, b ? b + (size_t)s * VH : nullptr,
                                yf + (size_t)s * VH * VD, KH, KD, VH, VD, eps, 0, pr, pr ? pr + VH : nullptr,
                                pr ? pr + 2 * VH : nullptr))
                return 0;
        }
    }
    CK(launch_f32_to_bf16(yf, y, (size_t)S * VH * VD, stream()));
    g_launches += 1;
    return linear_dev(out_t, y, S, od, 0);
}

// resid + delta -> resid_out; rmsnorm_zc(., post_ln) -> nrm; router logits;
// all three read back (the route tail of the Vulkan backend,
// c/backend_vulkan.c:2378-2406).
int route_tail(const float *rd, const float *delta, ColiCudaTensor *router, int ln_layer, float *resid_out,
               float *nrm_out, float *pr_out, int S, int D, int E, float eps)
{
    float *xo = (float *)scratch(S_RXO, (size_t)S * D * 4);
    float *nrm = (float *)scratch(S_RN, (size_t)S * D * 4);
    auto *nb = (__nv_bfloat16 *)scratch(S_RNB, (size_t)S * D * 2);
    float *pr = (float *)scratch(S_RP, (size_t)S * E * 4);
    if (!xo || !nrm || !nb || !pr) return 0;
    CK(launch_rmsnorm_zc_rows(rd, delta, G.ln_w[ln_layer] + D, xo, nrm, nb, S, D, eps, stream()));
    g_launches += 1;
    if (!linear_dev(router, nb, S, pr, 0)) return 0;
    if (!download(resid_out, xo, (size_t)S * D * 4) || !download(nrm_out, nrm, (size_t)S * D * 4) ||
        !download(pr_out, pr, (size_t)S * E * 4))
        return 0;
    return check_dev_error();
}

int route_checks(ColiCudaTensor *router, int ln_layer, int D, int Dout, int E)
{
    if (ln_layer < 0 || ln_layer >= MAX_LAYERS || !G.ln_w[ln_layer] || G.ln_D[ln_layer] != D)
        return fail("layer norm weights of layer %d not set for D = %d", ln_layer, D);
    if (Dout != D) return fail("the residual tail needs Dout == D");
    return tensor_shape(router, D, E, "router");
}

}  // namespace

extern "C" {

int coli_cuda_gqa_full(int layer, const float *x, int D, ColiCudaTensor *gq_t, ColiCudaTensor *gk_t,
                       ColiCudaTensor *gv_t, ColiCudaTensor *out_t, float *out, int S, int H, int KH, int hd,
                       int rot, int pos_base, int max_t, float eps, float theta, int Dout)
{
    READY();
    if (S < 1) return fail("bad S");
    const __nv_bfloat16 *xb = upload_bf16(x, (size_t)S * D);
    float *od = (float *)scratch(S_PY, (size_t)S * Dout * 4);
    if (!xb || !od) return 0;
    if (!gqa_block_dev(layer, xb, D, gq_t, gk_t, gv_t, out_t, od, S, H, KH, hd, rot, pos_base, max_t, eps, theta,
                       Dout))
        return 0;
    if (!download(out, od, (size_t)S * Dout * 4)) return 0;
    return check_dev_error();
}

static int gdn_full_rows(int layer, const float *x, int S, int D, ColiCudaTensor *gqkv_t, ColiCudaTensor *gz_t,
                         const float *params, ColiCudaTensor *out_t, float *out, int KH, int KD, int VH, int VD,
                         int conv_dim, int conv_k, float eps, int Dout)
{
    READY();
    if (S < 1 || !params) return fail("bad S / params");
    const __nv_bfloat16 *xb = upload_bf16(x, (size_t)S * D);
    const float *pd = (const float *)upload(S_PAR, params, (size_t)S * (2 * VH + VD) * 4);
    float *od = (float *)scratch(S_PY, (size_t)S * Dout * 4);
    if (!xb || !pd || !od) return 0;
    if (!gdn_block_dev(layer, xb, S, D, gqkv_t, gz_t, pd, out_t, od, KH, KD, VH, VD, conv_dim, conv_k, eps, Dout))
        return 0;
    if (!download(out, od, (size_t)S * Dout * 4)) return 0;
    return check_dev_error();
}

int coli_cuda_gdn_full(int layer, const float *x, int D, ColiCudaTensor *gqkv_t, ColiCudaTensor *gz_t,
                       const float *params, ColiCudaTensor *out_t, float *out, int KH, int KD, int VH, int VD,
                       int conv_dim, int conv_k, float eps, int Dout)
{
    return gdn_full_rows(layer, x, 1, D, gqkv_t, gz_t, params, out_t, out, KH, KD, VH, VD, conv_dim, conv_k, eps,
                         Dout);
}

int coli_cuda_gdn_full_seq(int layer, const float *x, int S, int D, ColiCudaTensor *gqkv_t, ColiCudaTensor *gz_t,
                           const float *params, ColiCudaTensor *out_t, float *out, int KH, int KD, int VH, int VD,
                           int conv_dim, int conv_k, float eps, int Dout)
{
    return gdn_full_rows(layer, x, S, D, gqkv_t, gz_t, params, out_t, out, KH, KD, VH, VD, conv_dim, conv_k, eps,
                         Dout);
}

int coli_cuda_gdn_full_ab(int layer, const float *x, int S, int D, ColiCudaTensor *gqkv_t, ColiCudaTensor *gz_t,
                          ColiCudaTensor *ga_t, ColiCudaTensor *gb_t, ColiCudaTensor *out_t, float *out, int KH,
                          int KD, int VH, int VD, int conv_dim, int conv_k, float eps, int Dout)
{
    READY();
    if (S < 1 || !x || !out) return fail("bad S / buffers");
    if (!ga_t || !gb_t) return fail("in_proj_a / in_proj_b required");
    const __nv_bfloat16 *xb = upload_bf16(x, (size_t)S * D);
    float *od = (float *)scratch(S_PY, (size_t)S * Dout * 4);
    if (!xb || !od) return 0;
    if (!gdn_block_dev(layer, xb, S, D, gqkv_t, gz_t, nullptr, out_t, od, KH, KD, VH, VD, conv_dim, conv_k, eps,
                       Dout, ga_t, gb_t))
        return 0;
    if (!download(out, od, (size_t)S * Dout * 4)) return 0;
    return check_dev_error();
}

int coli_cuda_moe_route_available(void) { return G.ready; }

int coli_cuda_layer_norm_weight(int layer, const float *in_ln, const float *post_ln, int D)
{
    READY();
    if (layer < 0 || layer >= MAX_LAYERS || D < 1 || !in_ln || !post_ln) return fail("bad layer norm weights");
    if (G.ln_w[layer] && G.ln_D[layer] != D) {
        dev_free(G.ln_w[layer], (size_t)2 * G.ln_D[layer] * 4);
        G.ln_w[layer] = nullptr;
    }
    if (!G.ln_w[layer]) {
        void *d = nullptr;
        if (!dev_alloc(&d, (size_t)2 * D * 4)) return 0;
        G.ln_w[layer] = (float *)d;
        G.ln_D[layer] = D;
    }
    CK(cudaMemcpyAsync(G.ln_w[layer], in_ln, (size_t)D * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaMemcpyAsync(G.ln_w[layer] + D, post_ln, (size_t)D * 4, cudaMemcpyHostToDevice, stream()));
    CK(cudaStreamSynchronize(stream()));
    return 1;
}

int coli_cuda_gqa_full_route(int layer, const float *resid, int D, ColiCudaTensor *gq_t, ColiCudaTensor *gk_t,
                             ColiCudaTensor *gv_t, ColiCudaTensor *out_t, ColiCudaTensor *router, int ln_layer,
                             float *resid_out, float *nrm_out, float *pr_out, int S, int H, int KH, int hd, int rot,
                             int pos_base, int max_t, float eps, float theta, int Dout, int E)
{
    READY();
    if (S < 1 || !resid || !resid_out || !nrm_out || !pr_out) return fail("bad route arguments");
    if (!route_checks(router, ln_layer, D, Dout, E)) return 0;
    const float *rd = (const float *)upload(S_RX, resid, (size_t)S * D * 4);
    auto *xb = (__nv_bfloat16 *)scratch(S_XB, (size_t)S * D * 2);
    float *od = (float *)scratch(S_PY, (size_t)S * Dout * 4);
    if (!rd || !xb || !od) return 0;
    // in_ln on the device: the attention input
    CK(launch_rmsnorm_zc_rows(rd, nullptr, G.ln_w[ln_layer], nullptr, nullptr, xb, S, D, eps, stream()));
    g_launches += 1;
    if (!gqa_block_dev(layer, xb, D, gq_t, gk_t, gv_t, out_t, od, S, H, KH, hd, rot, pos_base, max_t, eps, theta,
                       Dout))
        return 0;
    return route_tail(rd, od, router, ln_layer, resid_out, nrm_out, pr_out, S, D, E, eps);
}

int coli_cuda_gdn_full_route(int layer, const float *x_in, const float *resid, int D, ColiCudaTensor *gqkv_t,
                             ColiCudaTensor *gz_t, const float *params, ColiCudaTensor *out_t, ColiCudaTensor *router,
                             int ln_layer, float *resid_out, float *nrm_out, float *pr_out, int KH, int KD, int VH,
                             int VD, int conv_dim, int conv_k, float eps, int Dout, int E)
{
    READY();
    if (!x_in || !resid || !params || !resid_out || !nrm_out || !pr_out) return fail("bad route arguments");
    if (!route_checks(router, ln_layer, D, Dout, E)) return 0;
    const __nv_bfloat16 *xb = upload_bf16(x_in, (size_t)D);
    const float *rd = (const float *)upload(S_RX, resid, (size_t)D * 4);
    const float *pd = (const float *)upload(S_PAR, params, (size_t)(2 * VH + VD) * 4);
    float *od = (float *)scratch(S_PY, (size_t)Dout * 4);
    if (!xb || !rd || !pd || !od) return 0;
    if (!gdn_block_dev(layer, xb, 1, D, gqkv_t, gz_t, pd, out_t, od, KH, KD, VH, VD, conv_dim, conv_k, eps, Dout))
        return 0;
    return route_tail(rd, od, router, ln_layer, resid_out, nrm_out, pr_out, 1, D, E, eps);
}

}  // extern "C"

extern "C" {

int coli_cuda_gqa_project(int layer, const float *q, ColiCudaTensor *ot, float *out, int S, int H, int KH, int hd,
                          int max_t, int st0, int T, float scale, int Dout)
{
    READY();
    if (S < 1) return fail("bad S");
    if (!tensor_shape(ot, H * hd, Dout, "o_proj")) return 0;
    auto *ctx = (__nv_bfloat16 *)scratch(S_PCTX, (size_t)S * H * hd * 2);
    float *od = (float *)scratch(S_PY, (size_t)S * Dout * 4);
    if (!ctx || !od) return 0;
    if (!gqa_core(layer, q, ctx, 1, S, H, KH, hd, max_t, st0, T, scale)) return 0;
    if (!linear_dev(ot, ctx, S, od, 0)) return 0;
    if (!download(out, od, (size_t)S * Dout * 4)) return 0;
    return check_dev_error();
}

int coli_cuda_gdn_project(int layer, const float *qn, const float *kn, const float *v, const float *z,
                          const float *decay, const float *beta, const float *gnorm, ColiCudaTensor *ot, float *out,
                          int KH, int KD, int VH, int VD, float eps, int Dout)
{
    READY();
    if (!tensor_shape(ot, VH * VD, Dout, "out_proj")) return 0;
    float *yd = (float *)scratch(S_OUT, (size_t)VH * VD * 4);
    auto *yb = (__nv_bfloat16 *)scratch(S_PCTX, (size_t)VH * VD * 2);
    float *od = (float *)scratch(S_PY, (size_t)Dout * 4);
    if (!yd || !yb || !od) return 0;
    if (!gdn_core(layer, qn, kn, v, z, decay, beta, gnorm, yd, KH, KD, VH, VD, eps)) return 0;
    CK(launch_f32_to_bf16(yd, yb, (size_t)VH * VD, stream()));
    g_launches += 1;
    if (!linear_dev(ot, yb, 1, od, 0)) return 0;
    if (!download(out, od, (size_t)Dout * 4)) return 0;
    return check_dev_error();
}

}  // extern "C"
