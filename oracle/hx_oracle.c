/*
 * hx_oracle.c — TEST INFRASTRUCTURE ONLY (see hx_oracle.h): scalar C restatement of the
 * reference's quantized MoE expert path, used as the checker for the CUDA backend.
 * Each function names the reference lines it restates (paths inside pierce-lonergan/hearth).
 * Build with -ffp-contract=off: every float operation below is one rounded IEEE operation.
 */
#include "hx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define QK 64
#define CANON_NAN 0x7fc00000u

static float bits_to_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* engine/src/quant.c:17-35 (f16 -> f32, quiet NaNs; subnormals scaled exactly). */
float orc_f16(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0x1fu) return bits_to_f(s | 0x7f800000u | (m << 13) | (m ? 0x00400000u : 0u));
    if (e) return bits_to_f(s | ((e + 112u) << 23) | (m << 13));
    if (!m) return bits_to_f(s);
    {
        float f = (float)m * 5.9604644775390625e-8f; /* m * 2^-24: exact */
        uint32_t fb;
        memcpy(&fb, &f, 4);
        return bits_to_f(s | fb);
    }
}

static float bf16_to_f(uint16_t h) { return bits_to_f((uint32_t)h << 16); }

/* engine/src/quant.c:59-65: NaN results are stored as one quiet NaN. */
static float canon(float v) { return v != v ? bits_to_f(CANON_NAN) : v; }

/* engine/src/quant.c:46-49: round half to even for |v| < 2^22. */
static float rint_magic(float v) {
    volatile float t = v + 12582912.0f;
    return t - 12582912.0f;
}

/* engine/src/quant.c:80-90 */
size_t orc_row_bytes(int dtype, int64_t n) {
    if (n <= 0 || n > ((int64_t)1 << 40)) return 0;
    switch (dtype) {
    case ORC_F32: return (size_t)n * 4;
    case ORC_F16: case ORC_BF16: return (size_t)n * 2;
    case ORC_Q8: return n % QK ? 0 : (size_t)(n / QK) * 66;
    case ORC_Q4: return n % QK ? 0 : (size_t)(n / QK) * 34;
    default: return 0;
    }
}

/* engine/src/quant.c:311-315 */
size_t orc_act_bytes(int wdtype, int64_t n) {
    if (n <= 0) return 0;
    if (wdtype == ORC_Q8 || wdtype == ORC_Q4) return n % QK ? 0 : (size_t)(n / QK) * sizeof(orc_act_q8);
    return (size_t)n * 4;
}

/* engine/tests/test_quant.c:867-871 */
uint64_t orc_fnv1a(const void *p, size_t n, uint64_t h) {
    const uint8_t *b = (const uint8_t *)p;
    for (size_t i = 0; i < n; i++) h = (h ^ b[i]) * 0x100000001b3ull;
    return h;
}

/* engine/tests/test_quant.c:873-887: libm-free deterministic inputs of the pinned tests. */
void orc_det_fill(float *x, int64_t n, uint64_t seed) {
    uint64_t s = seed;
    for (int64_t i = 0; i < n; i++) {
        double v = 0.0;
        const int64_t blk = i / 64;
        for (int k = 0; k < 4; k++) {
            s = s * 6364136223846793005ull + 1442695040888963407ull;
            v += (double)((int64_t)(s >> 40) - (1 << 23)) * 0x1p-23;
        }
        v *= ldexp(1.0, (int)(blk % 7) - 3);
        if (blk % 13 == 5 && i % 64 == 17) v *= 40.0;
        if (blk % 11 == 3) v = 0.0;
        x[i] = (float)v;
    }
}

void orc_expf_batch(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = expf(x[i]);
}

/* engine/src/quant.c:325-348, docs/NUMERICS.md §2. NaN products become 0, +-inf saturates. */
void orc_act_quantize(const float *x, orc_act_q8 *out, int64_t n) {
    for (int64_t b = 0; b < n / QK; b++, x += QK) {
        float amax = 0.0f, d, id;
        int32_t sum = 0;
        for (int i = 0; i < QK; i++) {
            const float a = fabsf(x[i]);
            if (a > amax) amax = a;
        }
        d = amax / 127.0f;
        id = d != 0.0f ? 1.0f / d : 0.0f;
        for (int i = 0; i < QK; i++) {
            float v = x[i] * id;
            int q;
            if (v != v) v = 0.0f;
            if (v > 127.0f) v = 127.0f;
            if (v < -127.0f) v = -127.0f;
            q = (int)rint_magic(v);
            out[b].q[i] = (int8_t)q;
            sum += q;
        }
        out[b].d = d;
        out[b].sum = sum;
    }
}

/* docs/NUMERICS.md §1 (engine/src/quant.c:604-624): 16 lanes, then the 8/4/2/1 tree. */
static float tree16(float *L) {
    for (int s = 8; s >= 1; s >>= 1)
        for (int j = 0; j < s; j++) L[j] = L[j] + L[j + s];
    return L[0];
}

float orc_sum16(const float *a, int64_t n) {
    float L[16] = {0};
    for (int64_t i = 0; i < n; i++) L[i & 15] = L[i & 15] + a[i];
    return tree16(L);
}

float orc_dot16(const float *a, const float *b, int64_t n) {
    float L[16] = {0};
    for (int64_t i = 0; i < n; i++) {
        const float p = a[i] * b[i];
        L[i & 15] = L[i & 15] + p;
    }
    return tree16(L);
}

/* engine/src/quant.c:352-365: dot16 with the weight row converted to f32 first. */
static float dot16_row(int dt, const void *w, const float *x, int64_t n) {
    float L[16] = {0};
    for (int64_t i = 0; i < n; i++) {
        float wi, p;
        if (dt == ORC_F32) wi = ((const float *)w)[i];
        else if (dt == ORC_F16) wi = orc_f16(((const uint16_t *)w)[i]);
        else wi = bf16_to_f(((const uint16_t *)w)[i]);
        p = wi * x[i];
        L[i & 15] = L[i & 15] + p;
    }
    return tree16(L);
}

/* One quantized row against one activation, docs/NUMERICS.md §3 (quant.c:388-427). */
static float qrow(int dt, const uint8_t *row, const orc_act_q8 *a, int64_t nb) {
    float acc = 0.0f;
    const size_t bs = dt == ORC_Q8 ? 66 : 34;
    for (int64_t g = 0; g < nb; g++) {
        const uint8_t *blk = row + (size_t)g * bs;
        const uint16_t dh = (uint16_t)(blk[0] | (blk[1] << 8));
        int32_t isum = 0;
        float sc, p;
        if (dt == ORC_Q8) {
            for (int i = 0; i < QK; i++) isum += (int32_t)(int8_t)blk[2 + i] * (int32_t)a[g].q[i];
        } else {
            for (int j = 0; j < 32; j++) {
                isum += ((int32_t)(blk[2 + j] & 0x0f) - 8) * (int32_t)a[g].q[j];
                isum += ((int32_t)(blk[2 + j] >> 4) - 8) * (int32_t)a[g].q[j + 32];
            }
        }
        sc = orc_f16(dh) * a[g].d;
        p = (float)isum * sc;
        acc = acc + p;
    }
    return acc;
}

/* The row-range kernel contract of engine/src/hx_quant.h:49-57. */
void orc_matmul_rows(int dtype, const void *W, int64_t n_cols, const void *act, int T,
                     float *Y, int64_t ldy, int64_t r0, int64_t r1) {
    const size_t rb = orc_row_bytes(dtype, n_cols);
    for (int64_t r = r0; r < r1; r++) {
        const uint8_t *w = (const uint8_t *)W + (size_t)r * rb;
        for (int t = 0; t < T; t++) {
            float y;
            if (dtype == ORC_Q8 || dtype == ORC_Q4)
                y = qrow(dtype, w, (const orc_act_q8 *)act + (size_t)t * (size_t)(n_cols / QK), n_cols / QK);
            else
                y = dot16_row(dtype, w, (const float *)act + (size_t)t * (size_t)n_cols, n_cols);
            Y[(size_t)t * (size_t)ldy + (size_t)r] = canon(y);
        }
    }
}

/* engine/src/quant.c:574-600 (hearth_matmul): quantize each token, then all rows. */
int orc_matmul(int dtype, const void *W, int64_t n_rows, int64_t n_cols, const float *X, int T, float *Y) {
    const int quant = dtype == ORC_Q8 || dtype == ORC_Q4;
    void *buf = NULL;
    const void *act = X;
    if (dtype < ORC_F32 || dtype > ORC_Q4 || n_rows < 0 || T < 0 || orc_row_bytes(dtype, n_cols) == 0) return -1;
    if (T == 0 || n_rows == 0) return 0;
    if (!W || !X || !Y) return -1;
    if (quant) {
        const size_t ab = orc_act_bytes(dtype, n_cols);
        buf = malloc(ab * (size_t)T);
        if (!buf) return -3;
        for (int t = 0; t < T; t++)
            orc_act_quantize(X + (size_t)t * (size_t)n_cols, (orc_act_q8 *)((uint8_t *)buf + (size_t)t * ab), n_cols);
        act = buf;
    }
    orc_matmul_rows(dtype, W, n_cols, act, T, Y, n_rows, 0, n_rows);
    free(buf);
    return 0;
}

/* engine/src/quant.c:257-307 + 563-571 (hearth_dequantize) for the five float/quant dtypes. */
int orc_dequantize(int dtype, const void *src, int64_t n_rows, int64_t n_cols, float *dst) {
    const size_t rb = orc_row_bytes(dtype, n_cols);
    if (rb == 0 || n_rows < 0) return -1;
    for (int64_t r = 0; r < n_rows; r++) {
        const uint8_t *s = (const uint8_t *)src + (size_t)r * rb;
        float *o = dst + (size_t)r * (size_t)n_cols;
        for (int64_t i = 0; i < n_cols; i++) {
            switch (dtype) {
            case ORC_F32: memcpy(&o[i], s + 4 * i, 4); break;
            case ORC_F16: o[i] = orc_f16((uint16_t)(s[2 * i] | (s[2 * i + 1] << 8))); break;
            case ORC_BF16: o[i] = bf16_to_f((uint16_t)(s[2 * i] | (s[2 * i + 1] << 8))); break;
            case ORC_Q8: {
                const uint8_t *blk = s + (size_t)(i / QK) * 66;
                o[i] = orc_f16((uint16_t)(blk[0] | (blk[1] << 8))) * (float)(int8_t)blk[2 + i % QK];
                break;
            }
            default: {
                const uint8_t *blk = s + (size_t)(i / QK) * 34;
                const int j = (int)(i % QK);
                const int nib = j < 32 ? (blk[2 + j] & 15) : (blk[2 + j - 32] >> 4);
                o[i] = orc_f16((uint16_t)(blk[0] | (blk[1] << 8))) * (float)(nib - 8);
                break;
            }
            }
        }
    }
    return 0;
}

/* docs/NUMERICS.md §4 (engine/src/quant.c:626-651). */
void orc_rmsnorm(float *y, const float *x, const float *w, int64_t n, float eps) {
    float ms, r, den;
    if (n <= 0) return;
    ms = orc_dot16(x, x, n) / (float)n;
    den = sqrtf(ms + eps);
    r = 1.0f / den;
    for (int64_t i = 0; i < n; i++) {
        const float a = x[i] * r;
        y[i] = a * w[i];
    }
}

void orc_softmax(float *x, int64_t n) {
    float m, s;
    if (n <= 0) return;
    m = x[0];
    for (int64_t i = 1; i < n; i++) m = x[i] > m ? x[i] : m;
    for (int64_t i = 0; i < n; i++) x[i] = expf(x[i] - m);
    s = orc_sum16(x, n);
    for (int64_t i = 0; i < n; i++) x[i] = x[i] / s;
}

void orc_swiglu(float *out, const float *g, const float *u, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        const float gi = g[i], den = 1.0f + expf(-gi), s = gi / den;
        out[i] = s * u[i];
    }
}

float orc_sigmoid(float x) {
    const float den = 1.0f + expf(-x);
    return 1.0f / den;
}

/* engine/src/model.c:221-226: larger first, NaN last, ties to the lower index. */
static int ranks_before(float va, int ia, float vb, int ib) {
    const int na = va != va, nb = vb != vb;
    if (na || nb) return na == nb ? ia < ib : nb;
    if (va != vb) return va > vb;
    return ia < ib;
}

/* engine/src/model.c:793-831 (route_select), NUMERICS §5.3. */
void orc_route_select(const orc_route_cfg *c, const float *logits, const float *bias, int kk, int *ids, float *score) {
    const int E = c->E;
    float *sel = (float *)malloc(sizeof(float) * (size_t)E);
    unsigned char *taken = (unsigned char *)calloc((size_t)E, 1);
    memcpy(score, logits, sizeof(float) * (size_t)E);
    if (c->score_fn == ORC_SCORE_SOFTMAX) orc_softmax(score, E);
    else for (int e = 0; e < E; e++) score[e] = orc_sigmoid(score[e]);
    for (int e = 0; e < E; e++) sel[e] = (c->score_bias && bias) ? score[e] + bias[e] : score[e];
    if (c->n_group > 1) {
        const int ng = c->n_group, gs = E / ng;
        float *gsc = (float *)malloc(sizeof(float) * (size_t)ng);
        unsigned char *keep = (unsigned char *)calloc((size_t)ng, 1);
        for (int g = 0; g < ng; g++) {
            const float *v = sel + (size_t)g * gs;
            int i1 = 0, i2 = -1;
            for (int i = 1; i < gs; i++) {
                if (ranks_before(v[i], i, v[i1], i1)) { i2 = i1; i1 = i; }
                else if (i2 < 0 || ranks_before(v[i], i, v[i2], i2)) i2 = i;
            }
            gsc[g] = i2 >= 0 ? v[i1] + v[i2] : v[i1];
        }
        for (int r = 0; r < c->topk_group; r++) {
            int best = -1;
            for (int g = 0; g < ng; g++)
                if (!keep[g] && (best < 0 || ranks_before(gsc[g], g, gsc[best], best))) best = g;
            keep[best] = 1;
        }
        for (int g = 0; g < ng; g++)
            if (!keep[g]) for (int i = 0; i < gs; i++) sel[(size_t)g * gs + i] = 0.0f;
        free(gsc);
        free(keep);
    }
    for (int j = 0; j < kk; j++) {
        int best = -1;
        for (int e = 0; e < E; e++)
            if (!taken[e] && (best < 0 || ranks_before(sel[e], e, sel[best], best))) best = e;
        ids[j] = best;
        taken[best] = 1;
    }
    free(sel);
    free(taken);
}

/* engine/src/model.c:833-843 (route_weights). */
void orc_route_weights(const orc_route_cfg *c, const float *score, const int *ids, float *w) {
    for (int j = 0; j < c->K; j++) w[j] = score[ids[j]];
    if (c->norm_topk_prob) {
        float s = 0.0f, den;
        for (int j = 0; j < c->K; j++) s = s + w[j];
        den = s + 1e-20f;
        for (int j = 0; j < c->K; j++) w[j] = w[j] / den;
    }
    for (int j = 0; j < c->K; j++) w[j] = w[j] * c->routed_scale;
}

/* engine/src/model.c:1020-1037: union of experts (ascending), pairs grouped by expert and
 * tokens ascending within; pair_of[t*K+j] is the pair that holds token t's rank j. */
int orc_route_union(int E, int K, int T, const int *ids, int *ulist, int *u_p0, int *u_n, int *pair_tok, int *pair_of) {
    int *cnt = (int *)calloc((size_t)E, sizeof(int));
    int nu = 0;
    for (int i = 0; i < T * K; i++) cnt[ids[i]]++;
    for (int e = 0, p = 0; e < E; e++) {
        if (!cnt[e]) continue;
        ulist[nu] = e;
        u_p0[nu] = p;
        u_n[nu] = cnt[e];
        p += cnt[e];
        cnt[e] = u_p0[nu];
        nu++;
    }
    for (int i = 0; i < T; i++)
        for (int j = 0; j < K; j++) {
            const int p = cnt[ids[i * K + j]]++;
            pair_tok[p] = i;
            pair_of[i * K + j] = p;
        }
    free(cnt);
    return nu;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

/* docs/FORMAT.md §5 slab layout. */
void orc_slab_layout(int dtype, int64_t D, int64_t F, size_t *off_up, size_t *off_down, size_t *nbytes) {
    const size_t up = align_up((size_t)F * orc_row_bytes(dtype, D), 64);
    const size_t down = align_up(up + (size_t)F * orc_row_bytes(dtype, D), 64);
    const size_t end = down + (size_t)D * orc_row_bytes(dtype, F);
    if (off_up) *off_up = up;
    if (off_down) *off_down = down;
    if (nbytes) *nbytes = align_up(end, 4096);
}

/* One SwiGLU FFN for one token (engine/src/model.c:444-454 ffn and 847-897 compute_wave):
 * gate/up on x's activation, silu(g)*u, activation of that, down. */
static void ffn_one(int dt, const void *gate, const void *up, const void *down, int D, int F, const float *x, float *y) {
    const int quant = dt == ORC_Q8 || dt == ORC_Q4;
    float *g = (float *)malloc(sizeof(float) * (size_t)F), *u = (float *)malloc(sizeof(float) * (size_t)F);
    orc_act_q8 *ax = (orc_act_q8 *)malloc(orc_act_bytes(ORC_Q8, D)), *am = (orc_act_q8 *)malloc(orc_act_bytes(ORC_Q8, F));
    const void *act = x;
    if (quant) { orc_act_quantize(x, ax, D); act = ax; }
    orc_matmul_rows(dt, gate, D, act, 1, g, F, 0, F);
    orc_matmul_rows(dt, up, D, act, 1, u, F, 0, F);
    orc_swiglu(g, g, u, F);
    act = g;
    if (quant) { orc_act_quantize(g, am, F); act = am; }
    orc_matmul_rows(dt, down, F, act, 1, y, D, 0, D);
    free(g); free(u); free(ax); free(am);
}

/* engine/src/model.c:986-1131 (moe_layer) + 904-923 (moe_sum_range) + 925-934 (shared_expert),
 * evaluated token by token (INV-DET-2 makes the batched schedule equal to this). */
int orc_moe_layer_eval(const orc_moe_layer *L, const float *x, int T, float *out, int *ids_out, float *wts_out) {
    const int D = L->D, F = L->F, E = L->route.E, K = L->route.K;
    float *logits = (float *)malloc(sizeof(float) * (size_t)E), *score = (float *)malloc(sizeof(float) * (size_t)E);
    float *y = (float *)malloc(sizeof(float) * (size_t)D), *s = (float *)malloc(sizeof(float) * (size_t)D);
    int *ids = (int *)malloc(sizeof(int) * (size_t)K);
    float *w = (float *)malloc(sizeof(float) * (size_t)K);
    if (!L || D <= 0 || F <= 0 || K <= 0 || K > E) return -1;
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * (size_t)D;
        float *o = out + (size_t)t * (size_t)D;
        orc_matmul_rows(ORC_F32, L->router, D, xt, 1, logits, E, 0, E);
        orc_route_select(&L->route, logits, L->router_bias, K, ids, score);
        orc_route_weights(&L->route, score, ids, w);
        if (ids_out) memcpy(ids_out + (size_t)t * K, ids, sizeof(int) * (size_t)K);
        if (wts_out) memcpy(wts_out + (size_t)t * K, w, sizeof(float) * (size_t)K);
        for (int i = 0; i < D; i++) o[i] = 0.0f;
        for (int j = 0; j < K; j++) {
            const int e = ids[j], dt = L->slab_dtype[e];
            size_t ou, od;
            const uint8_t *slab = (const uint8_t *)L->slabs[e];
            orc_slab_layout(dt, D, F, &ou, &od, NULL);
            ffn_one(dt, slab, slab + ou, slab + od, D, F, xt, y);
            for (int i = 0; i < D; i++) {
                const float p = w[j] * y[i];
                o[i] = o[i] + p;
            }
        }
        if (L->Fs > 0) {
            ffn_one(L->sh_dtype, L->sh_gate, L->sh_up, L->sh_down, D, L->Fs, xt, s);
            if (L->sh_gate_inp) {
                const float g = orc_sigmoid(orc_dot16(L->sh_gate_inp, xt, D));
                for (int i = 0; i < D; i++) s[i] = s[i] * g;
            }
            for (int i = 0; i < D; i++) o[i] = o[i] + s[i];
        }
    }
    free(logits); free(score); free(y); free(s); free(ids); free(w);
    return 0;
}

/* docs/NUMERICS.md §5 FFN half of a layer: x = rmsnorm(h, ffn_norm); h = h + rs * moe(x). */
int orc_moe_forward(const orc_moe_layer *layers, int n_layers, float *h, int T) {
    for (int l = 0; l < n_layers; l++) {
        const orc_moe_layer *L = &layers[l];
        const int D = L->D;
        float *x = (float *)malloc(sizeof(float) * (size_t)D * (size_t)T);
        float *o = (float *)malloc(sizeof(float) * (size_t)D * (size_t)T);
        int rc;
        for (int t = 0; t < T; t++) orc_rmsnorm(x + (size_t)t * D, h + (size_t)t * D, L->ffn_norm, D, L->eps);
        rc = orc_moe_layer_eval(L, x, T, o, NULL, NULL);
        if (rc == 0)
            for (size_t i = 0; i < (size_t)D * (size_t)T; i++) {
                const float a = L->residual_scale * o[i];
                h[i] = h[i] + a;
            }
        free(x);
        free(o);
        if (rc) return rc;
    }
    return 0;
}
