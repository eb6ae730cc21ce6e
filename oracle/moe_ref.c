/*
 * moe_ref.c — TEST INFRASTRUCTURE ONLY: the timed CPU baseline.
 *
 * Runs the quantized MoE expert path on the host cores with the reference's own compiled
 * kernels (hx_kernels_get(): the AVX-512 VNNI Q4/Q8 matmuls, act_quantize_q8 and the F32
 * dot16 router of engine/src/quant.c / quant_avx512.c), its canonical helpers (hx_rmsnorm,
 * hx_swiglu) and its persistent thread pool (hx_pool_for_n, engine/src/pool.c).
 * The schedule mirrors engine/src/model.c moe_layer (986-1131): router for all tokens,
 * route_select/route_weights per token, union of experts, each expert's gate/up for all its
 * tokens in one parallel region of 16-row chunks (mm_run, model.c:307-339), SwiGLU + mid
 * activation, down, then the rank-order sum (moe_sum_range, model.c:904-923).
 * route_select / route_weights / the union are static in model.c and cannot be linked, so
 * the restatements in hx_oracle.c are used for them (integer work, negligible time).
 *
 * Built only where the reference sources exist (oracle/Makefile -> _ref/libmoe_ref.so).
 */
#include "hx_oracle.h"
#include "hx_pool.h"
#include "hx_quant.h"

#include <stdlib.h>
#include <string.h>

typedef struct moe_ref {
    hx_pool *pool;
    int n_threads;
    const hx_kernels *k;
} moe_ref;

typedef struct mtask {
    hx_matmul_fn fn;
    const void *W;
    int64_t cols, rows;
    const void *act;
    int T;
    float *Y;
    int64_t ldy;
} mtask;

typedef struct mjob {
    const mtask *t;
    const int64_t *start;
    int n;
    int64_t chunk;
} mjob;

static void mjob_range(void *ctx, int64_t b, int64_t e, int tid) {
    const mjob *j = (const mjob *)ctx;
    (void)tid;
    for (int64_t it = b; it < e; it++) {
        int lo = 0, hi = j->n - 1;
        while (lo < hi) {
            const int mid = lo + (hi - lo + 1) / 2;
            if (j->start[mid] <= it) lo = mid; else hi = mid - 1;
        }
        {
            const mtask *k = &j->t[lo];
            const int64_t r0 = (it - j->start[lo]) * j->chunk;
            const int64_t r1 = r0 + j->chunk < k->rows ? r0 + j->chunk : k->rows;
            k->fn(k->W, k->cols, k->act, k->T, k->Y, k->ldy, r0, r1);
        }
    }
}

/* All tasks' rows in chunks of a multiple of 16 rows over the whole pool. */
static void run_tasks(moe_ref *m, const mtask *t, int n) {
    int64_t total = 0, chunk, *start = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n + 1));
    mjob j;
    for (int i = 0; i < n; i++) total += t[i].rows;
    chunk = (total + (int64_t)m->n_threads * 4 - 1) / ((int64_t)m->n_threads * 4);
    chunk = (chunk + 15) & ~(int64_t)15;
    if (chunk < 16) chunk = 16;
    start[0] = 0;
    for (int i = 0; i < n; i++) start[i + 1] = start[i] + (t[i].rows + chunk - 1) / chunk;
    j.t = t; j.start = start; j.n = n; j.chunk = chunk;
    if (start[n] > 0) {
        if (m->n_threads <= 1) mjob_range(&j, 0, start[n], 0);
        else hx_pool_for_n(m->pool, m->n_threads, start[n], 1, mjob_range, &j);
    }
    free(start);
}

moe_ref *moe_ref_open(int n_threads, int isa) {
    moe_ref *m = (moe_ref *)calloc(1, sizeof *m);
    if (!m) return NULL;
    m->n_threads = n_threads > 0 ? n_threads : hx_num_physical_cores();
    m->k = isa ? hx_kernels_for(isa) : hx_kernels_get();
    if (!m->k) { free(m); return NULL; }
    m->pool = hx_pool_create(m->n_threads, 50);
    if (!m->pool) { free(m); return NULL; }
    return m;
}

void moe_ref_close(moe_ref *m) {
    if (!m) return;
    hx_pool_destroy(m->pool);
    free(m);
}

int moe_ref_threads(const moe_ref *m) { return m->n_threads; }
int moe_ref_isa(const moe_ref *m) { return m->k->isa; }

typedef struct swjob {
    const hx_kernels *k;
    float *G;
    const float *U;
    int F;
    uint8_t *mid;
    size_t abm;
} swjob;

static void swjob_range(void *ctx, int64_t b, int64_t e, int tid) {
    const swjob *j = (const swjob *)ctx;
    (void)tid;
    for (int64_t p = b; p < e; p++) {
        float *g = j->G + (size_t)p * (size_t)j->F;
        hx_swiglu(g, g, j->U + (size_t)p * (size_t)j->F, j->F);
        if (j->mid) j->k->act_quantize_q8(g, (hx_act_q8 *)(j->mid + (size_t)p * j->abm), j->F);
    }
}

/* One MoE FFN on normed x [T, D] -> out [T, D] (rank-order sum + shared). Experts must all be
 * Q4 or Q8; the shared expert (if any) uses sh_dtype. Returns 0 or -1. */
int moe_ref_layer(moe_ref *m, const orc_moe_layer *L, const float *x, int T, float *out) {
    const int D = L->D, F = L->F, E = L->route.E, K = L->route.K, P = T * K;
    const size_t ab = hx_act_bytes(HEARTH_Q8, D), abm = hx_act_bytes(HEARTH_Q8, F);
    float *logits = (float *)malloc(sizeof(float) * (size_t)T * E), *score = (float *)malloc(sizeof(float) * E);
    int *ids = (int *)malloc(sizeof(int) * (size_t)P), *ulist = (int *)malloc(sizeof(int) * (size_t)E);
    int *u_p0 = (int *)malloc(sizeof(int) * (size_t)E), *u_n = (int *)malloc(sizeof(int) * (size_t)E);
    int *pair_tok = (int *)malloc(sizeof(int) * (size_t)P), *pair_of = (int *)malloc(sizeof(int) * (size_t)P);
    float *w = (float *)malloc(sizeof(float) * (size_t)P);
    uint8_t *xact = (uint8_t *)hx_aligned_alloc(64, ab * (size_t)T);
    uint8_t *act_in = (uint8_t *)hx_aligned_alloc(64, ab * (size_t)P);
    uint8_t *mid = (uint8_t *)hx_aligned_alloc(64, abm * (size_t)P);
    float *G = (float *)hx_aligned_alloc(64, sizeof(float) * (size_t)P * F);
    float *U = (float *)hx_aligned_alloc(64, sizeof(float) * (size_t)P * F);
    float *Y = (float *)hx_aligned_alloc(64, sizeof(float) * (size_t)P * D);
    mtask *tk = (mtask *)malloc(sizeof(mtask) * (size_t)(3 * E + 3));
    int nu, nt, rc = 0;
    {   /* router (F32 dot16 kernel) and token activations */
        mtask r = {m->k->matmul[HEARTH_F32], L->router, D, E, x, T, logits, E};
        run_tasks(m, &r, 1);
        for (int t = 0; t < T; t++) m->k->act_quantize_q8(x + (size_t)t * D, (hx_act_q8 *)(xact + (size_t)t * ab), D);
    }
    for (int t = 0; t < T; t++) {
        orc_route_select(&L->route, logits + (size_t)t * E, L->router_bias, K, ids + (size_t)t * K, score);
        orc_route_weights(&L->route, score, ids + (size_t)t * K, w + (size_t)t * K);
    }
    nu = orc_route_union(E, K, T, ids, ulist, u_p0, u_n, pair_tok, pair_of);
    for (int u = 0; u < nu; u++)
        if (L->slab_dtype[ulist[u]] != HEARTH_Q4 && L->slab_dtype[ulist[u]] != HEARTH_Q8) rc = -1;
    if (!rc) {
        nt = 0;
        for (int u = 0; u < nu; u++) {
            const int e = ulist[u], dt = L->slab_dtype[e], p0 = u_p0[u], n = u_n[u];
            size_t ou, od;
            const uint8_t *slab = (const uint8_t *)L->slabs[e];
            uint8_t *a = act_in + (size_t)p0 * ab;
            orc_slab_layout(dt, D, F, &ou, &od, NULL);
            for (int i = 0; i < n; i++) memcpy(a + (size_t)i * ab, xact + (size_t)pair_tok[p0 + i] * ab, ab);
            tk[nt++] = (mtask){m->k->matmul[dt], slab, D, F, a, n, G + (size_t)p0 * F, F};
            tk[nt++] = (mtask){m->k->matmul[dt], slab + ou, D, F, a, n, U + (size_t)p0 * F, F};
        }
        run_tasks(m, tk, nt);
        {
            swjob sj = {m->k, G, U, F, mid, abm};
            if (m->n_threads <= 1 || P < 2) swjob_range(&sj, 0, P, 0);
            else hx_pool_for_n(m->pool, m->n_threads, P, 1, swjob_range, &sj);
        }
        nt = 0;
        for (int u = 0; u < nu; u++) {
            const int e = ulist[u], dt = L->slab_dtype[e], p0 = u_p0[u], n = u_n[u];
            size_t od;
            orc_slab_layout(dt, D, F, NULL, &od, NULL);
            tk[nt++] = (mtask){m->k->matmul[dt], (const uint8_t *)L->slabs[e] + od, F, D, mid + (size_t)p0 * abm, n,
                               Y + (size_t)p0 * D, D};
        }
        run_tasks(m, tk, nt);
        for (int t = 0; t < T; t++) {   /* rank-order sum (model.c:904-923) */
            float *o = out + (size_t)t * D;
            for (int i = 0; i < D; i++) o[i] = 0.0f;
            for (int j = 0; j < K; j++) {
                const float wj = w[(size_t)t * K + j];
                const float *y = Y + (size_t)pair_of[(size_t)t * K + j] * D;
                for (int i = 0; i < D; i++) o[i] = o[i] + wj * y[i];
            }
        }
        if (L->Fs > 0) {   /* shared expert (model.c:925-934) */
            const int Fs = L->Fs;
            const size_t abs_ = hx_act_bytes(HEARTH_Q8, Fs);
            float *g = (float *)malloc(sizeof(float) * (size_t)T * Fs), *uu = (float *)malloc(sizeof(float) * (size_t)T * Fs);
            float *s = (float *)malloc(sizeof(float) * (size_t)T * D);
            uint8_t *am = (uint8_t *)hx_aligned_alloc(64, abs_ * (size_t)T);
            mtask st[2] = {{m->k->matmul[L->sh_dtype], L->sh_gate, D, Fs, xact, T, g, Fs},
                           {m->k->matmul[L->sh_dtype], L->sh_up, D, Fs, xact, T, uu, Fs}};
            run_tasks(m, st, 2);
            for (int t = 0; t < T; t++) {
                hx_swiglu(g + (size_t)t * Fs, g + (size_t)t * Fs, uu + (size_t)t * Fs, Fs);
                m->k->act_quantize_q8(g + (size_t)t * Fs, (hx_act_q8 *)(am + (size_t)t * abs_), Fs);
            }
            st[0] = (mtask){m->k->matmul[L->sh_dtype], L->sh_down, Fs, D, am, T, s, D};
            run_tasks(m, st, 1);
            for (int t = 0; t < T; t++) {
                float *o = out + (size_t)t * D, *st_ = s + (size_t)t * D;
                if (L->sh_gate_inp) {
                    const float gg = hx_sigmoid(hx_dot16(L->sh_gate_inp, x + (size_t)t * D, D));
                    for (int i = 0; i < D; i++) st_[i] = st_[i] * gg;
                }
                for (int i = 0; i < D; i++) o[i] = o[i] + st_[i];
            }
            free(g); free(uu); free(s); hx_aligned_free(am);
        }
    }
    free(logits); free(score); free(ids); free(ulist); free(u_p0); free(u_n); free(pair_tok); free(pair_of); free(w);
    hx_aligned_free(xact); hx_aligned_free(act_in); hx_aligned_free(mid);
    hx_aligned_free(G); hx_aligned_free(U); hx_aligned_free(Y);
    free(tk);
    return rc;
}

/* Chained MoE stack: x = rmsnorm(h, ffn_norm_l); h = h + rs * moe_l(x) (NUMERICS §5). */
int moe_ref_forward(moe_ref *m, const orc_moe_layer *layers, int n_layers, float *h, int T) {
    for (int l = 0; l < n_layers; l++) {
        const orc_moe_layer *L = &layers[l];
        const int D = L->D;
        float *x = (float *)hx_aligned_alloc(64, sizeof(float) * (size_t)T * D);
        float *o = (float *)hx_aligned_alloc(64, sizeof(float) * (size_t)T * D);
        int rc;
        for (int t = 0; t < T; t++) hx_rmsnorm(x + (size_t)t * D, h + (size_t)t * D, L->ffn_norm, D, L->eps);
        rc = moe_ref_layer(m, L, x, T, o);
        if (!rc)
            for (size_t i = 0; i < (size_t)T * D; i++) h[i] = h[i] + L->residual_scale * o[i];
        hx_aligned_free(x);
        hx_aligned_free(o);
        if (rc) return rc;
    }
    return 0;
}

/* ---------------------------------------------------------------------------------------------
 * Synthetic weights for the benchmark's CPU leg: byte-identical to the backend's device
 * generator (splitmix64 integer hashing, Irwin-Hall(4) nibbles and scale jitter), so the CPU and
 * GPU legs compute on the same model and their outputs can be compared bit for bit.
 * ------------------------------------------------------------------------------------------- */

static uint64_t smix(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

static uint32_t half_scale_bits(float sigma) {
    const float v = sigma * 0.5f;
    uint32_t fb;
    memcpy(&fb, &v, 4);
    return (uint32_t)(((int)((fb >> 23) & 0xff) - 127 + 15) << 10) | ((fb >> 13) & 0x3ffu);
}

typedef struct synth_job {
    uint8_t *dst;
    int64_t slab_bytes, per_slab, nb_gate;
    size_t off_up, off_down;
    uint64_t seed;
    uint32_t scale_bits;
} synth_job;

static void synth_range(void *ctx, int64_t b0, int64_t b1, int tid) {
    const synth_job *j = (const synth_job *)ctx;
    (void)tid;
    for (int64_t i = b0; i < b1; i++) {
        const int64_t slab = i / j->per_slab, b = i - slab * j->per_slab;
        int64_t off;
        uint8_t *blk;
        uint64_t h = smix(j->seed ^ smix((uint64_t)i));
        uint32_t sc;
        if (b < j->nb_gate) off = b * 34;
        else if (b < 2 * j->nb_gate) off = (int64_t)j->off_up + (b - j->nb_gate) * 34;
        else off = (int64_t)j->off_down + (b - 2 * j->nb_gate) * 34;
        blk = j->dst + slab * j->slab_bytes + off;
        sc = j->scale_bits + (uint32_t)(h & 0x3f) - 32u;
        blk[0] = (uint8_t)(sc & 0xff);
        blk[1] = (uint8_t)(sc >> 8);
        for (int k = 0; k < 32; k++) {
            uint8_t v = 0;
            for (int half = 0; half < 2; half++) {
                int s4, q;
                h = smix(h);
                s4 = (int)(h & 0xff) + (int)((h >> 8) & 0xff) + (int)((h >> 16) & 0xff) + (int)((h >> 24) & 0xff);
                q = 8 + (s4 - 510 + 37 + 740) / 74 - 10;
                q = q < 0 ? 0 : (q > 15 ? 15 : q);
                v |= (uint8_t)(q << (4 * half));
            }
            blk[2 + k] = v;
        }
    }
}

/* Q4 expert slabs [n_slabs][slab_bytes] (padding zeroed). */
int moe_ref_synth_q4(moe_ref *m, uint8_t *dst, int64_t n_slabs, int64_t slab_bytes, int D, int F, uint64_t seed,
                     float sigma) {
    synth_job j;
    size_t ou, od, nb;
    orc_slab_layout(ORC_Q4, D, F, &ou, &od, &nb);
    if ((int64_t)nb > slab_bytes) return -1;
    memset(dst, 0, (size_t)(n_slabs * slab_bytes));
    j.dst = dst;
    j.slab_bytes = slab_bytes;
    j.nb_gate = (int64_t)F * (D / 64);
    j.per_slab = 2 * j.nb_gate + (int64_t)D * (F / 64);
    j.off_up = ou;
    j.off_down = od;
    j.seed = seed;
    j.scale_bits = half_scale_bits(sigma);
    if (m->n_threads <= 1) synth_range(&j, 0, n_slabs * j.per_slab, 0);
    else hx_pool_for_n(m->pool, m->n_threads, n_slabs * j.per_slab, 4096, synth_range, &j);
    return 0;
}

/* A [rows, cols] Q4 or Q8 matrix with the statistics of N(0, sigma) weights, byte-identical to the
 * backend's device generator for shared experts (k_synth_blocks): per 64-weight block a jittered
 * f16 scale (Q4 sigma/2, Q8 sigma/53) and Irwin-Hall(4) values over splitmix64 bytes. */
int moe_ref_synth_blocks(uint8_t *dst, int dtype, int64_t rows, int64_t cols, uint64_t seed, float sigma) {
    if ((dtype != ORC_Q4 && dtype != ORC_Q8) || rows <= 0 || cols <= 0 || cols % 64) return -1;
    const int64_t n = rows * (cols / 64);
    const int q8 = dtype == ORC_Q8;
    const uint32_t scale_bits = half_scale_bits(q8 ? 2.0f * (sigma / 53.0f) : sigma);
    for (int64_t i = 0; i < n; i++) {
        uint8_t *blk = dst + i * (q8 ? 66 : 34);
        uint64_t h = smix(seed ^ smix((uint64_t)i));
        const uint32_t sc = scale_bits + (uint32_t)(h & 0x3f) - 32u;
        blk[0] = (uint8_t)(sc & 0xff);
        blk[1] = (uint8_t)(sc >> 8);
        for (int j = 0; j < (q8 ? 64 : 32); j++) {
            h = smix(h);
            const int s4 = (int)(h & 0xff) + (int)((h >> 8) & 0xff) + (int)((h >> 16) & 0xff) + (int)((h >> 24) & 0xff);
            if (q8) {
                int q = ((s4 - 510) * 9 + (s4 >= 510 ? 12 : -12)) / 25;
                q = q < -127 ? -127 : (q > 127 ? 127 : q);
                blk[2 + j] = (uint8_t)(int8_t)q;
            } else {
                const int s4b = (int)((h >> 32) & 0xff) + (int)((h >> 40) & 0xff) + (int)((h >> 48) & 0xff) +
                                (int)((h >> 56) & 0xff);
                int lo = 8 + (s4 - 510 + 37 + 740) / 74 - 10, hi = 8 + (s4b - 510 + 37 + 740) / 74 - 10;
                lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
                hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
                blk[2 + j] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
    return 0;
}

/* f32 ~ N(0, sigma): (s4 - 510) * (sigma / 147.8f), one rounding. */
void moe_ref_synth_f32(float *dst, int64_t n, uint64_t seed, float sigma) {
    const float k = sigma / 147.8f;
    for (int64_t i = 0; i < n; i++) {
        const uint64_t h = smix(seed ^ smix((uint64_t)i));
        const int s4 = (int)(h & 0xff) + (int)((h >> 8) & 0xff) + (int)((h >> 16) & 0xff) + (int)((h >> 24) & 0xff);
        dst[i] = (float)(s4 - 510) * k;
    }
}
