/*
 * hearth_cuda_backend.c — the reference-side binding of the B200 MoE backend: what a maintainer of
 * the reference engine adds so that its public C API (engine/include/hearth.h, hearth_open /
 * hearth_eval) evaluates the MoE half of every layer on the GPU, and the Python toolkit that binds
 * that API (python/hearth/_native.py, engine.py) drives the GPU unchanged.
 *
 * It is compiled as part of the reference's engine/src/model.c: oracle/Makefile makes a build copy
 * of model.c with four anchored edits (the copy lives under oracle/_ref/, nothing is committed):
 *   1. `#include "hearth_cuda_backend.c"` just before forward() (after moe_layer(), model.c:986);
 *   2. forward() (model.c:1171) is renamed forward_cpu(); the forward() below takes its place;
 *   3. forward_cpu()'s `rc = moe_layer(m, w, l, T, pos0);` (model.c:1204) becomes hxc_moe_layer(...);
 *   4. hx_model_close() (model.c:1638) first calls hxc_close(m).
 *
 * Selection: the environment variable HEARTH_BACKEND=cuda, read when a model is first evaluated
 * (the same place the reference reads its other environment overrides is api.c:118-128; reading it
 * lazily keeps hearth_open and its options untouched). Then:
 *   - GQA / MHA containers: the whole forward() — embedding, every layer's attention with its KV
 *     cache, MoE or dense FFN, the output norm, the LM head — runs on the handle's GPU
 *     (hxb_model_forward), bit-identical to forward_cpu() (the backend's parity tests);
 *   - MLA containers, or HEARTH_CUDA_SCOPE=moe: only the MoE layer of forward() — x = rmsnorm(h,
 *     ffn_norm), router, routing, experts, rank-order sum, h += residual_scale * sum (model.c:1209-1214
 *     with moe_layer) — runs on the GPU (hxb_moe_forward); attention, the dense layers and the LM
 *     head stay on the CPU.
 * There is no CPU fallback: when the backend was asked for and cannot be opened (no device, a
 * container it cannot take) every evaluation fails with HX_E_IO, and the log says why.
 *   HEARTH_CUDA_DEVICE   CUDA device ordinal (default 0)
 *   HEARTH_CUDA_CACHE_GB HBM budget for expert slots in GiB (default 0: every expert resident)
 *   HEARTH_CUDA_SCOPE    "moe": the MoE layers only (default: the whole forward where supported)
 * Routing trace rows (hearth_trace_start, docs/FORMAT.md §9) are filled from the GPU routing; with a
 * route replay (hearth_route_replay) the replayed rows go to the GPU, the way moe_layer takes them
 * (model.c:1003-1009: row (pos + i) mod rows, the layer's K ids).
 */
#include "hearth_b200.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define HXC_MAX_MODELS 64
enum { HXC_UNSET = 0, HXC_CUDA = 1, HXC_CPU = 2, HXC_FULL = 3, HXC_FAILED = -1 };

typedef struct hxc_slot {
    hx_model *m;
    hxb_moe *b;        /* HXC_CUDA: the MoE layers' handle */
    hxb_model *full;   /* HXC_FULL: the whole decoder's handle */
    const uint16_t *replay;
    int replay_rows;
    int state;
} hxc_slot;

static hxc_slot hxc_slots[HXC_MAX_MODELS];
static pthread_mutex_t hxc_mu = PTHREAD_MUTEX_INITIALIZER;

static hxc_slot *hxc_slot_of(hx_model *m, int create) {
    hxc_slot *s = NULL;
    pthread_mutex_lock(&hxc_mu);
    for (int i = 0; i < HXC_MAX_MODELS && !s; i++)
        if (hxc_slots[i].m == m) s = &hxc_slots[i];
    for (int i = 0; i < HXC_MAX_MODELS && !s && create; i++)
        if (!hxc_slots[i].m) {
            s = &hxc_slots[i];
            s->m = m;
            s->b = NULL;
            s->full = NULL;
            s->replay = NULL;
            s->replay_rows = 0;
            s->state = HXC_UNSET;
        }
    pthread_mutex_unlock(&hxc_mu);
    return s;
}

/* Opens the backend handle of model m from its own container: the container's MoE shape and
 * routing, every MoE layer's router / bias / norm / shared expert and every expert slab. */
static int hxc_open(hxc_slot *s, hx_model *m) {
    hxb_moe_config cfg;
    hxb_container_info info;
    char err[512];
    const char *dev = getenv("HEARTH_CUDA_DEVICE"), *gb = getenv("HEARTH_CUDA_CACHE_GB");
    if (hxb_container_probe(m->mf->path, &cfg, &info, err, sizeof err) != HXB_OK) {
        hx_log(HX_LOG_ERROR, "cuda backend: %s", err);
        return HX_E_IO;
    }
    cfg.max_tokens = m->max_batch;
    cfg.device = dev && *dev ? atoi(dev) : 0;
    cfg.cache_gb = gb && *gb ? atof(gb) : 0.0;
    s->b = hxb_moe_open(&cfg, err, sizeof err);
    if (!s->b) {
        hx_log(HX_LOG_ERROR, "cuda backend: %s", err);
        return HX_E_IO;
    }
    if (hxb_moe_load_container(s->b, m->mf->path) != HXB_OK) {
        hx_log(HX_LOG_ERROR, "cuda backend: %s", hxb_last_error());
        hxb_moe_close(s->b);
        s->b = NULL;
        return HX_E_IO;
    }
    hx_log(HX_LOG_INFO, "cuda backend: MoE layers of %s on device %d (%s)", m->mf->path, cfg.device,
           hxb_moe_decode_path(s->b) ? "persistent decode kernel" : "per-phase kernels");
    return HX_OK;
}

/* Opens the whole-decoder handle of model m (GQA / MHA containers). */
static int hxc_open_full(hxc_slot *s, hx_model *m) {
    hxb_model_options o;
    char err[512];
    const char *dev = getenv("HEARTH_CUDA_DEVICE"), *gb = getenv("HEARTH_CUDA_CACHE_GB");
    hxb_model_default_options(&o);
    o.device = dev && *dev ? atoi(dev) : 0;
    o.cache_gb = gb && *gb ? atof(gb) : 0.0;
    o.max_batch = m->max_batch;
    o.max_seq = m->cap;
    s->full = hxb_model_open(m->mf->path, &o, err, sizeof err);
    if (!s->full) {
        hx_log(HX_LOG_ERROR, "cuda backend: %s", err);
        return HX_E_IO;
    }
    hx_log(HX_LOG_INFO, "cuda backend: the whole forward of %s on device %d", m->mf->path, o.device);
    return HX_OK;
}

/* The slot of model m with its backend decided (on the first evaluation). */
static hxc_slot *hxc_state(hx_model *m) {
    hxc_slot *s = hxc_slot_of(m, 1);
    if (!s) {
        hx_log(HX_LOG_ERROR, "cuda backend: more than %d open models", HXC_MAX_MODELS);
        return NULL;
    }
    if (s->state == HXC_UNSET) {
        const char *b = getenv("HEARTH_BACKEND"), *scope = getenv("HEARTH_CUDA_SCOPE");
        if (!(b && strcmp(b, "cuda") == 0)) s->state = HXC_CPU;
        else if (!m->mla && !(scope && strcmp(scope, "moe") == 0))
            s->state = hxc_open_full(s, m) == HX_OK ? HXC_FULL : HXC_FAILED;
        else s->state = hxc_open(s, m) == HX_OK ? HXC_CUDA : HXC_FAILED;
    }
    return s;
}

static int hxc_rc(int rc) {
    return rc == HXB_E_CAPACITY ? HX_E_CAPACITY : rc == HXB_E_NOMEM ? HX_E_NOMEM : rc == HXB_E_TOKEN ? HX_E_TOKEN
                                                                                                     : HX_E_IO;
}

static int forward_cpu(hx_model *m, const int32_t *tok, int T, int pos0, float *logits, int mode);

/* forward() (model.c:1171): the whole decoder on the GPU when the backend holds it, else the
 * reference's forward (whose MoE layers may still run on the GPU, hxc_moe_layer). The bookkeeping
 * of the reference's forward follows: counters, the call's routing trace rows, the store's ticks. */
static int forward(hx_model *m, const int32_t *tok, int T, int pos0, float *logits, int mode) {
    hxc_slot *s = hxc_state(m);
    if (!s) return HX_E_NOMEM;
    if (s->state != HXC_FULL) {
        if (s->state == HXC_FAILED) return HX_E_IO;
        return forward_cpu(m, tok, T, pos0, logits, mode);
    }
    if (m->replay != s->replay || m->replay_rows != s->replay_rows) {   /* hearth_route_replay changed it */
        if (hxb_model_set_replay(s->full, m->replay, (int)m->replay_rows) != HXB_OK) {
            hx_log(HX_LOG_ERROR, "cuda backend: route replay: %s", hxb_last_error());
            return HX_E_ARG;
        }
        s->replay = m->replay;
        s->replay_rows = (int)m->replay_rows;
    }
    const uint64_t t0 = hx_now_ns();
    const int rc = hxb_model_forward(s->full, tok, T, pos0, logits, mode);
    if (rc != HXB_OK) {
        hx_log(HX_LOG_ERROR, "cuda backend: forward: %s", hxb_last_error());
        return hxc_rc(rc);
    }
    if (m->n_moe && hxb_model_last_routes(s->full, m->routes, T) != HXB_OK) return HX_E_IO;
    m->st.dense_ns += hx_now_ns() - t0;
    m->st.forward_calls++;
    m->st.tokens += (uint64_t)T;
    m->st.expert_uses += (uint64_t)T * (uint64_t)m->n_moe * (uint64_t)m->K;
    if (m->trace && m->n_moe) trace_rows(m, T);
    for (int t = 0; t < T; t++) hx_store_tick(m->store);
    return HX_OK;
}

/* forward_cpu()'s MoE layer: on the GPU when HEARTH_BACKEND=cuda, else the reference's moe_layer. */
static int hxc_moe_layer(hx_model *m, const layer_w *w, int l, int T, int pos0) {
    hxc_slot *s = hxc_state(m);
    if (!s) return HX_E_NOMEM;
    if (s->state == HXC_CPU) return moe_layer(m, w, l, T, pos0);
    if (s->state != HXC_CUDA) return HX_E_IO;
    const int K = m->K, mi = m->moe_index[l];
    int rc;
    if (m->replay) {   /* the trace's ids for these tokens and this MoE layer */
        for (int i = 0; i < T; i++) {
            const uint16_t *row =
                m->replay + (size_t)((pos0 + i) % m->replay_rows) * (size_t)(m->n_moe * K) + (size_t)mi * K;
            for (int j = 0; j < K; j++) m->ids[(size_t)i * K + j] = row[j];
        }
        rc = hxb_moe_forward_routed(s->b, m->h, T, l, 1, m->ids);
    } else {
        rc = hxb_moe_forward(s->b, m->h, T, l, 1);   /* leaves m->h untouched on failure */
    }
    if (rc != HXB_OK) {
        hx_log(HX_LOG_ERROR, "cuda backend: layer %d: %s", l, hxb_last_error());
        return rc == HXB_E_CAPACITY ? HX_E_CAPACITY : rc == HXB_E_NOMEM ? HX_E_NOMEM : HX_E_IO;
    }
    /* routing of this layer into the per-token trace rows (model.c moe_layer, routes[]) */
    if (m->replay || hxb_moe_last_routing(s->b, m->ids, m->wts, T) == HXB_OK)
        for (int i = 0; i < T; i++)
            for (int j = 0; j < K; j++)
                m->routes[(size_t)i * (m->n_moe * K) + (size_t)mi * K + j] = (uint16_t)m->ids[(size_t)i * K + j];
    m->st.expert_uses += (uint64_t)T * (uint64_t)K;
    (void)w;
    return HX_OK;
}

/* hx_model_close(): the backend handle goes with its model. */
static void hxc_close(hx_model *m) {
    if (!m) return;
    hxc_slot *s = hxc_slot_of(m, 0);
    if (!s) return;
    if (s->b) hxb_moe_close(s->b);
    if (s->full) hxb_model_close(s->full);
    pthread_mutex_lock(&hxc_mu);
    s->b = NULL;
    s->full = NULL;
    s->state = HXC_UNSET;
    s->m = NULL;
    pthread_mutex_unlock(&hxc_mu);
}
