/*
 * hearth_b200.h — C ABI of the B200 (sm_100a) backend for Hearth's quantized MoE expert path.
 *
 * Plain C types only (pointers, sizes, ints); no CUDA or torch types. Device pointers are
 * passed as void* / float*, CUDA streams as void* (cudaStream_t). A NULL stream means, for the
 * hxb_moe_* calls on a handle, the handle's own non-blocking stream; for the handle-less
 * device-pointer calls (hxb_act_quantize_dev, hxb_matmul_dev, hxb_dequantize_dev, hxb_expf_dev,
 * hxb_matmul_noalloc), which have no stream of their own, CUDA's legacy default stream.
 *
 * The entry points replace these reference interfaces (pierce-lonergan/hearth):
 *   hxb_matmul          hearth_matmul       engine/include/hearth.h:157-158, engine/src/quant.c:574-600
 *   hxb_dequantize      hearth_dequantize   engine/include/hearth.h:153,     engine/src/quant.c:563-571
 *   hxb_row_bytes       hearth_row_bytes    engine/include/hearth.h:150,     engine/src/quant.c:507
 *   hxb_matmul_dev      hx_matmul_fn        engine/src/hx_quant.h:49-57 (row-range kernel contract)
 *   hxb_act_quantize_dev  act_quantize_q8   engine/src/hx_quant.h:62,        engine/src/quant.c:325-348
 *   hxb_moe_*           the MoE half of hx_model (engine/src/model.c:986-1131 moe_layer and the
 *                       FFN half of forward, model.c:1209-1214) plus the expert store it acquires
 *                       experts from (engine/src/hx_store.h:51-89), as a backend handle
 *   hxb_moe_stats       hx_store_stats      engine/src/hx_store.h:78-87 (+ hearth_stats timers)
 *
 * Return codes follow hx_model.h:60-68 (HX_E_*) where one exists.
 * Threading: a handle is used by one host thread at a time (engine/include/hearth.h:10-12).
 */
#ifndef HEARTH_B200_H
#define HEARTH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HXB_API __attribute__((visibility("default")))

enum {
    HXB_OK = 0,
    HXB_E_ARG = -1,          /* HX_E_ARG */
    HXB_E_TOKEN = -2,        /* HX_E_TOKEN: a token id outside [0, vocab_size) */
    HXB_E_CAPACITY = -3,     /* HX_E_CAPACITY: more tokens than the handle was opened for */
    HXB_E_IO = -4,           /* HX_E_IO: an expert could not be brought into HBM */
    HXB_E_NOMEM = -5,        /* HX_E_NOMEM */
    HXB_E_FORMAT = -6,       /* HX_E_FORMAT */
    HXB_E_DEVICE = -7,       /* CUDA error or a kernel's device error word */
    HXB_E_UNSUPPORTED = -8   /* a dtype / shape the kernels do not handle */
};

/* hearth_matmul's own codes (engine/src/quant.c:573): 0 ok, -1 bad args, -2 no device, -3 alloc. */
enum { HXB_MM_OK = 0, HXB_MM_E_ARG = -1, HXB_MM_E_NODEV = -2, HXB_MM_E_ALLOC = -3 };

/* ---- kernel-level boundary ------------------------------------------------------------------ */
HXB_API const char *hxb_version(void);
HXB_API const char *hxb_last_error(void);   /* message of the calling thread's last failure */
HXB_API int hxb_device_count(void);
HXB_API size_t hxb_row_bytes(int dtype, int64_t n_cols);

/* Y[T, n_rows] = W[n_rows, n_cols] . X[T, n_cols] with host buffers, NUMERICS §3 (bit-identical
 * to hearth_matmul on every dtype F32/F16/BF16/Q8/Q4). */
HXB_API int hxb_matmul(int dtype, const void *W, int64_t n_rows, int64_t n_cols, const float *X, int T,
                       float *Y);
HXB_API int hxb_dequantize(int dtype, const void *src, int64_t n_rows, int64_t n_cols, float *dst);

/* Device-pointer variants. act: T activations of n_cols (72-byte blocks for Q8/Q4 weights,
 * f32 vectors for float weights); Y[t * ldy + r] for rows [r0, r1). */
HXB_API int hxb_act_quantize_dev(const float *x, int64_t n, int T, void *act, void *stream);
HXB_API int hxb_matmul_dev(int dtype, const void *W, int64_t n_cols, const void *act, int T, float *Y,
                           int64_t ldy, int64_t r0, int64_t r1, void *stream);
HXB_API int hxb_dequantize_dev(int dtype, const void *W, int64_t n_rows, int64_t n_cols, float *out,
                               void *stream);
/* The device expf (the host libm's results) on the bit patterns [x0, x0 + n): self-check support. */
HXB_API int hxb_expf_dev(uint32_t x0, int64_t n, float *out, void *stream);

/* ---- allocation-free matmul ------------------------------------------------------------------
 * No counterpart in the reference (its hearth_matmul allocates a buffer on every call).
 * For callers that must not allocate device memory when they run a matmul: a serving engine
 * that reserved all of HBM for its own pool up front, code running while a CUDA graph is being
 * captured (cudaMalloc cannot be recorded into a graph), or an application that budgets device
 * memory once at start. W (n_rows rows of dtype), X [T, n_cols] f32 and Y [T, n_rows] f32 are
 * the caller's device buffers; the Q8/Q4 activation scratch is a 4 MiB static device array
 * (T * n_cols / 64 * 72 bytes at most, else HXB_E_CAPACITY with a message), held by every GPU
 * that loads the library until exit. The first call on a device looks up that array's address,
 * so make it before any stream capture. All calls share the array: calls that overlap on the
 * GPU race and must be serialised by the caller. Results equal hxb_matmul's bit for bit. The
 * work is enqueued on `stream` (NULL: the legacy default stream) and the call returns without
 * waiting for it. */
#define HXB_NOALLOC_SCRATCH_BYTES ((size_t)4 << 20)
HXB_API int hxb_matmul_noalloc(int dtype, const void *W, int64_t n_rows, int64_t n_cols, const float *X, int T,
                               float *Y, void *stream);

/* ---- MoE backend handle ---------------------------------------------------------------------- */
typedef struct hxb_moe hxb_moe;

typedef struct hxb_moe_config {
    int n_layers;          /* MoE layers held by this handle */
    int d_model;           /* D */
    int expert_ffn_dim;    /* F */
    int n_experts;         /* E (<= 384) */
    int top_k;             /* K (<= 32) */
    int score_fn;          /* 0 softmax, 1 sigmoid (HX_SCORE_*) */
    int score_bias;        /* 1: selection adds the router bias */
    int n_group, topk_group;
    int norm_topk_prob;
    float routed_scale, residual_scale, norm_eps;
    int expert_dtype;      /* HEARTH_Q4 or HEARTH_Q8 */
    int shared_ffn_dim;    /* 0 = no shared expert */
    int shared_dtype;      /* HEARTH_Q8 or HEARTH_Q4 */
    int shared_gate;       /* 1: shared output scaled by sigmoid(dot16(gate_inp, x)) */
    int max_tokens;        /* largest T per call */
    double cache_gb;       /* HBM budget for expert slots in GiB; 0 = every expert resident */
    int policy;            /* HEARTH_POLICY_LRU (0) / HEARTH_POLICY_LFU (1) */
    float heat_decay;      /* LFU per-token decay (default 0.995) */
    int device;            /* CUDA device ordinal */
    int ep_size, ep_rank;  /* expert parallelism: this handle holds and computes the experts e with
                              e % ep_size == ep_rank (default 1, 0: every expert) */
    int prefetch_next;     /* streaming store (cache_gb below the model): after routing layer l, route
                              layer l+1 with layer l's input (its ffn_norm and router) and hand the
                              predicted experts to the store as prefetch hints, so their copies run
                              while layer l computes (HEARTH_PREFETCH_NEXT, engine/src/model.c:944-973).
                              Default 1; 0 = demand copies only. */
} hxb_moe_config;

typedef struct hxb_moe_stats {
    uint64_t tokens, forward_calls;
    uint64_t expert_uses, expert_loads_unique;
    uint64_t hits, misses, evictions;
    uint64_t prefetch_issued, prefetch_used, prefetch_wasted;
    uint64_t bytes_copied, copies, copy_errors;
    int n_slots, resident, pinned;
    uint64_t slot_bytes;
    double wall_s, stall_s;
    uint64_t host_bytes;   /* pinned host bytes of the store's host tier (shared sources counted once) */
} hxb_moe_stats;

HXB_API void hxb_moe_default_config(hxb_moe_config *c);
HXB_API hxb_moe *hxb_moe_open(const hxb_moe_config *c, char *err, size_t errlen);
HXB_API void hxb_moe_close(hxb_moe *m);

/* Dense per-layer weights (host buffers, copied to HBM): router [E, D] f32, router_bias [E] or
 * NULL, ffn_norm [D] or NULL (then the input is used as given), shared expert gate/up [Fs, D],
 * down [D, Fs] in shared_dtype and gate_inp [D] (all NULL without a shared expert). */
HXB_API int hxb_moe_set_layer(hxb_moe *m, int layer, const float *router, const float *router_bias,
                              const float *ffn_norm, const void *sh_gate, const void *sh_up, const void *sh_down,
                              const float *sh_gate_inp);
/* One routed expert's slab (docs/FORMAT.md §5 layout, nbytes = the slab size) from host memory.
 * The store keeps a pinned host copy (the host tier) and moves it into HBM when needed. */
HXB_API int hxb_moe_set_expert(hxb_moe *m, int layer, int expert, const void *slab, size_t nbytes);
/* The bytes of one expert's slab as the handle holds them in HBM (every expert resident; nbytes >= the
 * slab size), e.g. to hand a synthesized stack to a streaming handle. No counterpart in the
 * reference (its slabs are read from the container file). */
HXB_API int hxb_moe_get_expert(hxb_moe *m, int layer, int expert, void *dst, size_t nbytes);
/* Benchmarks without a container: deterministic synthetic router (N(0, sigma_router)), selection
 * bias (N(0, sigma_router / 2), score_bias handles), unit norms, Q4 expert slabs and the Q4/Q8
 * shared expert (with its gate input) for every layer, generated in HBM. A handle whose HBM budget
 * holds every expert keeps them resident; a smaller budget gets the same bytes in the store's pinned
 * host tier (each slab generated on the device and copied out), streamed like a container's.
 * With expert parallelism each rank generates only the slabs it owns, byte for byte the slabs of
 * the same seed on one GPU. */
HXB_API int hxb_moe_synthesize(hxb_moe *m, uint64_t seed, float sigma_router, float sigma_expert);
HXB_API size_t hxb_moe_slab_bytes(const hxb_moe *m);
/* Expert (layer, expert) uses the slab of (src_layer, src_expert), which must already be set: the
 * pinned host copy is shared, not duplicated (a .hearth entry with the aliased flag names another
 * entry's slab, FORMAT §5); the expert keeps its own HBM slot and store counters. Setting either
 * expert again later gives both the new bytes. */
HXB_API int hxb_moe_share_expert(hxb_moe *m, int layer, int expert, int src_layer, int src_expert);

/* ---- .hearth containers (docs/FORMAT.md of the reference; the reference reads them in
 * engine/src/modelfile.c and builds its model from them in hx_model_open, engine/src/model.c:1651).
 * hxb_container_probe reads and validates a container (preamble, metadata, tensor and expert
 * directories, alignment, sizes, aliases, no overlaps; host only, no device work) and fills a
 * configuration for it: hxb_moe_default_config values plus the container's MoE shape and routing
 * (n_layers = the container's layers: one handle slot per layer, dense layers stay unset). The
 * caller then sets max_tokens, cache_gb, policy, device, ep_size / ep_rank and opens the handle.
 * Returns HXB_E_IO for a file that cannot be read, HXB_E_FORMAT (message in err) for one that breaks
 * the format's rules. */
typedef struct hxb_container_info {
    int n_layers;            /* transformer blocks in the file */
    int n_moe_layers;        /* of them MoE (layer_kind 1) */
    int n_expert_entries;    /* n_layers * n_experts */
    int n_physical_slabs;    /* distinct slabs among the MoE layers' entries */
    int n_aliased;           /* entries that share another entry's slab (synthetic benchmark files) */
    int expert_dtype;        /* dtype of every slab, -1 when the slabs mix dtypes */
    uint64_t slab_bytes;     /* bytes of one slab */
} hxb_container_info;
HXB_API int hxb_container_probe(const char *path, hxb_moe_config *cfg, hxb_container_info *info, char *err,
                                size_t errlen);
/* Loads a container's MoE weights into a handle opened with a configuration from
 * hxb_container_probe: per MoE layer hxb_moe_set_layer (moe_router, moe_router_bias, ffn_norm,
 * shexp_gate/up/down, shexp_gate_inp), then hxb_moe_set_expert for every expert this handle holds.
 * Each physical slab is read once; the entries that name it share one pinned host copy. HXB_E_ARG if the handle
 * and the container disagree on the shape or routing, HXB_E_UNSUPPORTED for slabs that are not all
 * Q4 or all Q8 or a shexp_gate_inp that is not F32, HXB_E_FORMAT / HXB_E_IO as above. */
HXB_API int hxb_moe_load_container(hxb_moe *m, const char *path);

/* h[T, D] (host, in place): for l in [layer0, layer0 + n_layers): x = rmsnorm(h, ffn_norm_l);
 * h = h + residual_scale * moe_l(x)   (docs/NUMERICS.md §5, the FFN half of each layer). */
HXB_API int hxb_moe_forward(hxb_moe *m, float *h, int T, int layer0, int n_layers);
HXB_API int hxb_moe_forward_dev(hxb_moe *m, float *h, int T, int layer0, int n_layers, void *stream);
/* Route replay (hearth_route_replay, engine/include/hearth.h:144-147; engine/src/model.c:1003-1009):
 * like hxb_moe_forward, but every token's K expert ids of every layer come from the caller (ids
 * [n_layers][T][K], host, each in [0, n_experts)) instead of the selection; scores and weights are
 * computed as usual. Synchronous; used to measure throughput under a recorded routing skew. */
HXB_API int hxb_moe_forward_routed(hxb_moe *m, float *h, int T, int layer0, int n_layers, const int *ids);
/* One MoE FFN on x[T, D] as given (no norm, no residual): out[T, D] = rank-order expert sum
 * (+ shared expert). Host and device variants. */
HXB_API int hxb_moe_layer(hxb_moe *m, int layer, const float *x, int T, float *out);
HXB_API int hxb_moe_layer_dev(hxb_moe *m, int layer, const float *x, int T, float *out, void *stream);
/* The *_dev calls are asynchronous on their stream; this waits for the stream and returns the
 * status of the device work since the last check (HXB_E_IO if an expert was not resident,
 * HXB_E_DEVICE if a bounded device wait gave up). */
HXB_API int hxb_moe_sync(hxb_moe *m, void *stream);
/* Average device time in microseconds of each kernel stage of one layer at T tokens (every
 * expert resident; eager launches between CUDA events): us[0] rmsnorm + activations, us[1]
 * router + routing, us[2] gate/up + SwiGLU + mid activations, us[3] down + rank-order sum. */
HXB_API int hxb_moe_profile(hxb_moe *m, int T, int iters, double *us);
/* Phase timeline of the last single-token persistent launch, for handles opened with the
 * environment variable HXB_TRACE=1: out[layer][cta][stamp] SM clock cycles of thread 0 (per-SM
 * counter: compare stamps of one CTA only). 21 stamps per layer, in order: start, h polled, rmsnorm
 * chain, router rows in, x, logit stored, activation blocks, predicted-logit partial, logits polled,
 * routed, routing barrier, first gate/up chunk landed, its SwiGLU values stored, exchange reset, mid
 * polled, mid blocks, down rows landed, down rows computed, y stored, y polled, h stored. Returns the
 * number of values (call with out = NULL to size the buffer), 0 when not tracing. */
HXB_API int64_t hxb_moe_phase_trace(hxb_moe *m, uint64_t *out, int64_t max_values);
/* Expert parallelism over ep_size handles (one per GPU, each holding its own experts), one MoE layer
 * in two steps around an exchange the caller makes (an all-gather over NCCL, for example):
 * 1. hxb_moe_ep_layer_dev: x = rmsnorm(h, ffn_norm), router, routing of the T tokens (identical on
 *    every rank), and the outputs of the (token, rank) pairs whose expert this handle owns, written
 *    to y [T*K, D] at the pair's index in the routing's expert-ascending bucket order (the same on
 *    every rank); rows of other ranks' pairs are left as they are. The shared expert, if any, is
 *    computed on every rank.
 * 2. hxb_moe_ep_combine_dev: with y_all [ep_size][T*K][D] holding every rank's y, h += residual_scale
 *    * (rank-order sum of w_j * y_all[owner of expert][pair] + shared output): the single-GPU result
 *    bit for bit. It uses the routing of step 1, so no other call on the handle may come between.
 * Device buffers, asynchronous on `stream`; every owned expert of the layer must be in HBM
 * (HXB_E_IO otherwise). No counterpart in the reference (one process, one CPU). */
HXB_API int hxb_moe_ep_layer_dev(hxb_moe *m, int layer, const float *h, int T, float *y, void *stream);
HXB_API int hxb_moe_ep_combine_dev(hxb_moe *m, int layer, const float *y_all, int T, float *h, void *stream);
/* Expert parallelism in the persistent single-token kernel (every GPU launches one kernel per token,
 * each computes the rank-order terms of the experts it owns and stores their y rows straight into
 * every GPU's memory over NVLink): each rank exports its y-word buffer with hxb_moe_ep_ipc_handle
 * (64 bytes), the ranks exchange the handles (an all-gather over any channel), and each passes all of
 * them, in rank order, to hxb_moe_ep_connect. From then on hxb_moe_forward / hxb_moe_forward_dev with
 * T = 1 on every rank, in the same order and with the same h, give every rank the single-GPU h bit
 * for bit. All ranks must launch the same number of tokens (each launch waits for the other ranks'
 * words of the same launch). No counterpart in the reference (one process, one CPU). */
HXB_API int hxb_moe_ep_ipc_handle(hxb_moe *m, void *handle);
HXB_API int hxb_moe_ep_connect(hxb_moe *m, const void *handles);
/* Which kernel evaluates a single-token forward over every layer (every expert resident):
 * 0 per-phase kernels (one launch per phase and layer), 1 the persistent decode kernel (one launch
 * for all layers). Chosen at open from the shape; the environment variable HXB_PERSISTENT=0 forces
 * 0. No counterpart in the reference (one CPU path). */
HXB_API int hxb_moe_decode_path(const hxb_moe *m);
/* Routing of the last evaluated layer: ids / weights [T, K] (host). */
HXB_API int hxb_moe_last_routing(hxb_moe *m, int *ids, float *weights, int T);

HXB_API int hxb_moe_get_stats(hxb_moe *m, hxb_moe_stats *out);
HXB_API void hxb_moe_reset_stats(hxb_moe *m);
HXB_API int hxb_moe_is_resident(hxb_moe *m, int layer, int expert);
/* Token boundary for the store (heat clock, prefetch protection): hx_store_tick
 * (engine/src/hx_store.h:70). */
HXB_API void hxb_moe_tick(hxb_moe *m);
/* Low-priority hints (hx_store_prefetch, engine/src/hx_store.h:67-69): copies start at once into
 * free or cold unprotected slots, and are dropped otherwise. */
HXB_API int hxb_moe_prefetch(hxb_moe *m, int layer, const int *experts, int n);
/* Heat profile (FORMAT.md §8 counts, n_keys = n_layers * n_experts): pins the hottest
 * pin_fraction of the slots and, with warm_start, fills the rest (engine/src/store.c:815-860). */
HXB_API int hxb_moe_seed_heat(hxb_moe *m, const float *counts, int n_keys, float pin_fraction, int warm_start);
/* Test seam (the counterpart of hx_store_set_read_hook, engine/src/store.c:614-622): called
 * before every host->HBM expert copy; a nonzero return fails that copy. NULL removes it. */
typedef int (*hxb_copy_hook)(void *ctx, int layer, int expert);
HXB_API void hxb_moe_set_copy_hook(hxb_moe *m, hxb_copy_hook fn, void *ctx);

/* ---- the whole decoder on the GPU -----------------------------------------------------------
 * forward() of engine/src/model.c:1171-1236 for GQA / MHA containers (attn_kind 0; MLA containers
 * are refused with HXB_E_UNSUPPORTED): the embedding row times emb_scale; per layer
 * x = rmsnorm(h, attn_norm), q/k/v projections (+ biases), qk-norm per head or full width, RoPE
 * (cos/sin tables computed on the host with its libm, as rope_tables, model.c:386-397), the (k, v)
 * rows appended to an f32 KV cache [layer][kv head][position][head_dim] in HBM, attention per head
 * (dot16 scores times attn_scale, softmax, the value sum in position order; model.c:484-629),
 * the o projection, h += residual_scale * out; then x = rmsnorm(h, ffn_norm) and the MoE layer (the
 * hxb_moe path above: routing, experts, rank-order sum) or the dense SwiGLU FFN (model.c:444-460,
 * 1133-1143), h += residual_scale * out; finally rmsnorm(h, out_norm), the LM head and logit_scale.
 * Every value follows the canonical order of docs/NUMERICS.md, so the logits equal hearth_eval's bit
 * for bit on the same host. Dense matrices may be F32, F16, BF16, Q8 or Q4; experts Q4 or Q8. */
typedef struct hxb_model hxb_model;
typedef struct hxb_model_options {
    int device;        /* CUDA device ordinal */
    int max_batch;     /* tokens per forward call (0: 512) */
    int max_seq;       /* KV cache positions (0: the container's max_seq) */
    double cache_gb;   /* HBM budget for expert slots in GiB (0: every expert resident) */
    int policy;        /* expert store policy (HEARTH_POLICY_LRU / LFU) */
} hxb_model_options;
HXB_API void hxb_model_default_options(hxb_model_options *o);
/* Opens the container at path: every dense tensor and expert slab goes to HBM (experts through the
 * store, as hxb_moe_load_container). NULL with a message in err on failure. */
HXB_API hxb_model *hxb_model_open(const char *path, const hxb_model_options *o, char *err, size_t errlen);
HXB_API void hxb_model_close(hxb_model *m);
/* n_layers, d_model, vocab_size, KV positions, MoE layers, top_k (any pointer may be NULL). */
HXB_API int hxb_model_info(const hxb_model *m, int *n_layers, int *d_model, int *vocab, int *max_seq,
                           int *n_moe_layers, int *top_k);
/* forward(m, tok, T, pos0, logits, mode) (model.c:1171): T tokens (host ids) at positions
 * pos0 .. pos0+T-1, their (k, v) rows written into the cache; mode 0 no logits, 1 the last token's
 * logits[V], 2 every token's logits[T][V] (host). HXB_E_TOKEN for an id outside the vocabulary,
 * HXB_E_CAPACITY beyond max_batch or max_seq. Synchronous. */
HXB_API int hxb_model_forward(hxb_model *m, const int32_t *tokens, int T, int pos0, float *logits, int mode);
/* forward() on device buffers, asynchronous on stream (NULL: the handle's own stream): tokens [T]
 * (device ids; an id outside the vocabulary gives a NaN embedding row instead of HXB_E_TOKEN),
 * logits [1 or T][V] (device, or NULL for mode 0). Every expert must be resident. A single-token
 * forward replays a CUDA graph of the whole decoder after its first use. Errors of the device work
 * (the MoE layers' error word) are reported by hxb_model_sync. */
HXB_API int hxb_model_forward_dev(hxb_model *m, const int32_t *tokens, int T, int pos0, float *logits, int mode,
                                  void *stream);
HXB_API int hxb_model_sync(hxb_model *m, void *stream);
/* The last forward's routing in the layout of model.c's routes[] (the FORMAT §9 trace rows): per
 * token, MoE layer by MoE layer, the K expert ids in rank order: routes[T][n_moe_layers * K]. */
HXB_API int hxb_model_last_routes(hxb_model *m, uint16_t *routes, int T);
/* Route replay (hearth_route_replay, model.c:1003-1009): the MoE layers of later forwards take the
 * ids of row (pos mod n_rows) of rows[n_rows][n_moe_layers * K] instead of their own selection (the
 * scores and weights computed as usual). rows NULL stops the replay. */
HXB_API int hxb_model_set_replay(hxb_model *m, const uint16_t *rows, int n_rows);
/* The MoE backend handle inside (statistics, store control); owned by the model. */
HXB_API hxb_moe *hxb_model_moe(hxb_model *m);
/* Benchmarks without a container: a decoder whose every layer is MoE, generated in HBM from seed.
 * Attention, embedding and LM head matrices in dense_dtype (Q8 or Q4) with the statistics of
 * N(0, sigma_dense) weights (the embedding N(0, 1)), unit norms, RoPE over the whole head with
 * inv_freq[j] = rope_theta^(-2j / head_dim); the MoE layers as hxb_moe_synthesize(seed). No
 * counterpart in the reference (its synthetic models are containers written by synth.py). */
typedef struct hxb_model_arch {
    int vocab_size, n_heads, n_kv_heads, head_dim;
    int qk_norm;            /* 0 none, 1 per head, 2 full width */
    float rope_theta;
    int dense_dtype;        /* HEARTH_Q8 or HEARTH_Q4 */
    float sigma_dense;
    hxb_moe_config moe;     /* the MoE layers: n_layers, d_model, routing, experts (every expert resident) */
} hxb_model_arch;
HXB_API hxb_model *hxb_model_synthesize(const hxb_model_arch *a, const hxb_model_options *o, uint64_t seed,
                                        char *err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif /* HEARTH_B200_H */
