/*
 * hx_oracle.h — TEST INFRASTRUCTURE ONLY: the CPU checker for the CUDA backend.
 *
 * A plain-C restatement of Hearth's quantized MoE expert path (pierce-lonergan/hearth,
 * engine/src/quant.c, engine/src/model.c, docs/NUMERICS.md), written from the reference's
 * normative numerics so that the CUDA kernels can be compared with it bit for bit.
 * Only tests, the smoke check and the benchmark's CPU-baseline leg load it; the product
 * (hearth_b200/) never links, loads or calls it.
 *
 * Pinning: orc_matmul reproduces the reference's pinned FNV-1a hashes PIN_Y_F32 .. PIN_Y_Q4
 * (engine/tests/test_quant.c:58-62) on the reference-quantized golden weights in
 * tests/golden/, and the MoE layer is compared with the reference's own kernels driven by
 * moe_ref.c (built from the reference sources into _ref/).
 *
 * Every function is scalar and single-threaded, compiled with -ffp-contract=off (the
 * reference's NUMERICS "no FMA contraction" rule) and calls the host libm expf exactly
 * where the reference does (quant.c:639,647,651).
 */
#ifndef HX_ORACLE_H
#define HX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2, ORC_Q8 = 3, ORC_Q4 = 4 };
enum { ORC_SCORE_SOFTMAX = 0, ORC_SCORE_SIGMOID = 1 };

/* Activation block, engine/src/hx_quant.h:24 (72 bytes). */
typedef struct { float d; int32_t sum; int8_t q[64]; } orc_act_q8;

size_t   orc_row_bytes(int dtype, int64_t n);
size_t   orc_act_bytes(int wdtype, int64_t n);
float    orc_f16(uint16_t h);
uint64_t orc_fnv1a(const void *p, size_t n, uint64_t h);
void     orc_det_fill(float *x, int64_t n, uint64_t seed);
void     orc_expf_batch(const float *x, float *y, int64_t n);

void orc_act_quantize(const float *x, orc_act_q8 *out, int64_t n);
void orc_matmul_rows(int dtype, const void *W, int64_t n_cols, const void *act, int T,
                     float *Y, int64_t ldy, int64_t r0, int64_t r1);
int  orc_matmul(int dtype, const void *W, int64_t n_rows, int64_t n_cols, const float *X, int T, float *Y);
int  orc_dequantize(int dtype, const void *src, int64_t n_rows, int64_t n_cols, float *dst);

float orc_sum16(const float *a, int64_t n);
float orc_dot16(const float *a, const float *b, int64_t n);
void  orc_rmsnorm(float *y, const float *x, const float *w, int64_t n, float eps);
void  orc_softmax(float *x, int64_t n);
void  orc_swiglu(float *out, const float *g, const float *u, int64_t n);
float orc_sigmoid(float x);

typedef struct orc_route_cfg {
    int E, K;
    int score_fn;        /* ORC_SCORE_* */
    int score_bias;      /* 1: selection adds router_bias */
    int n_group, topk_group;
    int norm_topk_prob;
    float routed_scale;
} orc_route_cfg;

void orc_route_select(const orc_route_cfg *c, const float *logits, const float *bias, int kk, int *ids, float *score);
void orc_route_weights(const orc_route_cfg *c, const float *score, const int *ids, float *w);
int  orc_route_union(int E, int K, int T, const int *ids, int *ulist, int *u_p0, int *u_n, int *pair_tok, int *pair_of);

/* FORMAT §5 slab: gate [F,D] at 0, up [F,D] at align64, down [D,F] at align64, size align4096. */
void orc_slab_layout(int dtype, int64_t D, int64_t F, size_t *off_up, size_t *off_down, size_t *nbytes);

typedef struct orc_moe_layer {
    int D, F;
    orc_route_cfg route;
    const float *router;          /* [E, D] f32 */
    const float *router_bias;     /* [E] or NULL */
    const void *const *slabs;     /* [E] expert slabs */
    const int *slab_dtype;        /* [E] dtype of each slab's three matrices */
    int Fs, sh_dtype;             /* shared expert width (0 = none) and dtype */
    const void *sh_gate, *sh_up, *sh_down;
    const float *sh_gate_inp;     /* [D] or NULL */
    const float *ffn_norm;        /* [D], used by orc_moe_forward */
    float eps, residual_scale;
} orc_moe_layer;

/* One MoE FFN on already-normed x [T, D]: out [T, D] = rank-order expert sum (+ shared).
 * ids/wts (optional, [T, K]) receive the routing. Returns 0, or -1 on bad arguments. */
int orc_moe_layer_eval(const orc_moe_layer *L, const float *x, int T, float *out, int *ids, float *wts);
/* Chained: for each layer, x = rmsnorm(h, ffn_norm); h = h + residual_scale * moe(x). */
int orc_moe_forward(const orc_moe_layer *layers, int n_layers, float *h, int T);

#ifdef __cplusplus
}
#endif
#endif
