// hx_kernels.h — launch interface of the sm_100a kernels (host side, C++).
//
// Kernel inventory (all in hx_kernels.cu):
//   act_quantize      NUMERICS §2 activation blocks           (engine/src/quant.c:325-348)
//   matmul            hearth_matmul rows for F32/F16/BF16/Q8/Q4 (quant.c:352-427, 574-600)
//   dequantize        hearth_dequantize                         (quant.c:257-307)
//   moe_norm_act      x = rmsnorm(h, ffn_norm), its Q8 activations (model.c:1209-1210, 1050)
//   moe_router        F32 router + shared-gate logits; the last CTA routes small batches
//                     (route_select/route_weights model.c:793-843, union model.c:1020-1037)
//   route_select      one warp per token (large batches)
//   route_union       expert buckets (large batches)
//   moe_gateup        Q4/Q8 gate+up rows, SwiGLU, mid activation blocks (model.c:847-897, 419-439)
//   moe_down          Q4/Q8 down rows; for small batches also the rank-order sum + shared expert +
//                     residual (model.c:904-923)
//   moe_sum           rank-order sum for large batches
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <cuda_runtime.h>

namespace hx {

struct act_q8;

// Routing configuration of one MoE layer (hx_config fields, engine/src/hx_modelfile.h:39-40).
struct RouteCfg {
    int E, K;
    int score_fn, score_bias, n_group, topk_group, norm_topk_prob;
    float routed_scale;
};

// Device scratch of one MoE evaluation (sized for max_tokens by the engine).
struct MoeScratch {
    float *x;            // [T, D] normed input
    act_q8 *xact;        // [T, D/64]
    float *logits;       // [T, E]
    float *sh_logit;     // [T] shared-expert gate logit
    int *ids;            // [T, K]
    float *wts;          // [T, K]
    int *nu;             // [1] unique experts
    int *ulist, *u_p0, *u_n;   // [E]
    int *pair_tok, *pair_of;   // [T*K]
    act_q8 *act_mid;     // [T*K + T, Fmax/64]
    float *Y;            // [T*K, D] per (token, rank) outputs (large batches)
    float *S;            // [T, D] shared expert output (large batches)
    int *ujob, *nu_job;  // expert parallelism: buckets of this rank's experts [E], their count [1]
    unsigned *ticket;    // [1] last-CTA counter of moe_router (returns to 0 after every launch)
    int *err;            // [1] device error word
    const int *forced_ids = nullptr;   // [T, K] route replay: the ids to use instead of the selection
};

// Tensor maps (CUtensorMap, 128 bytes each) of the staged tensor-core expert kernels, encoded on
// the host per layer and passed to the kernels by value. Views: the expert store as
// [slot][row][row bytes] for gate, up and down (down rows in groups of down_rg rows, so that a group
// is a multiple of 16 bytes), this layer's shared expert, the batch's activation rows (token order)
// and the mid activation rows (pair order).
struct alignas(64) TcMaps {
    uint64_t gate[16], up[16], down[16], sh_gate[16], sh_up[16], sh_down[16], xact[16], mid[16];
    const uint8_t *arena = nullptr;   // slot 0 of the expert store
    int64_t slot_bytes = 0;
    int n_slots = 0, down_rg = 0;
    int xact_rows = 0;                   // token rows the xact map covers
    float zero = 0.0f;                   // a zero the device code cannot constant-fold
    bool gu_ok = false, dn_ok = false;   // the staged gate/up and down kernels can take this layer
};

// What encode_tc_maps needs to know about a layer and the handle's buffers.
struct TcMapSrc {
    const uint8_t *arena;
    int64_t slot_bytes;
    int n_slots;
    int64_t off_up, off_down;
    int D, F, E, Fs, expert_dtype, sh_dtype;
    const uint8_t *sh_gate, *sh_up, *sh_down;
    const void *xact;
    int T;                    // rows of xact
    const void *mid;
    int64_t mid_rows;         // rows of act_mid (pairs + shared tokens)
    int fmax_nb;              // blocks per act_mid row
};

// Fills m (gu_ok / dn_ok false where a kernel's shape or alignment rules are not met or the driver
// cannot encode a map; those stages then run the register-fed tensor-core kernels).
void encode_tc_maps(TcMaps &m, const TcMapSrc &src);

// One MoE layer's weights on the device.
struct MoeLayerDev {
    const float *router;        // [E, D] f32
    const float *router_bias;   // [E] or null
    const float *ffn_norm;      // [D] or null (then x = h as given)
    const uint8_t *const *slab; // [E] device pointers of the resident slabs (null = not resident)
    int expert_dtype;           // Q4 or Q8 (uniform per layer)
    int64_t off_up, off_down;   // FORMAT §5 slab layout
    // shared expert (Fs = 0: none)
    int Fs, sh_dtype;
    const uint8_t *sh_gate, *sh_up, *sh_down;
    const float *sh_gate_inp;   // [D] or null
    const TcMaps *tc = nullptr; // host copy of this layer's tensor maps (staged tensor-core kernels)
};

struct MoeShape {
    int D, F, E, K, T;
    float eps, residual_scale;
    RouteCfg route;
    int ep_size = 1, ep_rank = 0;   // expert parallelism: this rank computes experts e % ep_size == ep_rank
};

// Chooses the fused small-batch path (routing in moe_router's last CTA, sum in moe_down) when
// T * K is at most this many pairs.
constexpr int kFusedMaxPairs = 64;

// Raises the dynamic shared-memory limit of the staged kernels to the device maximum (once per
// device, before any launch or stream capture).
cudaError_t init_kernel_attributes();
cudaError_t init_tc_attributes();   // the staged tensor-core kernels (hx_prefill_tc.cu)

// Launchers return cudaGetLastError() of their launches.
cudaError_t launch_act_quantize(const float *x, int64_t ldx, act_q8 *out, int64_t n, int T, cudaStream_t s);
cudaError_t launch_matmul(int dtype, const void *W, int64_t n_cols, const void *act, int T, float *Y,
                          int64_t ldy, int64_t r0, int64_t r1, cudaStream_t s);
// One token through the staged decode GEMV with x = rmsnorm(h, nw) formed in every CTA (the same
// bits as a separate rmsnorm + activation quantization): Y[r] (or resid[r] += rs * y). Returns
// cudaErrorNotSupported when the staged kernel does not take the shape (then norm and matmul separately).
// early_weights: the staged kernel may start, and stream its weights, while the previous kernel in
// the stream still runs (programmatic dependent launch); only for weights no kernel writes meanwhile.
cudaError_t launch_gemv_norm(int dtype, const void *W, int64_t n_cols, int64_t rows, const float *h, const float *nw,
                             float eps, float *Y, float *resid, float rs, cudaStream_t s, bool early_weights = false);
// The same with a residual epilogue: resid[t * ldy + r] += rs * y (Y unused) when resid is not null.
cudaError_t launch_matmul_resid(int dtype, const void *W, int64_t n_cols, const void *act, int T, float *Y,
                                int64_t ldy, int64_t r0, int64_t r1, float *resid, float rs, cudaStream_t s,
                                bool early_weights = false);
cudaError_t launch_dequantize(int dtype, const void *W, int64_t n_rows, int64_t n_cols, float *out,
                              cudaStream_t s);

// Expert gate/up (which & 1) and down (which & 2) of the unfused path on the tensor cores (tcgen05,
// hx_prefill_tc.cu): the same outputs as the SIMT stages, bit for bit.
cudaError_t launch_moe_experts_tc(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, int which,
                                  cudaStream_t s);
// Pairs (T * K) from which the unfused path runs its expert stages on the tensor cores.
constexpr int kTcMinPairs = kFusedMaxPairs + 1;

// Expert-parallel combine: h += rs * (rank-order sum over j of w_j * y_all[owner rank][pair(t, j)] +
// shared output) with the routing and shared output of the preceding launch_moe_layer.
cudaError_t launch_moe_ep_combine(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc,
                                  const float *y_all, float *h, cudaStream_t s);

// One MoE FFN. Input: h [T, D] (when L.ffn_norm is set, x = rmsnorm(h); otherwise x = h).
// Output: if out != null, out [T, D] = rank-order expert sum (+ shared); if resid, h += rs * sum.
cudaError_t launch_moe_layer(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, float *h,
                             float *out, bool resid, cudaStream_t s);

// Pieces of launch_moe_layer, for hosts that must look at the routing before the experts run
// (the streaming expert store): routing only, then the experts.
cudaError_t launch_moe_route(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, const float *h,
                             cudaStream_t s);
cudaError_t launch_moe_experts(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, float *h,
                               float *out, bool resid, cudaStream_t s);

// One stage of launch_moe_layer (0 norm+activations, 1 router+routing, 2 gate/up, 3 down+sum),
// for per-kernel timing.
cudaError_t launch_moe_stage(int stage, const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, float *h,
                             float *out, bool resid, cudaStream_t s);

// The persistent single-token decode kernel (hx_decode.cu): every layer of [0, n_layers) in one
// cooperative launch with one CTA per SM (every expert resident, no shared expert).
struct DecodeParams {
    int n_layers, D, F, E, K, dtype;
    RouteCfg route;
    float eps, rs;
    int64_t off_up, off_down;
    const float *const *router;   // [n_layers] device pointers
    const float *const *norm;
    const float *const *bias;
    const uint8_t *const *slab;   // [n_layers * E]
    float *h;                     // [D]
    float *xbuf;                  // decode_xbuf_floats(buf_layers, ...) floats, 0xffffffff at allocation
    int buf_layers;               // layers the exchange buffers hold (>= n_layers)
    unsigned *epoch;              // [4] launch counter, arrival count, buffer layers last used by set 0 / 1;
                                  // zero at allocation
    int *err;
    int *ids_out;
    float *w_out;
    unsigned long long *trace;    // null, or [n_layers][grid][decode_stamps()] phase timestamps
    int ep_size = 1, ep_rank = 0; // expert parallelism: this GPU computes the experts e % ep_size == ep_rank
    uint64_t *const *ep_y = nullptr;   // [ep_size] device pointers: every GPU's y words [buf_layers][K][D]
};
int decode_grid();
int decode_stamps();
int decode_max_layers();
int64_t decode_xbuf_floats(int buf_layers, int D, int F, int E, int K);
bool decode_supported(int D, int F, int E, int K, int dtype, bool shared, int ep, std::string *why);
cudaError_t init_decode_attributes();
cudaError_t launch_moe_decode(const DecodeParams &p, cudaStream_t s);

// Fills every expert slab of `n` slabs at dev with deterministic synthetic Q4 blocks (the
// statistics of N(0, sigma) weights packed to Q4), for benchmarks without a container.
// first_slab: index of dev's first slab in the generator's sequence (slab i's bytes depend only on
// seed and i, so a subset of slabs can be generated anywhere).
cudaError_t launch_synth_q4(uint8_t *dev, int64_t n_slabs, int64_t slab_bytes, int D, int F, uint64_t seed,
                            float sigma, cudaStream_t s, int64_t first_slab = 0);
cudaError_t launch_synth_f32(float *dev, int64_t n, uint64_t seed, float sigma, cudaStream_t s);
// A [rows, cols] Q4 or Q8 matrix (rows of cols/64 blocks) with the statistics of N(0, sigma) weights.
cudaError_t launch_synth_blocks(uint8_t *dev, int dtype, int64_t rows, int64_t cols, uint64_t seed, float sigma,
                                cudaStream_t s);

// Device expf restatement over [x0, x0 + n) bit patterns (self-check support).
cudaError_t launch_expf_bits(uint32_t x0, int64_t n, float *out, cudaStream_t s);

}  // namespace hx
