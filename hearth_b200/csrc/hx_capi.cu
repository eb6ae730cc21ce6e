// hx_capi.cu — the C ABI (include/hearth_b200.h): kernel-level entry points and the MoE backend
// handle (device weights, HBM expert store, per-call scratch, CUDA-graph replay).
#include "../../include/hearth_b200.h"
#include "hx_common.cuh"
#include "hx_kernels.h"
#include "hx_store.h"
#include "hx_container.h"
#include "hx_moe_internal.h"

#include <algorithm>
#include <chrono>
#include <sys/stat.h>
#include <cstdlib>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

using namespace hx;

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

bool cuda_ok(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    g_err = std::string(what) + ": " + cudaGetErrorString(e);
    cudaGetLastError();
    return false;
}

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// A device buffer owned by the handle.
struct DevBuf {
    void *p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    ~DevBuf() { release(); }
    bool alloc(size_t bytes) {
        release();
        if (bytes == 0) bytes = 16;
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
            cudaGetLastError();
            p = nullptr;
            return false;
        }
        n = bytes;
        cudaMemset(p, 0, bytes);
        return true;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    template <class T>
    T *as() const {
        return static_cast<T *>(p);
    }
};

// Host scratch for the kernel-level entry points, grown on demand (device).
struct Scratch1 {
    DevBuf w, x, act, y;
};

}  // namespace

namespace hx {
void set_last_error(const char *msg) { g_err = msg; }
}  // namespace hx

// =============================================================================================
// Kernel-level boundary
// =============================================================================================

extern "C" HXB_API const char *hxb_version(void) { return "hearth-b200 0.1.0 (sm_100a)"; }
extern "C" HXB_API const char *hxb_last_error(void) { return g_err.c_str(); }

extern "C" HXB_API int hxb_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

extern "C" HXB_API size_t hxb_row_bytes(int dtype, int64_t n_cols) {
    if (dtype < F32 || dtype > Q4) return 0;
    return (size_t)row_bytes(dtype, n_cols);
}

extern "C" HXB_API int hxb_act_quantize_dev(const float *x, int64_t n, int T, void *act, void *stream) {
    if (!x || !act || n <= 0 || n % QK || T < 0) return fail(HXB_E_ARG, "act_quantize: bad arguments");
    if (!cuda_ok(launch_act_quantize(x, n, (act_q8 *)act, n, T, (cudaStream_t)stream), "act_quantize"))
        return HXB_E_DEVICE;
    return HXB_OK;
}

extern "C" HXB_API int hxb_matmul_dev(int dtype, const void *W, int64_t n_cols, const void *act, int T, float *Y,
                                      int64_t ldy, int64_t r0, int64_t r1, void *stream) {
    if (dtype < F32 || dtype > Q4 || row_bytes(dtype, n_cols) == 0 || T < 0 || r0 < 0 || r1 < r0)
        return fail(HXB_E_ARG, "matmul_dev: bad arguments");
    if (T == 0 || r1 == r0) return HXB_OK;
    if (!W || !act || !Y) return fail(HXB_E_ARG, "matmul_dev: null pointer");
    if (!cuda_ok(launch_matmul(dtype, W, n_cols, act, T, Y, ldy, r0, r1, (cudaStream_t)stream), "matmul"))
        return HXB_E_DEVICE;
    return HXB_OK;
}

extern "C" HXB_API int hxb_dequantize_dev(int dtype, const void *W, int64_t n_rows, int64_t n_cols, float *out,
                                          void *stream) {
    if (dtype < F32 || dtype > Q4 || row_bytes(dtype, n_cols) == 0 || n_rows < 0)
        return fail(HXB_E_ARG, "dequantize_dev: bad arguments");
    if (n_rows == 0) return HXB_OK;
    if (!W || !out) return fail(HXB_E_ARG, "dequantize_dev: null pointer");
    if (!cuda_ok(launch_dequantize(dtype, W, n_rows, n_cols, out, (cudaStream_t)stream), "dequantize"))
        return HXB_E_DEVICE;
    return HXB_OK;
}

extern "C" HXB_API int hxb_expf_dev(uint32_t x0, int64_t n, float *out, void *stream) {
    if (n < 0 || (n && !out)) return fail(HXB_E_ARG, "expf_dev: bad arguments");
    if (!cuda_ok(launch_expf_bits(x0, n, out, (cudaStream_t)stream), "expf")) return HXB_E_DEVICE;
    return HXB_OK;
}

// hearth_matmul with host buffers (engine/src/quant.c:574-600): same argument checks and codes.
extern "C" HXB_API int hxb_matmul(int dtype, const void *W, int64_t n_rows, int64_t n_cols, const float *X, int T,
                                  float *Y) {
    if (dtype < F32 || dtype > Q4 || n_rows < 0 || T < 0 || row_bytes(dtype, n_cols) == 0) {
        fail(HXB_MM_E_ARG, "hxb_matmul: bad arguments");
        return HXB_MM_E_ARG;
    }
    if (T == 0 || n_rows == 0) return HXB_MM_OK;
    if (!W || !X || !Y) {
        fail(HXB_MM_E_ARG, "hxb_matmul: null pointer");
        return HXB_MM_E_ARG;
    }
    if (hxb_device_count() <= 0) {
        fail(HXB_MM_E_NODEV, "hxb_matmul: no CUDA device");
        return HXB_MM_E_NODEV;
    }
    const size_t wb = (size_t)row_bytes(dtype, n_cols) * (size_t)n_rows;
    const size_t xb = sizeof(float) * (size_t)n_cols * (size_t)T;
    const size_t ab = is_quant(dtype) ? (size_t)(n_cols / QK) * ACT_BLOCK * (size_t)T : 0;
    const size_t yb = sizeof(float) * (size_t)n_rows * (size_t)T;
    Scratch1 s;
    if (!s.w.alloc(wb) || !s.x.alloc(xb) || !s.act.alloc(ab) || !s.y.alloc(yb)) {
        fail(HXB_MM_E_ALLOC, "hxb_matmul: device allocation failed");
        return HXB_MM_E_ALLOC;
    }
    cudaStream_t st = nullptr;
    bool ok = cuda_ok(cudaMemcpy(s.w.p, W, wb, cudaMemcpyHostToDevice), "copy W") &&
              cuda_ok(cudaMemcpy(s.x.p, X, xb, cudaMemcpyHostToDevice), "copy X");
    const void *act = s.x.p;
    if (ok && is_quant(dtype)) {
        ok = cuda_ok(launch_act_quantize(s.x.as<float>(), n_cols, s.act.as<act_q8>(), n_cols, T, st), "act");
        act = s.act.p;
    }
    ok = ok && cuda_ok(launch_matmul(dtype, s.w.p, n_cols, act, T, s.y.as<float>(), n_rows, 0, n_rows, st), "mm");
    ok = ok && cuda_ok(cudaMemcpy(Y, s.y.p, yb, cudaMemcpyDeviceToHost), "copy Y");
    if (!ok) return HXB_MM_E_NODEV;
    return HXB_MM_OK;
}

extern "C" HXB_API int hxb_dequantize(int dtype, const void *src, int64_t n_rows, int64_t n_cols, float *dst) {
    if (dtype < F32 || dtype > Q4 || row_bytes(dtype, n_cols) == 0 || n_rows < 0)
        return fail(HXB_E_ARG, "hxb_dequantize: bad arguments");
    if (n_rows == 0) return HXB_OK;
    if (!src || !dst) return fail(HXB_E_ARG, "hxb_dequantize: null pointer");
    const size_t wb = (size_t)row_bytes(dtype, n_cols) * (size_t)n_rows;
    const size_t ob = sizeof(float) * (size_t)n_rows * (size_t)n_cols;
    DevBuf w, o;
    if (!w.alloc(wb) || !o.alloc(ob)) return fail(HXB_E_NOMEM, "hxb_dequantize: device allocation failed");
    bool ok = cuda_ok(cudaMemcpy(w.p, src, wb, cudaMemcpyHostToDevice), "copy") &&
              cuda_ok(launch_dequantize(dtype, w.p, n_rows, n_cols, o.as<float>(), nullptr), "dequantize") &&
              cuda_ok(cudaMemcpy(dst, o.p, ob, cudaMemcpyDeviceToHost), "copy back");
    return ok ? HXB_OK : HXB_E_DEVICE;
}

// =============================================================================================
// MoE backend handle
// =============================================================================================

struct LayerBufs {
    DevBuf router, bias, norm, sh_gate, sh_up, sh_down, sh_gate_inp;
    TcMaps maps;   // tensor maps of the staged tensor-core kernels (encoded when the layer is set)
    bool set = false;
};

struct GraphKey {
    int T, l0, nl;
    const void *h;
    cudaStream_t s;
    bool operator<(const GraphKey &o) const {
        return std::tie(T, l0, nl, h, s) < std::tie(o.T, o.l0, o.nl, o.h, o.s);
    }
};

struct hxb_moe {
    hxb_moe_config cfg{};
    int device = 0;
    size_t slab_bytes = 0;
    slab_layout lay{};
    cudaStream_t stream = nullptr;
    HbmStore store;
    bool resident_mode = false;          // every expert has a slot: no host round trip per layer
    std::unique_ptr<LayerBufs[]> layers;
    DevBuf table;                        // [L*E] device slab pointers
    const uint8_t **host_table = nullptr;  // pinned mirror
    // scratch
    DevBuf x, xact, logits, sh_logit, ids, wts, nu, ulist, u_p0, u_n, pair_tok, pair_of, act_mid, Y, S, ticket, err;
    DevBuf hbuf, obuf;                   // device copies of host inputs/outputs
    DevBuf forced;                       // route replay: [n_layers][max_tokens][K] expert ids
    // streaming store, next-layer prediction: the routing stages' own outputs for layer l+1
    DevBuf px, pxact, plogits, psh_logit, pids, pwts, pnu, pulist, pu_p0, pu_n, ppair_tok, ppair_of, pticket;
    cudaEvent_t pred_ready = nullptr;
    float *hpin = nullptr;               // pinned staging [max_tokens, D]
    int *epin = nullptr;                 // pinned: error word, nu, ulist
    std::map<GraphKey, cudaGraphExec_t> graphs;
    hxb_moe_stats st{};
    int last_T = 0;
    // persistent single-token decode kernel (every expert resident)
    DevBuf ujob, nu_job;                 // expert parallelism: this rank's buckets
    bool use_decode = false, dec_dirty = true;
    DevBuf dec_router, dec_norm, dec_bias;
    DevBuf dec_xbuf, dec_epoch;          // exchange buffers (two sets) and the launch counter
    DevBuf dec_trace;                    // phase timeline of the last launch (HXB_TRACE=1)
    // expert parallelism in the persistent kernel: this GPU's y words (written by every GPU) and the
    // table of every GPU's y words, filled by hxb_moe_ep_connect from the other ranks' IPC handles
    DevBuf ep_y, ep_peers;
    std::vector<void *> ep_opened;       // peer mappings to close
    bool ep_connected = false;

    MoeScratch scratch() const {
        MoeScratch s;
        s.x = x.as<float>();
        s.xact = xact.as<act_q8>();
        s.logits = logits.as<float>();
        s.sh_logit = sh_logit.as<float>();
        s.ids = ids.as<int>();
        s.wts = wts.as<float>();
        s.nu = nu.as<int>();
        s.ulist = ulist.as<int>();
        s.u_p0 = u_p0.as<int>();
        s.u_n = u_n.as<int>();
        s.pair_tok = pair_tok.as<int>();
        s.pair_of = pair_of.as<int>();
        s.act_mid = act_mid.as<act_q8>();
        s.Y = Y.as<float>();
        s.S = S.as<float>();
        s.ujob = ujob.as<int>();
        s.nu_job = nu_job.as<int>();
        s.ticket = ticket.as<unsigned>();
        s.err = err.as<int>();
        return s;
    }

    // The scratch of a prediction: the routing stages write only into their own buffers.
    MoeScratch pred_scratch() const {
        MoeScratch s = scratch();
        s.x = px.as<float>();
        s.xact = pxact.as<act_q8>();
        s.logits = plogits.as<float>();
        s.sh_logit = psh_logit.as<float>();
        s.ids = pids.as<int>();
        s.wts = pwts.as<float>();
        s.nu = pnu.as<int>();
        s.ulist = pulist.as<int>();
        s.u_p0 = pu_p0.as<int>();
        s.u_n = pu_n.as<int>();
        s.pair_tok = ppair_tok.as<int>();
        s.pair_of = ppair_of.as<int>();
        s.ticket = pticket.as<unsigned>();
        return s;
    }

    MoeShape shape(int T) const {
        MoeShape sh;
        sh.D = cfg.d_model;
        sh.F = cfg.expert_ffn_dim;
        sh.E = cfg.n_experts;
        sh.K = cfg.top_k;
        sh.T = T;
        sh.eps = cfg.norm_eps;
        sh.residual_scale = cfg.residual_scale;
        sh.route.E = cfg.n_experts;
        sh.route.K = cfg.top_k;
        sh.route.score_fn = cfg.score_fn;
        sh.route.score_bias = cfg.score_bias;
        sh.route.n_group = cfg.n_group;
        sh.route.topk_group = cfg.topk_group;
        sh.route.norm_topk_prob = cfg.norm_topk_prob;
        sh.route.routed_scale = cfg.routed_scale;
        sh.ep_size = cfg.ep_size;
        sh.ep_rank = cfg.ep_rank;
        return sh;
    }

    bool owns(int e) const { return e % cfg.ep_size == cfg.ep_rank; }
    int owned_experts() const {
        int n = 0;
        for (int e = 0; e < cfg.n_experts; e++) n += owns(e) ? 1 : 0;
        return n;
    }

    MoeLayerDev layer_dev(int l, bool with_norm) const {
        const LayerBufs &b = layers[(size_t)l];
        MoeLayerDev d;
        d.router = b.router.as<float>();
        d.router_bias = cfg.score_bias ? b.bias.as<float>() : nullptr;
        d.ffn_norm = with_norm ? b.norm.as<float>() : nullptr;
        d.slab = table.as<const uint8_t *>() + (size_t)l * cfg.n_experts;
        d.expert_dtype = cfg.expert_dtype;
        d.off_up = lay.off_up;
        d.off_down = lay.off_down;
        d.Fs = cfg.shared_ffn_dim;
        d.sh_dtype = cfg.shared_dtype;
        d.sh_gate = b.sh_gate.as<uint8_t>();
        d.sh_up = b.sh_up.as<uint8_t>();
        d.sh_down = b.sh_down.as<uint8_t>();
        d.sh_gate_inp = cfg.shared_gate ? b.sh_gate_inp.as<float>() : nullptr;
        d.tc = &b.maps;
        return d;
    }

    // (Re)encodes layer l's tensor maps: the store views, its shared expert and the scratch rows.
    void refresh_maps(int l) {
        LayerBufs &b = layers[(size_t)l];
        TcMapSrc a;
        a.arena = store.n_slots() ? store.slot_ptr(0) : nullptr;
        a.slot_bytes = (int64_t)slab_bytes;
        a.n_slots = store.n_slots();
        a.off_up = lay.off_up;
        a.off_down = lay.off_down;
        a.D = cfg.d_model;
        a.F = cfg.expert_ffn_dim;
        a.E = cfg.n_experts;
        a.Fs = cfg.shared_ffn_dim;
        a.expert_dtype = cfg.expert_dtype;
        a.sh_dtype = cfg.shared_dtype;
        a.sh_gate = b.sh_gate.as<uint8_t>();
        a.sh_up = b.sh_up.as<uint8_t>();
        a.sh_down = b.sh_down.as<uint8_t>();
        a.xact = xact.p;
        a.T = cfg.max_tokens;
        a.mid = act_mid.p;
        a.fmax_nb = std::max(cfg.expert_ffn_dim, cfg.shared_ffn_dim) / QK;
        a.mid_rows = (int64_t)cfg.max_tokens * cfg.top_k + cfg.max_tokens;
        encode_tc_maps(b.maps, a);
    }

    ~hxb_moe() {
        if (stream) cudaStreamSynchronize(stream);
        for (void *p : ep_opened) cudaIpcCloseMemHandle(p);
        for (auto &g : graphs) cudaGraphExecDestroy(g.second);
        graphs.clear();
        if (hpin) cudaFreeHost(hpin);
        if (epin) cudaFreeHost(epin);
        if (host_table) cudaFreeHost(host_table);
        if (pred_ready) cudaEventDestroy(pred_ready);
        store.close();
        if (stream) cudaStreamDestroy(stream);
    }
};

extern "C" HXB_API void hxb_moe_default_config(hxb_moe_config *c) {
    if (!c) return;
    std::memset(c, 0, sizeof *c);
    c->n_layers = 1;
    c->top_k = 1;
    c->n_group = 1;
    c->topk_group = 1;
    c->norm_topk_prob = 1;
    c->routed_scale = 1.0f;
    c->prefetch_next = 1;
    c->residual_scale = 1.0f;
    c->norm_eps = 1e-6f;
    c->expert_dtype = Q4;
    c->shared_dtype = Q8;
    c->max_tokens = 1;
    c->cache_gb = 0.0;
    c->policy = POLICY_LFU;
    c->heat_decay = 0.995f;
    c->ep_size = 1;
    c->ep_rank = 0;
}

static void set_errbuf(char *err, size_t errlen, const std::string &msg) {
    g_err = msg;
    if (err && errlen) {
        std::snprintf(err, errlen, "%s", msg.c_str());
    }
}

extern "C" HXB_API hxb_moe *hxb_moe_open(const hxb_moe_config *c, char *err, size_t errlen) {
    if (!c) {
        set_errbuf(err, errlen, "hxb_moe_open: null config");
        return nullptr;
    }
    const hxb_moe_config &k = *c;
    std::string why;
    if (k.n_layers <= 0) why = "n_layers must be positive";
    else if (k.d_model <= 0 || k.d_model % QK != 0 || k.d_model > 8192) why = "d_model must be a multiple of 64 up to 8192";
    else if (k.expert_ffn_dim <= 0 || k.expert_ffn_dim % QK) why = "expert_ffn_dim must be a positive multiple of 64";
    else if (k.n_experts <= 0 || k.n_experts > 384) why = "n_experts must be 1..384";
    else if (k.top_k <= 0 || k.top_k > 32 || k.top_k > k.n_experts) why = "top_k must be 1..min(32, n_experts)";
    else if (k.expert_dtype != Q4 && k.expert_dtype != Q8) why = "expert_dtype must be Q4 or Q8";
    else if (k.shared_ffn_dim < 0 || k.shared_ffn_dim % QK) why = "shared_ffn_dim must be a multiple of 64";
    else if (k.shared_ffn_dim && k.shared_dtype != Q4 && k.shared_dtype != Q8) why = "shared_dtype must be Q4 or Q8";
    else if (k.n_group > 1 && (k.n_experts % k.n_group || k.n_group > 32 || k.topk_group < 1 || k.topk_group > k.n_group))
        why = "bad expert grouping";
    else if (k.max_tokens <= 0 || k.max_tokens > 8192) why = "max_tokens must be 1..8192";
    else if (k.ep_size < 1 || k.ep_size > 64 || k.ep_rank < 0 || k.ep_rank >= k.ep_size || k.ep_size > k.n_experts)
        why = "expert parallelism: need 1 <= ep_size <= min(64, n_experts) and 0 <= ep_rank < ep_size";
    if (!why.empty()) {
        set_errbuf(err, errlen, "hxb_moe_open: " + why);
        return nullptr;
    }
    if (hxb_device_count() <= k.device) {
        set_errbuf(err, errlen, "hxb_moe_open: CUDA device " + std::to_string(k.device) + " not available");
        return nullptr;
    }
    std::unique_ptr<hxb_moe> m(new hxb_moe());
    m->cfg = k;
    m->device = k.device;
    cudaSetDevice(k.device);
    m->lay = make_slab_layout(k.expert_dtype, k.d_model, k.expert_ffn_dim);
    m->slab_bytes = (size_t)m->lay.nbytes;
    const int L = k.n_layers, E = k.n_experts, D = k.d_model, T = k.max_tokens, K = k.top_k;
    const int64_t nkeys = (int64_t)L * E;
    const int64_t owned_keys = (int64_t)L * m->owned_experts();   // all keys without expert parallelism
    int64_t n_slots = owned_keys;
    if (k.cache_gb > 0.0) {
        const int64_t by_budget = (int64_t)(k.cache_gb * 1073741824.0 / (double)m->slab_bytes);
        n_slots = std::min<int64_t>(owned_keys, std::max<int64_t>(by_budget, (int64_t)E + 2));
    }
    m->resident_mode = n_slots >= owned_keys;
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) {
        set_errbuf(err, errlen, "hxb_moe_open: cannot create a stream");
        return nullptr;
    }
    if (!m->store.open(L, E, m->slab_bytes, (int)n_slots, k.policy, k.heat_decay, why)) {
        set_errbuf(err, errlen, "hxb_moe_open: " + why);
        return nullptr;
    }
    m->layers.reset(new LayerBufs[(size_t)L]);
    const int Fmax = std::max(k.expert_ffn_dim, k.shared_ffn_dim);
    const size_t P = (size_t)T * K;
    bool ok = m->table.alloc(sizeof(void *) * (size_t)nkeys) && m->x.alloc(sizeof(float) * (size_t)T * D) &&
              m->xact.alloc((size_t)T * (D / QK) * ACT_BLOCK) && m->logits.alloc(sizeof(float) * (size_t)T * E) &&
              m->sh_logit.alloc(sizeof(float) * (size_t)T) && m->ids.alloc(sizeof(int) * P) &&
              m->wts.alloc(sizeof(float) * P) && m->nu.alloc(sizeof(int) * 4) && m->ulist.alloc(sizeof(int) * E) &&
              m->u_p0.alloc(sizeof(int) * E) && m->u_n.alloc(sizeof(int) * E) &&
              m->pair_tok.alloc(sizeof(int) * P) && m->pair_of.alloc(sizeof(int) * P) &&
              m->act_mid.alloc((P + (size_t)T) * (size_t)(Fmax / QK) * ACT_BLOCK) &&
              m->Y.alloc(P * kFusedMaxPairs > 0 && (int)P > kFusedMaxPairs ? sizeof(float) * P * D : 16) &&
              m->S.alloc(k.shared_ffn_dim && ((int)P > kFusedMaxPairs || k.ep_size > 1) ? sizeof(float) * (size_t)T * D
                                                                                          : 16) &&
              m->ujob.alloc(sizeof(int) * (size_t)E) && m->nu_job.alloc(sizeof(int) * 4) &&
              m->ticket.alloc(64) && m->err.alloc(64) && m->hbuf.alloc(sizeof(float) * (size_t)T * D) &&
              m->forced.alloc(sizeof(int) * P * (size_t)L) &&
              m->obuf.alloc(sizeof(float) * (size_t)T * D);
    if (ok && !m->resident_mode && k.prefetch_next)   // the prediction's own routing buffers
        ok = m->px.alloc(sizeof(float) * (size_t)T * D) && m->pxact.alloc((size_t)T * (D / QK) * ACT_BLOCK) &&
             m->plogits.alloc(sizeof(float) * (size_t)T * E) && m->psh_logit.alloc(sizeof(float) * (size_t)T) &&
             m->pids.alloc(sizeof(int) * P) && m->pwts.alloc(sizeof(float) * P) && m->pnu.alloc(sizeof(int) * 4) &&
             m->pulist.alloc(sizeof(int) * E) && m->pu_p0.alloc(sizeof(int) * E) && m->pu_n.alloc(sizeof(int) * E) &&
             m->ppair_tok.alloc(sizeof(int) * P) && m->ppair_of.alloc(sizeof(int) * P) && m->pticket.alloc(64) &&
             cudaMemset(m->pticket.p, 0, 64) == cudaSuccess &&
             cudaEventCreateWithFlags(&m->pred_ready, cudaEventDisableTiming) == cudaSuccess;
    ok = ok && cudaHostAlloc((void **)&m->hpin, sizeof(float) * (size_t)T * D, cudaHostAllocDefault) == cudaSuccess;
    ok = ok && cudaHostAlloc((void **)&m->epin, sizeof(int) * (size_t)(9 + 3 * E), cudaHostAllocDefault) == cudaSuccess;
    ok = ok && cudaHostAlloc((void **)&m->host_table, sizeof(void *) * (size_t)nkeys, cudaHostAllocDefault) ==
                   cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        set_errbuf(err, errlen, "hxb_moe_open: out of device or pinned memory");
        return nullptr;
    }
    std::memset(m->host_table, 0, sizeof(void *) * (size_t)nkeys);
    if (m->resident_mode) {
        // HXB_PERSISTENT=0: per-phase kernels only
        const char *env = std::getenv("HXB_PERSISTENT");
        std::string why_not;
        const bool off = env && env[0] == '0';
        m->use_decode = !off &&
                        decode_supported(D, k.expert_ffn_dim, E, K, k.expert_dtype, k.shared_ffn_dim > 0, k.ep_size,
                                         &why_not);
        if (m->use_decode) {
            const size_t xb = sizeof(float) * (size_t)decode_xbuf_floats(L, D, k.expert_ffn_dim, E, K);
            if (!m->dec_router.alloc(sizeof(void *) * (size_t)L) || !m->dec_norm.alloc(sizeof(void *) * (size_t)L) ||
                !m->dec_bias.alloc(sizeof(void *) * (size_t)L) || !m->dec_xbuf.alloc(xb) || !m->dec_epoch.alloc(64) ||
                !cuda_ok(cudaMemset(m->dec_xbuf.p, 0xff, xb), "decode buffers") ||
                !cuda_ok(cudaMemset(m->dec_epoch.p, 0, 64), "decode buffers") ||
                !cuda_ok(init_decode_attributes(), "decode attributes")) {
                set_errbuf(err, errlen, "hxb_moe_open: persistent decode setup failed: " + g_err);
                return nullptr;
            }
            if (k.ep_size > 1 &&
                (!m->ep_y.alloc(sizeof(uint64_t) * (size_t)L * K * D) || !m->ep_peers.alloc(sizeof(void *) * 64) ||
                 !cuda_ok(cudaMemset(m->ep_y.p, 0, m->ep_y.n), "ep words"))) {
                set_errbuf(err, errlen, "hxb_moe_open: expert-parallel exchange words: " + g_err);
                return nullptr;
            }
            const char *tr = std::getenv("HXB_TRACE");
            if (tr && tr[0] == '1' &&
                !m->dec_trace.alloc(sizeof(unsigned long long) * (size_t)L * decode_grid() * decode_stamps())) {
                set_errbuf(err, errlen, "hxb_moe_open: trace buffer");
                return nullptr;
            }
        }
    }
    if (!cuda_ok(init_kernel_attributes(), "kernel attributes")) {
        set_errbuf(err, errlen, "hxb_moe_open: " + g_err);
        return nullptr;
    }
    cudaDeviceSynchronize();
    m->st.n_slots = m->store.n_slots();
    m->st.slot_bytes = m->slab_bytes;
    return m.release();
}

extern "C" HXB_API void hxb_moe_close(hxb_moe *m) { delete m; }

extern "C" HXB_API size_t hxb_moe_slab_bytes(const hxb_moe *m) { return m ? m->slab_bytes : 0; }

static bool upload(DevBuf &b, const void *src, size_t bytes) {
    if (!src) {
        b.release();
        return true;
    }
    if (!b.alloc(bytes)) return false;
    return cudaMemcpy(b.p, src, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
}

static void drop_graphs(hxb_moe *m) {
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (auto &g : m->graphs) cudaGraphExecDestroy(g.second);
    m->graphs.clear();
}

extern "C" HXB_API int hxb_moe_set_layer(hxb_moe *m, int layer, const float *router, const float *router_bias,
                                         const float *ffn_norm, const void *sh_gate, const void *sh_up,
                                         const void *sh_down, const float *sh_gate_inp) {
    if (!m || layer < 0 || layer >= m->cfg.n_layers || !router) return fail(HXB_E_ARG, "set_layer: bad arguments");
    const hxb_moe_config &k = m->cfg;
    if (k.score_bias && !router_bias) return fail(HXB_E_ARG, "set_layer: score_bias needs router_bias");
    if (k.shared_ffn_dim && (!sh_gate || !sh_up || !sh_down)) return fail(HXB_E_ARG, "set_layer: shared expert missing");
    if (k.shared_gate && !sh_gate_inp) return fail(HXB_E_ARG, "set_layer: shared gate input missing");
    cudaSetDevice(m->device);
    LayerBufs &b = m->layers[(size_t)layer];
    const size_t D = (size_t)k.d_model, E = (size_t)k.n_experts, Fs = (size_t)k.shared_ffn_dim;
    const size_t shb = Fs ? (size_t)row_bytes(k.shared_dtype, (int64_t)D) * Fs : 0;
    const size_t shd = Fs ? (size_t)row_bytes(k.shared_dtype, (int64_t)Fs) * D : 0;
    bool ok = upload(b.router, router, sizeof(float) * E * D) && upload(b.bias, router_bias, sizeof(float) * E) &&
              upload(b.sh_gate, Fs ? sh_gate : nullptr, shb) && upload(b.sh_up, Fs ? sh_up : nullptr, shb) &&
              upload(b.sh_down, Fs ? sh_down : nullptr, shd) &&
              upload(b.sh_gate_inp, k.shared_gate ? sh_gate_inp : nullptr, sizeof(float) * D);
    if (ok) {
        if (ffn_norm) ok = upload(b.norm, ffn_norm, sizeof(float) * D);
        else {
            std::vector<float> ones(D, 1.0f);
            ok = upload(b.norm, ones.data(), sizeof(float) * D);
        }
    }
    if (!ok) {
        cudaGetLastError();
        return fail(HXB_E_NOMEM, "set_layer: device allocation or copy failed");
    }
    b.set = true;
    m->refresh_maps(layer);
    m->dec_dirty = true;
    drop_graphs(m);
    return HXB_OK;
}

// Resident mode: (re)places an expert's slab in its HBM slot from its host source and points both
// pointer tables at it.
static int place_resident_expert(hxb_moe *m, int layer, int expert) {
    cudaEvent_t ev = nullptr;
    const uint8_t *p = m->store.acquire_async(layer, expert, &ev);
    if (!p) return fail(HXB_E_IO, "set_expert: could not place the expert in HBM");
    m->store.release(layer, expert, m->store.copy_stream());
    cudaStreamSynchronize(m->store.copy_stream());
    m->host_table[(size_t)layer * m->cfg.n_experts + expert] = p;
    if (!cuda_ok(cudaMemcpy(m->table.as<const uint8_t *>() + (size_t)layer * m->cfg.n_experts + expert, &p, sizeof p,
                            cudaMemcpyHostToDevice),
                 "set_expert table"))
        return HXB_E_DEVICE;
    return HXB_OK;
}

extern "C" HXB_API int hxb_moe_set_expert(hxb_moe *m, int layer, int expert, const void *slab, size_t nbytes) {
    if (!m || layer < 0 || layer >= m->cfg.n_layers || expert < 0 || expert >= m->cfg.n_experts || !slab ||
        nbytes < (size_t)m->lay.end || nbytes > m->slab_bytes)
        return fail(HXB_E_ARG, "set_expert: bad arguments (slab must be %zu bytes)", m ? m->slab_bytes : (size_t)0);
    if (!m->owns(expert)) return HXB_OK;   // expert parallelism: another rank's expert, not held here
    cudaSetDevice(m->device);
    std::string why;
    if (!m->store.set_source(layer, expert, slab, nbytes, why)) return fail(HXB_E_NOMEM, "set_expert: %s", why.c_str());
    if (m->resident_mode) {   // every expert keeps a slot: copy it in now (and the experts sharing its bytes)
        int rc = place_resident_expert(m, layer, expert);
        for (int k : m->store.aliases_of(layer, expert))
            if (rc == HXB_OK) rc = place_resident_expert(m, k / m->cfg.n_experts, k % m->cfg.n_experts);
        if (rc != HXB_OK) return rc;
        m->store.reset_stats();
    }
    drop_graphs(m);
    return HXB_OK;
}

extern "C" HXB_API int hxb_moe_get_expert(hxb_moe *m, int layer, int expert, void *dst, size_t nbytes) {
    if (!m || layer < 0 || layer >= m->cfg.n_layers || expert < 0 || expert >= m->cfg.n_experts || !dst ||
        nbytes < m->slab_bytes)
        return fail(HXB_E_ARG, "get_expert: bad arguments (dst must hold %zu bytes)", m ? m->slab_bytes : (size_t)0);
    if (!m->resident_mode) return fail(HXB_E_UNSUPPORTED, "get_expert: the handle does not hold every expert in HBM");
    const uint8_t *p = m->host_table[(size_t)layer * m->cfg.n_experts + expert];
    if (!p) return fail(HXB_E_ARG, "get_expert: expert (%d, %d) is not held by this handle", layer, expert);
    cudaSetDevice(m->device);
    if (!cuda_ok(cudaStreamSynchronize(m->stream), "get_expert") ||
        !cuda_ok(cudaMemcpy(dst, p, m->slab_bytes, cudaMemcpyDeviceToHost), "get_expert"))
        return HXB_E_DEVICE;
    return HXB_OK;
}

extern "C" HXB_API int hxb_moe_share_expert(hxb_moe *m, int layer, int expert, int src_layer, int src_expert) {
    if (!m || layer < 0 || layer >= m->cfg.n_layers || expert < 0 || expert >= m->cfg.n_experts || src_layer < 0 ||
        src_layer >= m->cfg.n_layers || src_expert < 0 || src_expert >= m->cfg.n_experts)
        return fail(HXB_E_ARG, "share_expert: bad arguments");
    if (!m->owns(expert)) return HXB_OK;
    if (!m->owns(src_expert)) return fail(HXB_E_ARG, "share_expert: the source expert is not held by this handle");
    cudaSetDevice(m->device);
    std::string why;
    if (!m->store.share_source(layer, expert, src_layer, src_expert, why))
        return fail(HXB_E_ARG, "share_expert: %s", why.c_str());
    if (m->resident_mode) {
        const int rc = place_resident_expert(m, layer, expert);
        if (rc != HXB_OK) return rc;
        m->store.reset_stats();
    }
    drop_graphs(m);
    return HXB_OK;
}

extern "C" HXB_API int hxb_moe_synthesize(hxb_moe *m, uint64_t seed, float sigma_router, float sigma_expert) {
    if (!m) return fail(HXB_E_ARG, "synthesize: null handle");
    if (m->cfg.expert_dtype != Q4) return fail(HXB_E_UNSUPPORTED, "synthesize: Q4 experts only");
    if (m->cfg.shared_ffn_dim && m->cfg.shared_dtype != Q4 && m->cfg.shared_dtype != Q8)
        return fail(HXB_E_UNSUPPORTED, "synthesize: Q4/Q8 shared experts only");
    cudaSetDevice(m->device);
    const hxb_moe_config &k = m->cfg;
    const int L = k.n_layers, E = k.n_experts, D = k.d_model, Fs = k.shared_ffn_dim;
    for (int l = 0; l < L; l++) {
        LayerBufs &b = m->layers[(size_t)l];
        const uint64_t ls = seed * 1000003ull + (uint64_t)l;
        const size_t shb = Fs ? (size_t)row_bytes(k.shared_dtype, (int64_t)D) * Fs : 0;
        const size_t shd = Fs ? (size_t)row_bytes(k.shared_dtype, (int64_t)Fs) * D : 0;
        bool ok = b.router.alloc(sizeof(float) * (size_t)E * D) && b.norm.alloc(sizeof(float) * (size_t)D) &&
                  (!k.score_bias || b.bias.alloc(sizeof(float) * (size_t)E)) &&
                  (!Fs || (b.sh_gate.alloc(shb) && b.sh_up.alloc(shb) && b.sh_down.alloc(shd))) &&
                  (!k.shared_gate || b.sh_gate_inp.alloc(sizeof(float) * (size_t)D));
        if (!ok) return fail(HXB_E_NOMEM, "synthesize: out of device memory");
        if (!cuda_ok(launch_synth_f32(b.router.as<float>(), (int64_t)E * D, ls, sigma_router, m->stream),
                     "synth router"))
            return HXB_E_DEVICE;
        // the selection bias (sigmoid routers) at half the router's spread; the shared expert's
        // matrices like the routed experts'; its gate input like the router
        if (k.score_bias &&
            !cuda_ok(launch_synth_f32(b.bias.as<float>(), E, ls ^ 0xb1a5b1a5ull, 0.5f * sigma_router, m->stream),
                     "synth bias"))
            return HXB_E_DEVICE;
        if (Fs && !(cuda_ok(launch_synth_blocks(b.sh_gate.as<uint8_t>(), k.shared_dtype, Fs, D, ls ^ 0x5a1ull,
                                                sigma_expert, m->stream),
                            "synth shared gate") &&
                    cuda_ok(launch_synth_blocks(b.sh_up.as<uint8_t>(), k.shared_dtype, Fs, D, ls ^ 0x5a2ull,
                                                sigma_expert, m->stream),
                            "synth shared up") &&
                    cuda_ok(launch_synth_blocks(b.sh_down.as<uint8_t>(), k.shared_dtype, D, Fs, ls ^ 0x5a3ull,
                                                sigma_expert, m->stream),
                            "synth shared down")))
            return HXB_E_DEVICE;
        if (k.shared_gate && !cuda_ok(launch_synth_f32(b.sh_gate_inp.as<float>(), D, ls ^ 0x5a4ull, sigma_router,
                                                       m->stream),
                                      "synth shared gate input"))
            return HXB_E_DEVICE;
        std::vector<float> ones((size_t)D, 1.0f);
        cudaMemcpy(b.norm.p, ones.data(), sizeof(float) * D, cudaMemcpyHostToDevice);
        b.set = true;
        m->refresh_maps(l);
        if (!m->resident_mode) continue;
        for (int e = 0; e < E; e++) {
            if (!m->owns(e)) continue;
            uint8_t *p = m->store.place_resident(l, e);
            if (!p) return fail(HXB_E_NOMEM, "synthesize: no slot");
            m->host_table[(size_t)l * E + e] = p;
        }
    }
    if (!m->resident_mode) {   // the store's host tier: each slab generated on the device, then handed over
        DevBuf tmp;
        std::vector<uint8_t> host(m->slab_bytes);
        if (!tmp.alloc(m->slab_bytes)) return fail(HXB_E_NOMEM, "synthesize: out of device memory");
        for (int64_t i = 0; i < (int64_t)L * E; i++) {
            if (!m->owns((int)(i % E))) continue;
            if (!cuda_ok(launch_synth_q4(tmp.as<uint8_t>(), 1, (int64_t)m->slab_bytes, D, k.expert_ffn_dim, seed,
                                         sigma_expert, m->stream, i),
                         "synth experts") ||
                !cuda_ok(cudaMemcpyAsync(host.data(), tmp.p, m->slab_bytes, cudaMemcpyDeviceToHost, m->stream),
                         "synth copy") ||
                !cuda_ok(cudaStreamSynchronize(m->stream), "synth copy"))
                return HXB_E_DEVICE;
            std::string why;
            if (!m->store.set_source((int)(i / E), (int)(i % E), host.data(), m->slab_bytes, why))
                return fail(HXB_E_NOMEM, "synthesize: %s", why.c_str());
        }
        m->dec_dirty = true;
        drop_graphs(m);
        return cuda_ok(cudaStreamSynchronize(m->stream), "synthesize") ? HXB_OK : HXB_E_DEVICE;
    }
    if (k.ep_size > 1) {   // this rank's slabs, each the bytes of its place in the whole sequence
        for (int64_t i = 0; i < (int64_t)L * E; i++)
            if (m->owns((int)(i % E)) &&
                !cuda_ok(launch_synth_q4(const_cast<uint8_t *>(m->host_table[i]), 1, (int64_t)m->slab_bytes, D,
                                         k.expert_ffn_dim, seed, sigma_expert, m->stream, i),
                         "synth experts"))
                return HXB_E_DEVICE;
    } else {
        // slots were handed out in order, so the L*E slabs are contiguous: one launch fills them all
        const uint8_t *base = m->host_table[0];
        for (int64_t i = 0; i < (int64_t)L * E; i++)
            if (m->host_table[i] != base + (size_t)i * m->slab_bytes)
                return fail(HXB_E_ARG, "synthesize: expert slots are not contiguous (experts were set before)");
        if (!cuda_ok(launch_synth_q4(const_cast<uint8_t *>(base), (int64_t)L * E, (int64_t)m->slab_bytes, D,
                                     k.expert_ffn_dim, seed, sigma_expert, m->stream),
                     "synth experts"))
            return HXB_E_DEVICE;
    }
    if (!cuda_ok(cudaMemcpyAsync(m->table.p, m->host_table, sizeof(void *) * (size_t)L * E, cudaMemcpyHostToDevice,
                                 m->stream),
                 "table"))
        return HXB_E_DEVICE;
    if (!cuda_ok(cudaStreamSynchronize(m->stream), "synthesize")) return HXB_E_DEVICE;
    m->dec_dirty = true;
    drop_graphs(m);
    return HXB_OK;
}

// ---------------------------------------------------------------------------------------------
// Evaluation
// ---------------------------------------------------------------------------------------------

// Reads and clears the device error word (after the stream was synchronised).
static int take_device_error(hxb_moe *m, int word) {
    if (!word) return HXB_OK;
    cudaMemset(m->err.p, 0, sizeof(int));
    if (word == 2) return fail(HXB_E_IO, "an expert was not resident in HBM");
    if (word == 3) return fail(HXB_E_UNSUPPORTED, "expert dtype not handled by the kernels");
    return fail(HXB_E_DEVICE, "device error word %d (a bounded wait gave up)", word);
}

// Every expert resident: the whole range is device work only (capturable).
static int enqueue_resident(hxb_moe *m, float *h, float *out, int T, int l0, int nl, bool with_norm, bool resid,
                            cudaStream_t s) {
    const MoeScratch sc = m->scratch();
    const MoeShape sh = m->shape(T);
    for (int l = l0; l < l0 + nl; l++) {
        const MoeLayerDev L = m->layer_dev(l, with_norm);
        if (!cuda_ok(launch_moe_layer(sh, L, sc, h, out, resid, s), "moe layer")) return HXB_E_DEVICE;
    }
    return HXB_OK;
}

// Experts may be missing from HBM: route on the device, read the bucket list back, acquire the
// experts from the store (copies on its copy stream, waited for on the device), then run them.
static int run_streaming(hxb_moe *m, float *h, float *out, int T, int l0, int nl, bool with_norm, bool resid,
                         cudaStream_t s, const int *forced = nullptr) {
    MoeScratch sc = m->scratch();
    const MoeShape sh = m->shape(T);
    const int E = m->cfg.n_experts;
    for (int l = l0; l < l0 + nl; l++) {
        const MoeLayerDev L = m->layer_dev(l, with_norm);
        sc.forced_ids = forced ? forced + (size_t)(l - l0) * T * m->cfg.top_k : nullptr;
        if (!cuda_ok(launch_moe_route(sh, L, sc, h, s), "route")) return HXB_E_DEVICE;
        int *nu_h = m->epin + 1, *ul_h = m->epin + 8, *un_h = m->epin + 8 + E;
        bool ok = cuda_ok(cudaMemcpyAsync(nu_h, sc.nu, sizeof(int), cudaMemcpyDeviceToHost, s), "nu") &&
                  cuda_ok(cudaMemcpyAsync(ul_h, sc.ulist, sizeof(int) * (size_t)E, cudaMemcpyDeviceToHost, s), "ulist") &&
                  cuda_ok(cudaMemcpyAsync(un_h, sc.u_n, sizeof(int) * (size_t)E, cudaMemcpyDeviceToHost, s), "u_n") &&
                  cuda_ok(cudaMemcpyAsync(m->epin, sc.err, sizeof(int), cudaMemcpyDeviceToHost, s), "err");
        const double t0 = now_s();
        ok = ok && cuda_ok(cudaStreamSynchronize(s), "route sync");
        m->st.stall_s += now_s() - t0;
        if (!ok) return HXB_E_DEVICE;
        if (m->epin[0]) return take_device_error(m, m->epin[0]);
        const int nu = *nu_h;
        std::vector<int> got;
        int rc = HXB_OK;
        for (int u = 0; u < nu; u++) {
            const int e = ul_h[u];
            cudaEvent_t ev = nullptr;
            const uint8_t *p = m->store.acquire_async(l, e, &ev);
            if (!p) {
                rc = fail(HXB_E_IO, "layer %d expert %d could not be brought into HBM", l, e);
                break;
            }
            got.push_back(e);
            // one use per (token, rank) routed here, as sequential evaluation counts them
            if (un_h[u] > 1) m->store.count_uses(l, e, (uint32_t)(un_h[u] - 1));
            if (ev && !cuda_ok(cudaStreamWaitEvent(s, ev, 0), "wait copy")) {
                rc = HXB_E_DEVICE;
                break;
            }
            m->host_table[(size_t)l * E + e] = p;
        }
        if (rc == HXB_OK &&
            !cuda_ok(cudaMemcpyAsync(m->table.as<const uint8_t *>() + (size_t)l * E, m->host_table + (size_t)l * E,
                                     sizeof(void *) * (size_t)E, cudaMemcpyHostToDevice, s),
                     "table"))
            rc = HXB_E_DEVICE;
        // next-layer prediction (engine/src/model.c:944-973, HEARTH_PREFETCH_NEXT): route layer l+1 with
        // this layer's input h (before this layer's residual) and hand its experts to the store as
        // prefetch hints; their copies follow this layer's demand copies on the copy stream
        const bool predict = rc == HXB_OK && m->pred_ready && !forced && l + 1 < l0 + nl && m->layers[(size_t)l + 1].set;
        int *pnu_h = m->epin + 8 + 2 * E + 0, *pul_h = m->epin + 8 + 2 * E + 1;
        if (predict) {
            const MoeScratch ps = m->pred_scratch();
            if (!cuda_ok(launch_moe_route(sh, m->layer_dev(l + 1, with_norm), ps, h, s), "predict") ||
                !cuda_ok(cudaMemcpyAsync(pnu_h, ps.nu, sizeof(int), cudaMemcpyDeviceToHost, s), "predicted nu") ||
                !cuda_ok(cudaMemcpyAsync(pul_h, ps.ulist, sizeof(int) * (size_t)E, cudaMemcpyDeviceToHost, s),
                         "predicted experts") ||
                !cuda_ok(cudaEventRecord(m->pred_ready, s), "predict event"))
                rc = HXB_E_DEVICE;
        }
        if (rc == HXB_OK && !cuda_ok(launch_moe_experts(sh, L, sc, h, out, resid, s), "experts")) rc = HXB_E_DEVICE;
        if (rc == HXB_OK && predict) {   // the experts run meanwhile; the hints go out as soon as they are known
            if (!cuda_ok(cudaEventSynchronize(m->pred_ready), "predict wait")) rc = HXB_E_DEVICE;
            else m->store.prefetch(l + 1, pul_h, std::min(*pnu_h, E));
        }
        for (int e : got) m->store.release(l, e, s);
        if (rc != HXB_OK) {
            cudaStreamSynchronize(s);   // nothing of this call may still run when it returns
            return rc;
        }
    }
    return HXB_OK;
}

// Device pointer tables of the per-layer dense weights for the persistent kernel.
static bool refresh_decode_tables(hxb_moe *m) {
    if (!m->dec_dirty) return true;
    const int L = m->cfg.n_layers;
    std::vector<const void *> r((size_t)L), n((size_t)L), b((size_t)L);
    for (int l = 0; l < L; l++) {
        r[(size_t)l] = m->layers[(size_t)l].router.p;
        n[(size_t)l] = m->layers[(size_t)l].norm.p;
        b[(size_t)l] = m->cfg.score_bias ? m->layers[(size_t)l].bias.p : nullptr;
    }
    if (!cuda_ok(cudaMemcpy(m->dec_router.p, r.data(), sizeof(void *) * (size_t)L, cudaMemcpyHostToDevice), "tables") ||
        !cuda_ok(cudaMemcpy(m->dec_norm.p, n.data(), sizeof(void *) * (size_t)L, cudaMemcpyHostToDevice), "tables") ||
        !cuda_ok(cudaMemcpy(m->dec_bias.p, b.data(), sizeof(void *) * (size_t)L, cudaMemcpyHostToDevice), "tables"))
        return false;
    m->dec_dirty = false;
    return true;
}

static cudaError_t enqueue_decode(hxb_moe *m, float *h, int l0, int nl, cudaStream_t s) {
    const hxb_moe_config &k = m->cfg;
    DecodeParams p;
    p.n_layers = nl;
    p.D = k.d_model;
    p.F = k.expert_ffn_dim;
    p.E = k.n_experts;
    p.K = k.top_k;
    p.dtype = k.expert_dtype;
    p.route = m->shape(1).route;
    p.eps = k.norm_eps;
    p.rs = k.residual_scale;
    p.off_up = m->lay.off_up;
    p.off_down = m->lay.off_down;
    p.router = m->dec_router.as<const float *>() + l0;
    p.norm = m->dec_norm.as<const float *>() + l0;
    p.bias = m->dec_bias.as<const float *>() + l0;
    p.slab = m->table.as<const uint8_t *>() + (size_t)l0 * k.n_experts;
    p.h = h;
    p.xbuf = m->dec_xbuf.as<float>();
    p.buf_layers = k.n_layers;
    p.epoch = m->dec_epoch.as<unsigned>();
    p.err = m->err.as<int>();
    p.ids_out = m->ids.as<int>();
    p.w_out = m->wts.as<float>();
    p.trace = m->dec_trace.as<unsigned long long>();
    p.ep_size = k.ep_size;
    p.ep_rank = k.ep_rank;
    p.ep_y = k.ep_size > 1 ? m->ep_peers.as<uint64_t *const>() : nullptr;
    return launch_moe_decode(p, s);
}

// After a device error the persistent kernel's exchange buffers may hold values of the failed launch.
static void reset_decode_state(hxb_moe *m) {
    if (!m->use_decode) return;
    cudaDeviceSynchronize();
    cudaMemset(m->dec_xbuf.p, 0xff, m->dec_xbuf.n);
    cudaMemset(m->dec_epoch.p, 0, m->dec_epoch.n);
}

static int run_range(hxb_moe *m, float *h, float *out, int T, int l0, int nl, bool with_norm, bool resid,
                     cudaStream_t user, bool host_io, const float *hin, float *hout) {
    if (m->cfg.ep_size > 1 && !(m->use_decode && m->ep_connected && T == 1 && with_norm && resid && !out))
        return fail(HXB_E_UNSUPPORTED, "an expert-parallel handle evaluates batches through hxb_moe_ep_*, and "
                                       "single tokens once hxb_moe_ep_connect has run");
    cudaStream_t s = user ? user : m->stream;
    const size_t bytes = sizeof(float) * (size_t)T * m->cfg.d_model;
    const double t0 = now_s();
    int rc = HXB_OK;
    if (m->resident_mode && m->use_decode && T == 1 && with_norm && resid && !out && nl <= decode_max_layers()) {
        if (!refresh_decode_tables(m)) return HXB_E_DEVICE;
        float *dh = host_io ? m->hbuf.as<float>() : h;
        if (host_io) {
            std::memcpy(m->hpin, hin, bytes);
            if (!cuda_ok(cudaMemcpyAsync(dh, m->hpin, bytes, cudaMemcpyHostToDevice, s), "h in")) return HXB_E_DEVICE;
        }
        if (!cuda_ok(enqueue_decode(m, dh, l0, nl, s), "decode launch")) return HXB_E_DEVICE;
        if (host_io) {
            if (!cuda_ok(cudaMemcpyAsync(m->hpin, dh, bytes, cudaMemcpyDeviceToHost, s), "h out") ||
                !cuda_ok(cudaMemcpyAsync(m->epin, m->err.p, sizeof(int), cudaMemcpyDeviceToHost, s), "err") ||
                !cuda_ok(cudaStreamSynchronize(s), "sync"))
                return HXB_E_DEVICE;
            rc = take_device_error(m, m->epin[0]);
            if (rc != HXB_OK) {
                reset_decode_state(m);
                return rc;
            }
            std::memcpy(hout, m->hpin, bytes);
        }
    } else if (m->resident_mode) {
        // one CUDA graph per (T, range, buffers): the host copies (host variants) are part of it
        GraphKey key{T, l0 * 2 + (with_norm ? 1 : 0), nl * 2 + (resid ? 1 : 0), host_io ? nullptr : (const void *)h,
                     (cudaStream_t)(uintptr_t)(out ? 1 : 0)};
        if (!host_io) key.s = (cudaStream_t)(uintptr_t)((uintptr_t)out ^ 0x5);
        auto it = m->graphs.find(key);
        if (it == m->graphs.end() && m->graphs.size() >= 256) drop_graphs(m);   // bound the cache
        if (it == m->graphs.end()) {
            cudaGraph_t g = nullptr;
            cudaGraphExec_t ex = nullptr;
            if (!cuda_ok(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "capture")) return HXB_E_DEVICE;
            float *dh = host_io ? m->hbuf.as<float>() : h;
            float *dout = host_io ? (out ? m->obuf.as<float>() : nullptr) : out;
            if (host_io) cudaMemcpyAsync(dh, m->hpin, bytes, cudaMemcpyHostToDevice, m->stream);
            rc = enqueue_resident(m, dh, dout, T, l0, nl, with_norm, resid, m->stream);
            if (host_io) cudaMemcpyAsync(m->hpin, out ? dout : dh, bytes, cudaMemcpyDeviceToHost, m->stream);
            cudaMemcpyAsync(m->epin, m->err.p, sizeof(int), cudaMemcpyDeviceToHost, m->stream);
            const cudaError_t ce = cudaStreamEndCapture(m->stream, &g);
            if (rc != HXB_OK || !cuda_ok(ce, "end capture")) {
                if (g) cudaGraphDestroy(g);
                return rc != HXB_OK ? rc : HXB_E_DEVICE;
            }
            const bool iok = cuda_ok(cudaGraphInstantiate(&ex, g, 0), "instantiate");
            cudaGraphDestroy(g);
            if (!iok) return HXB_E_DEVICE;
            it = m->graphs.emplace(key, ex).first;
        }
        if (host_io) std::memcpy(m->hpin, hin, bytes);
        if (!cuda_ok(cudaGraphLaunch(it->second, s), "graph launch")) return HXB_E_DEVICE;
        if (host_io) {   // device variants stay asynchronous: hxb_moe_sync reports their errors
            if (!cuda_ok(cudaStreamSynchronize(s), "sync")) return HXB_E_DEVICE;
            rc = take_device_error(m, m->epin[0]);
            if (rc == HXB_OK) std::memcpy(hout, m->hpin, bytes);
        }
    } else {
        float *dh = h, *dout = out;
        if (host_io) {
            dh = m->hbuf.as<float>();
            dout = out ? m->obuf.as<float>() : nullptr;
            std::memcpy(m->hpin, hin, bytes);
            if (!cuda_ok(cudaMemcpyAsync(dh, m->hpin, bytes, cudaMemcpyHostToDevice, s), "h in")) return HXB_E_DEVICE;
        }
        rc = run_streaming(m, dh, dout, T, l0, nl, with_norm, resid, s);
        if (rc == HXB_OK && host_io) {
            if (!cuda_ok(cudaMemcpyAsync(m->hpin, out ? dout : dh, bytes, cudaMemcpyDeviceToHost, s), "h out") ||
                !cuda_ok(cudaStreamSynchronize(s), "sync"))
                return HXB_E_DEVICE;
            std::memcpy(hout, m->hpin, bytes);
        } else if (rc == HXB_OK && !user) {
            if (!cuda_ok(cudaStreamSynchronize(s), "sync")) return HXB_E_DEVICE;
        }
    }
    if (rc != HXB_OK) return rc;
    m->st.tokens += (uint64_t)T;
    m->st.forward_calls++;
    m->st.expert_uses += (uint64_t)T * (uint64_t)m->cfg.top_k * (uint64_t)nl;
    m->st.wall_s += now_s() - t0;
    m->last_T = T;
    return HXB_OK;
}

static int check_eval(hxb_moe *m, int T, int l0, int nl) {
    if (!m) return fail(HXB_E_ARG, "null handle");
    if (T <= 0 || l0 < 0 || nl <= 0 || l0 + nl > m->cfg.n_layers) return fail(HXB_E_ARG, "bad token count or layer range");
    if (T > m->cfg.max_tokens) return fail(HXB_E_CAPACITY, "T=%d exceeds max_tokens=%d", T, m->cfg.max_tokens);
    for (int l = l0; l < l0 + nl; l++)
        if (!m->layers[(size_t)l].set) return fail(HXB_E_ARG, "layer %d has no weights", l);
    cudaSetDevice(m->device);
    return HXB_OK;
}

extern "C" HXB_API int hxb_moe_forward(hxb_moe *m, float *h, int T, int layer0, int n_layers) {
    int rc = check_eval(m, T, layer0, n_layers);
    if (rc) return rc;
    if (!h) return fail(HXB_E_ARG, "null h");
    return run_range(m, nullptr, nullptr, T, layer0, n_layers, true, true, nullptr, true, h, h);
}

extern "C" HXB_API int hxb_moe_forward_dev(hxb_moe *m, float *h, int T, int layer0, int n_layers, void *stream) {
    int rc = check_eval(m, T, layer0, n_layers);
    if (rc) return rc;
    if (!h) return fail(HXB_E_ARG, "null h");
    return run_range(m, h, nullptr, T, layer0, n_layers, true, true, (cudaStream_t)stream, false, nullptr, nullptr);
}

// Route replay (hearth_route_replay, engine/src/model.c:1003-1009 and 1885-1959): the layers of
// [layer0, layer0 + n_layers) with every token's K expert ids given (ids [n_layers][T][K], host), the
// scores and weights computed as usual. Synchronous, host h in place; never the persistent kernel.
extern "C" HXB_API int hxb_moe_forward_routed(hxb_moe *m, float *h, int T, int layer0, int n_layers, const int *ids) {
    int rc = check_eval(m, T, layer0, n_layers);
    if (rc) return rc;
    if (!h || !ids) return fail(HXB_E_ARG, "forward_routed: null h or ids");
    if (m->cfg.ep_size > 1) return fail(HXB_E_UNSUPPORTED, "forward_routed: not on an expert-parallel handle");
    const int K = m->cfg.top_k, E = m->cfg.n_experts;
    const size_t n = (size_t)n_layers * T * K;
    for (size_t i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= E) return fail(HXB_E_ARG, "forward_routed: expert id %d outside [0, %d)", ids[i], E);
    cudaStream_t s = m->stream;
    const size_t bytes = sizeof(float) * (size_t)T * m->cfg.d_model;
    const double t0 = now_s();
    float *dh = m->hbuf.as<float>();
    std::memcpy(m->hpin, h, bytes);
    if (!cuda_ok(cudaMemcpyAsync(dh, m->hpin, bytes, cudaMemcpyHostToDevice, s), "h in") ||
        !cuda_ok(cudaMemcpyAsync(m->forced.p, ids, sizeof(int) * n, cudaMemcpyHostToDevice, s), "ids in"))
        return HXB_E_DEVICE;
    const int *fd = m->forced.as<int>();
    if (m->resident_mode) {
        MoeScratch sc = m->scratch();
        for (int l = layer0; l < layer0 + n_layers; l++) {
            sc.forced_ids = fd + (size_t)(l - layer0) * T * K;
            if (!cuda_ok(launch_moe_layer(m->shape(T), m->layer_dev(l, true), sc, dh, nullptr, true, s), "layer"))
                return HXB_E_DEVICE;
        }
    } else {
        rc = run_streaming(m, dh, nullptr, T, layer0, n_layers, true, true, s, fd);
        if (rc != HXB_OK) return rc;
    }
    if (!cuda_ok(cudaMemcpyAsync(m->hpin, dh, bytes, cudaMemcpyDeviceToHost, s), "h out") ||
        !cuda_ok(cudaMemcpyAsync(m->epin, m->err.p, sizeof(int), cudaMemcpyDeviceToHost, s), "err") ||
        !cuda_ok(cudaStreamSynchronize(s), "sync"))
        return HXB_E_DEVICE;
    rc = take_device_error(m, m->epin[0]);
    if (rc != HXB_OK) return rc;
    std::memcpy(h, m->hpin, bytes);
    m->st.tokens += (uint64_t)T;
    m->st.forward_calls++;
    m->st.expert_uses += (uint64_t)T * (uint64_t)K * (uint64_t)n_layers;
    m->st.wall_s += now_s() - t0;
    m->last_T = T;
    return HXB_OK;
}

// ---- inside the library: the MoE layers of a whole-model handle (hx_model.cu)

namespace hx {

int moe_layer_for_model(hxb_moe *m, float *h, int T, int l, cudaStream_t s, const int *forced) {
    int rc = check_eval(m, T, l, 1);
    if (rc) return rc;
    if (m->cfg.ep_size > 1) return fail(HXB_E_UNSUPPORTED, "whole-model evaluation on an expert-parallel handle");
    if (m->resident_mode) {
        if (m->use_decode && T == 1 && !forced) {
            if (!refresh_decode_tables(m)) return HXB_E_DEVICE;
            if (!cuda_ok(enqueue_decode(m, h, l, 1, s), "decode launch")) return HXB_E_DEVICE;
        } else {
            MoeScratch sc = m->scratch();
            sc.forced_ids = forced;
            if (!cuda_ok(launch_moe_layer(m->shape(T), m->layer_dev(l, true), sc, h, nullptr, true, s), "moe layer"))
                return HXB_E_DEVICE;
        }
    } else {
        rc = run_streaming(m, h, nullptr, T, l, 1, true, true, s, forced);
        if (rc != HXB_OK) return rc;
    }
    m->st.expert_uses += (uint64_t)T * (uint64_t)m->cfg.top_k;
    m->last_T = T;
    return HXB_OK;
}

const int *moe_ids_dev(const hxb_moe *m) { return m->ids.as<int>(); }
bool moe_resident(const hxb_moe *m) { return m->resident_mode; }
const int *moe_err_dev(const hxb_moe *m) { return m->err.as<int>(); }
int moe_take_error(hxb_moe *m, int word) { return take_device_error(m, word); }

}  // namespace hx

extern "C" HXB_API int hxb_moe_layer(hxb_moe *m, int layer, const float *x, int T, float *out) {
    int rc = check_eval(m, T, layer, 1);
    if (rc) return rc;
    if (!x || !out) return fail(HXB_E_ARG, "null buffer");
    return run_range(m, nullptr, m->obuf.as<float>(), T, layer, 1, false, false, nullptr, true, x, out);
}

extern "C" HXB_API int hxb_moe_layer_dev(hxb_moe *m, int layer, const float *x, int T, float *out, void *stream) {
    int rc = check_eval(m, T, layer, 1);
    if (rc) return rc;
    if (!x || !out) return fail(HXB_E_ARG, "null buffer");
    return run_range(m, const_cast<float *>(x), out, T, layer, 1, false, false, (cudaStream_t)stream, false, nullptr,
                     nullptr);
}

extern "C" HXB_API int hxb_moe_last_routing(hxb_moe *m, int *ids, float *weights, int T) {
    if (!m || T <= 0 || T > m->last_T) return fail(HXB_E_ARG, "last_routing: bad arguments");
    const size_t n = (size_t)T * m->cfg.top_k;
    cudaSetDevice(m->device);
    if (ids && !cuda_ok(cudaMemcpy(ids, m->ids.p, sizeof(int) * n, cudaMemcpyDeviceToHost), "ids")) return HXB_E_DEVICE;
    if (weights && !cuda_ok(cudaMemcpy(weights, m->wts.p, sizeof(float) * n, cudaMemcpyDeviceToHost), "wts"))
        return HXB_E_DEVICE;
    return HXB_OK;
}

extern "C" HXB_API int hxb_moe_get_stats(hxb_moe *m, hxb_moe_stats *out) {
    if (!m || !out) return fail(HXB_E_ARG, "get_stats: bad arguments");
    *out = m->st;
    const StoreStats ss = m->store.stats();
    if (m->resident_mode) {
        out->hits = out->expert_uses;
        out->misses = 0;
    } else {
        out->hits = ss.hits;
        out->misses = ss.misses;
    }
    out->evictions = ss.evictions;
    out->prefetch_issued = ss.prefetch_issued;
    out->prefetch_used = ss.prefetch_used;
    out->prefetch_wasted = ss.prefetch_wasted;
    out->bytes_copied = ss.bytes_copied;
    out->copies = ss.copies;
    out->copy_errors = ss.copy_errors;
    out->n_slots = m->store.n_slots();
    out->resident = m->store.n_ready();
    out->pinned = m->store.n_pinned();
    out->slot_bytes = m->slab_bytes;
    out->host_bytes = (uint64_t)m->store.host_bytes();
    return HXB_OK;
}

extern "C" HXB_API void hxb_moe_reset_stats(hxb_moe *m) {
    if (!m) return;
    const int ns = m->st.n_slots;
    m->st = hxb_moe_stats();
    m->st.n_slots = ns;
    m->store.reset_stats();
}

extern "C" HXB_API int hxb_moe_is_resident(hxb_moe *m, int layer, int expert) {
    if (!m || layer < 0 || layer >= m->cfg.n_layers || expert < 0 || expert >= m->cfg.n_experts) return 0;
    return m->store.is_resident(layer, expert) ? 1 : 0;
}

extern "C" HXB_API void hxb_moe_tick(hxb_moe *m) {
    if (m) m->store.tick();
}

extern "C" HXB_API int hxb_moe_prefetch(hxb_moe *m, int layer, const int *experts, int n) {
    if (!m || layer < 0 || layer >= m->cfg.n_layers || n < 0 || (n && !experts)) return fail(HXB_E_ARG, "prefetch: bad arguments");
    cudaSetDevice(m->device);
    m->store.prefetch(layer, experts, n);
    return HXB_OK;
}

extern "C" HXB_API int hxb_moe_seed_heat(hxb_moe *m, const float *counts, int n_keys, float pin_fraction,
                                         int warm_start) {
    if (!m || !counts || n_keys != m->cfg.n_layers * m->cfg.n_experts) return fail(HXB_E_ARG, "seed_heat: bad arguments");
    cudaSetDevice(m->device);
    m->store.seed_heat(counts, n_keys, pin_fraction, warm_start != 0);
    cudaStreamSynchronize(m->store.copy_stream());
    return HXB_OK;
}

extern "C" HXB_API void hxb_moe_set_copy_hook(hxb_moe *m, hxb_copy_hook fn, void *ctx) {
    if (!m) return;
    if (!fn) m->store.set_copy_hook(nullptr);
    else m->store.set_copy_hook([fn, ctx](int layer, int expert) { return fn(ctx, layer, expert); });
}

extern "C" HXB_API int hxb_moe_sync(hxb_moe *m, void *stream) {
    if (!m) return fail(HXB_E_ARG, "sync: null handle");
    cudaSetDevice(m->device);
    cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
    if (!cuda_ok(cudaStreamSynchronize(s), "sync")) return HXB_E_DEVICE;
    int word = 0;
    if (!cuda_ok(cudaMemcpy(&word, m->err.p, sizeof word, cudaMemcpyDeviceToHost), "error word")) return HXB_E_DEVICE;
    if (word) reset_decode_state(m);
    return take_device_error(m, word);
}

// Per-kernel device times of one resident layer evaluation (eager launches bracketed by CUDA
// events on the handle's stream, averaged over iters x layers): us[0] norm+activation,
// us[1] router+routing, us[2] gate/up+SwiGLU, us[3] down+rank-order sum. For roofline accounting;
// the graph path runs the same kernels back to back.
extern "C" HXB_API int hxb_moe_profile(hxb_moe *m, int T, int iters, double *us) {
    int rc = check_eval(m, T, 0, m ? m->cfg.n_layers : 1);
    if (rc) return rc;
    if (!m->resident_mode || iters <= 0 || !us) return fail(HXB_E_ARG, "profile: needs every expert resident");
    const MoeScratch sc = m->scratch();
    const MoeShape sh = m->shape(T);
    cudaEvent_t ev[5];
    for (auto &e : ev) cudaEventCreate(&e);
    double acc[4] = {0, 0, 0, 0};
    float *h = m->hbuf.as<float>();
    cudaMemsetAsync(h, 0, sizeof(float) * (size_t)T * m->cfg.d_model, m->stream);
    launch_synth_f32(h, (int64_t)T * m->cfg.d_model, 77, 1.0f, m->stream);
    int n = 0;
    for (int it = 0; it < iters; it++)
        for (int l = 0; l < m->cfg.n_layers; l++) {
            const MoeLayerDev L = m->layer_dev(l, true);
            cudaEventRecord(ev[0], m->stream);
            launch_moe_stage(0, sh, L, sc, h, nullptr, true, m->stream);
            cudaEventRecord(ev[1], m->stream);
            launch_moe_stage(1, sh, L, sc, h, nullptr, true, m->stream);
            cudaEventRecord(ev[2], m->stream);
            launch_moe_stage(2, sh, L, sc, h, nullptr, true, m->stream);
            cudaEventRecord(ev[3], m->stream);
            launch_moe_stage(3, sh, L, sc, h, nullptr, true, m->stream);
            cudaEventRecord(ev[4], m->stream);
            if (!cuda_ok(cudaEventSynchronize(ev[4]), "profile")) return HXB_E_DEVICE;
            for (int k = 0; k < 4; k++) {
                float ms = 0;
                cudaEventElapsedTime(&ms, ev[k], ev[k + 1]);
                acc[k] += ms * 1000.0;
            }
            n++;
        }
    for (auto &e : ev) cudaEventDestroy(e);
    for (int k = 0; k < 4; k++) us[k] = acc[k] / n;
    int word = 0;
    cudaMemcpy(&word, m->err.p, sizeof word, cudaMemcpyDeviceToHost);
    return take_device_error(m, word);
}

// Expert parallelism, step 1: routing of every token and this rank's pairs' outputs into y.
extern "C" HXB_API int hxb_moe_ep_layer_dev(hxb_moe *m, int layer, const float *h, int T, float *y, void *stream) {
    if (!m || layer < 0 || layer >= m->cfg.n_layers || T <= 0 || T > m->cfg.max_tokens || !h || !y)
        return fail(HXB_E_ARG, "ep_layer: bad arguments");
    if (!m->layers[(size_t)layer].set) return fail(HXB_E_ARG, "ep_layer: layer %d has no weights", layer);
    cudaSetDevice(m->device);
    const int E = m->cfg.n_experts;
    for (int e = 0; e < E; e++)
        if (m->owns(e) && !m->host_table[(size_t)layer * E + e])
            return fail(HXB_E_IO, "ep_layer: expert %d of layer %d is not in HBM", e, layer);
    MoeScratch sc = m->scratch();
    sc.Y = y;
    const MoeShape sh = m->shape(T);
    const MoeLayerDev L = m->layer_dev(layer, true);
    if (!cuda_ok(launch_moe_layer(sh, L, sc, const_cast<float *>(h), nullptr, false, (cudaStream_t)stream),
                 "ep layer"))
        return HXB_E_DEVICE;
    m->st.expert_uses += (uint64_t)T * m->cfg.top_k;
    return HXB_OK;
}

// Expert parallelism, step 2: rank-order sum over the gathered outputs, shared expert, residual.
extern "C" HXB_API int hxb_moe_ep_combine_dev(hxb_moe *m, int layer, const float *y_all, int T, float *h,
                                              void *stream) {
    if (!m || layer < 0 || layer >= m->cfg.n_layers || T <= 0 || T > m->cfg.max_tokens || !h || !y_all)
        return fail(HXB_E_ARG, "ep_combine: bad arguments");
    cudaSetDevice(m->device);
    if (!cuda_ok(launch_moe_ep_combine(m->shape(T), m->layer_dev(layer, true), m->scratch(), y_all, h,
                                       (cudaStream_t)stream),
                 "ep combine"))
        return HXB_E_DEVICE;
    return HXB_OK;
}

// Expert parallelism in the persistent decode kernel: this GPU's y-word buffer as a CUDA IPC handle
// (64 bytes), for the other ranks' hxb_moe_ep_connect.
extern "C" HXB_API int hxb_moe_ep_ipc_handle(hxb_moe *m, void *handle) {
    if (!m || !handle) return fail(HXB_E_ARG, "ep_ipc_handle: bad arguments");
    if (m->cfg.ep_size <= 1 || !m->ep_y.p) return fail(HXB_E_UNSUPPORTED, "ep_ipc_handle: not an expert-parallel decode handle");
    cudaSetDevice(m->device);
    cudaIpcMemHandle_t h;
    if (!cuda_ok(cudaIpcGetMemHandle(&h, m->ep_y.p), "ipc handle")) return HXB_E_DEVICE;
    std::memcpy(handle, &h, sizeof h);
    return HXB_OK;
}

// handles [ep_size][64]: every rank's hxb_moe_ep_ipc_handle (this rank's own entry is ignored).
extern "C" HXB_API int hxb_moe_ep_connect(hxb_moe *m, const void *handles) {
    if (!m || !handles) return fail(HXB_E_ARG, "ep_connect: bad arguments");
    const int N = m->cfg.ep_size;
    if (N <= 1 || !m->ep_y.p || N > 64) return fail(HXB_E_UNSUPPORTED, "ep_connect: not an expert-parallel decode handle");
    if (m->ep_connected) return HXB_OK;
    cudaSetDevice(m->device);
    std::vector<void *> ptrs((size_t)N, nullptr);
    for (int r = 0; r < N; r++) {
        if (r == m->cfg.ep_rank) {
            ptrs[(size_t)r] = m->ep_y.p;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)r * sizeof h, sizeof h);
        void *p = nullptr;
        if (!cuda_ok(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "ipc open")) return HXB_E_DEVICE;
        m->ep_opened.push_back(p);
        ptrs[(size_t)r] = p;
    }
    if (!cuda_ok(cudaMemcpy(m->ep_peers.p, ptrs.data(), sizeof(void *) * (size_t)N, cudaMemcpyHostToDevice), "peers"))
        return HXB_E_DEVICE;
    m->ep_connected = true;
    return HXB_OK;
}

extern "C" HXB_API int hxb_moe_decode_path(const hxb_moe *m) {
    if (!m) return HXB_E_ARG;
    return m->use_decode ? 1 : 0;
}

// Phase timeline of the last persistent decode launch (handles opened with HXB_TRACE=1):
// out[layer][cta][stamp] SM clock cycles; returns the number of values (0 without a trace).
extern "C" HXB_API int64_t hxb_moe_phase_trace(hxb_moe *m, uint64_t *out, int64_t max_values) {
    if (!m || !m->dec_trace.p) return 0;
    const int64_t n = (int64_t)(m->dec_trace.n / sizeof(unsigned long long));
    if (!out || max_values < n) return n;
    cudaSetDevice(m->device);
    if (cudaMemcpy(out, m->dec_trace.p, sizeof(uint64_t) * (size_t)n, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return n;
}

// ------------------------------------------------------------------------------- .hearth containers

extern "C" HXB_API int hxb_container_probe(const char *path, hxb_moe_config *cfg, hxb_container_info *info, char *err,
                                           size_t errlen) {
    if (!path) {
        set_errbuf(err, errlen, "hxb_container_probe: null path");
        return HXB_E_ARG;
    }
    ContainerFile f;
    std::string why;
    if (!f.open(path, why)) {
        set_errbuf(err, errlen, "hxb_container_probe: " + why);
        struct stat st;
        return stat(path, &st) == 0 ? HXB_E_FORMAT : HXB_E_IO;
    }
    const Container &c = f.info();
    if (cfg) {
        hxb_moe_default_config(cfg);
        cfg->n_layers = (int)c.n_layers;
        cfg->d_model = (int)c.d_model;
        cfg->expert_ffn_dim = (int)c.expert_ffn_dim;
        cfg->n_experts = (int)c.n_experts;
        cfg->top_k = (int)c.top_k;
        cfg->score_fn = (int)c.score_fn;
        cfg->score_bias = (int)c.score_bias;
        cfg->n_group = (int)c.n_group;
        cfg->topk_group = (int)c.topk_group;
        cfg->norm_topk_prob = (int)c.norm_topk_prob;
        cfg->routed_scale = c.routed_scale;
        cfg->residual_scale = c.residual_scale;
        cfg->norm_eps = c.norm_eps;
        if (c.expert_dtype >= 0) cfg->expert_dtype = c.expert_dtype;
        cfg->shared_ffn_dim = (int)c.shared_ffn_dim;
        cfg->shared_gate = (int)c.shared_gate;
        for (uint32_t l = 0; l < c.n_layers && c.shared_ffn_dim; l++) {   // the shared expert's dtype
            const CtTensor *t = c.find("blk." + std::to_string(l) + ".shexp_gate");
            if (c.layer_kind[l] && t) {
                cfg->shared_dtype = (int)t->dtype;
                break;
            }
        }
    }
    if (info) {
        info->n_layers = (int)c.n_layers;
        info->n_moe_layers = c.n_moe_layers;
        info->n_expert_entries = (int)c.experts.size();
        info->n_physical_slabs = c.n_physical;
        info->n_aliased = c.n_aliased;
        info->expert_dtype = c.expert_dtype;
        info->slab_bytes = 0;
        for (const CtExpert &x : c.experts)
            if (x.nbytes) {
                info->slab_bytes = x.nbytes;
                break;
            }
    }
    return HXB_OK;
}

// Float settings compared bit for bit: the kernels compute with exactly these values.
static bool same_bits(float a, float b) { return std::memcmp(&a, &b, sizeof a) == 0; }

extern "C" HXB_API int hxb_moe_load_container(hxb_moe *m, const char *path) {
    if (!m || !path) return fail(HXB_E_ARG, "load_container: bad arguments");
    ContainerFile f;
    std::string why;
    if (!f.open(path, why)) {
        struct stat st;
        return fail(stat(path, &st) == 0 ? HXB_E_FORMAT : HXB_E_IO, "load_container: %s", why.c_str());
    }
    const Container &c = f.info();
    const hxb_moe_config &k = m->cfg;
    const char *diff = nullptr;
    if ((int)c.n_layers != k.n_layers) diff = "n_layers";
    else if ((int)c.d_model != k.d_model) diff = "d_model";
    else if ((int)c.n_experts != k.n_experts || (int)c.top_k != k.top_k) diff = "n_experts / top_k";
    else if ((int)c.expert_ffn_dim != k.expert_ffn_dim) diff = "expert_ffn_dim";
    else if ((int)c.score_fn != k.score_fn || (int)c.score_bias != k.score_bias || (int)c.n_group != k.n_group ||
             (int)c.topk_group != k.topk_group || (int)c.norm_topk_prob != k.norm_topk_prob ||
             !same_bits(c.routed_scale, k.routed_scale))
        diff = "routing";
    else if ((int)c.shared_ffn_dim != k.shared_ffn_dim || (int)c.shared_gate != k.shared_gate) diff = "shared expert";
    else if (!same_bits(c.norm_eps, k.norm_eps)) diff = "norm_eps";
    else if (!same_bits(c.residual_scale, k.residual_scale)) diff = "residual_scale";
    if (diff) return fail(HXB_E_ARG, "load_container: the handle and the container disagree on %s", diff);
    if (c.n_moe_layers && c.expert_dtype != k.expert_dtype)
        return fail(HXB_E_UNSUPPORTED, "load_container: slabs must all have the handle's expert dtype");
    const size_t D = (size_t)k.d_model, E = (size_t)k.n_experts;

    // dense per-layer weights of every MoE layer
    auto tensor = [&](uint32_t l, const char *name, uint32_t dtype, uint64_t nbytes, std::vector<uint8_t> &out,
                      bool required) -> int {
        const CtTensor *t = c.find("blk." + std::to_string(l) + "." + name);
        if (!t) {
            out.clear();
            return required ? fail(HXB_E_FORMAT, "load_container: layer %u has no %s", l, name) : HXB_OK;
        }
        if ((dtype != ~0u && t->dtype != dtype) || t->nbytes != nbytes)
            return fail(HXB_E_UNSUPPORTED, "load_container: layer %u %s has dtype %u and %llu bytes (expected %llu)", l,
                        name, t->dtype, (unsigned long long)t->nbytes, (unsigned long long)nbytes);
        out.resize(nbytes);
        if (!f.read(t->off, out.data(), nbytes, why)) return fail(HXB_E_IO, "load_container: %s", why.c_str());
        return HXB_OK;
    };
    std::vector<uint8_t> router, bias, norm, sg, su, sd, sgi;
    const size_t Fs = (size_t)k.shared_ffn_dim;
    const uint64_t shb = Fs ? (uint64_t)row_bytes(k.shared_dtype, (int64_t)D) * Fs : 0;
    const uint64_t shd = Fs ? (uint64_t)row_bytes(k.shared_dtype, (int64_t)Fs) * D : 0;
    for (uint32_t l = 0; l < c.n_layers; l++) {
        if (!c.layer_kind[l]) continue;
        int rc;
        if ((rc = tensor(l, "moe_router", 0, 4 * E * D, router, true)) != HXB_OK ||
            (rc = tensor(l, "moe_router_bias", 0, 4 * E, bias, k.score_bias != 0)) != HXB_OK ||
            (rc = tensor(l, "ffn_norm", 0, 4 * D, norm, true)) != HXB_OK)
            return rc;
        if (Fs && ((rc = tensor(l, "shexp_gate", (uint32_t)k.shared_dtype, shb, sg, true)) != HXB_OK ||
                   (rc = tensor(l, "shexp_up", (uint32_t)k.shared_dtype, shb, su, true)) != HXB_OK ||
                   (rc = tensor(l, "shexp_down", (uint32_t)k.shared_dtype, shd, sd, true)) != HXB_OK ||
                   (k.shared_gate && (rc = tensor(l, "shexp_gate_inp", 0, 4 * D, sgi, true)) != HXB_OK)))
            return rc;
        rc = hxb_moe_set_layer(m, (int)l, reinterpret_cast<const float *>(router.data()),
                               k.score_bias ? reinterpret_cast<const float *>(bias.data()) : nullptr,
                               reinterpret_cast<const float *>(norm.data()), Fs ? sg.data() : nullptr,
                               Fs ? su.data() : nullptr, Fs ? sd.data() : nullptr,
                               Fs && k.shared_gate ? reinterpret_cast<const float *>(sgi.data()) : nullptr);
        if (rc != HXB_OK) return rc;
    }

    // expert slabs: each physical slab read once, in file order; the entries naming it share one host
    // copy (hxb_moe_share_expert)
    std::vector<size_t> order;
    for (size_t i = 0; i < c.experts.size(); i++)
        if (c.experts[i].nbytes) order.push_back(i);
    std::sort(order.begin(), order.end(),
              [&](size_t a, size_t b) { return c.experts[a].off < c.experts[b].off || (c.experts[a].off == c.experts[b].off && a < b); });
    std::vector<uint8_t> slab;
    for (size_t q = 0; q < order.size();) {
        size_t q1 = q;
        bool wanted = false;
        while (q1 < order.size() && c.experts[order[q1]].off == c.experts[order[q]].off) {
            wanted = wanted || m->owns((int)(order[q1] % E));
            q1++;
        }
        if (wanted) {
            const CtExpert &x = c.experts[order[q]];
            slab.resize(x.nbytes);
            if (!f.read(x.off, slab.data(), x.nbytes, why)) return fail(HXB_E_IO, "load_container: %s", why.c_str());
            int first = -1;   // the first entry this handle holds gets the bytes; the others share them
            for (size_t r = q; r < q1; r++) {
                const int l = (int)(order[r] / E), e = (int)(order[r] % E);
                if (!m->owns(e)) continue;
                const int rc = first < 0 ? hxb_moe_set_expert(m, l, e, slab.data(), x.nbytes)
                                         : hxb_moe_share_expert(m, l, e, first / (int)E, first % (int)E);
                if (rc != HXB_OK) return rc;
                if (first < 0) first = (int)order[r];
            }
        }
        q = q1;
    }
    return HXB_OK;
}
