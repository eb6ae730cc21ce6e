// hx_model.cu — the whole decoder on the GPU (hxb_model_*): embedding, GQA/MHA attention with an
// f32 KV cache in HBM, dense SwiGLU FFN layers, the MoE layers through the MoE backend handle
// (hx_capi.cu), the output norm and the LM head. The order of every float operation is the
// reference's (engine/src/model.c:386-629 and 1133-1236; docs/NUMERICS.md §1-§5), so the logits
// equal hearth_eval's bit for bit.
#include "../../include/hearth_b200.h"
#include "hx_container.h"
#include "hx_device.cuh"
#include "hx_kernels.h"
#include "hx_moe_internal.h"
#include "hx_route.cuh"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace hx {
void set_last_error(const char *msg);
}

namespace {

using namespace hx;

int mfail(int code, const char *f, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, f);
    vsnprintf(buf, sizeof buf, f, ap);
    va_end(ap);
    set_last_error(buf);
    return code;
}

bool mcuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    mfail(HXB_E_DEVICE, "%s: %s", what, cudaGetErrorString(e));
    return false;
}

struct Buf {
    void *p = nullptr;
    size_t n = 0;
    bool alloc(size_t bytes) {
        release();
        if (!bytes) bytes = 16;
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

// A matrix [rows, cols] of any dtype in HBM (FORMAT §4 rows).
struct Mat {
    Buf w;
    int dtype = -1;
    int64_t rows = 0, cols = 0, rb = 0;
};

struct DLayer {
    bool moe = false;
    Buf attn_norm, ffn_norm, bq, bk, bv, qn, kn;
    Mat q, k, v, o, gate, up, down;
    Mat qkv;   // q, k and v rows in one matrix when they share a dtype (one launch for the three)
};

// The host libm's cosf / sinf as separate calls, as the reference makes them
// (engine/src/model.c:201-202): never fused into a sincos.
__attribute__((noinline)) float libm_cosf(float x) { return cosf(x); }
__attribute__((noinline)) float libm_sinf(float x) { return sinf(x); }

}  // namespace

struct hxb_model {
    int device = 0;
    cudaStream_t stream = nullptr;
    hxb_moe *moe = nullptr;
    // shape (engine/src/model.c:1394-1439 setup_dims, GQA)
    int L = 0, D = 0, V = 0, H = 0, Hkv = 0, hd = 0, q_dim = 0, kv_dim = 0, rope_dim = 0, rope_half = 0;
    int rope_style = 0, qk_norm = 0, qkv_bias = 0, Fd = 0, n_moe = 0, K = 0, E = 0, max_in = 0, dc = 64, vthreads = 0;
    size_t vsmem = 0, vsmem1 = 0;   // value kernel: batches, one decode token
    int vnst1 = 0;                  // one decode token: ring stages, softmax fused
    bool vfuse1 = false;
    float eps = 1e-6f, rs = 1.0f, es = 1.0f, ls = 1.0f, attn_scale = 1.0f, rope_factor = 1.0f;
    int max_batch = 0, max_seq = 0, kv_seq = 0;   // kv_seq: max_seq rounded up to 32, the cache's stride
    std::vector<float> inv_freq;
    Mat tok_embd, lm_head;
    Buf out_norm;
    std::vector<DLayer> layers;
    std::vector<int> moe_index;
    Buf kc, vc;                                      // [L][Hkv][max_seq][hd] f32
    Buf tok, h, x, act, q, kk, S, att, f1, f2, logits, cs, routes, forced, dpos;   // q: [T][q|k|v]
    int32_t *tok_pin = nullptr;
    float *logit_pin = nullptr;
    int next_pos = -1;                               // the device position counter's value, if known
    bool resident = false;                           // every expert in HBM: a forward is device work only
    bool warm = false;                               // a single-token forward ran (tables settled)
    bool graphs_ok = true;
    cudaGraphExec_t graph[3] = {nullptr, nullptr, nullptr};   // single-token forward per mode
    int *route_pin = nullptr, *forced_pin = nullptr, *err_pin = nullptr;
    std::vector<uint16_t> replay;
    int replay_rows = 0;
    int last_T = 0;
};

namespace hx {
namespace {

// ---------------------------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------------------------

// h[t] = emb_scale * dequant(tok_embd[tok[t]]) (model.c:1178-1182); a NaN element stays as the
// host's multiply leaves it.
__global__ void k_embed(const int32_t *__restrict__ tok, int T, const uint8_t *__restrict__ W, int dtype, int64_t rb,
                        int D, int V, float es, float *__restrict__ h) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * D) return;
    const int64_t t = i / D, c = i - t * D;
    const int id = tok[t];
    if (id < 0 || id >= V) {   // the host entry points refuse such ids; device ids give a NaN row
        h[i] = __uint_as_float(CANON_NAN);
        return;
    }
    const float v = dequant_elem(dtype, W + (int64_t)id * rb, c);
    h[i] = v != v ? v : __fmul_rn(es, v);
}

// y = rmsnorm(x, w) per row (NUMERICS §4: ms = dot16(x, x) / n, r = 1 / sqrtf(ms + eps),
// y_i = (x_i * r) * w_i), optionally y's activation blocks. One CTA per row, the row in shared memory.
__global__ void __launch_bounds__(256) k_rmsnorm_rows(const float *__restrict__ x, int64_t ldx,
                                                      const float *__restrict__ w, int n, float eps,
                                                      float *__restrict__ y, int64_t ldy, act_q8 *__restrict__ act) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float rsh;
    const int t = blockIdx.x, tid = threadIdx.x;
    const float *xr = x + (int64_t)t * ldx;
    if (n % 4 == 0 && ldx % 4 == 0) {   // 16-byte loads, several in flight per thread
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        float4 *s4 = reinterpret_cast<float4 *>(xs);
#pragma unroll 4
        for (int i = tid; i < n / 4; i += blockDim.x) s4[i] = x4[i];
    } else {
        for (int i = tid; i < n; i += blockDim.x) xs[i] = xr[i];
    }
    __syncthreads();
    if (tid < 16) {
        float L = 0.0f;
        for (int i = tid; i < n; i += 16) L = __fadd_rn(L, __fmul_rn(xs[i], xs[i]));
        L = tree16(L, 0xffffu);
        if (tid == 0) rsh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(L, (float)n), eps)));
    }
    __syncthreads();
    const float r = rsh;
#pragma unroll 4
    for (int i = tid; i < n; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], r), w[i]);
    __syncthreads();
    if (y) {
        float *yr = y + (int64_t)t * ldy;
        for (int i = tid; i < n; i += blockDim.x) yr[i] = xs[i];
    }
    if (act) {
        const int warp = tid >> 5, lane = tid & 31, nb = n / QK;
        for (int b = warp; b < nb; b += blockDim.x >> 5)
            act_quant_warp(xs[b * QK + lane], xs[b * QK + lane + 32], act + (int64_t)t * nb + b, lane);
    }
}

struct PostArgs {
    const float *qkv;                        // [T][ld]: q | k | v of each token
    int64_t ld;
    float *qout;                             // [T][q_dim]: q after bias, qk-norm and RoPE
    const float *bq, *bk, *bv, *qn, *kn;     // biases and qk-norm weights (null when absent)
    const float *cs;                         // [max_seq][rope_dim]: (cos, sin) pairs per position
    float *kc, *vc;                          // this layer's caches: [Hkv][max_seq][hd]
    const int *dpos;                         // position of token 0
    int H, Hkv, hd, qk_norm, rope_half, rope_style, max_seq;
    float eps;
};

// rmsnorm of n values in shared memory with weights w, by the calling warp (lanes 0..15 hold the
// dot16 chains; the result is broadcast to the warp).
__device__ __forceinline__ void warp_rmsnorm(float *x, const float *w, int n, float eps) {
    const int lane = threadIdx.x & 31;
    float L = 0.0f;
    if (lane < 16)
        for (int i = lane; i < n; i += 16) L = __fadd_rn(L, __fmul_rn(x[i], x[i]));
    L = tree16(L, 0xffffffffu);
    const float sum = __shfl_sync(0xffffffffu, L, 0);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)n), eps)));
    __syncwarp();
    for (int i = lane; i < n; i += 32) x[i] = __fmul_rn(__fmul_rn(x[i], r), w[i]);
    __syncwarp();
}

// RoPE of one head's first rope_dim values (NUMERICS §4, model.c:400-411) by the calling warp.
__device__ __forceinline__ void warp_rope(float *x, const float *cs, int half, int style) {
    for (int j = threadIdx.x & 31; j < half; j += 32) {
        const int ia = style == 1 ? 2 * j : j, ib = style == 1 ? 2 * j + 1 : j + half;
        const float a = x[ia], b = x[ib], c = cs[2 * j], s = cs[2 * j + 1];
        x[ia] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        x[ib] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    }
    __syncwarp();
}

// Biases, qk-norm, RoPE, the (k, v) rows into the cache (gqa_post_range, model.c:484-517).
// Per-head qk-norm or none: one warp per head (q heads, then kv heads), 8 heads per CTA, grid
// (tokens, heads / 8). Full-width qk-norm: one CTA per token over the whole q and k rows.
// Shared memory: q [q_dim], k [kv_dim] (full width) or 8 x head_dim (per head).
__global__ void __launch_bounds__(256) k_attn_post(PostArgs a) {
    extern __shared__ float sm[];
    const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int qd = a.H * a.hd, kd = a.Hkv * a.hd;
    const float *qg = a.qkv + (int64_t)t * a.ld;
    const float *kg = qg + qd, *vg = qg + qd + kd;
    float *qo = a.qout + (int64_t)t * qd;
    const int pos = *a.dpos + t;
    const float *cs = a.cs + (int64_t)pos * 2 * a.rope_half;
    if (a.qk_norm != 2) {
        const int hh = blockIdx.y * nw + warp;
        if (hh >= a.H + a.Hkv) return;
        const bool isq = hh < a.H;
        const int off = isq ? hh * a.hd : (hh - a.H) * a.hd;
        const float *src = isq ? qg + off : kg + off;
        const float *bias = isq ? a.bq : a.bk;
        float *x = sm + warp * a.hd;
        for (int i = lane; i < a.hd; i += 32) x[i] = bias ? __fadd_rn(src[i], bias[off + i]) : src[i];
        __syncwarp();
        if (a.qk_norm == 1) warp_rmsnorm(x, isq ? a.qn : a.kn, a.hd, a.eps);
        if (a.rope_half) warp_rope(x, cs, a.rope_half, a.rope_style);
        if (isq) {
            for (int i = lane; i < a.hd; i += 32) qo[off + i] = x[i];
        } else {
            const int g = hh - a.H;
            const int64_t o = ((int64_t)g * a.max_seq + pos) * a.hd;
            for (int i = lane; i < a.hd; i += 32) {
                a.kc[o + i] = x[i];
                a.vc[o + i] = a.bv ? __fadd_rn(vg[off + i], a.bv[off + i]) : vg[off + i];
            }
        }
        return;
    }
    float *q = sm, *k = sm + qd;
    for (int i = tid; i < qd; i += blockDim.x) q[i] = a.bq ? __fadd_rn(qg[i], a.bq[i]) : qg[i];
    for (int i = tid; i < kd; i += blockDim.x) k[i] = a.bk ? __fadd_rn(kg[i], a.bk[i]) : kg[i];
    __syncthreads();
    if (warp == 0) warp_rmsnorm(q, a.qn, qd, a.eps);
    else if (warp == 1) warp_rmsnorm(k, a.kn, kd, a.eps);
    __syncthreads();
    if (a.rope_half)
        for (int hh = warp; hh < a.H + a.Hkv; hh += nw)
            warp_rope(hh < a.H ? q + hh * a.hd : k + (hh - a.H) * a.hd, cs, a.rope_half, a.rope_style);
    __syncthreads();
    for (int i = tid; i < qd; i += blockDim.x) qo[i] = q[i];
    for (int i = tid; i < kd; i += blockDim.x) {
        const int g = i / a.hd, d = i - g * a.hd;
        const int64_t o = ((int64_t)g * a.max_seq + pos) * a.hd + d;
        a.kc[o] = k[i];
        a.vc[o] = a.bv ? __fadd_rn(vg[i], a.bv[i]) : vg[i];
    }
}

// Lane j's chain of a 16-lane dot16 (NUMERICS §1) of a K row with q: k[j] q[j] + k[j+16] q[j+16] + ...
// in order. Rows up to 256 floats load all their values before the chain, so the loads overlap.
__device__ __forceinline__ float qk_chain(const float *kr, const float *q, int n, int j) {
    float L = 0.0f;
    if (n <= 256) {
        float kv[16];
#pragma unroll
        for (int u = 0; u < 16; u++) kv[u] = j + 16 * u < n ? kr[j + 16 * u] : 0.0f;
#pragma unroll
        for (int u = 0; u < 16; u++)
            if (j + 16 * u < n) L = __fadd_rn(L, __fmul_rn(kv[u], q[j + 16 * u]));
    } else {
        for (int i = j; i < n; i += 16) L = __fadd_rn(L, __fmul_rn(kr[i], q[i]));
    }
    return L;
}

// Scores S[t][h][r] = attn_scale * dot16(q_h, k_r) for r <= pos (gqa_scores through the F32
// matmul kernel, then gqa_softmax's scaling; model.c:519-550). One 16-lane group per (h, r); the
// CTAs of a (token, head) stride over the positions.
__global__ void __launch_bounds__(256) k_attn_scores(const float *__restrict__ q, const float *__restrict__ kc,
                                                     float *__restrict__ S, int H, int Hkv, int hd, int max_seq,
                                                     const int *__restrict__ dpos, float scale) {
    const int t = blockIdx.z, h = blockIdx.y, grp = threadIdx.x >> 4, j = threadIdx.x & 15;
    const int pos = *dpos + t;
    const int g = h / (H / Hkv);
    const float *qh = q + ((int64_t)t * H + h) * hd;
    for (int r0 = blockIdx.x * 16; r0 <= pos; r0 += gridDim.x * 16) {
        const int r = r0 + grp;
        const bool valid = r <= pos;
        float L = 0.0f;
        if (valid) {
            L = qk_chain(kc + ((int64_t)g * max_seq + r) * hd, qh, hd, j);
        }
        L = tree16(L, 0xffffffffu);
        if (valid && j == 0) {
            const float s = canon(L);
            S[((int64_t)t * H + h) * max_seq + r] = s != s ? s : __fmul_rn(scale, s);
        }
    }
}

// One token with per-head or no qk-norm: the post-processing folded into the score kernel. Each CTA
// forms its head's q and the token's own k row (bias, qk-norm, RoPE: the same arithmetic as
// k_attn_post) in shared memory, scores the cache rows r < pos and that k row for r = pos; the first
// CTA of each kv group's first head writes the token's (k, v) rows into the cache for later kernels.
__global__ void __launch_bounds__(256) k_attn_scores1(PostArgs a, float *__restrict__ S, float scale) {
    __shared__ float qh[1024], kp[1024];
    const int h = blockIdx.y, grp16 = threadIdx.x >> 4, j = threadIdx.x & 15, warp = threadIdx.x >> 5;
    const int grp = a.H / a.Hkv, g = h / grp;
    const int pos = *a.dpos;
    const int qd = a.H * a.hd, kd = a.Hkv * a.hd;
    const float *qg = a.qkv + h * a.hd, *kg = a.qkv + qd + g * a.hd, *vg = a.qkv + qd + kd + g * a.hd;
    const float *cs = a.cs + (int64_t)pos * 2 * a.rope_half;
    pdl_trigger();
    pdl_wait();   // q|k|v is the previous kernel's output
    if (warp < 2) {   // warp 0: this head's q; warp 1: the kv group's k row of this token
        float *x = warp == 0 ? qh : kp;
        const float *src = warp == 0 ? qg : kg;
        const float *bias = warp == 0 ? (a.bq ? a.bq + h * a.hd : nullptr) : (a.bk ? a.bk + g * a.hd : nullptr);
        const int lane = threadIdx.x & 31;
        for (int i = lane; i < a.hd; i += 32) x[i] = bias ? __fadd_rn(src[i], bias[i]) : src[i];
        __syncwarp();
        if (a.qk_norm == 1) warp_rmsnorm(x, warp == 0 ? a.qn : a.kn, a.hd, a.eps);
        if (a.rope_half) warp_rope(x, cs, a.rope_half, a.rope_style);
    }
    __syncthreads();
    if (blockIdx.x == 0 && h % grp == 0) {   // the token's (k, v) rows into the cache
        const int64_t o = ((int64_t)g * a.max_seq + pos) * a.hd;
        for (int i = threadIdx.x; i < a.hd; i += blockDim.x) {
            a.kc[o + i] = kp[i];
            a.vc[o + i] = a.bv ? __fadd_rn(vg[i], a.bv[g * a.hd + i]) : vg[i];
        }
    }
    for (int r0 = blockIdx.x * 16; r0 <= pos; r0 += gridDim.x * 16) {
        const int r = r0 + grp16;
        const bool valid = r <= pos;
        float L = 0.0f;
        if (valid) {
            L = qk_chain(r == pos ? kp : a.kc + ((int64_t)g * a.max_seq + r) * a.hd, qh, a.hd, j);
        }
        L = tree16(L, 0xffffffffu);
        if (valid && j == 0) {
            const float sv = canon(L);
            S[(int64_t)h * a.max_seq + r] = sv != sv ? sv : __fmul_rn(scale, sv);
        }
    }
}

__global__ void k_set_pos(int *dpos, int v) { *dpos = v; }
__global__ void k_advance_pos(int *dpos, int T) { *dpos += T; }

// Per (token, head), one CTA: p = softmax(S[0..pos]) in place (hx_softmax, model.c:534-550: max,
// expf(x - m), sum16, x / s). The row is staged in shared memory, so the 16 sum16 chains read it
// there. Shared memory: pos + 1 floats.
__global__ void __launch_bounds__(256) k_attn_softmax(float *__restrict__ S, int H, int max_seq,
                                                      const int *__restrict__ dpos) {
    extern __shared__ float p[];
    __shared__ float red[8];
    __shared__ float ssum;
    const int t = blockIdx.y, h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = *dpos + t + 1;
    float *s = S + ((int64_t)t * H + h) * max_seq;
    // m = x[0] if it is NaN, else the largest non-NaN value (the comparison `x > m` skips NaNs)
    float m = -__uint_as_float(0x7f800000u);
    for (int i = tid; i < n; i += blockDim.x) {
        const float v = s[i];
        p[i] = v;
        m = fmaxf(m, v);
    }
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) m = fmaxf(m, red[w]);
    if (p[0] != p[0]) m = p[0];
    for (int i = tid; i < n; i += blockDim.x) p[i] = host_expf(__fsub_rn(p[i], m));
    __syncthreads();
    if (tid < 16) {   // sum16 (NUMERICS §1): lane chains in index order, then the 8/4/2/1 tree
        float L = 0.0f;
        for (int i = tid; i < n; i += 16) L = __fadd_rn(L, p[i]);
        L = tree16(L, 0xffffu);
        if (tid == 0) ssum = L;
    }
    __syncthreads();
    const float sum = ssum;
    for (int i = tid; i < n; i += blockDim.x) s[i] = __fdiv_rn(p[i], sum);
}

// o_h[d] = sum_r p_h[r] * v_r[d] in position order from 0.0f (value_sum, model.c:552-590), one CTA
// per (token, kv group g, hpc of the group's heads, DC dims): thread (hh, d) runs the chain of head
// g*grp + hs*hpc + hh, dim dc*DC + d. Tiles of VT positions stream into a ring of nst shared-memory
// stages by 1-D bulk copies (the V rows of the tile, contiguous in the cache, and the VT
// probabilities of each of the CTA's heads), so each V row a CTA loads serves all its heads while the
// chains run on the previous tiles. Batches take the whole group per CTA (hpc = grp, each V row read
// once per group); a decode token takes one head per CTA (hpc = 1, DC = hd) and a deeper ring, so the
// group's heads run on separate SMs; it also forms its head's probabilities itself (fuse_sm, the
// softmax kernel's steps on the score row in shared memory) while the first V tiles stream in. With DC
// a multiple of 64 the CTA also forms the o projection's activation blocks of its dims (act not
// null). max_seq is a multiple of VT.
constexpr int VT = 32, V_NST = 4, V_NST1 = 10;
__global__ void __launch_bounds__(1024) k_attn_values(const float *__restrict__ S, const float *__restrict__ vc,
                                                      float *__restrict__ att, act_q8 *__restrict__ act, int H,
                                                      int Hkv, int hd, int DC, int hpc, int nst, int max_seq,
                                                      const int *__restrict__ dpos, int fuse_sm) {
    extern __shared__ __align__(128) uint8_t smv[];
    const int grp = H / Hkv, nd = hd / DC, nh = grp / hpc;
    const int t = blockIdx.y, g = blockIdx.x / (nh * nd), rem = blockIdx.x - g * nh * nd;
    const int hs = rem / nd, dc = rem - hs * nd;
    const int h0 = g * grp + hs * hpc;   // the CTA's first head
    const int tid = threadIdx.x;
    const int hh = tid / DC, d = tid - hh * DC;
    const bool chain = tid < hpc * DC;
    const int n = *dpos + t + 1;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smv);
    float *vbuf = reinterpret_cast<float *>(smv + 128);          // [nst][VT][hd]
    float *pbuf = vbuf + (size_t)nst * VT * hd;                  // [nst][hpc][VT]
    float *ost = pbuf + (size_t)nst * hpc * VT;                  // [hpc][DC]
    float *prow = ost + (size_t)hpc * DC;                        // fuse_sm: the head's probabilities [max_seq]
    const float *vg = vc + (int64_t)g * max_seq * hd;
    const float *pg = S + ((int64_t)t * H + h0) * max_seq;
    const int ntile = (n + VT - 1) / VT;
    if (tid == 0) {
        for (int st = 0; st < nst; st++) mbar_init(&bars[st], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int it) {
        const int st = it % nst, r0 = it * VT;
        mbar_expect_tx(&bars[st], (uint32_t)(VT * hd * 4 + (fuse_sm ? 0 : hpc * VT * 4)));
        bulk_g2s(vbuf + (size_t)st * VT * hd, vg + (int64_t)r0 * hd, (uint32_t)(VT * hd * 4), &bars[st]);
        for (int j = 0; j < hpc && !fuse_sm; j++)
            bulk_g2s(pbuf + ((size_t)st * hpc + j) * VT, pg + (int64_t)j * max_seq + r0, (uint32_t)(VT * 4), &bars[st]);
    };
    // V tiles wholly before this token's position were written by earlier forwards: with the softmax
    // fused (no probability rows to copy) they stream in before the previous kernel is done
    pdl_trigger();
    const int first = fuse_sm ? min(min(nst, ntile), (n - 1) / VT) : 0;
    if (tid == 0)
        for (int it = 0; it < first; it++) issue(it);
    pdl_wait();
    if (tid == 0)
        for (int it = first; it < min(nst, ntile); it++) issue(it);
    if (fuse_sm) {   // hpc == 1: k_attn_softmax's steps on the head's score row, in shared memory
        __shared__ float red[32];
        __shared__ float ssum;
        const int lane = tid & 31, warp = tid >> 5, nw = (int)(blockDim.x >> 5);
        float mx = -__uint_as_float(0x7f800000u);
        for (int i = tid; i < n; i += blockDim.x) {
            const float v = pg[i];
            prow[i] = v;
            mx = fmaxf(mx, v);
        }
        for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        mx = red[0];
        for (int w = 1; w < nw; w++) mx = fmaxf(mx, red[w]);
        if (prow[0] != prow[0]) mx = prow[0];
        for (int i = tid; i < n; i += blockDim.x) prow[i] = host_expf(__fsub_rn(prow[i], mx));
        __syncthreads();
        if (tid < 16) {   // sum16 (NUMERICS §1)
            float L = 0.0f;
            for (int i = tid; i < n; i += 16) L = __fadd_rn(L, prow[i]);
            L = tree16(L, 0xffffu);
            if (tid == 0) ssum = L;
        }
        __syncthreads();
        const float sum = ssum;
        for (int i = tid; i < n; i += blockDim.x) prow[i] = __fdiv_rn(prow[i], sum);
        __syncthreads();
    }
    float acc = 0.0f;
    bool ok = true;
    for (int it = 0; it < ntile; it++) {
        const int st = it % nst;
        ok = ok && mbar_wait(&bars[st], (uint32_t)((it / nst) & 1), nullptr);
        if (ok && chain) {
            const float *vb = vbuf + (size_t)st * VT * hd + dc * DC + d;
            const float *pb = fuse_sm ? prow + it * VT : pbuf + ((size_t)st * hpc + hh) * VT;
            const int m = min(VT, n - it * VT);
            if (m == VT) {   // a whole tile: the loads go ahead of the dependent adds
                float pv[VT];
#pragma unroll
                for (int r = 0; r < VT; r++) pv[r] = __fmul_rn(pb[r], vb[r * hd]);
#pragma unroll
                for (int r = 0; r < VT; r++) acc = __fadd_rn(acc, pv[r]);
            } else {
                for (int r = 0; r < m; r++) acc = __fadd_rn(acc, __fmul_rn(pb[r], vb[r * hd]));
            }
        }
        __syncthreads();   // every chain is done with this stage
        if (tid == 0 && it + nst < ntile) {
            fence_proxy_async();
            issue(it + nst);
        }
    }
    if (chain) att[((int64_t)t * H + h0 + hh) * hd + dc * DC + d] = acc;
    if (act) {   // DC a multiple of 64: the activation blocks of the CTA's (head, 64 dims)
        if (chain) ost[tid] = acc;
        __syncthreads();
        const int warp = tid >> 5, lane = tid & 31, nb = H * hd / QK, bpc = DC / QK;
        for (int w = warp; w < hpc * bpc; w += (int)(blockDim.x >> 5)) {
            const int wh = w / bpc, sb = w - wh * bpc;
            act_quant_warp(ost[wh * DC + sb * QK + lane], ost[wh * DC + sb * QK + lane + 32],
                           act + (int64_t)t * nb + ((int64_t)(h0 + wh) * hd + dc * DC + sb * QK) / QK, lane);
        }
    }
}

// g = silu(g) * u (hx_swiglu, NUMERICS §4).
__global__ void k_swiglu(float *__restrict__ g, const float *__restrict__ u, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) g[i] = swiglu_c(g[i], u[i]);
}

// logits = logit_scale * logits (model.c:1225); the canonical NaN of the matmul stays as it is.
__global__ void k_scale(float *__restrict__ y, int64_t n, float ls) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float v = y[i];
        y[i] = v != v ? v : __fmul_rn(ls, v);
    }
}

unsigned blocks(int64_t n, int b) { return (unsigned)((n + b - 1) / b); }

// x[T][n] (ld ldx) times matrix W into Y[T][rows] (ld ldy): act_of + mm_run of the reference
// (model.c:287-384): quantized weights take x's activation blocks (quantized once into act by the
// caller, or here when act_ready is false), float weights take x itself.
int matmul(hxb_model *m, const Mat &W, const float *x, int64_t ldx, act_q8 *act, bool &act_ready, int T, float *Y,
           int64_t ldy, cudaStream_t s, float *resid = nullptr, float rs = 0.0f) {
    (void)m;
    const void *in = x;
    if (is_quant(W.dtype)) {
        if (!act_ready) {
            if (!mcuda(launch_act_quantize(x, ldx, act, W.cols, T, s), "act quantize")) return HXB_E_DEVICE;
            act_ready = true;
        }
        in = act;
    } else if (ldx != W.cols) {
        return mfail(HXB_E_ARG, "float matmul input stride");
    }
    // the model's weights are written once at open: the GEMV may stream them while the previous kernel runs
    if (!mcuda(launch_matmul_resid(W.dtype, W.w.p, W.cols, in, T, Y, ldy, 0, W.rows, resid, rs, s, true), "matmul"))
        return HXB_E_DEVICE;
    return HXB_OK;
}

// ---------------------------------------------------------------------------------------------
// Loading
// ---------------------------------------------------------------------------------------------

struct Loader {
    hxb_model *m;
    const ContainerFile &f;
    std::string err;
    bool upload(Buf &b, const CtTensor &t) {
        std::vector<uint8_t> host(t.nbytes);
        if (!f.read(t.off, host.data(), host.size(), err)) return false;
        if (!b.alloc(t.nbytes)) {
            err = "out of device memory";
            return false;
        }
        if (cudaMemcpy(b.p, host.data(), t.nbytes, cudaMemcpyHostToDevice) != cudaSuccess) {
            err = "copy to the device failed";
            return false;
        }
        return true;
    }
    const CtTensor *find(int layer, const char *name) {
        char full[96];
        if (layer < 0) snprintf(full, sizeof full, "%s", name);
        else snprintf(full, sizeof full, "blk.%d.%s", layer, name);
        const CtTensor *t = f.info().find(full);
        if (!t) err = std::string("tensor '") + full + "' is missing";
        return t;
    }
    // a vector of n F32 values (model.c:1369-1387 bind_vec)
    bool vec(Buf &b, int layer, const char *name, int64_t n) {
        const CtTensor *t = find(layer, name);
        if (!t) return false;
        if (t->dtype != F32 || (int64_t)t->nbytes != n * 4) {
            err = std::string(name) + ": expected an F32 vector of the model's width";
            return false;
        }
        return upload(b, *t);
    }
    // a matrix [rows, cols] of any dtype the kernels take (model.c:1344-1367 bind_mat)
    bool mat(Mat &M, int layer, const char *name, int64_t rows, int64_t cols) {
        const CtTensor *t = find(layer, name);
        if (!t) return false;
        const int64_t rb = row_bytes((int)t->dtype, cols);
        if (t->dtype > Q4 || !rb || (int64_t)t->nbytes != rows * rb) {
            err = std::string(name) + ": dtype or shape does not fit the model";
            return false;
        }
        M.dtype = (int)t->dtype;
        M.rows = rows;
        M.cols = cols;
        M.rb = rb;
        return upload(M.w, *t);
    }
};

}  // namespace
}  // namespace hx

using namespace hx;

extern "C" HXB_API void hxb_model_default_options(hxb_model_options *o) {
    if (!o) return;
    std::memset(o, 0, sizeof *o);
    o->policy = 1;
}

extern "C" HXB_API void hxb_model_close(hxb_model *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (auto &g : m->graph)
        if (g) cudaGraphExecDestroy(g);
    if (m->moe) hxb_moe_close(m->moe);
    for (auto &l : m->layers)
        for (Buf *b : {&l.attn_norm, &l.ffn_norm, &l.bq, &l.bk, &l.bv, &l.qn, &l.kn, &l.q.w, &l.k.w, &l.v.w, &l.o.w,
                       &l.gate.w, &l.up.w, &l.down.w, &l.qkv.w})
            b->release();
    for (Buf *b : {&m->tok_embd.w, &m->lm_head.w, &m->out_norm, &m->kc, &m->vc, &m->tok, &m->h, &m->x, &m->act, &m->q,
                   &m->kk, &m->S, &m->att, &m->f1, &m->f2, &m->logits, &m->cs, &m->routes, &m->forced,
                   &m->dpos})
        b->release();
    for (void *p : {(void *)m->tok_pin, (void *)m->logit_pin, (void *)m->route_pin,
                    (void *)m->forced_pin, (void *)m->err_pin})
        if (p) cudaFreeHost(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

static hxb_model *open_fail(hxb_model *m, char *err, size_t errlen, const std::string &msg) {
    if (err && errlen) snprintf(err, errlen, "%s", msg.c_str());
    set_last_error(msg.c_str());
    hxb_model_close(m);
    return nullptr;
}

// q, k and v of one dtype go into one matrix (rows q | k | v), so one launch computes the three.
static bool fuse_qkv(DLayer &w) {
    if (w.q.dtype != w.k.dtype || w.q.dtype != w.v.dtype) return true;
    Mat &f = w.qkv;
    f.dtype = w.q.dtype;
    f.cols = w.q.cols;
    f.rb = w.q.rb;
    f.rows = w.q.rows + w.k.rows + w.v.rows;
    if (!f.w.alloc((size_t)(f.rows * f.rb))) return false;
    uint8_t *d = f.w.as<uint8_t>();
    const size_t bq = (size_t)(w.q.rows * f.rb), bk = (size_t)(w.k.rows * f.rb), bv = (size_t)(w.v.rows * f.rb);
    if (cudaMemcpy(d, w.q.w.p, bq, cudaMemcpyDeviceToDevice) != cudaSuccess ||
        cudaMemcpy(d + bq, w.k.w.p, bk, cudaMemcpyDeviceToDevice) != cudaSuccess ||
        cudaMemcpy(d + bq + bk, w.v.w.p, bv, cudaMemcpyDeviceToDevice) != cudaSuccess)
        return false;
    w.q.w.release();
    w.k.w.release();
    w.v.w.release();
    return true;
}

// The KV cache, the scratch of a forward of max_batch tokens and the attention kernels' shared
// memory; null, or why not.
static const char *alloc_runtime(hxb_model *m) {
    m->kv_seq = (m->max_seq + 31) / 32 * 32;
    // dynamic shared memory of the attention kernels: q and k rows of a token, a head's scores
    const size_t post_smem = sizeof(float) * (size_t)(m->q_dim + m->kv_dim), sm_smem = sizeof(float) * (size_t)m->max_seq;
    const int grp = m->H / m->Hkv;
    m->dc = m->hd % 64 == 0 ? 64 : m->hd;   // value-kernel dims per CTA (64: whole activation blocks)
    m->vthreads = (grp * m->dc + 31) / 32 * 32;
    m->vsmem = 128 + sizeof(float) * (size_t)(V_NST * VT * m->hd + V_NST * grp * VT + grp * m->dc);
    if (m->vthreads > 1024 || m->hd % 4)
        return "model_open: attention heads per kv group times head_dim beyond the value kernel's CTA";
    int smem_max = 0;
    cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device);
    // one decode token: as many ring stages as fit beside the score row (the fused softmax), else the
    // batch kernel's ring and the separate softmax
    {
        const size_t fixed = 128 + 1024 + sizeof(float) * (size_t)(m->hd + m->kv_seq), stage = sizeof(float) * (VT * m->hd + VT);
        const size_t room = (size_t)smem_max > fixed ? (size_t)smem_max - fixed : 0;
        m->vnst1 = (int)std::min<size_t>(V_NST1, room / stage);
        m->vfuse1 = m->vnst1 >= 2 && m->hd <= 1024;
        if (!m->vfuse1) m->vnst1 = V_NST;
        m->vsmem1 = 128 + sizeof(float) * (size_t)(m->vnst1 * (VT * m->hd + VT) + m->hd + (m->vfuse1 ? m->kv_seq : 0));
    }
    if (post_smem + 1024 > (size_t)smem_max || sizeof(float) * 8 * (size_t)m->hd + 1024 > (size_t)smem_max ||
        sm_smem + 1024 > (size_t)smem_max || m->vsmem + 1024 > (size_t)smem_max || m->vsmem1 + 1024 > (size_t)smem_max ||
        sizeof(float) * (size_t)m->D > 48 * 1024)
        return "model_open: max_seq or the attention width exceeds shared memory";
    // the attribute is the device's limit, not this model's need: it is per function, shared by every
    // model of the process
    cudaFuncAttributes fp{}, fs{}, fv{};
    if (cudaFuncGetAttributes(&fp, (const void *)k_attn_post) != cudaSuccess ||
        cudaFuncGetAttributes(&fs, (const void *)k_attn_softmax) != cudaSuccess ||
        cudaFuncGetAttributes(&fv, (const void *)k_attn_values) != cudaSuccess ||
        cudaFuncSetAttribute(k_attn_values, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_max - (int)fv.sharedSizeBytes) != cudaSuccess ||
        cudaFuncSetAttribute(k_attn_post, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_max - (int)fp.sharedSizeBytes) != cudaSuccess ||
        cudaFuncSetAttribute(k_attn_softmax, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_max - (int)fs.sharedSizeBytes) != cudaSuccess)
        return "model_open: shared memory attributes refused";
    // KV cache and scratch
    const size_t T = (size_t)m->max_batch, S = (size_t)m->kv_seq;
    const size_t kvb = sizeof(float) * (size_t)m->L * m->Hkv * S * m->hd;
    const size_t actb = T * ((size_t)m->max_in / QK + 1) * sizeof(act_q8);
    const size_t rows = std::max<size_t>(1, (size_t)m->n_moe * T * m->K);
    bool ok = m->kc.alloc(kvb) && m->vc.alloc(kvb) && m->tok.alloc(4 * T) && m->h.alloc(4 * T * m->D) &&
              m->x.alloc(4 * T * m->max_in) && m->act.alloc(actb) && m->q.alloc(4 * T * (m->q_dim + 2 * m->kv_dim)) &&
              m->kk.alloc(4 * T * m->q_dim) &&
              m->S.alloc(4 * T * m->H * S) && m->att.alloc(4 * T * m->q_dim) &&
              m->f1.alloc(4 * T * std::max(1, m->Fd)) && m->f2.alloc(4 * T * std::max(1, m->Fd)) &&
              m->logits.alloc(4 * T * m->V) && m->cs.alloc(4 * S * std::max(2, m->rope_dim)) &&
              m->routes.alloc(4 * rows) && m->forced.alloc(4 * rows) && m->dpos.alloc(4);
    if (!ok) return "model_open: out of device memory (KV cache or scratch)";
    // the RoPE (cos, sin) table of every position, computed on the host as rope_tables computes it
    // for the positions of a call (model.c:386-397): th = p * inv_freq[j], cosf(th) * f, sinf(th) * f
    if (m->rope_half) {
        std::vector<float> cs(S * (size_t)m->rope_dim);
        for (size_t p = 0; p < S; p++) {
            const float pf = (float)p;
            for (int j = 0; j < m->rope_half; j++) {
                const float th = pf * m->inv_freq[(size_t)j];
                cs[p * m->rope_dim + 2 * j] = libm_cosf(th) * m->rope_factor;
                cs[p * m->rope_dim + 2 * j + 1] = libm_sinf(th) * m->rope_factor;
            }
        }
        if (cudaMemcpy(m->cs.p, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice) != cudaSuccess)
            return "model_open: RoPE table upload failed";
    }
    m->resident = !m->moe || moe_resident(m->moe);
    ok = cudaHostAlloc((void **)&m->tok_pin, 4 * T, 0) == cudaSuccess &&
         cudaHostAlloc((void **)&m->logit_pin, 4 * T * m->V, 0) == cudaSuccess &&
         cudaHostAlloc((void **)&m->route_pin, 4 * rows, 0) == cudaSuccess &&
         cudaHostAlloc((void **)&m->forced_pin, 4 * rows, 0) == cudaSuccess &&
         cudaHostAlloc((void **)&m->err_pin, 16, 0) == cudaSuccess;
    if (!ok) return "model_open: out of pinned host memory";
    return nullptr;
}

extern "C" HXB_API hxb_model *hxb_model_open(const char *path, const hxb_model_options *opt, char *err, size_t errlen) {
    hxb_model_options o;
    hxb_model_default_options(&o);
    if (opt) o = *opt;
    if (!path) return open_fail(nullptr, err, errlen, "model_open: null path");
    ContainerFile f;
    std::string e;
    if (!f.open(path, e)) return open_fail(nullptr, err, errlen, e);
    const Container &c = f.info();
    if (c.attn_kind != 0)
        return open_fail(nullptr, err, errlen, "model_open: MLA attention (attn_kind 1) is not on the GPU path");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || o.device < 0 || o.device >= ndev) {
        cudaGetLastError();
        return open_fail(nullptr, err, errlen, "model_open: no such CUDA device");
    }
    hxb_model *m = new hxb_model();
    m->device = o.device;
    cudaSetDevice(m->device);
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        return open_fail(m, err, errlen, "model_open: stream creation failed");
    m->L = (int)c.n_layers;
    m->D = (int)c.d_model;
    m->V = (int)c.vocab_size;
    m->H = (int)c.n_heads;
    m->Hkv = (int)c.n_kv_heads;
    m->hd = (int)c.head_dim;
    m->q_dim = m->H * m->hd;
    m->kv_dim = m->Hkv * m->hd;
    m->rope_dim = (int)c.rope_dim;
    m->rope_half = m->rope_dim / 2;
    m->rope_style = (int)c.rope_style;
    m->qk_norm = (int)c.qk_norm;
    m->qkv_bias = (int)c.qkv_bias;
    m->Fd = (int)c.dense_ffn_dim;
    m->n_moe = c.n_moe_layers;
    m->K = c.n_moe_layers ? (int)c.top_k : 0;
    m->E = c.n_moe_layers ? (int)c.n_experts : 0;
    m->eps = c.norm_eps;
    m->rs = c.residual_scale;
    m->es = c.emb_scale;
    m->ls = c.logit_scale;
    m->attn_scale = c.attn_scale;
    m->rope_factor = c.rope_attn_factor;
    m->max_batch = o.max_batch > 0 ? o.max_batch : 512;
    m->max_seq = o.max_seq > 0 ? o.max_seq : (int)c.max_seq;
    if (m->D > 8192 || m->q_dim > 16384 || m->kv_dim > 16384 || m->hd > 1024 || m->H > 256)
        return open_fail(m, err, errlen, "model_open: shape beyond the kernels' limits");
    m->max_in = std::max(std::max(m->D, m->q_dim), std::max(m->Fd, (int)c.expert_ffn_dim));

    Loader ld{m, f, {}};
    if (!ld.mat(m->tok_embd, -1, "tok_embd", m->V, m->D)) return open_fail(m, err, errlen, ld.err);
    if (c.tie_embeddings) {
        m->lm_head.dtype = m->tok_embd.dtype;
        m->lm_head.rows = m->V;
        m->lm_head.cols = m->D;
        m->lm_head.rb = m->tok_embd.rb;
    } else if (!ld.mat(m->lm_head, -1, "lm_head", m->V, m->D)) {
        return open_fail(m, err, errlen, ld.err);
    }
    if (!ld.vec(m->out_norm, -1, "out_norm", m->D)) return open_fail(m, err, errlen, ld.err);
    if (m->rope_half) {
        const CtTensor *t = ld.find(-1, "rope_inv_freq");
        if (!t || t->dtype != F32 || t->nbytes != (uint64_t)m->rope_half * 4)
            return open_fail(m, err, errlen, "tensor 'rope_inv_freq' is missing or has the wrong size");
        m->inv_freq.resize((size_t)m->rope_half);
        if (!f.read(t->off, m->inv_freq.data(), t->nbytes, e)) return open_fail(m, err, errlen, e);
    }
    m->layers.resize((size_t)m->L);
    m->moe_index.assign((size_t)m->L, -1);
    for (int l = 0, mi = 0; l < m->L; l++) {
        DLayer &w = m->layers[(size_t)l];
        w.moe = c.layer_kind[(size_t)l] == 1;
        if (w.moe) m->moe_index[(size_t)l] = mi++;
        bool ok = ld.vec(w.attn_norm, l, "attn_norm", m->D) && ld.vec(w.ffn_norm, l, "ffn_norm", m->D) &&
                  ld.mat(w.q, l, "attn_q", m->q_dim, m->D) && ld.mat(w.k, l, "attn_k", m->kv_dim, m->D) &&
                  ld.mat(w.v, l, "attn_v", m->kv_dim, m->D) && ld.mat(w.o, l, "attn_o", m->D, m->q_dim);
        if (ok && m->qkv_bias)
            ok = ld.vec(w.bq, l, "attn_q_bias", m->q_dim) && ld.vec(w.bk, l, "attn_k_bias", m->kv_dim) &&
                 ld.vec(w.bv, l, "attn_v_bias", m->kv_dim);
        if (ok && m->qk_norm == 1) ok = ld.vec(w.qn, l, "attn_q_norm", m->hd) && ld.vec(w.kn, l, "attn_k_norm", m->hd);
        if (ok && m->qk_norm == 2)
            ok = ld.vec(w.qn, l, "attn_q_norm", m->q_dim) && ld.vec(w.kn, l, "attn_k_norm", m->kv_dim);
        if (ok && !w.moe)
            ok = ld.mat(w.gate, l, "ffn_gate", m->Fd, m->D) && ld.mat(w.up, l, "ffn_up", m->Fd, m->D) &&
                 ld.mat(w.down, l, "ffn_down", m->D, m->Fd);
        if (!ok) return open_fail(m, err, errlen, ld.err);
        if (!fuse_qkv(w)) return open_fail(m, err, errlen, "model_open: out of device memory");
    }
    // the MoE layers: the backend handle over the same container
    if (m->n_moe) {
        hxb_moe_config cfg;
        hxb_container_info info;
        char e2[512];
        if (hxb_container_probe(path, &cfg, &info, e2, sizeof e2) != HXB_OK) return open_fail(m, err, errlen, e2);
        cfg.max_tokens = m->max_batch;
        cfg.device = m->device;
        cfg.cache_gb = o.cache_gb;
        cfg.policy = o.policy;
        m->moe = hxb_moe_open(&cfg, e2, sizeof e2);
        if (!m->moe) return open_fail(m, err, errlen, e2);
        if (hxb_moe_load_container(m->moe, path) != HXB_OK) return open_fail(m, err, errlen, hxb_last_error());
    }
    const char *why = alloc_runtime(m);
    if (why) return open_fail(m, err, errlen, why);
    return m;
}

extern "C" HXB_API hxb_model *hxb_model_synthesize(const hxb_model_arch *a, const hxb_model_options *opt,
                                                   uint64_t seed, char *err, size_t errlen) {
    hxb_model_options o;
    hxb_model_default_options(&o);
    if (opt) o = *opt;
    if (!a) return open_fail(nullptr, err, errlen, "model_synthesize: null arch");
    const hxb_moe_config &c = a->moe;
    if (c.n_layers <= 0 || c.d_model <= 0 || a->vocab_size <= 0 || a->n_heads <= 0 || a->n_kv_heads <= 0 ||
        a->head_dim <= 0 || a->n_heads % a->n_kv_heads || a->head_dim % 2 || a->qk_norm < 0 || a->qk_norm > 2 ||
        (a->dense_dtype != Q8 && a->dense_dtype != Q4) || c.d_model % QK || (a->n_heads * a->head_dim) % QK)
        return open_fail(nullptr, err, errlen, "model_synthesize: bad shape");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || o.device < 0 || o.device >= ndev) {
        cudaGetLastError();
        return open_fail(nullptr, err, errlen, "model_synthesize: no such CUDA device");
    }
    hxb_model *m = new hxb_model();
    m->device = o.device;
    cudaSetDevice(m->device);
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        return open_fail(m, err, errlen, "model_synthesize: stream creation failed");
    m->L = c.n_layers;
    m->D = c.d_model;
    m->V = a->vocab_size;
    m->H = a->n_heads;
    m->Hkv = a->n_kv_heads;
    m->hd = a->head_dim;
    m->q_dim = m->H * m->hd;
    m->kv_dim = m->Hkv * m->hd;
    m->rope_dim = m->hd;
    m->rope_half = m->hd / 2;
    m->qk_norm = a->qk_norm;
    m->n_moe = m->L;
    m->K = c.top_k;
    m->E = c.n_experts;
    m->eps = c.norm_eps;
    m->rs = c.residual_scale;
    m->attn_scale = 1.0f / sqrtf((float)m->hd);
    m->max_batch = o.max_batch > 0 ? o.max_batch : 512;
    m->max_seq = o.max_seq > 0 ? o.max_seq : 4096;
    m->max_in = std::max(std::max(m->D, m->q_dim), c.expert_ffn_dim);
    if (m->D > 8192 || m->q_dim > 16384 || m->hd > 1024 || m->H > 256)
        return open_fail(m, err, errlen, "model_synthesize: shape beyond the kernels' limits");
    m->inv_freq.resize((size_t)m->rope_half);
    for (int j = 0; j < m->rope_half; j++)   // 1 / theta^(2j / rope_dim), in double, then f32
        m->inv_freq[(size_t)j] = (float)(1.0 / std::pow((double)a->rope_theta, (double)(2 * j) / (double)m->rope_dim));
    cudaStream_t s = m->stream;
    uint64_t tensor = 0;
    auto mat = [&](Mat &M, int64_t rows, int64_t cols, float sigma) {
        M.dtype = a->dense_dtype;
        M.rows = rows;
        M.cols = cols;
        M.rb = row_bytes(M.dtype, cols);
        return M.w.alloc((size_t)(rows * M.rb)) &&
               launch_synth_blocks(M.w.as<uint8_t>(), M.dtype, rows, cols, seed * 7919ull + (++tensor), sigma, s) ==
                   cudaSuccess;
    };
    std::vector<float> ones((size_t)std::max(m->D, m->q_dim), 1.0f);
    auto unit = [&](Buf &b, int64_t n) {
        return b.alloc(sizeof(float) * (size_t)n) &&
               cudaMemcpy(b.p, ones.data(), sizeof(float) * (size_t)n, cudaMemcpyHostToDevice) == cudaSuccess;
    };
    const float sd = a->sigma_dense > 0.0f ? a->sigma_dense : 0.02f;
    bool ok = mat(m->tok_embd, m->V, m->D, 1.0f) && mat(m->lm_head, m->V, m->D, sd) && unit(m->out_norm, m->D);
    m->layers.resize((size_t)m->L);
    m->moe_index.resize((size_t)m->L);
    for (int l = 0; l < m->L && ok; l++) {
        DLayer &w = m->layers[(size_t)l];
        w.moe = true;
        m->moe_index[(size_t)l] = l;
        ok = unit(w.attn_norm, m->D) && unit(w.ffn_norm, m->D) && mat(w.q, m->q_dim, m->D, sd) &&
             mat(w.k, m->kv_dim, m->D, sd) && mat(w.v, m->kv_dim, m->D, sd) && mat(w.o, m->D, m->q_dim, sd) &&
             (m->qk_norm != 1 || (unit(w.qn, m->hd) && unit(w.kn, m->hd))) &&
             (m->qk_norm != 2 || (unit(w.qn, m->q_dim) && unit(w.kn, m->kv_dim)));
        ok = ok && cudaStreamSynchronize(s) == cudaSuccess && fuse_qkv(w);
    }
    if (!ok) return open_fail(m, err, errlen, "model_synthesize: out of device memory");
    hxb_moe_config mc = c;
    mc.max_tokens = m->max_batch;
    mc.device = m->device;
    mc.cache_gb = 0.0;
    mc.ep_size = 1;
    mc.ep_rank = 0;
    char e2[512];
    m->moe = hxb_moe_open(&mc, e2, sizeof e2);
    if (!m->moe) return open_fail(m, err, errlen, e2);
    if (hxb_moe_synthesize(m->moe, seed, 0.02f, 0.02f) != HXB_OK) return open_fail(m, err, errlen, hxb_last_error());
    if (cudaStreamSynchronize(s) != cudaSuccess) return open_fail(m, err, errlen, "model_synthesize: generator failed");
    const char *why = alloc_runtime(m);
    if (why) return open_fail(m, err, errlen, why);
    return m;
}

extern "C" HXB_API int hxb_model_info(const hxb_model *m, int *n_layers, int *d_model, int *vocab, int *max_seq,
                                      int *n_moe_layers, int *top_k) {
    if (!m) return mfail(HXB_E_ARG, "model_info: null handle");
    if (n_layers) *n_layers = m->L;
    if (d_model) *d_model = m->D;
    if (vocab) *vocab = m->V;
    if (max_seq) *max_seq = m->max_seq;
    if (n_moe_layers) *n_moe_layers = m->n_moe;
    if (top_k) *top_k = m->K;
    return HXB_OK;
}

extern "C" HXB_API hxb_moe *hxb_model_moe(hxb_model *m) { return m ? m->moe : nullptr; }

extern "C" HXB_API int hxb_model_set_replay(hxb_model *m, const uint16_t *rows, int n_rows) {
    if (!m) return mfail(HXB_E_ARG, "set_replay: null handle");
    if (!rows) {
        m->replay.clear();
        m->replay_rows = 0;
        return HXB_OK;
    }
    if (n_rows <= 0 || !m->n_moe) return mfail(HXB_E_ARG, "set_replay: no rows or no MoE layers");
    const size_t w = (size_t)m->n_moe * m->K;
    for (size_t i = 0; i < (size_t)n_rows * w; i++)
        if (rows[i] >= m->E) return mfail(HXB_E_ARG, "set_replay: expert id %u outside [0, %d)", rows[i], m->E);
    m->replay.assign(rows, rows + (size_t)n_rows * w);
    m->replay_rows = n_rows;
    return HXB_OK;
}

// One attention sublayer for tokens [0, T) at the device position (attn_gqa, model.c:596-629):
// h += rs * o(attention(rmsnorm(h, attn_norm))).
static int attention(hxb_model *m, int l, int T, cudaStream_t s) {
    const DLayer &w = m->layers[(size_t)l];
    float *x = m->x.as<float>();
    act_q8 *act = m->act.as<act_q8>();
    const bool quant_in = is_quant(w.q.dtype) && is_quant(w.k.dtype) && is_quant(w.v.dtype);
    const int ld = m->q_dim + 2 * m->kv_dim;
    float *qkv = m->q.as<float>();
    int rc = HXB_OK;
    // one token and one q|k|v matrix: the GEMV's CTAs form rmsnorm(h, attn_norm) themselves
    cudaError_t fe = cudaErrorNotSupported;
    if (T == 1 && w.qkv.w.p)
        fe = launch_gemv_norm(w.qkv.dtype, w.qkv.w.p, m->D, w.qkv.rows, m->h.as<float>(), w.attn_norm.as<float>(),
                              m->eps, qkv, nullptr, 0.0f, s, true);
    if (fe != cudaErrorNotSupported) {
        if (!mcuda(fe, "q|k|v")) return HXB_E_DEVICE;
    } else {
    k_rmsnorm_rows<<<T, 256, sizeof(float) * m->D, s>>>(m->h.as<float>(), m->D, w.attn_norm.as<float>(), m->D, m->eps,
                                                          x, m->D, quant_in ? act : nullptr);
    if (!mcuda(cudaGetLastError(), "rmsnorm")) return HXB_E_DEVICE;
    bool ready = quant_in;
    if (w.qkv.w.p) {
        rc = matmul(m, w.qkv, x, m->D, act, ready, T, qkv, ld, s);
    } else {
        rc = matmul(m, w.q, x, m->D, act, ready, T, qkv, ld, s);
        if (!rc) rc = matmul(m, w.k, x, m->D, act, ready, T, qkv + m->q_dim, ld, s);
        if (!rc) rc = matmul(m, w.v, x, m->D, act, ready, T, qkv + m->q_dim + m->kv_dim, ld, s);
    }
    }
    if (rc) return rc;
    const size_t layer_kv = (size_t)m->Hkv * m->kv_seq * m->hd;
    PostArgs a;
    a.qkv = qkv;
    a.ld = ld;
    a.qout = m->kk.as<float>();
    a.bq = m->qkv_bias ? w.bq.as<float>() : nullptr;
    a.bk = m->qkv_bias ? w.bk.as<float>() : nullptr;
    a.bv = m->qkv_bias ? w.bv.as<float>() : nullptr;
    a.qn = m->qk_norm ? w.qn.as<float>() : nullptr;
    a.kn = m->qk_norm ? w.kn.as<float>() : nullptr;
    a.cs = m->cs.as<float>();
    a.kc = m->kc.as<float>() + (size_t)l * layer_kv;
    a.vc = m->vc.as<float>() + (size_t)l * layer_kv;
    a.dpos = m->dpos.as<int>();
    a.H = m->H;
    a.Hkv = m->Hkv;
    a.hd = m->hd;
    a.qk_norm = m->qk_norm;
    a.rope_half = m->rope_half;
    a.rope_style = m->rope_style;
    a.max_seq = m->kv_seq;
    a.eps = m->eps;
    // the score CTAs of a (token, head) stride over the positions: about 1200 CTAs in all (8 per SM)
    const int chunks = std::max(1, std::min((int)blocks(m->max_seq, 16), 1200 / (m->H * T)));
    if (T == 1 && m->qk_norm != 2 && m->hd <= 1024) {   // one token: post-processing inside the score kernel
        if (!mcuda(launch_pdl(true, k_attn_scores1, dim3(chunks, m->H, 1), dim3(256), 0, s, a, m->S.as<float>(),
                              m->attn_scale),
                   "attention scores"))
            return HXB_E_DEVICE;
    } else {
        if (m->qk_norm == 2)
            k_attn_post<<<dim3(T, 1), 256, sizeof(float) * (m->q_dim + m->kv_dim), s>>>(a);
        else
            k_attn_post<<<dim3(T, (m->H + m->Hkv + 7) / 8), 256, sizeof(float) * 8 * m->hd, s>>>(a);
        k_attn_scores<<<dim3(chunks, m->H, T), 256, 0, s>>>(a.qout, a.kc, m->S.as<float>(), m->H, m->Hkv, m->hd,
                                                             m->kv_seq, a.dpos, m->attn_scale);
    }
    // one decode token: a CTA per head (the group's heads on separate SMs); batches: a CTA per (group,
    // dc dims). The o projection's activation blocks come out of the value kernel when a CTA holds
    // whole blocks.
    if (T == 1) {
        if (!m->vfuse1)
            k_attn_softmax<<<dim3(m->H, T), 256, sizeof(float) * m->max_seq, s>>>(m->S.as<float>(), m->H, m->kv_seq, a.dpos);
        const bool fuse_act = is_quant(w.o.dtype) && m->hd % QK == 0;
        // after the separate softmax kernel the launch is an ordinary one
        if (!mcuda(launch_pdl(m->vfuse1, k_attn_values, dim3(m->H, 1), dim3((m->hd + 31) / 32 * 32), m->vsmem1, s,
                              m->S.as<float>(), a.vc, m->att.as<float>(), fuse_act ? act : nullptr, m->H, m->Hkv,
                              m->hd, m->hd, 1, m->vnst1, m->kv_seq, a.dpos, m->vfuse1 ? 1 : 0),
                   "attention"))
            return HXB_E_DEVICE;
        bool aready = fuse_act;
        return matmul(m, w.o, m->att.as<float>(), m->q_dim, act, aready, T, nullptr, m->D, s, m->h.as<float>(), m->rs);
    }
    k_attn_softmax<<<dim3(m->H, T), 256, sizeof(float) * m->max_seq, s>>>(m->S.as<float>(), m->H, m->kv_seq, a.dpos);
    const bool fuse_act = is_quant(w.o.dtype) && m->dc == 64;
    const int grp = m->H / m->Hkv;
    k_attn_values<<<dim3(m->Hkv * (m->hd / m->dc), T), m->vthreads, m->vsmem, s>>>(
        m->S.as<float>(), a.vc, m->att.as<float>(), fuse_act ? act : nullptr, m->H, m->Hkv, m->hd, m->dc, grp, V_NST,
        m->kv_seq, a.dpos, 0);
    if (!mcuda(cudaGetLastError(), "attention")) return HXB_E_DEVICE;
    bool aready = fuse_act;
    // h += rs * (Wo att): the residual in the matmul's epilogue
    return matmul(m, w.o, m->att.as<float>(), m->q_dim, act, aready, T, nullptr, m->D, s, m->h.as<float>(), m->rs);
}

// A dense FFN sublayer (dense_layer + ffn, model.c:444-460, 1133-1143).
static int dense_ffn(hxb_model *m, int l, int T, cudaStream_t s) {
    const DLayer &w = m->layers[(size_t)l];
    float *x = m->x.as<float>();
    act_q8 *act = m->act.as<act_q8>();
    const bool quant_in = is_quant(w.gate.dtype) && is_quant(w.up.dtype);
    k_rmsnorm_rows<<<T, 256, sizeof(float) * m->D, s>>>(m->h.as<float>(), m->D, w.ffn_norm.as<float>(), m->D, m->eps,
                                                          x, m->D, quant_in ? act : nullptr);
    bool ready = quant_in;
    int rc = matmul(m, w.gate, x, m->D, act, ready, T, m->f1.as<float>(), m->Fd, s);
    if (!rc) rc = matmul(m, w.up, x, m->D, act, ready, T, m->f2.as<float>(), m->Fd, s);
    if (rc) return rc;
    k_swiglu<<<blocks((int64_t)T * m->Fd, 256), 256, 0, s>>>(m->f1.as<float>(), m->f2.as<float>(), (int64_t)T * m->Fd);
    bool dready = false;
    rc = matmul(m, w.down, m->f1.as<float>(), m->Fd, act, dready, T, nullptr, m->D, s, m->h.as<float>(), m->rs);
    if (rc) return rc;
    return mcuda(cudaGetLastError(), "dense ffn") ? HXB_OK : HXB_E_DEVICE;
}

// forward() of T tokens from m->tok at the device position, on stream s: the embedding, every
// layer, and for mode 1 / 2 the last / every row's logits into m->logits; the device position then
// advances by T. Device work only when every expert is resident (then capturable).
static int enqueue_forward(hxb_model *m, int T, int mode, bool replay, cudaStream_t s) {
    k_embed<<<blocks((int64_t)T * m->D, 256), 256, 0, s>>>(m->tok.as<int32_t>(), T, m->tok_embd.w.as<uint8_t>(),
                                                          m->tok_embd.dtype, m->tok_embd.rb, m->D, m->V, m->es,
                                                          m->h.as<float>());
    if (!mcuda(cudaGetLastError(), "embed")) return HXB_E_DEVICE;
    int rc = HXB_OK;
    for (int l = 0; l < m->L && rc == HXB_OK; l++) {
        rc = attention(m, l, T, s);
        if (rc) break;
        const int mi = m->moe_index[(size_t)l];
        if (mi >= 0) {
            const int *forced = replay ? m->forced.as<int>() + (size_t)mi * T * m->K : nullptr;
            rc = moe_layer_for_model(m->moe, m->h.as<float>(), T, l, s, forced);
            if (rc == HXB_OK &&
                !mcuda(cudaMemcpyAsync(m->routes.as<int>() + (size_t)mi * T * m->K, moe_ids_dev(m->moe),
                                       sizeof(int) * (size_t)T * m->K, cudaMemcpyDeviceToDevice, s),
                       "routes"))
                rc = HXB_E_DEVICE;
        } else {
            rc = dense_ffn(m, l, T, s);
        }
    }
    if (rc == HXB_OK && mode) {
        const int first = mode == 1 ? T - 1 : 0, n = mode == 1 ? 1 : T;
        float *x = m->x.as<float>();
        act_q8 *act = m->act.as<act_q8>();
        const bool q = is_quant(m->lm_head.dtype);
        Mat head = m->lm_head;
        head.w.p = m->lm_head.w.p ? m->lm_head.w.p : m->tok_embd.w.p;
        cudaError_t fe = cudaErrorNotSupported;
        if (n == 1)   // one row: the LM head's CTAs form rmsnorm(h, out_norm) themselves
            fe = launch_gemv_norm(head.dtype, head.w.p, m->D, m->V, m->h.as<float>() + (size_t)first * m->D,
                                  m->out_norm.as<float>(), m->eps, m->logits.as<float>(), nullptr, 0.0f, s, true);
        if (fe != cudaErrorNotSupported) {
            rc = mcuda(fe, "lm head") ? HXB_OK : HXB_E_DEVICE;
        } else {
            k_rmsnorm_rows<<<n, 256, sizeof(float) * m->D, s>>>(m->h.as<float>() + (size_t)first * m->D, m->D,
                                                                  m->out_norm.as<float>(), m->D, m->eps, x, m->D,
                                                                  q ? act : nullptr);
            bool ready = q;
            rc = matmul(m, head, x, m->D, act, ready, n, m->logits.as<float>(), m->V, s);
        }
        if (rc == HXB_OK)
            k_scale<<<blocks((int64_t)n * m->V, 256), 256, 0, s>>>(m->logits.as<float>(), (int64_t)n * m->V, m->ls);
    }
    if (rc == HXB_OK) k_advance_pos<<<1, 1, 0, s>>>(m->dpos.as<int>(), T);
    if (rc == HXB_OK && !mcuda(cudaGetLastError(), "forward")) rc = HXB_E_DEVICE;
    return rc;
}

// Everything before the device work of a forward: arguments, the device position, the replay ids.
static int prepare(hxb_model *m, int T, int pos0, int mode, cudaStream_t s, bool &replay) {
    if (T <= 0 || pos0 < 0 || mode < 0 || mode > 2) return mfail(HXB_E_ARG, "model_forward: bad arguments");
    if (T > m->max_batch) return mfail(HXB_E_CAPACITY, "model_forward: T=%d exceeds max_batch=%d", T, m->max_batch);
    if (pos0 + T > m->max_seq)
        return mfail(HXB_E_CAPACITY, "model_forward: positions up to %d exceed max_seq=%d", pos0 + T, m->max_seq);
    cudaSetDevice(m->device);
    if (m->next_pos != pos0) {
        k_set_pos<<<1, 1, 0, s>>>(m->dpos.as<int>(), pos0);
        if (!mcuda(cudaGetLastError(), "position")) return HXB_E_DEVICE;
    }
    replay = m->replay_rows > 0;
    if (replay) {   // forced ids [n_moe][T][K] from rows (pos mod n_rows)
        const size_t w = (size_t)m->n_moe * m->K;
        for (int t = 0; t < T; t++) {
            const uint16_t *row = m->replay.data() + (size_t)((pos0 + t) % m->replay_rows) * w;
            for (int mi = 0; mi < m->n_moe; mi++)
                for (int j = 0; j < m->K; j++)
                    m->forced_pin[((size_t)mi * T + t) * m->K + j] = row[(size_t)mi * m->K + j];
        }
        if (!mcuda(cudaMemcpyAsync(m->forced.p, m->forced_pin, sizeof(int) * (size_t)m->n_moe * T * m->K,
                                   cudaMemcpyHostToDevice, s),
                   "replay ids"))
            return HXB_E_DEVICE;
    }
    return HXB_OK;
}

// The device work of a forward: a single-token forward of a resident model replays its CUDA graph
// (captured on its second use, once the first has settled the MoE tables); the rest launches
// directly. On failure the device position is unknown until the next forward sets it.
static int run_forward(hxb_model *m, int T, int pos0, int mode, bool replay, cudaStream_t s) {
    m->next_pos = -1;
    int rc = HXB_OK;
    const bool graphable = T == 1 && !replay && m->resident && m->graphs_ok;
    if (graphable && m->warm && !m->graph[mode]) {
        cudaGraph_t g = nullptr;
        if (!mcuda(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "capture")) return HXB_E_DEVICE;
        rc = enqueue_forward(m, T, mode, false, m->stream);
        const cudaError_t ce = cudaStreamEndCapture(m->stream, &g);
        cudaGraphExec_t ex = nullptr;
        if (rc == HXB_OK && ce == cudaSuccess && g && cudaGraphInstantiate(&ex, g, 0) == cudaSuccess) {
            m->graph[mode] = ex;
        } else {   // not capturable here: launch directly from now on
            cudaGetLastError();
            m->graphs_ok = false;
        }
        if (g) cudaGraphDestroy(g);
        rc = HXB_OK;
    }
    if (graphable && m->graph[mode]) {
        if (!mcuda(cudaGraphLaunch(m->graph[mode], s), "graph launch")) return HXB_E_DEVICE;
    } else {
        rc = enqueue_forward(m, T, mode, replay, s);
        if (rc != HXB_OK) return rc;
        if (T == 1 && !replay) m->warm = true;
    }
    m->next_pos = pos0 + T;
    return HXB_OK;
}

extern "C" HXB_API int hxb_model_forward(hxb_model *m, const int32_t *tokens, int T, int pos0, float *logits, int mode) {
    if (!m || !tokens || (mode && !logits)) return mfail(HXB_E_ARG, "model_forward: bad arguments");
    for (int t = 0; t < T; t++)
        if (tokens[t] < 0 || tokens[t] >= m->V)
            return mfail(HXB_E_TOKEN, "model_forward: token %d outside [0, %d)", tokens[t], m->V);
    cudaStream_t s = m->stream;
    bool replay = false;
    int rc = prepare(m, T, pos0, mode, s, replay);
    if (rc != HXB_OK) return rc;
    std::memcpy(m->tok_pin, tokens, sizeof(int32_t) * (size_t)T);
    if (!mcuda(cudaMemcpyAsync(m->tok.p, m->tok_pin, sizeof(int32_t) * T, cudaMemcpyHostToDevice, s), "tokens"))
        return HXB_E_DEVICE;
    rc = run_forward(m, T, pos0, mode, replay, s);
    const size_t nl = (size_t)(mode == 1 ? 1 : T) * m->V;
    if (rc == HXB_OK && mode &&
        !mcuda(cudaMemcpyAsync(m->logit_pin, m->logits.p, sizeof(float) * nl, cudaMemcpyDeviceToHost, s), "logits"))
        rc = HXB_E_DEVICE;
    if (m->moe && !mcuda(cudaMemcpyAsync(m->err_pin, moe_err_dev(m->moe), sizeof(int), cudaMemcpyDeviceToHost, s), "err"))
        rc = rc ? rc : HXB_E_DEVICE;
    if (!mcuda(cudaStreamSynchronize(s), "forward")) return HXB_E_DEVICE;
    if (rc != HXB_OK) {
        m->next_pos = -1;
        return rc;
    }
    if (m->moe && m->err_pin[0]) {
        m->next_pos = -1;
        return moe_take_error(m->moe, m->err_pin[0]);
    }
    if (mode) std::memcpy(logits, m->logit_pin, sizeof(float) * nl);
    m->last_T = T;
    return HXB_OK;
}

extern "C" HXB_API int hxb_model_forward_dev(hxb_model *m, const int32_t *tokens, int T, int pos0, float *logits,
                                             int mode, void *stream) {
    if (!m || !tokens || (mode && !logits)) return mfail(HXB_E_ARG, "model_forward_dev: bad arguments");
    if (!m->resident) return mfail(HXB_E_UNSUPPORTED, "model_forward_dev: needs every expert resident");
    cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
    bool replay = false;
    int rc = prepare(m, T, pos0, mode, s, replay);
    if (rc != HXB_OK) return rc;
    if (!mcuda(cudaMemcpyAsync(m->tok.p, tokens, sizeof(int32_t) * T, cudaMemcpyDeviceToDevice, s), "tokens"))
        return HXB_E_DEVICE;
    rc = run_forward(m, T, pos0, mode, replay, s);
    if (rc == HXB_OK && mode &&
        !mcuda(cudaMemcpyAsync(logits, m->logits.p, sizeof(float) * (size_t)(mode == 1 ? 1 : T) * m->V,
                               cudaMemcpyDeviceToDevice, s),
               "logits"))
        rc = HXB_E_DEVICE;
    if (rc == HXB_OK) m->last_T = T;
    return rc;
}

extern "C" HXB_API int hxb_model_sync(hxb_model *m, void *stream) {
    if (!m) return mfail(HXB_E_ARG, "model_sync: null handle");
    cudaSetDevice(m->device);
    if (!mcuda(cudaStreamSynchronize(stream ? (cudaStream_t)stream : m->stream), "model_sync")) return HXB_E_DEVICE;
    if (m->moe) {
        int word = 0;
        if (!mcuda(cudaMemcpy(&word, moe_err_dev(m->moe), sizeof(int), cudaMemcpyDeviceToHost), "err"))
            return HXB_E_DEVICE;
        if (word) {
            m->next_pos = -1;
            return moe_take_error(m->moe, word);
        }
    }
    return HXB_OK;
}

extern "C" HXB_API int hxb_model_last_routes(hxb_model *m, uint16_t *routes, int T) {
    if (!m || !routes || T <= 0 || T > m->last_T) return mfail(HXB_E_ARG, "last_routes: bad arguments");
    if (!m->n_moe) return HXB_OK;
    const size_t n = (size_t)m->n_moe * T * m->K;
    cudaSetDevice(m->device);
    if (!mcuda(cudaMemcpy(m->route_pin, m->routes.p, sizeof(int) * n, cudaMemcpyDeviceToHost), "routes"))
        return HXB_E_DEVICE;
    const size_t w = (size_t)m->n_moe * m->K;
    for (int t = 0; t < T; t++)
        for (int mi = 0; mi < m->n_moe; mi++)
            for (int j = 0; j < m->K; j++)
                routes[(size_t)t * w + (size_t)mi * m->K + j] = (uint16_t)m->route_pin[((size_t)mi * T + t) * m->K + j];
    return HXB_OK;
}
