// hx_decode.cu — single-token decode of a whole MoE stack in one persistent launch.
//
// One cooperative launch of one 512-thread CTA per SM evaluates every layer of the range for one
// token: rmsnorm, router, routing, Q4/Q8 gate/up + SwiGLU, mid activation blocks, down, rank-order
// sum and residual (engine/src/model.c:1203-1214 with moe_layer, model.c:857-930), each float
// result in the reference's canonical order (NUMERICS §1-§5), bit-identical to the per-phase kernels.
//
// The CTAs hand data to one another through exchange buffers in global memory whose words are their
// own readiness flags: every slot holds kEmpty (0xffffffff, a NaN bit pattern no canonicalised value
// has) until its producer stores the value, and a consumer polls exactly the words it needs. There
// is no grid barrier, no atomic and no fence on the data path. Per layer l:
//   P1  every CTA: h_l (layer 0: the input; later: polled from xh[l]), rmsnorm, x; CTA c computes
//       router row c (dot16) -> xlg[l][c];
//   P2  every CTA: every warp forms x's activation blocks, the CTA polls the E logits, warp 0 routes
//       the token (identical everywhere); then the bulk copies of its gate/up chunks and of its down
//       rows go out;
//   P3  CTA c: gate/up chunks [c*NCH/G, (c+1)*NCH/G) of the K x F/ch chunks of ch row pairs (warp q
//       takes chunk q as soon as it lands), SwiGLU -> xmid[l][j][f];
//   P4  CTA c belongs to the down group of rank j = c*K/G: polls expert j's F mid values, forms its
//       F/64 activation blocks (NUMERICS §2), computes its slice of expert j's down rows -> xy[l][j][d];
//   P5  CTA c owns h rows [c*D/G, (c+1)*D/G): polls y of the K experts for them, rank-order sum,
//       residual -> xh[l+1][d] (the last layer: the output h).
// Exchange slots are written once per launch. Two sets alternate by a launch counter kept in device
// memory; each launch resets the set the previous launch used (spread over its layers), so the next
// launch finds it empty — no end-of-launch barrier, and the launch can be captured in a CUDA graph.
// Every poll and every mbarrier wait is bounded: on expiry it records an error word and moves on.
//
// Expert parallelism (ep_size > 1, one launch per token on every GPU): rank r holds the experts e with
// e % ep_size == r. P1 and P2 run on every GPU (the same routing everywhere); P3 and P4 cover only the
// ranks j whose expert this GPU owns (the CTAs split those instead of all K); P4 stores each y row as
// a tagged 64-bit word (high half: the launch number + 1, the same on every GPU for the same token;
// low half: the value) into every GPU's y-word buffer over NVLink (plain peer stores, system scope);
// P5 polls its own GPU's y words. Nothing else crosses GPUs, so every GPU ends each layer with the
// single-GPU h, bit for bit.
#include "hx_device.cuh"
#include "hx_kernels.h"
#include "hx_route.cuh"

#include <string>

namespace hx {

constexpr int DEC_THREADS = 512;
constexpr int DEC_WARPS = DEC_THREADS / 32;
constexpr int DEC_PROWS = ROWS_1TOK;   // rows per warp_rows_1tok call (P buffer rows)
constexpr int DEC_MAXL = 128;      // layers per launch (router / norm / bias pointer tables in smem)
constexpr int DEC_MAXCH = 26;      // gate/up chunks per CTA (mbarriers 0..25)
constexpr int BAR_DOWN = 28, BAR_ROUTER = 29;
constexpr int kIssueWarp = DEC_WARPS - 1;   // issues the bulk copies of a layer
constexpr uint32_t kEmpty = 0xffffffffu;
constexpr uint32_t kPollLimit = 1u << 18;   // polls of one word before giving up (~30 ms)
enum : int { DEV_E_POLL = 4 };             // an exchange word never arrived

// Phase stamps of the optional timeline (thread 0 of every CTA, per layer).
// ST_H h polled; ST_RMS rmsnorm chain done; ST_NORM router rows in, barrier; ST_X x; ST_LOGIT logit
// stored; ST_ACT activation blocks; ST_LG logits polled; ST_RT routed; ST_ROUTE barrier after
// routing; ST_CH0 thread 0's chunk landed; ST_CHD its SwiGLU values stored; ST_RESET other set's slots reset; ST_MIDP mid polled; ST_MIDQ mid blocks; ST_DNW down rows
// landed; ST_DOWN down rows computed; ST_YST y stored; ST_Y y polled; ST_SUM h stored.
enum : int { ST_START, ST_H, ST_RMS, ST_NORM, ST_X, ST_LOGIT, ST_ACT, ST_LG, ST_RT, ST_ROUTE, ST_CH0,
             ST_CHD, ST_RESET, ST_MIDP, ST_MIDQ, ST_DNW, ST_DOWN, ST_YST, ST_Y, ST_SUM, DEC_STAMPS };

// Work split of one launch (identical on host and device).
struct DecodePlan {
    int G, ch, nch, ch_max;       // CTAs, row pairs per chunk, gate/up chunks (K * F / ch), chunks per CTA at most
    int prows;                    // down rows per single-token row loop call
    int ra, dr_max, hr_max;       // down-row alignment, down rows / CTA at most, h rows / CTA at most
    int rpc;                      // router rows per CTA
};

HX_HD inline void chunk_range(int c, int G, int nch, int *c0, int *c1) {
    *c0 = (int)((int64_t)nch * c / G);
    *c1 = (int)((int64_t)nch * (c + 1) / G);
}
HX_HD inline int down_group(int c, int G, int K) { return (int)((int64_t)c * K / G); }
HX_HD inline int group_first(int j, int G, int K) { return (int)(((int64_t)j * G + K - 1) / K); }
// down rows [*r0, *r1) of CTA c: its group's CTAs split expert j's D rows in multiples of ra
HX_HD inline void down_rows(int c, int G, int K, int D, int ra, int *r0, int *r1) {
    const int j = down_group(c, G, K), g0 = group_first(j, G, K), g1 = group_first(j + 1, G, K);
    const int n = g1 - g0, r = c - g0;
    *r0 = (int)((int64_t)D * r / n) / ra * ra;
    *r1 = r + 1 == n ? D : (int)((int64_t)D * (r + 1) / n) / ra * ra;
}
HX_HD inline void h_rows(int c, int G, int D, int *r0, int *r1) {
    *r0 = (int)((int64_t)D * c / G);
    *r1 = (int)((int64_t)D * (c + 1) / G);
}

HX_HD inline DecodePlan decode_plan(int G, int D, int F, int E, int K, int dtype, int ep) {
    DecodePlan P{};
    P.G = G;
    // gate/up row pairs per chunk (one mbarrier, two bulk copies): 4 (3 measured no faster on the
    // Qwen3 shape), 2 when F is not a multiple of 4. With expert parallelism a GPU computes about K/ep
    // of the ranks: chunks of 2 pairs keep every warp busy with half the dependent rows each, and the
    // down rows go 4 to a warp call for the same reason.
    P.ch = F % 4 == 0 && ep <= 1 ? 4 : 2;
    P.prows = ep <= 1 ? 8 : 4;
    P.nch = K * F / P.ch;
    P.ch_max = (P.nch + G - 1) / G;
    const int64_t rbF = row_bytes(dtype, F);
    P.ra = 1;
    while ((P.ra * rbF) % 16) P.ra++;
    const int nmin = G / K;   // smallest down group
    P.dr_max = (D + nmin - 1) / nmin + P.ra;
    P.hr_max = (D + G - 1) / G + 1;
    P.rpc = (E + G - 1) / G;
    return P;
}

// Shared-memory carve-up of one CTA (identical on host and device).
struct DecodeLayout {
    DecodePlan plan;
    int nbD, nbF;
    int64_t rbD, rbF;
    size_t off_hs, off_xs, off_xact, off_stab, off_rrow, off_norm, off_gu, off_dn, off_mid, off_amid, off_y, off_p,
        off_gout, off_lg, off_score, off_sel, off_key, off_gsc, off_keep, off_ids, off_w, off_yv, off_ptrs,
        off_chain, total;
    int cs;   // floats per lane row of the chain buffer
};

HX_HD inline size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

HX_HD inline DecodeLayout decode_layout(int G, int D, int F, int E, int K, int dtype, int ep) {
    DecodeLayout L{};
    L.plan = decode_plan(G, D, F, E, K, dtype, ep);
    L.nbD = D / QK;
    L.nbF = F / QK;
    L.rbD = row_bytes(dtype, D);
    L.rbF = row_bytes(dtype, F);
    const DecodePlan &P = L.plan;
    const int Ek = E > 128 ? E : 128;
    size_t o = 512;   // mbarriers
    L.off_hs = o; o = align16(o + (size_t)D * 4);
    L.off_xs = o; o = align16(o + (size_t)D * 4);
    L.off_xact = o; o = align16(o + (size_t)L.nbD * ACT_BLOCK);
    L.off_stab = o; o = align16(o + (size_t)E * 8);
    L.off_rrow = o; o = align16(o + (size_t)P.rpc * D * 4);
    L.off_norm = o; o = align16(o + (size_t)D * 4);
    // tiles keep 16 readable bytes after them (the padded block loaders read up to 2 past a block)
    L.off_gu = o; o = align16(o + (size_t)P.ch_max * 2 * P.ch * L.rbD + 16);
    L.off_dn = o; o = align16(o + (size_t)P.dr_max * L.rbF + 16);
    L.off_mid = o; o = align16(o + (size_t)F * 4);
    L.off_amid = o; o = align16(o + (size_t)L.nbF * ACT_BLOCK);
    L.off_y = o; o = align16(o + (size_t)P.dr_max * 4);
    L.off_p = o; o = align16(o + (size_t)DEC_WARPS * DEC_PROWS * 33 * 4);
    L.off_gout = o; o = align16(o + (size_t)DEC_WARPS * DEC_PROWS * 4);
    L.off_lg = o; o = align16(o + (size_t)Ek * 4);
    L.off_score = o; o = align16(o + (size_t)E * 4);
    L.off_sel = o; o = align16(o + (size_t)E * 4);
    L.off_key = o; o = align16(o + (size_t)Ek * 8);
    L.off_gsc = o; o = align16(o + 64 * 4);
    L.off_keep = o; o = align16(o + 64 * 4);
    L.off_ids = o; o = align16(o + 16 * 4);
    L.off_w = o; o = align16(o + 16 * 4);
    L.off_yv = o; o = align16(o + (size_t)K * P.hr_max * 4);
    L.off_ptrs = o; o = align16(o + (size_t)3 * DEC_MAXL * 8);
    // the 16-lane chains of NUMERICS §1 read their terms from here, lane j's D/16 terms contiguous:
    // the squares of h (rmsnorm), then the router row's products (one router row per CTA)
    L.cs = D / 16 + 4;
    L.off_chain = o; o = align16(o + (size_t)16 * L.cs * 4);
    L.total = o;
    return L;
}

// Exchange buffers of one set, in floats: xlg [Lb][E], xmid [Lb][K][F], xy [Lb][K][D],
// xh [Lb][D] (Lb = buffer layers, at least the layers of any launch).
HX_HD inline int64_t xset_floats(int Lb, int D, int F, int E, int K) {
    return (int64_t)Lb * ((int64_t)E + (int64_t)K * F + (int64_t)K * D + D);
}

struct DecodeArgs {
    int Lyr, D, F, E, K, dtype;
    RouteCfg route;
    float eps, rs;
    int64_t off_up, off_down;
    const float *const *router;   // [Lyr] router [E, D]
    const float *const *norm;     // [Lyr] ffn_norm [D]
    const float *const *bias;     // [Lyr] router bias [E] (null entries without score_bias)
    const uint8_t *const *slab;   // [Lyr * E]
    float *h;                     // [D] in / out
    float *xbuf;                  // two exchange sets of xset_floats(Lb, ...) floats, kEmpty at rest
    int Lb;
    unsigned *epoch;              // [4]: launch counter (set = epoch & 1), CTAs done with this launch,
                                  // buffer layers last used in set 0 / set 1
    int *err;
    int *ids_out;                 // [K] routing of the last layer
    float *w_out;
    unsigned long long *trace;    // null, or [Lyr][G][DEC_STAMPS] SM clock stamps of thread 0
    int ep_size, ep_rank;         // expert parallelism (1, 0: every expert here)
    uint64_t *const *ep_y;        // [ep_size] every GPU's y words [Lb][K][D] (this GPU's at ep_rank)
    DecodeLayout lay;
};

__device__ __forceinline__ unsigned long long sm_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %clock64;" : "=l"(t));
    return t;
}

__device__ __forceinline__ float ld_poll(const float *p) {
    float v;
    asm volatile("ld.relaxed.gpu.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float4 ld_poll4(const float *p) {
    float4 v;
    asm volatile("ld.relaxed.gpu.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

__device__ __forceinline__ void st_x(float *p, float v) {
    asm volatile("st.relaxed.gpu.global.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

__device__ __forceinline__ bool empty_word(float v) { return __float_as_uint(v) == kEmpty; }

// Tagged y words of expert parallelism (system scope: written by the GPU that owns the expert).
__device__ __forceinline__ void st_ep(uint64_t *p, uint32_t tag, float v) {
    const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

constexpr uint32_t kEpPollLimit = 1u << 20;   // a peer GPU's word: longer, a rank may start later
__device__ __forceinline__ float poll_ep(const uint64_t *p, uint32_t tag, int *err) {
    for (uint32_t spins = 0;; spins++) {
        uint64_t w;
        asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
        if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
        if (spins > kEpPollLimit || ((spins & 255u) == 255u && *(volatile int *)err)) {
            set_error(err, DEV_E_POLL);
            return 0.0f;
        }
        __nanosleep(64);
    }
}

// Polls one exchange word until it is filled (bounded; on expiry records an error and returns 0).
__device__ __forceinline__ float poll1(const float *p, int *err) {
    for (uint32_t spins = 0;; spins++) {
        const float v = ld_poll(p);
        if (!empty_word(v)) return v;
        if (spins > kPollLimit || ((spins & 255u) == 255u && *(volatile int *)err)) {
            set_error(err, DEV_E_POLL);
            return 0.0f;
        }
        __nanosleep(64);
    }
}

__device__ __forceinline__ float4 poll4(const float *p, int *err) {
    for (uint32_t spins = 0;; spins++) {
        const float4 v = ld_poll4(p);
        if (!empty_word(v.x) && !empty_word(v.y) && !empty_word(v.z) && !empty_word(v.w)) return v;
        if (spins > kPollLimit || ((spins & 255u) == 255u && *(volatile int *)err)) {
            set_error(err, DEV_E_POLL);
            return make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        __nanosleep(64);
    }
}

// n consecutive exchange floats (n % 4 == 0, 16-byte aligned) -> shared dst, by the whole CTA.
__device__ __forceinline__ void poll_vec(const float *src, float *dst, int n, int *err) {
    for (int i = threadIdx.x * 4; i < n; i += DEC_THREADS * 4)
        *reinterpret_cast<float4 *>(dst + i) = poll4(src + i, err);
}

// The 16-lane chain of NUMERICS §1 over the chain buffer: lane j < 16 adds c[j*cs + k], k = 0..4*n4-1,
// in order (its own terms are contiguous: 16-byte loads, several in flight ahead of the adds), then
// the 8/4/2/1 tree; the result lands in lane 0.
__device__ __forceinline__ float chain16_regs(const float *c, int cs, int n4) {
    const int lane = threadIdx.x & 31;
    float L = 0.0f;
    if (lane < 16) {
        const float4 *r = reinterpret_cast<const float4 *>(c + lane * cs);
#pragma unroll 8
        for (int k = 0; k < n4; k++) {
            const float4 v = r[k];
            L = __fadd_rn(L, v.x);
            L = __fadd_rn(L, v.y);
            L = __fadd_rn(L, v.z);
            L = __fadd_rn(L, v.w);
        }
    }
    return tree16(L, 0xffffffffu);
}

template <int DT>
__device__ void decode_body(const DecodeArgs &a, uint8_t *smem) {
    const DecodeLayout &ly = a.lay;
    const DecodePlan &pl = ly.plan;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, G = gridDim.x;
    const int D = a.D, F = a.F, E = a.E, K = a.K;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    float *hs = reinterpret_cast<float *>(smem + ly.off_hs);
    float *xs = reinterpret_cast<float *>(smem + ly.off_xs);
    act_q8 *xact = reinterpret_cast<act_q8 *>(smem + ly.off_xact);
    const uint8_t **stab = reinterpret_cast<const uint8_t **>(smem + ly.off_stab);   // this layer's slabs
    float *rrow = reinterpret_cast<float *>(smem + ly.off_rrow);
    float *normv = reinterpret_cast<float *>(smem + ly.off_norm);
    uint8_t *gu = smem + ly.off_gu;
    uint8_t *dn = smem + ly.off_dn;
    float *mids = reinterpret_cast<float *>(smem + ly.off_mid);
    act_q8 *amid = reinterpret_cast<act_q8 *>(smem + ly.off_amid);
    float *Ys = reinterpret_cast<float *>(smem + ly.off_y);
    float *P = reinterpret_cast<float *>(smem + ly.off_p) + warp * DEC_PROWS * 33;
    float *gout = reinterpret_cast<float *>(smem + ly.off_gout) + warp * DEC_PROWS;
    float *lgs = reinterpret_cast<float *>(smem + ly.off_lg);
    float *score = reinterpret_cast<float *>(smem + ly.off_score);
    float *sel = reinterpret_cast<float *>(smem + ly.off_sel);
    unsigned long long *rkey = reinterpret_cast<unsigned long long *>(smem + ly.off_key);
    float *gscr = reinterpret_cast<float *>(smem + ly.off_gsc);
    int *gkeep = reinterpret_cast<int *>(smem + ly.off_keep);
    int *ids = reinterpret_cast<int *>(smem + ly.off_ids);
    float *wts = reinterpret_cast<float *>(smem + ly.off_w);
    float *yv = reinterpret_cast<float *>(smem + ly.off_yv);
    const float **p_router = reinterpret_cast<const float **>(smem + ly.off_ptrs);
    const float **p_norm = p_router + DEC_MAXL, **p_bias = p_norm + DEC_MAXL;
    float *chb = reinterpret_cast<float *>(smem + ly.off_chain);
    __shared__ float rms_r;
    __shared__ unsigned s_epoch, s_prev;

    for (int i = tid; i < a.Lyr; i += DEC_THREADS) {
        p_router[i] = a.router[i];
        p_norm[i] = a.norm[i];
        p_bias[i] = a.bias[i];
    }
    if (tid == 0) {
        s_epoch = *(volatile unsigned *)a.epoch;
        // buffer layers the previous launch used in the other set (launches may differ in layers)
        s_prev = ((volatile unsigned *)a.epoch)[2 + ((s_epoch & 1u) ^ 1u)];
        for (int i = 0; i < 32; i++) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncthreads();

    // this launch's exchange set and the other one (reset during the launch for the next)
    const int64_t xset = xset_floats(a.Lb, D, F, E, K);
    float *X = a.xbuf + (int64_t)(s_epoch & 1u) * xset;
    float *Xo = a.xbuf + (int64_t)((s_epoch & 1u) ^ 1u) * xset;
    const int64_t o_lg = 0, o_mid = (int64_t)a.Lb * E,
                  o_y = o_mid + (int64_t)a.Lb * K * F, o_h = o_y + (int64_t)a.Lb * K * D;
    auto xlg = [&](int l) { return X + o_lg + (int64_t)l * E; };
    auto xmid = [&](int l, int j) { return X + o_mid + ((int64_t)l * K + j) * F; };
    auto xy = [&](int l, int j) { return X + o_y + ((int64_t)l * K + j) * D; };
    auto xh = [&](int l) { return X + o_h + (int64_t)l * D; };

    // this CTA's work (with expert parallelism the chunks and down groups follow, per layer, the ranks
    // whose expert this GPU owns: s_own[0..s_nown))
    int ch0, ch1;
    chunk_range(c, G, pl.nch, &ch0, &ch1);
    int nch_c = ch1 - ch0;
    int jd = down_group(c, G, K);
    int dr0, dr1, hr0, hr1;
    down_rows(c, G, K, D, pl.ra, &dr0, &dr1);
    h_rows(c, G, D, &hr0, &hr1);
    int ndr = dr1 - dr0;
    const int nhr = hr1 - hr0;
    const bool ep = a.ep_size > 1;
    __shared__ int s_own[16], s_nown;
    const uint32_t ep_tag = s_epoch + 1u;   // y words of this launch (buffers start at 0)
    const int CH = pl.ch;
    const int cpe = F / CH;   // chunks per expert
    const uint32_t chunk_bytes = (uint32_t)(CH * ly.rbD);
    const bool small_route = E <= 128 && a.route.n_group <= 1;

    auto issue_router = [&](int l) {   // router rows e = c + t*G, ffn_norm and the slab pointers of layer l
        uint32_t bytes = (uint32_t)D * 4 + (uint32_t)E * 8;
        for (int t = 0; t < pl.rpc; t++)
            if (c + t * G < E) bytes += (uint32_t)D * 4;
        mbar_expect_tx(&bars[BAR_ROUTER], bytes);
        bulk_g2s(normv, p_norm[l], (uint32_t)D * 4, &bars[BAR_ROUTER]);
        bulk_g2s(stab, a.slab + (size_t)l * E, (uint32_t)E * 8, &bars[BAR_ROUTER]);
        for (int t = 0; t < pl.rpc; t++)
            if (c + t * G < E)
                bulk_g2s(rrow + (size_t)t * D, p_router[l] + (size_t)(c + t * G) * D, (uint32_t)D * 4,
                         &bars[BAR_ROUTER]);
    };
    if (tid == 0) issue_router(0);

    unsigned long long *stamp = nullptr;
    for (int l = 0; l < a.Lyr; l++) {
        const uint32_t par = (uint32_t)(l & 1);
        if (a.trace) stamp = a.trace + ((size_t)l * G + c) * DEC_STAMPS;
#define HX_STAMP(i) \
    if (stamp && tid == 0) stamp[i] = sm_clock()
        HX_STAMP(ST_START);
        // ---------------- P1: h, rmsnorm, x, router rows
        for (int i4 = tid; i4 * 4 < D; i4 += DEC_THREADS) {   // h, and its squares for lane (i & 15)'s chain
            const float4 v = l == 0 ? __ldcg(reinterpret_cast<const float4 *>(a.h) + i4) : poll4(xh(l) + 4 * i4, a.err);
            reinterpret_cast<float4 *>(hs)[i4] = v;
            const float q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int i = 4 * i4 + k;
                chb[(i & 15) * ly.cs + (i >> 4)] = __fmul_rn(q[k], q[k]);
            }
        }
        __syncthreads();
        HX_STAMP(ST_H);
        if (warp == 0) {
            const float L = chain16_regs(chb, ly.cs, D / 64);
            if (lane == 0) rms_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(L, (float)D), a.eps)));
            HX_STAMP(ST_RMS);
        }
        mbar_wait(&bars[BAR_ROUTER], par, a.err);
        __syncthreads();
        HX_STAMP(ST_NORM);
        const bool one_row = pl.rpc == 1;   // the router row's products go through the chain buffer
        {
            const float r = rms_r;
            for (int i = tid; i < D; i += DEC_THREADS) {
                const float x = __fmul_rn(__fmul_rn(hs[i], r), normv[i]);
                xs[i] = x;
                if (one_row && c < E) chb[(i & 15) * ly.cs + (i >> 4)] = __fmul_rn(rrow[i], x);
            }
        }
        __syncthreads();
        HX_STAMP(ST_X);
        if (one_row) {   // router row c first (the logits are on every CTA's path)
            if (warp == 0 && c < E) {
                const float L = chain16_regs(chb, ly.cs, D / 64);
                if (lane == 0) st_x(xlg(l) + c, canon(L));
            }
        } else {   // router rows: one 16-lane group each
            const int t = tid >> 4, j = tid & 15;
            const bool active = t < pl.rpc && c + t * G < E;
            float L = 0.0f;
            if (active) {
                const float *w = rrow + (size_t)t * D;
#pragma unroll 8
                for (int i = j; i < D; i += 16) L = __fadd_rn(L, __fmul_rn(w[i], xs[i]));
            }
            if (warp < (pl.rpc + 1) / 2) {
                L = tree16(L, 0xffffffffu);
                if (active && j == 0) st_x(xlg(l) + c + t * G, canon(L));
            }
        }
        HX_STAMP(ST_LOGIT);
        for (int b = warp; b < ly.nbD; b += DEC_WARPS) act_quant_warp(xs[b * QK + lane], xs[b * QK + lane + 32], xact + b, lane);
        HX_STAMP(ST_ACT);
        poll_vec(xlg(l), lgs, E, a.err);
        __syncthreads();
        HX_STAMP(ST_LG);
        if (warp == 0) {
            if (small_route) route_token_warp128<true>(a.route, lgs, p_bias[l], ids, wts, gscr);
            else route_token_warp1<true>(a.route, lgs, p_bias[l], lgs, rkey, score, sel, gscr, gkeep, ids, wts);
            HX_STAMP(ST_RT);
        }
        if (ep && tid == 0) {   // the ranks whose expert this GPU owns, in rank order
            int n = 0;
            for (int j = 0; j < K; j++)
                if (ids[j] % a.ep_size == a.ep_rank) s_own[n++] = j;
            s_nown = n;
        }
        __syncthreads();
        const int nown = ep ? s_nown : K;
        if (ep) {
            chunk_range(c, G, nown * cpe, &ch0, &ch1);
            nch_c = ch1 - ch0;
            if (nown > 0) {
                const int gi = down_group(c, G, nown);
                jd = s_own[gi];
                down_rows(c, G, nown, D, pl.ra, &dr0, &dr1);
                ndr = dr1 - dr0;
            } else {
                jd = 0;
                ndr = 0;
            }
        }
        // chunk index g -> (rank j, chunk p within the expert)
        auto chunk_rank = [&](int g, int *p) {
            const int o = g / cpe;
            *p = g - o * cpe;
            return ep ? s_own[o] : o;
        };
        if (warp == kIssueWarp) {   // a warp without a chunk (when nch_c < 16): the others start at once
            fence_proxy_async();
            for (int q = lane; q < pl.ch_max; q += 32) {   // chunk q: rows ch*p.. of gate and up, rank j
                if (q >= nch_c) {   // every chunk barrier completes one phase per layer
                    mbar_expect_tx(&bars[q], 0);
                    continue;
                }
                int p;
                const int g = ch0 + q, j = chunk_rank(g, &p);
                const uint8_t *slab = stab[ids[j]];
                if (!slab) {
                    set_error(a.err, DEV_E_NOT_RESIDENT);
                    mbar_expect_tx(&bars[q], 0);
                } else {
                    const int64_t r0 = (int64_t)p * CH;
                    uint8_t *dst = gu + (size_t)q * 2 * chunk_bytes;
                    mbar_expect_tx(&bars[q], 2 * chunk_bytes);
                    bulk_g2s(dst, slab + r0 * ly.rbD, chunk_bytes, &bars[q]);
                    bulk_g2s(dst + chunk_bytes, slab + a.off_up + r0 * ly.rbD, chunk_bytes, &bars[q]);
                }
            }
            if (lane == 0) {   // this CTA's slice of the rank-jd expert's down rows
                const uint8_t *slab = ndr > 0 ? stab[ids[jd]] : nullptr;
                if (ndr == 0) {
                    mbar_expect_tx(&bars[BAR_DOWN], 0);
                } else if (!slab) {
                    set_error(a.err, DEV_E_NOT_RESIDENT);
                    mbar_expect_tx(&bars[BAR_DOWN], 0);
                } else {
                    mbar_expect_tx(&bars[BAR_DOWN], (uint32_t)(ndr * ly.rbF));
                    bulk_g2s(dn, slab + a.off_down + (int64_t)dr0 * ly.rbF, (uint32_t)(ndr * ly.rbF), &bars[BAR_DOWN]);
                }
            }
            __syncwarp();
            if (lane == 0 && l + 1 < a.Lyr) {   // rrow / normv / stab are consumed
                fence_proxy_async();
                issue_router(l + 1);
            }
        }
        HX_STAMP(ST_ROUTE);

        // ---------------- P3: gate/up chunks -> SwiGLU -> mid exchange
        for (int q = warp; q < nch_c; q += DEC_WARPS) {
            int p;
            const int g = ch0 + q, j = chunk_rank(g, &p);
            if (mbar_wait(&bars[q], par, a.err)) {
                if (q == 0) HX_STAMP(ST_CH0);
                warp_rows_1tok<DT>(gu + (size_t)q * 2 * chunk_bytes, ly.rbD, ly.nbD, 2 * CH, xact, P, gout);
                if (lane < CH) st_x(xmid(l, j) + p * CH + lane, canon(swiglu_c(gout[lane], gout[CH + lane])));
                if (q == 0) HX_STAMP(ST_CHD);
            }
        }
        {   // reset this CTA's share of the other set's slots of buffer layers [b0, b1) for the next launch
            // (while this CTA waits for the other CTAs' mid values anyway)
            const int np = (int)min(s_prev, (unsigned)a.Lb);
            const int b0 = (int)((int64_t)np * l / a.Lyr), b1 = (int)((int64_t)np * (l + 1) / a.Lyr);
            const int64_t per_layer[4] = {E, (int64_t)K * F, (int64_t)K * D, D};
            const int64_t base[4] = {o_lg, o_mid, o_y, o_h};
            for (int k = 0; k < 4; k++)
                for (int b = b0; b < b1; b++) {
                    float *s0 = Xo + base[k] + (int64_t)b * per_layer[k];
                    for (int64_t i = (int64_t)c * DEC_THREADS + tid; i < per_layer[k]; i += (int64_t)G * DEC_THREADS)
                        s0[i] = __uint_as_float(kEmpty);
                }
        }
        HX_STAMP(ST_RESET);

        // ---------------- P4: expert jd's mid -> activation blocks -> this CTA's down rows -> y exchange
        if (ndr > 0) poll_vec(xmid(l, jd), mids, F, a.err);
        __syncthreads();
        HX_STAMP(ST_MIDP);
        for (int b = warp; b < ly.nbF && ndr > 0; b += DEC_WARPS)
            act_quant_warp(mids[b * QK + lane], mids[b * QK + lane + 32], amid + b, lane);
        __syncthreads();
        HX_STAMP(ST_MIDQ);
        {
            const bool ok = mbar_wait(&bars[BAR_DOWN], par, a.err);
            HX_STAMP(ST_DNW);
            const int pr = pl.prows;
            for (int r0 = warp * pr; r0 < ndr && ok; r0 += DEC_WARPS * pr)
                warp_rows_1tok<DT>(dn + (size_t)r0 * ly.rbF, ly.rbF, ly.nbF, min(pr, ndr - r0), amid, P, Ys + r0);
        }
        __syncthreads();
        HX_STAMP(ST_DOWN);
        if (!ep) {
            for (int r = tid; r < ndr; r += DEC_THREADS) st_x(xy(l, jd) + dr0 + r, Ys[r]);
        } else {   // every GPU's y words (its own included)
            const int64_t o = ((int64_t)l * K + jd) * D + dr0;
            for (int i = tid; i < ndr * a.ep_size; i += DEC_THREADS) {
                const int p = i / ndr, r = i - p * ndr;
                st_ep(a.ep_y[p] + o + r, ep_tag, Ys[r]);
            }
        }
        HX_STAMP(ST_YST);

        // ---------------- P5: y of the K experts for this CTA's h rows -> rank-order sum -> residual
        for (int i = tid; i < K * nhr; i += DEC_THREADS) {
            const int j = i / nhr, r = i - j * nhr;
            yv[i] = ep ? poll_ep(a.ep_y[a.ep_rank] + ((int64_t)l * K + j) * D + hr0 + r, ep_tag, a.err)
                       : poll1(xy(l, j) + hr0 + r, a.err);
        }
        __syncthreads();
        HX_STAMP(ST_Y);
        if (tid < nhr) {
            float o = 0.0f;   // rank-order sum (engine/src/model.c:904-923)
            for (int j = 0; j < K; j++) o = __fadd_rn(o, __fmul_rn(wts[j], yv[j * nhr + tid]));
            const float hn = __fadd_rn(hs[hr0 + tid], __fmul_rn(a.rs, o));
            if (l + 1 < a.Lyr) st_x(xh(l + 1) + hr0 + tid, canon(hn));
            else a.h[hr0 + tid] = hn;
        }
        if (l == a.Lyr - 1 && c == 0 && tid < K) {
            a.ids_out[tid] = ids[tid];
            a.w_out[tid] = wts[tid];
        }
        HX_STAMP(ST_SUM);
        __syncthreads();   // hs rows of P5 are read before the next layer's h lands in hs
#undef HX_STAMP
    }
    // every bulk copy this CTA issued has landed before it exits (already true unless a wait gave up)
    if (tid == 0 && a.Lyr > 0) {
        const uint32_t last = (uint32_t)((a.Lyr - 1) & 1);
        for (int q = 0; q < pl.ch_max; q++) mbar_wait(&bars[q], last, nullptr);
        mbar_wait(&bars[BAR_DOWN], last, nullptr);
        mbar_wait(&bars[BAR_ROUTER], last, nullptr);
        // the last CTA to finish advances the launch counter (every CTA read it at its start)
        if (atomicAdd(a.epoch + 1, 1u) == (unsigned)G - 1) {
            a.epoch[1] = 0u;
            a.epoch[2 + (s_epoch & 1u)] = (unsigned)a.Lyr;   // what the next launch resets of this set
            a.epoch[0] = s_epoch + 1u;
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(DEC_THREADS, 1) k_moe_decode(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    // a kernel launched after this one with programmatic stream serialization (the whole decoder's
    // next GEMV) may start as SMs free up and stream its weights; it waits for this grid before it
    // reads h
    pdl_trigger();
    if (a.dtype == Q4) decode_body<Q4>(a, smem);
    else decode_body<Q8>(a, smem);
}

// ------------------------------------------------------------------------------------- host side

int decode_stamps() { return DEC_STAMPS; }
int decode_max_layers() { return DEC_MAXL; }

int decode_grid() {
    static int cached[64] = {};
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (dev >= 0 && dev < 64) cached[dev] = sms;
    return sms;
}

int64_t decode_xbuf_floats(int Lb, int D, int F, int E, int K) { return 2 * xset_floats(Lb, D, F, E, K); }

bool decode_supported(int D, int F, int E, int K, int dtype, bool shared, int ep, std::string *why) {
    auto no = [&](const char *w) {
        if (why) *why = w;
        return false;
    };
    if (shared) return no("shared expert");
    if (dtype != Q4 && dtype != Q8) return no("dtype");
    if (row_bytes(dtype, D) % 16) return no("gate/up rows not a multiple of 16 bytes");
    if (K > 16) return no("top_k > 16");
    if (E % 4 || D % 4 || F % 4) return no("exchange vectors (D, F, E multiples of 4)");
    const int G = decode_grid();
    const DecodeLayout ly = decode_layout(G, D, F, E, K, dtype, ep);
    const DecodePlan &pl = ly.plan;
    if (pl.rpc > 2 * DEC_WARPS) return no("router rows per CTA");
    if (pl.ch_max > DEC_MAXCH) return no("gate/up chunks per CTA");
    if (G < K || D % pl.ra) return no("down groups");
    if (D / (G / K) < 2 * pl.ra) return no("down rows per CTA");
    int lim = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&lim, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, (const void *)k_moe_decode) != cudaSuccess) return no("kernel");
    if (ly.total + fa.sharedSizeBytes > (size_t)lim) return no("shared memory");
    return true;
}

cudaError_t init_decode_attributes() {
    int lim = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&lim, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, (const void *)k_moe_decode);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_moe_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, lim - (int)fa.sharedSizeBytes);
    return e;
}

cudaError_t launch_moe_decode(const DecodeParams &p, cudaStream_t s) {
    if (p.n_layers > p.buf_layers || p.n_layers > DEC_MAXL) return cudaErrorInvalidValue;
    DecodeArgs a;
    a.Lyr = p.n_layers;
    a.D = p.D;
    a.F = p.F;
    a.E = p.E;
    a.K = p.K;
    a.dtype = p.dtype;
    a.route = p.route;
    a.eps = p.eps;
    a.rs = p.rs;
    a.off_up = p.off_up;
    a.off_down = p.off_down;
    a.router = p.router;
    a.norm = p.norm;
    a.bias = p.bias;
    a.slab = p.slab;
    a.h = p.h;
    a.xbuf = p.xbuf;
    a.Lb = p.buf_layers;
    a.epoch = p.epoch;
    a.err = p.err;
    a.ids_out = p.ids_out;
    a.w_out = p.w_out;
    a.trace = p.trace;
    a.ep_size = p.ep_size;
    a.ep_rank = p.ep_rank;
    a.ep_y = p.ep_y;
    if (a.ep_size > 1 && !a.ep_y) return cudaErrorInvalidValue;
    const int G = decode_grid();
    a.lay = decode_layout(G, p.D, p.F, p.E, p.K, p.dtype, p.ep_size);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)G);
    cfg.blockDim = dim3(DEC_THREADS);
    cfg.dynamicSmemBytes = a.lay.total;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_moe_decode, a);
}

}  // namespace hx
