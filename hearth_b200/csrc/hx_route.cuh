// hx_route.cuh — device routines shared by the MoE kernels: activation quantization of one
// 64-block by a warp (NUMERICS §2), top-k routing of one token by a warp (route_select +
// route_weights) and the expert buckets of a batch (the union).
#pragma once

#include "hx_device.cuh"
#include "hx_kernels.h"

namespace hx {

// Activation quantization (NUMERICS §2, engine/src/quant.c:325-348) of the 64 values a warp holds
// as (x0 = element lane, x1 = element lane + 32).
__device__ __forceinline__ void act_quant_warp(float x0, float x1, act_q8 *o, int lane) {
    float amax = fmaxf(fabsf(x0), fabsf(x1));   // fmaxf drops NaN, like `a > amax` in C
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, s));
    amax = fmaxf(amax, 0.0f);
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    float v0 = __fmul_rn(x0, id), v1 = __fmul_rn(x1, id);
    if (v0 != v0) v0 = 0.0f;
    if (v1 != v1) v1 = 0.0f;
    v0 = v0 > 127.0f ? 127.0f : (v0 < -127.0f ? -127.0f : v0);
    v1 = v1 > 127.0f ? 127.0f : (v1 < -127.0f ? -127.0f : v1);
    const int q0 = __float2int_rn(v0), q1 = __float2int_rn(v1);   // round half to even
    int sum = q0 + q1;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
    o->q[lane] = (int8_t)q0;
    o->q[lane + 32] = (int8_t)q1;
    if (lane == 0) {
        o->d = d;
        o->sum = sum;
    }
}

// Top-k routing of one token by one warp (engine/src/model.c:793-843, NUMERICS §5.3).
// logit: [E] (global, written by other CTAs: read through L2), score/sel: [E] shared scratch.
// forced: null, or the token's K expert ids to use instead of the selection (route replay,
// engine/src/model.c:1003-1009: the scores are computed as usual, the ids come from a trace).
__device__ __forceinline__ void route_token_warp(const RouteCfg &R, const float *logit, const float *bias, float *score,
                                 float *sel, int *ids_out, float *w_out, const int *forced = nullptr) {
    const int lane = threadIdx.x & 31, E = R.E, K = R.K;
    if (R.score_fn == SCORE_SOFTMAX) {
        float m = -__uint_as_float(0x7f800000u);
        for (int i = lane; i < E; i += 32) m = fmaxf(m, __ldcg(logit + i));
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
        const float x0 = __ldcg(logit);
        if (x0 != x0) m = x0;   // `m = x[0]; m = x[i] > m ? x[i] : m` keeps a leading NaN
        for (int i = lane; i < E; i += 32) score[i] = host_expf(__fsub_rn(__ldcg(logit + i), m));
        __syncwarp();
        float L = 0.0f;
        if (lane < 16)
            for (int i = lane; i < E; i += 16) L = __fadd_rn(L, score[i]);
        L = tree16(L, 0xffffffffu);
        const float ssum = __shfl_sync(0xffffffffu, L, 0);
        for (int i = lane; i < E; i += 32) score[i] = __fdiv_rn(score[i], ssum);
    } else {
        for (int i = lane; i < E; i += 32) score[i] = sigmoid_c(__ldcg(logit + i));
    }
    __syncwarp();
    for (int i = lane; i < E; i += 32) sel[i] = (R.score_bias && bias) ? __fadd_rn(score[i], bias[i]) : score[i];
    __syncwarp();
    if (R.n_group > 1) {
        const int ng = R.n_group, gs = E / ng;
        // group score: sum of the group's top-2 selection values (model.c:801-812)
        float gsc = 0.0f;
        if (lane < ng) {
            const float *v = sel + lane * gs;
            int i1 = 0, i2 = -1;
            for (int i = 1; i < gs; i++) {
                if (ranks_before(v[i], i, v[i1], i1)) {
                    i2 = i1;
                    i1 = i;
                } else if (i2 < 0 || ranks_before(v[i], i, v[i2], i2)) {
                    i2 = i;
                }
            }
            gsc = i2 >= 0 ? __fadd_rn(v[i1], v[i2]) : v[i1];
        }
        unsigned keep = 0;
        for (int r = 0; r < R.topk_group; r++) {
            float bv = gsc;
            int bi = (lane < ng && !((keep >> lane) & 1u)) ? lane : -1;
#pragma unroll
            for (int s = 16; s >= 1; s >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, s);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, s);
                if (oi >= 0 && (bi < 0 || ranks_before(ov, oi, bv, bi))) {
                    bv = ov;
                    bi = oi;
                }
            }
            keep |= 1u << bi;
        }
        for (int i = lane; i < E; i += 32)
            if (!((keep >> (i / gs)) & 1u)) sel[i] = 0.0f;
        __syncwarp();
    }
    // top-K by selection value, descending, ties to the lower index, NaN last
    unsigned taken[12] = {0};   // E <= 384: lane owns i = lane + 32 m
    int myid = -1;
    if (forced) {   // replayed ids: no selection
        if (lane < K) myid = forced[lane];
    }
    for (int j = 0; j < K && !forced; j++) {
        float bv = 0.0f;
        int bi = -1;
        for (int m = 0, i = lane; i < E; m++, i += 32) {
            if (taken[m]) continue;
            const float v = sel[i];
            if (bi < 0 || ranks_before(v, i, bv, bi)) {
                bv = v;
                bi = i;
            }
        }
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, s);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, s);
            if (oi >= 0 && (bi < 0 || ranks_before(ov, oi, bv, bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if ((bi & 31) == lane) taken[bi >> 5] = 1u;
        if (lane == j) myid = bi;
    }
    // weights (route_weights, model.c:833-843): score of the chosen expert, optional
    // renormalisation by the rank-order sum + 1e-20f, then routed_scale
    // gather the K ids to every lane
    int idj = -1;
    float wj = 0.0f;
    if (lane < K) {
        idj = myid;
        wj = score[myid];
    }
    // sequential renormalisation sum in rank order (lane 0), then divide and scale
    float den = 1.0f;
    if (R.norm_topk_prob) {
        float s = 0.0f;
        for (int j = 0; j < K; j++) s = __fadd_rn(s, __shfl_sync(0xffffffffu, wj, j));
        den = __fadd_rn(s, 1e-20f);
    }
    if (lane < K) {
        float v = wj;
        if (R.norm_topk_prob) v = __fdiv_rn(v, den);
        v = __fmul_rn(v, R.routed_scale);
        ids_out[lane] = idj;
        w_out[lane] = v;
    }
}

// Expert buckets of the batch (engine/src/model.c:1020-1037), by one CTA: experts ascending,
// tokens ascending within an expert; pair_of[t*K + j] is the pair of token t's rank j.
// The union of routed experts and the bucket order (engine/src/model.c:1020-1037): experts
// ascending, and within an expert the pairs i = t*K + j ascending. One CTA, a stable counting sort
// in three barriers: warp w owns a contiguous range of pairs and counts its experts (lanes holding
// the same expert find each other with __match_any_sync, one leader adds their number); warp 0 scans
// the per-expert totals into bucket starts and the bucket list; each warp's first position in a
// bucket follows the lower warps' pairs of that bucket; then every warp walks its range in order and
// places its pairs. blockDim is a multiple of 32. Shared scratch: cnt [E], start [E] and
// wcnt [blockDim/32][E].
__device__ __forceinline__ void route_union_cta(int T, int K, int E, const int *ids, int *cnt, int *start, int *nu_out,
                                int *ulist, int *u_p0, int *u_n, int *pair_tok, int *pair_of, int *wcnt) {
    const int tid = threadIdx.x, nt = blockDim.x, TK = T * K, lane = tid & 31, warp = tid >> 5;
    const int nwarps = nt >> 5;   // blockDim is a multiple of 32
    const int per = (TK + nwarps - 1) / nwarps, i0 = min(TK, warp * per), i1 = min(TK, i0 + per);
    int *wh = wcnt + warp * E;    // this warp's counts per expert, then its next position per expert
    for (int k = tid; k < nwarps * E; k += nt) wcnt[k] = 0;
    __syncthreads();
    // 1. every warp counts the experts of its contiguous range of pairs (one leader per expert per round)
    for (int b = i0; b < i1; b += 32) {
        const int i = b + lane;
        const bool live = i < i1;
        const int e = live ? __ldcg(ids + i) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (live && (peers & ((1u << lane) - 1u)) == 0) wh[e] += __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    for (int e = tid; e < E; e += nt) {
        int c = 0;
        for (int w = 0; w < nwarps; w++) c += wcnt[w * E + e];
        cnt[e] = c;
    }
    __syncthreads();
    // 2. warp 0: bucket starts in expert order (exclusive scan of the counts) and the list of buckets
    if (warp == 0) {
        int run = 0, nrun = 0;
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < E ? cnt[e] : 0, f = c > 0 ? 1 : 0;
            int incl = c, fincl = f;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o), fv = __shfl_up_sync(0xffffffffu, fincl, o);
                if (lane >= o) {
                    incl += v;
                    fincl += fv;
                }
            }
            const int st = run + incl - c, u = nrun + fincl - f;
            if (e < E) {
                start[e] = st;
                if (c) {
                    ulist[u] = e;
                    u_p0[u] = st;
                    u_n[u] = c;
                }
            }
            run += __shfl_sync(0xffffffffu, incl, 31);
            nrun += __shfl_sync(0xffffffffu, fincl, 31);
        }
        if (lane == 0) *nu_out = nrun;
    }
    __syncthreads();
    for (int e = tid; e < E; e += nt) {   // warp w's first position in bucket e: after the lower warps' pairs
        int p = start[e];
        for (int w = 0; w < nwarps; w++) {
            const int c = wcnt[w * E + e];
            wcnt[w * E + e] = p;
            p += c;
        }
    }
    __syncthreads();
    // 3. every warp places its pairs, in pair order (so each bucket lists its tokens in ascending order)
    for (int b = i0; b < i1; b += 32) {
        const int i = b + lane;
        const bool live = i < i1;
        const int e = live ? __ldcg(ids + i) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        if (live) {
            const int p = wh[e] + rank;
            pair_tok[p] = i / K;
            pair_of[i] = p;
        }
        __syncwarp();
        if (live && rank == 0) wh[e] += __popc(peers);
        __syncwarp();
    }
}

// A key whose unsigned order is ranks_before's order (engine/src/model.c:221-226): larger values
// first, NaN after every number, -0 equal to +0, and among equal values the lower index first.
__device__ __forceinline__ unsigned long long rank_key(float v, int i) {
    uint32_t u;
    if (v != v) u = 0u;
    else {
        const uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
        u = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    }
    return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
}

// Top-k routing of one token by ONE warp, warp-synchronous (no CTA barrier), for the decode path:
// logits -> score (softmax or sigmoid) -> selection value (+ bias) -> group mask -> top-K.
// The top-K comes from ranks: rank(i) = #{o : key(o) > key(i)} with rank_key's order, which is
// route_select's (engine/src/model.c:793-831), so the experts with rank < K are its ids in order.
// lg/score/sel [E], key [E] (8-byte aligned), gsc/keep [n_group]: this warp's shared scratch.
// Results: ids[K], w[K] in shared memory, valid after the call for this warp (and for the CTA
// after its next barrier). kSharedLogits: logit_g is already this warp's shared copy (lg unused).
template <bool kSharedLogits = false>
__device__ __forceinline__ void route_token_warp1(const RouteCfg &R, const float *logit_g, const float *bias,
                                                  float *lg, unsigned long long *key, float *score, float *sel,
                                                  float *gsc, int *keep, int *ids, float *w) {
    const int lane = threadIdx.x & 31;
    const int E = R.E, K = R.K;
    if constexpr (kSharedLogits) {
        lg = const_cast<float *>(logit_g);
    } else {
        for (int i = lane; i < E; i += 32) lg[i] = __ldcg(logit_g + i);
    }
    __syncwarp();
    if (R.score_fn == SCORE_SOFTMAX) {
        float m = -__uint_as_float(0x7f800000u);   // m = x[0]; m = x[i] > m ? x[i] : m
        for (int i = lane; i < E; i += 32) m = fmaxf(m, lg[i]);
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
        if (lg[0] != lg[0]) m = lg[0];
        for (int i = lane; i < E; i += 32) score[i] = host_expf(__fsub_rn(lg[i], m));
        __syncwarp();
        float L = 0.0f;   // sum16 (NUMERICS §1)
        if (lane < 16) {
#pragma unroll 8
            for (int i = lane; i < E; i += 16) L = __fadd_rn(L, score[i]);
        }
        L = tree16(L, 0xffffffffu);
        const float ssum = __shfl_sync(0xffffffffu, L, 0);
        for (int i = lane; i < E; i += 32) score[i] = __fdiv_rn(score[i], ssum);
    } else {
        for (int i = lane; i < E; i += 32) score[i] = sigmoid_c(lg[i]);
    }
    __syncwarp();
    for (int i = lane; i < E; i += 32) sel[i] = (R.score_bias && bias) ? __fadd_rn(score[i], __ldg(bias + i)) : score[i];
    __syncwarp();
    if (R.n_group > 1) {
        const int ng = R.n_group, gs = E / ng;
        if (lane < ng) {   // group score: sum of the group's top-2 (model.c:801-812)
            const float *v = sel + lane * gs;
            int i1 = 0, i2 = -1;
            for (int i = 1; i < gs; i++) {
                if (ranks_before(v[i], i, v[i1], i1)) {
                    i2 = i1;
                    i1 = i;
                } else if (i2 < 0 || ranks_before(v[i], i, v[i2], i2)) {
                    i2 = i;
                }
            }
            gsc[lane] = i2 >= 0 ? __fadd_rn(v[i1], v[i2]) : v[i1];
        }
        __syncwarp();
        if (lane < ng) {   // keep the topk_group best groups
            int rk = 0;
            for (int o = 0; o < ng; o++) rk += ranks_before(gsc[o], o, gsc[lane], lane) ? 1 : 0;
            keep[lane] = rk < R.topk_group;
        }
        __syncwarp();
        for (int i = lane; i < E; i += 32)
            if (!keep[i / gs]) sel[i] = 0.0f;
        __syncwarp();
    }
    for (int i = lane; i < E; i += 32) key[i] = rank_key(sel[i], i);
    __syncwarp();
    for (int i0 = 0; i0 < E; i0 += 128) {   // up to 4 of this lane's experts ranked per sweep
        unsigned long long k4[4];
        int r4[4] = {0, 0, 0, 0};
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const int i = i0 + t * 32 + lane;
            k4[t] = i < E ? key[i] : ~0ull;
        }
#pragma unroll 4
        for (int o = 0; o < E; o++) {
            const unsigned long long ko = key[o];
#pragma unroll
            for (int t = 0; t < 4; t++) r4[t] += ko > k4[t] ? 1 : 0;
        }
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const int i = i0 + t * 32 + lane;
            if (i < E && r4[t] < K) ids[r4[t]] = i;
        }
    }
    __syncwarp();
    // route_weights (model.c:833-843): rank-order renormalisation sum, division, routed_scale
    float wj = lane < K ? score[ids[lane]] : 0.0f;
    float sacc = 0.0f;
    for (int j = 0; j < K; j++) sacc = __fadd_rn(sacc, __shfl_sync(0xffffffffu, wj, j));
    const float den = __fadd_rn(sacc, 1e-20f);
    if (lane < K) {
        if (R.norm_topk_prob) wj = __fdiv_rn(wj, den);
        w[lane] = __fmul_rn(wj, R.routed_scale);
    }
    __syncwarp();
}

// Top-k routing of one token by ONE warp, for E <= 128 and K <= 16 without expert groups, with no
// CTA barrier: lane l holds experts l, l + 32, l + 64, l + 96 in registers. Softmax: the maximum by
// shuffles (a NaN x[0] is kept, as `m = x[0]; m = x[i] > m ? x[i] : m`), exp per expert, the sum16
// in NUMERICS §1 order (lane j < 16 adds e[j + 16k], k = 0..7: its own values and lane j + 16's),
// then one division per expert; sigmoid scores need none of it. Selection (route_select,
// engine/src/model.c:793-831): each lane sorts its 4 rank_keys, then K rounds take the warp maximum of
// the lanes' heads (the high words by one reduction, then the low words of the lanes that hold that
// high word; a low word encodes the expert, so one lane wins) and the winner records pick r and pops
// its head. Weights as route_weights (model.c:833-843). ids / w / vs (K floats of scratch) are shared
// memory; the warp's lanes see ids and w after the call, the CTA after its next barrier.
template <bool kSharedLogits = false>
__device__ __forceinline__ void route_token_warp128(const RouteCfg &R, const float *logit, const float *bias, int *ids,
                                                    float *w, float *vs) {
    const int lane = threadIdx.x & 31;
    const int E = R.E, K = R.K;
    float x[4], sc[4];
#pragma unroll
    for (int t = 0; t < 4; t++) {
        const int i = t * 32 + lane;
        x[t] = i < E ? (kSharedLogits ? logit[i] : __ldcg(logit + i)) : 0.0f;
    }
    if (R.score_fn == SCORE_SOFTMAX) {
        float m = -__uint_as_float(0x7f800000u);
#pragma unroll
        for (int t = 0; t < 4; t++)
            if (t * 32 + lane < E) m = fmaxf(m, x[t]);
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
        const float x0 = __shfl_sync(0xffffffffu, x[0], 0);
        if (x0 != x0) m = x0;
        float e[4], o[4];
#pragma unroll
        for (int t = 0; t < 4; t++) e[t] = t * 32 + lane < E ? host_expf(__fsub_rn(x[t], m)) : 0.0f;
#pragma unroll
        for (int t = 0; t < 4; t++) o[t] = __shfl_down_sync(0xffffffffu, e[t], 16);   // lane j + 16's
        float L = 0.0f;
        if (lane < 16) {
#pragma unroll
            for (int k = 0; k < 8; k++)   // expert lane + 16k: k even in this lane (slot k/2), odd in lane + 16
                if (lane + 16 * k < E) L = __fadd_rn(L, (k & 1) ? o[k >> 1] : e[k >> 1]);
        }
        L = tree16(L, 0xffffffffu);
        const float den = __shfl_sync(0xffffffffu, L, 0);
#pragma unroll
        for (int t = 0; t < 4; t++) sc[t] = __fdiv_rn(e[t], den);
    } else {
#pragma unroll
        for (int t = 0; t < 4; t++) sc[t] = sigmoid_c(x[t]);
    }
    uint32_t kh[4], kl[4];   // rank_key halves; (0, 0) below every expert's key
#pragma unroll
    for (int t = 0; t < 4; t++) {
        const int i = t * 32 + lane;
        kh[t] = kl[t] = 0u;
        if (i < E) {
            const float sv = (R.score_bias && bias) ? __fadd_rn(sc[t], __ldg(bias + i)) : sc[t];
            const unsigned long long k = rank_key(sv, i);
            kh[t] = (uint32_t)(k >> 32);
            kl[t] = (uint32_t)k;
        }
    }
    auto cswap = [&](int a, int b) {   // slot a keeps the larger key
        const bool sw = kh[b] > kh[a] || (kh[b] == kh[a] && kl[b] > kl[a]);
        if (sw) {
            const uint32_t th = kh[a], tl = kl[a];
            const float ts = sc[a];
            kh[a] = kh[b]; kl[a] = kl[b]; sc[a] = sc[b];
            kh[b] = th; kl[b] = tl; sc[b] = ts;
        }
    };
    cswap(0, 1);
    cswap(2, 3);
    cswap(0, 2);
    cswap(1, 3);
    cswap(1, 2);
    for (int r = 0; r < K; r++) {
        const uint32_t mh = __reduce_max_sync(0xffffffffu, kh[0]);
        const bool cand = kh[0] == mh;
        const uint32_t ml = __reduce_max_sync(0xffffffffu, cand ? kl[0] : 0u);
        if (cand && kl[0] == ml) {   // the winner: pick r, then its next key moves up
            ids[r] = (int)(0xffffffffu - ml);
            vs[r] = sc[0];
            kh[0] = kh[1]; kl[0] = kl[1]; sc[0] = sc[1];
            kh[1] = kh[2]; kl[1] = kl[2]; sc[1] = sc[2];
            kh[2] = kh[3]; kl[2] = kl[3]; sc[2] = sc[3];
            kh[3] = kl[3] = 0u;
        }
    }
    __syncwarp();
    float sacc = 0.0f, wj = 0.0f;   // route_weights: every lane forms the rank-order sum itself
#pragma unroll
    for (int j = 0; j < 16; j++)
        if (j < K) {
            const float vj = vs[j];
            sacc = __fadd_rn(sacc, vj);
            if (j == lane) wj = vj;
        }
    const float den = __fadd_rn(sacc, 1e-20f);
    if (lane < K) {
        if (R.norm_topk_prob) wj = __fdiv_rn(wj, den);
        w[lane] = __fmul_rn(wj, R.routed_scale);
    }
    __syncwarp();
}

}  // namespace hx
