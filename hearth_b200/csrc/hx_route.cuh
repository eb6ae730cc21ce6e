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
__device__ __forceinline__ void route_token_warp(const RouteCfg &R, const float *logit, const float *bias, float *score,
                                 float *sel, int *ids_out, float *w_out) {
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
    for (int j = 0; j < K; j++) {
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
__device__ __forceinline__ void route_union_cta(int T, int K, int E, const int *ids, int *cnt, int *start, int *nu_out,
                                int *ulist, int *u_p0, int *u_n, int *pair_tok, int *pair_of) {
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int e = tid; e < E; e += nt) cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < T * K; i += nt) atomicAdd(&cnt[__ldcg(ids + i)], 1);
    __syncthreads();
    if (tid == 0) {
        int nu = 0, p = 0;
        for (int e = 0; e < E; e++) {
            start[e] = p;
            if (!cnt[e]) continue;
            ulist[nu] = e;
            u_p0[nu] = p;
            u_n[nu] = cnt[e];
            p += cnt[e];
            nu++;
        }
        *nu_out = nu;
    }
    __syncthreads();
    for (int e = tid; e < E; e += nt) {
        if (!cnt[e]) continue;
        int p = start[e];
        for (int t = 0; t < T; t++)
            for (int j = 0; j < K; j++)
                if (__ldcg(ids + t * K + j) == e) {
                    pair_tok[p] = t;
                    pair_of[t * K + j] = p;
                    p++;
                }
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

// Top-k routing of one token by a whole CTA (engine/src/model.c:793-843), for the decode path:
// logits -> score (softmax or sigmoid) -> selection value (+ bias) -> group mask -> top-K by rank.
// Each thread ranks its experts against all E: rank(i) = #{k : k ranks before i}; the order is
// total (ties to the lower index, NaN last), so the K experts with rank < K are exactly
// route_select's ids in descending order. lg, score, sel: [E] shared, key: [E] shared (8-byte
// aligned); gsc/keep: [n_group] shared; red: 4 floats.
// Results land in ids/w (shared, K each). Every thread of the CTA must call it.
__device__ __forceinline__ void route_token_cta(const RouteCfg &R, const float *logit_g, const float *bias,
                                                float *lg, unsigned long long *key, float *score, float *sel,
                                                float *gsc, int *keep, float *red, int *ids, float *w) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int E = R.E, K = R.K;
    for (int i = tid; i < E; i += nt) lg[i] = __ldcg(logit_g + i);
    __syncthreads();
    if (R.score_fn == SCORE_SOFTMAX) {
        if (warp == 0) {   // m = x[0]; m = x[i] > m ? x[i] : m  (a leading NaN stays)
            float m = -__uint_as_float(0x7f800000u);
            for (int i = lane; i < E; i += 32) m = fmaxf(m, lg[i]);
#pragma unroll
            for (int s = 16; s >= 1; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
            if (lane == 0) red[0] = lg[0] != lg[0] ? lg[0] : m;
        }
        __syncthreads();
        const float m = red[0];
        for (int i = tid; i < E; i += nt) score[i] = host_expf(__fsub_rn(lg[i], m));
        __syncthreads();
        if (warp == 0) {   // sum16 over E, then every score divided by it
            float L = 0.0f;
            if (lane < 16) {
#pragma unroll 8
                for (int i = lane; i < E; i += 16) L = __fadd_rn(L, score[i]);
            }
            L = tree16(L, 0xffffffffu);
            if (lane == 0) red[1] = L;
        }
        __syncthreads();
        const float ssum = red[1];
        for (int i = tid; i < E; i += nt) score[i] = __fdiv_rn(score[i], ssum);
    } else {
        for (int i = tid; i < E; i += nt) score[i] = sigmoid_c(lg[i]);
    }
    __syncthreads();
    for (int i = tid; i < E; i += nt) sel[i] = (R.score_bias && bias) ? __fadd_rn(score[i], bias[i]) : score[i];
    __syncthreads();
    if (R.n_group > 1) {
        const int ng = R.n_group, gs = E / ng;
        for (int g = tid; g < ng; g += nt) {   // group score: sum of the group's top-2 (model.c:801-812)
            const float *v = sel + g * gs;
            int i1 = 0, i2 = -1;
            for (int i = 1; i < gs; i++) {
                if (ranks_before(v[i], i, v[i1], i1)) {
                    i2 = i1;
                    i1 = i;
                } else if (i2 < 0 || ranks_before(v[i], i, v[i2], i2)) {
                    i2 = i;
                }
            }
            gsc[g] = i2 >= 0 ? __fadd_rn(v[i1], v[i2]) : v[i1];
        }
        __syncthreads();
        for (int g = tid; g < ng; g += nt) {   // keep the topk_group best groups
            int rk = 0;
            for (int o = 0; o < ng; o++) rk += ranks_before(gsc[o], o, gsc[g], g) ? 1 : 0;
            keep[g] = rk < R.topk_group;
        }
        __syncthreads();
        for (int i = tid; i < E; i += nt)
            if (!keep[i / gs]) sel[i] = 0.0f;
        __syncthreads();
    }
    // rank of each expert by a 64-bit key with the order of ranks_before: order-preserving bits of
    // the value (NaN lowest, -0 counted as +0), then the lower index first
    for (int i = tid; i < E; i += nt) key[i] = rank_key(sel[i], i);
    __syncthreads();
    {
        int P = 1;   // lanes per expert (a power of two <= 32 with E * P <= threads)
        while (P < 32 && E * (P * 2) <= nt) P *= 2;
        const int per = (E + P - 1) / P;
        for (int base = 0; base < E * P; base += nt) {
            const int t = base + tid, i = t / P, part = t - i * P;
            int rk = 0;
            unsigned long long ki = 0;
            if (i < E) {
                ki = key[i];
                const int o0 = part * per, o1 = min(E, o0 + per);
#pragma unroll 8
                for (int o = o0; o < o1; o++) rk += key[o] > ki ? 1 : 0;
            }
            for (int s = 1; s < P; s <<= 1) rk += __shfl_xor_sync(0xffffffffu, rk, s, P);
            if (i < E && part == 0 && rk < K) ids[rk] = i;
        }
    }
    __syncthreads();
    // route_weights (model.c:833-843): the renormalisation sum runs in rank order on one thread,
    // the divisions and routed_scale on K threads
    if (tid == 0) {
        float sacc = 0.0f;
        for (int j = 0; j < K; j++) sacc = __fadd_rn(sacc, score[ids[j]]);
        red[2] = __fadd_rn(sacc, 1e-20f);
    }
    __syncthreads();
    if (tid < K) {
        float v = score[ids[tid]];
        if (R.norm_topk_prob) v = __fdiv_rn(v, red[2]);
        w[tid] = __fmul_rn(v, R.routed_scale);
    }
    __syncthreads();
}

}  // namespace hx
