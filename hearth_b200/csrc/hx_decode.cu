// hx_decode.cu — the persistent single-token decode kernel of the MoE stack.
//
// One cooperative launch evaluates every layer of the stack for one token, with one CTA per SM.
// Per layer (engine/src/model.c:1209-1214 FFN half of forward, 986-1131 moe_layer):
//   A  every CTA: x = rmsnorm(h, ffn_norm) (redundantly), the activation blocks of x, and its share
//      of the F32 router rows (dot16);                                   grid barrier
//   B  every CTA: softmax/sigmoid top-k routing of the 128 logits (redundantly), then it bulk-copies
//      its contiguous share of the K experts' gate/up rows AND its share of the down rows into
//      shared memory at once, computes gate/up, SwiGLU, and the mid activation block of every
//      64-row block it completes (per-block arrival counters);          grid barrier
//   C  every CTA: its down rows of all K experts, the rank-order weighted sum and h += rs * sum for
//      those rows;                                                       grid barrier
// The router rows and ffn_norm of layer l+1 are copied in while layer l runs.
// Every float result follows the canonical order of the reference's NUMERICS §1-§5, exactly as the
// multi-kernel path does (same device routines).
//
// Grid barriers are sense-reversing arrival counters in global memory with bounded spins; a wait
// that runs out records an error in the device error word and lets the CTA continue, so a fault of
// the protocol ends the launch with an error status instead of a hang.
#include "hx_device.cuh"
#include "hx_kernels.h"
#include "hx_route.cuh"

#include <algorithm>
#include <string>

namespace hx {

enum : int { DEV_E_BARRIER = 4 };
constexpr uint32_t kBarrierSpinLimit = 1u << 21;
constexpr int DEC_THREADS = 512;
constexpr int DEC_WARPS = DEC_THREADS / 32;
constexpr int DEC_CH = 4;          // gate/up row pairs per chunk (one bulk-copy group)
constexpr int DEC_PROWS = 8;       // rows per warp_rows_1tok call (P buffer rows)
constexpr int DEC_MAXL = 128;      // layers per launch (router / norm / bias pointer tables in smem)
constexpr int BAR_DOWN = 28, BAR_ROUTER = 29;
// Phase stamps of the optional timeline (thread 0 of every CTA, per layer).
enum : int { ST_START, ST_NORM, ST_ROUTER, ST_BAR1, ST_ROUTE, ST_GATEUP, ST_MID, ST_BAR2, ST_DOWN, ST_SUM, ST_BAR3,
             DEC_STAMPS };

// Shared-memory carve-up of one CTA (identical on host and device). The router rows and ffn_norm
// of a layer share the gate/up region: they are read in phase A and copied in after the previous
// layer's gate/up rows were consumed.
struct DecodeLayout {
    int G, R, rpc, units;              // CTAs, down rows / CTA, router rows / CTA, gate/up units (64-row blocks)
    int nbD, nbF;
    int64_t rbD, rbF;
    size_t off_hs, off_stab, off_xact, off_gu, off_rrow, off_norm, off_dn, off_amid, off_y, off_p, off_gout,
        off_mloc, off_lg, off_score, off_sel, off_key, off_gsc, off_keep, off_ids, off_w, off_ptrs, total;
};

HX_HD inline size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

HX_HD inline DecodeLayout decode_layout(int G, int D, int F, int E, int K, int dtype) {
    DecodeLayout L{};
    L.G = G;
    L.nbD = D / QK;
    L.nbF = F / QK;
    L.rbD = row_bytes(dtype, D);
    L.rbF = row_bytes(dtype, F);
    // down rows per CTA: R * rbF must be a multiple of 16 bytes for the bulk copies
    int ra = 1;
    while ((ra * L.rbF) % 16) ra++;
    L.R = (D + G - 1) / G;
    L.R = (L.R + ra - 1) / ra * ra;
    L.rpc = (E + G - 1) / G;
    L.units = K * L.nbF;
    size_t o = 512;   // mbarriers
    L.off_hs = o; o = align16(o + (size_t)D * 4);
    L.off_stab = o; o = align16(o + (size_t)E * 8);
    L.off_xact = o; o = align16(o + (size_t)L.nbD * ACT_BLOCK);
    L.off_gu = o;
    const size_t gu_bytes = (size_t)QK * 2 * L.rbD, rr_bytes = (size_t)(L.rpc + 1) * D * 4;
    L.off_rrow = o;
    L.off_norm = o + (size_t)L.rpc * D * 4;
    o = align16(o + (gu_bytes > rr_bytes ? gu_bytes : rr_bytes));
    L.off_dn = o; o = align16(o + (size_t)K * L.R * L.rbF);
    L.off_amid = o; o = align16(o + (size_t)K * L.nbF * ACT_BLOCK);
    L.off_y = o; o = align16(o + (size_t)K * L.R * 4);
    L.off_p = o; o = align16(o + (size_t)DEC_WARPS * DEC_PROWS * 33 * 4);
    L.off_gout = o; o = align16(o + (size_t)DEC_WARPS * DEC_PROWS * 4);
    L.off_mloc = o; o = align16(o + (size_t)QK * 4);
    L.off_lg = o; o = align16(o + (size_t)E * 4);
    L.off_score = o; o = align16(o + (size_t)E * 4);
    L.off_sel = o; o = align16(o + (size_t)E * 4);
    L.off_key = o; o = align16(o + (size_t)((E + 3) / 4 * 4) * 8);
    L.off_gsc = o; o = align16(o + 64 * 4);
    L.off_keep = o; o = align16(o + 64 * 4);
    L.off_ids = o; o = align16(o + (size_t)K * 4);
    L.off_w = o; o = align16(o + (size_t)K * 4);
    L.off_ptrs = o; o = align16(o + (size_t)3 * DEC_MAXL * 8);
    L.total = o;
    return L;
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
    float *logits;                // [E]
    float *mbuf;                  // [K, F] SwiGLU outputs
    act_q8 *act_mid;              // [K, F/64]
    unsigned *bar;                // [DEC_BAR_LINES * 32] barrier counters (zero at allocation)
    unsigned bar_base;            // barriers completed by earlier launches (3 * layers per launch)
    unsigned *blk_cnt;            // [Lyr, K, F/64] arrival counters (zero between launches)
    int *err;
    int *ids_out;                 // [K] routing of the last layer
    float *w_out;
    unsigned long long *trace;    // null, or [Lyr][G][DEC_STAMPS] SM clock stamps of thread 0
    DecodeLayout lay;
};

__device__ __forceinline__ unsigned long long sm_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %clock64;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned atom_add_release(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.release.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier on one counter: after the block barrier, thread 0 adds 1 with a release reduction
// (the block barrier orders the other threads' writes before it, so no separate fence), and lane 0..
// of warp 0 poll with acquire loads until the counter reaches the target. The target grows by the
// grid size with every barrier and across launches (the host passes each launch's first barrier
// number), so nothing is ever reset; the 32-bit counts are compared wrap-safely. Counters spread
// over several 128-byte lines measured slower than one on B200 (2482 vs 2290 cycles a barrier), so
// DEC_BAR_LINES is 1; the code keeps the general form.
constexpr int DEC_BAR_LINES = 1;

__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void grid_sync(unsigned *ctr, unsigned target, int *err) {
    __syncthreads();
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        if (lane == 0) red_release_add(ctr + (blockIdx.x % DEC_BAR_LINES) * 32, 1u);
        for (uint32_t spins = 0;; spins++) {
            const unsigned v = lane < DEC_BAR_LINES ? ld_acquire(ctr + lane * 32) : 0u;
            const unsigned sum = __reduce_add_sync(0xffffffffu, v);
            if ((int)(sum - target) >= 0) break;
            if (spins > kBarrierSpinLimit || ((spins & 1023u) == 0 && *(volatile int *)err)) {
                if (lane == 0) set_error(err, DEV_E_BARRIER);
                break;
            }
        }
    }
    __syncthreads();
}

// Rows [0, nr) of a tile whose rows are consecutive in shared memory, against one activation row
// of nb blocks. out[k] = canonical NUMERICS §3 value of row k. nr <= DEC_PROWS.
template <int DT>
__device__ __forceinline__ void warp_rows_1tok(const uint8_t *tile, int64_t rb, int nb, int nr, const act_q8 *act,
                                               float *P, float *out) {
    const int lane = threadIdx.x & 31;
    constexpr int BS = DT == Q4 ? Q4_BLOCK : Q8_BLOCK;
    float acc = 0.0f;
    for (int g0 = 0; g0 < nb; g0 += 32) {
        const int gn = min(32, nb - g0);
        if (gn == 32) {   // lane = block: its activation block stays in registers for every row
            act_regs ar;
            load_act(act + g0 + lane, ar);
            const uint8_t *col = tile + (int64_t)(g0 + lane) * BS;
            for (int k = 0; k < nr; k++) {
                const uint8_t *blk = col + (int64_t)k * rb;
                int isum;
                uint32_t sc;
                if constexpr (DT == Q4) {
                    uint32_t nib[8];
                    sc = load_q4_block(blk, nib);
                    isum = q4_isum(nib, ar.q, ar.sum);
                } else {
                    uint32_t q[16];
                    sc = load_q8_block(blk, q);
                    isum = q8_isum(q, ar.q);
                }
                P[k * 33 + lane] = __fmul_rn(__int2float_rn(isum), __fmul_rn(f16_to_f32(sc), ar.d));
            }
        } else {
            for (int it = lane; it < nr * gn; it += 32) {
                const int k = it / gn, g = it - k * gn;
                const uint8_t *blk = tile + (int64_t)k * rb + (int64_t)(g0 + g) * BS;
                act_regs ar;
                load_act(act + g0 + g, ar);
                int isum;
                uint32_t sc;
                if constexpr (DT == Q4) {
                    uint32_t nib[8];
                    sc = load_q4_block(blk, nib);
                    isum = q4_isum(nib, ar.q, ar.sum);
                } else {
                    uint32_t q[16];
                    sc = load_q8_block(blk, q);
                    isum = q8_isum(q, ar.q);
                }
                P[k * 33 + g] = __fmul_rn(__int2float_rn(isum), __fmul_rn(f16_to_f32(sc), ar.d));
            }
        }
        __syncwarp();
        if (lane < nr) {
            const float *p = P + lane * 33;
#pragma unroll 8
            for (int g = 0; g < gn; g++) acc = __fadd_rn(acc, p[g]);
        }
        __syncwarp();
    }
    if (lane < nr) out[lane] = canon(acc);
    __syncwarp();
}

template <int DT>
__device__ void decode_body(const DecodeArgs &a, uint8_t *smem) {
    const DecodeLayout &ly = a.lay;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, G = gridDim.x;
    const int D = a.D, E = a.E, K = a.K;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    float *hs = reinterpret_cast<float *>(smem + ly.off_hs);   // h, then x in place
    const uint8_t **stab = reinterpret_cast<const uint8_t **>(smem + ly.off_stab);   // this layer's slabs
    act_q8 *xact = reinterpret_cast<act_q8 *>(smem + ly.off_xact);
    uint8_t *gu = smem + ly.off_gu;
    float *rrow = reinterpret_cast<float *>(smem + ly.off_rrow);
    float *normv = reinterpret_cast<float *>(smem + ly.off_norm);
    uint8_t *dn = smem + ly.off_dn;
    act_q8 *amid = reinterpret_cast<act_q8 *>(smem + ly.off_amid);
    float *Y = reinterpret_cast<float *>(smem + ly.off_y);
    float *P = reinterpret_cast<float *>(smem + ly.off_p) + warp * DEC_PROWS * 33;
    float *gout = reinterpret_cast<float *>(smem + ly.off_gout) + warp * DEC_PROWS;
    float *mloc = reinterpret_cast<float *>(smem + ly.off_mloc);
    float *lgs = reinterpret_cast<float *>(smem + ly.off_lg);
    float *score = reinterpret_cast<float *>(smem + ly.off_score);
    float *sel = reinterpret_cast<float *>(smem + ly.off_sel);
    unsigned long long *rkey = reinterpret_cast<unsigned long long *>(smem + ly.off_key);
    float *gscr = reinterpret_cast<float *>(smem + ly.off_gsc);
    int *gkeep = reinterpret_cast<int *>(smem + ly.off_keep);
    int *ids = reinterpret_cast<int *>(smem + ly.off_ids);
    float *wts = reinterpret_cast<float *>(smem + ly.off_w);
    const float **p_router = reinterpret_cast<const float **>(smem + ly.off_ptrs);
    const float **p_norm = p_router + DEC_MAXL, **p_bias = p_norm + DEC_MAXL;
    __shared__ float rms_r;
    for (int i = tid; i < a.Lyr; i += DEC_THREADS) {
        p_router[i] = a.router[i];
        p_norm[i] = a.norm[i];
        p_bias[i] = a.bias[i];
    }

    // this CTA's gate/up unit: the 64-row block b of the rank-j expert (one mid activation block)
    const bool has_unit = c < ly.units;
    const int uj = has_unit ? c / ly.nbF : 0, ub = has_unit ? c - uj * ly.nbF : 0;
    const int d0 = c * ly.R, d1 = min(D, d0 + ly.R), nrow = max(0, d1 - d0);
    const uint32_t chunk_bytes = (uint32_t)(DEC_CH * ly.rbD);
    const bool small_route = E <= 128 && a.route.n_group <= 1;

    if (tid == 0) {
        for (int i = 0; i < 32; i++) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue_router = [&](int l) {   // router rows e = c + t*G, ffn_norm and the slab pointers of layer l
        uint32_t bytes = (uint32_t)D * 4 + (uint32_t)E * 8;
        for (int t = 0; t < ly.rpc; t++)
            if (c + t * G < E) bytes += (uint32_t)D * 4;
        mbar_expect_tx(&bars[BAR_ROUTER], bytes);
        bulk_g2s(normv, p_norm[l], (uint32_t)D * 4, &bars[BAR_ROUTER]);
        bulk_g2s(stab, a.slab + (size_t)l * E, (uint32_t)E * 8, &bars[BAR_ROUTER]);
        for (int t = 0; t < ly.rpc; t++)
            if (c + t * G < E)
                bulk_g2s(rrow + (size_t)t * D, p_router[l] + (size_t)(c + t * G) * D, (uint32_t)D * 4,
                         &bars[BAR_ROUTER]);
    };
    if (tid == 0) issue_router(0);

    unsigned long long *stamp = nullptr;
    unsigned nbar = a.bar_base;   // barriers passed so far
    auto barrier = [&]() { grid_sync(a.bar, (++nbar) * (unsigned)G, a.err); };
    for (int l = 0; l < a.Lyr; l++) {
        const uint32_t par = (uint32_t)(l & 1);
        if (a.trace) stamp = a.trace + ((size_t)l * G + c) * DEC_STAMPS;
#define HX_STAMP(i) \
    if (stamp && tid == 0) stamp[i] = sm_clock()
        HX_STAMP(ST_START);
        // ---------------- phase A: rmsnorm, activations, router rows
        for (int i = tid; i < D; i += DEC_THREADS) hs[i] = __ldcg(a.h + i);
        __syncthreads();
        if (warp == 0) {
            float L = 0.0f;
            if (lane < 16) {
#pragma unroll 8
                for (int i = lane; i < D; i += 16) L = __fadd_rn(L, __fmul_rn(hs[i], hs[i]));
            }
            L = tree16(L, 0xffffffffu);
            if (lane == 0) rms_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(L, (float)D), a.eps)));
        }
        mbar_wait(&bars[BAR_ROUTER], par, a.err);
        __syncthreads();
        HX_STAMP(ST_NORM);
        {
            const float r = rms_r;
            for (int i = tid; i < D; i += DEC_THREADS) hs[i] = __fmul_rn(__fmul_rn(hs[i], r), normv[i]);
        }
        __syncthreads();
        for (int b = warp; b < ly.nbD; b += DEC_WARPS) act_quant_warp(hs[b * QK + lane], hs[b * QK + lane + 32], xact + b, lane);
        {   // router rows: one 16-lane group each (warp-uniform tree; idle groups add zeros)
            const int t = tid >> 4, j = tid & 15;
            const bool active = t < ly.rpc && c + t * G < E;
            float L = 0.0f;
            if (active) {
                const float *w = rrow + (size_t)t * D;
#pragma unroll 8
                for (int i = j; i < D; i += 16) L = __fadd_rn(L, __fmul_rn(w[i], hs[i]));
            }
            if (warp < (ly.rpc + 1) / 2) {
                L = tree16(L, 0xffffffffu);
                if (active && j == 0) a.logits[c + t * G] = canon(L);
            }
        }
        HX_STAMP(ST_ROUTER);
        barrier();
        HX_STAMP(ST_BAR1);

        // ---------------- phase B: routing (warp 0), copies in flight, gate/up + SwiGLU, mid block
        if (small_route) route_token_cta_small(a.route, a.logits, p_bias[l], score, rkey, ids, wts);
        if (warp == 0) {
            if (!small_route)
                route_token_warp1(a.route, a.logits, p_bias[l], lgs, rkey, score, sel, gscr, gkeep, ids, wts);
            if (lane == 0) HX_STAMP(ST_ROUTE);
            fence_proxy_async();
            if (has_unit) {   // gate/up rows of the unit: chunk q = rows 4q..4q+3 of gate and of up
                const uint8_t *slab = stab[ids[uj]];
                if (lane < QK / DEC_CH) {
                    if (!slab) {
                        if (lane == 0) set_error(a.err, DEV_E_NOT_RESIDENT);
                        mbar_expect_tx(&bars[lane], 0);
                    } else {
                        const int64_t r0 = (int64_t)ub * QK + lane * DEC_CH;
                        uint8_t *dst = gu + (size_t)lane * 2 * chunk_bytes;
                        mbar_expect_tx(&bars[lane], 2 * chunk_bytes);
                        bulk_g2s(dst, slab + r0 * ly.rbD, chunk_bytes, &bars[lane]);
                        bulk_g2s(dst + chunk_bytes, slab + a.off_up + r0 * ly.rbD, chunk_bytes, &bars[lane]);
                    }
                }
            }
            if (nrow > 0) {   // down rows [d0, d1) of the K experts on one barrier
                const uint8_t *slab = lane < K ? stab[ids[lane]] : nullptr;
                const bool have = slab != nullptr;
                if (lane < K && !have) set_error(a.err, DEV_E_NOT_RESIDENT);
                const unsigned nhave = __popc(__ballot_sync(0xffffffffu, have));
                if (lane == 0) mbar_expect_tx(&bars[BAR_DOWN], nhave * (uint32_t)(nrow * ly.rbF));
                __syncwarp();
                if (have)
                    bulk_g2s(dn + (size_t)lane * ly.R * ly.rbF, slab + a.off_down + (int64_t)d0 * ly.rbF,
                             (uint32_t)(nrow * ly.rbF), &bars[BAR_DOWN]);
            }
            __syncwarp();
        }
        if (has_unit) {   // warp q: chunk q (4 gate rows then 4 up rows) -> 4 SwiGLU values
            const int q = warp;
            if (q < QK / DEC_CH && mbar_wait(&bars[q], par, a.err)) {
                warp_rows_1tok<DT>(gu + (size_t)q * 2 * chunk_bytes, ly.rbD, ly.nbD, 2 * DEC_CH, xact, P, gout);
                if (lane < DEC_CH) mloc[q * DEC_CH + lane] = swiglu_c(gout[lane], gout[DEC_CH + lane]);
            }
        }
        __syncthreads();
        HX_STAMP(ST_GATEUP);
        if (has_unit && warp == 0) {   // the unit's mid activation block (NUMERICS §2)
            act_quant_warp(mloc[lane], mloc[lane + 32], a.act_mid + (size_t)uj * ly.nbF + ub, lane);
            __threadfence();
        }
        if (tid == 0) {   // gate/up rows are consumed: the next layer's router rows may land there
            fence_proxy_async();
            if (l + 1 < a.Lyr) issue_router(l + 1);
        }
        HX_STAMP(ST_MID);
        barrier();
        HX_STAMP(ST_BAR2);

        // ---------------- phase C: down rows, rank-order sum, residual
        {
            const uint32_t *src = reinterpret_cast<const uint32_t *>(a.act_mid);
            uint32_t *dst = reinterpret_cast<uint32_t *>(amid);
            for (int i = tid; i < K * ly.nbF * (ACT_BLOCK / 4); i += DEC_THREADS) dst[i] = __ldcg(src + i);
        }
        __syncthreads();
        if (nrow > 0) {
            const bool ok = mbar_wait(&bars[BAR_DOWN], par, a.err);
            const int per = (nrow + DEC_PROWS - 1) / DEC_PROWS;   // row groups per expert
            for (int u = warp; u < K * per && ok; u += DEC_WARPS) {
                const int j = u / per, r0 = (u - j * per) * DEC_PROWS, nr = min(DEC_PROWS, nrow - r0);
                warp_rows_1tok<DT>(dn + ((size_t)j * ly.R + r0) * ly.rbF, ly.rbF, ly.nbF, nr,
                                   amid + (size_t)j * ly.nbF, P, Y + (size_t)j * ly.R + r0);
            }
        }
        __syncthreads();
        HX_STAMP(ST_DOWN);
        if (tid < nrow) {
            float o = 0.0f;
            for (int j = 0; j < K; j++) o = __fadd_rn(o, __fmul_rn(wts[j], Y[(size_t)j * ly.R + tid]));
            float *hp = a.h + d0 + tid;
            __stcg(hp, __fadd_rn(__ldcg(hp), __fmul_rn(a.rs, o)));
        }
        if (l == a.Lyr - 1 && c == 0 && tid < K) {
            a.ids_out[tid] = ids[tid];
            a.w_out[tid] = wts[tid];
        }
        HX_STAMP(ST_SUM);
        barrier();
        HX_STAMP(ST_BAR3);
#undef HX_STAMP
    }
    // every bulk copy this CTA issued has landed before it exits (already true unless a wait gave up)
    if (tid == 0 && a.Lyr > 0) {
        const uint32_t last = (uint32_t)((a.Lyr - 1) & 1);
        if (has_unit)
            for (int q = 0; q < QK / DEC_CH; q++) mbar_wait(&bars[q], last, nullptr);
        if (nrow > 0) mbar_wait(&bars[BAR_DOWN], last, nullptr);
        mbar_wait(&bars[BAR_ROUTER], last, nullptr);
    }
    __syncthreads();
}

__global__ void __launch_bounds__(DEC_THREADS, 1) k_moe_decode(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
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

size_t decode_smem_bytes(int D, int F, int E, int K, int dtype) {
    return decode_layout(decode_grid(), D, F, E, K, dtype).total;
}

bool decode_supported(int D, int F, int E, int K, int dtype, bool shared, std::string *why) {
    auto no = [&](const char *w) {
        if (why) *why = w;
        return false;
    };
    if (shared) return no("shared expert");
    if (dtype != Q4 && dtype != Q8) return no("dtype");
    if (row_bytes(dtype, D) % 16) return no("gate/up rows not a multiple of 16 bytes");
    if (K > 16) return no("top_k > 16");
    if (E % 2) return no("odd expert count (slab pointer row not a multiple of 16 bytes)");
    const int G = decode_grid();
    const DecodeLayout ly = decode_layout(G, D, F, E, K, dtype);
    if (ly.rpc > 2 * DEC_WARPS) return no("router rows per CTA");
    if (ly.R > DEC_PROWS * DEC_WARPS) return no("down rows per CTA");
    if (ly.units > G) return no("more gate/up blocks (top_k * F / 64) than SMs");
    (void)0;
    if (QK / DEC_CH > DEC_WARPS || QK / DEC_CH > BAR_DOWN) return no("chunking");
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
    a.logits = p.logits;
    a.mbuf = p.mbuf;
    a.act_mid = p.act_mid;
    a.bar = p.bar;
    a.bar_base = p.bar_base;
    a.blk_cnt = p.blk_cnt;
    a.err = p.err;
    a.ids_out = p.ids_out;
    a.w_out = p.w_out;
    a.trace = p.trace;
    const int G = decode_grid();
    a.lay = decode_layout(G, p.D, p.F, p.E, p.K, p.dtype);
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
