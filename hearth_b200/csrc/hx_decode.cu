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
constexpr int DEC_MAXQ = 24;       // chunks per CTA
constexpr int BAR_DOWN = 28, BAR_ROUTER = 29;
// Phase stamps of the optional timeline (thread 0 of every CTA, per layer).
enum : int { ST_START, ST_NORM, ST_ROUTER, ST_BAR1, ST_ROUTE, ST_GATEUP, ST_MID, ST_BAR2, ST_DOWN, ST_SUM, ST_BAR3,
             DEC_STAMPS };

// Shared-memory carve-up of one CTA (identical on host and device).
struct DecodeLayout {
    int G, R, rpc, ppc;                // CTAs, down rows / CTA, router rows / CTA, gate/up pairs / CTA
    int nbD, nbF;
    int64_t rbD, rbF;
    size_t off_hs, off_xs, off_norm, off_rrow, off_stab, off_xact, off_gu, off_dn, off_amid, off_y, off_p, off_gout,
        off_score, off_ids, off_w, off_done, total;
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
    L.ppc = (K * F + G - 1) / G;
    size_t o = 512;   // mbarriers
    L.off_hs = o; o = align16(o + (size_t)D * 4);
    L.off_xs = o; o = align16(o + (size_t)D * 4);
    L.off_norm = o; o = align16(o + (size_t)D * 4);
    L.off_rrow = o; o = align16(o + (size_t)L.rpc * D * 4);
    L.off_stab = o; o = align16(o + (size_t)E * 8);
    L.off_xact = o; o = align16(o + (size_t)L.nbD * ACT_BLOCK);
    L.off_gu = o; o = align16(o + (size_t)(L.ppc + 1) * 2 * L.rbD);
    L.off_dn = o; o = align16(o + (size_t)K * L.R * L.rbF);
    L.off_amid = o; o = align16(o + (size_t)K * L.nbF * ACT_BLOCK);
    L.off_y = o; o = align16(o + (size_t)K * L.R * 4);
    L.off_p = o; o = align16(o + (size_t)DEC_WARPS * DEC_PROWS * 33 * 4);
    L.off_gout = o; o = align16(o + (size_t)DEC_WARPS * DEC_PROWS * 4);
    L.off_score = o; o = align16(o + (size_t)3 * E * 4 + 16 + (size_t)E * 8 + 64 * 4 + 16 + 64 * 4);
    L.off_ids = o; o = align16(o + (size_t)K * 4);
    L.off_w = o; o = align16(o + (size_t)K * 4);
    L.off_done = o; o = align16(o + (size_t)(2 * 32 + 1) * 4);
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
    unsigned *bar;                // grid barrier word
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

// Sense-reversing grid barrier: CTA 0 adds 2^31 - (G - 1), every other CTA adds 1, so the top bit
// of the word flips exactly when all G CTAs have arrived and the low bits return to their value.
__device__ __forceinline__ void grid_sync(unsigned *bar, int *err) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned inc = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1) : 1u;
        __threadfence();
        const unsigned old = atom_add_release(bar, inc);
        uint32_t spins = 0;
        while (((ld_acquire(bar) ^ old) & 0x80000000u) == 0) {
            // give up on the limit, or at once when another wait of this launch already gave up
            if (++spins > kBarrierSpinLimit || ((spins & 1023u) == 0 && *(volatile int *)err)) {
                set_error(err, DEV_E_BARRIER);
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

// The CTA's gate/up pairs: pair p in [0, K*F) is (rank j = p / F, row r = p % F); CTA c owns
// [c * K*F / G, (c+1) * K*F / G), cut into chunks of at most DEC_CH pairs that stay in one expert.
struct Chunk {
    int j, r0, n, pbase;   // expert rank, first row, pairs, index of its first pair within the CTA
};

__device__ __forceinline__ int cta_chunks(int c, int G, int K, int F, Chunk *out) {
    const int64_t P = (int64_t)K * F;
    const int p0 = (int)(P * c / G), p1 = (int)(P * (c + 1) / G);
    int n = 0;
    for (int p = p0; p < p1 && n < DEC_MAXQ;) {
        const int j = p / F, r = p - j * F;
        const int len = min(min(DEC_CH, F - r), p1 - p);
        out[n].j = j;
        out[n].r0 = r;
        out[n].n = len;
        out[n].pbase = p - p0;
        n++;
        p += len;
    }
    return n;
}

template <int DT>
__device__ void decode_body(const DecodeArgs &a, uint8_t *smem) {
    const DecodeLayout &ly = a.lay;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, G = gridDim.x;
    const int D = a.D, F = a.F, E = a.E, K = a.K;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    float *hs = reinterpret_cast<float *>(smem + ly.off_hs);
    float *xs = reinterpret_cast<float *>(smem + ly.off_xs);
    float *normv = reinterpret_cast<float *>(smem + ly.off_norm);
    float *rrow = reinterpret_cast<float *>(smem + ly.off_rrow);
    const uint8_t **stab = reinterpret_cast<const uint8_t **>(smem + ly.off_stab);   // this layer's slabs
    act_q8 *xact = reinterpret_cast<act_q8 *>(smem + ly.off_xact);
    uint8_t *gu = smem + ly.off_gu;
    uint8_t *dn = smem + ly.off_dn;
    act_q8 *amid = reinterpret_cast<act_q8 *>(smem + ly.off_amid);
    float *Y = reinterpret_cast<float *>(smem + ly.off_y);
    float *P = reinterpret_cast<float *>(smem + ly.off_p) + warp * DEC_PROWS * 33;
    float *gout = reinterpret_cast<float *>(smem + ly.off_gout) + warp * DEC_PROWS;
    float *score = reinterpret_cast<float *>(smem + ly.off_score), *sel = score + E, *lgs = sel + E;
    unsigned long long *rkey = reinterpret_cast<unsigned long long *>(
        smem + align16(ly.off_score + (size_t)3 * E * 4));
    float *gscr = reinterpret_cast<float *>(rkey + E), *red = gscr + 64;
    int *gkeep = reinterpret_cast<int *>(red + 4);
    int *ids = reinterpret_cast<int *>(smem + ly.off_ids);
    float *wts = reinterpret_cast<float *>(smem + ly.off_w);
    int *done = reinterpret_cast<int *>(smem + ly.off_done);   // [0] count, then (j, b) pairs
    __shared__ float rms_r;

    Chunk ch[DEC_MAXQ];
    const int nq = cta_chunks(c, G, K, F, ch);
    const int d0 = c * ly.R, d1 = min(D, d0 + ly.R), nrow = max(0, d1 - d0);
    const int pfirst = (int)((int64_t)K * F * c / G), plast = (int)((int64_t)K * F * (c + 1) / G);

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
        bulk_g2s(normv, a.norm[l], (uint32_t)D * 4, &bars[BAR_ROUTER]);
        bulk_g2s(stab, a.slab + (size_t)l * E, (uint32_t)E * 8, &bars[BAR_ROUTER]);
        for (int t = 0; t < ly.rpc; t++)
            if (c + t * G < E)
                bulk_g2s(rrow + (size_t)t * D, a.router[l] + (size_t)(c + t * G) * D, (uint32_t)D * 4,
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
            for (int i = tid; i < D; i += DEC_THREADS) xs[i] = __fmul_rn(__fmul_rn(hs[i], r), normv[i]);
        }
        __syncthreads();
        for (int b = warp; b < ly.nbD; b += DEC_WARPS) act_quant_warp(xs[b * QK + lane], xs[b * QK + lane + 32], xact + b, lane);
        {   // router rows: one 16-lane group each (warp-uniform tree; idle groups add zeros)
            const int t = tid >> 4, j = tid & 15;
            const bool active = t < ly.rpc && c + t * G < E;
            float L = 0.0f;
            if (active) {
                const float *w = rrow + (size_t)t * D;
#pragma unroll 8
                for (int i = j; i < D; i += 16) L = __fadd_rn(L, __fmul_rn(w[i], xs[i]));
            }
            if (warp < (ly.rpc + 1) / 2) {
                L = tree16(L, 0xffffffffu);
                if (active && j == 0) a.logits[c + t * G] = canon(L);
            }
        }
        HX_STAMP(ST_ROUTER);
        grid_sync(a.bar, a.err);
        HX_STAMP(ST_BAR1);

        // ---------------- phase B: routing, expert rows in flight, gate/up + SwiGLU + mid blocks
        route_token_cta(a.route, a.logits, a.bias[l], lgs, rkey, score, sel, gscr, gkeep, red, ids, wts);
        HX_STAMP(ST_ROUTE);
        if (warp == 0) {   // issue every copy of this layer from the 32 lanes (slab pointers in smem)
            fence_proxy_async();
            for (int q = lane; q < nq; q += 32) {   // gate/up chunks, one barrier each
                const uint8_t *slab = stab[ids[ch[q].j]];
                const uint32_t bytes = (uint32_t)(ch[q].n * ly.rbD);
                uint8_t *dst = gu + (size_t)ch[q].pbase * 2 * ly.rbD;
                if (!slab) {
                    set_error(a.err, DEV_E_NOT_RESIDENT);
                    mbar_expect_tx(&bars[q], 0);
                    continue;
                }
                mbar_expect_tx(&bars[q], 2 * bytes);
                bulk_g2s(dst, slab + (int64_t)ch[q].r0 * ly.rbD, bytes, &bars[q]);
                bulk_g2s(dst + bytes, slab + a.off_up + (int64_t)ch[q].r0 * ly.rbD, bytes, &bars[q]);
            }
            if (nrow > 0) {   // down rows [d0, d1) of the K experts on one barrier
                const bool have = lane < K && stab[ids[lane]] != nullptr;
                if (lane < K && !have) set_error(a.err, DEV_E_NOT_RESIDENT);
                const unsigned nhave = __popc(__ballot_sync(0xffffffffu, have));
                if (lane == 0) mbar_expect_tx(&bars[BAR_DOWN], nhave * (uint32_t)(nrow * ly.rbF));
                __syncwarp();
                if (have)
                    bulk_g2s(dn + (size_t)lane * ly.R * ly.rbF, stab[ids[lane]] + a.off_down + (int64_t)d0 * ly.rbF,
                             (uint32_t)(nrow * ly.rbF), &bars[BAR_DOWN]);
            }
            __syncwarp();
        }
        __syncthreads();   // every lane has read stab: the next layer's pointers may land there
        if (tid == 0) {
            fence_proxy_async();
            if (l + 1 < a.Lyr) issue_router(l + 1);
        }
        for (int q = warp; q < nq; q += DEC_WARPS) {
            if (!mbar_wait(&bars[q], par, a.err)) continue;
            const Chunk &k = ch[q];
            warp_rows_1tok<DT>(gu + (size_t)k.pbase * 2 * ly.rbD, ly.rbD, ly.nbD, 2 * k.n, xact, P, gout);
            if (lane < k.n) {
                const float m = swiglu_c(gout[lane], gout[k.n + lane]);
                __stcg(a.mbuf + (size_t)k.j * F + k.r0 + lane, m);
            }
            __syncwarp();
        }
        __threadfence();
        __syncthreads();
        HX_STAMP(ST_GATEUP);
        if (warp == 0) {   // arrivals per 64-row mid block; the CTA that completes a block quantizes it
            // the CTA's pair range [pfirst, plast) touches at most 32 blocks: lane i takes the i-th
            const int j0 = pfirst / F, b0 = (pfirst - j0 * F) / QK;
            const int gb = j0 * ly.nbF + b0 + lane;   // global block index = j * nbF + b
            const int j = gb / ly.nbF, b = gb - j * ly.nbF;
            const int bs = j * F + b * QK, be = bs + QK;
            const int lo = max(bs, pfirst), hi = min(be, plast);
            bool fin = false;
            if (lo < hi) {
                const unsigned cnt = (unsigned)(hi - lo);
                unsigned *ctr = a.blk_cnt + ((size_t)l * K + j) * ly.nbF + b;
                fin = atomicAdd(ctr, cnt) + cnt == (unsigned)QK;
            }
            const unsigned m = __ballot_sync(0xffffffffu, fin);
            if (fin) {
                const int slot = __popc(m & ((1u << lane) - 1u));
                done[1 + 2 * slot] = j;
                done[2 + 2 * slot] = b;
            }
            if (lane == 0) done[0] = __popc(m);
            __threadfence();
        }
        __syncthreads();
        for (int i = warp; i < done[0]; i += DEC_WARPS) {
            const int j = done[1 + 2 * i], b = done[2 + 2 * i];
            const float *m = a.mbuf + (size_t)j * F + (size_t)b * QK;
            act_quant_warp(__ldcg(m + lane), __ldcg(m + lane + 32), a.act_mid + (size_t)j * ly.nbF + b, lane);
        }
        HX_STAMP(ST_MID);
        grid_sync(a.bar, a.err);
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
        grid_sync(a.bar, a.err);
        HX_STAMP(ST_BAR3);
#undef HX_STAMP
    }
    // every bulk copy this CTA issued has landed before it exits (already true unless a wait gave up)
    if (tid == 0 && a.Lyr > 0) {
        const uint32_t last = (uint32_t)((a.Lyr - 1) & 1);
        for (int q = 0; q < nq; q++) mbar_wait(&bars[q], last, nullptr);
        if (nrow > 0) mbar_wait(&bars[BAR_DOWN], last, nullptr);
        mbar_wait(&bars[BAR_ROUTER], last, nullptr);
    }
    __syncthreads();
    // leave the arrival counters at zero for the next launch
    const int ncnt = a.Lyr * K * ly.nbF;
    for (int i = c * DEC_THREADS + tid; i < ncnt; i += G * DEC_THREADS) a.blk_cnt[i] = 0u;
}

__global__ void __launch_bounds__(DEC_THREADS, 1) k_moe_decode(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    if (a.dtype == Q4) decode_body<Q4>(a, smem);
    else decode_body<Q8>(a, smem);
}

// ------------------------------------------------------------------------------------- host side

int decode_stamps() { return DEC_STAMPS; }

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
    if (ly.R > 16) return no("down rows per CTA > 16");
    if (((int64_t)K * F + G - 1) / G > DEC_CH * (DEC_MAXQ - 2)) return no("gate/up pairs per CTA");
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
