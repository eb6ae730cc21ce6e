// hx_prefill_tc.cu — expert gate/up and down on the 5th-generation tensor cores (tcgen05) for
// prefill, speculative verification and batched decode (more than 64 token-expert pairs).
//
// NUMERICS §3 fixes each output as acc = ((0 + t_0) + t_1) + ... over the 64-weight blocks g of the
// row, t_g = (float)isum_g * (dw_g * dx_g), where isum_g is the exact int32 dot of the block. The
// tensor cores produce the isum_g of a whole tile of 128 rows x 32 token pairs (`tcgen05.mma
// .kind::i8`, K = 32 bytes per instruction, a fresh accumulation per block in tensor memory); the
// CUDA cores read the tile back (`tcgen05.ld`) and run every row's float chain in block order. Q4
// weights enter as unsigned nibbles (u8 x s8) and sum((nib-8)*xq) = sum(nib*xq) - 8*sum(xq) removes
// the offset exactly; Q8 weights enter as s8. Operands in shared memory use the K-major, unswizzled
// core-matrix layout of the UMMA descriptors (8 rows x 16 bytes per core matrix, K-chunks 128 bytes
// apart, 8-row groups 512 bytes apart).
//
// Two implementations:
//   * staged (k_moe_gateup_ws / k_moe_down_ws, Q4 experts, D a multiple of 512, down rows of 4, 8 or
//     12 blocks): persistent CTAs with warp roles, tensor-map loads into a stage ring, operand A in
//     tensor memory, the offset and the int -> float conversion folded into the accumulator (see the
//     section comment below);
//   * register-fed (k_moe_gateup_tc / k_moe_down_tc, every other shape, Q8 experts included): one
//     CTA per (row tile, job, pair tile), each thread loading its row's next block into registers
//     while the current block is multiplied.
// Gate/up tiles end with SwiGLU and the mid activation blocks (NUMERICS §2, one per 64 rows); down
// tiles write the canonical outputs into Y (routed) or S (shared) for the rank-order sum.
#include "hx_device.cuh"
#include "hx_kernels.h"
#include "hx_route.cuh"
#include "hx_moe_job.cuh"

#include <algorithm>
#include <cuda.h>

namespace hx {

namespace {

constexpr int TC_M = 128;   // rows per CTA (lanes of tensor memory)
constexpr int TC_N = 32;    // token pairs per CTA (tensor-memory columns per accumulator)
constexpr int TC_THREADS = 128;

__device__ __forceinline__ int op_off(int r, int chunk) { return (r >> 3) * 512 + chunk * 128 + (r & 7) * 16; }

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    // start address, LBO 128 B, SBO 512 B (16-byte units), descriptor version 1, no swizzle
    return (uint64_t)((saddr >> 4) & 0x3fff) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) |
           (1ull << 46);
}

// .kind::i8 instruction descriptor: D s32, A u8 or s8, B s8, both K-major, N = TC_N, M = TC_M.
__device__ __forceinline__ uint32_t umma_idesc_i8(bool a_signed) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | (1u << 10) | ((uint32_t)(TC_N >> 3) << 17) |
           ((uint32_t)(TC_M >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate ? 1u : 0u));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t v[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Tensor-memory allocation of one CTA (warp 0 allocates and frees).
__device__ __forceinline__ uint32_t tmem_alloc(uint32_t *slot, uint32_t ncols) {
    if ((threadIdx.x >> 5) == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    return *slot;
}

__device__ __forceinline__ void tmem_free(uint32_t tmem, uint32_t ncols) {
    tc_fence_before();
    __syncthreads();
    if ((threadIdx.x >> 5) == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
}

// One weight block of one row in registers: the 64 values as 16 words in MMA K order (Q4: unsigned
// nibbles, elements 0..31 then 32..63; Q8: signed bytes) and the f16 scale bits.
template <int DT>
struct WBlock {
    uint32_t w[16];
    uint32_t sc;
};

template <int DT>
__device__ __forceinline__ void load_wblock(const uint8_t *blk, bool valid, WBlock<DT> &b) {
    if (!valid) {
#pragma unroll
        for (int i = 0; i < 16; i++) b.w[i] = 0;
        b.sc = 0;
        return;
    }
    if constexpr (DT == Q4) {
        uint32_t nib[8];
        b.sc = load_q4_block(blk, nib);   // exact-bound loads (global memory)
#pragma unroll
        for (int i = 0; i < 8; i++) {
            b.w[i] = nib[i] & 0x0f0f0f0fu;
            b.w[8 + i] = (nib[i] >> 4) & 0x0f0f0f0fu;
        }
    } else {
        b.sc = load_q8_block(blk, b.w);
    }
}

__device__ __forceinline__ void store_operand_row(uint8_t *op, int r, const uint32_t w[16]) {
#pragma unroll
    for (int c = 0; c < 4; c++)
        *reinterpret_cast<uint4 *>(op + op_off(r, c)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// Activation operand of one block: thread t moves 16 of the 64 q bytes of pair t/4 (zeros past nn);
// threads with t%4 == 0 also keep the pair's d and sum.
struct ABlock {
    uint2 q0, q1;
    float d;
    int sum;
};

__device__ __forceinline__ void load_ablock(const act_q8 *a, bool valid, int quarter, ABlock &b) {
    if (!valid) {
        b.q0 = b.q1 = make_uint2(0, 0);
        b.d = 0.0f;
        b.sum = 0;
        return;
    }
    const uint2 *p = reinterpret_cast<const uint2 *>(a);   // 72-byte blocks are 8-byte aligned
    const uint2 h = p[0];
    b.d = __uint_as_float(h.x);
    b.sum = (int)h.y;
    b.q0 = p[1 + 2 * quarter];
    b.q1 = p[2 + 2 * quarter];
}

// Shared memory of one CTA.
struct TcSmem {
    uint8_t a0[TC_M * 64];   // operand A (gate, or down)
    uint8_t a1[TC_M * 64];   // operand A (up)
    uint8_t b[TC_N * 64];    // operand B (activations)
    float dx[TC_N];
    int asum[TC_N];
    float red[4][TC_N];      // epilogue reductions
    int ired[4][TC_N];
    uint64_t bar;
    uint32_t tmem;
};

// Drains one accumulator (TC_N columns at tcol) into the row's float chains.
template <int DT>
__device__ __forceinline__ void drain(uint32_t tmem, int tcol, float dw, const TcSmem &s, float acc[TC_N]) {
    uint32_t v[32];
    const uint32_t taddr = tmem + ((uint32_t)((threadIdx.x >> 5) * 32) << 16) + (uint32_t)tcol;
    tmem_ld32(taddr, v);
#pragma unroll
    for (int n = 0; n < TC_N; n++) {
        const int isum = DT == Q4 ? (int)v[n] - 8 * s.asum[n] : (int)v[n];
        acc[n] = __fadd_rn(acc[n], __fmul_rn(__int2float_rn(isum), __fmul_rn(dw, s.dx[n])));
    }
}

// NUMERICS §2 quantization of pair n's 64 values held by 64 threads (rows blk*64 .. +63, one per
// thread of warps 2*blk and 2*blk+1): the same amax, d, q and sum as act_quant_warp on one warp. The
// block of pair n goes to mid[(p + n) * fmax_nb + b0 + blk].
__device__ __forceinline__ void quant_epilogue(const float m[TC_N], bool rowvalid, TcSmem &s, act_q8 *mid,
                                               int64_t p, int fmax_nb, int b0, int nn) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, blk = warp >> 1;
    for (int n = 0; n < TC_N; n++) {
        float amax = rowvalid && n < nn ? fabsf(m[n]) : 0.0f;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0) s.red[warp][n] = amax;
    }
    __syncthreads();
    for (int n = 0; n < TC_N; n++) {
        const float amax = fmaxf(fmaxf(s.red[2 * blk][n], s.red[2 * blk + 1][n]), 0.0f);
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        float v = __fmul_rn(m[n], id);
        if (v != v) v = 0.0f;
        v = v > 127.0f ? 127.0f : (v < -127.0f ? -127.0f : v);
        const bool live = rowvalid && n < nn;
        const int q = live ? __float2int_rn(v) : 0;
        int sum = q;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) s.ired[warp][n] = sum;
        if (live) {
            act_q8 *o = mid + (p + n) * fmax_nb + b0 + blk;
            o->q[tid - blk * 64] = (int8_t)q;
            if ((tid & 63) == 0) o->d = d;
        }
    }
    __syncthreads();
    if ((tid & 63) == 0 && rowvalid)
        for (int n = 0; n < nn; n++) (mid + (p + n) * fmax_nb + b0 + blk)->sum = s.ired[2 * blk][n] + s.ired[2 * blk + 1][n];
}

template <int DT>
__device__ void gateup_tc_body(const MoeShape &sh, const MoeScratch &sc, const Job &job, int rt, int n0, int fmax_nb,
                               TcSmem &s) {
    const int tid = threadIdx.x, nbD = sh.D / QK;
    const int nn = min(TC_N, job.n - n0);
    const int64_t rbD = row_bytes(DT, sh.D);
    const int row = rt * TC_M + tid;
    const bool rowvalid = row < job.F;
    const uint8_t *grow = job.gate + (int64_t)row * rbD, *urow = job.up + (int64_t)row * rbD;
    constexpr int BS = DT == Q4 ? Q4_BLOCK : Q8_BLOCK;
    // the activation quarter this thread moves each block
    const int an = tid >> 2, aq = tid & 3;
    const bool avalid = an < nn;
    const act_q8 *arow = avalid ? sc.xact + (int64_t)job_token(sc, job, n0 + an) * nbD : nullptr;

    if (tid == 0) {
        mbar_init(&s.bar, 1);
        fence_mbar_init();
    }
    const uint32_t tmem = tmem_alloc(&s.tmem, 2 * TC_N);
    const uint32_t idesc = umma_idesc_i8(DT == Q8);
    float accG[TC_N], accU[TC_N];
#pragma unroll
    for (int n = 0; n < TC_N; n++) accG[n] = accU[n] = 0.0f;

    WBlock<DT> gn, un;
    ABlock an_;
    load_wblock<DT>(grow, rowvalid, gn);
    load_wblock<DT>(urow, rowvalid, un);
    load_ablock(avalid ? arow : nullptr, avalid, aq, an_);
    for (int g = 0; g < nbD; g++) {
        const WBlock<DT> gc = gn, uc = un;
        const ABlock ac = an_;
        if (g + 1 < nbD) {   // next block's loads in flight while this one is multiplied
            load_wblock<DT>(grow + (int64_t)(g + 1) * BS, rowvalid, gn);
            load_wblock<DT>(urow + (int64_t)(g + 1) * BS, rowvalid, un);
            load_ablock(avalid ? arow + g + 1 : nullptr, avalid, aq, an_);
        }
        store_operand_row(s.a0, tid, gc.w);
        store_operand_row(s.a1, tid, uc.w);
        *reinterpret_cast<uint4 *>(s.b + op_off(an, aq)) = make_uint4(ac.q0.x, ac.q0.y, ac.q1.x, ac.q1.y);
        if (aq == 0) {
            s.dx[an] = ac.d;
            s.asum[an] = ac.sum;
        }
        fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            const uint32_t sa0 = smem_u32(s.a0), sa1 = smem_u32(s.a1), sb = smem_u32(s.b);
            for (int k = 0; k < 2; k++) {
                umma_i8(tmem, umma_desc(sa0 + 256 * k), umma_desc(sb + 256 * k), idesc, k > 0);
                umma_i8(tmem + TC_N, umma_desc(sa1 + 256 * k), umma_desc(sb + 256 * k), idesc, k > 0);
            }
            umma_commit(&s.bar);
        }
        mbar_wait(&s.bar, (uint32_t)(g & 1), sc.err);
        tc_fence_after();
        drain<DT>(tmem, 0, f16_to_f32(gc.sc), s, accG);
        drain<DT>(tmem, TC_N, f16_to_f32(uc.sc), s, accU);
        tc_fence_before();
        __syncthreads();   // operands and tensor memory are reused by the next block
    }
    // SwiGLU and the mid activation blocks
    float m[TC_N];
#pragma unroll
    for (int n = 0; n < TC_N; n++) m[n] = swiglu_c(canon(accG[n]), canon(accU[n]));
    quant_epilogue(m, rowvalid, s, sc.act_mid, (int64_t)job.p0 + n0, fmax_nb, rt * 2, nn);
    tmem_free(tmem, 2 * TC_N);
}

template <int DT>
__device__ void down_tc_body(const MoeShape &sh, const MoeScratch &sc, const Job &job, int rt, int n0, int fmax_nb,
                             TcSmem &s) {
    const int tid = threadIdx.x;
    const int nn = min(TC_N, job.n - n0);
    const int nbF = job.nbF;
    const int64_t rbF = row_bytes(DT, job.F);
    const int row = rt * TC_M + tid;
    const bool rowvalid = row < sh.D;
    const uint8_t *drow = job.down + (int64_t)row * rbF;
    constexpr int BS = DT == Q4 ? Q4_BLOCK : Q8_BLOCK;
    const int an = tid >> 2, aq = tid & 3;
    const bool avalid = an < nn;
    const act_q8 *arow = avalid ? sc.act_mid + (int64_t)(job.p0 + n0 + an) * fmax_nb : nullptr;

    if (tid == 0) {
        mbar_init(&s.bar, 1);
        fence_mbar_init();
    }
    const uint32_t tmem = tmem_alloc(&s.tmem, TC_N);
    const uint32_t idesc = umma_idesc_i8(DT == Q8);
    float acc[TC_N];
#pragma unroll
    for (int n = 0; n < TC_N; n++) acc[n] = 0.0f;

    WBlock<DT> wn;
    ABlock an_;
    load_wblock<DT>(drow, rowvalid, wn);
    load_ablock(arow, avalid, aq, an_);
    for (int g = 0; g < nbF; g++) {
        const WBlock<DT> wc = wn;
        const ABlock ac = an_;
        if (g + 1 < nbF) {
            load_wblock<DT>(drow + (int64_t)(g + 1) * BS, rowvalid, wn);
            load_ablock(avalid ? arow + g + 1 : nullptr, avalid, aq, an_);
        }
        store_operand_row(s.a0, tid, wc.w);
        *reinterpret_cast<uint4 *>(s.b + op_off(an, aq)) = make_uint4(ac.q0.x, ac.q0.y, ac.q1.x, ac.q1.y);
        if (aq == 0) {
            s.dx[an] = ac.d;
            s.asum[an] = ac.sum;
        }
        fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            const uint32_t sa = smem_u32(s.a0), sb = smem_u32(s.b);
            for (int k = 0; k < 2; k++) umma_i8(tmem, umma_desc(sa + 256 * k), umma_desc(sb + 256 * k), idesc, k > 0);
            umma_commit(&s.bar);
        }
        mbar_wait(&s.bar, (uint32_t)(g & 1), sc.err);
        tc_fence_after();
        drain<DT>(tmem, 0, f16_to_f32(wc.sc), s, acc);
        tc_fence_before();
        __syncthreads();
    }
    if (rowvalid) {   // canonical outputs: Y [pair][D] (routed) or S [token][D] (shared)
        for (int n = 0; n < nn; n++) {
            float *out = job.shared ? sc.S + (int64_t)(n0 + n) * sh.D : sc.Y + (int64_t)(job.p0 + n0 + n) * sh.D;
            out[row] = canon(acc[n]);
        }
    }
    tmem_free(tmem, TC_N);
}

// =============================================================================================
// Staged persistent path (Q4 experts). One CTA per SM walks a static list of tiles; the weight rows
// and activation rows of each tile reach shared memory through tensor-map loads (one box of 128 rows
// per matrix and stage, gather4 boxes of four token rows, one box of 32 mid rows for down) into a
// two-slot ring that runs ahead across tiles, so that up to two stages (~176 KB) per SM are in
// flight while the CTA unpacks, multiplies and drains. Unpacking reads shared memory with 16- or
// 8-byte loads laid out to avoid bank conflicts; the row loads of the register path above touch one
// 32-byte sector per thread and instruction, which keeps the load/store unit, not HBM, busy.
//
// Tiles: job u (routed bucket or the shared expert) owns ceil(n_u / 32) x (row tiles) tiles, in
// job order and, inside a job, pair tile major and row tile minor, so that consecutive tiles read
// the same activations. Tile t goes to CTA t % gridDim.x.
// =============================================================================================

constexpr int SG_BLK = 8;                        // gate/up: blocks per stage
constexpr int SG_SEG = SG_BLK * Q4_BLOCK;        // 272: one row's bytes per stage
constexpr int SG_ASEG = SG_BLK * ACT_BLOCK;      // 576: one pair's activation bytes per stage
constexpr int SG_MAXJOBS = 1024 + 1;             // routed buckets (E <= 1024) + the shared expert
constexpr int SD_MAXNB = 12;                     // down: whole rows of at most 12 blocks (F <= 768)

struct TileInfo {
    const uint8_t *w0, *w1;   // gate and up rows (gate/up), down rows (down); null: the job cannot run
    int rt, n0, nn, p0;       // row tile, first pair of the tile in the job, pairs, job's first pair
    int F, shared;            // job's expert width, shared-expert job
    int slot;                 // expert-store slot of a routed job
};

// Tiles per job and their exclusive prefix pre[0..njobs]; returns the number of tiles.
// down = false: row tiles over the job's F (gate/up); down = true: over D.
__device__ int tile_prefix(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, int nu, int njobs,
                           bool down, int *pre) {
    const int tid = threadIdx.x, lane = tid & 31;
    for (int u = tid; u < njobs; u += blockDim.x) {
        int n, F;
        if (u < nu) {
            n = sc.u_n[sh.ep_size > 1 ? sc.ujob[u] : u];
            F = sh.F;
        } else {
            n = sh.T;
            F = L.Fs;
        }
        const int nrt = down ? (sh.D + TC_M - 1) / TC_M : (F + TC_M - 1) / TC_M;
        pre[u + 1] = (n + TC_N - 1) / TC_N * nrt;
    }
    __syncthreads();
    if (tid < 32) {   // warp 0: lane scans a contiguous chunk, then a shuffle scan of the chunk sums
        const int chunk = (njobs + 31) / 32, a = lane * chunk, b = min(njobs, a + chunk);
        int s = 0;
        for (int u = a; u < b; u++) s += pre[u + 1];
        int incl = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - s;
        for (int u = a; u < b; u++) {
            const int c = pre[u + 1];
            pre[u + 1] = run + c;
            run += c;
        }
        if (lane == 0) pre[0] = 0;
    }
    __syncthreads();
    return pre[njobs];
}

// Tile t -> its job and place (one thread). A job that cannot run (expert not resident) gives a
// tile with no rows and no pairs: its stages copy nothing and its epilogue writes nothing.
__device__ void decode_tile(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, const TcMaps &mp, int nu,
                            int njobs, const int *pre, int t, bool down, TileInfo &ti) {
    int lo = 0, hi = njobs;   // largest u with pre[u] <= t
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (pre[mid] <= t) lo = mid;
        else hi = mid;
    }
    Job job;
    bool ok = get_job(sh, L, sc, lo, nu, job);
    ti.slot = 0;
    if (ok && !job.shared) {   // the tensor maps address routed experts by store slot
        const int64_t off = job.gate - mp.arena;
        ok = off >= 0 && off % mp.slot_bytes == 0 && off / mp.slot_bytes < mp.n_slots;
        if (ok) ti.slot = (int)(off / mp.slot_bytes);
        else set_error(sc.err, DEV_E_NOT_RESIDENT);
    }
    const int F = ok ? job.F : 0;
    const int nrt = down ? (sh.D + TC_M - 1) / TC_M : (F + TC_M - 1) / TC_M;
    const int l = t - pre[lo];
    ti.rt = nrt ? l % nrt : 0;
    ti.n0 = nrt ? l / nrt * TC_N : 0;
    ti.nn = ok ? min(TC_N, job.n - ti.n0) : 0;
    ti.p0 = ok ? job.p0 : 0;
    ti.F = F;
    ti.shared = ok && job.shared;
    ti.w0 = ok ? (down ? job.down : job.gate) : nullptr;
    ti.w1 = ok ? job.up : nullptr;
}

// Q4 block starting O bytes (even, < 16) into the words W: the scale bits, and the 64 values as
// unsigned nibbles in MMA K order (elements 0..31 from the low nibbles, 32..63 from the high ones).
template <int O>
__device__ __forceinline__ uint32_t q4_words(const uint32_t *W, uint32_t w[16]) {
    const uint32_t sc = (O & 2) ? (W[O / 4] >> 16) : (W[O / 4] & 0xffffu);
    constexpr int B0 = O + 2;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        uint32_t nib;
        if constexpr ((B0 & 2) != 0) nib = __funnelshift_r(W[B0 / 4 + i], W[B0 / 4 + i + 1], 16);
        else nib = W[B0 / 4 + i];
        w[i] = nib & 0x0f0f0f0fu;
        w[8 + i] = (nib >> 4) & 0x0f0f0f0fu;
    }
    return sc;
}

// Block J (0..7) of a 272-byte gate/up stage row (16-byte aligned): it starts 2J bytes into
// 16-byte chunk 2J, so three 16-byte loads cover it.
template <int J>
__device__ __forceinline__ uint32_t seg_q4_block(const uint8_t *seg, uint32_t w[16]) {
    const uint4 *p = reinterpret_cast<const uint4 *>(seg) + 2 * J;
    const uint4 a = p[0], b = p[1], c = p[2];
    const uint32_t W[12] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w};
    return q4_words<2 * J>(W, w);
}

// Block j (j % 4 == JM) of a whole down row in shared memory (8-byte aligned): it starts
// 2 * JM bytes into 8-byte word 4j + j / 4, so five 8-byte loads cover it.
template <int JM>
__device__ __forceinline__ uint32_t row_q4_block(const uint8_t *row, int j, uint32_t w[16]) {
    const uint2 *p = reinterpret_cast<const uint2 *>(row) + 4 * j + (j >> 2);
    uint32_t W[10];
#pragma unroll
    for (int i = 0; i < 5; i++) {
        const uint2 v = p[i];
        W[2 * i] = v.x;
        W[2 * i + 1] = v.y;
    }
    return q4_words<2 * JM>(W, w);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t v[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Tensor-map loads into this CTA's own shared memory, completion counted on bar. The box
// origin's x times the element size is a multiple of 16 bytes for every call below.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const void *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Four rows r0..r3 (box one row high) of a 2-D map, stored one after another.
__device__ __forceinline__ void tma_gather4(void *dst, const void *map, int x, int r0, int r1, int r2, int r3,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------------------------------------
// Warp roles of the staged kernels (832 threads, one CTA per SM; many light warps per role, so that
// each scheduler always has a warp of every role ready while others wait on tensor memory or
// shared memory):
//   warps 0-15   drain: read a block's int32 tile from tensor memory and extend the float chains
//   warps 16-23  unpack: stage rows -> operand A in tensor memory (tcgen05.st), activations ->
//                operand B in shared memory, scales -> shared memory
//   warp 24      copies: decodes tiles and issues the tensor-map loads of the stage ring
//   warp 25      MMA: one thread issues each block's tcgen05.mma and commits
// Operands and accumulators rotate through WS_NBUF buffers by block; mbarriers hand each buffer from
// role to role, so unpacking, multiplication and draining of different blocks overlap.
//
// Two exact identities keep the tensor cores to the plain dots and the drain short. The accumulator
// starts at the bit pattern of 1.5 * 2^23 (0x4B400000); the u8 (nibble) x s8 dot X of a block
// changes only its low 23 mantissa bits (|X| <= 64 * 15 * 127 < 2^22), so the word read back, taken
// as a float, is exactly 12582912 + X. The unpackers store cm = 12582912 + 8 * sum(q) per pair (an
// integer below 2^24, exact in f32), and one subtraction gives the signed Q4 block dot
// isum = X - 8 * sum(q) exactly. The chain's multiplies run as packed f32x2 pairs (two IEEE
// round-to-nearest products per instruction); its adds stay scalar, in block order.
// ---------------------------------------------------------------------------------------------

constexpr int WS_THREADS = 832;
constexpr int WS_DRAIN = 512;                    // warps 0-15
constexpr int WS_UNPACK0 = 512, WS_UNPACK = 256; // warps 16-23
constexpr int WS_COPY_WARP = 24, WS_MMA_WARP = 25;
constexpr int WS_NBUF = 4;                       // blocks in flight between the roles
constexpr uint32_t kMagic = 0x4B400000u;         // bit pattern of 1.5 * 2^23
constexpr int kMagicI = 12582912;                // 1.5 * 2^23
static_assert(WS_THREADS == (WS_MMA_WARP + 1) * 32 && WS_COPY_WARP * 32 == WS_UNPACK0 + WS_UNPACK,
              "warp roles: drain, unpack, copy, MMA");

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One arrival for the whole warp, after every lane's preceding work (its fences included).
__device__ __forceinline__ void warp_arrive(uint64_t *bar) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// Load without the wait: the registers are valid after tmem_wait_ld().
__device__ __forceinline__ void tmem_ld8_async(uint32_t taddr, uint32_t v[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_fill8(uint32_t taddr, uint32_t x) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(x) : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t v[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// The same word into 16 consecutive columns of this warp's lanes.
__device__ __forceinline__ void tmem_fill16(uint32_t taddr, uint32_t x) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
        "r"(x)
        : "memory");
}

// D[tmem] += A[tmem] x B[smem] (kind::i8, A from tensor memory).
__device__ __forceinline__ void umma_i8_ts(uint32_t d, uint32_t a, uint64_t db, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 1, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(db), "r"(idesc));
}

__device__ __forceinline__ uint64_t pack2(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }
__device__ __forceinline__ uint64_t pack2f(float lo, float hi) { return pack2(__float_as_uint(lo), __float_as_uint(hi)); }

__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float lo_f(uint64_t x) { return __uint_as_float((uint32_t)x); }
__device__ __forceinline__ float hi_f(uint64_t x) { return __uint_as_float((uint32_t)(x >> 32)); }

// Per-block pair constants in shared memory, interleaved for the drain: entry i holds
// {cm[2i], cm[2i+1], dx[2i], dx[2i+1]}.
struct PairConst {
    float4 v[TC_N / 2];
};

// NC columns of block words v (magic-offset u8 x s8 dots) into the packed chains acc2[NC / 2]:
// acc = acc + isum * (dw * dx[n]), every operation a packed f32x2 pair rounded to nearest. The product
// term comes from fma(isum, dw * dx, z) with z a zero the compiler cannot see (a kernel argument):
// exactly the rounded product (the chains start at +0, so the sign of a zero product cannot
// matter), and, unlike a multiply, it is never contracted into the following add (a packed multiply
// feeding a packed add is contracted into a fused multiply-add even when both carry .rn).
template <int NC>
__device__ __forceinline__ void chain_f2(const uint32_t *v, float dw, const float4 *pc, uint64_t *acc2, float zero) {
    const uint64_t dw2 = pack2f(dw, dw), z2 = pack2f(zero, zero);
#pragma unroll
    for (int i = 0; i < NC / 2; i++) {
        const float4 q = pc[i];
        const uint64_t isum2 = f2_sub(pack2(v[2 * i], v[2 * i + 1]), pack2f(q.x, q.y));
        acc2[i] = f2_add(acc2[i], f2_fma(isum2, f2_mul(dw2, pack2f(q.z, q.w)), z2));
    }
}

// Activation operand of block J for the 32 pairs of a stage (pair rows `pitch` bytes apart, 16-byte
// aligned): 128 threads (u = 0..127) move one 16-byte chunk each; pairs past nn get zeros, and the
// thread holding chunk 0 of a pair also stores the pair's dx and cm. Thread u = 8k + i takes pair
// 8 (k & 3) + i and chunk ((i >> CSH) + (k >> 2)) & 3: the eight threads of a shared-memory phase
// write eight different operand rows, and read eight different 16-byte bank groups when the pitch
// in 16-byte units is 4 mod 8 (CSH = 1) or 2 or 6 mod 8 (CSH = 2).
template <int JP, int CSH>   // JP = J & 1: block J's quantized bytes start 16-byte aligned when J is odd
__device__ __forceinline__ void unpack_act_ws(const uint8_t *act, int pitch, int j, int nn, uint8_t *bop,
                                              PairConst &pc, int u) {
    const int k = u >> 3, i = u & 7;
    const int n = 8 * (k & 3) + i, c = ((i >> CSH) + (k >> 2)) & 3;
    const bool live = n < nn;
    const uint8_t *blk = act + n * pitch + j * ACT_BLOCK;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (live) {
        if constexpr (JP == 1) {
            v = *reinterpret_cast<const uint4 *>(blk + 8 + 16 * c);
        } else {
            const uint2 a = *reinterpret_cast<const uint2 *>(blk + 8 + 16 * c);
            const uint2 b = *reinterpret_cast<const uint2 *>(blk + 16 + 16 * c);
            v = make_uint4(a.x, a.y, b.x, b.y);
        }
    }
    *reinterpret_cast<uint4 *>(bop + op_off(n, c)) = v;
    if (c == 0) {
        const uint2 hd = live ? *reinterpret_cast<const uint2 *>(blk) : make_uint2(0, 0);
        float *e = reinterpret_cast<float *>(&pc.v[n >> 1]) + (n & 1);
        e[0] = __int2float_rn(kMagicI + 8 * (int)hd.y);   // cm: exact (below 2^24)
        e[2] = __uint_as_float(hd.x);                        // dx
    }
}

// The same operand as unpack_act_ws with two threads per chunk: thread (u, hm) moves bytes
// 8 hm .. 8 hm + 7 of chunk u's 16 (both reads and writes 8 bytes); hm == 0 also stores dx and cm.
template <int CSH>
__device__ __forceinline__ void unpack_act_half(const uint8_t *act, int pitch, int j, int nn, uint8_t *bop,
                                                PairConst &pc, int u, int hm) {
    const int k = u >> 3, i = u & 7;
    const int n = 8 * (k & 3) + i, c = ((i >> CSH) + (k >> 2)) & 3;
    const bool live = n < nn;
    const uint8_t *blk = act + n * pitch + j * ACT_BLOCK;
    const uint2 v = live ? *reinterpret_cast<const uint2 *>(blk + 8 + 16 * c + 8 * hm) : make_uint2(0, 0);
    *reinterpret_cast<uint2 *>(bop + op_off(n, c) + 8 * hm) = v;
    if (c == 0 && hm == 0) {
        const uint2 hd = live ? *reinterpret_cast<const uint2 *>(blk) : make_uint2(0, 0);
        float *e = reinterpret_cast<float *>(&pc.v[n >> 1]) + (n & 1);
        e[0] = __int2float_rn(kMagicI + 8 * (int)hd.y);   // cm: exact (below 2^24)
        e[2] = __uint_as_float(hd.x);                        // dx
    }
}

// NUMERICS §2 quantization of the mid values of a tile held in X[pair][128 rows] (shared): unit
// (pair n, 64-row block b) is quantized by 8 consecutive lanes, 8 rows each (amax and the q sum by
// 3-step shuffles; the same d, q and sum as act_quant_warp). Called by the 512 drain threads.
__device__ __forceinline__ void quant_tile(const float *X, const TileInfo &ti, act_q8 *mid, int fmax_nb, int tid) {
    static_assert(WS_DRAIN == TC_N * TC_M / 8, "one (pair, 8-row group) item per drain thread");
    {
        const int item = tid;                           // 512 items: (pair, 8-row group)
        const int n = item >> 4, grp = item & 15, b = grp >> 3, l8 = grp & 7;
        const bool live = n < ti.nn && ti.rt * TC_M + b * 64 < ti.F;   // uniform over the 8 lanes
        const float4 x0 = *reinterpret_cast<const float4 *>(X + n * TC_M + grp * 8);
        const float4 x1 = *reinterpret_cast<const float4 *>(X + n * TC_M + grp * 8 + 4);
        const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        float amax = fabsf(x[0]);
#pragma unroll
        for (int i = 1; i < 8; i++) amax = fmaxf(amax, fabsf(x[i]));   // fmaxf drops NaN
#pragma unroll
        for (int o = 4; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        amax = fmaxf(amax, 0.0f);
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint32_t qw[2] = {0, 0};
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float v = __fmul_rn(x[i], id);
            if (v != v) v = 0.0f;
            v = v > 127.0f ? 127.0f : (v < -127.0f ? -127.0f : v);
            const int q = __float2int_rn(v);
            sum += q;
            qw[i >> 2] |= ((uint32_t)q & 0xffu) << (8 * (i & 3));
        }
#pragma unroll
        for (int o = 4; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (live) {
            act_q8 *o = mid + (int64_t)(ti.p0 + ti.n0 + n) * fmax_nb + ti.rt * 2 + b;
            *reinterpret_cast<uint2 *>(o->q + 8 * l8) = make_uint2(qw[0], qw[1]);
            if (l8 == 0) {
                o->d = d;
                o->sum = sum;
            }
        }
    }
}

__device__ __forceinline__ void drain_bar() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// Barriers and scratch shared by both staged kernels.
struct WsSync {
    uint64_t full[2], empty[2];                       // stage ring: copies landed / unpackers done
    uint64_t aready[WS_NBUF], accfull[WS_NBUF], accempty[WS_NBUF];
    uint32_t tmem;
};

__device__ __forceinline__ void ws_init(WsSync &y) {
    for (int b = 0; b < 2; b++) {
        mbar_init(&y.full[b], 1);
        mbar_init(&y.empty[b], WS_UNPACK / 32);   // one arrival per warp
    }
    for (int b = 0; b < WS_NBUF; b++) {
        mbar_init(&y.aready[b], WS_UNPACK / 32);
        mbar_init(&y.accfull[b], 1);
        mbar_init(&y.accempty[b], WS_DRAIN / 32);
    }
    fence_mbar_init();
}

// ------------------------------------------------------------------------------------ gate/up

struct GuStage {
    uint8_t w[2 * TC_M][SG_SEG];    // rows 0..127: gate, 128..255: up (one tensor-map box each)
    uint8_t act[TC_N][SG_ASEG];     // pair rows (gather4 boxes of four rows)
};

struct GuSmem {
    GuStage st[2];
    uint8_t b[WS_NBUF][TC_N * 64];  // operand B (activations) per block buffer
    PairConst pc[WS_NBUF];
    float dw[WS_NBUF][2 * TC_M];    // block scales of gate rows, then up rows
    float X[TC_N * TC_M];           // epilogue: SwiGLU exchange and the mid values
    TileInfo ti[3];
    int pre[SG_MAXJOBS + 1];
    WsSync y;
};
static_assert(sizeof(GuStage) % 128 == 0 && (TC_M * SG_SEG) % 128 == 0 && (4 * SG_ASEG) % 128 == 0,
              "tensor-map destinations stay 128-byte aligned");

// Tensor-memory columns (512 allocated): accumulators [b] at 64b (gate +0, up +32), operand A [b][m]
// at 256 + 32b + 16m.
constexpr uint32_t GU_ACC = 0, GU_A = 256, GU_TMEM_COLS = 512;

// Tensor-map loads of gate/up stage qs (tile qs / nS, blocks 8 (qs % nS) ..) into slot qs & 1, by
// the copy warp. The stage's tile description is decoded into the info ring at its first stage.
__device__ __forceinline__ void gu_issue_stage(GuSmem &s, const MoeShape &sh, const MoeLayerDev &L,
                                               const MoeScratch &sc, const TcMaps &mp, int nu, int njobs, int ntiles,
                                               int nS, int qs) {
    const int i = qs / nS, s0 = qs % nS, t = blockIdx.x + i * gridDim.x, lane = threadIdx.x & 31;
    if (t >= ntiles) return;
    TileInfo &ti = s.ti[i % 3];
    if (s0 == 0 && lane == 0) decode_tile(sh, L, sc, mp, nu, njobs, s.pre, t, false, ti);
    __syncwarp();
    const int nn = ti.nn, ng = (nn + 3) / 4, slot = qs & 1;
    const bool wok = ti.w0 != nullptr;
    int tok = 0;
    if (lane < nn) {
        Job j;
        j.shared = ti.shared;
        j.p0 = ti.p0;
        tok = job_token(sc, j, ti.n0 + lane);
    }
    const int tok0 = __shfl_sync(0xffffffffu, tok, 0);
    if (lane >= nn) tok = tok0;   // gather4 fills its four rows; rows past nn are not used
    int t4[4];
#pragma unroll
    for (int e = 0; e < 4; e++) t4[e] = __shfl_sync(0xffffffffu, tok, (4 * lane + e) & 31);
    uint64_t *bar = &s.y.full[slot];
    if (lane == 0) {
        mbar_expect_tx(bar, (uint32_t)((wok ? 2 * TC_M * SG_SEG : 0) + ng * 4 * SG_ASEG));
        if (wok) {
            const int x = s0 * (SG_SEG / 4), yr = ti.rt * TC_M;
            if (ti.shared) {
                tma_load_2d(s.st[slot].w[0], mp.sh_gate, x, yr, bar);
                tma_load_2d(s.st[slot].w[TC_M], mp.sh_up, x, yr, bar);
            } else {
                tma_load_3d(s.st[slot].w[0], mp.gate, x, yr, ti.slot, bar);
                tma_load_3d(s.st[slot].w[TC_M], mp.up, x, yr, ti.slot, bar);
            }
        }
    }
    if (lane < ng) tma_gather4(s.st[slot].act[4 * lane], mp.xact, s0 * (SG_ASEG / 4), t4[0], t4[1], t4[2], t4[3], bar);
}

__global__ void __launch_bounds__(WS_THREADS, 1) k_moe_gateup_ws(MoeShape sh, MoeLayerDev L, MoeScratch sc,
                                                                  int fmax_nb, const __grid_constant__ TcMaps mp) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    GuSmem &s = *reinterpret_cast<GuSmem *>(smem_raw);
    WsSync &y = s.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nu = routed_jobs(sh, sc), njobs = nu + (L.Fs > 0 ? 1 : 0);
    const int ntiles = tile_prefix(sh, L, sc, nu, njobs, false, s.pre);
    if ((int)blockIdx.x >= ntiles) return;
    const int nbD = sh.D / QK, nS = nbD / SG_BLK;
    const int mytiles = (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

    if (tid == 0) ws_init(y);
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&y.tmem)),
                     "r"(GU_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = y.tmem;

    if (warp < 16) {
        // ------------------------------------------------------------------ drain warps
        // warp w: rows 32 (w & 3) .. of matrix (w >> 2) & 1 (gate, up), pairs 16 (w >> 3) .. + 15
        const int m = (warp >> 2) & 1, h = warp >> 3, q4 = warp & 3, r = q4 * 32 + lane;
        const uint32_t lanes = (uint32_t)(q4 * 32) << 16, col = GU_ACC + 32 * m + 16 * h;
        for (int b = 0; b < WS_NBUF; b++) tmem_fill16(tmem + lanes + col + 64 * b, kMagic);
        tmem_wait_st();
        tc_fence_before();
        for (int b = 0; b < WS_NBUF; b++) warp_arrive(&y.accempty[b]);
        uint32_t G = 0;
        for (int i = 0; i < mytiles; i++) {
            TileInfo ti;
            if (lane == 0) decode_tile(sh, L, sc, mp, nu, njobs, s.pre, blockIdx.x + i * gridDim.x, false, ti);
            ti.rt = __shfl_sync(0xffffffffu, ti.rt, 0);
            ti.n0 = __shfl_sync(0xffffffffu, ti.n0, 0);
            ti.nn = __shfl_sync(0xffffffffu, ti.nn, 0);
            ti.p0 = __shfl_sync(0xffffffffu, ti.p0, 0);
            ti.F = __shfl_sync(0xffffffffu, ti.F, 0);
            uint64_t acc2[8];
#pragma unroll
            for (int k = 0; k < 8; k++) acc2[k] = 0;
            for (int g = 0; g < nbD; g++, G++) {
                const int b = G % WS_NBUF;
                const uint32_t par = (G / WS_NBUF) & 1;
                mbar_wait(&y.accfull[b], par, sc.err);
                mbar_wait(&y.aready[b], par, sc.err);   // acquires the unpackers' scales
                tc_fence_after();
                if (16 * h < ti.nn) {   // columns of pairs past nn keep the magic start (zero operand rows)
                    uint32_t v[16];
                    const uint32_t ta = tmem + lanes + col + 64 * b;
                    tmem_ld16(ta, v);
                    tmem_fill16(ta, kMagic);
                    chain_f2<16>(v, s.dw[b][m * TC_M + r], s.pc[b].v + 8 * h, acc2, mp.zero);
                    tmem_wait_st();
                }
                tc_fence_before();
                warp_arrive(&y.accempty[b]);
            }
            // epilogue: SwiGLU (of its 16 pairs, a gate warp keeps the first 8 and an up warp the last
            // 8; each hands the other half of its values over through X), then the mid blocks
            float *X = s.X;
            float acc[16];
#pragma unroll
            for (int k = 0; k < 8; k++) {
                acc[2 * k] = lo_f(acc2[k]);
                acc[2 * k + 1] = hi_f(acc2[k]);
            }
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const bool give = m == 0 ? k >= 8 : k < 8;
                if (give) X[(16 * h + k) * TC_M + r] = canon(acc[k]);
            }
            drain_bar();
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const bool keep = m == 0 ? k < 8 : k >= 8;
                if (keep) {
                    const float a = canon(acc[k]);
                    float *x = X + (16 * h + k) * TC_M + r;
                    *x = m == 0 ? swiglu_c(a, *x) : swiglu_c(*x, a);
                }
            }
            drain_bar();
            quant_tile(X, ti, sc.act_mid, fmax_nb, tid);
            drain_bar();   // X is rewritten by the next tile
        }
    } else if (warp < WS_COPY_WARP) {
        // ------------------------------------------------------------------ unpack warps
        // warps 16-19: gate rows, warps 20-23: up rows; both halves of each activation chunk
        const int u = tid - WS_UNPACK0, m = u >> 7, r = u & (TC_M - 1), q4 = warp & 3;
        const uint32_t lanes = (uint32_t)(q4 * 32) << 16;
        uint32_t G = 0;
        for (int i = 0; i < mytiles; i++) {
            for (int s0 = 0; s0 < nS; s0++) {
                const int qs = i * nS + s0, slot = qs & 1;
                mbar_wait(&y.full[slot], (qs >> 1) & 1, sc.err);
                const TileInfo &ti = s.ti[i % 3];
                const bool rowok = ti.rt * TC_M + r < ti.F;
                const int nn = ti.nn;
                const uint8_t *row = s.st[slot].w[m * TC_M + r];
#pragma unroll
                for (int jj = 0; jj < SG_BLK; jj++, G++) {
                    const int b = G % WS_NBUF;
                    mbar_wait(&y.accempty[b], (G / WS_NBUF) & 1, sc.err);
                    tc_fence_after();
                    uint32_t w[16];
                    uint32_t scb = 0;
                    if (rowok) {
                        switch (jj) {
                        case 0: scb = seg_q4_block<0>(row, w); break;
                        case 1: scb = seg_q4_block<1>(row, w); break;
                        case 2: scb = seg_q4_block<2>(row, w); break;
                        case 3: scb = seg_q4_block<3>(row, w); break;
                        case 4: scb = seg_q4_block<4>(row, w); break;
                        case 5: scb = seg_q4_block<5>(row, w); break;
                        case 6: scb = seg_q4_block<6>(row, w); break;
                        default: scb = seg_q4_block<7>(row, w); break;
                        }
                    } else {
#pragma unroll
                        for (int k = 0; k < 16; k++) w[k] = 0;
                    }
                    tmem_st16(tmem + lanes + GU_A + 32 * b + 16 * m, w);
                    s.dw[b][m * TC_M + r] = f16_to_f32_hw(scb);   // chains are canonicalised before use
                    unpack_act_half<1>(&s.st[slot].act[0][0], SG_ASEG, jj, nn, s.b[b], s.pc[b], r, m);
                    if (jj == SG_BLK - 1) warp_arrive(&y.empty[slot]);   // this warp is done with the slot
                    tmem_wait_st();
                    fence_proxy_async();
                    tc_fence_before();
                    warp_arrive(&y.aready[b]);
                }
            }
        }
    } else if (warp == WS_COPY_WARP) {
        // ------------------------------------------------------------------ copy warp
        for (int qs = 0; qs < mytiles * nS; qs++) {
            if (qs >= 2) mbar_wait(&y.empty[qs & 1], ((qs >> 1) - 1) & 1, sc.err);
            gu_issue_stage(s, sh, L, sc, mp, nu, njobs, ntiles, nS, qs);
        }
    } else {
        // ------------------------------------------------------------------ MMA warp
        const uint32_t idesc = umma_idesc_i8(false);
        for (uint32_t G = 0; G < (uint32_t)(mytiles * nbD); G++) {
            const int b = G % WS_NBUF;
            const uint32_t par = (G / WS_NBUF) & 1;
            mbar_wait(&y.aready[b], par, sc.err);
            mbar_wait(&y.accempty[b], par, sc.err);
            tc_fence_after();
            if (lane == 0) {
                const uint32_t sb = smem_u32(s.b[b]);
#pragma unroll
                for (int m = 0; m < 2; m++) {
                    const uint32_t d = tmem + GU_ACC + 64 * b + 32 * m, a = tmem + GU_A + 32 * b + 16 * m;
#pragma unroll
                    for (int k = 0; k < 2; k++) umma_i8_ts(d, a + 8 * k, umma_desc(sb + 256 * k), idesc);
                }
                umma_commit(&y.accfull[b]);
            }
            __syncwarp();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GU_TMEM_COLS));
}

// --------------------------------------------------------------------------------------- down

constexpr int DN_SLOT = TC_M * SD_MAXNB * Q4_BLOCK + TC_N * SD_MAXNB * ACT_BLOCK;
static_assert(DN_SLOT % 128 == 0, "tensor-map destinations stay 128-byte aligned");

struct DnSmem {
    uint8_t st[2][DN_SLOT];         // one tile per slot: its 128 whole rows, then its 32 pair rows
    uint8_t b[WS_NBUF][TC_N * 64];
    PairConst pc[WS_NBUF];
    float dw[WS_NBUF][TC_M];
    TileInfo ti[3];
    int pre[SG_MAXJOBS + 1];
    WsSync y;
};

// Tensor-memory columns (256 allocated): accumulators [b] at 32b, operand A [b] at 128 + 16b.
constexpr uint32_t DN_ACC = 0, DN_A = 128, DN_TMEM_COLS = 256;

template <int JM>
__device__ __forceinline__ void dn_unpack_row(DnSmem &s, int slot, int b, int j, int rb, bool rowok, uint32_t tm_a,
                                              int r) {
    uint32_t w[16];
    uint32_t scb = 0;
    if (rowok) {
        scb = row_q4_block<JM>(s.st[slot] + r * rb, j, w);
    } else {
#pragma unroll
        for (int k = 0; k < 16; k++) w[k] = 0;
    }
    tmem_st16(tm_a, w);
    s.dw[b][r] = f16_to_f32_hw(scb);   // chains are canonicalised before use
}

// Tensor-map loads of down tile i (its 128 whole rows and 32 pair rows) into slot i & 1, by lane 0
// of the copy warp; the tile description goes into the info ring.
__device__ __forceinline__ void dn_issue_tile(DnSmem &s, const MoeShape &sh, const MoeLayerDev &L,
                                              const MoeScratch &sc, const TcMaps &mp, int nu, int njobs, int ntiles,
                                              int i, int rb, int pitch, int rg) {
    const int t = blockIdx.x + i * gridDim.x;
    if (t >= ntiles) return;
    if ((threadIdx.x & 31) == 0) {
        TileInfo &ti = s.ti[i % 3];
        decode_tile(sh, L, sc, mp, nu, njobs, s.pre, t, true, ti);
        uint64_t *bar = &s.y.full[i & 1];
        uint8_t *dst = s.st[i & 1];
        const bool wok = ti.w0 != nullptr;
        mbar_expect_tx(bar, (uint32_t)(wok ? TC_M * rb + TC_N * pitch : 0));
        if (wok) {
            const int yr = ti.rt * TC_M / rg;
            if (ti.shared) tma_load_2d(dst, mp.sh_down, 0, yr, bar);
            else tma_load_3d(dst, mp.down, 0, yr, ti.slot, bar);
            tma_load_2d(dst + TC_M * rb, mp.mid, 0, ti.p0 + ti.n0, bar);
        }
    }
    __syncwarp();
}

__global__ void __launch_bounds__(WS_THREADS, 1) k_moe_down_ws(MoeShape sh, MoeLayerDev L, MoeScratch sc,
                                                                int fmax_nb, int nbF, int rg,
                                                                const __grid_constant__ TcMaps mp) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    DnSmem &s = *reinterpret_cast<DnSmem *>(smem_raw);
    WsSync &y = s.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nu = routed_jobs(sh, sc), njobs = nu + (L.Fs > 0 ? 1 : 0);
    const int ntiles = tile_prefix(sh, L, sc, nu, njobs, true, s.pre);
    if ((int)blockIdx.x >= ntiles) return;
    const int mytiles = (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const int rb = nbF * Q4_BLOCK, pitch = nbF * ACT_BLOCK;
    const bool csh1 = ((pitch / 16) & 7) == 4;   // bank-group step of the pair rows

    if (tid == 0) ws_init(y);
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&y.tmem)),
                     "r"(DN_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = y.tmem;

    if (warp < 16) {
        // ------------------------------------------------------------------ drain warps
        // warp w: rows 32 (w & 3) .., pairs 8 (w >> 2) .. + 7
        const int c4 = warp >> 2, q4 = warp & 3, r = q4 * 32 + lane;
        const uint32_t lanes = (uint32_t)(q4 * 32) << 16, col = DN_ACC + 8 * c4;
        for (int b = 0; b < WS_NBUF; b++) tmem_fill8(tmem + lanes + col + 32 * b, kMagic);
        tmem_wait_st();
        tc_fence_before();
        for (int b = 0; b < WS_NBUF; b++) warp_arrive(&y.accempty[b]);
        uint32_t G = 0;
        for (int i = 0; i < mytiles; i++) {
            TileInfo ti;
            if (lane == 0) decode_tile(sh, L, sc, mp, nu, njobs, s.pre, blockIdx.x + i * gridDim.x, true, ti);
            const int rt = __shfl_sync(0xffffffffu, ti.rt, 0), n0 = __shfl_sync(0xffffffffu, ti.n0, 0);
            const int nn = __shfl_sync(0xffffffffu, ti.nn, 0), p0 = __shfl_sync(0xffffffffu, ti.p0, 0);
            const int shared = __shfl_sync(0xffffffffu, ti.shared, 0);
            const int ok = __shfl_sync(0xffffffffu, ti.w0 != nullptr ? 1 : 0, 0);
            uint64_t acc2[4];
#pragma unroll
            for (int k = 0; k < 4; k++) acc2[k] = 0;
            for (int g = 0; g < nbF; g += 2, G += 2) {   // two blocks per pass: one load latency
                const int b0 = G % WS_NBUF, b1 = (G + 1) % WS_NBUF;
                const uint32_t p0 = (G / WS_NBUF) & 1, p1 = ((G + 1) / WS_NBUF) & 1;
                mbar_wait(&y.accfull[b0], p0, sc.err);
                mbar_wait(&y.aready[b0], p0, sc.err);   // acquires the unpackers' scales
                mbar_wait(&y.accfull[b1], p1, sc.err);
                mbar_wait(&y.aready[b1], p1, sc.err);
                tc_fence_after();
                uint32_t v0[8], v1[8];
                const uint32_t t0 = tmem + lanes + col + 32 * b0, t1 = tmem + lanes + col + 32 * b1;
                tmem_ld8_async(t0, v0);
                tmem_ld8_async(t1, v1);
                tmem_wait_ld();
                tmem_fill8(t0, kMagic);
                tmem_fill8(t1, kMagic);
                chain_f2<8>(v0, s.dw[b0][r], s.pc[b0].v + 4 * c4, acc2, mp.zero);
                chain_f2<8>(v1, s.dw[b1][r], s.pc[b1].v + 4 * c4, acc2, mp.zero);
                tmem_wait_st();
                tc_fence_before();
                warp_arrive(&y.accempty[b0]);
                warp_arrive(&y.accempty[b1]);
            }
            const int row = rt * TC_M + r;
            if (ok && row < sh.D) {   // canonical outputs: Y [pair][D] (routed) or S [token][D] (shared)
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int n = 8 * c4 + k;
                    if (n < nn) {
                        float *out = shared ? sc.S + (int64_t)(n0 + n) * sh.D : sc.Y + (int64_t)(p0 + n0 + n) * sh.D;
                        out[row] = canon(k & 1 ? hi_f(acc2[k >> 1]) : lo_f(acc2[k >> 1]));
                    }
                }
            }
        }
    } else if (warp < WS_COPY_WARP) {
        // ------------------------------------------------------------------ unpack warps
        // warps 16-19: the 128 rows into operand A; warps 20-23: the 32 pair rows into operand B
        const int u = tid - WS_UNPACK0, q4 = warp & 3, r = u & (TC_M - 1);
        const bool rows_role = u < TC_M;
        const uint32_t lanes = (uint32_t)(q4 * 32) << 16;
        uint32_t G = 0;
        for (int i = 0; i < mytiles; i++) {
            const int slot = i & 1;
            mbar_wait(&y.full[slot], (i >> 1) & 1, sc.err);
            const TileInfo &ti = s.ti[i % 3];
            const bool rowok = ti.w0 != nullptr && ti.rt * TC_M + r < sh.D;
            const int nn = ti.nn;
            const uint8_t *act = s.st[slot] + TC_M * rb;
            for (int g0 = 0; g0 < nbF; g0 += 4) {
#pragma unroll
                for (int jm = 0; jm < 4; jm++, G++) {
                    const int b = G % WS_NBUF, j = g0 + jm;
                    mbar_wait(&y.accempty[b], (G / WS_NBUF) & 1, sc.err);
                    tc_fence_after();
                    if (rows_role) {
                        const uint32_t ta = tmem + lanes + DN_A + 16 * b;
                        switch (jm) {
                        case 0: dn_unpack_row<0>(s, slot, b, j, rb, rowok, ta, r); break;
                        case 1: dn_unpack_row<1>(s, slot, b, j, rb, rowok, ta, r); break;
                        case 2: dn_unpack_row<2>(s, slot, b, j, rb, rowok, ta, r); break;
                        default: dn_unpack_row<3>(s, slot, b, j, rb, rowok, ta, r); break;
                        }
                    } else if (csh1) {
                        if (jm & 1) unpack_act_ws<1, 1>(act, pitch, j, nn, s.b[b], s.pc[b], r);
                        else unpack_act_ws<0, 1>(act, pitch, j, nn, s.b[b], s.pc[b], r);
                    } else {
                        if (jm & 1) unpack_act_ws<1, 2>(act, pitch, j, nn, s.b[b], s.pc[b], r);
                        else unpack_act_ws<0, 2>(act, pitch, j, nn, s.b[b], s.pc[b], r);
                    }
                    if (j == nbF - 1) warp_arrive(&y.empty[slot]);
                    if (rows_role) tmem_wait_st();
                    fence_proxy_async();
                    tc_fence_before();
                    warp_arrive(&y.aready[b]);
                }
            }
        }
    } else if (warp == WS_COPY_WARP) {
        // ------------------------------------------------------------------ copy warp
        for (int i = 0; i < mytiles; i++) {
            if (i >= 2) mbar_wait(&y.empty[i & 1], ((i >> 1) - 1) & 1, sc.err);
            dn_issue_tile(s, sh, L, sc, mp, nu, njobs, ntiles, i, rb, pitch, rg);
        }
    } else {
        // ------------------------------------------------------------------ MMA warp
        const uint32_t idesc = umma_idesc_i8(false);
        for (uint32_t G = 0; G < (uint32_t)(mytiles * nbF); G++) {
            const int b = G % WS_NBUF;
            const uint32_t par = (G / WS_NBUF) & 1;
            mbar_wait(&y.aready[b], par, sc.err);
            mbar_wait(&y.accempty[b], par, sc.err);
            tc_fence_after();
            if (lane == 0) {
                const uint32_t sb = smem_u32(s.b[b]), d = tmem + DN_ACC + 32 * b, a = tmem + DN_A + 16 * b;
#pragma unroll
                for (int k = 0; k < 2; k++) umma_i8_ts(d, a + 8 * k, umma_desc(sb + 256 * k), idesc);
                umma_commit(&y.accfull[b]);
            }
            __syncwarp();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(DN_TMEM_COLS));
}

__global__ void __launch_bounds__(TC_THREADS, 3) k_moe_gateup_tc(MoeShape sh, MoeLayerDev L, MoeScratch sc,
                                                                  int fmax_nb) {
    __shared__ __align__(1024) TcSmem s;
    const int rt = blockIdx.x, u = blockIdx.y, n0 = blockIdx.z * TC_N;
    const int nu = routed_jobs(sh, sc);
    if (u >= nu + (L.Fs > 0 ? 1 : 0)) return;
    Job job;
    if (!get_job(sh, L, sc, u, nu, job)) return;
    if (rt * TC_M >= job.F || n0 >= job.n) return;
    if (job.dtype == Q4) gateup_tc_body<Q4>(sh, sc, job, rt, n0, fmax_nb, s);
    else gateup_tc_body<Q8>(sh, sc, job, rt, n0, fmax_nb, s);
}

__global__ void __launch_bounds__(TC_THREADS, 3) k_moe_down_tc(MoeShape sh, MoeLayerDev L, MoeScratch sc,
                                                                int fmax_nb) {
    __shared__ __align__(1024) TcSmem s;
    const int rt = blockIdx.x, u = blockIdx.y, n0 = blockIdx.z * TC_N;
    const int nu = routed_jobs(sh, sc);
    if (u >= nu + (L.Fs > 0 ? 1 : 0)) return;
    Job job;
    if (!get_job(sh, L, sc, u, nu, job)) return;
    if (n0 >= job.n) return;
    if (job.dtype == Q4) down_tc_body<Q4>(sh, sc, job, rt, n0, fmax_nb, s);
    else down_tc_body<Q8>(sh, sc, job, rt, n0, fmax_nb, s);
}

static int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 1;
    }
    return n;
}

static bool staged_on() {
    static const bool on = [] {
        const char *e = std::getenv("HXB_TC_STAGED");
        return !(e && e[0] == '0');
    }();
    return on;
}

}  // namespace

// ------------------------------------------------------------------------------ tensor maps

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// A map of 32-bit words: rank 2 or 3, dims innermost first, strides in bytes of dims 1.., box.
static bool encode_u32(uint64_t out[16], const void *base, int rank, const uint64_t *dims, const uint64_t *strides,
                       const uint32_t *box) {
    const EncodeTiledFn fn = encode_fn();
    if (!fn || !base || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    cuuint64_t gd[3], gs[2];
    cuuint32_t bx[3], es[3] = {1, 1, 1};
    for (int i = 0; i < rank; i++) {
        gd[i] = dims[i];
        bx[i] = box[i];
        if (i + 1 < rank) gs[i] = strides[i];
    }
    return fn(reinterpret_cast<CUtensorMap *>(out), CU_TENSOR_MAP_DATA_TYPE_UINT32, (cuuint32_t)rank,
              const_cast<void *>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void encode_tc_maps(TcMaps &m, const TcMapSrc &a) {
    m = TcMaps();
    m.arena = a.arena;
    m.slot_bytes = a.slot_bytes;
    m.n_slots = a.n_slots;
    m.xact_rows = a.T;
    const bool q4 = a.expert_dtype == Q4 && (a.Fs == 0 || a.sh_dtype == Q4);
    if (!q4 || !a.arena || a.slot_bytes % 16 || a.E + 1 > SG_MAXJOBS || a.D % QK || a.F % QK) return;
    const int nbD = a.D / QK, nbF = a.F / QK;
    const int64_t rbD = (int64_t)nbD * Q4_BLOCK;
    const uint64_t S = (uint64_t)a.n_slots, SB = (uint64_t)a.slot_bytes;
    // gate/up: 8-block stages of 128 rows; activations by gather4 rows of 8 blocks
    if (nbD % SG_BLK == 0 && a.off_up % 16 == 0) {
        const uint64_t d3[3] = {(uint64_t)rbD / 4, (uint64_t)a.F, S}, s3[2] = {(uint64_t)rbD, SB};
        const uint32_t b3[3] = {SG_SEG / 4, TC_M, 1};
        const uint64_t dx[2] = {(uint64_t)nbD * ACT_BLOCK / 4, (uint64_t)a.T}, sx[1] = {(uint64_t)nbD * ACT_BLOCK};
        const uint32_t bxa[2] = {SG_ASEG / 4, 1};
        bool ok = encode_u32(m.gate, a.arena, 3, d3, s3, b3) && encode_u32(m.up, a.arena + a.off_up, 3, d3, s3, b3) &&
                  encode_u32(m.xact, a.xact, 2, dx, sx, bxa);
        if (ok && a.Fs > 0) {
            const uint64_t d2[2] = {(uint64_t)rbD / 4, (uint64_t)a.Fs}, s2[1] = {(uint64_t)rbD};
            const uint32_t b2[2] = {SG_SEG / 4, TC_M};
            ok = encode_u32(m.sh_gate, a.sh_gate, 2, d2, s2, b2) && encode_u32(m.sh_up, a.sh_up, 2, d2, s2, b2);
        }
        m.gu_ok = ok;
    }
    // down: whole rows (nbF of 4, 8 or 12 blocks) in groups of rg rows; mid rows of 32 pairs
    if (nbF % 4 == 0 && nbF <= SD_MAXNB && (a.Fs == 0 || a.Fs == a.F) && a.fmax_nb == nbF && a.off_down % 16 == 0 &&
        a.D % TC_M == 0) {
        int rg = 1;
        while ((rg * nbF * Q4_BLOCK) % 16) rg <<= 1;
        const uint64_t gb = (uint64_t)rg * nbF * Q4_BLOCK;
        const uint64_t d3[3] = {gb / 4, (uint64_t)a.D / rg, S}, s3[2] = {gb, SB};
        const uint32_t b3[3] = {(uint32_t)(gb / 4), (uint32_t)(TC_M / rg), 1};
        const uint64_t dm[2] = {(uint64_t)a.fmax_nb * ACT_BLOCK / 4, (uint64_t)a.mid_rows},
                       sm[1] = {(uint64_t)a.fmax_nb * ACT_BLOCK};
        const uint32_t bm[2] = {(uint32_t)(nbF * ACT_BLOCK / 4), TC_N};
        bool ok = gb / 4 <= 256 && encode_u32(m.down, a.arena + a.off_down, 3, d3, s3, b3) &&
                  encode_u32(m.mid, a.mid, 2, dm, sm, bm);
        if (ok && a.Fs > 0) {
            const uint64_t d2[2] = {gb / 4, (uint64_t)a.D / rg}, s2[1] = {gb};
            const uint32_t b2[2] = {(uint32_t)(gb / 4), (uint32_t)(TC_M / rg)};
            ok = encode_u32(m.sh_down, a.sh_down, 2, d2, s2, b2);
        }
        m.down_rg = rg;
        m.dn_ok = ok;
    }
}

cudaError_t init_tc_attributes() {
    cudaError_t e = cudaFuncSetAttribute(k_moe_gateup_ws, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(GuSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_moe_down_ws, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(DnSmem));
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, (const void *)k_moe_gateup_tc);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, (const void *)k_moe_down_tc);
    return e;
}

cudaError_t launch_moe_experts_tc(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, int which,
                                  cudaStream_t s) {
    const int T = sh.T, K = sh.route.K, E = sh.route.E;
    const int fmax_nb = std::max(sh.F, L.Fs) / QK;
    const int maxjobs = std::min(E, T * K) + (L.Fs > 0 ? 1 : 0);
    const int maxn = std::max(T, 1);   // a bucket holds at most T pairs (one per token)
    if (which & 1) {
        if (staged_on() && L.tc && L.tc->gu_ok && sh.T <= L.tc->xact_rows) {
            k_moe_gateup_ws<<<sm_count(), WS_THREADS, sizeof(GuSmem), s>>>(sh, L, sc, fmax_nb, *L.tc);
        } else {
            const dim3 grid((unsigned)((std::max(sh.F, L.Fs) + TC_M - 1) / TC_M), (unsigned)maxjobs,
                            (unsigned)((maxn + TC_N - 1) / TC_N));
            k_moe_gateup_tc<<<grid, TC_THREADS, 0, s>>>(sh, L, sc, fmax_nb);
        }
    }
    if (which & 2) {
        if (staged_on() && L.tc && L.tc->dn_ok) {
            k_moe_down_ws<<<sm_count(), WS_THREADS, sizeof(DnSmem), s>>>(sh, L, sc, fmax_nb, sh.F / QK, L.tc->down_rg,
                                                                          *L.tc);
        } else {
            const dim3 grid((unsigned)((sh.D + TC_M - 1) / TC_M), (unsigned)maxjobs, (unsigned)((maxn + TC_N - 1) / TC_N));
            k_moe_down_tc<<<grid, TC_THREADS, 0, s>>>(sh, L, sc, fmax_nb);
        }
    }
    return cudaGetLastError();
}

}  // namespace hx
