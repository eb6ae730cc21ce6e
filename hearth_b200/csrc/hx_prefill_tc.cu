// hx_prefill_tc.cu — expert gate/up and down on the 5th-generation tensor cores (tcgen05) for
// prefill and verification batches (many tokens per expert).
//
// NUMERICS §3 fixes each output as acc = ((0 + t_0) + t_1) + ... over the 64-weight blocks g of the
// row, t_g = (float)isum_g * (dw_g * dx_g), where isum_g is the exact int32 dot of the block. The
// tensor cores produce the isum_g of a whole tile: per block, two `tcgen05.mma .kind::i8` (K = 32
// bytes each) write D[128 rows][32 tokens] (s32) into tensor memory, one fresh accumulation per block;
// the CTA then reads the tile back (`tcgen05.ld`) and each thread runs its row's float chain in
// registers, in block order. Q4 weights enter as unsigned nibbles (u8 x s8 MMA) and the identity
// sum((nib-8)*xq) = sum(nib*xq) - 8*sum(xq) removes the offset exactly; Q8 weights enter as s8.
//
// Operands in shared memory use the K-major, unswizzled core-matrix layout of the UMMA descriptors:
// a core matrix is 8 rows x 16 bytes (128 contiguous bytes), the four 16-byte K-chunks of a 64-byte
// block row are 128 bytes apart (LBO) and 8-row groups 512 bytes apart (SBO). Every thread loads its
// own row's block for the next iteration into registers while the current one is in flight.
//
// Gate/up CTA: 128 rows of gate and the same 128 rows of up x 32 token pairs of one job (routed expert
// bucket or the shared expert); epilogue SwiGLU and the mid activation blocks (NUMERICS §2, one per
// 64 rows). Down CTA: 128 rows of down x 32 pairs; epilogue the canonical outputs into Y (routed) or
// S (shared) for the rank-order sum.
#include "hx_device.cuh"
#include "hx_kernels.h"
#include "hx_route.cuh"
#include "hx_moe_job.cuh"

#include <algorithm>

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
// Staged persistent path (Q4 experts). One CTA of 256 threads per SM walks a static list of
// tiles; the weight rows and activation rows of each tile reach shared memory by 1-D bulk copies
// (cp.async.bulk, one per row segment) into a two-slot ring that runs ahead across tiles, so that
// up to two stages (~176 KB) per SM are in flight while the CTA unpacks, multiplies and drains.
// Unpacking reads shared memory with 16- or 8-byte loads that are free of bank conflicts; the row
// loads of the register path above touch one 32-byte sector per thread and instruction, which
// keeps the load/store unit, not HBM, busy.
//
// Tiles: job u (routed bucket or the shared expert) owns ceil(n_u / 32) x (row tiles) tiles, in
// job order and, inside a job, pair tile major and row tile minor, so that consecutive tiles read
// the same activations. Tile t goes to CTA t % gridDim.x.
// =============================================================================================

constexpr int SG_THREADS = 256;
constexpr int SG_BLK = 8;                        // gate/up: blocks per stage
constexpr int SG_SEG = SG_BLK * Q4_BLOCK;        // 272: one row's bytes per stage
constexpr int SG_ASEG = SG_BLK * ACT_BLOCK;      // 576: one pair's activation bytes per stage
constexpr int SG_MAXJOBS = 1024 + 1;             // routed buckets (E <= 1024) + the shared expert
constexpr int SD_MAXNB = 12;                     // down: whole rows of at most 12 blocks (F <= 768)

struct TileInfo {
    const uint8_t *w0, *w1;   // gate and up rows (gate/up), down rows (down)
    int rt, n0, nn, p0;       // row tile, first pair of the tile in the job, pairs, job's first pair
    int F, shared;            // job's expert width, shared-expert job
    int tok[TC_N];            // token of each pair (gate/up)
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
__device__ void decode_tile(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, int nu, int njobs,
                            const int *pre, int t, bool down, TileInfo &ti) {
    int lo = 0, hi = njobs;   // largest u with pre[u] <= t
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (pre[mid] <= t) lo = mid;
        else hi = mid;
    }
    Job job;
    const bool ok = get_job(sh, L, sc, lo, nu, job);
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

// Activation operand of block j for the 32 pairs of a stage (pair rows `pitch` bytes apart):
// `nthr` threads (tid - t0 in [0, nthr), nthr = 128 or 256) move 16 or 8 bytes each; pairs past nn
// get zeros. Thread t0 + n (n < 32) also stores the pair's d and -8 * sum (the Q4 offset term).
__device__ __forceinline__ void unpack_act(const uint8_t *act, int pitch, int j, int nn, uint8_t *bop, float *dx,
                                           int *c8, int t, int nthr) {
    const int n = t & 31;
    const bool live = n < nn;
    const uint8_t *src = act + n * pitch + j * ACT_BLOCK + 8;
    if (nthr == 256) {   // 8 bytes: chunk (t >> 5) & 3, half t >> 7
        const int c = (t >> 5) & 3, h = t >> 7;
        const uint2 v = live ? *reinterpret_cast<const uint2 *>(src + 16 * c + 8 * h) : make_uint2(0, 0);
        *reinterpret_cast<uint2 *>(bop + op_off(n, c) + 8 * h) = v;
    } else {             // 16 bytes: chunk t >> 5
        const int c = t >> 5;
        uint2 v0 = make_uint2(0, 0), v1 = make_uint2(0, 0);
        if (live) {
            v0 = *reinterpret_cast<const uint2 *>(src + 16 * c);
            v1 = *reinterpret_cast<const uint2 *>(src + 16 * c + 8);
        }
        *reinterpret_cast<uint4 *>(bop + op_off(n, c)) = make_uint4(v0.x, v0.y, v1.x, v1.y);
    }
    if (t < 32) {
        uint2 hd = make_uint2(0, 0);
        if (live) hd = *reinterpret_cast<const uint2 *>(src - 8);
        dx[n] = __uint_as_float(hd.x);
        c8[n] = -8 * (int)hd.y;
    }
}

// Q4 float chains of one drained accumulator: NC columns of v against pairs col0 + i.
template <int NC>
__device__ __forceinline__ void chain_q4(const uint32_t *v, float dw, const float *dx, const int *c8, int col0,
                                         float *acc) {
#pragma unroll
    for (int i = 0; i < NC; i++) {
        const int isum = (int)v[i] + c8[col0 + i];
        acc[i] = __fadd_rn(acc[i], __fmul_rn(__int2float_rn(isum), __fmul_rn(dw, dx[col0 + i])));
    }
}

// ------------------------------------------------------------------------------------ gate/up

struct GuStage {
    uint8_t w[2 * TC_M][SG_SEG];    // rows 0..127: gate, 128..255: up
    uint8_t act[TC_N][SG_ASEG];
};

struct GuSmem {
    GuStage st[2];
    uint8_t a[2][2][TC_M * 64];     // [operand buffer][gate, up]; the epilogue reuses them as floats
    uint8_t b[2][TC_N * 64];
    float dx[2][TC_N];
    int c8[2][TC_N];
    TileInfo ti[3];
    int pre[SG_MAXJOBS + 1];
    uint64_t full[2], mma;
    uint32_t tmem;
};
static_assert(sizeof(GuStage) % 16 == 0, "stage slots stay 16-byte aligned");

// Issues stage q of this CTA (tile q / nS, blocks 8 (q % nS) ..) into slot q & 1.
__device__ __forceinline__ void gu_issue(GuSmem &s, const MoeShape &sh, const MoeScratch &sc, int q, int nS,
                                         int ntiles) {
    const int i = q / nS, st = q % nS, t = blockIdx.x + i * gridDim.x;
    if (t >= ntiles) return;
    const TileInfo &ti = s.ti[i % 3];
    const int tid = threadIdx.x, slot = q & 1;
    uint64_t *bar = &s.full[slot];
    const int64_t rbD = (int64_t)(sh.D / QK) * Q4_BLOCK;
    const int m = tid >> 7, r = tid & (TC_M - 1), row = ti.rt * TC_M + r;
    fence_proxy_async();   // this thread's earlier shared-memory reads of the slot come first
    if (row < ti.F) bulk_g2s(s.st[slot].w[tid], (m ? ti.w1 : ti.w0) + row * rbD + st * SG_SEG, SG_SEG, bar);
    if (tid < ti.nn)
        bulk_g2s(s.st[slot].act[tid], reinterpret_cast<const uint8_t *>(sc.xact + (int64_t)ti.tok[tid] * (sh.D / QK)) +
                                          st * SG_ASEG,
                 SG_ASEG, bar);
    if (tid == 0) {
        const int rows = max(0, min(TC_M, ti.F - ti.rt * TC_M));
        mbar_expect_tx(bar, (uint32_t)(2 * rows * SG_SEG + ti.nn * SG_ASEG));
    }
}

__device__ __forceinline__ void gu_fill_info(GuSmem &s, const MoeShape &sh, const MoeLayerDev &L,
                                             const MoeScratch &sc, int nu, int njobs, int ntiles, int i) {
    // warp 1 fills the description of this CTA's tile i (if it exists)
    const int t = blockIdx.x + i * gridDim.x;
    if (t >= ntiles) return;
    TileInfo &ti = s.ti[i % 3];
    const int lane = threadIdx.x & 31;
    if (lane == 0) decode_tile(sh, L, sc, nu, njobs, s.pre, t, false, ti);
    __syncwarp();
    if (lane < ti.nn) {
        Job j;
        j.shared = ti.shared;
        j.p0 = ti.p0;
        ti.tok[lane] = job_token(sc, j, ti.n0 + lane);
    }
}

template <int J>
__device__ __forceinline__ uint32_t gu_unpack(GuSmem &s, const TileInfo &ti, int slot, int buf, int tid) {
    const int m = tid >> 7, r = tid & (TC_M - 1);
    uint32_t w[16];
    uint32_t scb = 0;
    if (ti.rt * TC_M + r < ti.F) {
        scb = seg_q4_block<J>(s.st[slot].w[tid], w);
    } else {
#pragma unroll
        for (int i = 0; i < 16; i++) w[i] = 0;
    }
    store_operand_row(s.a[buf][m], r, w);
    unpack_act(&s.st[slot].act[0][0], SG_ASEG, J, ti.nn, s.b[buf], s.dx[buf], s.c8[buf], tid, SG_THREADS);
    return scb;
}

// j in 0..7; inside the unrolled block loop j is a constant and the switch folds away.
__device__ __forceinline__ uint32_t gu_unpack_j(GuSmem &s, const TileInfo &ti, int slot, int buf, int tid, int j) {
    switch (j) {
    case 0: return gu_unpack<0>(s, ti, slot, buf, tid);
    case 1: return gu_unpack<1>(s, ti, slot, buf, tid);
    case 2: return gu_unpack<2>(s, ti, slot, buf, tid);
    case 3: return gu_unpack<3>(s, ti, slot, buf, tid);
    case 4: return gu_unpack<4>(s, ti, slot, buf, tid);
    case 5: return gu_unpack<5>(s, ti, slot, buf, tid);
    case 6: return gu_unpack<6>(s, ti, slot, buf, tid);
    default: return gu_unpack<7>(s, ti, slot, buf, tid);
    }
}

__device__ __forceinline__ void gu_mma(GuSmem &s, uint32_t tmem, uint32_t idesc, int buf) {
    const uint32_t sa0 = smem_u32(s.a[buf][0]), sa1 = smem_u32(s.a[buf][1]), sb = smem_u32(s.b[buf]);
#pragma unroll
    for (int k = 0; k < 2; k++) {
        umma_i8(tmem, umma_desc(sa0 + 256 * k), umma_desc(sb + 256 * k), idesc, k > 0);
        umma_i8(tmem + TC_N, umma_desc(sa1 + 256 * k), umma_desc(sb + 256 * k), idesc, k > 0);
    }
    umma_commit(&s.mma);
}

__device__ __forceinline__ void cta_sync_tc() {
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
}

__global__ void __launch_bounds__(SG_THREADS, 1) k_moe_gateup_tcs(MoeShape sh, MoeLayerDev L, MoeScratch sc,
                                                                   int fmax_nb) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    GuSmem &s = *reinterpret_cast<GuSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nu = routed_jobs(sh, sc), njobs = nu + (L.Fs > 0 ? 1 : 0);
    const int ntiles = tile_prefix(sh, L, sc, nu, njobs, false, s.pre);
    if ((int)blockIdx.x >= ntiles) return;
    const int nbD = sh.D / QK, nS = nbD / SG_BLK;
    const int mytiles = (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

    if (tid == 0) {
        mbar_init(&s.full[0], 1);
        mbar_init(&s.full[1], 1);
        mbar_init(&s.mma, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        gu_fill_info(s, sh, L, sc, nu, njobs, ntiles, 0);
        gu_fill_info(s, sh, L, sc, nu, njobs, ntiles, 1);
    }
    const uint32_t tmem = tmem_alloc(&s.tmem, 2 * TC_N);   // includes a CTA barrier
    gu_issue(s, sh, sc, 0, nS, ntiles);
    gu_issue(s, sh, sc, 1, nS, ntiles);
    const uint32_t idesc = umma_idesc_i8(false);
    const int m = tid >> 7;
    uint32_t mma_phase = 0;

    for (int i = 0; i < mytiles; i++) {
        const TileInfo &ti = s.ti[i % 3];
        if (warp == 1) gu_fill_info(s, sh, L, sc, nu, njobs, ntiles, i + 2);   // visible after the next barrier
        float acc[TC_N];
#pragma unroll
        for (int n = 0; n < TC_N; n++) acc[n] = 0.0f;
        float dw_next = 0.0f;
        for (int s0 = 0; s0 < nS; s0++) {
            const int q = i * nS + s0, slot = q & 1;
            mbar_wait(&s.full[slot], (uint32_t)((q >> 1) & 1), sc.err);
            if (s0 == 0) {   // prologue of the tile: block 0 unpacked and multiplied
                dw_next = f16_to_f32(gu_unpack<0>(s, ti, slot, 0, tid));
                cta_sync_tc();
                if (tid == 0) gu_mma(s, tmem, idesc, 0);
            }
#pragma unroll
            for (int jj = 0; jj < SG_BLK; jj++) {
                const int g = s0 * SG_BLK + jj;
                const float dw = dw_next;
                if (jj + 1 < SG_BLK) {
                    dw_next = f16_to_f32(gu_unpack_j(s, ti, slot, (g + 1) & 1, tid, jj + 1));
                } else if (s0 + 1 < nS) {   // block 0 of the next stage
                    const int q1 = q + 1;
                    mbar_wait(&s.full[q1 & 1], (uint32_t)((q1 >> 1) & 1), sc.err);
                    dw_next = f16_to_f32(gu_unpack<0>(s, ti, q1 & 1, (g + 1) & 1, tid));
                }
                mbar_wait(&s.mma, mma_phase, sc.err);
                mma_phase ^= 1;
                tc_fence_after();
                {
                    uint32_t v[32];
                    tmem_ld32(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(m * TC_N), v);
                    chain_q4<TC_N>(v, dw, s.dx[g & 1], s.c8[g & 1], 0, acc);
                }
                cta_sync_tc();
                if (jj == SG_BLK - 2) gu_issue(s, sh, sc, q + 2, nS, ntiles);   // slot of stage q is read
                if (g + 1 < nbD && tid == 0) gu_mma(s, tmem, idesc, (g + 1) & 1);
            }
        }
        // epilogue: SwiGLU through shared memory, then the mid activation blocks (NUMERICS §2)
        float *U = reinterpret_cast<float *>(s.a[0]);   // [32][128]
        float *M = reinterpret_cast<float *>(s.a[1]);   // [32][128]
        const int r = tid & (TC_M - 1);
        if (m == 1) {
#pragma unroll
            for (int n = 0; n < TC_N; n++) U[n * TC_M + r] = canon(acc[n]);
        }
        __syncthreads();
        if (m == 0) {
#pragma unroll
            for (int n = 0; n < TC_N; n++) M[n * TC_M + r] = swiglu_c(canon(acc[n]), U[n * TC_M + r]);
        }
        __syncthreads();
        for (int u = warp; u < 2 * TC_N; u += SG_THREADS / 32) {
            const int n = u >> 1, b = u & 1;
            if (n < ti.nn && ti.rt * TC_M + b * 64 < ti.F) {
                act_q8 *o = sc.act_mid + (int64_t)(ti.p0 + ti.n0 + n) * fmax_nb + ti.rt * 2 + b;
                act_quant_warp(M[n * TC_M + b * 64 + lane], M[n * TC_M + b * 64 + 32 + lane], o, lane);
            }
        }
        __syncthreads();   // U and M are operand buffers again
    }
    tmem_free(tmem, 2 * TC_N);
}

// --------------------------------------------------------------------------------------- down

struct DnSmem {
    uint8_t st[2][TC_M * SD_MAXNB * Q4_BLOCK + TC_N * SD_MAXNB * ACT_BLOCK];   // rows, then pairs
    uint8_t a[2][TC_M * 64];
    uint8_t b[2][TC_N * 64];
    float dx[2][TC_N];
    int c8[2][TC_N];
    float dw[2][TC_M];
    TileInfo ti[3];
    int pre[SG_MAXJOBS + 1];
    uint64_t full[2], mma;
    uint32_t tmem;
};
static_assert((TC_M * SD_MAXNB * Q4_BLOCK + TC_N * SD_MAXNB * ACT_BLOCK) % 16 == 0, "down slots 16-byte aligned");

// Issues tile i of this CTA (all nbF blocks of its 128 rows and 32 pairs) into slot i & 1.
// Rows go in groups of rg rows so that every copy is a multiple of 16 bytes.
__device__ __forceinline__ void dn_issue(DnSmem &s, const MoeShape &sh, const MoeScratch &sc, int i, int ntiles,
                                         int nbF, int rg, int fmax_nb) {
    const int t = blockIdx.x + i * gridDim.x;
    if (t >= ntiles) return;
    const TileInfo &ti = s.ti[i % 3];
    const int tid = threadIdx.x, slot = i & 1;
    uint64_t *bar = &s.full[slot];
    const int rb = nbF * Q4_BLOCK, pitch = nbF * ACT_BLOCK;
    const int ngroups = TC_M / rg;
    const int rows = ti.w0 ? max(0, min(TC_M, sh.D - ti.rt * TC_M)) : 0;
    fence_proxy_async();
    if (tid < ngroups && tid * rg < rows)
        bulk_g2s(s.st[slot] + tid * rg * rb, ti.w0 + (int64_t)(ti.rt * TC_M + tid * rg) * rb, (uint32_t)(rg * rb), bar);
    const int pn = tid - ngroups;
    if (pn >= 0 && pn < ti.nn)
        bulk_g2s(s.st[slot] + TC_M * rb + pn * pitch,
                 reinterpret_cast<const uint8_t *>(sc.act_mid + (int64_t)(ti.p0 + ti.n0 + pn) * fmax_nb), (uint32_t)pitch,
                 bar);
    if (tid == 0) mbar_expect_tx(bar, (uint32_t)(rows * rb + ti.nn * pitch));
}

__device__ __forceinline__ void dn_fill_info(DnSmem &s, const MoeShape &sh, const MoeLayerDev &L,
                                             const MoeScratch &sc, int nu, int njobs, int ntiles, int i) {
    const int t = blockIdx.x + i * gridDim.x;
    if (t >= ntiles) return;
    if ((threadIdx.x & 31) == 0) decode_tile(sh, L, sc, nu, njobs, s.pre, t, true, s.ti[i % 3]);
}

template <int JM>
__device__ __forceinline__ void dn_unpack(DnSmem &s, const TileInfo &ti, int slot, int buf, int j, int nbF, int D,
                                          int tid) {
    const int rb = nbF * Q4_BLOCK;
    if (tid < TC_M) {
        uint32_t w[16];
        float dw = 0.0f;
        if (ti.w0 && ti.rt * TC_M + tid < D) {
            dw = f16_to_f32(row_q4_block<JM>(s.st[slot] + tid * rb, j, w));
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++) w[i] = 0;
        }
        store_operand_row(s.a[buf], tid, w);
        s.dw[buf][tid] = dw;
    } else {
        unpack_act(s.st[slot] + TC_M * rb, nbF * ACT_BLOCK, j, ti.nn, s.b[buf], s.dx[buf], s.c8[buf], tid - TC_M, TC_M);
    }
}

__device__ __forceinline__ void dn_unpack_j(DnSmem &s, const TileInfo &ti, int slot, int buf, int j, int nbF, int D,
                                            int tid) {
    switch (j & 3) {
    case 0: dn_unpack<0>(s, ti, slot, buf, j, nbF, D, tid); break;
    case 1: dn_unpack<1>(s, ti, slot, buf, j, nbF, D, tid); break;
    case 2: dn_unpack<2>(s, ti, slot, buf, j, nbF, D, tid); break;
    default: dn_unpack<3>(s, ti, slot, buf, j, nbF, D, tid); break;
    }
}

__device__ __forceinline__ void dn_mma(DnSmem &s, uint32_t tmem, uint32_t idesc, int buf) {
    const uint32_t sa = smem_u32(s.a[buf]), sb = smem_u32(s.b[buf]);
#pragma unroll
    for (int k = 0; k < 2; k++) umma_i8(tmem, umma_desc(sa + 256 * k), umma_desc(sb + 256 * k), idesc, k > 0);
    umma_commit(&s.mma);
}

__global__ void __launch_bounds__(SG_THREADS, 1) k_moe_down_tcs(MoeShape sh, MoeLayerDev L, MoeScratch sc,
                                                                 int fmax_nb, int nbF, int rg) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    DnSmem &s = *reinterpret_cast<DnSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int nu = routed_jobs(sh, sc), njobs = nu + (L.Fs > 0 ? 1 : 0);
    const int ntiles = tile_prefix(sh, L, sc, nu, njobs, true, s.pre);
    if ((int)blockIdx.x >= ntiles) return;
    const int mytiles = (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

    if (tid == 0) {
        mbar_init(&s.full[0], 1);
        mbar_init(&s.full[1], 1);
        mbar_init(&s.mma, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        dn_fill_info(s, sh, L, sc, nu, njobs, ntiles, 0);
        dn_fill_info(s, sh, L, sc, nu, njobs, ntiles, 1);
    }
    const uint32_t tmem = tmem_alloc(&s.tmem, TC_N);
    dn_issue(s, sh, sc, 0, ntiles, nbF, rg, fmax_nb);
    dn_issue(s, sh, sc, 1, ntiles, nbF, rg, fmax_nb);
    const uint32_t idesc = umma_idesc_i8(false);
    const int h = warp >> 2, r = (warp & 3) * 32 + (tid & 31);
    uint32_t mma_phase = 0;

    for (int i = 0; i < mytiles; i++) {
        const TileInfo &ti = s.ti[i % 3];
        const int slot = i & 1;
        if (warp == 1) dn_fill_info(s, sh, L, sc, nu, njobs, ntiles, i + 2);
        float acc[TC_N / 2];
#pragma unroll
        for (int n = 0; n < TC_N / 2; n++) acc[n] = 0.0f;
        mbar_wait(&s.full[slot], (uint32_t)((i >> 1) & 1), sc.err);
        dn_unpack<0>(s, ti, slot, 0, 0, nbF, sh.D, tid);
        cta_sync_tc();
        if (tid == 0) dn_mma(s, tmem, idesc, 0);
        for (int g0 = 0; g0 < nbF; g0 += 4) {
#pragma unroll
            for (int jm = 0; jm < 4; jm++) {
                const int g = g0 + jm;
                if (g + 1 < nbF) dn_unpack_j(s, ti, slot, (g + 1) & 1, g + 1, nbF, sh.D, tid);
                mbar_wait(&s.mma, mma_phase, sc.err);
                mma_phase ^= 1;
                tc_fence_after();
                {
                    uint32_t v[16];
                    tmem_ld16(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(h * 16), v);
                    chain_q4<TC_N / 2>(v, s.dw[g & 1][r], s.dx[g & 1], s.c8[g & 1], h * 16, acc);
                }
                cta_sync_tc();
                if (g == nbF - 2) dn_issue(s, sh, sc, i + 2, ntiles, nbF, rg, fmax_nb);   // slot is read
                if (g + 1 < nbF && tid == 0) dn_mma(s, tmem, idesc, (g + 1) & 1);
            }
        }
        const int row = ti.rt * TC_M + r;
        if (ti.w0 && row < sh.D) {   // canonical outputs: Y [pair][D] (routed) or S [token][D] (shared)
#pragma unroll
            for (int k = 0; k < TC_N / 2; k++) {
                const int n = h * 16 + k;
                if (n < ti.nn) {
                    float *out = ti.shared ? sc.S + (int64_t)(ti.n0 + n) * sh.D
                                           : sc.Y + (int64_t)(ti.p0 + ti.n0 + n) * sh.D;
                    out[row] = canon(acc[k]);
                }
            }
        }
        __syncthreads();   // the next tile's warp 1 rewrites the info slot this epilogue read
    }
    tmem_free(tmem, TC_N);
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

// The staged kernels take Q4 experts (and a Q4 shared expert, if any) with D a multiple of 512 for
// gate/up (8-block stages) and, for down, F (and Fs) of 4, 8 or 12 blocks (whole rows in a slot).
static bool staged_gateup_ok(const MoeShape &sh, const MoeLayerDev &L) {
    const int64_t rbD = (int64_t)(sh.D / QK) * Q4_BLOCK;
    if (L.expert_dtype != Q4 || (L.Fs > 0 && L.sh_dtype != Q4)) return false;
    if ((sh.D / QK) % SG_BLK || sh.E + 1 > SG_MAXJOBS || L.off_up % 16) return false;
    if (L.Fs > 0 && ((reinterpret_cast<uintptr_t>(L.sh_gate) | reinterpret_cast<uintptr_t>(L.sh_up)) & 15)) return false;
    return rbD % 16 == 0;
}

static bool staged_down_ok(const MoeShape &sh, const MoeLayerDev &L, int fmax_nb) {
    if (L.expert_dtype != Q4 || (L.Fs > 0 && L.sh_dtype != Q4)) return false;
    const int nbF = sh.F / QK;
    if (L.Fs > 0 && L.Fs != sh.F) return false;   // one row width per launch (whole rows per slot)
    if (nbF % 4 || nbF > SD_MAXNB || fmax_nb % 2 || sh.E + 1 > SG_MAXJOBS || L.off_down % 16) return false;
    if (L.Fs > 0 && (reinterpret_cast<uintptr_t>(L.sh_down) & 15)) return false;
    return true;
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

cudaError_t init_tc_attributes() {
    cudaError_t e = cudaFuncSetAttribute(k_moe_gateup_tcs, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(GuSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_moe_down_tcs, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(DnSmem));
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
        if (staged_on() && staged_gateup_ok(sh, L)) {
            k_moe_gateup_tcs<<<sm_count(), SG_THREADS, sizeof(GuSmem), s>>>(sh, L, sc, fmax_nb);
        } else {
            const dim3 grid((unsigned)((std::max(sh.F, L.Fs) + TC_M - 1) / TC_M), (unsigned)maxjobs,
                            (unsigned)((maxn + TC_N - 1) / TC_N));
            k_moe_gateup_tc<<<grid, TC_THREADS, 0, s>>>(sh, L, sc, fmax_nb);
        }
    }
    if (which & 2) {
        if (staged_on() && staged_down_ok(sh, L, fmax_nb)) {
            const int nbF = sh.F / QK;
            int rg = 1;
            while ((rg * nbF * Q4_BLOCK) % 16) rg <<= 1;
            k_moe_down_tcs<<<sm_count(), SG_THREADS, sizeof(DnSmem), s>>>(sh, L, sc, fmax_nb, nbF, rg);
        } else {
            const dim3 grid((unsigned)((sh.D + TC_M - 1) / TC_M), (unsigned)maxjobs, (unsigned)((maxn + TC_N - 1) / TC_N));
            k_moe_down_tc<<<grid, TC_THREADS, 0, s>>>(sh, L, sc, fmax_nb);
        }
    }
    return cudaGetLastError();
}

}  // namespace hx
