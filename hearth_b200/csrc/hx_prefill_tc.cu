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

}  // namespace

cudaError_t launch_moe_experts_tc(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, int which,
                                  cudaStream_t s) {
    const int T = sh.T, K = sh.route.K, E = sh.route.E;
    const int fmax_nb = std::max(sh.F, L.Fs) / QK;
    const int maxjobs = std::min(E, T * K) + (L.Fs > 0 ? 1 : 0);
    const int maxn = std::max(T, 1);   // a bucket holds at most T pairs (one per token)
    const dim3 grid_z_rows((unsigned)((std::max(sh.F, L.Fs) + TC_M - 1) / TC_M), (unsigned)maxjobs,
                           (unsigned)((maxn + TC_N - 1) / TC_N));
    if (which & 1) k_moe_gateup_tc<<<grid_z_rows, TC_THREADS, 0, s>>>(sh, L, sc, fmax_nb);
    if (which & 2) {
        const dim3 grid((unsigned)((sh.D + TC_M - 1) / TC_M), (unsigned)maxjobs, (unsigned)((maxn + TC_N - 1) / TC_N));
        k_moe_down_tc<<<grid, TC_THREADS, 0, s>>>(sh, L, sc, fmax_nb);
    }
    return cudaGetLastError();
}

}  // namespace hx
