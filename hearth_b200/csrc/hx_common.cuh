// hx_common.cuh — formats and canonical device numerics of the B200 MoE backend.
//
// The reference defines one canonical order of float operations for every kernel
// (pierce-lonergan/hearth docs/NUMERICS.md §1-§5). Everything here is written with
// explicit round-to-nearest intrinsics (__fadd_rn, __fmul_rn, __fdiv_rn, __fsqrt_rn)
// and the library is built with -fmad=false, so no multiply-add is ever contracted.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

#ifndef HX_HD
#define HX_HD __host__ __device__
#endif

namespace hx {

// dtypes (engine/include/hearth.h:40-43)
enum : int { F32 = 0, F16 = 1, BF16 = 2, Q8 = 3, Q4 = 4 };
enum : int { SCORE_SOFTMAX = 0, SCORE_SIGMOID = 1 };

constexpr int QK = 64;            // weights and activations are quantized in blocks of 64
constexpr int Q4_BLOCK = 34;      // u16 f16 scale + 32 bytes of nibbles (FORMAT §6)
constexpr int Q8_BLOCK = 66;      // u16 f16 scale + 64 int8
constexpr int ACT_BLOCK = 72;     // {f32 d; i32 sum; i8 q[64]} (engine/src/hx_quant.h:24)
constexpr uint32_t CANON_NAN = 0x7fc00000u;

struct alignas(4) act_q8 {
    float d;
    int32_t sum;
    int8_t q[64];
};
static_assert(sizeof(act_q8) == ACT_BLOCK, "activation block is 72 bytes");

HX_HD inline int64_t row_bytes(int dtype, int64_t n) {
    if (n <= 0 || n > (int64_t(1) << 40)) return 0;
    switch (dtype) {
    case F32: return n * 4;
    case F16: case BF16: return n * 2;
    case Q8: return n % QK ? 0 : n / QK * Q8_BLOCK;
    case Q4: return n % QK ? 0 : n / QK * Q4_BLOCK;
    default: return 0;
    }
}

HX_HD inline bool is_quant(int dtype) { return dtype == Q8 || dtype == Q4; }

// FORMAT §5 slab: gate [F,D] at 0, up [F,D] and down [D,F] at 64-byte aligned offsets.
struct slab_layout {
    int64_t off_up, off_down, end, nbytes;
};
HX_HD inline slab_layout make_slab_layout(int dtype, int64_t D, int64_t F) {
    slab_layout s;
    const int64_t g = F * row_bytes(dtype, D);
    s.off_up = (g + 63) / 64 * 64;
    s.off_down = (s.off_up + g + 63) / 64 * 64;
    s.end = s.off_down + D * row_bytes(dtype, F);
    s.nbytes = (s.end + 4095) / 4096 * 4096;
    return s;
}

// ------------------------------------------------------------------ canonical scalar ops

#ifdef __CUDACC__

// f16 -> f32 exactly as the reference decodes block scales (engine/src/quant.c:17-35):
// NaNs come back quiet with their payload, subnormals are m * 2^-24.
__device__ __forceinline__ float f16_to_f32(uint32_t h) {
    const uint32_t s = (h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0x1fu) return __uint_as_float(s | 0x7f800000u | (m << 13) | (m ? 0x00400000u : 0u));
    if (e) return __uint_as_float(s | ((e + 112u) << 23) | (m << 13));
    if (!m) return __uint_as_float(s);
    return __uint_as_float(s | __float_as_uint(__fmul_rn(__uint2float_rn(m), 5.9604644775390625e-8f)));
}

__device__ __forceinline__ float bf16_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

__device__ __forceinline__ float canon(float v) { return v != v ? __uint_as_float(CANON_NAN) : v; }
#endif  // __CUDACC__

// expf with the results of the host C library the reference calls (glibc 2.39, x86-64, its FMA
// variant selected at run time). Restated from the published algorithm of that implementation
// (ARM optimized-routines expf, Szabolcs Nagy 2017, as shipped in glibc since 2.27): with N = 32,
// z = x * N/ln2 = k + r, exp(x) = 2^(k/N) * p(r) where 2^(k/N) comes from a 32-entry table of
// 2^(i/32) (each entry is the double nearest 2^(i/32) with i << 47 subtracted, so that adding
// k << 47 applies the exponent) and p is a cubic in r, all in double precision, rounded once to
// float. The table is derived from the mathematics; the host test suite checks this function
// against the host expf on all 2^32 inputs and recomputes the table.
#define HX_EXP2_TAB                                                                                \
    {0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,  \
     0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,  \
     0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,  \
     0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,  \
     0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,  \
     0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,  \
     0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,  \
     0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull}

#ifdef __CUDACC__
// global memory, read through the L1 / read-only path: the 32 lanes of a warp index the table
// independently, which the constant cache would serialise
static __device__ const uint64_t kExp2TabDev[32] = HX_EXP2_TAB;
#endif
static const uint64_t kExp2TabHost[32] = HX_EXP2_TAB;

#if defined(__CUDA_ARCH__)
#define HX_DFMA(a, b, c) __fma_rn((a), (b), (c))
#define HX_DMUL(a, b) __dmul_rn((a), (b))
#define HX_DSUB(a, b) __dsub_rn((a), (b))
#define HX_D2F(a) __double2float_rn(a)
#define HX_EXP2(i) __ldg(&kExp2TabDev[i])
#define HX_F2U(f) __float_as_uint(f)
#define HX_U2F(u) __uint_as_float(u)
#define HX_D2U(d) ((uint64_t)__double_as_longlong(d))
#define HX_U2D(u) __longlong_as_double((long long)(u))
#else
#define HX_DFMA(a, b, c) std::fma((a), (b), (c))
#define HX_DMUL(a, b) ((a) * (b))
#define HX_DSUB(a, b) ((a) - (b))
#define HX_D2F(a) ((float)(a))
#define HX_EXP2(i) kExp2TabHost[i]
#define HX_F2U(f) hx_bits_f(f)
#define HX_U2F(u) hx_f_bits(u)
#define HX_D2U(d) hx_bits_d(d)
#define HX_U2D(u) hx_d_bits(u)
inline uint32_t hx_bits_f(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float hx_f_bits(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint64_t hx_bits_d(double d) { uint64_t u; std::memcpy(&u, &d, 8); return u; }
inline double hx_d_bits(uint64_t u) { double d; std::memcpy(&d, &u, 8); return d; }
#endif

HX_HD inline float host_expf(float x) {
    const uint32_t ux = HX_F2U(x);
    const uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) {                     // |x| >= 88, or inf / NaN
        if (ux == 0xff800000u) return 0.0f;     // exp(-inf)
        if (abstop >= 0x7f8u) return x + x;     // +inf, NaN
        if (x > 0x1.62e42ep6f) return HX_U2F(0x7f800000u);
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
    const double c1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double xd = (double)x;
    double kd = HX_DFMA(inv_ln2_n, xd, shift);
    const uint64_t ki = HX_D2U(kd);
    kd = HX_DSUB(kd, shift);
    const double r = HX_DFMA(inv_ln2_n, xd, -kd);
    const uint64_t t = HX_EXP2(ki & 31u) + (ki << 47);
    const double s = HX_U2D(t);
    const double z = HX_DFMA(c0, r, c1);
    const double r2 = HX_DMUL(r, r);
    double y = HX_DFMA(c2, r, 1.0);
    y = HX_DFMA(z, r2, y);
    y = HX_DMUL(y, s);
    return HX_D2F(y);
}

#ifdef __CUDACC__
// NUMERICS §4: sigmoid = 1/(1+expf(-x)); silu(g)*u = (g/(1+expf(-g)))*u.
__device__ __forceinline__ float sigmoid_c(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, host_expf(-x)));
}
__device__ __forceinline__ float swiglu_c(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, host_expf(-g))), u);
}

// engine/src/model.c:221-226: a ranks before b (larger first, NaN last, ties to the lower index).
__device__ __forceinline__ bool ranks_before(float va, int ia, float vb, int ib) {
    const bool na = va != va, nb = vb != vb;
    if (na || nb) return na == nb ? ia < ib : nb;
    if (va != vb) return va > vb;
    return ia < ib;
}

// The 8/4/2/1 lane tree of NUMERICS §1 on a 16-lane group: lane j of the group holds L[j];
// the result lands in the group's first lane. (a + b == b + a exactly in IEEE arithmetic.)
__device__ __forceinline__ float tree16(float v, unsigned mask) {
#pragma unroll
    for (int s = 8; s >= 1; s >>= 1) v = __fadd_rn(v, __shfl_down_sync(mask, v, s, 16));
    return v;
}

// One 64-block integer dot: Q4 nibbles (stored q+8) against activation q, exact:
// sum (nib-8)*xq = sum nib*xq - 8*sum(xq) (NUMERICS §3 note).
__device__ __forceinline__ int q4_isum(const uint32_t nib[8], const int32_t aq[16], int32_t asum) {
    int a0 = 0, a1 = 0;   // two independent chains (integer sums: any order is exact)
#pragma unroll
    for (int k = 0; k < 8; k++) {
        a0 = __dp4a((int)(nib[k] & 0x0f0f0f0fu), aq[k], a0);
        a1 = __dp4a((int)((nib[k] >> 4) & 0x0f0f0f0fu), aq[8 + k], a1);
    }
    return a0 + a1 - 8 * asum;
}

__device__ __forceinline__ int q8_isum(const uint32_t w[16], const int32_t aq[16]) {
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
        a0 = __dp4a((int)w[k], aq[k], a0);
        a1 = __dp4a((int)w[k + 1], aq[k + 1], a1);
        a2 = __dp4a((int)w[k + 2], aq[k + 2], a2);
        a3 = __dp4a((int)w[k + 3], aq[k + 3], a3);
    }
    return (a0 + a1) + (a2 + a3);
}

// Loads a Q4 block that starts at a 2-byte aligned byte address with aligned loads that stay
// inside the block's 34 bytes: returns the f16 scale bits and the 8 nibble words. Works for
// shared and global pointers.
__device__ __forceinline__ uint32_t load_q4_block(const uint8_t *blk, uint32_t nib[8]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
    if (a & 2) {   // scale is the high half of the word before; the nibbles are word aligned
        const uint32_t *w = reinterpret_cast<const uint32_t *>(a + 2);
#pragma unroll
        for (int k = 0; k < 8; k++) nib[k] = w[k];
        return *reinterpret_cast<const uint16_t *>(blk);
    }
    // scale is the low half of w[0]; nibble word k straddles w[k] and w[k+1], the last one ends
    // with the block's final half word
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a);
    uint32_t prev = w[0];
    const uint32_t scale = prev & 0xffffu;
#pragma unroll
    for (int k = 0; k < 7; k++) {
        const uint32_t nx = w[k + 1];
        nib[k] = __funnelshift_r(prev, nx, 16);
        prev = nx;
    }
    nib[7] = __funnelshift_r(prev, (uint32_t)*reinterpret_cast<const uint16_t *>(blk + 32), 16);
    return scale;
}

__device__ __forceinline__ uint32_t load_q8_block(const uint8_t *blk, uint32_t q[16]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
    if (a & 2) {
        const uint32_t *w = reinterpret_cast<const uint32_t *>(a + 2);
#pragma unroll
        for (int k = 0; k < 16; k++) q[k] = w[k];
        return *reinterpret_cast<const uint16_t *>(blk);
    }
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a);
    uint32_t prev = w[0];
    const uint32_t scale = prev & 0xffffu;
#pragma unroll
    for (int k = 0; k < 15; k++) {
        const uint32_t nx = w[k + 1];
        q[k] = __funnelshift_r(prev, nx, 16);
        prev = nx;
    }
    q[15] = __funnelshift_r(prev, (uint32_t)*reinterpret_cast<const uint16_t *>(blk + 64), 16);
    return scale;
}

// Shared-memory block loaders: one aligned word per 4 bytes from the word that holds the block's
// first byte, the block bytes picked out with byte permutes (no branch on the block's 2-byte
// alignment). When the block starts on a word boundary the last word read extends 2 bytes past the
// block, so these are only for tiles in shared memory with readable bytes after them.
__device__ __forceinline__ uint32_t load_q4_block_pad(const uint8_t *blk, uint32_t nib[8]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
    const uint32_t o = (uint32_t)(a & 2u);
    const uint32_t sel = o ? 0x7654u : 0x5432u;
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    uint32_t v[9];
#pragma unroll
    for (int i = 0; i < 9; i++) v[i] = w[i];
#pragma unroll
    for (int k = 0; k < 8; k++) nib[k] = __byte_perm(v[k], v[k + 1], sel);
    return (v[0] >> (o * 8u)) & 0xffffu;
}

__device__ __forceinline__ uint32_t load_q8_block_pad(const uint8_t *blk, uint32_t q[16]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
    const uint32_t o = (uint32_t)(a & 2u);
    const uint32_t sel = o ? 0x7654u : 0x5432u;
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    uint32_t v[17];
#pragma unroll
    for (int i = 0; i < 17; i++) v[i] = w[i];
#pragma unroll
    for (int k = 0; k < 16; k++) q[k] = __byte_perm(v[k], v[k + 1], sel);
    return (v[0] >> (o * 8u)) & 0xffffu;
}

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// q4_isum with the high nibbles left in place: (nib & 0xf0f0f0f0) . aq = 16 * sum(hi * aq), an
// exact multiple of 16, so an arithmetic shift recovers the sum (one fewer operation per word).
__device__ __forceinline__ int q4_isum_hi(const uint32_t nib[8], const int32_t aq[16], int32_t asum) {
    int a0 = 0, a1 = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        a0 = __dp4a((int)(nib[k] & 0x0f0f0f0fu), aq[k], a0);
        a1 = dp4a_us(nib[k] & 0xf0f0f0f0u, aq[8 + k], a1);
    }
    return a0 + (a1 >> 4) - 8 * asum;
}

// Hardware f16 -> f32: exact for every finite value and infinity; a NaN keeps NaN-ness but not
// necessarily its payload, so this is for products whose sums are canonicalised (canon()) before
// they are stored, never for dequantized values.
__device__ __forceinline__ float f16_to_f32_hw(uint32_t h) {
    float f;
    asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"((unsigned short)h));
    return f;
}

// The product term of NUMERICS §3 for one block: (float)isum * (dw * dx), rounded per op.
__device__ __forceinline__ float block_term(int isum, uint32_t dw_bits, float dx) {
    return __fmul_rn(__int2float_rn(isum), __fmul_rn(f16_to_f32(dw_bits), dx));
}

// Activation block of one token, read as words (q first, then d and sum).
struct act_regs {
    int32_t q[16];
    float d;
    int32_t sum;
};
__device__ __forceinline__ void load_act(const act_q8 *a, act_regs &r) {
    const uint2 *p = reinterpret_cast<const uint2 *>(a);   // 72-byte blocks are 8-byte aligned
    const uint2 h = p[0];
    r.d = __uint_as_float(h.x);
    r.sum = (int32_t)h.y;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint2 v = p[1 + k];
        r.q[2 * k] = (int32_t)v.x;
        r.q[2 * k + 1] = (int32_t)v.y;
    }
}

#endif  // __CUDACC__

}  // namespace hx
