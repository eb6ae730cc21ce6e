// hx_kernels.cu — hand-written sm_100a kernels of the quantized MoE expert path.
//
// Every float result follows the canonical operation order of the reference
// (pierce-lonergan/hearth docs/NUMERICS.md): integer block dots are exact and may be computed in
// any order; every float sum runs in the reference's order with one rounding per operation.
#include "hx_device.cuh"
#include "hx_kernels.h"
#include "hx_route.cuh"
#include "hx_moe_job.cuh"

#include <algorithm>
#include <cstdlib>

namespace hx {

// =============================================================================================
// Activation quantization (NUMERICS §2, engine/src/quant.c:325-348): one warp per 64-block.
// =============================================================================================

__global__ void k_act_quantize(const float *__restrict__ x, int64_t ldx, act_q8 *__restrict__ out, int nb,
                               int T) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= (int64_t)T * nb) return;
    const int64_t t = w / nb, b = w - t * nb;
    const float *xb = x + t * ldx + b * QK;
    act_quant_warp(xb[lane], xb[lane + 32], out + w, lane);
}

cudaError_t launch_act_quantize(const float *x, int64_t ldx, act_q8 *out, int64_t n, int T, cudaStream_t s) {
    const int nb = (int)(n / QK);
    const int64_t warps = (int64_t)nb * T;
    if (warps == 0) return cudaSuccess;
    k_act_quantize<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(x, ldx, out, nb, T);
    return cudaGetLastError();
}

// =============================================================================================
// Generic row-range matmul (the hearth_matmul boundary, engine/src/quant.c:352-427, 574-600).
// =============================================================================================

// Quantized weights: one warp per row, up to 16 tokens per pass, block terms chained per
// (row, token) in block order.
// Epilogue of the row-range matmuls: Y = y, or with a residual target h: h = h + rs * y (the
// h_i + (rs * a_i) of engine/src/model.c:1194-1198 on the matmul's canonical output).
__device__ __forceinline__ void mm_store(float *Y, float *resid, float rs, int64_t i, float y) {
    if (resid) resid[i] = __fadd_rn(resid[i], __fmul_rn(rs, y));
    else Y[i] = y;
}

template <int DT>
__global__ void __launch_bounds__(256) k_matmul_q(const uint8_t *__restrict__ W, int nb, int64_t rb,
                                                  const act_q8 *__restrict__ act, int T, float *__restrict__ Y,
                                                  int64_t ldy, int64_t r0, int64_t r1, float *resid, float rs) {
    __shared__ float Pbuf[8][16 * 33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = r0 + (int64_t)blockIdx.x * 8 + warp;
    if (r >= r1) return;
    float *P = Pbuf[warp];
    constexpr int BS = DT == Q4 ? Q4_BLOCK : Q8_BLOCK;
    const uint8_t *row = W + r * rb;
    for (int t0 = blockIdx.y * 16; t0 < T; t0 += gridDim.y * 16) {
        const int nt = min(16, T - t0);
        float acc = 0.0f;
        for (int g0 = 0; g0 < nb; g0 += 32) {
            const int gn = min(32, nb - g0);
            if (lane < gn) {
                const int g = g0 + lane;
                const uint8_t *blk = row + (int64_t)g * BS;
                uint32_t wq[16];
                float dw;
                if constexpr (DT == Q4) dw = f16_to_f32(load_q4_block(blk, wq));
                else dw = f16_to_f32(load_q8_block(blk, wq));
                for (int i = 0; i < nt; i++) {
                    act_regs ar;
                    load_act(act + (int64_t)(t0 + i) * nb + g, ar);
                    int isum;
                    if constexpr (DT == Q4) isum = q4_isum(wq, ar.q, ar.sum);
                    else isum = q8_isum(wq, ar.q);
                    P[i * 33 + lane] = __fmul_rn(__int2float_rn(isum), __fmul_rn(dw, ar.d));
                }
            }
            __syncwarp();
            if (lane < nt)
                for (int g = 0; g < gn; g++) acc = __fadd_rn(acc, P[lane * 33 + g]);
            __syncwarp();
        }
        if (lane < nt) mm_store(Y, resid, rs, (int64_t)(t0 + lane) * ldy + r, canon(acc));
    }
}

// Quantized weights at few tokens (decode): every warp streams its own units of U consecutive rows
// (one 1-D bulk copy each) through two shared-memory slots of its own, so all warps of every SM keep
// copies in flight whatever the row width (16 slots of up to ~12 KB per SM, what the HBM stream
// needs) and no warp waits for another. Warp w of CTA b takes units w + 8b, then every 8*gridDim
// further. A unit runs through the single-token row loop (lane = block, the activation block in
// registers across the unit's rows, lanes 0..U-1 the rows' chains in block order: NUMERICS §3) once
// per token. Rows must be a multiple of 16 bytes and the matrix 16-byte aligned (every Q4/Q8 matrix
// with n_cols a multiple of 512, in cudaMalloc memory).
constexpr int GV_WARPS = 8;
constexpr int GV_SLOTS = 2;
constexpr int GV_TMAX = 4;

template <int DT>
__global__ void __launch_bounds__(GV_WARPS * 32) k_gemv_staged(const uint8_t *__restrict__ W, int64_t rows, int nb,
                                                               int64_t rb, int U, const act_q8 *__restrict__ act,
                                                               int T, float *__restrict__ Y, int64_t ldy, float *resid,
                                                               float rs, const float *__restrict__ nh,
                                                               const float *__restrict__ nw, float eps) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * GV_SLOTS;
    const int64_t slot = (int64_t)U * rb + 16;   // the padded block loads read up to 2 bytes past a row
    uint8_t *slots = smem + 128 + (size_t)warp * GV_SLOTS * slot;
    act_q8 *acts = reinterpret_cast<act_q8 *>(smem + 128 + (size_t)GV_WARPS * GV_SLOTS * slot);
    float *fbase = reinterpret_cast<float *>(acts + (int64_t)T * nb);
    float *P = fbase + warp * ROWS_1TOK * 33;
    float *outs = fbase + GV_WARPS * ROWS_1TOK * 33 + warp * GV_TMAX * ROWS_1TOK;
    float *xs = fbase + GV_WARPS * ROWS_1TOK * 33 + GV_WARPS * GV_TMAX * ROWS_1TOK;   // nh: x = rmsnorm(nh)
    const int64_t units = (rows + U - 1) / U;
    const int64_t gw = (int64_t)blockIdx.x * GV_WARPS + warp, nwarps = (int64_t)gridDim.x * GV_WARPS;
    const int64_t mine = gw < units ? (units - 1 - gw) / nwarps + 1 : 0;
    auto issue = [&](int64_t k) {
        const int64_t r0 = (gw + k * nwarps) * U;
        const int64_t nr = min((int64_t)U, rows - r0);
        const int st = (int)(k % GV_SLOTS);
        mbar_expect_tx(&bars[st], (uint32_t)(nr * rb));
        bulk_g2s(slots + st * slot, W + r0 * rb, (uint32_t)(nr * rb), &bars[st]);
    };
    pdl_trigger();
    if (lane == 0) {   // the weights stream in while the previous kernel may still run
        for (int st = 0; st < GV_SLOTS; st++) mbar_init(&bars[st], 1);
        fence_mbar_init();
        for (int64_t k = 0; k < min((int64_t)GV_SLOTS, mine); k++) issue(k);
    }
    pdl_wait();   // the activations, nh and the residual are the previous kernels' outputs
    if (nh) {   // one token: x = rmsnorm(nh, nw) (NUMERICS §4) and its activation blocks, formed here
        __shared__ float rsh;
        const int n = nb * QK;
        for (int i = tid; i < n; i += blockDim.x) xs[i] = nh[i];
        __syncthreads();
        if (tid < 16) {
            float L = 0.0f;
            for (int i = tid; i < n; i += 16) L = __fadd_rn(L, __fmul_rn(xs[i], xs[i]));
            L = tree16(L, 0xffffu);
            if (tid == 0) rsh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(L, (float)n), eps)));
        }
        __syncthreads();
        const float r = rsh;
        for (int i = tid; i < n; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], r), nw[i]);
        __syncthreads();
        for (int b = warp; b < nb; b += GV_WARPS) act_quant_warp(xs[b * QK + lane], xs[b * QK + lane + 32], acts + b, lane);
    } else {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(act);
        uint32_t *dst = reinterpret_cast<uint32_t *>(acts);
        for (int64_t i = tid; i < (int64_t)T * nb * (ACT_BLOCK / 4); i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    for (int64_t k = 0; k < mine; k++) {
        const int st = (int)(k % GV_SLOTS);
        if (!mbar_wait(&bars[st], (uint32_t)((k / GV_SLOTS) & 1), nullptr)) break;
        const int64_t r0 = (gw + k * nwarps) * U;
        const int nr = (int)min((int64_t)U, rows - r0);
        const uint8_t *tile = slots + st * slot;
        for (int i = 0; i < T; i++)   // the unit stays in shared memory for every token
            warp_rows_1tok<DT>(tile, rb, nb, nr, acts + (int64_t)i * nb, P, outs + i * ROWS_1TOK);
        if (lane < nr)
            for (int i = 0; i < T; i++) mm_store(Y, resid, rs, (int64_t)i * ldy + r0 + lane, outs[i * ROWS_1TOK + lane]);
        __syncwarp();
        if (lane == 0 && k + GV_SLOTS < mine) {
            fence_proxy_async();
            issue(k + GV_SLOTS);
        }
    }
}

// The staged kernel's rows per unit and shared memory for a launch (norm: the rmsnorm prologue's x),
// or 0 when it does not apply.
static int gemv_rows_per_stage(int dtype, const void *W, int64_t n_cols, int64_t rows, int T, bool norm,
                               size_t *smem) {
    if (!is_quant(dtype) || T > GV_TMAX || rows < 1 || (reinterpret_cast<uintptr_t>(W) & 15)) return 0;
    const int64_t rb = row_bytes(dtype, n_cols);
    const int64_t nb = n_cols / QK;
    if (rb % 16) return 0;
    const size_t fixed = 128 + (size_t)T * nb * ACT_BLOCK +
                         sizeof(float) * ((size_t)GV_WARPS * ROWS_1TOK * 33 + (size_t)GV_WARPS * GV_TMAX * ROWS_1TOK) +
                         (norm ? sizeof(float) * (size_t)n_cols : 0);
    if (fixed + (size_t)GV_WARPS * GV_SLOTS * (rb + 16) > 220 * 1024) return 0;
    const size_t per_slot = (220 * 1024 - fixed) / ((size_t)GV_WARPS * GV_SLOTS) - 16;
    const int U = (int)std::min<int64_t>(ROWS_1TOK, (int64_t)(per_slot / (size_t)rb));
    *smem = fixed + (size_t)GV_WARPS * GV_SLOTS * ((size_t)U * rb + 16);
    return U;
}

// Float weights: NUMERICS §1 dot16, one 16-lane group per (row, token).
template <int DT>
__device__ __forceinline__ float load_wf(const uint8_t *row, int64_t i) {
    if constexpr (DT == F32) return reinterpret_cast<const float *>(row)[i];
    else if constexpr (DT == F16) return f16_to_f32(reinterpret_cast<const uint16_t *>(row)[i]);
    else return bf16_to_f32(reinterpret_cast<const uint16_t *>(row)[i]);
}

template <int DT>
__device__ __forceinline__ float dot16_group(const uint8_t *row, const float *x, int64_t n, int j) {
    float L = 0.0f;
    for (int64_t i = j; i < n; i += 16) L = __fadd_rn(L, __fmul_rn(load_wf<DT>(row, i), x[i]));
    return L;
}

template <int DT>
__global__ void __launch_bounds__(256) k_matmul_f(const uint8_t *__restrict__ W, int64_t n, int64_t rb,
                                                  const float *__restrict__ X, int T, float *__restrict__ Y,
                                                  int64_t ldy, int64_t r0, int64_t r1, float *resid, float rs) {
    const int grp = threadIdx.x >> 4, j = threadIdx.x & 15;
    const int64_t item = (int64_t)blockIdx.x * 16 + grp;   // (row, token) item
    const int64_t rows = r1 - r0;
    const bool valid = item < rows * T;
    const int64_t r = valid ? r0 + item % rows : r0;
    const int64_t t = valid ? item / rows : 0;
    float L = valid ? dot16_group<DT>(W + r * rb, X + t * n, n, j) : 0.0f;
    const unsigned mask = 0xffffffffu;
    L = tree16(L, mask);
    if (valid && j == 0) mm_store(Y, resid, rs, t * ldy + r, canon(L));
}

// The staged GEMV's shared-memory attribute on the current device (once per device) and its SM count.
// Grid: enough CTAs for every unit's warp, at most one per SM.
static cudaError_t gemv_prepare(int dtype, int *sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr_set[64][2] = {};   // per device: the attribute belongs to the device's context
    const int di = dtype == Q4 ? 0 : 1;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev][di]) {
        cudaError_t e = dtype == Q4 ? cudaFuncSetAttribute(k_gemv_staged<Q4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                           220 * 1024)
                                    : cudaFuncSetAttribute(k_gemv_staged<Q8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                           220 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev][di] = true;
    }
    return cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
}

cudaError_t launch_gemv_norm(int dtype, const void *W, int64_t n_cols, int64_t rows, const float *h, const float *nw,
                             float eps, float *Y, float *resid, float rs, cudaStream_t s, bool early_weights) {
    size_t smem = 0;
    const int U = gemv_rows_per_stage(dtype, W, n_cols, rows, 1, true, &smem);
    if (U <= 0) return cudaErrorNotSupported;
    int sms = 148;
    cudaError_t e = gemv_prepare(dtype, &sms);
    if (e != cudaSuccess) return e;
    const int64_t rb = row_bytes(dtype, n_cols);
    const unsigned grid = (unsigned)std::min<int64_t>(((rows + U - 1) / U + GV_WARPS - 1) / GV_WARPS, sms);
    const int nb = (int)(n_cols / QK);
    const uint8_t *w = static_cast<const uint8_t *>(W);
    if (dtype == Q4)
        return launch_pdl(early_weights, k_gemv_staged<Q4>, grid, GV_WARPS * 32, smem, s, w, rows, nb, rb, U,
                          nullptr, 1, resid ? nullptr : Y, 0, resid, rs, h, nw, eps);
    return launch_pdl(early_weights, k_gemv_staged<Q8>, grid, GV_WARPS * 32, smem, s, w, rows, nb, rb, U, nullptr,
                      1, resid ? nullptr : Y, 0, resid, rs, h, nw, eps);
}

cudaError_t launch_matmul(int dtype, const void *W, int64_t n_cols, const void *act, int T, float *Y,
                          int64_t ldy, int64_t r0, int64_t r1, cudaStream_t s) {
    return launch_matmul_resid(dtype, W, n_cols, act, T, Y, ldy, r0, r1, nullptr, 0.0f, s);
}

cudaError_t launch_matmul_resid(int dtype, const void *W, int64_t n_cols, const void *act, int T, float *Y,
                                int64_t ldy, int64_t r0, int64_t r1, float *resid, float rs, cudaStream_t s,
                                bool early_weights) {
    const int64_t rows = r1 - r0;
    if (rows <= 0 || T <= 0) return cudaSuccess;
    const int64_t rb = row_bytes(dtype, n_cols);
    const uint8_t *w = static_cast<const uint8_t *>(W);
    size_t smem = 0;
    const int U = gemv_rows_per_stage(dtype, w + r0 * rb, n_cols, rows, T, false, &smem);
    if (U > 0) {   // few tokens: the rows stream through shared memory at the HBM rate
        int sms = 148;
        cudaError_t e = gemv_prepare(dtype, &sms);
        if (e != cudaSuccess) return e;
        const unsigned grid = (unsigned)std::min<int64_t>(((rows + U - 1) / U + GV_WARPS - 1) / GV_WARPS, sms);
        const int nb = (int)(n_cols / QK);
        float *Yr = resid ? nullptr : Y + r0;
        float *hr = resid ? resid + r0 : nullptr;
        if (dtype == Q4)
            return launch_pdl(early_weights, k_gemv_staged<Q4>, grid, GV_WARPS * 32, smem, s, w + r0 * rb, rows, nb,
                              rb, U, (const act_q8 *)act, T, Yr, ldy, hr, rs, nullptr, nullptr, 0.0f);
        return launch_pdl(early_weights, k_gemv_staged<Q8>, grid, GV_WARPS * 32, smem, s, w + r0 * rb, rows, nb, rb,
                          U, (const act_q8 *)act, T, Yr, ldy, hr, rs, nullptr, nullptr, 0.0f);
    }
    if (is_quant(dtype)) {
        const int nb = (int)(n_cols / QK);
        dim3 grid((unsigned)((rows + 7) / 8), (unsigned)std::min<int64_t>((T + 15) / 16, 65535));
        if (dtype == Q4)
            k_matmul_q<Q4><<<grid, 256, 0, s>>>(w, nb, rb, (const act_q8 *)act, T, Y, ldy, r0, r1, resid, rs);
        else
            k_matmul_q<Q8><<<grid, 256, 0, s>>>(w, nb, rb, (const act_q8 *)act, T, Y, ldy, r0, r1, resid, rs);
    } else {
        const int64_t items = rows * T;
        const unsigned grid = (unsigned)((items + 15) / 16);
        const float *x = static_cast<const float *>(act);
        if (dtype == F32) k_matmul_f<F32><<<grid, 256, 0, s>>>(w, n_cols, rb, x, T, Y, ldy, r0, r1, resid, rs);
        else if (dtype == F16) k_matmul_f<F16><<<grid, 256, 0, s>>>(w, n_cols, rb, x, T, Y, ldy, r0, r1, resid, rs);
        else k_matmul_f<BF16><<<grid, 256, 0, s>>>(w, n_cols, rb, x, T, Y, ldy, r0, r1, resid, rs);
    }
    return cudaGetLastError();
}

// hearth_dequantize (engine/src/quant.c:257-307): one element per thread.
__global__ void k_dequantize(int dtype, const uint8_t *__restrict__ W, int64_t n_rows, int64_t n_cols, int64_t rb,
                             float *__restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows * n_cols) return;
    const int64_t r = i / n_cols, c = i - r * n_cols;
    out[i] = dequant_elem(dtype, W + r * rb, c);
}

cudaError_t launch_dequantize(int dtype, const void *W, int64_t n_rows, int64_t n_cols, float *out,
                              cudaStream_t s) {
    const int64_t n = n_rows * n_cols;
    if (n <= 0) return cudaSuccess;
    k_dequantize<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dtype, (const uint8_t *)W, n_rows, n_cols,
                                                             row_bytes(dtype, n_cols), out);
    return cudaGetLastError();
}

// =============================================================================================
// MoE: normalisation + activation, router, routing.
// =============================================================================================

// One CTA per token: x = rmsnorm(h, w) (NUMERICS §4) or x = h, then x's activation blocks.
__global__ void __launch_bounds__(256) k_moe_norm_act(const float *__restrict__ h, const float *__restrict__ w,
                                                      float eps, int D, float *__restrict__ x,
                                                      act_q8 *__restrict__ xact) {
    __shared__ __align__(16) float xs[8192];
    __shared__ float rsh;
    const int t = blockIdx.x, tid = threadIdx.x;
    const float *ht = h + (int64_t)t * D;
    if (D % 4 == 0) {   // 16-byte loads, several in flight per thread
        const float4 *h4 = reinterpret_cast<const float4 *>(ht);
        float4 *x4 = reinterpret_cast<float4 *>(xs);
#pragma unroll 4
        for (int i = tid; i < D / 4; i += blockDim.x) x4[i] = h4[i];
    } else {
        for (int i = tid; i < D; i += blockDim.x) xs[i] = ht[i];
    }
    __syncthreads();
    if (w) {
        if (tid < 16) {   // ms = dot16(h, h) / n ; r = 1 / sqrtf(ms + eps)
            float L = 0.0f;
            for (int i = tid; i < D; i += 16) L = __fadd_rn(L, __fmul_rn(xs[i], xs[i]));
            L = tree16(L, 0xffffu);
            if (tid == 0) {
                const float ms = __fdiv_rn(L, (float)D);
                rsh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
            }
        }
        __syncthreads();
        const float r = rsh;
#pragma unroll 4
        for (int i = tid; i < D; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], r), w[i]);
        __syncthreads();
    }
    float *xt = x + (int64_t)t * D;
    for (int i = tid; i < D; i += blockDim.x) xt[i] = xs[i];
    const int warp = tid >> 5, lane = tid & 31, nb = D / QK;
    for (int b = warp; b < nb; b += blockDim.x >> 5)
        act_quant_warp(xs[b * QK + lane], xs[b * QK + lane + 32], xact + (int64_t)t * nb + b, lane);
}

// The opt-in shared memory per block of the current device.
static size_t smem_limit() {
    static size_t lim = 0;
    if (!lim) {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        lim = (size_t)v;
    }
    return lim;
}

// Routing of token t by one warp: the register-resident warp routing when E <= 128 without expert
// groups or forced ids, else the general warp routing (groups, E > 128, route replay).
// score / sel: 2 * E floats of this warp's shared scratch.
__device__ __forceinline__ void route_one(const MoeShape &sh, const MoeScratch &sc, int t, const float *bias,
                                          float *score, float *sel) {
    const int E = sh.route.E, K = sh.route.K;
    if (!sc.forced_ids && E <= 128 && sh.route.n_group <= 1 && K <= 16)
        route_token_warp128(sh.route, sc.logits + (int64_t)t * E, bias, sc.ids + t * K, sc.wts + t * K, score);
    else
        route_token_warp(sh.route, sc.logits + (int64_t)t * E, bias, score, sel, sc.ids + t * K, sc.wts + t * K,
                         sc.forced_ids ? sc.forced_ids + t * K : nullptr);
}

// Router logits (F32 dot16 rows, canonical NaN) and the shared-expert gate logit, one 16-lane
// group per (row, token). With fuse_route the last CTA to finish routes every token and builds
// the buckets.
// staged (one token): the CTA's rows and x arrive in shared memory by 1-D bulk copies first, so the
// chains read shared memory and every CTA keeps its whole share of the router in flight at once.
// staged == 2 also forms x = rmsnorm(h, norm) (or x = h without a norm) in every CTA from h, and each
// CTA writes its share of x's activation blocks (the separate norm kernel's work).
__global__ void __launch_bounds__(256) k_moe_router(MoeShape sh, const float *__restrict__ router,
                                                    const float *__restrict__ gate_inp,
                                                    const float *__restrict__ bias, MoeScratch sc, int fuse_route,
                                                    int staged, const float *__restrict__ h,
                                                    const float *__restrict__ norm) {
    extern __shared__ __align__(16) float rsm[];
    __shared__ int last;
    __shared__ float rsh;
    __shared__ __align__(8) uint64_t rbar;
    const int D = sh.D, E = sh.route.E, T = sh.T;
    const int rows = E + (gate_inp ? 1 : 0);
    const int grp = threadIdx.x >> 4, j = threadIdx.x & 15;
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 4) + grp;
    const bool valid = item < (int64_t)rows * T;
    const int r = valid ? (int)(item % rows) : 0;
    const int t = valid ? (int)(item / rows) : 0;
    float L = 0.0f;
    if (staged) {   // T == 1: item == row
        const int r0 = blockIdx.x * (blockDim.x >> 4), nr = min((int)(blockDim.x >> 4), rows - r0);
        const bool fnorm = staged == 2, wn = fnorm && norm;
        float *xs = rsm, *nws = rsm + D, *ws = rsm + (fnorm ? 2 * D : D);
        if (threadIdx.x == 0) {
            mbar_init(&rbar, 1);
            fence_mbar_init();
            mbar_expect_tx(&rbar, (uint32_t)((nr + (wn ? 2 : 1)) * D * 4));
            bulk_g2s(xs, fnorm ? h : sc.x, (uint32_t)(D * 4), &rbar);
            if (wn) bulk_g2s(nws, norm, (uint32_t)(D * 4), &rbar);
            for (int k = 0; k < nr; k++)
                bulk_g2s(ws + (int64_t)k * D, r0 + k < E ? router + (int64_t)(r0 + k) * D : gate_inp, (uint32_t)(D * 4),
                         &rbar);
        }
        __syncthreads();
        const bool ok = mbar_wait(&rbar, 0, sc.err);
        if (fnorm && ok) {
            if (wn) {   // x = rmsnorm(h, norm) (NUMERICS §4), as k_moe_norm_act forms it
                const int tid = threadIdx.x;
                if (tid < 16) {
                    float Ls = 0.0f;
                    for (int i = tid; i < D; i += 16) Ls = __fadd_rn(Ls, __fmul_rn(xs[i], xs[i]));
                    Ls = tree16(Ls, 0xffffu);
                    if (tid == 0) rsh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(Ls, (float)D), sh.eps)));
                }
                __syncthreads();
                const float rr = rsh;
                for (int i = tid; i < D; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], rr), nws[i]);
                __syncthreads();
            }
            // this CTA's share of x and its activation blocks (blocks blockIdx.x + k * gridDim.x)
            const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
            for (int b = blockIdx.x + warp * gridDim.x; b < D / QK; b += gridDim.x * nwarps) {
                const float x0 = xs[b * QK + lane], x1 = xs[b * QK + lane + 32];
                sc.x[b * QK + lane] = x0;
                sc.x[b * QK + lane + 32] = x1;
                act_quant_warp(x0, x1, sc.xact + b, lane);
            }
        }
        if (valid && ok) {
            const float *wr = ws + (int64_t)grp * D;
#pragma unroll 8
            for (int i = j; i < D; i += 16) L = __fadd_rn(L, __fmul_rn(wr[i], xs[i]));
        }
    } else if (valid) {
        const float *x = sc.x + (int64_t)t * D;
        const float *w = r < E ? router + (int64_t)r * D : gate_inp;
#pragma unroll 8
        for (int i = j; i < D; i += 16) L = __fadd_rn(L, __fmul_rn(__ldg(w + i), x[i]));
    }
    L = tree16(L, 0xffffffffu);
    if (valid && j == 0) {
        if (r < E) sc.logits[(int64_t)t * E + r] = canon(L);
        else sc.sh_logit[t] = L;
    }
    if (!fuse_route) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(sc.ticket, 1u);
        last = ticket == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // this CTA saw every other CTA's logits: route each token (one warp per token)
    const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    float *score = rsm + warp * 2 * E, *sel = score + E;
    for (int tt = warp; tt < T; tt += nwarps)
        route_one(sh, sc, tt, bias, score, sel);
    __syncthreads();
    __threadfence_block();
    int *cnt = reinterpret_cast<int *>(rsm), *start = cnt + E;
    route_union_cta(T, sh.route.K, E, sc.ids, cnt, start, sc.nu, sc.ulist, sc.u_p0, sc.u_n, sc.pair_tok,
                    sc.pair_of, start + E);
    if (threadIdx.x == 0) *sc.ticket = 0u;   // ready for the next launch
}

// Router logits of a large batch as a tiled GEMM on the CUDA cores, in the canonical dot16 order
// (NUMERICS §1): output (t, e) = tree16 over lanes j of L_j = ((0 + x_j w_j) + x_{j+16} w_{j+16}) + ...
// A CTA computes 16 tokens x 16 rows (router rows, and the shared-expert gate row as row E): thread
// (cell c, lane j) keeps lane j's chains of the 4 x 4 outputs of cell c, with K staged 64 columns at a
// time in shared memory; the 16 lanes of a cell form one half-warp for the final tree.
constexpr int RT_T = 16, RT_E = 16, RT_K = 64;
constexpr int kTiledRouterMinT = 64;   // below, the per-(row, token) router keeps every SM busy

__global__ void __launch_bounds__(256) k_moe_router_tiled(MoeShape sh, const float *__restrict__ router,
                                                          const float *__restrict__ gate_inp, MoeScratch sc) {
    __shared__ float xs[RT_T][RT_K + 1], ws[RT_E][RT_K + 1];
    const int D = sh.D, E = sh.route.E, T = sh.T;
    const int rows = E + (gate_inp ? 1 : 0);
    const int t0 = blockIdx.x * RT_T, e0 = blockIdx.y * RT_E;
    const int tid = threadIdx.x, j = tid & 15, cell = tid >> 4;   // 16 cells of 4 x 4 outputs
    const int ct = (cell >> 2) * 4, ce = (cell & 3) * 4;           // the cell's first token / row in the tile
    float L[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) L[a][b] = 0.0f;
    for (int k0 = 0; k0 < D; k0 += RT_K) {
        for (int i = tid; i < RT_T * RT_K; i += 256) {   // stage x and w (zeros outside the batch / rows)
            const int r = i / RT_K, k = i - r * RT_K, t = t0 + r, e = e0 + r;
            xs[r][k] = t < T ? sc.x[(int64_t)t * D + k0 + k] : 0.0f;
            ws[r][k] = e < E ? __ldg(router + (int64_t)e * D + k0 + k) : (e < rows ? __ldg(gate_inp + k0 + k) : 0.0f);
        }
        __syncthreads();
#pragma unroll
        for (int s = 0; s < RT_K / 16; s++) {   // columns k0 + j + 16 s, in order
            const int k = j + 16 * s;
            float xv[4], wv[4];
#pragma unroll
            for (int a = 0; a < 4; a++) xv[a] = xs[ct + a][k];
#pragma unroll
            for (int b = 0; b < 4; b++) wv[b] = ws[ce + b][k];
#pragma unroll
            for (int a = 0; a < 4; a++)
#pragma unroll
                for (int b = 0; b < 4; b++) L[a][b] = __fadd_rn(L[a][b], __fmul_rn(wv[b], xv[a]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const float v = tree16(L[a][b], 0xffffffffu);
            const int t = t0 + ct + a, e = e0 + ce + b;
            if (j == 0 && t < T && e < rows) {
                if (e < E) sc.logits[(int64_t)t * E + e] = canon(v);
                else sc.sh_logit[t] = v;
            }
        }
}

__global__ void __launch_bounds__(256) k_route_select(MoeShape sh, const float *__restrict__ bias, MoeScratch sc) {
    extern __shared__ float rsm[];
    const int warp = threadIdx.x >> 5, E = sh.route.E;
    const int t = blockIdx.x * 8 + warp;
    if (t >= sh.T) return;
    float *score = rsm + warp * 2 * E, *sel = score + E;
    route_one(sh, sc, t, bias, score, sel);
}

__global__ void __launch_bounds__(512) k_route_union(MoeShape sh, MoeScratch sc) {
    extern __shared__ int usm[];
    route_union_cta(sh.T, sh.route.K, sh.route.E, sc.ids, usm, usm + sh.route.E, sc.nu, sc.ulist, sc.u_p0,
                    sc.u_n, sc.pair_tok, sc.pair_of, usm + 2 * sh.route.E);
    if (sh.ep_size > 1) {   // the buckets of this rank's experts, in bucket order
        __syncthreads();
        if (threadIdx.x == 0) {
            int n = 0;
            for (int u = 0; u < *sc.nu; u++)
                if (sc.ulist[u] % sh.ep_size == sh.ep_rank) sc.ujob[n++] = u;
            *sc.nu_job = n;
        }
    }
}


// =============================================================================================
// MoE experts. A "job" is one routed expert bucket (jobs 0..nu-1, experts ascending) or the
// shared expert over all tokens (job nu). Activation rows of job pairs: routed pair p -> p,
// shared token t -> T*K + t.
// =============================================================================================



constexpr int GU_ROWS = 64;    // gate/up rows per CTA: one activation block of the mid vector
constexpr int GU_CH = 8;       // rows of gate (and of up) per pipeline stage
constexpr int GU_NCH = GU_ROWS / GU_CH;
constexpr int DN_ROWS = 16;    // down rows per CTA

struct GateUpCfg {
    int ntok;       // tokens per pass
    int64_t ring;   // bytes of the copy ring; each job cuts it into stages of its own row size
    int nbD;
    int fmax_nb;    // activation blocks per mid row (max of F, Fs over 64)
};

template <int DT>
__device__ void gateup_body(const MoeShape &sh, const MoeScratch &sc, const Job &job, const GateUpCfg &c,
                            uint8_t *smem, int rb) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nbD = c.nbD;
    const int64_t rbD = row_bytes(DT, sh.D);
    const int64_t chunk = (int64_t)GU_CH * rbD;   // bytes of one matrix's stage rows
    const int64_t stage = 2 * chunk;
    const int nst = (int)min((int64_t)GU_NCH, c.ring / stage);   // >= 1: the host sized the ring for the widest rows
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    uint8_t *ring = smem + 128;
    act_q8 *acts = reinterpret_cast<act_q8 *>(ring + c.ring);
    const int nw = blockDim.x >> 5;   // 16 warps: one row of each 16-row stage
    const int pw = c.ntok * 33;         // a warp's term buffer: ntok chains
    float *P = reinterpret_cast<float *>(acts + (int64_t)c.ntok * nbD) + warp * pw;
    float *GU = reinterpret_cast<float *>(acts + (int64_t)c.ntok * nbD) + nw * pw;   // [2][ntok][64]
    int *tok_off = reinterpret_cast<int *>(GU + 2 * c.ntok * GU_ROWS);                  // [ntok]

    const int npass = (job.n + c.ntok - 1) / c.ntok;
    const int total = npass * GU_NCH;
    const uint8_t *g0 = job.gate + (int64_t)rb * GU_ROWS * rbD, *u0 = job.up + (int64_t)rb * GU_ROWS * rbD;
    if (tid == 0) {
        for (int s = 0; s < nst; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int q) {   // thread 0: chunk q (pass q / GU_NCH, chunk q % GU_NCH)
        const int s = q % nst, ch = q % GU_NCH;
        uint8_t *dst = ring + (int64_t)s * stage;
        mbar_expect_tx(&bars[s], (uint32_t)(2 * chunk));
        bulk_g2s(dst, g0 + ch * chunk, (uint32_t)chunk, &bars[s]);
        bulk_g2s(dst + chunk, u0 + ch * chunk, (uint32_t)chunk, &bars[s]);
    };
    if (tid == 0)
        for (int q = 0; q < min(nst, total); q++) issue(q);
    bool ok = true;
    for (int pass = 0; pass < npass; pass++) {
        const int i0 = pass * c.ntok, nt = min(c.ntok, job.n - i0);
        // stage this pass's token activations (nbD blocks each) and their offsets
        for (int i = 0; i < nt; i++) {
            const int t = job_token(sc, job, i0 + i);
            const uint32_t *src = reinterpret_cast<const uint32_t *>(sc.xact + (int64_t)t * nbD);
            uint32_t *dst = reinterpret_cast<uint32_t *>(acts + (int64_t)i * nbD);
            for (int k = tid; k < nbD * (ACT_BLOCK / 4); k += blockDim.x) dst[k] = src[k];
        }
        if (tid < nt) tok_off[tid] = tid * nbD;
        __syncthreads();
        for (int ch = 0; ch < GU_NCH; ch++) {
            const int q = pass * GU_NCH + ch, s = q % nst;
            ok = ok && mbar_wait(&bars[s], (uint32_t)((q / nst) & 1), sc.err);
            if (ok) {
                const uint8_t *st = ring + (int64_t)s * stage;
                // warp w: row w of this stage (rows 0..7 gate, 8..15 up)
                const int rl[1] = {warp};
                const int row = ch * GU_CH + (warp & (GU_CH - 1));   // row within the CTA's 64
                float *out = GU + (warp >= GU_CH ? (int64_t)c.ntok * GU_ROWS : 0) + row;
                for (int tg = 0; tg < nt; tg += 16) {
                    const int ntg = min(16, nt - tg);
                    warp_rows<DT>(st, rbD, nbD, rl, 1, acts, tok_off + tg, ntg, P, out + (int64_t)tg * GU_ROWS, 0,
                                  GU_ROWS);
                }
            }
            __syncthreads();
            if (tid == 0 && q + nst < total) {
                fence_proxy_async();
                issue(q + nst);
            }
        }
        if (!ok) break;
        // SwiGLU and the mid activation block of each token (warp per token)
        for (int i = warp; i < nt; i += nw) {
            const float *G = GU + i * GU_ROWS, *U = GU + c.ntok * GU_ROWS + i * GU_ROWS;
            const float m0 = swiglu_c(G[lane], U[lane]), m1 = swiglu_c(G[lane + 32], U[lane + 32]);
            act_q8 *dst = sc.act_mid + (int64_t)(job.p0 + i0 + i) * c.fmax_nb + rb;
            act_quant_warp(m0, m1, dst, lane);
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(512) k_moe_gateup(MoeShape sh, MoeLayerDev L, MoeScratch sc, GateUpCfg c) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int u = blockIdx.y, rb = blockIdx.x;
    const int nu = routed_jobs(sh, sc);
    const int njobs = nu + (L.Fs > 0 ? 1 : 0);
    if (u >= njobs) return;
    Job job;
    if (!get_job(sh, L, sc, u, nu, job)) return;
    if (rb * GU_ROWS >= job.F) return;
    if (job.dtype == Q4) gateup_body<Q4>(sh, sc, job, c, smem, rb);
    else gateup_body<Q8>(sh, sc, job, c, smem, rb);
}

// ---- gate/up for single-token jobs (decode, T = 1): one CTA per (job, 64 mid rows), G1_WARPS warps.
// The CTA's 128 rows (64 gate, then the 64 up rows of the same mid rows) go in tiles of TR
// consecutive rows (TR rows of up to 32 KB: one 1-D bulk copy each), warp w taking tiles w,
// w + G1_WARPS, ... into its own shared-memory slot; each tile runs through the single-token row loop
// (lane = block, the activation block kept in registers across 8 rows, lanes 0..7 the rows' chains).
// SwiGLU and the mid activation block follow in the CTA. Used when rows are whole 16-byte units.
constexpr int G1_WARPS = 12;
constexpr int G1_SLOT = 16 * 1024;
constexpr int G1_HDR = (G1_WARPS * 8 + 127) / 128 * 128;   // the warps' mbarriers
constexpr int G1_TMAX = 4;   // tokens per job (decode, speculative verification of a few tokens)

__host__ __device__ inline int g1_tile_rows(int64_t rb) {   // largest power of two <= 32 with TR * rb <= G1_SLOT
    int tr = 32;
    while (tr > 1 && tr * rb > G1_SLOT) tr >>= 1;
    return tr;
}

template <int DT>
__device__ void gateup1_body(const MoeShape &sh, const MoeScratch &sc, const Job &job, int fmax_nb, uint8_t *smem,
                             int rb) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nbD = sh.D / QK;
    const int64_t rbD = row_bytes(DT, sh.D);
    const int TR = g1_tile_rows(rbD), ntile = 2 * GU_ROWS / TR;   // gate tiles, then up tiles
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem) + warp;
    uint8_t *slot = smem + G1_HDR + (size_t)warp * G1_SLOT;
    const int nt = job.n;   // <= G1_TMAX (host condition)
    act_q8 *acts = reinterpret_cast<act_q8 *>(smem + G1_HDR + (size_t)G1_WARPS * G1_SLOT);   // [nt][nbD]
    float *P = reinterpret_cast<float *>(acts + sh.T * nbD) + warp * ROWS_1TOK * 33;
    float *GU = reinterpret_cast<float *>(acts + sh.T * nbD) + G1_WARPS * ROWS_1TOK * 33;   // [nt][2][64]
    auto issue = [&](int tile) {
        const int r = tile * TR;   // row in [0, 128): gate rows, then up rows
        const uint8_t *src = (r < GU_ROWS ? job.gate : job.up) + ((int64_t)rb * GU_ROWS + (r % GU_ROWS)) * rbD;
        mbar_expect_tx(bar, (uint32_t)(TR * rbD));
        bulk_g2s(slot, src, (uint32_t)(TR * rbD), bar);
    };
    if (lane == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        if (warp < ntile) issue(warp);
    }
    for (int i = 0; i < nt; i++) {   // the tokens' activation blocks
        const int t = job_token(sc, job, i);
        const uint32_t *src = reinterpret_cast<const uint32_t *>(sc.xact + (int64_t)t * nbD);
        uint32_t *dst = reinterpret_cast<uint32_t *>(acts + (int64_t)i * nbD);
        for (int k = threadIdx.x; k < nbD * (ACT_BLOCK / 4); k += blockDim.x) dst[k] = src[k];
    }
    __syncthreads();
    bool ok = true;
    int k = 0;
    for (int tile = warp; tile < ntile; tile += G1_WARPS, k++) {
        ok = ok && mbar_wait(bar, (uint32_t)(k & 1), sc.err);
        if (ok)
            for (int i = 0; i < nt; i++)   // the tile stays in shared memory for every token
                for (int r8 = 0; r8 < TR; r8 += ROWS_1TOK)
                    warp_rows_1tok<DT>(slot + (int64_t)r8 * rbD, rbD, nbD, min(ROWS_1TOK, TR - r8), acts + (int64_t)i * nbD,
                                       P, GU + i * 2 * GU_ROWS + tile * TR + r8);
        if (lane == 0 && tile + G1_WARPS < ntile && ok) {
            fence_proxy_async();
            issue(tile + G1_WARPS);
        }
        __syncwarp();
    }
    __syncthreads();
    if (warp < nt && ok) {   // warp i: token i's SwiGLU and mid activation block
        const float *G = GU + warp * 2 * GU_ROWS, *U = G + GU_ROWS;
        act_quant_warp(swiglu_c(G[lane], U[lane]), swiglu_c(G[lane + 32], U[lane + 32]),
                       sc.act_mid + (int64_t)(job.p0 + warp) * fmax_nb + rb, lane);
    }
}

__global__ void __launch_bounds__(G1_WARPS * 32) k_moe_gateup1(MoeShape sh, MoeLayerDev L, MoeScratch sc,
                                                              int fmax_nb) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int u = blockIdx.y, rb = blockIdx.x;
    const int nu = routed_jobs(sh, sc);
    const int njobs = nu + (L.Fs > 0 ? 1 : 0);
    if (u >= njobs) return;
    Job job;
    if (!get_job(sh, L, sc, u, nu, job)) return;
    if (rb * GU_ROWS >= job.F) return;
    if (job.dtype == Q4) gateup1_body<Q4>(sh, sc, job, fmax_nb, smem, rb);
    else gateup1_body<Q8>(sh, sc, job, fmax_nb, smem, rb);
}

static size_t gateup1_smem(int nbD, int T) {
    return G1_HDR + (size_t)G1_WARPS * G1_SLOT + (size_t)T * nbD * ACT_BLOCK + (size_t)G1_WARPS * ROWS_1TOK * 33 * 4 +
           (size_t)T * 2 * GU_ROWS * 4 + 64;
}

struct DownCfg {
    int nst;          // pipeline stages
    int64_t stage;    // bytes per stage (DN_ROWS rows of the widest down matrix)
    int fmax_nb;      // activation blocks per mid row
    int fused;        // keep Y in shared memory and finish the rank-order sum here
    int max_pairs;    // fused: T*K (Y rows held in shared memory)
};

// One down tile (DN_ROWS rows of a job's down matrix) against the job's mid activations.
template <int DT>
__device__ void down_tile(const MoeShape &sh, const MoeScratch &sc, const Job &job, const DownCfg &c,
                          const uint8_t *tile, float *P, int *tok_off, float *Ys, float *Ss, int r0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rbF = row_bytes(DT, job.F);
    const int rl[1] = {warp};   // 16 warps: one row of the 16-row tile each
    for (int i0 = 0; i0 < job.n; i0 += 16) {
        const int nt = min(16, job.n - i0);
        if (lane < nt) tok_off[lane] = (job.p0 + i0 + lane) * c.fmax_nb;
        __syncwarp();
        float *out;
        int oi;
        if (c.fused) {
            out = job.shared ? Ss + (int64_t)i0 * DN_ROWS + warp : Ys + (int64_t)(job.p0 + i0) * DN_ROWS + warp;
            oi = DN_ROWS;
        } else {
            out = job.shared ? sc.S + (int64_t)i0 * sh.D + r0 + warp
                             : sc.Y + (int64_t)(job.p0 + i0) * sh.D + r0 + warp;
            oi = sh.D;
        }
        warp_rows<DT>(tile, rbF, job.nbF, rl, 1, sc.act_mid, tok_off, nt, P, out, 0, oi);
        __syncwarp();
    }
}

// Per (token, row): out = sum_j w_j * y_j in rank order from +0.0f, + shared (times its sigmoid
// gate), then h += rs * out and/or out written (engine/src/model.c:904-923, 925-934).
__device__ __forceinline__ void finish_row(const MoeShape &sh, const MoeScratch &sc, int t, int r, const float *Yrow,
                                           int ystride, float sval, bool has_shared, const float *sh_logit,
                                           float *h, float *out, bool resid) {
    const int K = sh.route.K;
    float o = 0.0f;
    for (int j = 0; j < K; j++) {
        const float wj = sc.wts[t * K + j];
        const float y = Yrow[(int64_t)sc.pair_of[t * K + j] * ystride];
        o = __fadd_rn(o, __fmul_rn(wj, y));
    }
    if (has_shared) {
        float s = sval;
        if (sh_logit) s = __fmul_rn(s, sigmoid_c(sh_logit[t]));
        o = __fadd_rn(o, s);
    }
    const int64_t idx = (int64_t)t * sh.D + r;
    if (out) out[idx] = o;
    if (resid) h[idx] = __fadd_rn(h[idx], __fmul_rn(sh.residual_scale, o));
}

__global__ void __launch_bounds__(512) k_moe_down(MoeShape sh, MoeLayerDev L, MoeScratch sc, DownCfg c, float *h,
                                                  float *out, int resid) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5;
    const int r0 = blockIdx.x * DN_ROWS;
    const int nu = routed_jobs(sh, sc);
    const int njobs = nu + (L.Fs > 0 ? 1 : 0);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    uint8_t *ring = smem + 128;
    // 16 warps: term buffers of 16 chains, token offsets, then the fused rows
    float *P = reinterpret_cast<float *>(ring + (int64_t)c.nst * c.stage) + warp * (16 * 33);
    int *tok_off = reinterpret_cast<int *>(reinterpret_cast<float *>(ring + (int64_t)c.nst * c.stage) + 16 * 16 * 33) +
                   warp * 16;
    float *Ys = reinterpret_cast<float *>(reinterpret_cast<int *>(reinterpret_cast<float *>(
                                               ring + (int64_t)c.nst * c.stage) + 16 * 16 * 33) + 16 * 16);
    float *Ss = Ys + (int64_t)(c.fused ? c.max_pairs : 0) * DN_ROWS;
    if (tid == 0) {
        for (int s = 0; s < c.nst; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int u) {
        Job j;
        if (!get_job(sh, L, sc, u, nu, j)) return false;
        const int64_t rbF = row_bytes(j.dtype, j.F);
        const int s = u % c.nst;
        mbar_expect_tx(&bars[s], (uint32_t)(DN_ROWS * rbF));
        bulk_g2s(ring + (int64_t)s * c.stage, j.down + (int64_t)r0 * rbF, (uint32_t)(DN_ROWS * rbF), &bars[s]);
        return true;
    };
    __shared__ int issued_ok;
    if (tid == 0) {
        int ok = 1;
        for (int u = 0; u < min(c.nst, njobs); u++) ok &= issue(u) ? 1 : 0;
        issued_ok = ok;
    }
    __syncthreads();
    bool ok = issued_ok != 0;
    for (int u = 0; u < njobs && ok; u++) {
        Job job;
        get_job(sh, L, sc, u, nu, job);
        const int s = u % c.nst;
        ok = mbar_wait(&bars[s], (uint32_t)((u / c.nst) & 1), sc.err);
        if (ok) {
            const uint8_t *tile = ring + (int64_t)s * c.stage;
            if (job.dtype == Q4) down_tile<Q4>(sh, sc, job, c, tile, P, tok_off, Ys, Ss, r0);
            else down_tile<Q8>(sh, sc, job, c, tile, P, tok_off, Ys, Ss, r0);
        }
        __syncthreads();
        if (tid == 0 && u + c.nst < njobs) {
            fence_proxy_async();
            if (!issue(u + c.nst)) issued_ok = 0;
        }
        __syncthreads();
        ok = ok && issued_ok != 0;
    }
    if (!ok) {
        // drain copies that may still be landing in this CTA's shared memory before exiting
        if (tid == 0)
            for (int u = 0; u < njobs && u < c.nst; u++) mbar_wait(&bars[u % c.nst], 0, nullptr);
        return;
    }
    if (!c.fused) return;
    const int T = sh.T;
    const bool has_shared = L.Fs > 0;
    for (int it = tid; it < T * DN_ROWS; it += blockDim.x) {
        const int t = it / DN_ROWS, rr = it - t * DN_ROWS;
        finish_row(sh, sc, t, r0 + rr, Ys + rr, DN_ROWS, has_shared ? Ss[t * DN_ROWS + rr] : 0.0f, has_shared,
                   L.sh_gate_inp ? sc.sh_logit : nullptr, h, out, resid != 0);
    }
}

__global__ void k_moe_sum(MoeShape sh, MoeLayerDev L, MoeScratch sc, float *h, float *out, int resid) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)sh.T * sh.D) return;
    const int t = (int)(i / sh.D), r = (int)(i - (int64_t)t * sh.D);
    const bool has_shared = L.Fs > 0;
    finish_row(sh, sc, t, r, sc.Y + r, sh.D, has_shared ? sc.S[i] : 0.0f, has_shared,
               L.sh_gate_inp ? sc.sh_logit : nullptr, h, out, resid != 0);
}

// ---- down for single-token jobs (decode, T = 1): one CTA per DN_ROWS rows of D, 8 warps; its work
// units are (job, 8 of its rows), warp w taking units w, w + 8, ...: each unit's 8 down rows are
// consecutive (one 1-D bulk copy into the warp's slot) and run through the single-token row loop.
// The pair outputs stay in shared memory and the CTA finishes its rows: rank-order sum, shared
// expert, residual. Used when 8 down rows fit D1_SLOT bytes.
constexpr int D1_SLOT = 20 * 1024;

__global__ void __launch_bounds__(256) k_moe_down1(MoeShape sh, MoeLayerDev L, MoeScratch sc, int fmax_nb, float *h,
                                                   float *out, int resid) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * DN_ROWS;
    const int nu = routed_jobs(sh, sc);
    const int njobs = nu + (L.Fs > 0 ? 1 : 0);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem) + warp;
    uint8_t *slot = smem + 128 + (size_t)warp * D1_SLOT;
    float *P = reinterpret_cast<float *>(smem + 128 + (size_t)8 * D1_SLOT) + warp * ROWS_1TOK * 33;
    // [T * K pairs + T shared rows][DN_ROWS], the fused down kernel's layout
    float *Ys = reinterpret_cast<float *>(smem + 128 + (size_t)8 * D1_SLOT) + 8 * ROWS_1TOK * 33;
    const int units = njobs * (DN_ROWS / ROWS_1TOK);
    auto issue = [&](int un) {
        const int u = un / (DN_ROWS / ROWS_1TOK), gi = un - u * (DN_ROWS / ROWS_1TOK);
        Job j;
        if (!get_job(sh, L, sc, u, nu, j)) return false;
        const int64_t rbF = row_bytes(j.dtype, j.F);
        mbar_expect_tx(bar, (uint32_t)(ROWS_1TOK * rbF));
        bulk_g2s(slot, j.down + (int64_t)(r0 + gi * ROWS_1TOK) * rbF, (uint32_t)(ROWS_1TOK * rbF), bar);
        return true;
    };
    bool ok = true;
    if (lane == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (warp < units) {
        int issued = 1;
        if (lane == 0) issued = issue(warp) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, issued, 0) != 0;
    }
    int k = 0;
    for (int un = warp; ok && un < units; un += 8, k++) {
        const int u = un / (DN_ROWS / ROWS_1TOK), gi = un - u * (DN_ROWS / ROWS_1TOK);
        Job job;
        get_job(sh, L, sc, u, nu, job);
        ok = mbar_wait(bar, (uint32_t)(k & 1), sc.err);
        if (!ok) break;
        // pair outputs by pair index, the shared expert's rows after the T * K pairs (one per token)
        for (int i = 0; i < job.n; i++) {
            float *yout = Ys + (job.shared ? sh.T * sh.route.K + i : job.p0 + i) * DN_ROWS + gi * ROWS_1TOK;
            const act_q8 *act = sc.act_mid + (int64_t)(job.p0 + i) * fmax_nb;
            if (job.dtype == Q4) warp_rows_1tok<Q4>(slot, row_bytes(Q4, job.F), job.F / QK, ROWS_1TOK, act, P, yout);
            else warp_rows_1tok<Q8>(slot, row_bytes(Q8, job.F), job.F / QK, ROWS_1TOK, act, P, yout);
        }
        if (un + 8 < units) {
            int issued = 1;
            if (lane == 0) {
                fence_proxy_async();
                issued = issue(un + 8) ? 1 : 0;
            }
            ok = __shfl_sync(0xffffffffu, issued, 0) != 0;
        }
    }
    __shared__ int all_ok;
    if (threadIdx.x == 0) all_ok = 1;
    __syncthreads();
    if (!ok) all_ok = 0;
    __syncthreads();
    if (!all_ok) return;
    // finish this CTA's rows: rank-order sum, shared expert, residual (as the fused down kernel)
    const bool has_shared = L.Fs > 0;
    const int npairs = sh.T * sh.route.K;
    for (int it = threadIdx.x; it < sh.T * DN_ROWS; it += blockDim.x) {
        const int t = it / DN_ROWS, rr = it - t * DN_ROWS;
        finish_row(sh, sc, t, r0 + rr, Ys + rr, DN_ROWS, has_shared ? Ys[(npairs + t) * DN_ROWS + rr] : 0.0f, has_shared,
                   L.sh_gate_inp ? sc.sh_logit : nullptr, h, out, resid != 0);
    }
}

static size_t down1_smem(int T, int K) {
    return 128 + (size_t)8 * D1_SLOT + (size_t)8 * ROWS_1TOK * 33 * 4 + (size_t)(T * K + T) * DN_ROWS * 4 + 64;
}

// Expert-parallel combine: pair (t, j) of expert e comes from rank e % ep_size's slice of y_all.
__global__ void k_moe_ep_combine(MoeShape sh, MoeLayerDev L, MoeScratch sc, const float *__restrict__ y_all,
                                 float *h) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)sh.T * sh.D) return;
    const int t = (int)(i / sh.D), r = (int)(i - (int64_t)t * sh.D), K = sh.route.K;
    const int64_t slice = (int64_t)sh.T * K * sh.D;
    float o = 0.0f;   // rank-order sum (engine/src/model.c:904-923)
    for (int j = 0; j < K; j++) {
        const int owner = sc.ids[t * K + j] % sh.ep_size;
        const float y = y_all[owner * slice + (int64_t)sc.pair_of[t * K + j] * sh.D + r];
        o = __fadd_rn(o, __fmul_rn(sc.wts[t * K + j], y));
    }
    if (L.Fs > 0) {
        float sv = sc.S[i];
        if (L.sh_gate_inp) sv = __fmul_rn(sv, sigmoid_c(sc.sh_logit[t]));
        o = __fadd_rn(o, sv);
    }
    h[i] = __fadd_rn(h[i], __fmul_rn(sh.residual_scale, o));
}

cudaError_t launch_moe_ep_combine(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc,
                                  const float *y_all, float *h, cudaStream_t s) {
    const int64_t n = (int64_t)sh.T * sh.D;
    k_moe_ep_combine<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(sh, L, sc, y_all, h);
    return cudaGetLastError();
}

// =============================================================================================
// Launch sequences.
// =============================================================================================

static int fmax_nb_of(const MoeShape &sh, const MoeLayerDev &L) { return std::max(sh.F, L.Fs) / QK; }

// Stage 0: x = rmsnorm(h) and its activations; stage 1: router logits and routing.
static void launch_route_stages(int which, const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc,
                                const float *h, cudaStream_t s) {
    const int T = sh.T, E = sh.route.E, K = sh.route.K;
    const bool fused = T * K <= kFusedMaxPairs && sh.ep_size == 1;
    constexpr int RT0 = 64;
    // one token: the router CTAs stage their rows (and h and the norm) through shared memory by bulk
    // copies; with both stages asked for they also form x and its activation blocks (no norm launch)
    const size_t stage_smem = (size_t)(RT0 / 16 + 2) * sh.D * sizeof(float);
    const bool staged = T == 1 && sh.D % QK == 0 && stage_smem + 1024 <= smem_limit() &&
                        (reinterpret_cast<uintptr_t>(sc.x) & 15) == 0 && (reinterpret_cast<uintptr_t>(h) & 15) == 0 &&
                        (!L.ffn_norm || (reinterpret_cast<uintptr_t>(L.ffn_norm) & 15) == 0);
    const bool fuse_norm = staged && which == 3;
    if ((which & 1) && !fuse_norm) k_moe_norm_act<<<T, 256, 0, s>>>(h, L.ffn_norm, sh.eps, sh.D, sc.x, sc.xact);
    if (which & 2) {
        const int rows = E + (L.sh_gate_inp ? 1 : 0);
        const int64_t items = (int64_t)rows * T;
        constexpr int RT = 64;   // 4 (row, token) items per CTA: E=128 rows -> 32 CTAs at T=1
        const unsigned grid = (unsigned)((items + RT / 16 - 1) / (RT / 16));
        const size_t route_smem = (size_t)8 * 2 * E * sizeof(float);
        if (T >= kTiledRouterMinT && !fused)   // large batches: tiled router GEMM
            k_moe_router_tiled<<<dim3((unsigned)((T + RT_T - 1) / RT_T), (unsigned)((rows + RT_E - 1) / RT_E)), 256, 0,
                                 s>>>(sh, L.router, L.sh_gate_inp, sc);
        else
        {
            static_assert(RT == RT0, "router CTA size");
            const size_t smem = std::max(fused ? route_smem : (size_t)0, staged ? stage_smem : (size_t)0);
            k_moe_router<<<grid, RT, smem, s>>>(sh, L.router, L.sh_gate_inp, L.router_bias, sc, fused ? 1 : 0,
                                                fuse_norm ? 2 : (staged ? 1 : 0), h, L.ffn_norm);
        }
        if (!fused) {
            k_route_select<<<(T + 7) / 8, 256, route_smem, s>>>(sh, L.router_bias, sc);
            k_route_union<<<1, 512, (size_t)(2 + 512 / 32) * E * sizeof(int), s>>>(sh, sc);
        }
    }
}

cudaError_t launch_moe_route(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, const float *h,
                             cudaStream_t s) {
    launch_route_stages(3, sh, L, sc, h, s);
    return cudaGetLastError();
}


cudaError_t init_kernel_attributes() {
    const int lim = (int)smem_limit();
    cudaFuncAttributes fa;
    // the dynamic limit is the opt-in maximum minus the kernel's static shared memory
    cudaError_t e = cudaFuncGetAttributes(&fa, (const void *)k_moe_gateup);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_moe_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, lim - (int)fa.sharedSizeBytes);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, (const void *)k_moe_gateup1);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_moe_gateup1, cudaFuncAttributeMaxDynamicSharedMemorySize, lim - (int)fa.sharedSizeBytes);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, (const void *)k_moe_down1);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_moe_down1, cudaFuncAttributeMaxDynamicSharedMemorySize, lim - (int)fa.sharedSizeBytes);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, (const void *)k_moe_router);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_moe_router, cudaFuncAttributeMaxDynamicSharedMemorySize, lim - (int)fa.sharedSizeBytes);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, (const void *)k_moe_down);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_moe_down, cudaFuncAttributeMaxDynamicSharedMemorySize, lim - (int)fa.sharedSizeBytes);
    // load every MoE kernel now, so no module loading happens inside a stream capture later
    const void *kernels[] = {(const void *)k_moe_norm_act, (const void *)k_moe_router, (const void *)k_route_select,
                             (const void *)k_route_union, (const void *)k_moe_sum};
    for (const void *k : kernels)
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, k);
    if (e == cudaSuccess) e = init_tc_attributes();
    return e;
}

// Stage 2 (which & 1): gate/up + SwiGLU + mid activations; stage 3 (which & 2): down (+ sum).
static cudaError_t launch_expert_stages(int which, const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc,
                                        float *h, float *out, bool resid, cudaStream_t s) {
    const int T = sh.T, K = sh.route.K, E = sh.route.E;
    const bool fused = T * K <= kFusedMaxPairs && sh.ep_size == 1;
    const size_t lim = smem_limit() - 1024;
    const int fmax_nb = fmax_nb_of(sh, L);
    // large batches: tensor-core expert stages (HXB_TC=0 keeps the SIMT stages)
    static const bool tc_on = [] {
        const char *e = std::getenv("HXB_TC");
        return !(e && e[0] == '0');
    }();
    const bool tc = tc_on && !fused && T * K >= kTcMinPairs;
    if (tc) {
        cudaError_t e = launch_moe_experts_tc(sh, L, sc, which & 3, s);
        if (e != cudaSuccess) return e;
        if ((which & 2) && sh.ep_size == 1) {
            const int64_t n = (int64_t)T * sh.D;
            k_moe_sum<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(sh, L, sc, h, out, resid ? 1 : 0);
        }
        return cudaGetLastError();
    }
    // ---- gate/up + SwiGLU + mid activations
    // up to G1_TMAX tokens: the single-token kernels (rows of whole 16-byte units; a row of the widest
    // gate/up dtype fits a slot)
    const int64_t rbD_max = std::max<int64_t>(row_bytes(L.expert_dtype, sh.D), L.Fs > 0 ? row_bytes(L.sh_dtype, sh.D) : 0);
    const bool one_token = T <= G1_TMAX && (sh.D / QK) % 8 == 0 && (sh.F % GU_ROWS) == 0 && (L.Fs % GU_ROWS) == 0 &&
                           rbD_max <= G1_SLOT && gateup1_smem(sh.D / QK, T) + 1024 <= smem_limit();
    if ((which & 1) && one_token) {
        const int maxjobs = std::min(E, T * K) + (L.Fs > 0 ? 1 : 0);
        dim3 grid((unsigned)(std::max(sh.F, L.Fs) / GU_ROWS), (unsigned)maxjobs);
        k_moe_gateup1<<<grid, G1_WARPS * 32, gateup1_smem(sh.D / QK, T), s>>>(sh, L, sc, fmax_nb);
    } else if (which & 1) {
        GateUpCfg c;
        c.nbD = sh.D / QK;
        c.fmax_nb = fmax_nb;
        int64_t rb = row_bytes(sh.F > 0 ? L.expert_dtype : Q4, sh.D);
        if (L.Fs > 0) rb = std::max<int64_t>(rb, row_bytes(L.sh_dtype, sh.D));
        const size_t stage_max = 2 * GU_CH * (size_t)rb;   // the widest job's stage
        c.ntok = std::min(8, std::max(1, T));
        auto fixed = [&](int ntok) {   // everything but the ring (P: ntok chains of 33 per warp, 16 warps)
            return (size_t)128 + (size_t)ntok * c.nbD * ACT_BLOCK + (size_t)16 * ntok * 33 * 4 +
                   (size_t)2 * ntok * GU_ROWS * 4 + (size_t)ntok * 4 + 64;
        };
        while (c.ntok > 1 && fixed(c.ntok) + stage_max > lim) c.ntok /= 2;
        if (fixed(c.ntok) + stage_max > lim) return cudaErrorInvalidConfiguration;
        // the ring: 4 stages of the routed experts' rows where they fit (small rows leave room for a
        // second CTA per SM), at least one stage of the widest rows
        const size_t rb_min = (size_t)row_bytes(sh.F > 0 ? L.expert_dtype : L.sh_dtype, sh.D);
        const size_t want = std::min(lim - fixed(c.ntok), (size_t)4 * 2 * GU_CH * rb_min) / 128 * 128;
        c.ring = (int64_t)std::max(want, (stage_max + 127) / 128 * 128);
        const size_t smem = fixed(c.ntok) + (size_t)c.ring;
        const int maxjobs = std::min(E, T * K) + (L.Fs > 0 ? 1 : 0);
        dim3 grid((unsigned)(std::max(sh.F, L.Fs) / GU_ROWS), (unsigned)maxjobs);
        k_moe_gateup<<<grid, 512, smem, s>>>(sh, L, sc, c);
    }
    // ---- down (+ rank-order sum for small batches)
    const int64_t rbF_max = std::max<int64_t>(row_bytes(L.expert_dtype, sh.F), L.Fs > 0 ? row_bytes(L.sh_dtype, L.Fs) : 0);
    const bool down_one = one_token && fused && sh.D % DN_ROWS == 0 && (sh.F / QK) % 8 == 0 && (L.Fs / QK) % 8 == 0 &&
                          ROWS_1TOK * rbF_max <= D1_SLOT && down1_smem(T, K) + 1024 <= smem_limit();
    if ((which & 2) && down_one) {
        k_moe_down1<<<(unsigned)(sh.D / DN_ROWS), 256, down1_smem(T, K), s>>>(sh, L, sc, fmax_nb, h, out,
                                                                            resid ? 1 : 0);
    } else if (which & 2) {
        DownCfg c;
        c.fmax_nb = fmax_nb;
        c.fused = fused ? 1 : 0;
        c.max_pairs = T * K;
        int64_t rbF = row_bytes(L.expert_dtype, sh.F);
        if (L.Fs > 0) rbF = std::max<int64_t>(rbF, row_bytes(L.sh_dtype, L.Fs));
        c.stage = ((int64_t)DN_ROWS * rbF + 127) / 128 * 128;
        const size_t fixed = 128 + (size_t)16 * 16 * 33 * 4 + (size_t)16 * 16 * 4 +
                             (fused ? (size_t)(T * K + T) * DN_ROWS * 4 : 0) + 64;
        const int maxjobs = std::min(E, T * K) + (L.Fs > 0 ? 1 : 0);
        c.nst = (int)std::min<int64_t>(std::min(maxjobs, 16), (int64_t)((lim - fixed) / (size_t)c.stage));
        if (c.nst < 1) return cudaErrorInvalidConfiguration;
        const size_t smem = fixed + (size_t)c.nst * c.stage;
        k_moe_down<<<(unsigned)(sh.D / DN_ROWS), 512, smem, s>>>(sh, L, sc, c, h, out, resid ? 1 : 0);
        if (!fused && sh.ep_size == 1) {   // expert parallelism: the sum waits for the exchange
            const int64_t n = (int64_t)T * sh.D;
            k_moe_sum<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(sh, L, sc, h, out, resid ? 1 : 0);
        }
    }
    return cudaGetLastError();
}

cudaError_t launch_moe_experts(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, float *h,
                               float *out, bool resid, cudaStream_t s) {
    return launch_expert_stages(3, sh, L, sc, h, out, resid, s);
}

cudaError_t launch_moe_stage(int stage, const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, float *h,
                             float *out, bool resid, cudaStream_t s) {
    if (stage < 2) {
        launch_route_stages(stage == 0 ? 1 : 2, sh, L, sc, h, s);
        return cudaGetLastError();
    }
    return launch_expert_stages(stage == 2 ? 1 : 2, sh, L, sc, h, out, resid, s);
}

cudaError_t launch_moe_layer(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, float *h, float *out,
                             bool resid, cudaStream_t s) {
    cudaError_t e = launch_moe_route(sh, L, sc, h, s);
    if (e != cudaSuccess) return e;
    return launch_moe_experts(sh, L, sc, h, out, resid, s);
}

// =============================================================================================
// Synthetic weights (benchmarks without a container) and the expf self-check.
// =============================================================================================

__host__ __device__ inline uint64_t splitmix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// Q4 blocks with the statistics of N(0, sigma) weights packed by the reference quantizer:
// nibbles follow a discretised Irwin-Hall(4) bell around 8, scales jitter around sigma/2.
// One thread per 34-byte block; padding bytes of the slab stay zero.
__global__ void k_synth_q4(uint8_t *dev, int64_t n_slabs, int64_t slab_bytes, int D, int F, uint64_t seed,
                           uint32_t scale_bits, int64_t first_slab) {
    const slab_layout lay = make_slab_layout(Q4, D, F);
    const int64_t nb_gate = (int64_t)F * (D / QK);      // blocks in gate (and in up)
    const int64_t nb_down = (int64_t)D * (F / QK);
    const int64_t per_slab = 2 * nb_gate + nb_down;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_slabs * per_slab) return;
    const int64_t slab = i / per_slab, b = i - slab * per_slab;
    int64_t off;
    if (b < nb_gate) off = b * Q4_BLOCK;
    else if (b < 2 * nb_gate) off = lay.off_up + (b - nb_gate) * Q4_BLOCK;
    else off = lay.off_down + (b - 2 * nb_gate) * Q4_BLOCK;
    uint8_t *blk = dev + slab * slab_bytes + off;
    uint64_t h = splitmix64(seed ^ splitmix64((uint64_t)(i + first_slab * per_slab)));
    const uint32_t sc = scale_bits + (uint32_t)(h & 0x3f) - 32u;
    blk[0] = (uint8_t)(sc & 0xff);
    blk[1] = (uint8_t)(sc >> 8);
    for (int j = 0; j < 32; j++) {
        uint8_t v = 0;
        for (int half = 0; half < 2; half++) {
            h = splitmix64(h);
            const int s4 = (int)(h & 0xff) + (int)((h >> 8) & 0xff) + (int)((h >> 16) & 0xff) + (int)((h >> 24) & 0xff);
            int q = 8 + (s4 - 510 + 37 + 740) / 74 - 10;   // ~ round((s4-510)/74): sd ~2
            q = q < 0 ? 0 : (q > 15 ? 15 : q);
            v |= (uint8_t)(q << (4 * half));
        }
        blk[2 + j] = v;
    }
}

cudaError_t launch_synth_q4(uint8_t *dev, int64_t n_slabs, int64_t slab_bytes, int D, int F, uint64_t seed,
                            float sigma, cudaStream_t s, int64_t first_slab) {
    // the f16 bits of sigma/2 (finite, normal for any sensible sigma)
    const float v = sigma * 0.5f;
    uint32_t fb;
    std::memcpy(&fb, &v, 4);
    const int e = (int)((fb >> 23) & 0xff) - 127 + 15;
    const uint32_t scale_bits = (uint32_t)(e << 10) | ((fb >> 13) & 0x3ffu);
    const int64_t per_slab = 2 * (int64_t)F * (D / QK) + (int64_t)D * (F / QK);
    const int64_t n = n_slabs * per_slab;
    cudaMemsetAsync(dev, 0, (size_t)(n_slabs * slab_bytes), s);
    k_synth_q4<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dev, n_slabs, slab_bytes, D, F, seed, scale_bits,
                                                          first_slab);
    return cudaGetLastError();
}

// A quantized matrix (Q4 or Q8 rows, `n_blocks` consecutive 64-weight blocks) with the statistics of
// N(0, sigma) weights: Q4 as in k_synth_q4; Q8 values an Irwin-Hall(4) bell of sd ~53 under a scale
// of sigma/53 (a 64-block of N(0, sigma) has amax ~2.4 sigma, so amax/127 ~ sigma/53). One thread
// per block.
__global__ void k_synth_blocks(uint8_t *dev, int64_t n_blocks, int dtype, uint64_t seed, uint32_t scale_bits) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_blocks) return;
    uint8_t *blk = dev + i * (dtype == Q8 ? Q8_BLOCK : Q4_BLOCK);
    uint64_t h = splitmix64(seed ^ splitmix64((uint64_t)i));
    const uint32_t sc = scale_bits + (uint32_t)(h & 0x3f) - 32u;
    blk[0] = (uint8_t)(sc & 0xff);
    blk[1] = (uint8_t)(sc >> 8);
    for (int j = 0; j < (dtype == Q8 ? 64 : 32); j++) {
        h = splitmix64(h);
        const int s4 = (int)(h & 0xff) + (int)((h >> 8) & 0xff) + (int)((h >> 16) & 0xff) + (int)((h >> 24) & 0xff);
        if (dtype == Q8) {
            int q = ((s4 - 510) * 9 + (s4 >= 510 ? 12 : -12)) / 25;   // ~ round((s4-510)*0.36): sd ~53
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            blk[2 + j] = (uint8_t)(int8_t)q;
        } else {
            int lo = 8 + (s4 - 510 + 37 + 740) / 74 - 10;
            const int s4b = (int)((h >> 32) & 0xff) + (int)((h >> 40) & 0xff) + (int)((h >> 48) & 0xff) +
                            (int)((h >> 56) & 0xff);
            int hi = 8 + (s4b - 510 + 37 + 740) / 74 - 10;
            lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
            hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
            blk[2 + j] = (uint8_t)(lo | (hi << 4));
        }
    }
}

// f16 bits of a positive normal float (truncated mantissa).
static uint32_t f16_bits_of(float v) {
    uint32_t fb;
    std::memcpy(&fb, &v, 4);
    const int e = (int)((fb >> 23) & 0xff) - 127 + 15;
    return (uint32_t)(e << 10) | ((fb >> 13) & 0x3ffu);
}

cudaError_t launch_synth_blocks(uint8_t *dev, int dtype, int64_t rows, int64_t cols, uint64_t seed, float sigma,
                                cudaStream_t s) {
    if (dtype != Q4 && dtype != Q8) return cudaErrorInvalidValue;
    if (rows <= 0 || cols <= 0 || cols % QK) return cudaErrorInvalidValue;
    const int64_t n = rows * (cols / QK);
    const uint32_t scale_bits = f16_bits_of(dtype == Q8 ? sigma / 53.0f : sigma * 0.5f);
    k_synth_blocks<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dev, n, dtype, seed, scale_bits);
    return cudaGetLastError();
}

// f32 ~ N(0, sigma) approximated by Irwin-Hall(4) over bytes, one rounding: (s4 - 510) * (sigma/147.8).
__global__ void k_synth_f32(float *dev, int64_t n, uint64_t seed, float k) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t h = splitmix64(seed ^ splitmix64((uint64_t)i));
    const int s4 = (int)(h & 0xff) + (int)((h >> 8) & 0xff) + (int)((h >> 16) & 0xff) + (int)((h >> 24) & 0xff);
    dev[i] = __fmul_rn(__int2float_rn(s4 - 510), k);
}

cudaError_t launch_synth_f32(float *dev, int64_t n, uint64_t seed, float sigma, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    k_synth_f32<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dev, n, seed, sigma / 147.8f);
    return cudaGetLastError();
}

__global__ void k_expf_bits(uint32_t x0, int64_t n, float *out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    out[i] = host_expf(__uint_as_float(x0 + (uint32_t)i));
}

cudaError_t launch_expf_bits(uint32_t x0, int64_t n, float *out, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    k_expf_bits<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x0, n, out);
    return cudaGetLastError();
}

}  // namespace hx
