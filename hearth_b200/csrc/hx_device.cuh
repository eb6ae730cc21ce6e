// hx_device.cuh — sm_100a plumbing shared by the kernels: shared-memory addresses, mbarriers with
// bounded waits, 1-D bulk copies (cp.async.bulk into this CTA only), the device error word,
// and the canonical row-chain machinery of the quantized GEMV tiles.
#pragma once

#include "hx_common.cuh"

namespace hx {

// Error codes a kernel leaves in the device error word (first one wins).
enum : int {
    DEV_OK = 0,
    DEV_E_WAIT_TIMEOUT = 1,   // a bulk copy did not complete within the spin limit
    DEV_E_NOT_RESIDENT = 2,   // a routed expert had no slab in HBM
    DEV_E_BAD_DTYPE = 3,      // an expert dtype the kernels do not handle
};

constexpr uint32_t kSpinLimit = 1u << 20;   // try_wait rounds before a wait is declared lost

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void set_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization may start
// while its predecessor in the stream still runs; pdl_wait() returns once the predecessor has
// completed and its memory is visible (at once for a kernel launched without the attribute), and
// pdl_trigger() lets the next such kernel start launching. Before pdl_wait() a kernel reads only data
// written before the stream work it follows (weights, older KV rows).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launches kernel k, with programmatic stream serialization when pdl is set (the kernel must
// pdl_wait() before it reads anything earlier stream work wrote).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(bool pdl, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completion counted on bar.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase: returns false (and records the error) when the limit is hit.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
    for (uint32_t i = 0; i < kSpinLimit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    set_error(err, DEV_E_WAIT_TIMEOUT);
    return false;
}

// ---------------------------------------------------------------------------------------------
// Quantized row tiles. A tile is `rows` consecutive rows of a Q4/Q8 matrix with nb blocks per
// row, resident in shared memory (row stride rb bytes). For each (row, token) the canonical
// NUMERICS §3 value is acc = ((0 + t_0) + t_1) + ... with t_g = (float)isum_g * (dw_g * dx_g).
//
// Work split inside one warp: the (row, block) items of the warp's rows are spread over the 32
// lanes; each lane writes its block terms into the warp's term buffer P[chain][g], one chain per
// (row, token); then one lane per chain adds its terms in block order. The integer dots and the
// products are independent, only the adds form a chain, and that chain runs in exactly the
// reference's order.
// ---------------------------------------------------------------------------------------------

// Warp-level: rows rlist[0..nr) of the tile (local row indices) against tokens 0..nt whose
// activation rows (nb blocks each) start at act + tok_off[i]. Writes the canonical value of
// (rlist[k], token i) to out[k * ok + i * oi]. Blocks are taken 32 at a time; the chain lane keeps
// its running sum across those chunks, so P holds nr * nt * 33 floats whatever nb is. nr * nt <= 32.
// d * (float)q with the NaN results of the host's SSE multiply, which the reference's dequantize
// stores unmodified: a NaN scale comes back as itself (already quiet after the f16 decode) and
// inf * 0 gives the x86 default NaN 0xffc00000. GPU arithmetic would return its own canonical NaN.
__device__ __forceinline__ float x86_mul_scale(float d, int q) {
    if (d != d) return d;
    if (q == 0 && fabsf(d) == __uint_as_float(0x7f800000u)) return __uint_as_float(0xffc00000u);
    return __fmul_rn(d, (float)q);
}

// Element c of a row of any dtype, as hx_dequantize_row (engine/src/quant.c:257-307) produces it.
__device__ __forceinline__ float dequant_elem(int dtype, const uint8_t *row, int64_t c) {
    switch (dtype) {
    case F32: return reinterpret_cast<const float *>(row)[c];
    case F16: return f16_to_f32(reinterpret_cast<const uint16_t *>(row)[c]);
    case BF16: return bf16_to_f32(reinterpret_cast<const uint16_t *>(row)[c]);
    case Q8: {
        const uint8_t *blk = row + (c / QK) * Q8_BLOCK;
        return x86_mul_scale(f16_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8)), (int)(int8_t)blk[2 + c % QK]);
    }
    default: {
        const uint8_t *blk = row + (c / QK) * Q4_BLOCK;
        const int j = (int)(c % QK);
        const int nib = j < 32 ? (blk[2 + j] & 15) : (blk[2 + j - 32] >> 4);
        return x86_mul_scale(f16_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8)), nib - 8);
    }
    }
}

template <int DT>
__device__ __forceinline__ void warp_rows(const uint8_t *tile, int64_t rb, int nb, const int *rlist, int nr,
                                          const act_q8 *act, const int *tok_off, int nt, float *P, float *out,
                                          int ok, int oi) {
    const int lane = threadIdx.x & 31;
    const int nch = nr * nt;
    constexpr int BS = DT == Q4 ? Q4_BLOCK : Q8_BLOCK;
    float acc = 0.0f;
    for (int g0 = 0; g0 < nb; g0 += 32) {
        const int gn = min(32, nb - g0);
        const int items = nr * gn;
        for (int it = lane; it < items; it += 32) {
            const int k = it / gn, g = it - k * gn;
            const uint8_t *blk = tile + (int64_t)rlist[k] * rb + (int64_t)(g0 + g) * BS;
            float *pk = P + (k * nt) * 33 + g;
            if constexpr (DT == Q4) {
                uint32_t nib[8];
                const float dw = f16_to_f32(load_q4_block(blk, nib));
                for (int i = 0; i < nt; i++) {
                    act_regs ar;
                    load_act(act + tok_off[i] + g0 + g, ar);
                    pk[i * 33] = __fmul_rn(__int2float_rn(q4_isum(nib, ar.q, ar.sum)), __fmul_rn(dw, ar.d));
                }
            } else {
                uint32_t q[16];
                const float dw = f16_to_f32(load_q8_block(blk, q));
                for (int i = 0; i < nt; i++) {
                    act_regs ar;
                    load_act(act + tok_off[i] + g0 + g, ar);
                    pk[i * 33] = __fmul_rn(__int2float_rn(q8_isum(q, ar.q)), __fmul_rn(dw, ar.d));
                }
            }
        }
        __syncwarp();
        if (lane < nch) {
            const float *p = P + lane * 33;
            for (int g = 0; g < gn; g++) acc = __fadd_rn(acc, p[g]);
        }
        __syncwarp();
    }
    if (lane < nch) {
        const int k = lane / nt, i = lane - k * nt;
        out[k * ok + i * oi] = canon(acc);
    }
}

// Single-token rows (the persistent decode kernel and the single-token expert kernels): P holds
// ROWS_1TOK x 33 floats per warp; tiles in shared memory may be read up to 2 bytes past a block.
constexpr int ROWS_1TOK = 8;

// Rows [0, nr) of a tile whose rows are consecutive in shared memory, against one activation row
// of nb blocks. out[k] = canonical NUMERICS §3 value of row k. nr <= ROWS_1TOK. The row loop is
// unrolled to ROWS_1TOK (predicated on nr) so that the rows' loads and dot chains overlap.
template <int DT>
__device__ __forceinline__ void warp_rows_1tok(const uint8_t *tile, int64_t rb, int nb, int nr, const act_q8 *act,
                                               float *P, float *out) {
    const int lane = threadIdx.x & 31;
    constexpr int BS = DT == Q4 ? Q4_BLOCK : Q8_BLOCK;
    auto term = [&](const uint8_t *blk, const act_regs &ar) {
        int isum;
        uint32_t sc;
        if constexpr (DT == Q4) {
            uint32_t nib[8];
            sc = load_q4_block_pad(blk, nib);
            isum = q4_isum_hi(nib, ar.q, ar.sum);
        } else {
            uint32_t q[16];
            sc = load_q8_block_pad(blk, q);
            isum = q8_isum(q, ar.q);
        }
        return __fmul_rn(__int2float_rn(isum), __fmul_rn(f16_to_f32_hw(sc), ar.d));
    };
    float acc = 0.0f;
    for (int g0 = 0; g0 < nb; g0 += 32) {
        const int gn = min(32, nb - g0);
        if (gn == 32) {   // lane = block: its activation block stays in registers for every row
            act_regs ar;
            load_act(act + g0 + lane, ar);
            const uint8_t *col = tile + (int64_t)(g0 + lane) * BS;
#pragma unroll
            for (int k = 0; k < ROWS_1TOK; k++)
                if (k < nr) P[k * 33 + lane] = term(col + (int64_t)k * rb, ar);
        } else if (gn <= 16) {   // lane = (row phase, block): each lane's activation block loaded once
            const int rp = 32 / gn, g = lane % gn, r2 = lane / gn;
            if (r2 < rp) {
                act_regs ar;
                load_act(act + g0 + g, ar);
                const uint8_t *col = tile + (int64_t)(g0 + g) * BS;
#pragma unroll
                for (int i = 0; i < ROWS_1TOK / 2; i++) {   // rp >= 2: rows r2, r2 + rp, ... (loads overlap)
                    const int k = r2 + i * rp;
                    if (k < nr) P[k * 33 + g] = term(col + (int64_t)k * rb, ar);
                }
            }
        } else {
            for (int it = lane; it < nr * gn; it += 32) {
                const int k = it / gn, g = it - k * gn;
                act_regs ar;
                load_act(act + g0 + g, ar);
                P[k * 33 + g] = term(tile + (int64_t)k * rb + (int64_t)(g0 + g) * BS, ar);
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

}  // namespace hx
