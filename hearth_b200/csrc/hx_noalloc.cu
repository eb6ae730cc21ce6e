// hx_noalloc.cu — hxb_matmul_noalloc: the Q8/Q4/F32/F16/BF16 matmul on caller-provided device
// buffers without allocating anything.
//
// Who needs it: callers that cannot call cudaMalloc at the time they want a matmul — a serving
// engine that reserved all of HBM up front for its own pool (KV cache, expert slots), code that
// runs while a CUDA graph is being captured (cudaMalloc is not a stream operation and cannot be
// recorded into the graph), or an embedding application that budgets device memory once at start
// and forbids allocation (and the implicit device synchronisation cudaMalloc may cause) later.
// hxb_matmul, by contrast, allocates device copies of W, X and Y plus the activation scratch on
// every call.
//
// The scratch that the quantized path needs — the 72-byte activation blocks of X (NUMERICS §2) —
// lives in a file-scope __device__ array of kNoAllocScratchBytes (4 MiB). Every GPU that loads this
// library holds that array until the process exits. All calls on a device share it and it keeps
// the previous call's contents; the activation kernel overwrites every block it later reads, so
// nothing needs clearing. Two calls whose work overlaps on the GPU (different streams, or
// threads) race on the array and must be serialised by the caller.
#include "../../include/hearth_b200.h"
#include "hx_common.cuh"
#include "hx_kernels.h"

#include <mutex>
#include <string>

using namespace hx;

namespace hx {
void set_last_error(const char *msg);   // hx_capi.cu: the message hxb_last_error() returns
}

static constexpr size_t kNoAllocScratchBytes = HXB_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_act_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;

// Host code cannot use g_act_scratch's name as a device address: it is a host-side stand-in.
// The device address is looked up once per device, with that device current.
void *g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

int noalloc_fail(int code, const std::string &msg) {
    hx::set_last_error(msg.c_str());
    return code;
}

// Returns the device address of g_act_scratch on the current device (looked up on first use).
int scratch_on_current_device(void **out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return noalloc_fail(HXB_E_DEVICE, "hxb_matmul_noalloc: no current CUDA device");
    }
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_act_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return noalloc_fail(HXB_E_DEVICE, std::string("hxb_matmul_noalloc: cudaGetSymbolAddress failed: ") +
                                                  cudaGetErrorString(e));
        }
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return HXB_OK;
}

}  // namespace

extern "C" HXB_API int hxb_matmul_noalloc(int dtype, const void *W, int64_t n_rows, int64_t n_cols, const float *X,
                                          int T, float *Y, void *stream) {
    if (dtype < F32 || dtype > Q4 || n_rows < 0 || T < 0 || row_bytes(dtype, n_cols) == 0)
        return noalloc_fail(HXB_E_ARG, "hxb_matmul_noalloc: bad dtype, shape or token count");
    if (T == 0 || n_rows == 0) return HXB_OK;
    if (!W || !X || !Y) return noalloc_fail(HXB_E_ARG, "hxb_matmul_noalloc: null device pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const void *act = X;
    if (is_quant(dtype)) {
        const size_t need = (size_t)T * (size_t)(n_cols / QK) * ACT_BLOCK;
        if (need > kNoAllocScratchBytes)
            return noalloc_fail(HXB_E_CAPACITY,
                                "hxb_matmul_noalloc: T * n_cols / 64 activation blocks need " + std::to_string(need) +
                                    " bytes, more than the " + std::to_string(kNoAllocScratchBytes) +
                                    "-byte static scratch");
        void *scratch = nullptr;
        const int rc = scratch_on_current_device(&scratch);
        if (rc != HXB_OK) return rc;
        if (launch_act_quantize(X, n_cols, static_cast<act_q8 *>(scratch), n_cols, T, s) != cudaSuccess)
            return noalloc_fail(HXB_E_DEVICE, "hxb_matmul_noalloc: activation kernel launch failed");
        act = scratch;
    }
    if (launch_matmul(dtype, W, n_cols, act, T, Y, n_rows, 0, n_rows, s) != cudaSuccess)
        return noalloc_fail(HXB_E_DEVICE, "hxb_matmul_noalloc: matmul kernel launch failed");
    return HXB_OK;
}
