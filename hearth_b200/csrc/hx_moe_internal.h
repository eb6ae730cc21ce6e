// hx_moe_internal.h — what the whole-model handle (hx_model.cu) uses of the MoE backend handle
// (hx_capi.cu) inside the library: one MoE layer on device memory on the caller's stream, the device
// routing of the last layer, the device error word. Not exported.
#pragma once

#include <cuda_runtime.h>

#include "../../include/hearth_b200.h"

namespace hx {

// h [T, D] (device) += residual_scale * moe(rmsnorm(h, ffn_norm)) for MoE layer `layer`, enqueued on s.
// forced (device, [T, K] or null): route replay ids. Resident handles enqueue device work only; a
// streaming handle reads each layer's routing back (it synchronises s).
int moe_layer_for_model(hxb_moe *m, float *h, int T, int layer, cudaStream_t s, const int *forced);
// The device ids [T, K] of the last layer run (valid once s reaches the end of that layer).
const int *moe_ids_dev(const hxb_moe *m);
// Every expert has an HBM slot (the MoE layers are device work only, capturable).
bool moe_resident(const hxb_moe *m);
// The device error word (0: no error) and its decoding into a return code (clears it).
const int *moe_err_dev(const hxb_moe *m);
int moe_take_error(hxb_moe *m, int word);

}  // namespace hx
