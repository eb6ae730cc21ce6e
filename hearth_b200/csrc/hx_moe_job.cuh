// hx_moe_job.cuh — the unit of expert work of the per-phase MoE kernels: a routed expert bucket
// (its expert's slab, tokens p0.. of the bucket order) or the shared expert over all tokens.
#pragma once
#include "hx_device.cuh"
#include "hx_kernels.h"

namespace hx {

// Routed jobs of a launch: every bucket, or under expert parallelism this rank's buckets.
__device__ __forceinline__ int routed_jobs(const MoeShape &sh, const MoeScratch &sc) {
    return sh.ep_size > 1 ? *sc.nu_job : *sc.nu;
}

struct Job {
    const uint8_t *gate, *up, *down;
    int dtype, F, nbF, n, p0;   // rows of gate/up, down's blocks per row, tokens, first pair
    bool shared;
};

__device__ __forceinline__ bool get_job(const MoeShape &sh, const MoeLayerDev &L, const MoeScratch &sc, int u,
                                        int nu, Job &j) {
    if (u < nu) {
        if (sh.ep_size > 1) u = sc.ujob[u];   // job -> bucket
        const int e = sc.ulist[u];
        const uint8_t *slab = L.slab[e];
        if (!slab) {
            set_error(sc.err, DEV_E_NOT_RESIDENT);
            return false;
        }
        j.gate = slab;
        j.up = slab + L.off_up;
        j.down = slab + L.off_down;
        j.dtype = L.expert_dtype;
        j.F = sh.F;
        j.n = sc.u_n[u];
        j.p0 = sc.u_p0[u];
        j.shared = false;
    } else {
        j.gate = L.sh_gate;
        j.up = L.sh_up;
        j.down = L.sh_down;
        j.dtype = L.sh_dtype;
        j.F = L.Fs;
        j.n = sh.T;
        j.p0 = sh.T * sh.route.K;
        j.shared = true;
    }
    j.nbF = j.F / QK;
    if (j.dtype != Q4 && j.dtype != Q8) {
        set_error(sc.err, DEV_E_BAD_DTYPE);
        return false;
    }
    return true;
}

__device__ __forceinline__ int job_token(const MoeScratch &sc, const Job &j, int i) {
    return j.shared ? i : sc.pair_tok[j.p0 + i];
}

}  // namespace hx
