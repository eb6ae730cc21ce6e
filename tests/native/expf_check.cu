// Host-side exhaustive check of the device expf restatement (hx::host_expf compiled for the
// host from the product header) against the host C library's expf. Test support only.
#include "../../hearth_b200/csrc/hx_common.cuh"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

extern "C" long long hxt_expf_mismatches(uint64_t lo, uint64_t hi, int n_threads, uint32_t *first_bad) {
    std::vector<long long> bad((size_t)n_threads, 0);
    std::vector<uint32_t> fb((size_t)n_threads, 0);
    std::vector<std::thread> th;
    for (int t = 0; t < n_threads; t++)
        th.emplace_back([&, t] {
            long long b = 0;
            for (uint64_t u = lo + (uint64_t)t; u < hi; u += (uint64_t)n_threads) {
                const uint32_t v = (uint32_t)u;
                float x;
                std::memcpy(&x, &v, 4);
                const float a = expf(x), c = hx::host_expf(x);
                uint32_t ua, uc;
                std::memcpy(&ua, &a, 4);
                std::memcpy(&uc, &c, 4);
                if (ua != uc && !(a != a && c != c)) {
                    if (!b) fb[(size_t)t] = v;
                    b++;
                }
            }
            bad[(size_t)t] = b;
        });
    long long tot = 0;
    for (int t = 0; t < n_threads; t++) {
        th[(size_t)t].join();
        if (bad[(size_t)t] && first_bad && !tot) *first_bad = fb[(size_t)t];
        tot += bad[(size_t)t];
    }
    return tot;
}

extern "C" void hxt_exp2_table(uint64_t *out) {
    for (int i = 0; i < 32; i++) out[i] = hx::kExp2TabHost[i];
}
