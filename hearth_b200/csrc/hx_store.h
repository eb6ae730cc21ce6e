// hx_store.h — the HBM-resident expert store of the B200 backend.
//
// Replaces the reference's NVMe -> DRAM store (engine/src/hx_store.h, engine/src/store.c) with a
// host DRAM -> HBM store: a fixed arena of slab-sized slots in device memory, slot_of[layer*E+e]
// direct indexing, LRU or LFU (decayed per-token heat) eviction, pinned slots from a heat profile,
// demand requests (never dropped) and prefetch hints (dropped when no unprotected, cold slot is
// free). A "read" is an asynchronous cudaMemcpyAsync from a pinned host copy of the slab on the
// store's copy stream; its completion is a CUDA event, so the compute stream waits for it on the
// device (cudaStreamWaitEvent) instead of a host thread blocking on a condition variable. A slot
// is overwritten only after the compute that last read it has finished (the copy stream waits on
// the slot's release event).
//
// Single caller thread (the engine's), like the reference's compute side; no reader threads are
// needed because the copy engines are the readers.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>
#include <vector>

#include <cuda_runtime.h>

namespace hx {

enum : int { POLICY_LRU = 0, POLICY_LFU = 1 };

struct StoreStats {
    uint64_t hits = 0, misses = 0, evictions = 0;
    uint64_t prefetch_issued = 0, prefetch_used = 0, prefetch_wasted = 0;
    uint64_t bytes_copied = 0, copies = 0, copy_errors = 0;
    double stall_s = 0.0;
};

class HbmStore {
public:
    // Test seam (the counterpart of hx_store_set_read_hook): called before every copy is issued;
    // a nonzero return fails that copy the way a failed slab read fails in the reference.
    using CopyHook = std::function<int(int layer, int expert)>;

    HbmStore() = default;
    ~HbmStore();
    HbmStore(const HbmStore &) = delete;
    HbmStore &operator=(const HbmStore &) = delete;

    // n_slots slots of slot_bytes in HBM for L*E keys. Returns false with a message on failure.
    bool open(int L, int E, size_t slot_bytes, int n_slots, int policy, float heat_decay, std::string &err);
    void close();

    // The host source of a key: the store copies the bytes into its own pinned host memory.
    bool set_source(int layer, int expert, const void *bytes, size_t n, std::string &err);
    // An aliased expert (a container entry that names another entry's slab): its host source is the
    // other expert's pinned copy, shared rather than copied. Its slot, counters and policy state stay
    // its own. A later set_source of either side gives the aliases the new bytes too.
    bool share_source(int layer, int expert, int src_layer, int src_expert, std::string &err);
    size_t host_bytes() const;   // pinned host bytes held by the host tier
    std::vector<int> aliases_of(int layer, int expert) const;   // experts sharing this one's source
    // Slab bytes generated directly in a slot (synthetic weights): makes the key resident.
    uint8_t *place_resident(int layer, int expert);

    // Non-blocking: resident -> the slab's device pointer (refs++) and *ready = nullptr; in flight
    // or just requested -> the slot's device pointer with *ready = the event the compute stream
    // must wait for (refs++ as well, so it is not evicted before use); nullptr when the expert
    // cannot be brought in now (no evictable slot, or its copy failed this token).
    const uint8_t *acquire_async(int layer, int expert, cudaEvent_t *ready);
    // Unpin; `done` (recorded on the compute stream after the last kernel that reads the slab)
    // guards the slot against being overwritten early. done may be null (already complete).
    void release(int layer, int expert, cudaStream_t compute);
    void count_uses(int layer, int expert, uint32_t n);
    void prefetch(int layer, const int *experts, int n);
    void tick();
    bool is_resident(int layer, int expert) const;
    bool all_resident() const { return n_ready_ == (int)slot_of_.size(); }

    // Heat profile (FORMAT.md §8 counts per key): pins the hottest pin_fraction * n_slots keys and,
    // with warm_start, fills the rest with the next hottest (loads issued at once).
    void seed_heat(const float *counts, int n_keys, float pin_fraction, bool warm_start);
    const std::vector<double> &counts() const { return count_; }

    void set_copy_hook(CopyHook h) { hook_ = std::move(h); }
    StoreStats stats() const { return st_; }
    void reset_stats() { st_ = StoreStats(); }
    int n_slots() const { return (int)slots_.size(); }
    int n_ready() const { return n_ready_; }
    int n_pinned() const { return n_pinned_; }
    size_t slot_bytes() const { return slot_bytes_; }
    cudaStream_t copy_stream() const { return copy_; }
    uint8_t *slot_ptr(int si) const { return arena_ + (size_t)si * slot_bytes_; }
    int slot_of(int layer, int expert) const { return slot_of_[(size_t)layer * E_ + expert]; }
    bool copy_failed_now(int layer, int expert) const { return failed_[(size_t)layer * E_ + expert] != 0; }

private:
    enum : int { FREE = 0, LOADING = 1, READY = 2 };
    struct Slot {
        int key = -1, state = FREE, refs = 0;
        bool pinned = false, pf_unused = false, used_once = false;
        uint64_t prot_tick = 0, last_seq = 0, last_tick = 0;
        cudaEvent_t ready = nullptr;   // copy completion
        cudaEvent_t done = nullptr;    // last compute use
        bool done_recorded = false;
    };
    double eff_heat(int key) const;
    bool evictable(const Slot &s) const;
    bool cheaper(int a, int b) const;
    int pick_victim(bool allow_protected) const;
    int slot_for(bool demand);
    bool issue_copy(int si, int key, bool demand);
    void settle(Slot &s);   // LOADING -> READY once its event completed
    void wait_loading(size_t key);      // the key's copy in flight (if any) has landed
    void refresh_slot(size_t key);      // after new source bytes: drop the key's slot, or re-copy a pinned one
    void count_use(int key, double n);

    int L_ = 0, E_ = 0, policy_ = POLICY_LFU;
    double decay_ = 0.995, hot_heat_ = 0.0;
    size_t slot_bytes_ = 0;
    uint8_t *arena_ = nullptr;
    cudaStream_t copy_ = nullptr;
    std::vector<Slot> slots_;
    std::vector<int> slot_of_, free_;
    std::vector<uint8_t *> host_;       // pinned host copies (host tier)
    std::vector<int64_t> host_owner_;   // key whose pinned buffer host_[key] is (-1: no source)
    std::vector<size_t> host_n_;
    std::vector<double> heat_, count_;
    std::vector<uint64_t> heat_tick_;
    std::vector<uint8_t> failed_;
    int n_ready_ = 0, n_pinned_ = 0;
    uint64_t now_ = 0, seq_ = 0;
    StoreStats st_;
    CopyHook hook_;
};

}  // namespace hx
