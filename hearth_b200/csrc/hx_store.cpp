// hx_store.cpp — the HBM expert store (see hx_store.h). Policy follows the reference's store
// (engine/src/store.c): victim choice pick_victim/cheaper (150-196), demand vs prefetch slot
// rules slot_for_demand/slot_for_prefetch (198-215), hits/misses per use (435-446), failed reads
// retried after the next tick (563-580), heat-profile pins and warm start (815-860).
#include "hx_store.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>

namespace hx {

HbmStore::~HbmStore() { close(); }

bool HbmStore::open(int L, int E, size_t slot_bytes, int n_slots, int policy, float heat_decay, std::string &err) {
    close();
    if (L <= 0 || E <= 0 || slot_bytes == 0 || n_slots <= 0) {
        err = "store: bad geometry";
        return false;
    }
    L_ = L;
    E_ = E;
    slot_bytes_ = slot_bytes;
    policy_ = policy == POLICY_LRU ? POLICY_LRU : POLICY_LFU;
    decay_ = heat_decay > 0.0f && heat_decay <= 1.0f ? heat_decay : 0.995;
    hot_heat_ = decay_ < 1.0 ? 0.5 / (1.0 - decay_) : 1e300;
    if (cudaMalloc(&arena_, slot_bytes * (size_t)n_slots) != cudaSuccess) {
        cudaGetLastError();
        arena_ = nullptr;
        err = "store: cannot allocate " + std::to_string(n_slots) + " HBM slots of " + std::to_string(slot_bytes) +
              " bytes";
        return false;
    }
    if (cudaStreamCreateWithFlags(&copy_, cudaStreamNonBlocking) != cudaSuccess) {
        err = "store: cannot create the copy stream";
        close();
        return false;
    }
    slots_.assign((size_t)n_slots, Slot());
    for (auto &s : slots_) {
        if (cudaEventCreateWithFlags(&s.ready, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming) != cudaSuccess) {
            err = "store: cannot create slot events";
            close();
            return false;
        }
    }
    free_.resize((size_t)n_slots);
    for (int i = 0; i < n_slots; i++) free_[(size_t)i] = n_slots - 1 - i;   // pop gives slot 0 first
    const size_t nk = (size_t)L * E;
    slot_of_.assign(nk, -1);
    host_.assign(nk, nullptr);
    host_n_.assign(nk, 0);
    host_owner_.assign(nk, -1);
    heat_.assign(nk, 0.0);
    count_.assign(nk, 0.0);
    heat_tick_.assign(nk, 0);
    failed_.assign(nk, 0);
    n_ready_ = n_pinned_ = 0;
    now_ = seq_ = 0;
    st_ = StoreStats();
    return true;
}

void HbmStore::close() {
    if (copy_) cudaStreamSynchronize(copy_);
    for (auto &s : slots_) {
        if (s.ready) cudaEventDestroy(s.ready);
        if (s.done) cudaEventDestroy(s.done);
    }
    slots_.clear();
    for (size_t k = 0; k < host_.size(); k++)
        if (host_[k] && host_owner_[k] == (int64_t)k) cudaFreeHost(host_[k]);
    host_.clear();
    host_owner_.clear();
    if (copy_) cudaStreamDestroy(copy_);
    copy_ = nullptr;
    if (arena_) cudaFree(arena_);
    arena_ = nullptr;
}

bool HbmStore::set_source(int layer, int expert, const void *bytes, size_t n, std::string &err) {
    if (layer < 0 || layer >= L_ || expert < 0 || expert >= E_ || !bytes || n == 0 || n > slot_bytes_) {
        err = "store: bad expert source";
        return false;
    }
    const size_t key = (size_t)layer * E_ + expert;
    const bool alias = host_owner_[key] >= 0 && host_owner_[key] != (int64_t)key;
    // every copy still reading the buffer this key reads (and, for an owner, its aliases' copies)
    // lands before the buffer is written or freed: no slot can receive half-old, half-new bytes
    wait_loading(key);
    if (!alias)
        for (size_t k = 0; k < host_.size(); k++)
            if (k != key && host_owner_[k] == (int64_t)key) wait_loading(k);
    if (alias || !host_[key] || host_n_[key] != n) {
        uint8_t *p = nullptr;
        if (cudaHostAlloc((void **)&p, n, cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            err = "store: cannot pin host memory for an expert";   // an alias keeps its shared source
            return false;
        }
        uint8_t *old = alias ? nullptr : host_[key];   // an alias detaches; the owner keeps its buffer
        host_[key] = p;
        host_n_[key] = n;
        host_owner_[key] = (int64_t)key;
        if (!alias)
            for (size_t k = 0; k < host_.size(); k++)   // the aliases of this key follow its new buffer
                if (k != key && host_owner_[k] == (int64_t)key) {
                    host_[k] = p;
                    host_n_[k] = n;
                }
        if (old) cudaFreeHost(old);
    }
    std::memcpy(host_[key], bytes, n);
    refresh_slot(key);
    for (size_t k = 0; k < host_.size(); k++)
        if (k != key && host_owner_[k] == (int64_t)key) refresh_slot(k);
    return true;
}

bool HbmStore::share_source(int layer, int expert, int src_layer, int src_expert, std::string &err) {
    if (layer < 0 || layer >= L_ || expert < 0 || expert >= E_ || src_layer < 0 || src_layer >= L_ || src_expert < 0 ||
        src_expert >= E_) {
        err = "store: bad expert";
        return false;
    }
    const size_t key = (size_t)layer * E_ + expert, src = (size_t)src_layer * E_ + src_expert;
    if (key == src) return true;
    if (!host_[src] || host_owner_[src] < 0) {
        err = "store: the shared expert has no source yet";
        return false;
    }
    if (host_owner_[key] == (int64_t)key) {   // its own buffer goes, unless other experts share it
        for (size_t k = 0; k < host_.size(); k++)
            if (k != key && host_owner_[k] == (int64_t)key) {
                err = "store: the expert is the source of other experts";
                return false;
            }
        wait_loading(key);   // a copy from the buffer lands before the buffer is freed
        cudaFreeHost(host_[key]);
    }
    host_[key] = host_[src];
    host_n_[key] = host_n_[src];
    host_owner_[key] = host_owner_[src];
    refresh_slot(key);
    return true;
}

size_t HbmStore::host_bytes() const {
    size_t n = 0;
    for (size_t k = 0; k < host_.size(); k++)
        if (host_[k] && host_owner_[k] == (int64_t)k) n += host_n_[k];
    return n;
}

std::vector<int> HbmStore::aliases_of(int layer, int expert) const {
    std::vector<int> out;
    const size_t key = (size_t)layer * E_ + expert;
    for (size_t k = 0; k < host_.size(); k++)
        if (k != key && host_owner_[k] == (int64_t)key) out.push_back((int)k);
    return out;
}

void HbmStore::wait_loading(size_t key) {
    const int si = slot_of_[key];
    if (si >= 0 && slots_[(size_t)si].state == LOADING) cudaEventSynchronize(slots_[(size_t)si].ready);
}

void HbmStore::refresh_slot(size_t key) {
    const int si = slot_of_[key];
    if (si < 0) return;
    Slot &s = slots_[(size_t)si];
    if (s.state == LOADING) {
        cudaEventSynchronize(s.ready);
        settle(s);
    }
    if (s.refs == 0 && !s.pinned) {   // a resident copy of the older bytes is dropped
        if (s.state == READY) n_ready_--;
        s.key = -1;
        s.state = FREE;
        slot_of_[key] = -1;
        free_.push_back(si);
        return;
    }
    // a pinned slot keeps its place and receives the new bytes (after the compute that last read it)
    if (s.done) cudaEventSynchronize(s.done);
    if (cudaMemcpy(slot_ptr(si), host_[key], host_n_[key], cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        st_.copy_errors++;
    }
}

uint8_t *HbmStore::place_resident(int layer, int expert) {
    const int key = layer * E_ + expert;
    int si = slot_of_[(size_t)key];
    if (si < 0) {
        if (free_.empty()) return nullptr;
        si = free_.back();
        free_.pop_back();
        Slot &s = slots_[(size_t)si];
        s.key = key;
        s.state = READY;
        s.refs = 0;
        s.pf_unused = false;
        slot_of_[(size_t)key] = si;
        n_ready_++;
    }
    return slot_ptr(si);
}

double HbmStore::eff_heat(int key) const {
    const uint64_t dt = now_ - heat_tick_[(size_t)key];
    return heat_[(size_t)key] * std::pow(decay_, (double)dt);
}

void HbmStore::count_use(int key, double n) {
    heat_[(size_t)key] = eff_heat(key) + n;
    heat_tick_[(size_t)key] = now_;
    count_[(size_t)key] += n;
    const int si = slot_of_[(size_t)key];
    if (si >= 0) {
        slots_[(size_t)si].last_seq = ++seq_;
        slots_[(size_t)si].last_tick = now_;
    }
}

bool HbmStore::evictable(const Slot &s) const { return s.state == READY && s.refs == 0 && !s.pinned; }

bool HbmStore::cheaper(int a, int b) const {
    const Slot &x = slots_[(size_t)a], &y = slots_[(size_t)b];
    const bool px = x.prot_tick == now_ + 1, py = y.prot_tick == now_ + 1;
    if (px != py) return px < py;
    if (policy_ == POLICY_LFU) {
        const double hx_ = eff_heat(x.key), hy = eff_heat(y.key);
        if (hx_ != hy) return hx_ < hy;
    }
    if (x.last_seq != y.last_seq) return x.last_seq < y.last_seq;
    return a < b;
}

int HbmStore::pick_victim(bool allow_protected) const {
    int best = -1;
    for (int c = 0; c < (int)slots_.size(); c++)
        if (evictable(slots_[(size_t)c]) && (best < 0 || cheaper(c, best))) best = c;
    if (best >= 0 && !allow_protected && slots_[(size_t)best].prot_tick == now_ + 1) return -1;
    return best;
}

int HbmStore::slot_for(bool demand) {
    if (!free_.empty()) {
        const int si = free_.back();
        free_.pop_back();
        return si;
    }
    // settle finished loads first: they may become victims
    for (auto &s : slots_) settle(s);
    const int v = pick_victim(demand);
    if (v < 0 || demand) return v;
    const Slot &s = slots_[(size_t)v];
    if (policy_ == POLICY_LFU ? eff_heat(s.key) >= hot_heat_ : s.last_tick == now_) return -1;
    return v;
}

void HbmStore::settle(Slot &s) {
    if (s.state == LOADING && cudaEventQuery(s.ready) == cudaSuccess) {
        s.state = READY;
        n_ready_++;
    }
}

bool HbmStore::issue_copy(int si, int key, bool demand) {
    Slot &s = slots_[(size_t)si];
    if (s.state == READY) {   // evict the victim
        slot_of_[(size_t)s.key] = -1;
        n_ready_--;
        st_.evictions++;
        if (s.pf_unused) st_.prefetch_wasted++;
    }
    s.key = -1;
    s.state = FREE;
    const int layer = key / E_, expert = key % E_;
    bool ok = host_[(size_t)key] != nullptr;
    if (ok && hook_ && hook_(layer, expert) != 0) ok = false;
    if (ok && s.done_recorded) ok = cudaStreamWaitEvent(copy_, s.done, 0) == cudaSuccess;
    if (ok)
        ok = cudaMemcpyAsync(slot_ptr(si), host_[(size_t)key], host_n_[(size_t)key], cudaMemcpyHostToDevice, copy_) ==
             cudaSuccess;
    if (ok) ok = cudaEventRecord(s.ready, copy_) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        failed_[(size_t)key] = 1;
        st_.copy_errors++;
        free_.push_back(si);
        return false;
    }
    s.key = key;
    s.state = LOADING;
    s.refs = 0;
    s.pf_unused = !demand;
    s.prot_tick = demand ? 0 : now_ + 1;
    slot_of_[(size_t)key] = si;
    st_.bytes_copied += host_n_[(size_t)key];
    st_.copies++;
    return true;
}

const uint8_t *HbmStore::acquire_async(int layer, int expert, cudaEvent_t *ready) {
    *ready = nullptr;
    if (layer < 0 || layer >= L_ || expert < 0 || expert >= E_) return nullptr;
    const int key = layer * E_ + expert;
    const int si = slot_of_[(size_t)key];
    if (si >= 0) {
        Slot &s = slots_[(size_t)si];
        settle(s);
        if (s.state == READY) st_.hits++;
        else {
            st_.misses++;
            *ready = s.ready;
        }
        if (s.pf_unused) {
            st_.prefetch_used++;
            s.pf_unused = false;
        }
        s.refs++;
        count_use(key, 1.0);
        return slot_ptr(si);
    }
    if (failed_[(size_t)key]) return nullptr;
    st_.misses++;
    const int v = slot_for(true);
    if (v < 0) return nullptr;
    if (!issue_copy(v, key, true)) return nullptr;
    Slot &s = slots_[(size_t)v];
    s.refs = 1;
    count_use(key, 1.0);
    *ready = s.ready;
    return slot_ptr(v);
}

void HbmStore::release(int layer, int expert, cudaStream_t compute) {
    const int key = layer * E_ + expert;
    const int si = slot_of_[(size_t)key];
    if (si < 0 || slots_[(size_t)si].refs <= 0) return;
    Slot &s = slots_[(size_t)si];
    s.refs--;
    if (cudaEventRecord(s.done, compute) == cudaSuccess) s.done_recorded = true;
    else cudaGetLastError();
}

void HbmStore::count_uses(int layer, int expert, uint32_t n) {
    const int key = layer * E_ + expert;
    if (n == 0 || slot_of_[(size_t)key] < 0) return;
    st_.hits += n;
    count_use(key, (double)n);
}

void HbmStore::prefetch(int layer, const int *experts, int n) {
    for (int i = 0; i < n; i++) {
        if (experts[i] < 0 || experts[i] >= E_) continue;
        const int key = layer * E_ + experts[i];
        const int si = slot_of_[(size_t)key];
        if (si >= 0) {
            slots_[(size_t)si].prot_tick = now_ + 1;
            continue;
        }
        if (failed_[(size_t)key] || !host_[(size_t)key]) continue;
        const int v = slot_for(false);
        if (v < 0) continue;   // dropped: no cold, unprotected slot
        if (issue_copy(v, key, false)) st_.prefetch_issued++;
    }
}

void HbmStore::tick() {
    now_++;
    std::fill(failed_.begin(), failed_.end(), (uint8_t)0);
}

bool HbmStore::is_resident(int layer, int expert) const {
    const int si = slot_of_[(size_t)layer * E_ + expert];
    if (si < 0) return false;
    const Slot &s = slots_[(size_t)si];
    return s.state == READY || (s.state == LOADING && cudaEventQuery(s.ready) == cudaSuccess);
}

void HbmStore::seed_heat(const float *counts, int n_keys, float pin_fraction, bool warm_start) {
    const int nk = std::min(n_keys, (int)slot_of_.size());
    std::vector<int> order;
    for (int k = 0; k < nk; k++) {
        heat_[(size_t)k] = count_[(size_t)k] = counts[k] > 0.0f ? (double)counts[k] : 0.0;
        if (counts[k] > 0.0f) order.push_back(k);
    }
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return count_[(size_t)a] > count_[(size_t)b]; });
    int n_pin = (int)(std::min(std::max(pin_fraction, 0.0f), 0.9f) * (float)slots_.size());
    n_pin = std::min(n_pin, (int)order.size());
    size_t i = 0;
    for (; i < order.size() && n_pinned_ < n_pin && !free_.empty(); i++) {
        const int key = order[i];
        if (slot_of_[(size_t)key] >= 0 || !host_[(size_t)key]) continue;
        const int si = free_.back();
        free_.pop_back();
        if (issue_copy(si, key, true)) {
            slots_[(size_t)si].pinned = true;
            n_pinned_++;
        }
    }
    if (warm_start)
        for (; i < order.size() && !free_.empty(); i++) {
            const int key = order[i];
            if (slot_of_[(size_t)key] >= 0 || !host_[(size_t)key]) continue;
            const int si = free_.back();
            free_.pop_back();
            issue_copy(si, key, true);
        }
}

}  // namespace hx
