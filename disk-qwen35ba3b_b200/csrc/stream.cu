// stream.cu -- pools larger than HBM: the reference's routed-expert cache
// (src/cache.c:140-214, include/ds4f/ds4f.h:181-232) over an HBM slot
// arena, filled from a pinned host copy of the packed pool instead of by
// pread from disk. Host code only.
//
// Policy (as the reference's, so a streamed run fetches exactly what the
// reference's cache would read): a slot holds EMPTY, INFLIGHT or the key
// (layer + 1, expert + 1). A request for n experts
//   1. reserves serially: a resident key is a hit; otherwise the victim is
//      the first EMPTY slot, else the non-pinned, non-INFLIGHT slot fetched
//      longest ago (hits do not refresh it); none left: a drop (slot -1);
//   2. fetches the reserved slots in pool-offset order;
//   3. publishes them in that order, each taking the next clock value.
// One departure, behind `guard` (the streaming model sets it): in the
// reference a slot answered as a hit in step 1 stays a victim candidate for
// the request's later misses, so two selections can end up on one slot and
// the earlier one reads the other expert's bytes (src/cache.c:150-170 with
// src/main.c:729-733). Guarded, the request's hits are not evicted and an
// expert named twice shares one slot; every other decision is the
// reference's.
#include <algorithm>
#include <cstring>
#include <set>
#include <new>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "matvec.cuh"
#include "model.cuh"
#include "../../include/ds4f/gpu_cuda.h"

namespace ds4f {

struct SlotCache {
    static constexpr uint64_t kEmpty = 0, kInflight = 1;
    static constexpr int kMaxReq = 64;           // DS4F_MAX_TOPK
    int nslot = 0;
    std::vector<uint64_t> key, used_at;
    std::vector<uint8_t> pinned;
    // live key -> the slots holding it (more than one only when a request
    // of the unguarded policy names an expert twice); a lookup answers the
    // lowest, as the reference's linear scan does
    std::unordered_map<uint64_t, std::set<int>> where;
    std::vector<uint8_t> held;                   // guard: this request's hits
    // The victim order kept sorted instead of scanned: free slots by index,
    // and the live slots that may be evicted (not pinned, not held) by their
    // fetch clock, which is unique per slot -- so the first of each is the
    // slot the reference's linear scan picks, in O(log n).
    std::set<int> empty_slots;
    std::set<std::pair<uint64_t, int>> lru;
    uint64_t clock = 0;
    int64_t nreq = 0, nhit = 0, ndrop = 0, nfetch = 0;
    bool guard = false;

    SlotCache(int n, bool g) : nslot(n), key(n, kEmpty), used_at(n, 0), pinned(n, 0), held(n, 0), guard(g) {
        for (int i = 0; i < n; i++) empty_slots.insert(empty_slots.end(), i);
    }

    static uint64_t expert_key(int layer, int expert) {
        return ((uint64_t)(uint32_t)(layer + 1) << 32) | (uint32_t)(expert + 1);
    }
    bool evictable(int s) const { return key[s] > kInflight && !pinned[s] && !held[s]; }
    // the first EMPTY slot, else the evictable slot fetched longest ago
    int victim() const {
        if (!empty_slots.empty()) return *empty_slots.begin();
        return lru.empty() ? -1 : lru.begin()->second;
    }
    void set_pin(int s, bool on) {
        const bool was = evictable(s);
        pinned[s] = on;
        const bool now = evictable(s);
        if (was && !now) lru.erase({used_at[s], s});
        if (!was && now) lru.insert({used_at[s], s});
    }
    void hold(int s) {
        if (held[s]) return;
        if (evictable(s)) lru.erase({used_at[s], s});
        held[s] = 1;
    }
    // Slot s stops holding its key: O(log n).
    void forget(int s) {
        auto it = where.find(key[s]);
        if (it == where.end()) return;
        it->second.erase(s);
        if (it->second.empty()) where.erase(it);
    }
    // out_slot[j]: the slot of experts[j] (-1: dropped); fetch[] receives the
    // (slot, expert) pairs to copy in, in pool-offset order, already
    // published. Returns their count.
    int getmany(int layer, const int *experts, int n, int *out_slot, std::vector<std::pair<int, int>> &fetch) {
        if (n > kMaxReq) n = kMaxReq;
        fetch.clear();
        nreq += n;
        for (int j = 0; j < n; j++) {
            const uint64_t k = expert_key(layer, experts[j]);
            auto it = where.find(k);
            if (it != where.end()) {
                const int hs = *it->second.begin();
                out_slot[j] = hs;
                nhit++;
                if (guard) hold(hs);
                continue;
            }
            if (guard) {                         // named earlier in this request
                int prev = -1;
                for (int q = 0; q < j && prev < 0; q++)
                    if (experts[q] == experts[j] && out_slot[q] >= 0) prev = out_slot[q];
                if (prev >= 0) { out_slot[j] = prev; nhit++; continue; }
            }
            const int s = victim();
            if (s < 0) { out_slot[j] = -1; ndrop++; continue; }
            if (key[s] == kEmpty) {
                empty_slots.erase(s);
            } else {
                lru.erase({used_at[s], s});
                forget(s);
            }
            key[s] = kInflight;
            fetch.emplace_back(s, experts[j]);
            out_slot[j] = s;
        }
        // pool offsets grow with the expert index within a layer; stable, as
        // the reference's insertion sort
        std::stable_sort(fetch.begin(), fetch.end(),
                         [](const std::pair<int, int> &a, const std::pair<int, int> &b) { return a.second < b.second; });
        for (const auto &f : fetch) {
            const uint64_t k = expert_key(layer, f.second);
            key[f.first] = k;
            used_at[f.first] = ++clock;
            if (evictable(f.first)) lru.insert({used_at[f.first], f.first});
            where[k].insert(f.first);
        }
        if (guard)
            for (int j = 0; j < n; j++) {
                const int h = out_slot[j];
                if (h >= 0 && held[h]) {
                    held[h] = 0;
                    if (evictable(h)) lru.insert({used_at[h], h});
                }
            }
        nfetch += (int64_t)fetch.size();
        return (int)fetch.size();
    }
};

// The streaming layer step's fetch: the K selections' routing (device,
// m->w.idx) read back, the cache consulted, the misses copied from the pinned
// host pool into their arena slots, and the selections' slots uploaded to
// m->slot_dev -- all ordered on `st` before the chain kernels.
int stream_fetch(Model *m, int L, cudaStream_t st) {
    const int K = m->d.topk, E = m->d.n_experts;
    const int64_t sb = m->slot.nbytes;
    DS4F_CUDA(cudaMemcpyAsync(m->idx_h, m->w.idx, K * 4, cudaMemcpyDeviceToHost, st));
    DS4F_CUDA(cudaStreamSynchronize(st));
    // the routing indexes the host pool: a value outside [0, E) (the top-K
    // always writes valid experts; this guards the host read) stops here
    for (int j = 0; j < K; j++)
        DS4F_REQUIRE(m->idx_h[j] >= 0 && m->idx_h[j] < E, "stream: selection %d of layer %d is expert %d, "
                     "outside [0, %d)", j, L, m->idx_h[j], E);
    std::vector<std::pair<int, int>> fetch;
    m->cache->getmany(L, m->idx_h, K, m->slot_h, fetch);
    for (int j = 0; j < K; j++)
        DS4F_REQUIRE(m->slot_h[j] >= 0, "stream: no free slot for expert %d of layer %d (every slot pinned or "
                     "in flight)", m->idx_h[j], L);
    for (const auto &f : fetch) {
        uint8_t *dst = m->pool + (int64_t)f.first * sb;
        DS4F_CUDA(cudaMemcpyAsync(dst, m->host_pool + ((int64_t)L * E + f.second) * sb, sb, cudaMemcpyHostToDevice,
                                  st));
        if (m->d.fmt == DS4F_FMT_FP8)    // e=15 bytes -> +-448, as on every upload
            for (int t = 0; t < 3; t++)
                if (launch_f8_canon(dst + m->slot.rel_v[t], m->slot.rel_s[t] - m->slot.rel_v[t], st)) return -1;
    }
    DS4F_CUDA(cudaMemcpyAsync(m->slot_dev, m->slot_h, K * 4, cudaMemcpyHostToDevice, st));
    return 0;
}

SlotCache *slot_cache_new(int n) { return new (std::nothrow) SlotCache(n, true); }
void slot_cache_delete(SlotCache *c) { delete c; }
void slot_cache_stats(const SlotCache *c, int64_t *req, int64_t *hit, int64_t *drop, int64_t *fetched) {
    if (req) *req = c->nreq;
    if (hit) *hit = c->nhit;
    if (drop) *drop = c->ndrop;
    if (fetched) *fetched = c->nfetch;
}

}  // namespace ds4f

// ---- the policy on its own (no device): for hosts that manage their own
// ---- arena, and for checking it against the reference's cache -----------
struct Ds4fSlotCache { ds4f::SlotCache c; Ds4fSlotCache(int n, bool g) : c(n, g) {} };

extern "C" {

int ds4f_slotcache_create(int n_slots, int flags, Ds4fSlotCache **out) {
    DS4F_REQUIRE(out && n_slots > 0 && !(flags & ~DS4F_SLOTCACHE_GUARD), "slotcache_create: bad arguments");
    *out = new (std::nothrow) Ds4fSlotCache(n_slots, (flags & DS4F_SLOTCACHE_GUARD) != 0);
    DS4F_REQUIRE(*out, "slotcache_create: out of host memory");
    return 0;
}

void ds4f_slotcache_free(Ds4fSlotCache *c) { delete c; }

int ds4f_slotcache_getmany(Ds4fSlotCache *c, int layer, const int *experts, int n, int *out_slot) {
    DS4F_REQUIRE(c && experts && out_slot && n >= 0, "slotcache_getmany: bad arguments");
    // the policy knows no pool, so the upper bound of an expert index is the
    // caller's to check against its own; a negative one (the reference's key
    // would then collide with the empty slot's) is refused
    for (int j = 0; j < n && j < ds4f::SlotCache::kMaxReq; j++)
        DS4F_REQUIRE(experts[j] >= 0 && layer >= 0, "slotcache_getmany: negative layer %d or expert %d (entry %d)",
                     layer, experts[j], j);
    std::vector<std::pair<int, int>> fetch;
    return c->c.getmany(layer, experts, n, out_slot, fetch);
}

int ds4f_slotcache_pin(Ds4fSlotCache *c, int slot, int pin) {
    DS4F_REQUIRE(c, "slotcache_pin: null cache");
    if (slot >= 0 && slot < c->c.nslot) c->c.set_pin(slot, pin != 0);
    return 0;
}

int ds4f_slotcache_stats(const Ds4fSlotCache *c, int64_t *requests, int64_t *hits, int64_t *drops,
                         int64_t *fetched) {
    DS4F_REQUIRE(c, "slotcache_stats: null cache");
    ds4f::slot_cache_stats(&c->c, requests, hits, drops, fetched);
    return 0;
}

}  // extern "C"
