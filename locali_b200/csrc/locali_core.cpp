// Slot-residency planner behind include/locali_core.h.
//
// Host policy that decides which arena slot each (layer, expert) key lives in
// (the role of the reference's native/locali_core.c, driven from
// dsv4_arena.py:68-127).  Behaviour follows the reference planner:
//   * SLRU: new keys enter a fixed-size probation segment; a hit promotes a
//     probation key to the protected segment (capped, the oldest protected key
//     is demoted back), locali_core.c:79-98.  A miss takes a free slot while
//     probation has room, otherwise evicts the least recent unpinned probation
//     key, then the least recent unpinned protected key (:112-141).
//   * LFU-decay: every access bumps a saturating counter and a clock; a miss
//     takes a free slot, else evicts the unpinned probation key with the lowest
//     counter, oldest first (:143-182); every 16 noted tokens halve all counters.
//   * Slots named in `pinned_slots` for a plan call are never evicted by it.
// Memory is allocated once in create(); plan() performs no allocation.
#include "../../include/locali_core.h"

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>
#include <vector>

namespace {

constexpr uint8_t kNone = 0, kProbation = 1, kProtected = 2;

struct Segment {
    int32_t head = -1, tail = -1, size = 0;
};

}  // namespace

struct locali_cache {
    int32_t nkeys = 0, nslots = 0, prot_cap = 0, prob_cap = 0, policy = 0;
    uint32_t tokens = 0, epoch = 0;
    uint64_t clock = 0;
    Segment seg[3];  // indexed by kProbation / kProtected
    std::vector<int32_t> slot_of, key_at, prev, next, free_stack;
    std::vector<uint8_t> where;
    std::vector<uint32_t> heat, pin_epoch;
    std::vector<uint64_t> stamp;

    bool valid(int32_t key) const { return key >= 0 && key < nkeys; }

    void unlink(int32_t key) {
        Segment &s = seg[where[key]];
        const int32_t p = prev[key], n = next[key];
        (p >= 0 ? next[p] : s.head) = n;
        (n >= 0 ? prev[n] : s.tail) = p;
        prev[key] = next[key] = -1;
        where[key] = kNone;
        --s.size;
    }

    void push_back(int32_t key, uint8_t which) {
        Segment &s = seg[which];
        prev[key] = s.tail;
        next[key] = -1;
        (s.tail >= 0 ? next[s.tail] : s.head) = key;
        s.tail = key;
        where[key] = which;
        ++s.size;
    }

    bool pinned(int32_t slot) const { return slot >= 0 && pin_epoch[slot] == epoch; }

    int32_t oldest_unpinned(uint8_t which) const {
        for (int32_t k = seg[which].head; k >= 0; k = next[k])
            if (!pinned(slot_of[k])) return k;
        return -1;
    }

    // Recency refresh on a hit (SLRU promotion when a protected segment exists).
    void refresh(int32_t key) {
        if (where[key] == kProtected) {
            unlink(key);
            push_back(key, kProtected);
        } else if (prot_cap == 0) {
            unlink(key);
            push_back(key, kProbation);
        } else {
            unlink(key);
            push_back(key, kProtected);
            if (seg[kProtected].size > prot_cap) {
                const int32_t old = seg[kProtected].head;
                unlink(old);
                push_back(old, kProbation);
            }
        }
    }

    void bind(int32_t key, int32_t slot) {
        slot_of[key] = slot;
        key_at[slot] = key;
        push_back(key, kProbation);
    }

    int32_t take_victim_slot(int32_t victim, int32_t *evicted) {
        const int32_t slot = slot_of[victim];
        *evicted = victim;
        unlink(victim);
        slot_of[victim] = -1;
        key_at[slot] = -1;
        return slot;
    }

    bool place_slru(int32_t key, int32_t *slot, int32_t *evicted) {
        const bool prob_full = seg[kProbation].size >= prob_cap;
        const bool have_free = !free_stack.empty();
        int32_t victim = -1;
        if (prob_full || !have_free) victim = oldest_unpinned(kProbation);
        if (victim < 0 && !prob_full && have_free) {
            *slot = free_stack.back();
            free_stack.pop_back();
        } else {
            if (victim < 0) victim = oldest_unpinned(kProtected);
            if (victim < 0) return false;
            *slot = take_victim_slot(victim, evicted);
        }
        bind(key, *slot);
        return true;
    }

    int32_t coldest_unpinned() const {
        int32_t best = -1;
        uint32_t best_heat = UINT32_MAX;
        uint64_t best_stamp = UINT64_MAX;
        for (int32_t k = seg[kProbation].head; k >= 0; k = next[k]) {
            if (pinned(slot_of[k])) continue;
            if (heat[k] < best_heat || (heat[k] == best_heat && stamp[k] < best_stamp)) {
                best = k;
                best_heat = heat[k];
                best_stamp = stamp[k];
            }
        }
        return best;
    }

    bool place_lfu(int32_t key, int32_t *slot, int32_t *evicted) {
        if (!free_stack.empty()) {
            *slot = free_stack.back();
            free_stack.pop_back();
        } else {
            const int32_t victim = coldest_unpinned();
            if (victim < 0) return false;
            *slot = take_victim_slot(victim, evicted);
        }
        bind(key, *slot);
        return true;
    }
};

extern "C" {

locali_cache *locali_cache_create(int32_t key_capacity, int32_t slots, int32_t protected_capacity) {
    return locali_cache_create_policy(key_capacity, slots, protected_capacity, LOCALI_CACHE_SLRU);
}

locali_cache *locali_cache_create_policy(int32_t key_capacity, int32_t slots, int32_t protected_capacity,
                                         int32_t policy) {
    if (key_capacity <= 0 || slots < 2 || protected_capacity < 0 || protected_capacity >= slots) return nullptr;
    if (policy != LOCALI_CACHE_SLRU && policy != LOCALI_CACHE_LFU_DECAY) return nullptr;
    locali_cache *c = new (std::nothrow) locali_cache();
    if (!c) return nullptr;
    try {
        c->nkeys = key_capacity;
        c->nslots = slots;
        c->policy = policy;
        c->prot_cap = policy == LOCALI_CACHE_LFU_DECAY ? 0 : protected_capacity;
        c->prob_cap = slots - 1 - c->prot_cap;
        c->slot_of.assign(key_capacity, -1);
        c->prev.assign(key_capacity, -1);
        c->next.assign(key_capacity, -1);
        c->where.assign(key_capacity, kNone);
        c->heat.assign(key_capacity, 0);
        c->stamp.assign(key_capacity, 0);
        c->key_at.assign(slots, -1);
        c->pin_epoch.assign(slots, 0);
        // slot 0 is the reserved zero slot; the stack hands out the highest first
        c->free_stack.reserve(slots - 1);
        for (int32_t s = 1; s < slots; ++s) c->free_stack.push_back(s);
    } catch (...) {
        delete c;
        return nullptr;
    }
    return c;
}

void locali_cache_destroy(locali_cache *cache) { delete cache; }

void locali_cache_note_token(locali_cache *cache) {
    if (!cache || cache->policy != LOCALI_CACHE_LFU_DECAY) return;
    if (++cache->tokens % 16u != 0u) return;
    for (uint32_t &h : cache->heat) h >>= 1;
}

int locali_cache_plan(locali_cache *cache, const int32_t *keys, size_t key_count, const int32_t *pinned_slots,
                      size_t pinned_count, int touch_hits, locali_cache_result *results) {
    if (!cache || (!keys && key_count) || (!results && key_count)) return -1;
    if (++cache->epoch == 0) {
        std::fill(cache->pin_epoch.begin(), cache->pin_epoch.end(), 0u);
        cache->epoch = 1;
    }
    for (size_t i = 0; i < pinned_count; ++i) {
        const int32_t s = pinned_slots[i];
        if (s > 0 && s < cache->nslots) cache->pin_epoch[s] = cache->epoch;
    }
    const bool lfu = cache->policy == LOCALI_CACHE_LFU_DECAY;
    for (size_t i = 0; i < key_count; ++i) {
        const int32_t key = keys[i];
        if (!cache->valid(key)) return -3;
        locali_cache_result r;
        r.key = key;
        r.slot = -1;
        r.evicted_key = -1;
        r.hit = 0;
        r.placed = 0;
        if (lfu) {
            if (cache->heat[key] < UINT32_MAX) ++cache->heat[key];
            cache->stamp[key] = ++cache->clock;
        }
        if (cache->slot_of[key] >= 0) {
            r.hit = 1;
            r.placed = 1;
            r.slot = cache->slot_of[key];
            if (touch_hits && !lfu) cache->refresh(key);
        } else {
            const bool ok = lfu ? cache->place_lfu(key, &r.slot, &r.evicted_key)
                                : cache->place_slru(key, &r.slot, &r.evicted_key);
            r.placed = ok ? 1 : 0;
        }
        results[i] = r;
    }
    return 0;
}

int32_t locali_cache_peek(const locali_cache *cache, int32_t key) {
    return (cache && cache->valid(key)) ? cache->slot_of[key] : -1;
}

int32_t locali_cache_probation_size(const locali_cache *cache) {
    return cache ? cache->seg[kProbation].size : -1;
}

int32_t locali_cache_protected_size(const locali_cache *cache) {
    return cache ? cache->seg[kProtected].size : -1;
}

}  // extern "C"
