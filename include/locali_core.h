/*
 * locali_core.h - slot-residency planner ABI (liblocali_core.so).
 *
 * Same C interface as the reference's native/locali_core.h (declarations
 * there at native/locali_core.h:12-48) so that locali_native.py-style ctypes
 * bindings and the arena's _place_keys (dsv4_arena.py:68-127) keep working
 * unchanged; the implementation (locali_b200/csrc/locali_core.cpp) is this
 * project's own C++.  Host-side policy only: SLRU (probation + protected
 * segments, pinned-slot aware) or LFU with periodic decay.  Allocation-free
 * after create; not thread-safe (single caller).
 */
#ifndef LOCALI_CORE_H
#define LOCALI_CORE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct locali_cache locali_cache;

enum {
    LOCALI_CACHE_SLRU = 0,      /* reference locali_core.h:14 */
    LOCALI_CACHE_LFU_DECAY = 1, /* reference locali_core.h:15 */
};

/* One planned key (reference locali_core.h:18-24). */
typedef struct {
    int32_t key;
    int32_t slot;        /* arena slot, -1 when not placed */
    int32_t evicted_key; /* key that lost the slot, -1 if none */
    uint8_t hit;
    uint8_t placed;
} locali_cache_result;

/* SLRU planner; NULL on invalid sizes (reference locali_cache_create). */
locali_cache *locali_cache_create(int32_t key_capacity, int32_t slots, int32_t protected_capacity);
/* Planner with an explicit policy (reference locali_cache_create_policy). */
locali_cache *locali_cache_create_policy(int32_t key_capacity, int32_t slots,
                                         int32_t protected_capacity, int32_t policy);
void locali_cache_destroy(locali_cache *cache);
/* One decode token passed (LFU: halve every counter each 16 tokens). */
void locali_cache_note_token(locali_cache *cache);
/* Plan keys in order; pinned slots are never evicted.  0 ok, -1 bad
 * arguments, -3 invalid key (reference locali_core.c:259-313). */
int locali_cache_plan(locali_cache *cache, const int32_t *keys, size_t key_count,
                      const int32_t *pinned_slots, size_t pinned_count, int touch_hits,
                      locali_cache_result *results);
int32_t locali_cache_peek(const locali_cache *cache, int32_t key);
int32_t locali_cache_probation_size(const locali_cache *cache);
int32_t locali_cache_protected_size(const locali_cache *cache);

#ifdef __cplusplus
}
#endif

#endif
