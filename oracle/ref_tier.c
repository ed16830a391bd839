/* ref_tier.c -- build harness around the REFERENCE header include/tier.h.
 *
 * TEST INFRASTRUCTURE ONLY.  tier.h is #included from where it lies (the
 * Makefile puts the reference's include/ on the path) and compiled into
 * oracle/_ref/libref_tier.so; its static functions are exported under
 * ref_tier_* names, unchanged, so tests can compare the restatement in
 * moe_oracle.c (and the library's own policy) with them. */
#include <stdint.h>

#include "tier.h"

int ref_tier_pick_swap(const uint32_t *heat, int nexpert, const int *pinned, int npin, int *slot, int *eid,
                       long *gain) {
    return tier_pick_swap(heat, nexpert, pinned, npin, slot, eid, gain);
}

uint64_t ref_tier_lfru_score(uint32_t heat, uint32_t last, uint32_t clock) { return tier_lfru_score(heat, last, clock); }

int ref_tier_pick_lfru(const uint32_t *heat, const uint32_t *last, uint32_t clock, int nexpert, const int *pinned,
                       int npin, int *slot, int *eid, long *gain) {
    return tier_pick_lfru(heat, last, clock, nexpert, pinned, npin, slot, eid, gain);
}

void ref_tier_decay(uint32_t *heat, int nexpert) { tier_decay(heat, nexpert); }
