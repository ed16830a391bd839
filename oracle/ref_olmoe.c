/* ref_olmoe.c -- build harness around the REFERENCE engine engines/olmoe.c.
 *
 * TEST INFRASTRUCTURE ONLY.  The reference source is not copied: it is
 * #included from where it lies (REF_OLMOE_C, passed by oracle/Makefile) and
 * compiled into oracle/_ref/libref_olmoe.so.  Its `main` is renamed
 * ref_olmoe_main so the unmodified file links as a library.
 *
 * ref_olmoe_moe() calls the reference's own static moe()
 * (engines/olmoe.c:344-402) on caller-supplied weights: the harness fills the
 * per-layer LRU cache (engines/olmoe.c:52-53) with every expert up front
 * (cap = n = E), so expert_get (engines/olmoe.c:250-272) always hits and
 * never touches disk.
 */
#define main ref_olmoe_main
#include REF_OLMOE_C
#undef main

int ref_olmoe_moe(int D, int E, int K, int I, int norm_topk,
                  const float *x, int S, const float *gate,
                  const int8_t *g, const float *gs, const int8_t *u, const float *us,
                  const int8_t *d, const float *ds, float *out) {
    Model m;
    memset(&m, 0, sizeof(m));
    m.c.hidden = D; m.c.n_experts = E; m.c.topk = K; m.c.inter = I;
    m.c.norm_topk = norm_topk; m.c.n_layers = 1; m.quant_bits = 8;
    Layer L;
    memset(&L, 0, sizeof(L));
    L.gate = (float *)gate;
    Slot *slots = calloc((size_t)E, sizeof(Slot));
    if (!slots) return -1;
    for (int e = 0; e < E; e++) {
        slots[e].eid = e;
        slots[e].g  = (int8_t *)g + (int64_t)e * I * D;
        slots[e].u  = (int8_t *)u + (int64_t)e * I * D;
        slots[e].d  = (int8_t *)d + (int64_t)e * D * I;
        slots[e].gs = (float *)gs + (int64_t)e * I;
        slots[e].us = (float *)us + (int64_t)e * I;
        slots[e].ds = (float *)ds + (int64_t)e * D;
    }
    LCache lc = { slots, E, E };
    m.cache = &lc;
    m.L = &L;
    moe(&m, &L, 0, (float *)x, S, out);
    free(slots);
    return 0;
}
