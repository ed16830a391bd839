/* ref_qwen.c -- build harness around the REFERENCE engine engines/qwen.c.
 *
 * TEST INFRASTRUCTURE ONLY.  The reference source is #included from where it
 * lies (REF_QWEN_C, passed by oracle/Makefile) and compiled into
 * oracle/_ref/libref_qwen.so; its `main` is renamed ref_qwen_main.
 *
 * ref_qwen_moe() runs the reference's own static moe_step()
 * (engines/qwen.c:453-495) in stream mode (m->stream = 1: int8 router,
 * int8 shared expert, int8 routed experts through the LRU), token by token
 * as the engine does (engines/qwen.c:588,637).  The LRU (engines/qwen.c:
 * 428-450) is pre-filled with every expert, so it never reads disk.
 *
 * ref_qwen_tiny_moe() loads a snapshot with the reference's model_init
 * (engines/qwen.c:211-298, f32-resident when the experts are f32) and runs
 * moe_step of one layer: used to dump golden vectors from the reference's
 * own fixture model oracle/qwen_tiny.
 */
#define main ref_qwen_main
#include REF_QWEN_C
#undef main

int ref_qwen_moe(int D, int E, int K, int MI, int SI,
                 const int8_t *router_q, const float *router_s,
                 const int8_t *sh_g, const float *sh_gs, const int8_t *sh_u, const float *sh_us,
                 const int8_t *sh_d, const float *sh_ds, const float *sh_gate,
                 const int8_t *g, const float *gs, const int8_t *u, const float *us,
                 const int8_t *d, const float *ds,
                 const float *x, int T, float *out) {
    Model m;
    memset(&m, 0, sizeof(m));
    m.c.hidden = D; m.c.n_exp = E; m.c.topk = K; m.c.moe_inter = MI; m.c.shared_inter = SI;
    m.c.n_layers = 1; m.stream = 1;
    Layer L;
    memset(&L, 0, sizeof(L));
    L.Qgate = (QW){ (int8_t *)router_q, (float *)router_s };
    L.Qsg = (QW){ (int8_t *)sh_g, (float *)sh_gs };
    L.Qsu = (QW){ (int8_t *)sh_u, (float *)sh_us };
    L.Qsd = (QW){ (int8_t *)sh_d, (float *)sh_ds };
    L.sh_gate = (float *)sh_gate;
    Slot *slots = calloc((size_t)E, sizeof(Slot));
    if (!slots) return -1;
    for (int e = 0; e < E; e++) {
        slots[e].eid = e + 1;                     /* qwen.c stores eid+1 (:430,448) */
        slots[e].g  = (int8_t *)g + (int64_t)e * MI * D;
        slots[e].u  = (int8_t *)u + (int64_t)e * MI * D;
        slots[e].d  = (int8_t *)d + (int64_t)e * D * MI;
        slots[e].gs = (float *)gs + (int64_t)e * MI;
        slots[e].us = (float *)us + (int64_t)e * MI;
        slots[e].ds = (float *)ds + (int64_t)e * D;
    }
    LCache lc = { slots, E, E };
    m.cache = &lc;
    m.L = &L;
    for (int t = 0; t < T; t++)
        moe_step(&m, &L, x + (int64_t)t * D, out + (int64_t)t * D);
    free(slots);
    return 0;
}

static Model g_tiny;
static int g_tiny_loaded;

/* Loads the snapshot once (f32-resident for the shipped tiny fixture). */
int ref_qwen_tiny_load(const char *snap) {
    if (g_tiny_loaded) return 0;
    memset(&g_tiny, 0, sizeof(g_tiny));
    model_init(&g_tiny, snap, 64);
    g_tiny_loaded = 1;
    return 0;
}

int ref_qwen_tiny_dims(int *dims) {
    if (!g_tiny_loaded) return -1;
    dims[0] = g_tiny.c.hidden; dims[1] = g_tiny.c.n_exp; dims[2] = g_tiny.c.topk;
    dims[3] = g_tiny.c.moe_inter; dims[4] = g_tiny.c.shared_inter; dims[5] = g_tiny.c.n_layers;
    dims[6] = g_tiny.stream;
    return 0;
}

/* Copies out layer `li`'s MoE weights (f32) so tests can quantise them. */
int ref_qwen_tiny_weights(int li, float *gate, float *sh_g, float *sh_u, float *sh_d, float *sh_gate,
                          float *eg, float *eu, float *ed) {
    if (!g_tiny_loaded || g_tiny.stream) return -1;
    Cfg *c = &g_tiny.c; Layer *l = &g_tiny.L[li];
    int D = c->hidden, E = c->n_exp, MI = c->moe_inter, SI = c->shared_inter;
    memcpy(gate, l->gate, sizeof(float) * E * D);
    memcpy(sh_g, l->sh_g, sizeof(float) * SI * D);
    memcpy(sh_u, l->sh_u, sizeof(float) * SI * D);
    memcpy(sh_d, l->sh_d, sizeof(float) * D * SI);
    memcpy(sh_gate, l->sh_gate, sizeof(float) * D);
    for (int e = 0; e < E; e++) {
        memcpy(eg + (int64_t)e * MI * D, l->eg[e], sizeof(float) * MI * D);
        memcpy(eu + (int64_t)e * MI * D, l->eu[e], sizeof(float) * MI * D);
        memcpy(ed + (int64_t)e * D * MI, l->ed[e], sizeof(float) * D * MI);
    }
    return 0;
}

int ref_qwen_tiny_moe(int li, const float *x, int T, float *out) {
    if (!g_tiny_loaded) return -1;
    int D = g_tiny.c.hidden;
    for (int t = 0; t < T; t++)
        moe_step(&g_tiny, &g_tiny.L[li], x + (int64_t)t * D, out + (int64_t)t * D);
    return 0;
}
