/* omc_engine_hook.h -- the OLMoE engine's MoE layer on the GPU (level 2).
 *
 * Included into a build-time copy of the unmodified engines/olmoe.c just
 * above moe() (engines/olmoe.c:344), whose first statement becomes
 *
 *     #ifdef OM_CUDA
 *         if (omc_engine_moe(m, l, layer, x, S, out)) return;
 *     #endif
 *
 * (oracle/Makefile makes that copy in a temporary directory; nothing of the
 * engine is kept).  The hook uses the engine's own types and loader, so it
 * must be included after them, inside the engine's translation unit.
 *
 * On a layer's first call it creates the library layer from the engine's
 * router (l->gate, f32 [E][D], engines/olmoe.c:226), top-k and
 * norm_topk_prob (engines/olmoe.c:194), and uploads all E experts with the
 * engine's loader load_expert_w (engines/olmoe.c:237-247: the int8
 * container's rows and .qs scales, or quantise-on-load).  From then on every
 * call is one omc_moe_forward over the S tokens: routing, dispatch, expert
 * SwiGLU and the weighted combine all run on the GPU, replacing
 * engines/olmoe.c:346-401.  There is no CPU fallback: a failure is reported
 * and the process exits with status 2.
 *
 * Environment: OMC_DEVICE selects the CUDA device (default 0).
 * OMC_TIER_SLOTS=n (0 < n < experts) keeps only n experts of each layer in
 * HBM and the rest in pinned host memory, moved in by the library's hot-store
 * policy (omc_tier_enable: a model larger than its HBM share); the heat is
 * halved every OMC_TIER_DECAY forwards (default 0: never).  Unset: every
 * expert in HBM.
 */
#ifndef OMC_ENGINE_HOOK_H
#define OMC_ENGINE_HOOK_H
#include "om_cuda.h"

static unsigned char *omc_hook_ready;   /* per layer: created and uploaded */

static void omc_hook_fail(const char *what, int rc) {
    fprintf(stderr, "omc: %s failed: %s (%s)\n", what, omc_strerror(rc), omc_last_error());
    exit(2);
}

static void omc_hook_upload(Model *m, Layer *l, int layer) {
    Cfg *c = &m->c;
    int rc;
    omc_moe_desc d;
    memset(&d, 0, sizeof(d));
    d.family = OMC_FAMILY_OLMOE;
    d.D = c->hidden;
    d.I = c->inter;
    d.E = c->n_experts;
    d.k = c->topk;
    d.renorm = c->norm_topk;
    d.router_dtype = OMC_ROUTER_F32;
    if ((rc = omc_layer_init(layer, &d, l->gate, NULL))) omc_hook_fail("omc_layer_init", rc);
    {
        const char *ts = getenv("OMC_TIER_SLOTS"), *td = getenv("OMC_TIER_DECAY");
        const int slots = ts ? atoi(ts) : 0;
        if (slots > 0 && slots < d.E && (rc = omc_tier_enable(layer, slots, 1, td ? atoi(td) : 0)))
            omc_hook_fail("omc_tier_enable", rc);
    }
    const int64_t n = (int64_t)c->inter * c->hidden;
    int8_t *g = malloc(n), *u = malloc(n), *dn = malloc(n);
    float *gs = falloc(c->inter), *us = falloc(c->inter), *ds = falloc(c->hidden), *tmp = falloc(n);
    if (!g || !u || !dn) omc_hook_fail("host buffers", OMC_ENOMEM);
    char nm[256];
    for (int e = 0; e < c->n_experts; e++) {
        snprintf(nm, sizeof(nm), "model.layers.%d.mlp.experts.%d.gate_proj.weight", layer, e);
        load_expert_w(m, nm, g, gs, c->inter, c->hidden, tmp);
        snprintf(nm, sizeof(nm), "model.layers.%d.mlp.experts.%d.up_proj.weight", layer, e);
        load_expert_w(m, nm, u, us, c->inter, c->hidden, tmp);
        snprintf(nm, sizeof(nm), "model.layers.%d.mlp.experts.%d.down_proj.weight", layer, e);
        load_expert_w(m, nm, dn, ds, c->hidden, c->inter, tmp);
        if ((rc = omc_expert_set(layer, e, g, gs, u, us, dn, ds))) omc_hook_fail("omc_expert_set", rc);
    }
    free(g);
    free(u);
    free(dn);
    free(gs);
    free(us);
    free(ds);
    free(tmp);
}

/* The engine's moe(): out[S][D] = MoE(x[S][D]) for layer `layer`.  Returns 1
 * (handled); never returns on failure. */
static int omc_engine_moe(Model *m, Layer *l, int layer, float *x, int S, float *out) {
    int rc;
    if (!omc_hook_ready) {
        const char *dev = getenv("OMC_DEVICE");
        if ((rc = omc_init(dev ? atoi(dev) : 0, 0))) omc_hook_fail("omc_init", rc);
        omc_hook_ready = calloc((size_t)m->c.n_layers, 1);
        if (!omc_hook_ready) omc_hook_fail("host buffers", OMC_ENOMEM);
    }
    if (!omc_hook_ready[layer]) {
        omc_hook_upload(m, l, layer);
        omc_hook_ready[layer] = 1;
    }
    if ((rc = omc_moe_forward(layer, x, S, out, NULL, NULL))) omc_hook_fail("omc_moe_forward", rc);
    return 1;
}

#endif /* OMC_ENGINE_HOOK_H */
