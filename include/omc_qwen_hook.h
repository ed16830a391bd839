/* omc_qwen_hook.h -- the Qwen engine's MoE layer on the GPU (level 2).
 *
 * Included into a build-time copy of the unmodified engines/qwen.c just above
 * moe_step() (engines/qwen.c:453), whose first statement becomes
 *
 *     #ifdef OM_CUDA
 *         if (omc_qwen_engine_moe(m, l, x, out)) return;
 *     #endif
 *
 * (oracle/Makefile makes that copy in a temporary directory; nothing of the
 * engine is kept).  The hook uses the engine's own types and container
 * reader, so it must be included after them, inside the engine's
 * translation unit.
 *
 * The engine calls moe_step once per token (step(), engines/qwen.c:515), so
 * every call is one omc_moe_forward of T = 1: the shared expert behind its
 * sigmoid gate, the int8 router, softmax (double sum), top-k, renorm, the k
 * routed experts and the combine, all on the GPU, replacing
 * engines/qwen.c:454-494.
 *
 * On a layer's first call it creates the library layer from what the engine
 * holds in stream mode (engines/qwen.c:283-288): the router and the shared
 * expert as the engine quantised them at load (qw_make: int8 rows + f32
 * scales, l->Qgate, l->Qsg, l->Qsu, l->Qsd) and the f32 gate vector
 * l->sh_gate; and it uploads all E routed experts, read from the int8
 * container the way expert_get reads one on a miss (engines/qwen.c:428-450:
 * "name" int8 rows and "name.qs" f32 scales).
 *
 * The f32-resident mode (engines/qwen.c:289-296: a snapshot whose experts are
 * not int8) has no int8 expert weights for the library to run; the hook
 * reports that and exits, as it does on any failure (status 2).  There is no
 * CPU fallback.
 *
 * Environment: OMC_DEVICE selects the CUDA device (default 0).
 */
#ifndef OMC_QWEN_HOOK_H
#define OMC_QWEN_HOOK_H
#include "om_cuda.h"

static unsigned char *omc_qh_ready;   /* per layer: created and uploaded */

static void omc_qh_fail(const char *what, int rc) {
    fprintf(stderr, "omc: %s failed: %s (%s)\n", what, omc_strerror(rc), omc_last_error());
    exit(2);
}

static void omc_qh_upload(Model *m, Layer *l, int li) {
    Cfg *c = &m->c;
    int rc;
    if (!m->stream) {
        fprintf(stderr, "omc: the Qwen MoE hook needs the int8 container (stream mode, engines/qwen.c:215-218); "
                        "this snapshot keeps its experts f32\n");
        exit(2);
    }
    omc_moe_desc d;
    memset(&d, 0, sizeof(d));
    d.family = OMC_FAMILY_QWEN;
    d.D = c->hidden;
    d.I = c->moe_inter;
    d.E = c->n_exp;
    d.k = c->topk;
    d.renorm = 1;                          /* engines/qwen.c:476-477 */
    d.router_dtype = OMC_ROUTER_I8;        /* l->Qgate, engines/qwen.c:284,465 */
    d.has_shared = c->shared_inter > 0;
    d.Is = c->shared_inter;
    if ((rc = omc_layer_init(li, &d, l->Qgate.q, l->Qgate.s))) omc_qh_fail("omc_layer_init", rc);
    if (d.has_shared &&
        (rc = omc_shared_set(li, l->Qsg.q, l->Qsg.s, l->Qsu.q, l->Qsu.s, l->Qsd.q, l->Qsd.s, l->sh_gate)))
        omc_qh_fail("omc_shared_set", rc);
    const int64_t ng = (int64_t)c->moe_inter * c->hidden;
    int8_t *g = malloc(ng), *u = malloc(ng), *dn = malloc(ng);
    float *gs = falloc(c->moe_inter), *us = falloc(c->moe_inter), *ds = falloc(c->hidden);
    if (!g || !u || !dn) omc_qh_fail("host buffers", OMC_ENOMEM);
    char nm[320], qs[336];
    for (int e = 0; e < c->n_exp; e++) {
#define OMC_QH_READ(W, SC, proj)                                                                  \
        do {                                                                                      \
            snprintf(nm, sizeof(nm), "model.layers.%d.mlp.experts.%d." proj ".weight", li, e);    \
            snprintf(qs, sizeof(qs), "%s.qs", nm);                                                \
            st_read_raw(&m->S, nm, (W), 1);                                                       \
            st_read_f32(&m->S, qs, (SC), 1);                                                      \
        } while (0)
        OMC_QH_READ(g, gs, "gate_proj");
        OMC_QH_READ(u, us, "up_proj");
        OMC_QH_READ(dn, ds, "down_proj");
#undef OMC_QH_READ
        if ((rc = omc_expert_set(li, e, g, gs, u, us, dn, ds))) omc_qh_fail("omc_expert_set", rc);
    }
    free(g);
    free(u);
    free(dn);
    free(gs);
    free(us);
    free(ds);
}

/* The engine's moe_step(): out[D] = MoE(x[D]) of one token for layer l.
 * Returns 1 (handled); never returns on failure. */
static int omc_qwen_engine_moe(Model *m, Layer *l, const float *x, float *out) {
    int rc;
    const int li = (int)(l - m->L);
    if (!omc_qh_ready) {
        const char *dev = getenv("OMC_DEVICE");
        if ((rc = omc_init(dev ? atoi(dev) : 0, 0))) omc_qh_fail("omc_init", rc);
        omc_qh_ready = calloc((size_t)m->c.n_layers, 1);
        if (!omc_qh_ready) omc_qh_fail("host buffers", OMC_ENOMEM);
    }
    if (!omc_qh_ready[li]) {
        omc_qh_upload(m, l, li);
        omc_qh_ready[li] = 1;
    }
    if ((rc = omc_moe_forward(li, x, 1, out, NULL, NULL))) omc_qh_fail("omc_moe_forward", rc);
    return 1;
}

#endif /* OMC_QWEN_HOOK_H */
