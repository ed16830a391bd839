/* omc_gemma_hook.h -- the Gemma engine's MoE block on the GPU (level 2).
 *
 * Included into a build-time copy of the unmodified engines/gemma.c just
 * above step_batch() (engines/gemma.c:483); inside its layer loop, right
 * after the expert union's output is zeroed (engines/gemma.c:609-611), the
 * copy gains
 *
 *     #ifdef OM_CUDA
 *         if (omc_gemma_engine_moe(m, l, li, x, S, moe)) gpu_done = 1;
 *     #endif
 *
 * so the engine's CPU union (engines/gemma.c:632-686) is skipped and `moe`
 * holds the block's output, which the engine then normalises with
 * post_feedforward_layernorm_2 (:691) as before.  oracle/Makefile makes that
 * copy in a temporary directory; nothing of the engine is kept.
 *
 * The library takes the residual rows x as they are: routing
 * (route_token, :455-478, with its rmsnorm, router.scale and
 * per_expert_scale) and the experts' input norm (pre_feedforward_layernorm_2,
 * :608) run on the GPU, so the engine's own CPU routing of the same rows
 * (:581-583) is not used.  On a layer's first call the hook creates the
 * library layer from the engine's router (l->rproj: int8 + scales as the
 * converter writes it, or f32) and norms, and uploads every expert from the
 * int8 container (model.layers.N.experts.E.gate_up_proj [2I,D] + .qs, and
 * down_proj [D,I] + .qs, as expert_get reads them, :335-365).  The
 * f32-resident fixture layout (no per-expert int8 tensors) is not served: the
 * hook reports it and exits with status 2, as it does on any failure.  There
 * is no CPU fallback.
 *
 * Environment: OMC_DEVICE selects the CUDA device (default 0).
 * OMC_TIER_SLOTS=n (0 < n < experts) keeps only n experts of each layer in
 * HBM and the rest in pinned host memory, moved in by the library's hot-store
 * policy (omc_tier_enable: a model larger than its HBM share); the heat is
 * halved every OMC_TIER_DECAY forwards (default 0: never).  Unset: every
 * expert in HBM.
 */
#ifndef OMC_GEMMA_HOOK_H
#define OMC_GEMMA_HOOK_H
#include "om_cuda.h"

static unsigned char *omc_gh_ready;   /* per layer: created and uploaded */

static void omc_gh_fail(const char *what, int rc) {
    fprintf(stderr, "omc: %s failed: %s (%s)\n", what, omc_strerror(rc), omc_last_error());
    exit(2);
}

static void omc_gh_upload(Model *m, Layer *l, int li) {
    Cfg *c = &m->c;
    int rc;
    if (!m->stream) {
        fprintf(stderr, "omc: the Gemma hook needs the int8 expert container (per-expert gate_up_proj)\n");
        exit(2);
    }
    omc_moe_desc d;
    memset(&d, 0, sizeof(d));
    d.family = OMC_FAMILY_GEMMA;
    d.D = c->hidden;
    d.I = c->moe_inter;
    d.E = c->n_experts;
    d.k = c->topk;
    d.renorm = 1;
    d.router_dtype = l->rproj.q ? OMC_ROUTER_I8 : OMC_ROUTER_F32;
    const void *rw = l->rproj.q ? (const void *)l->rproj.q : (const void *)l->rproj.f;
    if ((rc = omc_layer_init(li, &d, rw, l->rproj.s))) omc_gh_fail("omc_layer_init", rc);
    {
        const char *ts = getenv("OMC_TIER_SLOTS"), *td = getenv("OMC_TIER_DECAY");
        const int slots = ts ? atoi(ts) : 0;
        if (slots > 0 && slots < d.E && (rc = omc_tier_enable(li, slots, 1, td ? atoi(td) : 0)))
            omc_gh_fail("omc_tier_enable", rc);
    }
    if ((rc = omc_layer_gemma_norms(li, c->eps, l->rscale, l->pes, l->pre_ffw2)))
        omc_gh_fail("omc_layer_gemma_norms", rc);
    const int D = c->hidden, mi = c->moe_inter;
    int8_t *gq = malloc((size_t)2 * mi * D), *dq = malloc((size_t)D * mi);
    float *gs = falloc(2 * mi), *ds = falloc(D);
    if (!gq || !dq) omc_gh_fail("host buffers", OMC_ENOMEM);
    char nm[300];
    for (int e = 0; e < c->n_experts; e++) {
        snprintf(nm, sizeof(nm), "model.layers.%d.experts.%d.gate_up_proj", li, e);
        st_read_raw(&m->S, nm, gq, 0);
        snprintf(nm, sizeof(nm), "model.layers.%d.experts.%d.gate_up_proj.qs", li, e);
        st_read_f32(&m->S, nm, gs, 0);
        snprintf(nm, sizeof(nm), "model.layers.%d.experts.%d.down_proj", li, e);
        st_read_raw(&m->S, nm, dq, 0);
        snprintf(nm, sizeof(nm), "model.layers.%d.experts.%d.down_proj.qs", li, e);
        st_read_f32(&m->S, nm, ds, 0);
        /* the fused gate_up: gate rows [0, I), up rows [I, 2I) */
        if ((rc = omc_expert_set(li, e, gq, gs, gq + (size_t)mi * D, gs + mi, dq, ds)))
            omc_gh_fail("omc_expert_set", rc);
    }
    free(gq);
    free(dq);
    free(gs);
    free(ds);
}

/* The MoE term of layer li for the S residual rows x: moe[S][D].  Returns 1
 * (handled); never returns on failure. */
static int omc_gemma_engine_moe(Model *m, Layer *l, int li, const float *x, int S, float *moe) {
    int rc;
    if (!omc_gh_ready) {
        const char *dev = getenv("OMC_DEVICE");
        if ((rc = omc_init(dev ? atoi(dev) : 0, 0))) omc_gh_fail("omc_init", rc);
        omc_gh_ready = calloc((size_t)m->c.n_layers, 1);
        if (!omc_gh_ready) omc_gh_fail("host buffers", OMC_ENOMEM);
    }
    if (!omc_gh_ready[li]) {
        omc_gh_upload(m, l, li);
        omc_gh_ready[li] = 1;
    }
    if ((rc = omc_moe_forward(li, x, S, moe, NULL, NULL))) omc_gh_fail("omc_moe_forward", rc);
    return 1;
}

#endif /* OMC_GEMMA_HOOK_H */
