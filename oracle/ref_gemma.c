/* ref_gemma.c -- build harness around the REFERENCE engine engines/gemma.c.
 *
 * TEST INFRASTRUCTURE ONLY.  The reference source is #included from where it
 * lies (REF_GEMMA_C, passed by oracle/Makefile) and compiled into
 * oracle/_ref/libref_gemma.so; its `main` is renamed ref_gemma_main.
 *
 * ref_gemma_route() runs the reference's own static route_token()
 * (engines/gemma.c:455-478) token by token on a layer built from the
 * caller's arrays: router.proj f32 [E,D] (the f32-resident path, matvec) or
 * int8 [E,D] + f32 .qs [E] (the container path, matmul_q), router.scale [D]
 * and router.per_expert_scale [E].
 *
 * ref_gemma_moe() is the MoE part of step_batch() (engines/gemma.c:580-685)
 * on the CPU path in stream mode: route_token for every token, the expert
 * input rmsnorm(x, pre_feedforward_layernorm_2) (:608), then the expert
 * union -- hits collected for e = 0..E-1, s, k (:641-659), each hit through
 * the reference's matmul_q_st / gelu_tanh (:663-672), and the hits reduced
 * into moe[s] in hit order (:680-685).  Every arithmetic step is a call of
 * the reference's compiled function; only the loop nest is restated here.
 * Expert weights are the container's fused gate_up int8 [2*MI, D] (gate rows
 * first) with .qs [2*MI], and down int8 [D, MI] with .qs [D], per expert.
 *
 * ref_gemma_tiny_*() load the reference's own fixture model
 * (oracle/gemma_tiny, tools/make_gemma_oracle.py) with its model_init
 * (engines/gemma.c:381-437) and expose one layer's MoE weights and its
 * route_token, to derive golden vectors from the real fixture.
 */
#define main ref_gemma_main
#include REF_GEMMA_C
#undef main

static void build_layer(Layer *L, int router_i8, const void *router_w, const float *router_s,
                        const float *rscale, const float *pes) {
    memset(L, 0, sizeof(*L));
    if (router_i8) {
        L->rproj.q = (int8_t *)router_w;
        L->rproj.s = (float *)router_s;
    } else {
        L->rproj.f = (float *)router_w;
    }
    L->rscale = (float *)rscale;
    L->pes = (float *)pes;
}

int ref_gemma_route(int D, int E, int K, float eps, int router_i8, const void *router_w, const float *router_s,
                    const float *rscale, const float *pes, const float *x, int T, int32_t *top, float *tw) {
    if (E > 512) return -1;                       /* route_token's probs[512] */
    Model m;
    memset(&m, 0, sizeof(m));
    m.c.hidden = D; m.c.n_experts = E; m.c.topk = K; m.c.eps = eps;
    Layer L;
    build_layer(&L, router_i8, router_w, router_s, rscale, pes);
    float *nrm = falloc(D);
    int ti[64];
    for (int t = 0; t < T; t++) {
        route_token(&m, &L, x + (int64_t)t * D, nrm, ti, tw + (int64_t)t * K);
        for (int k = 0; k < K; k++) top[(int64_t)t * K + k] = ti[k];
    }
    free(nrm);
    return 0;
}

int ref_gemma_moe(int D, int E, int K, int MI, float eps, int router_i8, const void *router_w,
                  const float *router_s, const float *rscale, const float *pes, const float *enorm,
                  const int8_t *gq, const float *gs, const int8_t *dq, const float *ds,
                  const float *x, int S, float *moe) {
    if (E > 512 || K > 64) return -1;
    Model m;
    memset(&m, 0, sizeof(m));
    m.c.hidden = D; m.c.n_experts = E; m.c.topk = K; m.c.eps = eps; m.c.moe_inter = MI;
    Layer L;
    build_layer(&L, router_i8, router_w, router_s, rscale, pes);
    float *nrm = falloc((int64_t)S * D);
    int *top = malloc((size_t)S * K * sizeof(int));
    float *tw = malloc((size_t)S * K * sizeof(float));
    for (int s = 0; s < S; s++)
        route_token(&m, &L, x + (int64_t)s * D, nrm + (int64_t)s * D, top + s * K, tw + s * K);
    for (int s = 0; s < S; s++)
        rmsnorm(nrm + (int64_t)s * D, x + (int64_t)s * D, enorm, D, eps);
    memset(moe, 0, (size_t)S * D * sizeof(float));
    typedef struct { int e, s; float w; } Hit;
    Hit *hits = malloc((size_t)S * K * sizeof(Hit));
    int nh = 0;
    for (int e = 0; e < E; e++)
        for (int s = 0; s < S; s++)
            for (int k = 0; k < K; k++)
                if (top[s * K + k] == e) hits[nh++] = (Hit){e, s, tw[s * K + k]};
    float *hbuf = falloc((int64_t)(nh > 0 ? nh : 1) * D);
    #pragma omp parallel for schedule(dynamic)
    for (int h = 0; h < nh; h++) {
        float a[MI], b[MI];
        const int e = hits[h].e;
        const int8_t *g = gq + (int64_t)e * 2 * MI * D;
        const float *sc = gs + (int64_t)e * 2 * MI;
        const float *xin = nrm + (int64_t)hits[h].s * D;
        matmul_q_st(a, xin, g, sc, D, MI);
        matmul_q_st(b, xin, g + (int64_t)MI * D, sc + MI, D, MI);
        for (int i = 0; i < MI; i++) a[i] = gelu_tanh(a[i]) * b[i];
        matmul_q_st(hbuf + (int64_t)h * D, a, dq + (int64_t)e * D * MI, ds + (int64_t)e * D, MI, D);
    }
    for (int h = 0; h < nh; h++) {
        float *mo = moe + (int64_t)hits[h].s * D;
        const float *hb = hbuf + (int64_t)h * D;
        for (int i = 0; i < D; i++) mo[i] += hits[h].w * hb[i];
    }
    free(hbuf); free(hits); free(tw); free(top); free(nrm);
    return 0;
}

static Model g_tiny;
static int g_tiny_loaded;

int ref_gemma_tiny_load(const char *snap) {
    if (g_tiny_loaded) return 0;
    model_init(&g_tiny, snap, 64, 8);
    g_tiny_loaded = 1;
    return 0;
}

/* dims: hidden, experts, top-k, moe_inter, layers, stream, then eps bits */
int ref_gemma_tiny_dims(int *dims, float *eps) {
    if (!g_tiny_loaded) return -1;
    dims[0] = g_tiny.c.hidden; dims[1] = g_tiny.c.n_experts; dims[2] = g_tiny.c.topk;
    dims[3] = g_tiny.c.moe_inter; dims[4] = g_tiny.c.n_layers; dims[5] = g_tiny.stream;
    *eps = g_tiny.c.eps;
    return 0;
}

/* Layer li's MoE weights of the f32-resident fixture: router.proj [E,D],
 * router.scale [D], per_expert_scale [E], pre_feedforward_layernorm_2 [D],
 * experts.gate_up_proj [E,2MI,D], experts.down_proj [E,D,MI]. */
int ref_gemma_tiny_weights(int li, float *router, float *rscale, float *pes, float *enorm, float *eg, float *ed) {
    if (!g_tiny_loaded || g_tiny.stream) return -1;
    Cfg *c = &g_tiny.c;
    Layer *l = &g_tiny.L[li];
    if (!l->rproj.f) return -2;
    const int D = c->hidden, E = c->n_experts, MI = c->moe_inter;
    memcpy(router, l->rproj.f, sizeof(float) * E * D);
    memcpy(rscale, l->rscale, sizeof(float) * D);
    memcpy(pes, l->pes, sizeof(float) * E);
    memcpy(enorm, l->pre_ffw2, sizeof(float) * D);
    memcpy(eg, l->eg, sizeof(float) * (int64_t)E * 2 * MI * D);
    memcpy(ed, l->ed, sizeof(float) * (int64_t)E * D * MI);
    return 0;
}

int ref_gemma_tiny_route(int li, const float *x, int T, int32_t *top, float *tw) {
    if (!g_tiny_loaded) return -1;
    const int D = g_tiny.c.hidden, K = g_tiny.c.topk;
    float *nrm = falloc(D);
    int ti[64];
    for (int t = 0; t < T; t++) {
        route_token(&g_tiny, &g_tiny.L[li], x + (int64_t)t * D, nrm, ti, tw + (int64_t)t * K);
        for (int k = 0; k < K; k++) top[(int64_t)t * K + k] = ti[k];
    }
    free(nrm);
    return 0;
}
