/* moe_oracle.c -- CPU oracle for the overhang MoE block (TEST INFRASTRUCTURE
 * ONLY; see moe_oracle.h).  Every function below restates a reference
 * function operation for operation; the citation is on each one.
 *
 * Build: gcc -O3 -fPIC -ffp-contract=off (no -ffast-math, no -march): the
 * same x86-64 SSE2 scalar arithmetic the reference engines get from
 * `gcc -O3 -fopenmp` (Makefile:5-11 with gcc in place of clang).
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- reference arithmetic kernels ------------------------------------ */

/* engines/olmoe.c:74-85 (matmul) and engines/qwen.c:70-77 (matvec):
 * y[o] = sum_i x[i]*W[o,i], one sequential fp32 chain per output. */
static void ref_matvec_f32(float *y, const float *x, const float *W, int I, int O) {
    for (int o = 0; o < O; o++) {
        const float *w = W + (int64_t)o * I;
        float acc = 0.f;
        for (int i = 0; i < I; i++) acc += x[i] * w[i];
        y[o] = acc;
    }
}

/* engines/olmoe.c:134-140, engines/qwen.c:116-121 (x86 scalar matmul_q):
 * y[o] = (sum_i x[i]*(float)q[o,i]) * scale[o]. */
static void ref_matmul_q(float *y, const float *x, const int8_t *q, const float *scale, int I, int O) {
    for (int o = 0; o < O; o++) {
        const int8_t *w = q + (int64_t)o * I;
        float acc = 0.f;
        for (int i = 0; i < I; i++) acc += x[i] * (float)w[i];
        y[o] = acc * scale[o];
    }
}

/* engines/olmoe.c:170-174 softmax_row: float running sum. */
static void ref_softmax_f32sum(float *x, int n) {
    float m = -1e30f;
    for (int i = 0; i < n; i++) if (x[i] > m) m = x[i];
    float s = 0;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - m); s += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= s;
}

/* engines/qwen.c:161-165 softmax_: double running sum, divide by (float)sum. */
static void ref_softmax_f64sum(float *x, int n) {
    float m = -1e30f;
    for (int i = 0; i < n; i++) if (x[i] > m) m = x[i];
    double s = 0;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - m); s += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= (float)s;
}

/* engines/olmoe.c:355-362, engines/qwen.c:468-475: k passes of argmax over the
 * probabilities with strict '>' from bv=-1e30 and taken ids skipped, so an
 * equal probability keeps the lower expert id. */
static void ref_topk(const float *pr, int E, int K, int *idx, float *val) {
    for (int kk = 0; kk < K; kk++) {
        int best = -1; float bv = -1e30f;
        for (int e = 0; e < E; e++) {
            int taken = 0;
            for (int j = 0; j < kk; j++) if (idx[j] == e) { taken = 1; break; }
            if (!taken && pr[e] > bv) { bv = pr[e]; best = e; }
        }
        idx[kk] = best; val[kk] = bv;
    }
}

/* engines/olmoe.c:363 and engines/qwen.c:476-477: float sum, then divide. */
static void ref_renorm(float *val, int K) {
    float sm = 0;
    for (int kk = 0; kk < K; kk++) sm += val[kk];
    for (int kk = 0; kk < K; kk++) val[kk] /= sm;
}

/* engines/qwen.c:158-159 */
static float ref_sigmoidf(float z) { return 1.f / (1.f + expf(-z)); }
static float ref_siluf(float z) { return z * ref_sigmoidf(z); }

/* ---- routing ------------------------------------------------------- */

static int desc_ok(const orc_desc *d) {
    if (!d || d->D <= 0 || d->I <= 0 || d->E <= 0 || d->k <= 0 || d->k > d->E || d->k > 64) return 0;
    if (d->family != ORC_FAMILY_OLMOE && d->family != ORC_FAMILY_QWEN && d->family != ORC_FAMILY_GEMMA) return 0;
    if (d->has_shared && (d->family != ORC_FAMILY_QWEN || d->Is <= 0)) return 0;
    return 1;
}

static int gemma_ok(const orc_desc *d, const orc_weights *w) {
    return d->family != ORC_FAMILY_GEMMA || (w->g_rscale && w->g_pes);
}

/* ---- gemma ---------------------------------------------------------- */

/* engines/gemma.c:313-317 rmsnorm's factor: double running sum of x^2,
 * (float)(ms/n) + eps, then powf(., -0.5f) (ORC_RSQRT_LIBM) or the double
 * 1/sqrt rounded once to float (ORC_RSQRT_CR). */
static float gemma_norm_factor(const orc_desc *d, const float *x) {
    double ms = 0;
    for (int i = 0; i < d->D; i++) ms += (double)x[i] * x[i];
    const float y = (float)(ms / d->D) + d->eps;
    if (d->rsqrt_mode == ORC_RSQRT_LIBM) return powf(y, -0.5f);
    return (float)(1.0 / sqrt((double)y));
}

/* engines/gemma.c:458-460 (router input: rmsnorm without weight, then
 * *= router.scale[i] * D^-0.5) and :608 (expert input: rmsnorm with
 * pre_feedforward_layernorm_2).  rmsnorm writes x[i]*r*w[i] left to right,
 * with w[i] = 1.f when there is no weight. */
static void gemma_inputs(const orc_desc *d, const orc_weights *w, const float *x, float *xr, float *xe,
                         float *rout) {
    const float r = gemma_norm_factor(d, x);
    const float rroot = 1.f / sqrtf((float)d->D);
    for (int i = 0; i < d->D; i++) {
        const float n = x[i] * r;
        if (xr) xr[i] = (n * 1.f) * (w->g_rscale[i] * rroot);
        if (xe) xe[i] = n * (w->g_enorm ? w->g_enorm[i] : 1.f);
    }
    if (rout) *rout = r;
}

/* engines/gemma.c:319-321 */
static float ref_gelu_tanh(float x) {
    return 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

/* engines/gemma.c:461-477: router logits of the pre-scaled input, e_i =
 * expf(l_i - max) with a float running sum, top-k over the e_i (strict '>'
 * from -1, so ties keep the lower id), w_k = e_k/sum renormalised by the
 * float sum of those quotients in selection order, times per_expert_scale. */
static void gemma_route(const orc_desc *d, const orc_weights *w, const float *xr, float *pr, int *idx, float *val) {
    const int E = d->E, K = d->k;
    if (d->router_i8) ref_matmul_q(pr, xr, (const int8_t *)w->router, w->router_s, d->D, E);
    else              ref_matvec_f32(pr, xr, (const float *)w->router, d->D, E);
    if (w->router_bias) for (int e = 0; e < E; e++) pr[e] += w->router_bias[e];
    float pmx = -1e30f;
    for (int e = 0; e < E; e++) if (pr[e] > pmx) pmx = pr[e];
    float psum = 0.f;
    for (int e = 0; e < E; e++) { pr[e] = expf(pr[e] - pmx); psum += pr[e]; }
    float wsum = 0.f;
    for (int kk = 0; kk < K; kk++) {
        int best = -1; float bv = -1.f;
        for (int e = 0; e < E; e++) {
            int taken = 0;
            for (int j = 0; j < kk; j++) if (idx[j] == e) taken = 1;
            if (!taken && pr[e] > bv) { bv = pr[e]; best = e; }
        }
        idx[kk] = best; val[kk] = bv / psum; wsum += bv / psum;
    }
    for (int kk = 0; kk < K; kk++) val[kk] = val[kk] / wsum * w->g_pes[idx[kk]];
}

int orc_gemma_prenorm(const orc_desc *d, const orc_weights *w, const float *x, int T, float *xr, float *xe,
                      float *r) {
    if (!desc_ok(d) || d->family != ORC_FAMILY_GEMMA || !gemma_ok(d, w) || T < 0) return -1;
    for (int t = 0; t < T; t++)
        gemma_inputs(d, w, x + (int64_t)t * d->D, xr ? xr + (int64_t)t * d->D : NULL,
                     xe ? xe + (int64_t)t * d->D : NULL, r ? r + t : NULL);
    return 0;
}

/* Routes one token: logits -> softmax -> top-k -> renorm.
 * olmoe: engines/olmoe.c:347 (logits), :351-364 (softmax_row, top-k, renorm)
 * qwen : engines/qwen.c:465-477 (DM router, softmax_, top-k, renorm) */
static void route_one(const orc_desc *d, const orc_weights *w, const float *xs, float *pr,
                      int *idx, float *val) {
    if (d->family == ORC_FAMILY_GEMMA) {
        float *xr = malloc(sizeof(float) * d->D);
        gemma_inputs(d, w, xs, xr, NULL, NULL);
        gemma_route(d, w, xr, pr, idx, val);
        free(xr);
        return;
    }
    if (d->router_i8) ref_matmul_q(pr, xs, (const int8_t *)w->router, w->router_s, d->D, d->E);
    else              ref_matvec_f32(pr, xs, (const float *)w->router, d->D, d->E);
    /* the harness's optional router bias, one float add per logit */
    if (w->router_bias) for (int e = 0; e < d->E; e++) pr[e] += w->router_bias[e];
    if (d->family == ORC_FAMILY_QWEN) ref_softmax_f64sum(pr, d->E);
    else                              ref_softmax_f32sum(pr, d->E);
    ref_topk(pr, d->E, d->k, idx, val);
    if (d->family == ORC_FAMILY_QWEN || d->renorm) ref_renorm(val, d->k);
}

int orc_route(const orc_desc *d, const orc_weights *w, const float *x, int T,
              int32_t *topk_idx, float *topk_w) {
    if (!desc_ok(d) || !gemma_ok(d, w) || T < 0) return -1;
    #pragma omp parallel
    {
        float *pr = malloc(sizeof(float) * d->E);
        int idx[64]; float val[64];
        #pragma omp for schedule(static)
        for (int s = 0; s < T; s++) {
            route_one(d, w, x + (int64_t)s * d->D, pr, idx, val);
            for (int kk = 0; kk < d->k; kk++) {
                if (topk_idx) topk_idx[(int64_t)s * d->k + kk] = idx[kk];
                if (topk_w)   topk_w[(int64_t)s * d->k + kk] = val[kk];
            }
        }
        free(pr);
    }
    return 0;
}

/* ---- the block ------------------------------------------------------ */

/* Tokens are independent in the reference (every buffer below is per token),
 * so they are spread over OpenMP threads; each token's arithmetic is the
 * reference's, in the reference's order. */
/* One routed expert e on one input row: g,u = int8 GEMVs, the family's
 * activation, then the down GEMV into y.
 * olmoe: engines/olmoe.c:386-394 (g/(1+exp(-g))*u)
 * qwen : engines/qwen.c:480-491 (silu(g)*u)
 * gemma: engines/gemma.c:667-672 (gelu_tanh(g)*u; gate_up rows [0,mi) and
 *        [mi,2mi) are the g and u matrices here) */
static int family_act(const orc_desc *d) { return d->family; }   /* ORC_ACT_* equals the family */

static void expert_apply(const orc_desc *d, const orc_weights *w, int act, int e, const float *xs, float *g, float *u,
                         float *y) {
    const int D = d->D, I = d->I;
    const int8_t *qg = w->g + (int64_t)e * I * D, *qu = w->u + (int64_t)e * I * D;
    const int8_t *qd = w->d + (int64_t)e * D * I;
    ref_matmul_q(g, xs, qg, w->gs + (int64_t)e * I, D, I);
    ref_matmul_q(u, xs, qu, w->us + (int64_t)e * I, D, I);
    if (act == ORC_ACT_SILU_SIG) {
        for (int i = 0; i < I; i++) g[i] = ref_siluf(g[i]) * u[i];          /* qwen.c:485 */
    } else if (act == ORC_ACT_GELU_TANH) {
        for (int i = 0; i < I; i++) g[i] = ref_gelu_tanh(g[i]) * u[i];      /* gemma.c:671 */
    } else {
        for (int i = 0; i < I; i++) { float gv = g[i]; g[i] = (gv / (1.f + expf(-gv))) * u[i]; } /* olmoe.c:393 */
    }
    ref_matmul_q(y, g, qd, w->ds + (int64_t)e * D, I, D);
}

/* Tokens are independent in the reference (every buffer below is per token),
 * so they are spread over OpenMP threads; each token's arithmetic is the
 * reference's, in the reference's order. */
int orc_moe(const orc_desc *d, const orc_weights *w, const float *x, int T,
            float *out, int32_t *topk_idx, float *topk_w) {
    if (!desc_ok(d) || !gemma_ok(d, w) || T < 0) return -1;
    const int D = d->D, I = d->I, E = d->E, K = d->k;
    const int Wmax = (d->has_shared && d->Is > I) ? d->Is : I;
    #pragma omp parallel
    {
        float *pr = malloc(sizeof(float) * E);
        float *g = malloc(sizeof(float) * Wmax), *u = malloc(sizeof(float) * Wmax);
        float *hh = malloc(sizeof(float) * D), *xe = malloc(sizeof(float) * D);
        int idx[64]; float val[64];
        #pragma omp for schedule(dynamic, 1)
        for (int s = 0; s < T; s++) {
            const float *xs = x + (int64_t)s * D;
            float *os = out + (int64_t)s * D;
            if (d->family == ORC_FAMILY_QWEN && d->has_shared) {
                /* engines/qwen.c:455-462: shared expert, then x sigmoid gate */
                const int SI = d->Is;
                ref_matmul_q(g, xs, w->sh_g, w->sh_gs, D, SI);
                ref_matmul_q(u, xs, w->sh_u, w->sh_us, D, SI);
                for (int i = 0; i < SI; i++) g[i] = ref_siluf(g[i]) * u[i];
                ref_matmul_q(os, g, w->sh_d, w->sh_ds, SI, D);
                float sg = 0;
                for (int i = 0; i < D; i++) sg += w->sh_gate[i] * xs[i];
                sg = ref_sigmoidf(sg);
                for (int i = 0; i < D; i++) os[i] *= sg;
            } else {
                memset(os, 0, sizeof(float) * D);        /* engines/olmoe.c:348, gemma.c:610 */
            }
            route_one(d, w, xs, pr, idx, val);
            for (int kk = 0; kk < K; kk++) {
                if (topk_idx) topk_idx[(int64_t)s * K + kk] = idx[kk];
                if (topk_w)   topk_w[(int64_t)s * K + kk] = val[kk];
            }
            if (d->family == ORC_FAMILY_GEMMA) {
                /* gemma.c:608 expert input; hits combined in ascending expert
                 * id (the union loop over e, gemma.c:641-659, reduced in hit
                 * order at :680-685) */
                gemma_inputs(d, w, xs, NULL, xe, NULL);
                for (int e = 0; e < E; e++)
                    for (int kk = 0; kk < K; kk++) {
                        if (idx[kk] != e) continue;
                        expert_apply(d, w, family_act(d), e, xe, g, u, hh);
                        for (int i = 0; i < D; i++) os[i] += val[kk] * hh[i];
                    }
                continue;
            }
            for (int kk = 0; kk < K; kk++) {
                expert_apply(d, w, family_act(d), idx[kk], xs, g, u, hh);
                const float wk = val[kk];
                for (int i = 0; i < D; i++) os[i] += wk * hh[i];   /* olmoe.c:395-397, qwen.c:492 */
            }
        }
        free(pr); free(g); free(u); free(hh); free(xe);
    }
    return 0;
}

int orc_shared_gate(const orc_desc *d, const orc_weights *w, const float *x, int T, float *sg) {
    if (!desc_ok(d) || T < 0 || !d->has_shared) return -1;
    for (int t = 0; t < T; t++) {
        const float *xs = x + (int64_t)t * d->D;
        float s = 0;
        for (int i = 0; i < d->D; i++) s += w->sh_gate[i] * xs[i];
        sg[t] = ref_sigmoidf(s);
    }
    return 0;
}

int orc_expert_rows(const orc_desc *d, const orc_weights *w, const float *x, int R, const int32_t *ids,
                    float *y) {
    if (!desc_ok(d) || !gemma_ok(d, w) || R < 0) return -1;
    for (int r = 0; r < R; r++)
        if (ids[r] < 0 || ids[r] > d->E || (ids[r] == d->E && !d->has_shared)) return -1;
    const int D = d->D, I = d->I, E = d->E;
    const int Wmax = (d->has_shared && d->Is > I) ? d->Is : I;
    #pragma omp parallel
    {
        float *g = malloc(sizeof(float) * Wmax), *u = malloc(sizeof(float) * Wmax);
        float *xe = malloc(sizeof(float) * D);
        #pragma omp for schedule(dynamic, 1)
        for (int r = 0; r < R; r++) {
            const float *xs = x + (int64_t)r * D;
            float *ys = y + (int64_t)r * D;
            const int e = ids[r];
            if (e == E) {
                /* engines/qwen.c:455-459: shared expert, sigmoid gate applied by the caller */
                const int SI = d->Is;
                ref_matmul_q(g, xs, w->sh_g, w->sh_gs, D, SI);
                ref_matmul_q(u, xs, w->sh_u, w->sh_us, D, SI);
                for (int i = 0; i < SI; i++) g[i] = ref_siluf(g[i]) * u[i];
                ref_matmul_q(ys, g, w->sh_d, w->sh_ds, SI, D);
                continue;
            }
            if (d->family == ORC_FAMILY_GEMMA) {     /* rows are residual rows: gemma.c:608 first */
                gemma_inputs(d, w, xs, NULL, xe, NULL);
                xs = xe;
            }
            expert_apply(d, w, family_act(d), e, xs, g, u, ys);
        }
        free(g); free(u); free(xe);
    }
    return 0;
}

int orc_expert_rows_act(const orc_desc *d, const orc_weights *w, const float *x, int R, const int32_t *ids, int act,
                        float *y) {
    if (!desc_ok(d) || R < 0 || act < ORC_ACT_SILU_DIV || act > ORC_ACT_GELU_TANH) return -1;
    for (int r = 0; r < R; r++)
        if (ids[r] < 0 || ids[r] >= d->E) return -1;
    #pragma omp parallel
    {
        float *g = malloc(sizeof(float) * d->I), *u = malloc(sizeof(float) * d->I);
        #pragma omp for schedule(dynamic, 1)
        for (int r = 0; r < R; r++)
            expert_apply(d, w, act, ids[r], x + (int64_t)r * d->D, g, u, y + (int64_t)r * d->D);
        free(g); free(u);
    }
    return 0;
}

/* ---- quantisers and inputs ----------------------------------------- */

/* tools/convert_olmoe.py:32-38 (same rule in convert_qwen.py / convert_gemma.py) */
void orc_quantize_rows_py(const float *w, int O, int I, int8_t *q, float *s) {
    for (int o = 0; o < O; o++) {
        const float *wr = w + (int64_t)o * I;
        float amax = 0.f;
        for (int i = 0; i < I; i++) { float a = fabsf(wr[i]); if (a > amax) amax = a; }
        if (amax < 1e-12f) amax = 1e-12f;
        const float sc = amax / 127.0f;
        s[o] = sc;
        for (int i = 0; i < I; i++) {
            float v = nearbyintf(wr[i] / sc);              /* torch.round: half to even */
            if (v > 127.f) v = 127.f;
            if (v < -128.f) v = -128.f;
            q[(int64_t)o * I + i] = (int8_t)v;
        }
    }
}

/* engines/qwen.c:124-138 */
void orc_quantize_rows_c(const float *w, int O, int I, int8_t *q, float *s) {
    for (int o = 0; o < O; o++) {
        const float *wr = w + (int64_t)o * I;
        float am = 0.f;
        for (int i = 0; i < I; i++) { float a = fabsf(wr[i]); if (a > am) am = a; }
        float sc = am / 127.f;
        if (sc < 1e-8f) sc = 1e-8f;
        s[o] = sc;
        for (int i = 0; i < I; i++) {
            int v = (int)lrintf(wr[i] / sc);
            if (v > 127) v = 127;
            if (v < -128) v = -128;
            q[(int64_t)o * I + i] = (int8_t)v;
        }
    }
}

static uint64_t splitmix64(uint64_t *st) {
    uint64_t z = (*st += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* Blocks of 65536 values, each block seeded from (seed, block index), so the
 * stream is the same whatever the thread count. */
void orc_fill_normal(uint64_t seed, float *dst, int64_t n, float sigma) {
    const int64_t BLK = 65536;
    const int64_t nb = (n + BLK - 1) / BLK;
    #pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; b++) {
        uint64_t st = seed ^ (0xD1B54A32D192ED03ULL * (uint64_t)(b + 1));
        splitmix64(&st);
        const int64_t lo = b * BLK, hi = (lo + BLK < n) ? lo + BLK : n;
        for (int64_t i = lo; i < hi; i += 2) {
            double u1 = ((splitmix64(&st) >> 11) + 1.0) * 0x1.0p-53;   /* (0,1] */
            double u2 = (splitmix64(&st) >> 11) * 0x1.0p-53;
            double r = sqrt(-2.0 * log(u1)), th = 6.283185307179586 * u2;
            dst[i] = (float)(sigma * r * cos(th));
            if (i + 1 < hi) dst[i + 1] = (float)(sigma * r * sin(th));
        }
    }
}

float orc_expf(float x) { return expf(x); }

void orc_expf_array(const float *x, float *y, int64_t n) {
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) y[i] = expf(x[i]);
}

/* ------------------------------------------------------------ hot store -- */
/* include/tier.h:30-33 */
uint64_t orc_tier_score(uint32_t heat, uint32_t last, uint32_t clock) {
    const uint32_t age = clock - last;
    const uint64_t recency = age < 255u ? (uint64_t)(255u - age) : 0u;
    return ((uint64_t)heat << 8) | recency;
}

/* Residency of expert e: is it named by any of the npin slots
 * (tier.h:17,45 scan the slots per expert; a flag array is the same set). */
static unsigned char *tier_resident(int nexpert, const int *pinned, int npin) {
    unsigned char *r = calloc((size_t)nexpert, 1);
    if (!r) return NULL;
    for (int z = 0; z < npin; z++)
        if (pinned[z] >= 0 && pinned[z] < nexpert) r[pinned[z]] = 1;
    return r;
}

/* include/tier.h:35-54 */
int orc_tier_pick_lfru(const uint32_t *heat, const uint32_t *last, uint32_t clock, int nexpert, const int *pinned,
                       int npin, int *slot, int *eid, long *gain) {
    if (!heat || !last || !pinned || npin < 1 || nexpert < 1) return 0;
    int cold = 0;
    uint64_t cs = orc_tier_score(heat[pinned[0]], last[pinned[0]], clock);
    for (int z = 1; z < npin; z++) {
        const uint64_t v = orc_tier_score(heat[pinned[z]], last[pinned[z]], clock);
        if (v < cs) {
            cs = v;
            cold = z;
        }
    }
    unsigned char *res = tier_resident(nexpert, pinned, npin);
    if (!res) return 0;
    int hot = -1;
    uint64_t hs = 0;
    for (int e = 0; e < nexpert; e++) {
        if (res[e]) continue;
        const uint64_t v = orc_tier_score(heat[e], last[e], clock);
        if (hot < 0 || v > hs) {
            hot = e;
            hs = v;
        }
    }
    free(res);
    if (hot < 0 || hs <= cs + (cs >> 2) + (4u << 8)) return 0;
    *slot = cold;
    *eid = hot;
    *gain = (long)((hs - cs) >> 8);
    return 1;
}

/* include/tier.h:9-24 */
int orc_tier_pick_heat(const uint32_t *heat, int nexpert, const int *pinned, int npin, int *slot, int *eid,
                       long *gain) {
    if (!heat || !pinned || npin < 1 || nexpert < 1) return 0;
    int cold = 0;
    for (int z = 1; z < npin; z++)
        if (heat[pinned[z]] < heat[pinned[cold]]) cold = z;
    unsigned char *res = tier_resident(nexpert, pinned, npin);
    if (!res) return 0;
    int hot = -1;
    uint32_t hh = 0;
    for (int e = 0; e < nexpert; e++)
        if (!res[e] && heat[e] > hh) {
            hh = heat[e];
            hot = e;
        }
    free(res);
    if (hot < 0) return 0;
    const uint32_t hc = heat[pinned[cold]];
    /* the margin is computed in 32-bit unsigned arithmetic, as tier.h:20 */
    if (hh <= (uint32_t)(hc + (hc >> 2) + 4u)) return 0;
    *slot = cold;
    *eid = hot;
    *gain = (long)hh - (long)hc;
    return 1;
}

/* include/tier.h:56-58 */
void orc_tier_decay(uint32_t *heat, int nexpert) {
    for (int e = 0; e < nexpert; e++) heat[e] >>= 1;
}

void orc_tier_account(const int32_t *topk_idx, int nslots, int nexpert, uint32_t *heat, uint32_t *last,
                      uint32_t *clock, int decay_every) {
    const uint32_t clk = *clock + 1u;
    uint32_t *n = calloc((size_t)(nexpert > 0 ? nexpert : 1), sizeof(uint32_t));
    if (!n) return;
    for (int s = 0; s < nslots; s++)
        if (topk_idx[s] >= 0 && topk_idx[s] < nexpert) n[topk_idx[s]]++;
    for (int e = 0; e < nexpert; e++) {
        if (n[e]) {
            const uint64_t h = (uint64_t)heat[e] + n[e];
            heat[e] = h > 0xFFFFFFFFull ? 0xFFFFFFFFu : (uint32_t)h;
            last[e] = clk;
        }
        if (decay_every > 0 && clk % (uint32_t)decay_every == 0) heat[e] >>= 1;
    }
    *clock = clk;
    free(n);
}
