/* moe_oracle.h -- CPU oracle for the overhang MoE block.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load this code, and only as the checker.
 * The product (libomc.so) never links, loads or calls it.
 *
 * It restates, operation for operation, the reference C engines' MoE math:
 *   - OLMoE  moe()       engines/olmoe.c:344-402
 *   - Qwen   moe_step()  engines/qwen.c:453-495   (stream mode: int8 router,
 *                                                  int8 shared expert)
 *   - Gemma  route_token() engines/gemma.c:455-478 and the expert union of
 *                         step_batch() engines/gemma.c:606-685 (CPU path,
 *                         int8 stream-mode experts)
 * in the same floating-point order (sequential fp32 sums, no FMA
 * contraction, glibc expf), so that on identical inputs its outputs are
 * bit-identical to the reference built with gcc -O3 on x86-64.  That
 * bit-identity is checked against the reference itself (oracle/_ref) and
 * against golden vectors generated from it (tests/golden/).
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Model family: fixes the reference's arithmetic for routing, the SwiGLU
 * form and the combine order.  Same values as OMC_FAMILY_* in om_cuda.h. */
enum { ORC_FAMILY_OLMOE = 0, ORC_FAMILY_QWEN = 1, ORC_FAMILY_GEMMA = 2 };

/* Gemma's router norm takes (mean(x^2) + eps)^-0.5 with powf
 * (engines/gemma.c:313-317).  libm's powf is not correctly rounded: glibc
 * 2.39 on x86-64 is 1 ulp off the correctly rounded value for 207,500 of the
 * 335,544,321 floats in [2^-20, 2^20].  ORC_RSQRT_LIBM calls powf (the
 * reference on this host, bit for bit); ORC_RSQRT_CR rounds the double
 * 1/sqrt once to float, the value the device computes. */
enum { ORC_RSQRT_CR = 0, ORC_RSQRT_LIBM = 1 };

typedef struct {
    int family;        /* ORC_FAMILY_* */
    int D, I, E, k;    /* hidden, expert FFN width, experts, top-k */
    int renorm;        /* olmoe: config norm_topk_prob (olmoe.c:194,363); qwen: always 1 (qwen.c:476-477) */
    int router_i8;     /* 0: f32 router [E,D] (olmoe.c:74-85); 1: int8 [E,D] + f32 scale[E] (qwen.c:284,465) */
    int has_shared;    /* qwen shared expert (qwen.c:455-462) */
    int Is;            /* shared expert FFN width */
    float eps;         /* gemma: rms_norm_eps (gemma.c:94) */
    int rsqrt_mode;    /* gemma: ORC_RSQRT_* */
} orc_desc;

/* Expert weights, packed expert-major (the int8 container layout of
 * tools/convert_olmoe.py:32-38 per expert, concatenated):
 *   g, u : int8 [E][I][D]   gs, us : f32 [E][I]
 *   d    : int8 [E][D][I]   ds     : f32 [E][D]
 * Shared expert (qwen): sh_g, sh_u int8 [Is][D], sh_d int8 [D][Is], their
 * f32 row scales, and sh_gate f32 [D] (kept f32 by qwen.c:282,460). */
typedef struct {
    const void   *router;   const float *router_s;
    const int8_t *g, *u, *d;
    const float  *gs, *us, *ds;
    const int8_t *sh_g, *sh_u, *sh_d;
    const float  *sh_gs, *sh_us, *sh_ds, *sh_gate;
    /* gemma (gemma.c:422-424, :608): router.scale [D], router.per_expert_scale
     * [E], pre_feedforward_layernorm_2 [D] (nullable: ones) */
    const float  *g_rscale, *g_pes, *g_enorm;
    /* router bias [E] (nullable): added to each routed logit before the
     * softmax.  A harness input with no counterpart in the reference (the
     * engines have no bias term); benchmarks use it to skew expert load. */
    const float  *router_bias;
} orc_weights;

/* For the GEMMA family, x is the layer's residual stream (the row
 * route_token reads, gemma.c:582): the router input is
 * rms(x) * router.scale * D^-0.5 and the experts' input rms(x) *
 * pre_feedforward_layernorm_2, both computed here (and on the device).  The
 * experts are gelu_tanh(g) * u (gemma.c:319-321, :671), and a token's hits are
 * combined in ascending expert id (the union order of gemma.c:641-685). */

/* out[T,D] = MoE(x[T,D]).  topk_idx/topk_w [T,k] (nullable) receive the
 * routing in selection order.  Returns 0, or -1 on a bad descriptor. */
int orc_moe(const orc_desc *dsc, const orc_weights *w, const float *x, int T,
            float *out, int32_t *topk_idx, float *topk_w);

/* Routing only (router GEMV + softmax + top-k + optional renorm), same rules. */
/* One expert per row, unweighted: y[r] = expert ids[r] applied to x[r]
 * ([D] -> [D]), with the reference's arithmetic for one expert of moe() /
 * moe_step() (engines/olmoe.c:386-394, engines/qwen.c:480-491); id E is the
 * shared expert (engines/qwen.c:455-459, before its sigmoid gate).  Returns
 * -1 on a bad descriptor or id.  (Expert-parallel tests sum these rows.) */
int orc_expert_rows(const orc_desc *dsc, const orc_weights *w, const float *x, int R, const int32_t *ids,
                    float *y);

/* GEMMA: the router input xr and the expert input xe [T,D] of residual rows x,
 * and the norm factor r [T] (engines/gemma.c:313-317, :458-460, :608). */
int orc_gemma_prenorm(const orc_desc *dsc, const orc_weights *w, const float *x, int T,
                      float *xr, float *xe, float *r);

/* Expert activations (h = act(g) * u); ORC_ACT_x equals the family whose
 * form it is: olmoe.c:393, qwen.c:158,485, gemma.c:319-321,671. */
enum { ORC_ACT_SILU_DIV = 0, ORC_ACT_SILU_SIG = 1, ORC_ACT_GELU_TANH = 2 };

/* Like orc_expert_rows for routed experts, with the activation given and the
 * rows taken as the experts' input as they are (no GEMMA norm): the
 * omm_moe_act job pass (metal/om_metal.h:49-51, `gelu` selects gelu_tanh). */
int orc_expert_rows_act(const orc_desc *dsc, const orc_weights *w, const float *x, int R, const int32_t *ids,
                        int act, float *y);

/* sg[t] = sigmoid(sum_i sh_gate[i] * x[t][i]) (engines/qwen.c:460-461). */
int orc_shared_gate(const orc_desc *dsc, const orc_weights *w, const float *x, int T, float *sg);

int orc_route(const orc_desc *dsc, const orc_weights *w, const float *x, int T,
              int32_t *topk_idx, float *topk_w);

/* Per-row symmetric int8 quantiser of the container converters
 * (tools/convert_olmoe.py:32-38): s = max(amax,1e-12)/127,
 * q = clamp(round_half_even(w/s), -128, 127). */
void orc_quantize_rows_py(const float *w, int O, int I, int8_t *q, float *s);

/* The engines' load-time quantiser (qwen.c:124-138, olmoe.c:145-161 with
 * bits=8): s = max(amax/127, 1e-8), q = clamp(lrintf(w/s), -128, 127).
 * qwen.c uses it for the router and the shared expert in stream mode. */
void orc_quantize_rows_c(const float *w, int O, int I, int8_t *q, float *s);

/* SplitMix64 + Box-Muller generator shared by tests and bench so that CPU
 * and GPU legs see identical seeded inputs.  fills n floats ~ N(0, sigma). */
void orc_fill_normal(uint64_t seed, float *dst, int64_t n, float sigma);

/* glibc expf as called by the reference (exposed so tests can compare the
 * device restatement of the same function against it). */
float orc_expf(float x);
void orc_expf_array(const float *x, float *y, int64_t n);

/* The hot-store replacement policy of include/tier.h (the reference header
 * has no caller in its engines; these restate its three functions).
 *
 * orc_tier_score (tier.h:30-33): (heat << 8) | recency, recency = 255 - age
 * for age = clock - last (unsigned, wraps) below 255, else 0.
 *
 * orc_tier_pick_lfru (tier.h:35-54): the coldest resident slot (lowest score,
 * first slot on ties) and the hottest non-resident expert (highest score,
 * lowest id on ties, the first one taken even at score 0); a swap only when
 * hot > cold + cold/4 + 4*256.  Returns 1 and fills slot/eid/gain
 * ((hot-cold) >> 8) on a swap, else 0; 0 on a null array, npin < 1 or
 * nexpert < 1.
 *
 * orc_tier_pick_heat (tier.h:9-24): the same on heat alone (margin
 * cold/4 + 4, a zero-heat expert is never picked).
 *
 * orc_tier_decay (tier.h:56-58): heat >>= 1 for every expert. */
uint64_t orc_tier_score(uint32_t heat, uint32_t last, uint32_t clock);
int orc_tier_pick_lfru(const uint32_t *heat, const uint32_t *last, uint32_t clock, int nexpert, const int *pinned,
                       int npin, int *slot, int *eid, long *gain);
int orc_tier_pick_heat(const uint32_t *heat, int nexpert, const int *pinned, int npin, int *slot, int *eid,
                       long *gain);
void orc_tier_decay(uint32_t *heat, int nexpert);

/* The heat a tiered layer gathers from one forward's routing (the library's
 * own accounting, which the reference leaves to its caller): clock += 1;
 * for every expert e routed n > 0 times among the T*k slots, heat[e] += n
 * (saturating at 2^32-1) and last[e] = clock; then, when decay_every > 0 and
 * clock % decay_every == 0, heat >>= 1 for every expert. */
void orc_tier_account(const int32_t *topk_idx, int nslots, int nexpert, uint32_t *heat, uint32_t *last,
                      uint32_t *clock, int decay_every);

#ifdef __cplusplus
}
#endif
#endif
