/* om_cuda.h -- B200 (sm_100a) mixture-of-experts block, C ABI.
 *
 * This is the device-side replacement for the MoE layer of the overhang C
 * engines.  Routing, token->expert dispatch, the int8-dequant expert SwiGLU
 * products and the weighted combine all run on the GPU; the caller hands in
 * the post-norm activations x[T,D] and receives out[T,D].
 *
 * Reference interfaces this header replaces:
 *   - moe()       engines/olmoe.c:344-402  (router + top-k + experts + combine)
 *   - moe_step()  engines/qwen.c:453-495   (shared expert + router + experts)
 *   - route_token() + the expert union of step_batch()
 *                 engines/gemma.c:455-478, :580-685 (GEMMA family)
 *   - the GPU seam metal/om_metal.h:14-46 (omm_*), whose prototypes are
 *     mirrored one-for-one by om_metal.h in this directory.
 *
 * Conventions
 *   - Plain C types only: pointers, sizes, ints.  No CUDA or torch types.
 *   - Every entry point returns an OMC_* status (0 = OK, < 0 = error); there
 *     is no CPU fallback.  omc_strerror() names a status; omc_last_error()
 *     returns the detail string of the last failure on this thread.
 *   - One process drives one GPU (omc_init(device, ...)); expert parallelism
 *     across GPUs is joined with omc_ep_init().
 *   - Calls are made from one host thread, as the engines do
 *     (engines/olmoe.c:405-427).
 */
#ifndef OM_CUDA_H
#define OM_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define OMC_OK          0
#define OMC_EINVAL     -1   /* bad argument / descriptor / shape          */
#define OMC_ENOMEM     -2   /* device, pinned or slab allocation failed   */
#define OMC_ENOINIT    -3   /* omc_init / omc_layer_init not called        */
#define OMC_ECUDA      -4   /* CUDA runtime error                          */
#define OMC_EDEVICE    -5   /* a kernel reported an error (bounds, wait)   */
#define OMC_ETIMEOUT   -6   /* a bounded wait expired (device or NCCL)     */
#define OMC_ENCCL      -7   /* NCCL error or NCCL unavailable              */
#define OMC_EUNSUPPORTED -8 /* valid request this build does not handle    */
#define OMC_ERANGE     -9   /* an activation outside the tensor-core path's
                               f16 operand range (|v| >= 65520 or NaN): the
                               forward's results are not valid.  The blocking
                               entry omc_moe_forward recomputes such a forward
                               on the f32 CUDA-core path and never returns it */

/* ---- layer descriptor ------------------------------------------------ */
/* Model family fixes the reference's arithmetic: the router's softmax sum
 * precision, the SwiGLU form and the combine order.
 *   OLMOE: softmax_row float sum (engines/olmoe.c:170-174), silu as
 *          g/(1+exp(-g)) (olmoe.c:393), out = sum_k w_k*y_k (olmoe.c:395-397)
 *   QWEN : softmax_ double sum (engines/qwen.c:161-165), silu as
 *          g*sigmoid(g) (qwen.c:158-159), renormalised top-k, out =
 *          sigmoid(sh_gate.x)*shared(x) + sum_k w_k*y_k (qwen.c:455-492)
 *   GEMMA: x is the RESIDUAL row (engines/gemma.c:582).  The router reads
 *          rms(x)*router.scale*D^-0.5 and the experts rms(x)*
 *          pre_feedforward_layernorm_2 (gemma.c:458-460, :608); top-k over
 *          the softmax numerators, renormalised, times per_expert_scale
 *          (gemma.c:461-477); experts gelu_tanh(g)*u (gemma.c:319-321,
 *          :671); no shared expert.  Needs omc_layer_gemma_norms().
 *          out = sum_k w_k*y_k, the MoE term before post_feedforward_
 *          layernorm_2 (gemma.c:691). */
#define OMC_FAMILY_OLMOE 0
#define OMC_FAMILY_QWEN  1
#define OMC_FAMILY_GEMMA 2

#define OMC_ROUTER_F32 0    /* router weights f32 [E,D]                       */
#define OMC_ROUTER_I8  1    /* int8 [E,D] + f32 scale [E] (qwen.c:284 stream)  */

typedef struct omc_moe_desc {
    int family;        /* OMC_FAMILY_*                                          */
    int D;             /* hidden size (multiple of 64)                          */
    int I;             /* routed-expert FFN width (multiple of 16)              */
    int E;             /* routed experts (<= 1024)                              */
    int k;             /* experts per token (<= 32)                             */
    int renorm;        /* 1: top-k weights divided by their sum (forced for QWEN, GEMMA) */
    int router_dtype;  /* OMC_ROUTER_*                                          */
    int has_shared;    /* 1: always-on shared expert behind a sigmoid gate (QWEN) */
    int Is;            /* shared-expert FFN width (multiple of 64)               */
} omc_moe_desc;

/* ---- lifetime ------------------------------------------------------- */

/* Bind this process to CUDA `device` and reserve the HBM expert slab.
 * slab_bytes = 0: use free HBM minus a 4 GiB reserve.  An upload past the
 * budget fails with OMC_ENOMEM (a layer larger than its share of HBM uses
 * omc_tier_enable).  Replaces omm_init (metal/om_metal.h:13-14). */
int omc_init(int device, size_t slab_bytes);

/* Free every device and pinned resource (and the NCCL communicator). */
void omc_shutdown(void);

/* Describe layer `layer` and upload its router.  router_w is f32 [E,D] or
 * int8 [E,D] with router_s f32 [E].  Replaces the router weights the engines
 * keep resident (engines/olmoe.c:226, engines/qwen.c:278,284). */
int omc_layer_init(int layer, const omc_moe_desc *desc,
                   const void *router_w, const float *router_s);

/* GEMMA layers: the router's norm parameters and the experts' input norm
 * (engines/gemma.c:409, :423-424): router_scale [D] (router.scale),
 * per_expert_scale [E] (router.per_expert_scale), expert_norm [D]
 * (pre_feedforward_layernorm_2 weight; NULL = ones) and eps
 * (rms_norm_eps).  Call after omc_layer_init, before the first forward.
 * The router's rms factor (mean(x^2)+eps)^-0.5 is the correctly rounded
 * value; the reference's libm powf is up to 1 ulp from it (0.06% of rows on
 * glibc), which moves those rows' top-k weights by a few ulps. */
int omc_layer_gemma_norms(int layer, float eps, const float *router_scale, const float *per_expert_scale,
                          const float *expert_norm);

/* Router bias: bias [E] is added to expert e's router logit before the
 * softmax (one f32 add: p = softmax(logit + bias)); NULL removes it.  This
 * input has no counterpart in the reference: it lets a benchmark skew the
 * expert load (e.g. bias_e = -1.1*ln(rank_e), a Zipf(1.1) preference over a
 * permutation of the experts) on random-init weights.  The oracle adds it at
 * the same point, so routing stays bit-exact with it.  Every value must be
 * finite (OMC_EINVAL otherwise). */
int omc_layer_router_bias(int layer, const float *bias);

/* Router of the forwards with T >= 16 (OLMoE- and Qwen-family layers with
 * D % 8 == 0; T < 16 and GEMMA layers always take the exact router).
 *   mode 1, exact:   the reference's sequential fp32 chain (engines/olmoe.c:
 *                    74-85, engines/qwen.c:116-121) for every (token, expert);
 *                    topk_idx and topk_w bit-exact.
 *   mode 2, bounded: approximate logits on the tensor cores with a proven
 *                    error interval, the exact chain only for the experts
 *                    whose interval can reach the top k and for the shared
 *                    gate, and every row exact for the rare token whose
 *                    selection order could depend on the rest.  topk_idx is
 *                    bit-exact; topk_w is within a few ulps of the reference's
 *                    (its softmax sum includes the approximated logits of
 *                    experts that cannot be selected).
 *   mode 0 (the default): bounded for layers of 128 experts or more, exact
 *                    below (where the dense exact kernel moves less data). */
int omc_set_router_exact(int mode);
/* Counters of the library's last bounded-router pass: out[0] exact chains
 * run, out[1] chains of retried tokens, out[2] tokens taken whole from the
 * start (non-finite or out-of-range values, too many candidates), out[3]
 * tokens retried.  Synchronises the library's stream. */
int omc_router_stats(int *out);

/* The fused decode forward (T <= 8 tokens, one launch) starts streaming the
 * experts' weights as soon as intervals on the logits decide every token's
 * top-k set; the exact chains, the selection's weights and order, and the
 * combine follow.  out[0] = forwards the intervals decided, out[1] = forwards
 * that waited for the exact selection (a near-tie at the k-th expert, a
 * non-finite value), since the last reset; reset != 0 zeroes them.
 * Synchronises the device. */
int omc_decode_stats(int *out, int reset);

/* Upload routed expert e of a layer into the HBM slab (re-tiled for the
 * kernels).  Row-major int8 container tensors as written by the converters
 * (tools/convert_olmoe.py:93-99): g,u [I,D], d [D,I], per-row f32 scales
 * gs,us [I], ds [D].  Replaces expert_get's disk fill
 * (engines/olmoe.c:250-272, engines/qwen.c:428-450). */
int omc_expert_set(int layer, int e,
                   const int8_t *g, const float *gs, const int8_t *u, const float *us,
                   const int8_t *d, const float *ds);

/* The same for all E experts at once from expert-major packed arrays:
 * g,u [E,I,D], d [E,D,I], gs,us [E,I], ds [E,D]. */
int omc_experts_set_packed(int layer,
                           const int8_t *g, const float *gs, const int8_t *u, const float *us,
                           const int8_t *d, const float *ds);

/* GEMMA's container keeps gate and up fused (gate_up_proj int8 [2I,D] with
 * .qs [2I], engines/gemma.c:342-361): pass g = gate_up, u = gate_up + I*D,
 * gs = qs, us = qs + I. */

/* Upload the routed experts of `layer` that this process holds straight from
 * the engines' int8 container: every *.safetensors file of directory
 * `snapshot` (one shard each).  name_g, name_u, name_d are printf patterns
 * taking the container's layer index `src_layer` (the engine's layer, which
 * the engines' hooks also use as the library's layer id) then the expert id,
 * e.g.
 *   "model.layers.%d.mlp.experts.%d.gate_proj.weight"   (OLMoE, Qwen)
 * each tensor int8 [rows][cols] with its f32 row scales at name + ".qs"
 * (tools/convert_olmoe.py:93-99).  name_u = NULL: name_g is the fused
 * gate_up [2I,D] (Gemma, "model.layers.%d.experts.%d.gate_up_proj",
 * tools/convert_gemma.py:386-394).  nthreads reader threads (0 = 8) read
 * the tensors into pinned staging while the caller's thread uploads the
 * finished experts in order.  Replaces the engines' per-expert disk fill
 * (expert_get, engines/olmoe.c:250-272) at load time.  A missing tensor or
 * a dtype/shape that differs from the layer: OMC_EINVAL, naming it. */
int omc_experts_load(int layer, const char *snapshot, int src_layer, const char *name_g, const char *name_u,
                     const char *name_d, int nthreads);

/* ---- tiered expert store (layers larger than their HBM share) -------- */

/* Keep only `hbm_slots` of the layer's routed experts in HBM; every expert
 * gets a home copy in mapped pinned host memory.  A forward that routes to
 * a non-resident expert copies it from its home into an HBM miss area right
 * after routing (one crossing of the host link); kernels read HBM only.  The
 * T = 1 forward of a tiered layer takes the router + CUDA-core path, not the
 * fused decode kernel.  Replaces the engines' RAM expert
 * cache (expert_get, engines/olmoe.c:250-272) one level up, with the
 * reference's hot-store policy (include/tier.h:30-58): the device counts
 * each forward's routings per expert (heat += slots, last = clock, clock
 * += 1 per forward; heat halved every `decay_every` forwards, 0 = never);
 * every `interval` forwards (0 = only omc_tier_step) the counters are read
 * asynchronously and at most one swap is made -- the coldest slot by LFRU
 * score (heat << 8 | recency) for the hottest non-resident expert, only past
 * a 25% + 4-routing margin.  A swap is stream-ordered ahead of the next
 * forward and changes no result.  Call after omc_layer_init and before the
 * experts are uploaded (the first hbm_slots uploaded start resident).  Not
 * with expert parallelism.  Forwards of a tiered layer must be ordered
 * (one stream, or synchronised by the caller). */
int omc_tier_enable(int layer, int hbm_slots, int interval, int decay_every);

/* Synchronously read the counters and apply at most one swap now; *eid
 * (nullable) = the expert moved into HBM, or -1. */
int omc_tier_step(int layer, int *eid);

/* The counters (heat, last [E], clock; each nullable), the expert in each
 * HBM slot ([hbm_slots], -1 = not filled yet), the swaps made so far and
 * the misses so far (routed non-resident experts copied in, summed over
 * forwards). */
int omc_tier_stats(int layer, uint32_t *heat, uint32_t *last, uint32_t *clock, int32_t *slot_expert,
                   long long *swaps, long long *misses);

/* The replacement rule alone (no device needed): include/tier.h:35-54's
 * tier_pick_lfru with the same arguments and result. */
int omc_tier_pick(const uint32_t *heat, const uint32_t *last, uint32_t clock, int nexpert, const int *pinned,
                  int npin, int *slot, int *eid, long *gain);

/* QWEN shared expert: g,u int8 [Is,D], d int8 [D,Is], their row scales, and
 * the f32 gate vector sh_gate [D] (engines/qwen.c:279-287). */
int omc_shared_set(int layer,
                   const int8_t *g, const float *gs, const int8_t *u, const float *us,
                   const int8_t *d, const float *ds, const float *sh_gate);

/* ---- forward -------------------------------------------------------- */

/* out[T,D] = MoE_layer(x[T,D]) with HOST pointers (blocking).  topk_idx and
 * topk_w (nullable, [T,k]) receive the routing in selection order.
 * Drop-in for moe(m, l, layer, x, S, out) (engines/olmoe.c:344). */
int omc_moe_forward(int layer, const float *x, int T, float *out,
                    int32_t *topk_idx, float *topk_w);

/* omc_moe_forward as a pipeline: enqueues the upload of x, the forward and
 * the download of out / topk_idx / topk_w (nullable) and returns at once
 * with *ticket; omc_moe_wait(ticket) returns when that call's results are in
 * the host buffers.  Consecutive calls overlap: the upload of the next call's
 * x and the download of the previous call's out run on their own copy
 * streams while a forward runs, so a serving loop that keeps two or three
 * calls in flight pays for the host<->device copies only where they exceed
 * the forward.  x must stay unchanged until the call's ticket is waited for
 * (or the next three calls were submitted), and out/topk until its wait;
 * pinned host memory (cudaHostAlloc / cudaHostRegister) makes the copies
 * asynchronous.  At most three calls are in flight: a fourth first waits for
 * the oldest.  A device-side error is reported by the next omc_moe_wait; an
 * OMC_ERANGE forward is not recomputed here (omc_moe_forward does that).  Not
 * for expert-parallel layers (OMC_EUNSUPPORTED). */
int omc_moe_forward_async(int layer, const float *x, int T, float *out,
                          int32_t *topk_idx, float *topk_w, long long *ticket);
int omc_moe_wait(long long ticket);

/* The same with DEVICE pointers, enqueued on `stream` (a cudaStream_t; NULL
 * = the library's stream).  Returns once enqueued; the caller synchronises.
 * x and out must be 16-byte aligned (OMC_EINVAL otherwise): rows are moved
 * with 16-byte bulk copies and vector stores. */
int omc_moe_forward_dev(int layer, const float *x, int T, float *out,
                        int32_t *topk_idx, float *topk_w, void *stream);

/* The same as omc_moe_forward_dev, but it allocates nothing: no cudaMalloc,
 * cudaFree or other allocating call, on any call.  This entry has no
 * counterpart in the reference.
 *
 * It is for callers that must not allocate device memory per call: an engine
 * that has reserved its whole HBM budget up front (expert slab, KV cache) and
 * must keep a fixed footprint, or a serving loop that may not stall in the
 * driver's allocator between tokens.  The other forward entries grow their
 * workspace with cudaMalloc when T grows; this one takes it from a fixed
 * 32 MiB device array that the library holds on every GPU it is loaded on
 * until the process exits (its address is looked up once, in omc_init).
 *
 * Limit: a forward whose workspace does not fit those 32 MiB is rejected with
 * OMC_EINVAL and a message giving the largest T for the layer (for the
 * OLMoE-shaped layer, D=2048 E=64 k=8 I=1024, T=238; for the Qwen-shaped
 * one, E=256 I=512 with its shared expert, T=273).  The caller still
 * passes x, out and the optional top-k buffers as device pointers.  Every call
 * uses the same array, which keeps the previous call's contents; the counters
 * that must start at zero are cleared on `stream` by each call.  Two calls
 * that can run at the same time on the GPU (different streams with no
 * ordering between them) race on the array: order them on one stream.  The
 * T = 1 fused decode kernel's counters (set up by omc_layer_init) and a
 * tiered layer's miss area are shared with the other forward entries as
 * well, so a no-alloc forward must also be ordered with every other forward
 * of the library (one stream, or events). */
int omc_moe_forward_noalloc(int layer, const float *x, int T, float *out,
                            int32_t *topk_idx, float *topk_w, void *stream);

/* ---- building blocks for expert parallelism ------------------------ */
/* A caller that spreads the experts of a layer over GPUs (one process per
 * GPU, its own exchange, e.g. torch.distributed) composes a forward from
 * these two.  Both take device pointers and enqueue on `stream`.
 *
 * omc_moe_route_dev: the router alone (the first half of moe(),
 * engines/olmoe.c:347-364 / moe_step(), engines/qwen.c:463-477): topk_idx,
 * topk_w [T,k] in selection order, and for layers with a shared expert the
 * sigmoid gate shared_gate [T] (nullable) of engines/qwen.c:460-461.
 *
 * omc_moe_experts_dev: y[r] = weight[r] * expert[r](x_rows[r]) for R rows of
 * D floats, each with its own expert: a routed expert resident on this
 * process (see omc_ep_init for the resident range; all of them when no
 * group was joined) or E for the layer's shared expert (weight 1 then gives
 * the unweighted shared output).  The product is rounded exactly as the
 * forward rounds w * y (engines/olmoe.c:396), so summing a token's rows in
 * selection order after sigmoid(gate) * shared reproduces omc_moe_forward
 * bit for bit.  A row naming a non-resident expert is skipped and reported
 * as OMC_EDEVICE by the next omc_sync.  x_rows and y are 16-byte aligned. */
int omc_moe_route_dev(int layer, const float *x, int T, int32_t *topk_idx, float *topk_w, float *shared_gate,
                      void *stream);
int omc_moe_experts_dev(int layer, const float *x_rows, int R, const int32_t *expert, const float *weight,
                        float *y, void *stream);

/* Wait for all work of the library; reports a pending device error. */
int omc_sync(void);

/* ---- expert parallelism (1 process per GPU) ------------------------- */

/* Declare this process rank `rank` of `world` expert-parallel ranks, one
 * process per GPU (call after omc_init, before the first omc_layer_init;
 * world <= 16).  Layers initialised afterwards hold only routed experts
 * [rank*E/world, (rank+1)*E/world) in the slab (omc_expert_set ignores the
 * others) plus the shared expert; E must be divisible by world.
 *
 * unique_id = the 128 bytes rank 0 got from omc_ep_unique_id, passed to
 * every rank by the caller (any channel): the ranks join one NCCL group
 * (NCCL is loaded at run time; OMC_ENCCL if absent), and omc_moe_forward /
 * omc_moe_forward_dev on a layer run the whole expert-parallel forward of
 * this rank's own T tokens (any T >= 0, every rank calling for the same
 * layer in the same order): route, each token sent once to every rank
 * holding one of its experts (f16 rows), the experts there, the weighted f32
 * partials back, and the combine at home in the reference's order; the
 * result equals one GPU's tensor-core forward bit for bit.  One host wait per
 * forward (the per-peer row counts) is bounded, see omc_ep_set_timeout.
 *
 * unique_id = NULL: no group; the caller composes a forward from
 * omc_moe_route_dev and omc_moe_experts_dev over its own transport, and
 * omc_moe_forward[_dev] on such a layer returns OMC_EUNSUPPORTED. */
int omc_ep_init(int rank, int world, const void *unique_id);

/* A new NCCL unique id (rank 0; len >= 128 bytes) for omc_ep_init. */
int omc_ep_unique_id(void *buf, size_t len);

/* The deadline of every host wait of an expert-parallel forward (default
 * 30000 ms): the wait polls the work's completion and the NCCL
 * communicator's asynchronous error; past the deadline (a peer rank that
 * left or stopped calling) or on an NCCL error the communicator is aborted
 * and the call returns OMC_ETIMEOUT or OMC_ENCCL.  Later expert-parallel
 * forwards return OMC_ENCCL until omc_ep_init joins a new group. */
int omc_ep_set_timeout(int timeout_ms);

/* How the expert ranks return their results (every rank of a group must use
 * the same mode):
 *   OMC_EP_EXACT   one f32 row per routed slot, summed at home in selection
 *                  order: the result equals one GPU's forward bit for bit
 *                  (the default);
 *   OMC_EP_RANKSUM one f32 row per (token, expert rank), the sum of the
 *                  token's slots on that rank in selection order, added at
 *                  home rank by rank: fewer bytes back (one row per token and
 *                  rank instead of one per slot: 4x fewer at 2 ranks of top-8),
 *                  the same terms in another order (within the parity
 *                  tolerance of the reference, not bit-equal to one GPU). */
#define OMC_EP_EXACT   0
#define OMC_EP_RANKSUM 1
int omc_ep_set_combine(int mode);

/* Waits, with that deadline, for the last expert-parallel forward enqueued by
 * omc_moe_forward_dev (its stream), then reports a pending device error.
 * omc_sync does the same first when a group was joined. */
int omc_ep_wait(void);

/* ---- introspection -------------------------------------------------- */

const char *omc_strerror(int status);
const char *omc_last_error(void);

/* Per-stage device time of the last forward (milliseconds, CUDA events on
 * the launching stream) when profiling is on: stages are router, dispatch,
 * expert gate/up, expert down, combine, exchange.  Returns the number of
 * stages written. */
int omc_set_profiling(int on);
int omc_stage_times(float *ms, int n);

/* Name of stage i of the last profiled forward ("router", "dispatch",
 * "gemm_gateup", "gemm_down", "combine", "gemv_gateup", ...), or NULL. */
const char *omc_stage_name(int i);

/* Stage timer for benchmarks: from this call on, every forward records one
 * pair of CUDA events on its launching stream, at the boundaries just before
 * and just after the stage called `name` (a name omc_stage_name reports, e.g.
 * "gemm_gateup"); no other event is kept and nothing is synchronised, so the
 * forwards run as they do untimed.  name = NULL stops.  omc_stage_timer
 * returns the mean duration of that stage over the timed forwards (the last
 * 1023 when more ran) and how many it averaged. */
int omc_time_stage(const char *name);
int omc_stage_timer(float *mean_ms, int *count);

/* Number of kernels the library launched since the last reset (a count of
 * its own launches, not of library calls it makes). */
long long omc_launch_count(int reset);

/* Build and version string. */
const char *omc_version(void);

#ifdef __cplusplus
}
#endif
#endif
