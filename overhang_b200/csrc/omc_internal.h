/* omc_internal.h -- internal types shared by the C host runtime (omc_host.c)
 * and the CUDA kernel files.  Not part of the public ABI (include/om_cuda.h).
 *
 * Expert weight layout in HBM ("tiled int8"): a row-major int8 matrix
 * W[O][K] is padded to O_pad = roundup(O,128), K_pad = roundup(K,64) with
 * zeros and stored as blocks of 128 rows x 64 columns (8 KiB each), blocks
 * ordered [row tile][K block]; inside a block the 16-byte chunk c (columns
 * 16c..16c+15) of row r sits at byte (c*128 + r)*16.  A warp reading 32
 * consecutive rows' chunk c reads 512 contiguous bytes, and one K block of a
 * row tile is one contiguous 8 KiB bulk copy.  Row scales are f32 padded with
 * zeros to O_pad.
 *
 * Activation operands of the tensor-core path ("AOL"): f16 rows of 64
 * elements (128 B) per K block, 8-row atoms of 1024 B with the 128-byte
 * swizzle (16-byte chunk c of row r stored at chunk c ^ (r & 7)), K blocks
 * outermost: element (row, k) of a [R][K_pad] operand lives at
 *   (k/64)*R*128 + row*128 + ((((k%64)/8) ^ (row&7)) * 16) + (k%8)*2.
 * A contiguous run of rows of one K block is a valid K-major SWIZZLE_128B
 * UMMA operand once copied 1024-byte aligned into shared memory.
 */
#ifndef OMC_INTERNAL_H
#define OMC_INTERNAL_H
#include <stdint.h>
#include <stddef.h>
#include <cuda_runtime.h>

#include "om_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define OMC_TM 128          /* rows per weight tile                       */
#define OMC_KB 64           /* int8 columns per K block                   */
#define OMC_BLK_BYTES (OMC_TM * OMC_KB)
#define OMC_ROW_ALIGN 16    /* expert row groups padded to 16 rows (UMMA N) */
#define OMC_MAX_K 32
#define OMC_MAX_E 1024
#define OMC_MAX_DEVICES 64

/* Size of the static device scratch behind omc_moe_forward_noalloc(). */
#define OMC_NOALLOC_SCRATCH_BYTES (32u << 20)

/* device error codes written into the error word */
#define OMC_DEVERR_TIMEOUT 1
#define OMC_DEVERR_BOUNDS  2
#define OMC_DEVERR_ROUTE   3
#define OMC_DEVERR_CONFIG  4
#define OMC_DEVERR_RANGE   5   /* an activation outside the f16 operand range */

/* error sites (err[1]) */
#define OMC_SITE_GEMM_PRODUCER 10
#define OMC_SITE_GEMM_DEQUANT  11
#define OMC_SITE_GEMM_MMA      12
#define OMC_SITE_GEMM_EPILOGUE 13
#define OMC_SITE_ROUTER        20
#define OMC_SITE_DISPATCH      21
#define OMC_SITE_GEMV          22
#define OMC_SITE_COMBINE       23
#define OMC_SITE_DECODE        24
#define OMC_SITE_TEST_WAIT     90

static inline int omc_round_up(int x, int m) { return (x + m - 1) / m * m; }

/* One expert's three tiled matrices and padded scales.
 *
 * Weights are stored as 128-row x 64-column int8 blocks (8 KiB; inside a
 * block, 16-byte chunk c of row r sits at (c*128 + r)*16) grouped in tile
 * PAIRS whose K blocks interleave: block kb of member m of pair p is at
 * ((p*nkb + kb)*2 + m) * 8 KiB, so one K block of a pair is 16 KiB of
 * contiguous memory (one bulk copy).  g and u share one buffer as members
 * 0 and 1 of pair mt (u = g + 8 KiB); the down matrix pairs its consecutive
 * row tiles 2p and 2p+1.  OMC_PAIR_STRIDE is the distance between two K
 * blocks of one tile. */
typedef struct {
    const int8_t *g, *u, *d;
    const float *gs, *us, *ds;
} omc_expert_ptrs;

#define OMC_PAIR_STRIDE (2 * OMC_BLK_BYTES)

/* Byte offset of block (row tile t, K block kb) of a matrix whose tiles pair
 * up consecutively (the down matrix). */
static inline __host__ __device__ size_t omc_dblk(int t, int kb, int nkb) {
    return ((size_t)((t >> 1) * nkb + kb) * 2 + (t & 1)) * OMC_BLK_BYTES;
}

/* Layer parameters handed to kernels by value. */
/* expert activation, h = act(g) * u */
#define OMC_ACT_SILU_DIV  0   /* g/(1+exp(-g))      engines/olmoe.c:393   */
#define OMC_ACT_SILU_SIG  1   /* g*(1/(1+exp(-g)))  engines/qwen.c:158,485 */
#define OMC_ACT_GELU_TANH 2   /* gelu_tanh(g)       engines/gemma.c:319,671 */

typedef struct {
    int family, D, I, E, k, renorm, router_i8, has_shared, Is;
    int act;                      /* OMC_ACT_* (the family's, or the caller's for job passes) */
    int D_pad, I_pad, Is_pad;     /* roundup(.., 64): K extent of a tiled matrix   */
    int D_rows, I_rows, Is_rows;  /* roundup(.., 128): row extent of a tiled matrix */
    const float *router;          /* f32 [E][D] (int8 routers stored as their exact f32 values) */
    const float *router_s;        /* [E] for int8 routers, else NULL */
    const float *sh_gate;         /* [D] or NULL */
    const omc_expert_ptrs *experts;  /* device table [E + 1]; entry E = shared expert */
    /* GEMMA only (NULL / 0 otherwise) */
    float eps;                    /* rms_norm_eps                                   */
    const float *g_s2;            /* [D] router.scale[i] * D^-0.5 (float product)   */
    const float *g_en;            /* [D] expert-input norm weight, NULL = ones      */
    const float *g_pes;           /* [E] per_expert_scale                           */
    const float *rbias;           /* [E] added to every router logit, or NULL       */
    /* bounded router (router_fast.cu; rf_tab NULL = exact router only): f16
     * tiles of the router rows as a one-matrix layer (rf_tab[0].d, .ds = ones),
     * rf_rows = E (int8 router: its values are exact in f16) or 2E (f32
     * router: the f16 rounding of each row, then the f16 rounding of the
     * remainder); rf_wn = [E] ||w_e||_2 then [E] ||w_e||_1, rounded up */
    const omc_expert_ptrs *rf_tab;
    int rf_rows, rf_split;
    const float *rf_wn;
    const unsigned char *rf_wc;   /* the router rows chunk-major for the chains' staging: chunk c
                                     (64 int8 or 16 f32 columns) of row e is 64 bytes at
                                     (c * E + e) * 64, its 16-byte piece p at slot
                                     p ^ ((e >> 1) & 3); NULL when D is not a multiple of the
                                     chunk.  OMC_RF_NREP copies rf_wc_stride bytes apart: the
                                     blocks of a pass walk the chunks in step (each chain's order
                                     is fixed), and block b reading copy b % OMC_RF_NREP spreads
                                     the same chunk's reads over more L2 slices */
    size_t rf_wc_stride;
    /* the exact router's rows in 16-row blocks (router.cu, router_tile2): block
     * rb, 128-column chunk c is 16 rows x 128 f32 (8 KB) at ((rb * (D/128) + c)
     * * 16 + r) * 128, the 16-byte unit u of row r at slot (u + r) % 32 (rows
     * read together differ in bank); row E is the shared gate (written by
     * omc_shared_set), rows past it zero; NULL when D % 128 != 0 */
    const float *rt_w;
    int rt_nrb;
} omc_layer_dev;

#define OMC_NMAX 128              /* token rows per grouped-GEMM work item (MMA N) */

/* The dispatch plan of a tensor-core forward (the batch union of
 * engines/olmoe.c:366-378, on the device): built by the last block of the
 * router's select kernel once every token's routing is written. */
typedef struct {
    int E, K, T, has_shared;
    int rows_mode;                /* 1: every slot is an explicit row (K = 1) whose
                                     expert id may be E (the shared expert); no
                                     implicit shared rows                          */
    int e_lo, e_hi;               /* routed experts resident here: [e_lo, e_hi)  */
    int I_rows, Is_rows, D_rows;  /* row extents of gate/up (routed, shared) and down */
    int R_cap, cap1, cap2;        /* operand rows and work-list capacities      */
    int *counts;                  /* [E + 1] rows per group (shared group: T)   */
    int *offsets;                 /* [E + 2] 16-row-padded row offsets          */
    int *nwork;                   /* [0] gate/up items [1] down items [2] rows  */
    int *slotrow;                 /* [T * K] rank of each routed slot in its expert */
    int *work1, *work2;           /* work items (g, mt, n0, n) as 4 ints        */
    int *rowinfo;                 /* [R] slot of each operand row (-1 padding)  */
    float *roww;                  /* [R] routing weight of each operand row     */
    int *done;                    /* select blocks finished; zero at start      */
} omc_plan_args;

/* Per-forward workspace (device pointers, grow-only). */
typedef struct {
    int T_cap, R_cap;             /* capacity in tokens and activation rows */
    float *x;                     /* [T][D] staging for host inputs       */
    float *out;                   /* [T][D] staging for host outputs      */
    float *logits;                /* [T][E + 1]                           */
    int32_t *topk_idx;            /* [T][k]                               */
    float *topk_w;                /* [T][k]                               */
    float *sg;                    /* [T] shared-gate sigmoid              */
    int *counts;                  /* [E + 2] rows per expert (+ shared)   */
    int *offsets;                 /* [E + 3] padded row offsets           */
    int *done;                    /* [1] select blocks finished (plan trigger) */
    int *slotrow;                 /* [T * k] rank of each routed slot in its expert */
    int *rowinfo;                 /* [R]: routed slot t*k+kk, T*k+t shared, -1 pad */
    float *roww;                  /* [R]: routing weight of the row (1 shared, 0 pad) */
    int *work;                    /* tile work list                       */
    int *nwork;                   /* [4] work counts                      */
    uint16_t *xh;                 /* [T][D] f16 token operand (tensor-core path) */
    uint16_t *hp;                 /* AOL f16 [Imax_pad/64][R][64]         */
    float *ypart;                 /* [T][k + 1][D]                        */
    float *hbuf;                  /* [T*k + T][Imax_pad] (GEMV path)      */
    float *xg_r, *xg_e;           /* GEMMA: [T][D] router and expert inputs */
    int *err;                     /* [4] device error word                */
    /* bounded router (router_fast.cu), NULL until a forward takes it */
    int rf_R;                     /* operand rows (>= 2T, a multiple of 128) */
    uint16_t *rf_act;             /* AOL f16 [D_pad/64][rf_R][64]: x_hi rows, then x_lo rows */
    float *rf_y;                  /* [2T][rf_rows] products of the row parts */
    int *rf_rowinfo;              /* [rf_R] identity rows (-1 padding) */
    float *rf_roww;               /* [rf_R] ones */
    int *rf_work;                 /* GEMM work items (int4) */
    int *rf_ctl;                  /* [16]: [0..3] GEMM nwork, [4] jobs, [5] retry jobs,
                                     [6] tokens taken whole from the start, [7] retried tokens */
    float *rf_xn;                 /* [T][D_pad/256][2] per 256-column segment: sum x^2, sum |x| (rounded up) */
    int *rf_tok;                  /* [T][4] first job, groups of 4, groups done, whole */
    int *rf_jobs;                 /* [cap][2] (token, row) chains; row -1 = padding */
    int *rf_jobs2;                /* [cap][2] retry chains */
    int rf_jcap;                  /* capacity of each job list */
} omc_ws;

/* ---- launchers (CUDA files), all enqueue on `s` ---------------------- */
/* member >= 0: tile t of src becomes member `member` of pair t (g, u);
 * member < 0: tiles pair up consecutively (d). */
int omc_launch_relayout(const int8_t *src, int O, int K, int8_t *dst, int O_pad, int K_pad, int member,
                        cudaStream_t s);
int omc_launch_i8_to_f32(const int8_t *src, float *dst, long long n, cudaStream_t s);
/* plan != NULL: the select kernel's last block also builds the dispatch plan
 * (and, except for GEMMA, the logits kernel writes the f16 token operand
 * ws->xh from x) */
int omc_launch_router(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                      int32_t *topk_idx, float *topk_w, const omc_plan_args *plan, cudaStream_t s);
/* fills the plan arguments of a tensor-core forward over workspace ws */
void omc_plan_setup(const omc_layer_dev *L, int T, const omc_ws *ws, omc_plan_args *pa);
int omc_launch_gemv_ffn(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                        const int32_t *topk_idx, const float *topk_w, float *out, cudaStream_t s);
int omc_launch_mma_ffn(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                       const int32_t *topk_idx, const float *topk_w, float *out, cudaStream_t s);
int omc_launch_test_wait(int *err, cudaStream_t s);
/* fused decode forward (decode.cu): the state (counters, zeroed once, and
 * pieces) serves every T <= 8 of a layer on a grid of G CTAs */
int omc_decode_state_size(const omc_layer_dev *L, int G, size_t *ctr_ints, size_t *part_floats);
int omc_decode_supported(const omc_layer_dev *L, int T, int G, size_t ctr_ints, size_t part_floats);
/* x = the input rows (GEMMA: the residual rows, normed in the kernel); xr =
 * the rows the router CTAs stage (x) */
int omc_launch_decode(const omc_layer_dev *L, const float *x, const float *xr, int T, const omc_ws *ws, int G, int *ctr,
                      float *part, int32_t *topk_idx, float *topk_w, float *out, cudaStream_t s);
/* GEMMA: router input xr, expert input xe (f32) and xh (f16 token operand)
 * of residual rows x, each nullable; r [T] the norm factor (nullable) */
int omc_launch_gemma_prenorm(const omc_layer_dev *L, const float *x, int T, float *xr, float *xe, uint16_t *xh,
                             float *r, int *err, cudaStream_t s);
long long omc_mma_work_items(const omc_layer_dev *L, int R);
/* job-driven pass helpers: rows[r] = x[pos[r]]; out[s] += y[list[j]] over j in [off[s], off[s+1]) in order */
int omc_launch_gather_rows(const float *x, const int *pos, int R, int S, int D, float *rows, int *err, cudaStream_t s);
int omc_launch_ordered_add(float *out, const float *y, const int *off, const int *list, int S, int D, cudaStream_t s);
/* explicit-rows pass: y[r] = w[r] * expert ids[r] (x[r]), ids in [e_lo, e_hi) or E (shared) */
int omc_launch_mma_rows(const omc_layer_dev *L, const float *x, int R, const omc_ws *ws, const int32_t *ids,
                        const float *w, int e_lo, int e_hi, float *y, cudaStream_t s);
/* dense pass: y[S][N] = x[S][K] . (ds * Wd)^T, Wd the down matrix of L's
 * expert 0 (L: E = 1, D = N, I = K with K % 64 == 0) */
int omc_launch_dense_i8(const omc_layer_dev *L, const float *x, int S, const omc_ws *ws, float *y, cudaStream_t s);
/* expert-parallel pass over explicit slots (ffn_mma.cu): y[s] = slot_w[s] *
 * expert slot_e[s] (operand row slot_tok[s] of xh); the slots were counted
 * into ws->counts / ws->slotrow already */
int omc_launch_mma_slots(const omc_layer_dev *L, const uint16_t *xh, int nslots, const int32_t *slot_tok,
                         const int32_t *slot_e, const float *slot_w, const omc_ws *ws, int e_lo, int e_hi, float *y,
                         cudaStream_t s);
/* expert-parallel exchange kernels (ep.cu; index arithmetic in omc_ep_plan.h) */
int omc_launch_ep_layout(const int32_t *idx, int T, int k, int ne, int P, int32_t *tok_pos, int32_t *slot_pos,
                         int32_t *counts, int32_t *pairs, cudaStream_t s);
int omc_launch_ep_pack(const float *x, const int32_t *idx, const float *w, int T, int D, int k, int ne, int P,
                       const int32_t *tok_pos, const int32_t *slot_pos, const int32_t *counts, uint16_t *send_x,
                       int32_t *send_meta, uint16_t *home_xh, int *err, cudaStream_t s);
int omc_launch_ep_unpack(const int32_t *meta, int Rr, int k, int P, const int *recv_base, const int *slot_base,
                         int Thome, int E, int e_lo, int e_hi, int has_shared, int Sr, int32_t *slot_tok,
                         int32_t *slot_e, float *slot_w, int *counts_e, int *slotrow, int *err, cudaStream_t s);
int omc_launch_ep_combine(const float *ret, const int32_t *slot_pos, const float *y_shared, const float *sg, int T,
                          int D, int k, int has_shared, float *out, cudaStream_t s);
int omc_launch_ep_ranksum(const int32_t *meta, int Rr, int k, int P, const int *recv_base, const int *slot_base,
                          const float *y, int D, float *rows, cudaStream_t s);
int omc_launch_ep_combine_ranksum(const float *ret, const int32_t *tok_pos, const int32_t *idx, const float *y_shared,
                                  const float *sg, int T, int D, int k, int ne, int P, int has_shared, float *out,
                                  cudaStream_t s);
/* omm_dense on the tensor cores: f16 weight tiles of a row-major f32 [N][K]
 * (K % 8 == 0; omc_f16_tiles_bytes bytes), and y[S][N] = x[S][K] . W^T with
 * L a one-matrix layer whose expert 0 has d = those tiles, ds = ones */
size_t omc_f16_tiles_bytes(int N, int K);
int omc_launch_f16_tiles(const float *W, int N, int K, uint16_t *dst, int *err, cudaStream_t s);
int omc_launch_dense_f16(const omc_layer_dev *L, const float *x, int S, const omc_ws *ws, float *y, cudaStream_t s);
/* bounded router: per-layer tiles and norms (host side, at omc_layer_init),
 * the GEMM over a prepared operand (ffn_mma.cu), and the forward's launches */
int omc_launch_rf_split_rows(const float *W, int E, int D, float *dst, cudaStream_t s);
/* rows row0.. row0+nr-1 of the exact router's row blocks from W [nr][D] */
int omc_launch_rt_blocks(const float *W, int row0, int nr, int D, float *dst, cudaStream_t s);
int omc_launch_gemm_dense_op(const omc_layer_dev *Ld, const uint16_t *act, int R, const int *rowinfo,
                             const float *roww, const int *work, const int *nwork, float *y, int *err,
                             cudaStream_t s);
int omc_rf_eligible(const omc_layer_dev *L, int T, const omc_ws *ws);
int omc_launch_router_fast(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws, uint16_t *xh,
                           cudaStream_t s);
/* smallest T, and by default the smallest E, that take the bounded router
 * (below: the exact router).  Under 128 experts the dense exact kernel, whose
 * register tiles share every staged operand, moves less data per routed
 * token than the candidates' chains, each with its own router row. */
#define OMC_RF_TMIN 16
#define OMC_RF_EMIN 128
#define OMC_RF_NREP 8
/* router mode (omc_set_router_exact): 0 auto, 1 exact, 2 bounded */
extern int omc_router_exact;
/* test hook: 1 = every token of a bounded pass is retried whole */
extern int omc_rf_force_retry;
/* fused decode: 1 = stream once the logit intervals decide the top-k sets */
extern int omc_decode_early;
/* decode state words: forwards the intervals decided, forwards that waited */
#define OMC_DEC_CTR_STATS 4
/* dst = f16(src), n % 8 == 0 */
int omc_launch_f32_to_f16(const float *src, long long n, uint16_t *dst, cudaStream_t s);
int omc_noalloc_setup(int device);
void *omc_noalloc_scratch_ptr(int device);
int omc_launch_expf_probe(const float *x, float *y, long long n, cudaStream_t s);

/* anything that changes what a forward enqueues calls this: the host entry's
 * replayed forwards are rebuilt */
void omc_graphs_invalidate(void);

/* a tiered layer after routing (tier.cu): hot-store counters (stats =
 * [heat E][last E][clock]), routed non-resident experts listed and pointed
 * at miss-area images, which are then filled from their home images.
 * layout = {image bytes, off_d, off_gs, off_us, off_ds}; list [1 + E];
 * total accumulates the misses. */
int omc_launch_tier_route(const int32_t *idx, int nslots, int E, uint32_t *stats, int decay_every,
                          omc_expert_ptrs *tab, const void *slots_lo, const void *slots_hi, const void *home,
                          void *miss, int miss_cap, const size_t *layout, int *list,
                          unsigned long long *total, int *err, int grid, cudaStream_t s);

/* profiling: ends the named stage on stream s (no-op unless profiling) */
void omc_prof_mark(cudaStream_t s, const char *name);

/* number of kernels launched by this library (launchers add to it) */
extern long long omc_g_launches;

#ifdef __cplusplus
}
#endif
#endif
