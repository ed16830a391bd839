// decode.cu -- the whole MoE block for decode-sized batches in one launch.
//
// For T <= 8 tokens the block is HBM-bound on the selected experts' int8
// weights (OLMoE T=1: 50 MB, 7.8 us at 6.4 TB/s) after a router whose exact
// fp32 chain (D dependent adds, ~4.5 us) cannot be shortened -- but only the
// routing weights and order need the chain; the weight stream needs only the
// set of selected experts.  One cooperative launch of one CTA per SM:
//
//  1. router: CTAs 0..nrc-1 each take rr = ceil((E + shared)/G) router rows
//     and bulk-copy them in four column chunks.  Their select warp runs the
//     reference's chain for every (token, row) (engines/olmoe.c:74-85,
//     engines/qwen.c:116-121: acc = RN(acc + RN(x*w)), i ascending) as the
//     chunks land, and counts itself done.  Meanwhile the other warps sum the
//     same products in double, with their prefix sums, into an interval that
//     provably holds the chain's logit (dec_interval), publish it and count.
//  2. select: every CTA waits for the interval count and takes each token's
//     top-k set from the intervals (omc_bounds.cuh).  When every set is
//     decided (exactly k candidates) it plans and streams at once; the
//     select warp then waits for the exact logits and runs select_token
//     (softmax, top-k, renorm, shared gate: bit-exact, omc_select.cuh) beside
//     the stream, for the combine.  A set that is not decided (a near tie at
//     the k-th place, a non-finite value) makes every CTA wait for the exact
//     logits and select first, as the reference does.  The select warp of
//     CTA 0 writes the routing out.
//  3. plan: one warp groups the routed slots by expert (ascending id, slot
//     order inside a group: a bitmap and match masks), plus the shared expert
//     with every token (engines/qwen.c:459-462).
//  4. stream: the gate/up blocks of all groups (list A: group, row tile, K
//     block) and the down blocks (list B: group, row-tile pair, K block) are
//     16 KiB each in the paired tile layout and are split evenly over the
//     CTAs.  Warp 0 streams a CTA's blocks through a ring of bulk copies
//     (evict-first); warp 1 brings the h tiles list B needs into a small
//     ring as they are published; 16 consumer warps dequantise each block
//     in registers (a thread: 16 columns of rows r and r+128 -- gate and up,
//     or two down tiles -- so one x load feeds two rows) and accumulate it
//     against x (list A) or h (list B) for every token of the group.
//  5. reduce: a CTA's run of K blocks inside one segment (group x row tile)
//     is a piece.  The CTA holding the segment's first block reaches it last
//     (it ends that CTA's range) and finalises it: it keeps its own piece in
//     shared memory, waits until the other CTAs' pieces are stored (they
//     store and count without waiting) and sums them in CTA order
//     (deterministic), then
//       list A: h = act(gs*g) * (us*u) for the tile's 128 rows
//               (engines/olmoe.c:391-393, engines/qwen.c:484-485) and a
//               release flag for that tile;
//       list B: y = sum * ds (matmul_q: acc * scale); when all of a token's
//               k (+ shared) down segments of a row-tile pair are done, that
//               CTA combines them in the reference's order (the select
//               warp's; slot positions map it onto the plan's):
//               out = [sigmoid gate * shared] + sum_kk w_kk * y_kk
//               (engines/olmoe.c:394-397, engines/qwen.c:486-492).
//     A down block needs only the h tile of its 64 columns; down weights do
//     not depend on h, so they are already in flight while a CTA waits.
//
// Every cross-CTA wait is on a flag or count with a time limit (about a
// second); a lost wait reports OMC_DEVERR_TIMEOUT and the kernel runs on
// instead of hanging.  Counters reset themselves when their last user is
// done and flags carry a per-launch tag kept in device memory, so the launch
// can be replayed from a CUDA graph.  All CTAs are co-resident (cooperative
// launch).
#include "omc_bounds.cuh"
#include "omc_select.cuh"
#include "omc_rms.cuh"

namespace {

constexpr int DC_CW = 16;                       // consumer warps
constexpr int DC_MT = 32 * (2 + DC_CW);         // warp 0: weight producer, warp 1: h tiles, consumers
constexpr int DC_SELW = 2 + DC_CW;              // the select warp: exact chains and selection
constexpr int DC_THREADS = DC_MT + 32;
constexpr int DC_CT = 32 * DC_CW;               // consumer threads
constexpr int DC_BW = 16;                       // warps that compute the logit intervals
constexpr int DC_ROWS = 2 * OMC_TM;             // rows per block
constexpr int DC_BLK = 2 * OMC_BLK_BYTES;       // one K block of a tile pair: 256 rows x 64 int8
constexpr int DC_NCH = 4;                       // 16-column chunks of a block
constexpr int DC_TMAX = 8;                      // tokens
constexpr int DC_SLOTS_MAX = 64;                // T * k
constexpr int DC_GMAX = DC_SLOTS_MAX + 1;       // groups (routed + shared)
constexpr int DC_TILES_MAX = 64;                // gate/up row tiles of an expert (I <= 8192)
constexpr int DC_RCH = 4;                       // router staging chunks
constexpr int DC_MAXG = 256;                    // CTAs
constexpr int DC_NPMAX = 64;                    // pieces of one segment
constexpr int DC_HB = 4;                        // h tile ring

// State words (ctr[]).  Flags hold launch tags and are never reset, so they
// live at fixed places for every layer and T; the counters (zero between
// forwards) follow at offsets that depend on the geometry.
constexpr int CTR_EPOCH = 0, CTR_EXIT = 1, CTR_ROUTER = 2, CTR_RFAST = 3;
// forwards whose sets the intervals decided, and forwards that waited for the
// exact selection (never reset by the kernel; omc_decode_stats reads them)
constexpr int CTR_NEARLY = OMC_DEC_CTR_STATS, CTR_NFALL = OMC_DEC_CTR_STATS + 1;
static_assert(CTR_NFALL < 8, "fixed state words");
constexpr int CTR_HFLAG = 8;                                 // [DC_GMAX][DC_TILES_MAX] h tile published
constexpr int CTR_FIXED = CTR_HFLAG + DC_GMAX * DC_TILES_MAX;

struct DecArgs {
    omc_layer_dev L;
    const float *x;       // the input rows (GEMMA: the residual rows, normed here)
    int T;
    int32_t *topk_idx;
    float *topk_w, *logits;
    int ldl;
    float *hbuf;          // [slot][ldh] h of every slot (routed t*k+kk, shared T*k+t)
    int ldh;
    float *ybuf;          // [T][k+1][D] y of every slot
    float *out;           // [T][D]
    float *partA, *partB; // pieces: [cta][T][256]
    int *ctr;
    int offSA, offSB, offC;
    int *err;
    int ns;               // ring stages (the reserved router slots follow them)
    int ldx;              // smem stride of a token row of x (floats)
    int rr, nrc;          // router rows per router CTA, router CTAs
    int rres;             // bytes reserved after the ring for the router rows (+ Gemma's router
                          // input); 0: they are staged in the ring and the sets wait for the
                          // exact selection (the ring is free only after it)
    float2 *rbnd;         // [T][E] interval of each routed logit (bias included)
    int bnw;              // warps per interval team
    int early;            // 1: stream as soon as the intervals decide every token's set
};

__device__ __forceinline__ int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(int *p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_add(int *p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Release/acquire fence at GPU scope.  After a block (or named) barrier it
// also releases what the other threads wrote before the barrier (the
// pattern CUTLASS's inter-CTA barrier uses); it is weaker, and cheaper, than
// the sequentially consistent fence of __threadfence().
__device__ __forceinline__ void fence_acqrel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void cons_bar() { asm volatile("bar.sync 1, %0;" ::"n"(DC_CT) : "memory"); }
// every warp but the select warp
__device__ __forceinline__ void main_bar() { asm volatile("bar.sync 2, %0;" ::"n"(DC_MT) : "memory"); }

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}

// Bounded wait for *p == want (acquire).  False on timeout, or at once when
// an error is already reported (the forward is lost either way).
__device__ bool wait_value(const int *p, int want, int *err, int detail) {
    if (ld_acquire(p) == want) return true;
    OmcDeadline dl;
    dl.start();
    for (;;) {
        __nanosleep(64);
        if (ld_acquire(p) == want) return true;
        if (*(volatile int *)err != 0) return false;
        if (dl.over()) {
            omc_dev_error(err, OMC_DEVERR_TIMEOUT, OMC_SITE_DECODE, detail);
            return false;
        }
    }
}

// Bounded mbarrier wait that lets the thread sleep in the hardware until the
// phase flips: waiting warps take no issue slots from working ones.
__device__ __forceinline__ void mbar_wait_s(uint64_t *bar, uint32_t parity, int *err) {
    if (mbar_try_wait(bar, parity)) return;
    OmcDeadline dl;
    dl.start();
    while (!mbar_try_wait_sleep(bar, parity, 256u)) {   // short hint: wake-up latency stays small
        if (dl.over()) {
            omc_dev_error(err, OMC_DEVERR_TIMEOUT, OMC_SITE_DECODE, (int)parity);
            return;
        }
    }
}

// Bounded wait for a shared-memory flag another warp of the CTA sets.
__device__ bool wait_smem_flag(volatile int *f, int *err, int detail) {
    if (*f) return true;
    OmcDeadline dl;
    dl.start();
    for (;;) {
        __nanosleep(64);
        if (*f) return true;
        if (*(volatile int *)err != 0) return false;
        if (dl.over()) {
            omc_dev_error(err, OMC_DEVERR_TIMEOUT, OMC_SITE_DECODE, detail);
            return false;
        }
    }
}

// The interval that holds the reference's chain acc = RN(acc + p_j), j = 0..D-1
// (p_j = RN(x_j * w_j), the products the chain adds), from one pass of
// double sums over the same products:
//   c  ~ S_D, the exact sum of the p_j;   B ~ sum_j |S_j| (prefix sums);
//   P >= sum_j |p_j| (float, rounded up).
// Each chain add rounds with |err_j| <= u |acc_j| (u = 2^-24), so the chain
// is within u * sum_j |acc_j| <= u B' / (1 - D u) of S_D, where B' bounds
// sum_j |S_j|; every double partial sum here is within (D + 64) 2^-52 P of
// its exact value, which bounds both |c - S_D| and B' - B / D.  A subnormal
// partial sum adds at most 2^-150 per add.  The router's int8 row scale and
// the bias then widen the ends with directed rounding.
__device__ float2 dec_interval(double c, double B, float P, int D, const float *scale, const float *bias) {
    const double u = 5.9604644775390625e-08, Dd = (double)D;
    const double em = __dmul_ru(__dmul_ru(Dd + 64.0, 2.220446049250313e-16), (double)P);
    const double Bp = __dadd_ru(B, __dmul_ru(Dd, em));
    double beta = __dmul_ru(__dmul_ru(u, Bp), __dadd_ru(1.0, __dmul_ru(2.0 * Dd, u)));
    beta = __dadd_ru(__dadd_ru(beta, em), __dmul_ru(Dd, 7.006492321624085e-46));
    float lo = __double2float_rd(__dsub_rd(c, beta)), hi = __double2float_ru(__dadd_ru(c, beta));
    if (scale) {
        const float s = *scale, l = lo;
        lo = s >= 0.f ? __fmul_rd(lo, s) : __fmul_rd(hi, s);
        hi = s >= 0.f ? __fmul_ru(hi, s) : __fmul_ru(l, s);
    }
    if (bias) {
        lo = __fadd_rd(lo, *bias);
        hi = __fadd_ru(hi, *bias);
    }
    return make_float2(lo, hi);
}

// pointer words of the expert table in shared memory (5 per expert, even count)
__host__ __device__ constexpr int dc_ptab_words(int E) { return (5 * (E + 1) + 1) & ~1; }

// A ring position: slot and the parity of its current use.
struct RingPos {
    int slot, phase;
    __device__ void next(int n) {
        if (++slot == n) {
            slot = 0;
            phase ^= 1;
        }
    }
};

// 4 int8 (already xor 0x80808080) -> 4 exact floats as two pairs:
// (2^23 + 128 + q) as a float minus the bias, one packed add per pair.
__device__ __forceinline__ void u8x4_f2(uint32_t u, float2 &lo, float2 &hi) {
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);
    lo = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)),
                                __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441))),
                    bias);
    hi = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)),
                                __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443))),
                    bias);
}

__device__ __forceinline__ float swiglu(int act, float g, float u) {
    if (act == OMC_ACT_GELU_TANH) return __fmul_rn(omc_gelu_tanh(g), u);   // engines/gemma.c:671
    const float e = omc_expf_glibc(-g);
    if (act == OMC_ACT_SILU_SIG) return __fmul_rn(__fmul_rn(g, __fdiv_rn(1.f, __fadd_rn(1.f, e))), u);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, e)), u);
}

// first item of CTA c in an even split of n items over G CTAs, and the CTA
// whose range holds item b (ranges may be empty when n < G)
__device__ __forceinline__ long long split_start(int c, long long n, int G) { return (long long)c * n / G; }
__device__ __forceinline__ int split_owner(long long b, long long n, int G) {
    return (int)(((b + 1) * G - 1) / n);
}

// The work lists, identical in every CTA once the routing is known.
struct Lists {
    int ngr;                       // routed groups (the shared group, if any, is group ngr)
    int ntr, nts, nkbA;            // gate/up row tiles (routed, shared), K blocks
    int npair, nkbr, nkbs;         // down row-tile pairs, K blocks (routed, shared)
    long long NA, NBr, NB;
    __device__ int segA(long long b) const { return (int)(b / nkbA); }
    __device__ long long segA_start(int S) const { return (long long)S * nkbA; }
    __device__ void decA(int S, int &g, int &mt) const {
        if (S < ngr * ntr) {
            g = S / ntr;
            mt = S - g * ntr;
        } else {
            g = ngr;
            mt = S - ngr * ntr;
        }
    }
    __device__ int segB(long long b) const {
        if (b < NBr) return (int)(b / nkbr);
        return ngr * npair + (int)((b - NBr) / nkbs);
    }
    __device__ long long segB_start(int S) const {
        return S < ngr * npair ? (long long)S * nkbr : NBr + (long long)(S - ngr * npair) * nkbs;
    }
    __device__ int segB_nkb(int S) const { return S < ngr * npair ? nkbr : nkbs; }
    __device__ void decB(int S, int &g, int &p) const {
        if (S < ngr * npair) {
            g = S / npair;
            p = S - g * npair;
        } else {
            g = ngr;
            p = S - ngr * npair;
        }
    }
};

// Walks the blocks [b0, b1) of list B in order, calling f(S, g, p, kb, nkb)
// for each; the producer, the h-tile warp and the consumers share this order.
template <class F>
__device__ __forceinline__ void walk_B(const Lists &W, long long b0, long long b1, F f) {
    if (b0 >= b1) return;
    int S = W.segB(b0), kb = (int)(b0 - W.segB_start(S));
    for (long long b = b0; b < b1; ++S, kb = 0) {
        int g, p;
        W.decB(S, g, p);
        const int nkb = W.segB_nkb(S);
        for (; kb < nkb && b < b1; ++kb, ++b) f(S, g, p, kb, nkb);
    }
}

template <int NV, int TM>
__global__ void __launch_bounds__(DC_THREADS, 1) decode_moe_kernel(const DecArgs a) {
    extern __shared__ __align__(1024) uint8_t dsm[];
    const omc_layer_dev &L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, K = L.k, E = L.E, D = L.D, D_pad = L.D_pad;
    const int G = gridDim.x, c = blockIdx.x;
    const int nslots = T * K, hsh = L.has_shared ? 1 : 0;
    // dynamic shared memory: ring | x [T][ldx] | h tiles [HB][T][128] |
    // chunk partials [T][4][256] | own piece [T][256] | expert table | barriers
    uint8_t *ring = dsm;
    float *xs = reinterpret_cast<float *>(dsm + (size_t)a.ns * DC_BLK + a.rres);
    float *hsm = xs + (size_t)T * a.ldx;
    float *xch = hsm + (size_t)DC_HB * T * OMC_TM;
    float *xown = xch + (size_t)T * DC_NCH * DC_ROWS;
    float *selscr = xown + (size_t)T * DC_ROWS;                                // the select warp's scratch
    // every expert's matrices and scales (g, d, gs, us, ds), copied while the router runs
    const void **ptab = reinterpret_cast<const void **>(selscr + (size_t)NV * 32);
    uint64_t *full = reinterpret_cast<uint64_t *>(ptab + dc_ptab_words(E));
    uint64_t *empty = full + a.ns, *rbar = empty + a.ns, *hfull = rbar + DC_RCH, *hempty = hfull + DC_HB;
    // the routing and the plan
    __shared__ int s_tidx[DC_SLOTS_MAX];
    __shared__ float s_tw[DC_SLOTS_MAX], s_sg[DC_TMAX];
    __shared__ int s_ge[DC_GMAX], s_gn[DC_GMAX], s_c0[DC_GMAX];
    __shared__ int s_gslot[DC_GMAX * DC_TMAX], s_gtok[DC_GMAX * DC_TMAX];
    __shared__ uint32_t s_bits[OMC_MAX_E / 32];
    __shared__ int s_wbase[32];
    __shared__ const int8_t *s_gp[DC_GMAX], *s_dp[DC_GMAX];   // group's gate/up and down matrices
    __shared__ int s_pcta[DC_NPMAX];                            // other CTAs holding pieces of a segment
    __shared__ int s_epoch, s_abort, s_ngr, s_np;
    __shared__ float s_r[DC_TMAX];                              // GEMMA: each token's rms factor
    __shared__ int s_comb[DC_TMAX];
    // the reference's selection (the select warp): indices, weights, shared
    // gates, and where each selected expert's y lies among the plan's slots
    __shared__ int s_xidx[DC_SLOTS_MAX], s_pos[DC_SLOTS_MAX];
    __shared__ float s_xw[DC_SLOTS_MAX], s_xsg[DC_TMAX];
    __shared__ int s_det[DC_TMAX], s_planned, s_seldone;
    __shared__ double s_bt[DC_BW], s_bb[DC_BW];                 // interval teams: warp totals, sum |S_j|
    __shared__ float s_bp[DC_BW];                               // and sum |p_j|
    int *ctr = a.ctr;
    const bool router = c < a.nrc;

    if (tid == 0) {
        s_epoch = *(volatile int *)(ctr + CTR_EPOCH);
        s_abort = 0;
        s_planned = 0;
        s_seldone = 0;
        for (int i = 0; i < a.ns; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], DC_CW);
        }
        for (int i = 0; i < DC_RCH; ++i) mbar_init(&rbar[i], 1);
        for (int i = 0; i < DC_HB; ++i) {
            mbar_init(&hfull[i], 1);
            mbar_init(&hempty[i], DC_CW);
        }
        fence_barrier_init();
    }
    // ---- 1. x (every CTA) and the router rows (router CTAs) ---------------
    // A router CTA stages its rows (and, for Gemma, the token rows it scales
    // into the router's input) in the reserved bytes after the ring: its
    // chains run on there while the ring streams the experts' weights.
    // Without the reserve they go into the ring, which then streams only
    // after every chain is done (the sets wait for the exact selection).
    const int rr = a.rr, r0 = c * rr, ldw = a.ldx, nrows = E + hsh;
    const bool gemma = L.family == OMC_FAMILY_GEMMA;
    float *rws = reinterpret_cast<float *>(ring + (a.rres ? (size_t)a.ns * DC_BLK : 0));   // [rr][ldw] router rows
    // Gemma: the router's input is (x*r)*router scale, the experts' (x*r)*
    // pre_feedforward_layernorm_2.  With the reserve the router's has its own
    // copy; without it the router CTAs scale xs for the router and rebuild the
    // experts' input once every chain is done (before the ring streams).
    const bool gx = gemma && a.rres != 0, gx_late = gemma && !a.rres && router;
    float *rxs = gx ? rws + (size_t)rr * ldw : xs;                             // [T][ldw] the router's input
    if (router && tid == 0) {   // (the barriers above are this thread's own: no sync needed)
        const int cw = D / DC_RCH, nr = min(rr, nrows - r0);
        for (int ch = 0; ch < DC_RCH; ++ch) {
            mbar_arrive_expect_tx(&rbar[ch], (uint32_t)(((gx ? T : 0) + nr) * cw * 4));
            if (gx)
                for (int t = 0; t < T; ++t)
                    bulk_g2s(rxs + (size_t)t * ldw + ch * cw, a.x + (size_t)t * D + ch * cw, cw * 4, &rbar[ch]);
            for (int r = 0; r < nr; ++r) {
                const int gr = r0 + r;
                const float *src = gr < E ? L.router + (size_t)gr * D : L.sh_gate;
                bulk_g2s(rws + (size_t)r * ldw + ch * cw, src + ch * cw, cw * 4, &rbar[ch]);
            }
        }
    }
    for (int i = tid; i < T * (D / 4); i += DC_THREADS) {
        const int t = i / (D / 4), col = (i - t * (D / 4)) * 4;
        cp_async16(xs + (size_t)t * a.ldx + col, a.x + (size_t)t * D + col);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int e = tid; e <= E; e += DC_THREADS) {
        const omc_expert_ptrs *P = L.experts + e;
        ptab[5 * e] = P->g;
        ptab[5 * e + 1] = P->d;
        ptab[5 * e + 2] = P->gs;
        ptab[5 * e + 3] = P->us;
        ptab[5 * e + 4] = P->ds;
    }
    __syncthreads();   // barriers initialised; s_epoch read
    const int tag = s_epoch + 1;
    for (int i = tid; i < T * (D_pad - D); i += DC_THREADS) {
        const int t = i / (D_pad - D), col = D + (i - t * (D_pad - D));
        xs[(size_t)t * a.ldx + col] = 0.f;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();   // every thread's copies of x have landed
    if (gemma) {
        // x is the residual row.  Each CTA takes every token's rms factor
        // from its copy (warp t, token t; omc_rms.cuh); the router's input is
        // (x*r)*router_scale*rroot (router CTAs), the experts' input
        // (x*r)*pre_feedforward_layernorm_2
        if (warp < T) {
            const float r = omc_gemma_rms_factor(xs + (size_t)warp * a.ldx, D, L.eps);
            if (lane == 0) s_r[warp] = r;
        }
        __syncthreads();
        if (gx && router) {
            for (int ch = 0; ch < DC_RCH; ++ch) mbar_wait(&rbar[ch], 0, a.err, OMC_SITE_DECODE);
            for (int i = tid; i < T * D; i += DC_THREADS) {
                const int t = i / D, col = i - t * D;
                float *v = rxs + (size_t)t * ldw + col;
                *v = __fmul_rn(__fmul_rn(*v, s_r[t]), L.g_s2[col]);
            }
        }
        for (int i = tid; i < T * D; i += DC_THREADS) {
            const int t = i / D, col = i - t * D;
            float *v = xs + (size_t)t * a.ldx + col;
            *v = __fmul_rn(__fmul_rn(*v, s_r[t]), gx_late ? L.g_s2[col] : (L.g_en ? L.g_en[col] : 1.f));
        }
        __syncthreads();
    }

    if (warp == DC_SELW) {
        // ---- the select warp: this CTA's exact chains (the reference's
        // order, engines/olmoe.c:74-85, engines/qwen.c:116-121; about 5.5
        // cycles an element), then the reference's selection of every token
        // from the exact logits, while the other warps stream.  The combine
        // takes its weights, order and shared gates from here.
        if (router) {
            if (lane < T * rr) {
                const int t = lane / rr, r = lane - t * rr, gr = r0 + r;
                const float *xr = rxs + (size_t)t * ldw, *wr = rws + (size_t)r * ldw;
                const int cw = D / DC_RCH;
                float acc = 0.f;
                for (int ch = 0; ch < DC_RCH; ++ch) {
                    mbar_wait(&rbar[ch], 0, a.err, OMC_SITE_DECODE);
#pragma unroll 8
                    for (int col = ch * cw; col < (ch + 1) * cw; col += 4) {
                        const float4 xv = *reinterpret_cast<const float4 *>(xr + col);
                        const float4 wv = *reinterpret_cast<const float4 *>(wr + col);
                        acc = __fadd_rn(acc, __fmul_rn(xv.x, wv.x));
                        acc = __fadd_rn(acc, __fmul_rn(xv.y, wv.y));
                        acc = __fadd_rn(acc, __fmul_rn(xv.z, wv.z));
                        acc = __fadd_rn(acc, __fmul_rn(xv.w, wv.w));
                    }
                }
                if (gr < nrows)
                    a.logits[(size_t)t * a.ldl + gr] = (L.router_i8 && gr < E) ? __fmul_rn(acc, L.router_s[gr]) : acc;
            }
            __syncwarp();
            if (lane == 0) {
                fence_acqrel_gpu();
                red_release_add(ctr + CTR_ROUTER, 1);
            }
        }
        int ok = 1;
        if (lane == 0) ok = wait_value(ctr + CTR_ROUTER, a.nrc, a.err, -1);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok)
            for (int t = 0; t < T; ++t)
                select_token<NV>(a.logits, a.ldl, t, E, K, L.family, L.renorm, L.has_shared, L.g_pes, L.rbias, s_xidx,
                                 s_xw, s_xsg, a.err, selscr);
        // the plan's slots: the interval sets (experts in ascending id) or
        // these same indices; map each selected expert to its slot
        if (lane == 0) wait_smem_flag(&s_planned, a.err, -3);
        __syncwarp();
        __threadfence_block();
        const bool use = ok && !s_abort;
        for (int i = lane; i < nslots; i += 32) {
            const int t = i / K;
            int pos = i - t * K;
            if (use) {
                int f = -1;
                for (int j = 0; j < K; ++j)
                    if (s_tidx[t * K + j] == s_xidx[i]) f = j;
                if (f < 0) omc_dev_error(a.err, OMC_DEVERR_ROUTE, OMC_SITE_DECODE, i);
                else pos = f;
                if (c == 0) {
                    a.topk_idx[i] = s_xidx[i];
                    a.topk_w[i] = s_xw[i];
                }
            }
            s_pos[i] = pos;
        }
        __syncwarp();
        __threadfence_block();
        if (lane == 0) *(volatile int *)&s_seldone = 1;
    } else {
    if (router) {
        // ---- intervals of this CTA's routed logits: teams of a.bnw warps, one
        // (token, row) pair a team; a thread sums a contiguous run of the
        // products in double, the team scans the runs (prefix sums S_j)
        const int np = T * rr, nw = a.bnw, nteam = DC_BW / nw;
        const int team = warp < DC_BW ? warp / nw : -1, wq = warp - (team < 0 ? 0 : team) * nw;
        const int nq = 32 * nw, q = wq * 32 + lane;
        bool landed = false;
        for (int b0 = 0; b0 < np; b0 += nteam) {
            const int b = b0 + team;
            const bool act = team >= 0 && b < np;   // warp-uniform
            const int t = act ? b / rr : 0, r = act ? b - t * rr : 0, gr = r0 + r;
            const float *xv = rxs + (size_t)t * ldw, *wv = rws + (size_t)r * ldw;
            const int j0 = (int)((long long)q * D / nq), j1 = (int)((long long)(q + 1) * D / nq);
            if (act && !landed) {
                for (int ch = 0; ch < DC_RCH; ++ch) mbar_wait(&rbar[ch], 0, a.err, OMC_SITE_DECODE);
                landed = true;
            }
            double loc = 0.0;
            float pab = 0.f;
            if (act)
                for (int j = j0; j < j1; ++j) {
                    const float p = __fmul_rn(xv[j], wv[j]);
                    loc = __dadd_rn(loc, (double)p);
                    pab = __fadd_ru(pab, fabsf(p));
                }
            double inc = loc;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double v = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc = __dadd_rn(inc, v);
            }
            if (act && lane == 31) s_bt[warp] = inc;
            main_bar();
            double babs = 0.0;
            const double ex = __shfl_up_sync(0xffffffffu, inc, 1);
            if (act) {
                double sp = 0.0;
                for (int w2 = team * nw; w2 < warp; ++w2) sp = __dadd_rn(sp, s_bt[w2]);
                if (lane > 0) sp = __dadd_rn(sp, ex);
                for (int j = j0; j < j1; ++j) {
                    sp = __dadd_rn(sp, (double)__fmul_rn(xv[j], wv[j]));
                    babs = __dadd_ru(babs, fabs(sp));
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                babs = __dadd_ru(babs, __shfl_xor_sync(0xffffffffu, babs, o));
                pab = __fadd_ru(pab, __shfl_xor_sync(0xffffffffu, pab, o));
            }
            if (act && lane == 0) {
                s_bb[warp] = babs;
                s_bp[warp] = pab;
            }
            main_bar();
            if (act && wq == 0) {   // the team's first warp: the team's sums (lane w: warp w)
                const int w2 = team * nw + lane;
                double B = lane < nw ? s_bb[w2] : 0.0, cs = lane < nw ? s_bt[w2] : 0.0;
                float P = lane < nw ? s_bp[w2] : 0.f;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    B = __dadd_ru(B, __shfl_xor_sync(0xffffffffu, B, o));
                    P = __fadd_ru(P, __shfl_xor_sync(0xffffffffu, P, o));
                    cs = __dadd_rn(cs, __shfl_xor_sync(0xffffffffu, cs, o));
                }
                if (lane == 0 && gr < E)
                    a.rbnd[(size_t)t * E + gr] = dec_interval(cs, B, P, D, L.router_i8 ? L.router_s + gr : nullptr,
                                                              L.rbias ? L.rbias + gr : nullptr);
            }
            main_bar();   // the intervals are written before the count; s_bt, s_bb are the next round's
        }
        if (tid == 0) {
            fence_acqrel_gpu();
            red_release_add(ctr + CTR_RFAST, 1);
        }
    }

    // ---- 2. every token's top-k set from the intervals, in every CTA: with
    // exactly k candidates (omc_bounds.cuh) the set is the reference's, and
    // the weights and order can wait for the select warp.  Otherwise the
    // reference's selection from the exact logits, here, first.
    if (tid == 0 && !wait_value(ctr + CTR_RFAST, a.nrc, a.err, -1)) s_abort = 1;
    main_bar();
    if (!s_abort && warp < T) {
        float lo[NV], hi[NV];
        bool bad = false;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int e = lane + 32 * j;
            lo[j] = hi[j] = -INFINITY;
            if (e < E) {
                const float2 v = __ldcg(a.rbnd + (size_t)warp * E + e);
                lo[j] = v.x;
                hi[j] = v.y;
                bad |= !(fabsf(v.x) < 1e30f) || !(fabsf(v.y) < 1e30f);
            }
        }
        int nc = -1;
        if (!__any_sync(0xffffffffu, bad)) nc = omc_topk_candidates<NV>(lo, hi, E, K, K, s_tidx + warp * K);
        if (lane == 0) s_det[warp] = nc == K;
    }
    main_bar();
    bool early = a.early != 0 && a.rres != 0;
    for (int t = 0; t < T; ++t) early = early && s_det[t] != 0;
    if (c == 0 && tid == 0 && !s_abort) atomicAdd(ctr + (early ? CTR_NEARLY : CTR_NFALL), 1);
    if (!s_abort && !early) {
        if (tid == 0 && !wait_value(ctr + CTR_ROUTER, a.nrc, a.err, -1)) s_abort = 1;
        main_bar();
        if (gx_late) {   // every chain is done: the experts' input from the residual rows
            for (int i = tid; i < T * D; i += DC_MT) {
                const int t = i / D, col = i - t * D;
                xs[(size_t)t * a.ldx + col] =
                    __fmul_rn(__fmul_rn(__ldg(a.x + (size_t)t * D + col), s_r[t]), L.g_en ? L.g_en[col] : 1.f);
            }
            main_bar();
        }
        if (!s_abort && warp < T)
            select_token<NV>(a.logits, a.ldl, warp, E, K, L.family, L.renorm, L.has_shared, L.g_pes, L.rbias, s_tidx,
                             s_tw, s_sg, a.err, reinterpret_cast<float *>(ring) + warp * NV * 32);
        main_bar();
    }
    if (tid == 0) {
        __threadfence_block();
        *(volatile int *)&s_planned = 1;   // s_tidx is final (the select warp maps onto it)
    }

    // With one token and a decided set the groups are the set itself (the
    // candidates, ascending): the weight producer starts at once and warp 1
    // plans beside it for the other warps.
    const bool fast = early && T == 1 && !s_abort;

    // ---- 3. plan (one warp): groups in ascending expert id ---------------------
    if (warp == 1 && !s_abort) {
        const int nw = (E + 31) >> 5;
        for (int i = lane; i < nw; i += 32) s_bits[i] = 0u;
        for (int g = lane; g < DC_GMAX; g += 32) s_gn[g] = 0;
        __syncwarp();
        const int e0 = lane < nslots ? s_tidx[lane] : -1;
        const int e1 = lane + 32 < nslots ? s_tidx[lane + 32] : -1;
        const bool bad = (lane < nslots && (e0 < 0 || e0 >= E)) || (lane + 32 < nslots && (e1 < 0 || e1 >= E));
        if (__any_sync(0xffffffffu, bad)) {
            if (lane == 0) {
                s_abort = 1;
                omc_dev_error(a.err, OMC_DEVERR_ROUTE, OMC_SITE_DECODE, c);
            }
        } else {
            if (e0 >= 0) atomicOr(&s_bits[e0 >> 5], 1u << (e0 & 31));
            if (e1 >= 0) atomicOr(&s_bits[e1 >> 5], 1u << (e1 & 31));
            __syncwarp();
            const int pcnt = lane < nw ? __popc(s_bits[lane]) : 0;
            int incl = pcnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            s_wbase[lane] = incl - pcnt;
            const int ngr = __shfl_sync(0xffffffffu, incl, 31);
            __syncwarp();
            auto gid = [&](int e) { return s_wbase[e >> 5] + __popc(s_bits[e >> 5] & ((1u << (e & 31)) - 1u)); };
            // rank inside a group = earlier slots with the same expert
            const unsigned lt = (1u << lane) - 1u;
            const unsigned m0 = __match_any_sync(0xffffffffu, e0), m1 = __match_any_sync(0xffffffffu, e1);
            const int rk0 = __popc(m0 & lt), rk1 = __popc(m1 & lt);
            const int g0 = e0 >= 0 ? gid(e0) : 0, g1 = e1 >= 0 ? gid(e1) : 0;
            if (e1 >= 0) s_c0[g1] = 0;
            __syncwarp();
            if (e0 >= 0 && rk0 == 0) s_c0[g0] = __popc(m0);   // slots 0..31 of this expert
            __syncwarp();
            if (e0 >= 0) {
                s_gslot[g0 * DC_TMAX + rk0] = lane;
                s_gtok[g0 * DC_TMAX + rk0] = lane / K;
                s_ge[g0] = e0;
                atomicMax(&s_gn[g0], rk0 + 1);
            }
            if (e1 >= 0) {
                const int rk = s_c0[g1] + rk1;
                s_gslot[g1 * DC_TMAX + rk] = lane + 32;
                s_gtok[g1 * DC_TMAX + rk] = (lane + 32) / K;
                s_ge[g1] = e1;
                atomicMax(&s_gn[g1], rk + 1);
            }
            if (L.has_shared && lane < T) {
                s_gslot[ngr * DC_TMAX + lane] = nslots + lane;
                s_gtok[ngr * DC_TMAX + lane] = lane;
            }
            if (lane == 0) {
                s_ngr = ngr;
                if (L.has_shared) {
                    s_ge[ngr] = E;
                    s_gn[ngr] = T;
                }
            }
            __syncwarp();
            for (int g = lane; g < ngr + hsh; g += 32) {
                s_gp[g] = static_cast<const int8_t *>(ptab[5 * s_ge[g]]);
                s_dp[g] = static_cast<const int8_t *>(ptab[5 * s_ge[g] + 1]);
            }
        }
    }
    if (!fast) {
        fence_proxy_async_smem();   // select scratch (generic) before bulk copies into the ring
        main_bar();
    } else if (warp != 0) {
        // (the fast path wrote nothing generic to the ring: no proxy fence)
        asm volatile("bar.sync 3, %0;" ::"n"(DC_MT - 32) : "memory");   // the plan, for warps 1..17
    }

    Lists W;
    W.ngr = fast ? K : s_ngr;
    W.ntr = L.I_rows / OMC_TM;
    W.nts = L.has_shared ? L.Is_rows / OMC_TM : 0;
    W.nkbA = D_pad / OMC_KB;
    W.npair = (L.D_rows / OMC_TM + 1) / 2;
    W.nkbr = L.I_pad / OMC_KB;
    W.nkbs = L.has_shared ? L.Is_pad / OMC_KB : 1;
    W.NA = ((long long)W.ngr * W.ntr + W.nts) * W.nkbA;
    W.NBr = (long long)W.ngr * W.npair * W.nkbr;
    W.NB = W.NBr + (long long)hsh * W.npair * W.nkbs;
    const long long a0b = split_start(c, W.NA, G), a1b = split_start(c + 1, W.NA, G);
    const long long b0b = split_start(c, W.NB, G), b1b = split_start(c + 1, W.NB, G);
    const int ldh = a.ldh;

    if (s_abort) {
        // nothing streamed
    } else if (warp == 0) {
        // ---- 4a. weight producer: one bulk copy per block, in list order --
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            RingPos rp{0, 0};
            int seq = 0;
            auto produce = [&](const int8_t *src) {
                if (seq >= a.ns) mbar_wait_s(&empty[rp.slot], rp.phase ^ 1, a.err);
                mbar_arrive_expect_tx(&full[rp.slot], DC_BLK);
                bulk_g2s_hint(ring + (size_t)rp.slot * DC_BLK, src, DC_BLK, &full[rp.slot], pol);
                rp.next(a.ns);
                ++seq;
            };
            // group g's matrices: the plan's, or (fast path) group g < K is the
            // set's g-th expert and group K the shared expert
            auto mat = [&](int g, int which) -> const int8_t * {
                if (!fast) return which ? s_dp[g] : s_gp[g];
                return static_cast<const int8_t *>(ptab[5 * (g < K ? s_tidx[g] : E) + which]);
            };
            if (a0b < a1b) {
                int S = W.segA(a0b), kb = (int)(a0b - W.segA_start(S));
                for (long long b = a0b; b < a1b; ++S, kb = 0) {
                    int g, mt;
                    W.decA(S, g, mt);
                    const int8_t *base = mat(g, 0) + (size_t)mt * W.nkbA * DC_BLK;
                    for (; kb < W.nkbA && b < a1b; ++kb, ++b) produce(base + (size_t)kb * DC_BLK);
                }
            }
            walk_B(W, b0b, b1b, [&](int, int g, int p, int kb, int nkb) {
                produce(mat(g, 1) + ((size_t)p * nkb + kb) * DC_BLK);
            });
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- 4b. h tiles of list B, in the consumers' order ---------------
        if (lane == 0) {
            RingPos hp{0, 0};
            int hseq = 0;
            bool first = true;
            walk_B(W, b0b, b1b, [&](int, int g, int, int kb, int) {
                if (!first && (kb & 1)) return;   // the second block of a tile
                first = false;
                const int mt = kb >> 1, n = s_gn[g];
                if (hseq >= DC_HB) mbar_wait_s(&hempty[hp.slot], hp.phase ^ 1, a.err);
                wait_value(ctr + CTR_HFLAG + g * DC_TILES_MAX + mt, tag, a.err, g);
                mbar_arrive_expect_tx(&hfull[hp.slot], (uint32_t)(n * OMC_TM * 4));
                float *dst = hsm + (size_t)hp.slot * T * OMC_TM;
                for (int j = 0; j < n; ++j)
                    bulk_g2s(dst + j * OMC_TM, a.hbuf + (size_t)s_gslot[g * DC_TMAX + j] * ldh + mt * OMC_TM,
                             OMC_TM * 4, &hfull[hp.slot]);
                hp.next(DC_HB);
                ++hseq;
            });
        }
        __syncwarp();
    } else {
        // ---- 4c. consumers: thread (chunk, r) owns 16 columns of rows r and
        // r + 128 of every block; the chunk is warp-uniform (broadcast loads)
        const int ci = tid - 64, cw = ci >> 5, ch = cw >> 2, r = (cw & 3) * 32 + lane;
        float2 acc0[TM], acc1[TM];
        RingPos rp{0, 0}, hp{0, 0};
        bool sel_seen = false;   // the select warp's results are in shared memory

        // rows r and r + 128 of chunk ch of the next block, dequantised; then
        // the slot is released (every loaded word is used before the arrive)
        auto take = [&](float2 (&w0)[8], float2 (&w1)[8]) {
            mbar_wait_s(&full[rp.slot], rp.phase, a.err);
            const uint8_t *p = ring + (size_t)rp.slot * DC_BLK + ch * 2048 + r * 16;
            const uint4 q0 = *reinterpret_cast<const uint4 *>(p);
            const uint4 q1 = *reinterpret_cast<const uint4 *>(p + OMC_BLK_BYTES);
            const uint32_t u0x = q0.x ^ 0x80808080u, u0y = q0.y ^ 0x80808080u, u0z = q0.z ^ 0x80808080u,
                           u0w = q0.w ^ 0x80808080u, u1x = q1.x ^ 0x80808080u, u1y = q1.y ^ 0x80808080u,
                           u1z = q1.z ^ 0x80808080u, u1w = q1.w ^ 0x80808080u;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[rp.slot]);
            rp.next(a.ns);
            u8x4_f2(u0x, w0[0], w0[1]);
            u8x4_f2(u0y, w0[2], w0[3]);
            u8x4_f2(u0z, w0[4], w0[5]);
            u8x4_f2(u0w, w0[6], w0[7]);
            u8x4_f2(u1x, w1[0], w1[1]);
            u8x4_f2(u1y, w1[2], w1[3]);
            u8x4_f2(u1z, w1[4], w1[5]);
            u8x4_f2(u1w, w1[6], w1[7]);
        };
        auto zero = [&]() {
#pragma unroll
            for (int j = 0; j < TM; ++j) acc0[j] = acc1[j] = make_float2(0.f, 0.f);
        };
        // acc[j] += w . operand row j (16 floats at base + roff[j]): rows r, r+128
        auto dot = [&](const float2 (&w0)[8], const float2 (&w1)[8], const float *base, const int (&roff)[TM],
                       int n) {
#pragma unroll
            for (int j = 0; j < TM; ++j) {
                if (j < n) {
                    const float4 *o = reinterpret_cast<const float4 *>(base + roff[j]);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 v = o[q];
                        const float2 xa = make_float2(v.x, v.y), xb = make_float2(v.z, v.w);
                        acc0[j] = __ffma2_rn(w0[2 * q], xa, acc0[j]);
                        acc1[j] = __ffma2_rn(w1[2 * q], xa, acc1[j]);
                        acc0[j] = __ffma2_rn(w0[2 * q + 1], xb, acc0[j]);
                        acc1[j] = __ffma2_rn(w1[2 * q + 1], xb, acc1[j]);
                    }
                }
            }
        };
        // The piece of segment [s0, s1) of a list of N blocks is done: its
        // row sums (chunks added in order).  Not the segment's first-block
        // owner: store it, count it, go on (false).  The owner: keep it in
        // shared memory, wait for the other pieces, list their CTAs in s_pcta
        // (true, in every consumer thread).
        auto piece = [&](float *part, int *cnt, long long s0, long long s1, long long N, int n) -> bool {
#pragma unroll
            for (int j = 0; j < TM; ++j)
                if (j < n) {
                    xch[(j * DC_NCH + ch) * DC_ROWS + r] = __fadd_rn(acc0[j].x, acc0[j].y);
                    xch[(j * DC_NCH + ch) * DC_ROWS + OMC_TM + r] = __fadd_rn(acc1[j].x, acc1[j].y);
                }
            cons_bar();
            const bool owner = split_owner(s0, N, G) == c;
            float *dst = owner ? xown : part + (size_t)c * T * DC_ROWS;
            for (int q = ci; q < n * DC_ROWS; q += DC_CT) {
                const float *s = xch + (size_t)(q >> 8) * DC_NCH * DC_ROWS + (q & (DC_ROWS - 1));
                dst[q] = __fadd_rn(__fadd_rn(s[0], s[DC_ROWS]), __fadd_rn(s[2 * DC_ROWS], s[3 * DC_ROWS]));
            }
            cons_bar();
            if (!owner) {
                if (ci == 0) {
                    fence_acqrel_gpu();
                    red_release_add(cnt, 1);
                }
                return false;
            }
            if (ci == 0) {
                int np = 0;
                for (long long b = split_start(c + 1, N, G); b < s1 && np < DC_NPMAX;) {
                    const int cc = split_owner(b, N, G);
                    s_pcta[np++] = cc;
                    b = split_start(cc + 1, N, G);
                }
                s_np = np;
                if (np > 0) {
                    wait_value(cnt, np, a.err, -2);
                    *cnt = 0;
                    fence_acqrel_gpu();
                }
            }
            cons_bar();
            return true;
        };
        // a row of the segment: own piece + the others', CTA order
        auto gather = [&](const float *part, int j, int rw) {
            float v = xown[j * DC_ROWS + rw];
            const int np = s_np;
            for (int k = 0; k < np; ++k) v = __fadd_rn(v, __ldcg(part + ((size_t)s_pcta[k] * T + j) * DC_ROWS + rw));
            return v;
        };

        // list A: gate/up, x rows of the group's tokens
        if (a0b < a1b) {
            int S = W.segA(a0b), kb = (int)(a0b - W.segA_start(S));
            for (long long b = a0b; b < a1b; ++S, kb = 0) {
                int g, mt;
                W.decA(S, g, mt);
                const int n = s_gn[g];
                int roff[TM];
#pragma unroll
                for (int j = 0; j < TM; ++j) roff[j] = j < n ? s_gtok[g * DC_TMAX + j] * a.ldx : 0;
                zero();
                for (; kb < W.nkbA && b < a1b; ++kb, ++b) {
                    float2 w0[8], w1[8];
                    take(w0, w1);
                    dot(w0, w1, xs + kb * OMC_KB + ch * 16, roff, n);
                }
                const long long s0 = W.segA_start(S);
                if (!piece(a.partA, ctr + a.offSA + S, s0, s0 + W.nkbA, W.NA, n)) continue;
                // ---- the tile's h: rows (member 0: gate, member 1: up) of 128
                const int e = s_ge[g];
                const float *gs = static_cast<const float *>(ptab[5 * e + 2]);
                const float *us = static_cast<const float *>(ptab[5 * e + 3]);
                const int Iw = e == E ? L.Is : L.I;
                for (int q = ci; q < n * OMC_TM; q += DC_CT) {
                    const int j = q >> 7, rt = q & (OMC_TM - 1), hrow = mt * OMC_TM + rt;
                    const float gsum = gather(a.partA, j, rt), usum = gather(a.partA, j, OMC_TM + rt);
                    a.hbuf[(size_t)s_gslot[g * DC_TMAX + j] * ldh + hrow] =
                        hrow < Iw ? swiglu(L.act, __fmul_rn(gsum, gs[hrow]), __fmul_rn(usum, us[hrow])) : 0.f;
                }
                cons_bar();
                if (ci == 0) {
                    fence_acqrel_gpu();
                    st_release(ctr + CTR_HFLAG + g * DC_TILES_MAX + mt, tag);
                }
            }
        }

        // list B: down + combine; a block reads the h tile of its 64 columns
        if (b0b < b1b) {
            int S = W.segB(b0b), kb = (int)(b0b - W.segB_start(S));
            bool first = true;
            for (long long b = b0b; b < b1b; ++S, kb = 0) {
                int g, p;
                W.decB(S, g, p);
                const int n = s_gn[g], nkb = W.segB_nkb(S);
                int roff[TM];
#pragma unroll
                for (int j = 0; j < TM; ++j) roff[j] = j * OMC_TM;
                zero();
                for (; kb < nkb && b < b1b; ++kb, ++b) {
                    if (first || !(kb & 1)) {
                        // next h tile (same order as warp 1 brings them)
                        if (!first) {
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&hempty[hp.slot]);
                            hp.next(DC_HB);
                        }
                        first = false;
                        mbar_wait_s(&hfull[hp.slot], hp.phase, a.err);
                    }
                    float2 w0[8], w1[8];
                    take(w0, w1);
                    dot(w0, w1, hsm + (size_t)hp.slot * T * OMC_TM + (kb & 1) * OMC_KB + ch * 16, roff, n);
                }
                const long long s0 = W.segB_start(S);
                if (!piece(a.partB, ctr + a.offSB + S, s0, s0 + nkb, W.NB, n)) continue;
                // ---- y = sum * ds for the group's tokens, rows p*256 ..
                const float *ds = static_cast<const float *>(ptab[5 * s_ge[g] + 4]);
                for (int q = ci; q < n * DC_ROWS; q += DC_CT) {
                    const int j = q >> 8, rw = q & (DC_ROWS - 1), d = p * DC_ROWS + rw;
                    const float ysum = gather(a.partB, j, rw);
                    const int sl = s_gslot[g * DC_TMAX + j];
                    const int t = sl < nslots ? sl / K : sl - nslots, kk = sl < nslots ? sl - t * K : K;
                    if (d < D) a.ybuf[((size_t)t * (K + 1) + kk) * D + d] = __fmul_rn(ysum, ds[d]);
                }
                cons_bar();
                if (ci == 0) {
                    fence_acqrel_gpu();
                    const int nsl = K + hsh;
                    bool any = false;
                    for (int j = 0; j < n; ++j) {
                        int *cc = ctr + a.offC + s_gtok[g * DC_TMAX + j] * W.npair + p;
                        const int old = atomicAdd(cc, 1);
                        s_comb[j] = old + 1 == nsl;
                        any |= s_comb[j] != 0;
                        if (s_comb[j]) *cc = 0;
                    }
                    fence_acqrel_gpu();
                    if (any && !sel_seen) {
                        wait_smem_flag(&s_seldone, a.err, -4);
                        __threadfence_block();
                        sel_seen = true;
                    }
                }
                cons_bar();
                // tokens whose every y of these rows is written: combine in the
                // reference's order (the select warp's order and weights; the
                // y of selected expert kk is at the plan's slot s_pos)
                for (int q = ci; q < n * DC_ROWS; q += DC_CT) {
                    const int j = q >> 8, rw = q & (DC_ROWS - 1), d = p * DC_ROWS + rw;
                    if (!s_comb[j] || d >= D) continue;
                    const int t = s_gtok[g * DC_TMAX + j];
                    const float *yt = a.ybuf + (size_t)t * (K + 1) * D + d;
                    float o = 0.f;
                    if (L.has_shared) o = __fmul_rn(__ldcg(yt + (size_t)K * D), s_xsg[t]);
                    for (int kk = 0; kk < K; ++kk)
                        o = __fadd_rn(o, __fmul_rn(s_xw[t * K + kk], __ldcg(yt + (size_t)s_pos[t * K + kk] * D)));
                    a.out[(size_t)t * D + d] = o;
                }
            }
        }
    }
    }   // the main warps

    // ---- exit: the last CTA resets the router counts, advances the tag ----
    __syncthreads();
    if (tid == 0) {
        fence_acqrel_gpu();
        if (atomicAdd(ctr + CTR_EXIT, 1) == G - 1) {
            atomicExch(ctr + CTR_EXIT, 0);
            atomicExch(ctr + CTR_ROUTER, 0);
            atomicExch(ctr + CTR_RFAST, 0);
            fence_acqrel_gpu();
            atomicExch(ctr + CTR_EPOCH, tag);
        }
    }
}

struct DecGeom {
    int G, ns, rres, ldx, rr, nrc, bnw;
    int offSA, offSB, offC, nctr;
    size_t smem, partA_floats, partB_floats, rbnd_floats;
};

// ceil(E / 32) rounded up to a power of two: the select template's NV
static int dec_nv(int E) {
    int nv = 1;
    while (nv * 32 < E) nv *= 2;
    return nv;
}

constexpr size_t DC_SMEM_MAX = 216 * 1024;   // dynamic; the static plan needs the rest of 227 KiB
constexpr int DC_NS_EARLY = 4;                // ring stages left beside the reserved router rows

// Everything about a launch that follows from the shapes (not the routing):
// for T tokens, the worst case over routings.
static int dec_geometry(const omc_layer_dev *L, int T, int G, DecGeom *g) {
    if (T < 1 || T > DC_TMAX || T * L->k > DC_SLOTS_MAX || (L->D % (4 * DC_RCH)) || L->E > OMC_MAX_E ||
        G > DC_MAXG || L->I_rows / OMC_TM > DC_TILES_MAX || (L->has_shared && L->Is_rows / OMC_TM > DC_TILES_MAX) ||
        L->D_pad / OMC_KB > DC_NPMAX || L->I_pad / OMC_KB > DC_NPMAX || L->Is_pad / OMC_KB > DC_NPMAX)
        return OMC_EUNSUPPORTED;   // (a segment has at most DC_NPMAX pieces: one K block each)
    g->G = G;
    g->ldx = L->D_pad + 4;
    const int nrows = L->E + (L->has_shared ? 1 : 0);
    g->rr = (nrows + G - 1) / G;
    g->nrc = (nrows + g->rr - 1) / g->rr;
    if (T * g->rr > 32 || (L->D % 32)) return OMC_EUNSUPPORTED;   // chains: one select-warp lane each
    const size_t fixed = (size_t)T * g->ldx * 4 + (size_t)DC_HB * T * OMC_TM * 4 +
                         (size_t)T * DC_NCH * DC_ROWS * 4 + (size_t)T * DC_ROWS * 4 + (size_t)dec_nv(L->E) * 32 * 4 +
                         (size_t)dc_ptab_words(L->E) * 8 + (DC_RCH + 2 * DC_HB) * 8;
    // reserved bytes after the ring: the router rows and Gemma's router input
    // (1 KiB granules), when a ring of at least DC_NS_EARLY stages remains;
    // otherwise the rows go into the ring
    const size_t rows = (size_t)g->rr * g->ldx * 4;
    const size_t rbytes = (rows + (L->family == OMC_FAMILY_GEMMA ? (size_t)T * g->ldx * 4 : 0) + 1023) & ~(size_t)1023;
    if (fixed + 4 * ((size_t)DC_BLK + 16) > DC_SMEM_MAX) return OMC_EUNSUPPORTED;
    int ns;
    if (fixed + rbytes + DC_NS_EARLY * ((size_t)DC_BLK + 16) <= DC_SMEM_MAX) {
        g->rres = (int)rbytes;
        ns = (int)((DC_SMEM_MAX - fixed - rbytes) / (DC_BLK + 16));
    } else {   // the rows in the ring (Gemma's router input in xs)
        g->rres = 0;
        ns = (int)((DC_SMEM_MAX - fixed) / (DC_BLK + 16));
        if (rows > (size_t)ns * DC_BLK) return OMC_EUNSUPPORTED;
    }
    if (ns > 12) ns = 12;
    g->ns = ns;
    g->smem = (size_t)ns * DC_BLK + g->rres + fixed + (size_t)2 * ns * 8;
    // interval teams: DC_BW warps split over the T * rr (token, row) pairs
    int p2 = 1;
    while (p2 < T * g->rr) p2 *= 2;
    g->bnw = p2 >= DC_BW ? 1 : DC_BW / p2;
    // worst-case lists: every slot its own expert
    const int gmax = (T * L->k < L->E ? T * L->k : L->E);
    const int ntr = L->I_rows / OMC_TM, nts = L->has_shared ? L->Is_rows / OMC_TM : 0;
    const int npair = (L->D_rows / OMC_TM + 1) / 2;
    g->partA_floats = (size_t)G * T * DC_ROWS;
    g->partB_floats = (size_t)G * T * DC_ROWS;
    g->rbnd_floats = (size_t)2 * T * L->E;
    const int nsegA = gmax * ntr + nts, nsegB = (gmax + 1) * npair;
    g->offSA = CTR_FIXED;
    g->offSB = g->offSA + nsegA;
    g->offC = g->offSB + nsegB;
    g->nctr = g->offC + T * npair;
    return 0;
}

template <int NV, int TM>
static int launch_tm(const DecArgs &a, const DecGeom &g, cudaStream_t s) {
    static int attr_done = 0;
    if (!attr_done) {
        if (cudaFuncSetAttribute(decode_moe_kernel<NV, TM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)DC_SMEM_MAX) != cudaSuccess)
            return OMC_ECUDA;
        attr_done = 1;
    }
    void *args[] = {(void *)&a};
    if (cudaLaunchCooperativeKernel((const void *)decode_moe_kernel<NV, TM>, dim3(g.G), dim3(DC_THREADS), args, g.smem,
                                    s) != cudaSuccess)
        return OMC_ECUDA;
    return 0;
}

// the token count is a template bound (accumulators in registers)
template <int NV>
static int launch_nv(const DecArgs &a, const DecGeom &g, cudaStream_t s) {
    if (a.T <= 1) return launch_tm<NV, 1>(a, g, s);
    if (a.T <= 2) return launch_tm<NV, 2>(a, g, s);
    if (a.T <= 4) return launch_tm<NV, 4>(a, g, s);
    return launch_tm<NV, 8>(a, g, s);
}

}  // namespace

int omc_decode_early = 1;

// Test hook: 0 = the fused decode waits for the exact selection before it
// streams, whatever the intervals decide (the output is the same bit for bit).
extern "C" int omc_debug_decode_early(int on) {
    if (on != 0 && on != 1) return OMC_EINVAL;
    omc_decode_early = on;
    omc_graphs_invalidate();
    return 0;
}

// Sizes of the decode state (counters and pieces) that serve every T <= 8
// for this layer on a grid of G CTAs.
extern "C" int omc_decode_state_size(const omc_layer_dev *L, int G, size_t *ctr_ints, size_t *part_floats) {
    size_t ci = 0, pf = 0;
    int any = 0;
    for (int T = 1; T <= DC_TMAX; ++T) {
        DecGeom g;
        if (dec_geometry(L, T, G, &g)) continue;
        any = 1;
        if ((size_t)g.nctr > ci) ci = (size_t)g.nctr;
        if (g.partA_floats + g.partB_floats + g.rbnd_floats > pf) pf = g.partA_floats + g.partB_floats + g.rbnd_floats;
    }
    *ctr_ints = ci;
    *part_floats = pf;
    return any ? 0 : OMC_EUNSUPPORTED;
}

// 1 when the fused decode forward serves (L, T) with a state of the given sizes.
extern "C" int omc_decode_supported(const omc_layer_dev *L, int T, int G, size_t ctr_ints, size_t part_floats) {
    DecGeom g;
    if (dec_geometry(L, T, G, &g)) return 0;
    return (size_t)g.nctr <= ctr_ints && g.partA_floats + g.partB_floats + g.rbnd_floats <= part_floats;
}

extern "C" int omc_launch_decode(const omc_layer_dev *L, const float *x, const float *xr, int T, const omc_ws *ws,
                                 int G, int *ctr, float *part, int32_t *topk_idx, float *topk_w, float *out,
                                 cudaStream_t s) {
    if (T <= 0) return 0;
    if (xr && xr != x) return OMC_EINVAL;   // the router's input is the experts' (Gemma: both from x)
    DecGeom g;
    int rc;
    if ((rc = dec_geometry(L, T, G, &g))) return rc;
    DecArgs a;
    a.L = *L;
    a.x = x;
    a.T = T;
    a.topk_idx = topk_idx;
    a.topk_w = topk_w;
    a.logits = ws->logits;
    a.ldl = L->E + 1;
    a.hbuf = ws->hbuf;
    a.ldh = L->has_shared && L->Is_rows > L->I_rows ? L->Is_rows : L->I_rows;
    a.ybuf = ws->ypart;
    a.out = out;
    a.partA = part;
    a.partB = part + g.partA_floats;
    a.ctr = ctr;
    a.offSA = g.offSA;
    a.offSB = g.offSB;
    a.offC = g.offC;
    a.err = ws->err;
    a.ns = g.ns;
    a.rres = g.rres;
    a.ldx = g.ldx;
    a.rr = g.rr;
    a.nrc = g.nrc;
    a.rbnd = reinterpret_cast<float2 *>(part + g.partA_floats + g.partB_floats);
    a.bnw = g.bnw;
    a.early = omc_decode_early;
    const int nv = (L->E + 31) / 32;
    if (nv <= 1) rc = launch_nv<1>(a, g, s);
    else if (nv <= 2) rc = launch_nv<2>(a, g, s);
    else if (nv <= 4) rc = launch_nv<4>(a, g, s);
    else if (nv <= 8) rc = launch_nv<8>(a, g, s);
    else if (nv <= 16) rc = launch_nv<16>(a, g, s);
    else rc = launch_nv<32>(a, g, s);
    if (rc) return rc;
    omc_prof_mark(s, "decode_moe");
    omc_g_launches += 1;
    return 0;
}
