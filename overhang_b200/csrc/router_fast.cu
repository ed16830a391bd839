// router_fast.cu -- the bounded router: the reference's routing (indices bit for
// bit) without running the exact fp32 chain for every (token, expert).
//
// The exact router (router.cu) runs one sequential fp32 chain of D separately
// rounded products and sums per (token, expert) -- the reference's matmul /
// matmul_q order (engines/olmoe.c:74-85, engines/qwen.c:116-121).  That is
// T*E*D dependent CUDA-core steps: at T = 8192 on a 256-expert router it
// costs as much as the expert GEMMs.  Routing only needs the exact value of
// the experts that can be selected, so the bounded router
//
//   1. prep   splits each token row into f16 parts, x = x_hi + x_lo + r with
//             |r| <= 2^-22|x| + 2^-24, writes them as the rows of a GEMM
//             operand (x_hi rows, then x_lo rows), writes x_hi as the expert
//             GEMMs' f16 token operand, and ||x||_2, ||x||_1 rounded up;
//   2. GEMM   on the tensor cores (the library's grouped GEMM, f16 weight
//             tiles in tensor memory): the router rows as f16 (int8 routers
//             are exact in f16; an f32 router contributes its f16 rounding and
//             the f16 rounding of the remainder as two row sets), every
//             product part of every (token, row) summed in f32;
//   3. cand   per token: a_e = the sum of the parts, an interval that provably
//             holds the exact chain's logit, and the candidates -- every
//             expert whose interval reaches the k-th largest lower end (less
//             a margin that keeps the non-candidates' probabilities strictly
//             below the k-th).  Approximate logits go to the logits rows; the
//             candidates (and the shared-gate row) become chain jobs;
//   4. chain  the exact chain of every job, written over the approximation,
//             then a check per token: candidates whose exp values (computed as
//             the select kernel computes them) lie within 2^-21 of each other
//             but differ, or a k-th value below 2^-100, could order
//             differently under the approximate softmax sum, and the token is
//             retried with every row exact (5.);
//   5. chain  the retried tokens' remaining rows.
// The select kernel (router.cu) then routes from the logits rows as before.
// Non-candidates only enter through the softmax sum, so the routing weights
// agree with the reference's within a few ulps, and the indices exactly.
//
// The interval (per token t, expert e, in the chain's units before the row
// scale):  |a_e - c_e| <= coef * ||x_t||_2 ||w_e||_2 + 2^-23 (||w_e||_1 +
// split * ||x_t||_1),  c_e the exact chain, where coef (host, rf_coef) adds
//   gamma_D = D u/(1 - D u), u = 2^-24: sequential dot product of D separately
//             rounded products vs the real value (Higham, Accuracy and
//             Stability of Numerical Algorithms, 2nd ed., eq. 3.5);
//   2^-21:    the f16 split of x (and w) against the real products;
//   17 * 2^-23 * (D_pad/16 + 1) * 1.003: the tensor-core f32 accumulation.
//             Products of f16 operands are exact in f32; each K=16 MMA step
//             is taken to add its 16 products and the accumulator with an
//             error below 17 units of 2^-23 of (|acc| + sum|p|): a truncating
//             aligned adder loses less than one unit in the last place of the
//             largest term per addend, a serial one rounds 16 times.  This is
//             a model of the hardware, generous against the published
//             measurements of NVIDIA tensor-core accumulation (Fasi, Higham,
//             Mikaitis, Pranesh, PeerJ CS 7:e330, 2021);
//   4u:       the three f32 adds of the parts.
// Sum |x_d||w_d| <= ||x||_2 ||w||_2 (Cauchy-Schwarz).  The row scale and the
// router bias are applied to the interval ends with directed rounding.
#include <math.h>
#include <string.h>

#include "omc_common.cuh"
#include "omc_bounds.cuh"

namespace {

constexpr int RF_CAPC = 28;          // candidates beyond this: the token is taken whole from the start

__device__ __forceinline__ void rf_cp16(void *smem_dst, const void *gsrc, bool valid) {
    const uint32_t d = smem_u32(smem_dst);
    const int n = valid ? 16 : 0;   // 0 source bytes: zero fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(n) : "memory");
}
__device__ __forceinline__ void rf_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void rf_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// f16 split of two values: hi = RN_f16(v) (saturated), lo = RN_f16(v - hi).
// v - f32(hi) is exact in f32 (hi is within half an f16 unit of v).
__device__ __forceinline__ void rf_split2(float a, float b, uint32_t &hi, uint32_t &lo) {
    hi = f32x2_to_f16x2_sat(a, b);
    const __half2 h = *reinterpret_cast<const __half2 *>(&hi);
    const float2 hf = __half22float2(h);
    lo = f32x2_to_f16x2_sat(a - hf.x, b - hf.y);
}

// rows 0..T-1 of the operand: x_hi; rows T..2T-1: x_lo (AOL layout: element
// (r, k) at (k/64)*R*128 + r*128 + ((k%64)/8 ^ (r&7))*16 + (k%8)*2); xh row t
// = x_hi (when xh); xn[t][seg] = (sum x^2, sum |x|) of each 256-column
// segment, rounded up.  Block 0 also
// writes the identity row map, the GEMM's work items over the Sp operand
// rows, and zeroes the job counters.
__global__ void __launch_bounds__(256) rf_prep_kernel(const float *__restrict__ x, int T, int D, int D_pad, int R,
                                                      uint16_t *__restrict__ act, uint16_t *__restrict__ xh,
                                                      float *__restrict__ xn, int *__restrict__ rowinfo,
                                                      float *__restrict__ roww, int4 *__restrict__ work,
                                                      int *__restrict__ ctl, int ntiles, int *err) {
    const int tid = blockIdx.x * blockDim.x + threadIdx.x, nthr = gridDim.x * blockDim.x;
    const int Sp = (2 * T + OMC_ROW_ALIGN - 1) / OMC_ROW_ALIGN * OMC_ROW_ALIGN;
    for (int r = tid; r < R; r += nthr) {
        rowinfo[r] = r < 2 * T ? r : -1;
        roww[r] = 1.f;
    }
    if (blockIdx.x == 0) {
        const int nch = (Sp + OMC_NMAX - 1) / OMC_NMAX;
        for (int j = threadIdx.x; j < nch * ntiles; j += blockDim.x) {
            const int ch = j / ntiles, p = j - ch * ntiles, n0 = ch * OMC_NMAX;
            work[j] = make_int4(0, p, n0, min(OMC_NMAX, Sp - n0));
        }
        if (threadIdx.x == 0) {
            ctl[0] = 0;
            ctl[1] = nch * ntiles;
            ctl[4] = ctl[5] = ctl[6] = ctl[7] = 0;
        }
    }
    // one warp per (token, 256-column segment); xn holds each segment's sums
    const int lane = threadIdx.x & 31;
    const int nseg = (D_pad + 255) / 256;
    for (int w = tid >> 5; w < T * nseg; w += nthr >> 5) {
        const int t = w / nseg, seg = w - t * nseg;
        const int k0 = seg * 256 + lane * 8;
        const float *xr = x + (size_t)t * D;
        float s2 = 0.f, s1 = 0.f;
        bool outside = false;
        if (k0 < D_pad) {
            float v[8];
            if (k0 < D) {
                const float4 a = *reinterpret_cast<const float4 *>(xr + k0);
                const float4 b = *reinterpret_cast<const float4 *>(xr + k0 + 4);
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
#pragma unroll
                for (int q = 0; q < 8; ++q) v[q] = 0.f;
            }
            uint4 hi, lo;
            rf_split2(v[0], v[1], hi.x, lo.x);
            rf_split2(v[2], v[3], hi.y, lo.y);
            rf_split2(v[4], v[5], hi.z, lo.z);
            rf_split2(v[6], v[7], hi.w, lo.w);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                outside |= omc_f16_outside(v[q]);
                s2 = __fmaf_ru(v[q], v[q], s2);
                s1 = __fadd_ru(s1, fabsf(v[q]));
            }
            const int kb = k0 >> 6, c = (k0 & 63) >> 3;
            uint8_t *base = reinterpret_cast<uint8_t *>(act) + (size_t)kb * R * 128;
            *reinterpret_cast<uint4 *>(base + (size_t)t * 128 + ((c ^ (t & 7)) << 4)) = hi;
            *reinterpret_cast<uint4 *>(base + (size_t)(T + t) * 128 + ((c ^ ((T + t) & 7)) << 4)) = lo;
            if (xh && k0 < D) *reinterpret_cast<uint4 *>(xh + (size_t)t * D + k0) = hi;

        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            s2 = __fadd_ru(s2, __shfl_xor_sync(0xffffffffu, s2, o));
            s1 = __fadd_ru(s1, __shfl_xor_sync(0xffffffffu, s1, o));
        }
        // a value outside the f16 range (NaN too) saturates x_hi: the
        // segment's sums are made infinite, so the candidate pass takes the
        // token whole (every row exact).  It is an error only where x_hi is
        // the expert GEMMs' operand (xh): the host then redoes the forward on
        // the f32 path.
        const bool out_any = __any_sync(0xffffffffu, outside);
        if (lane == 0) {
            xn[2 * w] = out_any ? INFINITY : s2;
            xn[2 * w + 1] = out_any ? INFINITY : s1;
            if (out_any && xh) omc_dev_error(err, OMC_DEVERR_RANGE, OMC_SITE_ROUTER, t);
        }
    }
}

// ---- candidates of one token (one warp) -------------------------------------
// a_e = the sum of the GEMM's product parts; the interval [lo_e, hi_e] holds
// the exact chain's logit (row scale and bias applied with directed rounding);
// the candidates are the experts with hi_e >= (k-th largest lo) - mu.  Writes
// every approximate logit (RN(a_e * s_e)) to the token's logits row and the
// candidates, ascending, to cand[0..nc).  Returns nc, or -1 when the token is
// taken whole (a non-finite or huge value, more than RF_CAPC candidates, or a
// k-th value that may underflow the softmax).
template <int MAXV>
__device__ __forceinline__ int rf_token_candidates(const float *__restrict__ y, int M, int T, int t, int E, int K,
                                                   int split, const float *__restrict__ Ws,
                                                   const float *__restrict__ bias, const float *__restrict__ wn,
                                                   const float *__restrict__ xn, int nseg, float coef,
                                                   float *__restrict__ lrow, int16_t *cand) {
    const int lane = threadIdx.x & 31;
    const float *y0 = y + (size_t)t * M, *y1 = y + (size_t)(T + t) * M;
    // every load first, at in-range indices (the experts past E of the last
    // column are clamped and discarded), so that they are in flight together
    float s2 = lane < nseg ? __ldcg(xn + 2 * (t * nseg + lane)) : 0.f;
    float s1 = lane < nseg ? __ldcg(xn + 2 * (t * nseg + lane) + 1) : 0.f;
    float v0[MAXV], v1[MAXV], v2[MAXV], v3[MAXV], n2[MAXV], n1[MAXV], sc[MAXV], bi[MAXV];
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
        const int e = min(lane + 32 * j, E - 1);
        v0[j] = __ldcg(y0 + e);
        v1[j] = __ldcg(y1 + e);
        v2[j] = split ? __ldcg(y0 + E + e) : 0.f;
        v3[j] = split ? __ldcg(y1 + E + e) : 0.f;
        n2[j] = __ldg(wn + e);
        n1[j] = __ldg(wn + E + e);
        sc[j] = Ws ? __ldg(Ws + e) : 1.f;
        bi[j] = bias ? __ldg(bias + e) : 0.f;
    }
    // ||x||_2 and ||x||_1 from the segments' sums, rounded up
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s2 = __fadd_ru(s2, __shfl_xor_sync(0xffffffffu, s2, o));
        s1 = __fadd_ru(s1, __shfl_xor_sync(0xffffffffu, s1, o));
    }
    const float x2 = __fsqrt_ru(s2), x1 = split ? s1 : 0.f;
    float hi[MAXV], lo[MAXV];
    bool bad = false;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
        const int e = lane + 32 * j;
        hi[j] = -INFINITY;
        lo[j] = -INFINITY;
        if (e >= E) continue;
        float a = __fadd_rn(v0[j], v1[j]);
        if (split) a = __fadd_rn(__fadd_rn(a, v2[j]), v3[j]);
        const float B = __fadd_ru(__fmul_ru(coef, __fmul_ru(x2, n2[j])),
                                  __fmul_ru(1.1920928955078125e-7f, __fadd_ru(n1[j], x1)));
        const float cl = __fsub_rd(a, B), ch = __fadd_ru(a, B);
        float l1 = cl, h1 = ch, ap = a;
        if (Ws) {
            const float s = sc[j];
            l1 = s >= 0.f ? __fmul_rd(cl, s) : __fmul_rd(ch, s);
            h1 = s >= 0.f ? __fmul_ru(ch, s) : __fmul_ru(cl, s);
            ap = __fmul_rn(a, s);
        }
        if (bias) {
            const float b = bi[j];
            l1 = __fadd_rd(l1, b);
            h1 = __fadd_ru(h1, b);
        }
        lo[j] = l1;
        hi[j] = h1;
        bad |= !(fabsf(h1) < 1e30f) || !(fabsf(l1) < 1e30f) || !isfinite(ap);
        lrow[e] = ap;
    }
    if (__any_sync(0xffffffffu, bad)) return -1;
    const int nc = omc_topk_candidates<MAXV>(lo, hi, E, K, RF_CAPC, cand);
    return nc > RF_CAPC ? -1 : nc;
}

// int8 -> f32, exact: the byte (biased to unsigned) is placed in the low
// mantissa bits of 2^23 and the bias subtracted.
__device__ __forceinline__ float rf_i8f(uint32_t u4, uint32_t sel) {
    return __fsub_rn(__uint_as_float(__byte_perm(u4, 0x4B000000u, sel)), 8388736.f);   // 2^23 + 128
}

// ---- bounded pass: candidates and their exact chains, a block of RX_TB tokens
// Every block stages, per chunk (64 int8 or 16 f32 columns), all E router
// rows (64 bytes each, from the chunk-major copy rf_wc: one 1-D bulk copy),
// the shared-gate row and its tokens' rows (one bulk copy each) into a ring of
// RX_ST stages completed on mbarriers: the router is streamed once per RX_TB
// tokens and shared by all their chains, and bulk copies keep a chunk's bytes
// in flight without per-thread requests.  While the first chunks land, each
// warp finds the candidates of two tokens (rf_token_candidates).  Warps 0..6
// then run the candidates' chains (the reference's sequential fp32 order), up
// to RX_MAXJ a thread advanced element by element together so that their adds
// overlap; warp 7 issues the copies and runs the shared-gate chains (an f32
// row: no divergence from the int8 rows).  Last, one warp per token checks
// the order-sensitive near-ties and appends the token's retry chains.  Tokens
// taken whole go to the retry list at once.
constexpr int RX_TB = 16;
constexpr int RX_NT = 256;
constexpr int RX_RW = 7;                         // warps on the routed chains
constexpr int RX_MAXJ = 2;                       // routed chains a thread: 7*32*2 >= RX_TB*RF_CAPC
constexpr int RX_ST = 4;
static_assert(RX_RW * 32 * RX_MAXJ >= RX_TB * RF_CAPC, "routed chain slots");
static_assert(RX_TB <= 30, "one shared-gate chain a lane of warp 7; lanes 2.. copy the token rows");

__host__ __device__ constexpr int rx_kc(int w8) { return w8 ? 64 : 16; }
// a stage: the chunk of every router row, then the shared gate's chunk
__host__ __device__ constexpr int rx_stage_bytes(int E, int w8, int has_shared) {
    return E * 64 + (has_shared ? rx_kc(w8) * 4 : 0);
}
// the block's token rows stay resident (D f32 each, padded by 16 bytes so
// that rows differ in bank), then the stages, barriers and job tables
__host__ __device__ constexpr int rx_xrow(int D) { return D * 4 + 16; }
__host__ __device__ constexpr int rx_smem_bytes(int E, int w8, int has_shared, int D) {
    return RX_TB * rx_xrow(D) + RX_ST * rx_stage_bytes(E, w8, has_shared) + (RX_ST + 1) * 8 + RX_TB * RF_CAPC * 2 +
           RX_TB * 8 + RX_RW * 32 * RX_MAXJ * 8 + 32;
}

// One chunk of one chain: the chunk's rounded products first (independent of
// the chain, so they issue back to back), then their adds in column order
// (the only dependent steps).  wrow: the row's 64-byte chunk (pieces at slot
// p ^ sw), xr: the token's staged columns.
template <bool W8>
__device__ __forceinline__ float rx_chunk(float a, const unsigned char *wrow, int sw, const float *xr) {
    constexpr int KC = W8 ? 64 : 16;
    float p[KC];
#pragma unroll
    for (int pc = 0; pc < 4; ++pc) {
        const uint4 q = *reinterpret_cast<const uint4 *>(wrow + ((pc ^ sw) << 4));
        if (W8) {
            const uint32_t u[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const float4 xv = *reinterpret_cast<const float4 *>(xr + pc * 16 + 4 * g);
                p[pc * 16 + 4 * g + 0] = __fmul_rn(xv.x, rf_i8f(u[g], 0x7540u));
                p[pc * 16 + 4 * g + 1] = __fmul_rn(xv.y, rf_i8f(u[g], 0x7541u));
                p[pc * 16 + 4 * g + 2] = __fmul_rn(xv.z, rf_i8f(u[g], 0x7542u));
                p[pc * 16 + 4 * g + 3] = __fmul_rn(xv.w, rf_i8f(u[g], 0x7543u));
            }
        } else {
            const float4 wv = *reinterpret_cast<const float4 *>(&q);
            const float4 xv = *reinterpret_cast<const float4 *>(xr + pc * 4);
            p[pc * 4 + 0] = __fmul_rn(xv.x, wv.x);
            p[pc * 4 + 1] = __fmul_rn(xv.y, wv.y);
            p[pc * 4 + 2] = __fmul_rn(xv.z, wv.z);
            p[pc * 4 + 3] = __fmul_rn(xv.w, wv.w);
        }
    }
#pragma unroll
    for (int i = 0; i < KC; ++i) a = __fadd_rn(a, p[i]);
    return a;
}

template <int MAXV, bool W8>
__global__ void __launch_bounds__(RX_NT, 1) rf_exact_kernel(const float *__restrict__ x, int T, int D,
                                                            const float *__restrict__ y, int M, int split, float coef,
                                                            const unsigned char *__restrict__ Wc, size_t wc_stride,
                                                            const float *__restrict__ Ws,
                                                            const float *__restrict__ sh_gate, int E, int K,
                                                            int has_shared, const float *__restrict__ bias,
                                                            const float *__restrict__ wn, const float *__restrict__ xn,
                                                            int nseg, float *__restrict__ logits, int ldl,
                                                            int2 *__restrict__ jobs2, int jcap,
                                                            int *__restrict__ ctl, int force_retry, int *err) {
    extern __shared__ __align__(128) unsigned char xsm[];
    constexpr int KC = W8 ? 64 : 16;                                          // columns a chunk
    const int XROW = rx_xrow(D);
    const unsigned char *wcb = Wc + (size_t)(blockIdx.x % OMC_RF_NREP) * wc_stride;
    constexpr int NJ = RX_RW * 32 * RX_MAXJ;                                  // routed chain slots
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int sb = rx_stage_bytes(E, W8 ? 1 : 0, has_shared);
    unsigned char *xrows = xsm;                                               // [TB][XROW]
    unsigned char *stages = xsm + RX_TB * XROW;                               // [ST][sb]
    uint64_t *full = reinterpret_cast<uint64_t *>(stages + RX_ST * sb);       // [ST], then the rows' barrier
    uint64_t *xbar = full + RX_ST;
    int16_t *s_cand = reinterpret_cast<int16_t *>(xbar + 1);                  // [TB][CAPC]
    int *s_nc = reinterpret_cast<int *>(s_cand + RX_TB * RF_CAPC);            // [TB] (-1: whole)
    int *s_off = s_nc + RX_TB;                                                // [TB] first chain slot
    int *s_job = s_off + RX_TB;                                               // [NJ] tok << 16 | row, -1
    float *s_val = reinterpret_cast<float *>(s_job + NJ);                    // [NJ]
    int *s_abort = reinterpret_cast<int *>(s_val + NJ);
    const int t0 = blockIdx.x * RX_TB;
    const int ntok = min(RX_TB, T - t0);
    const int nch = D / KC;
    const int shb = has_shared ? KC * 4 : 0;
    if (tid == 0) {
        for (int i = 0; i < RX_ST + 1; ++i) mbar_init(&full[i], 1);
        *s_abort = 0;
        fence_barrier_init();
    }
    __syncthreads();
    // warp 7: chunk ch into stage ch % ST (its previous chunk was read by every
    // thread before the barrier that precedes this call): two bulk copies
    auto issue = [&](int ch) {
        unsigned char *st = stages + (ch % RX_ST) * sb;
        if (lane == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&full[ch % RX_ST], (uint32_t)(E * 64 + shb));
        }
        __syncwarp();
        if (lane == 0) bulk_g2s(st, wcb + (size_t)ch * E * 64, (uint32_t)(E * 64), &full[ch % RX_ST]);
        if (lane == 1 && has_shared) bulk_g2s(st + E * 64, sh_gate + (size_t)ch * KC, (uint32_t)(KC * 4), &full[ch % RX_ST]);
    };
    if (warp == RX_RW) {
        // the token rows, once
        if (lane == 0) mbar_arrive_expect_tx(xbar, (uint32_t)(ntok * D * 4));
        __syncwarp();
        if (lane < ntok) bulk_g2s(xrows + lane * XROW, x + (size_t)(t0 + lane) * D, (uint32_t)(D * 4), xbar);
        for (int c = 0; c < RX_ST - 1 && c < nch; ++c) issue(c);
    }
    // candidates, two tokens a warp, while the first chunks land
    for (int tl = warp; tl < RX_TB; tl += RX_NT / 32) {
        int nc = 0;
        if (tl < ntok) {
            const int t = t0 + tl;
            nc = rf_token_candidates<MAXV>(y, M, T, t, E, K, split, Ws, bias, wn, xn, nseg, coef,
                                           logits + (size_t)t * ldl, s_cand + tl * RF_CAPC);
            if (nc < 0 && lane == 0) {
                // taken whole: every row (and the shared gate) in the retry pass
                const int n2 = (E + has_shared + 3) & ~3;
                const int b = atomicAdd(ctl + 5, n2);
                if (b + n2 > jcap) {
                    omc_dev_error(err, OMC_DEVERR_BOUNDS, OMC_SITE_ROUTER, b + n2);
                } else {
                    for (int i = 0; i < n2; ++i) jobs2[b + i] = make_int2(t, i < E + has_shared ? i : -1);
                }
                atomicAdd(ctl + 6, 1);
            }
        }
        if (lane == 0) s_nc[tl] = nc;
    }
    __syncthreads();
    // the routed chains, token by token, dealt to the routed warps' slots
    if (warp == 0) {
        const int nc = lane < RX_TB && s_nc[lane] > 0 ? s_nc[lane] : 0;
        int inc = nc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += v;
        }
        const int off = inc - nc, total = __shfl_sync(0xffffffffu, inc, 31);
        if (lane < RX_TB) s_off[lane] = off;
        for (int j = 0; j < nc; ++j) s_job[off + j] = (lane << 16) | s_cand[lane * RF_CAPC + j];
        for (int j = total + lane; j < NJ; j += 32) s_job[j] = -1;
    }
    // slot q of routed thread u = tid (< 224) is chain u + 224 q
    int jt[RX_MAXJ], je[RX_MAXJ];
    float acc[RX_MAXJ];
    const bool routed = warp < RX_RW;
    __syncthreads();
    const bool shared_lane = !routed && has_shared && lane < ntok && s_nc[lane] >= 0;
#pragma unroll
    for (int q = 0; q < RX_MAXJ; ++q) {
        const int code = routed ? s_job[tid + q * RX_RW * 32] : -1;
        jt[q] = code >= 0 ? code >> 16 : 0;
        je[q] = code >= 0 ? code & 0xffff : -1;
        acc[q] = 0.f;
    }
    // a routed warp advances two chains a lane only when some lane has two
    const bool two = __any_sync(0xffffffffu, je[1] >= 0);
    const bool busy = __any_sync(0xffffffffu, je[0] >= 0);
    const int sw0 = ((je[0] > 0 ? je[0] : 0) >> 1) & 3, sw1 = ((je[1] > 0 ? je[1] : 0) >> 1) & 3;
    if (!mbar_wait(xbar, 0, err, OMC_SITE_ROUTER)) atomicExch(s_abort, 1);
    for (int ch = 0; ch < nch; ++ch) {
        if (ch > 0) __syncthreads();           // every thread is done with chunk ch-1's stage
        if (warp == RX_RW && ch + RX_ST - 1 < nch) issue(ch + RX_ST - 1);
        if (!*reinterpret_cast<volatile int *>(s_abort) &&
            !mbar_wait(&full[ch % RX_ST], (uint32_t)((ch / RX_ST) & 1), err, OMC_SITE_ROUTER))
            atomicExch(s_abort, 1);
        if (*reinterpret_cast<volatile int *>(s_abort)) continue;
        const unsigned char *st = stages + (ch % RX_ST) * sb;
        const unsigned char *xs = xrows + ch * KC * 4;         // column ch*KC of token row 0
        if (routed && busy) {
            acc[0] = rx_chunk<W8>(acc[0], st + (je[0] >= 0 ? je[0] : 0) * 64, sw0,
                                  reinterpret_cast<const float *>(xs + jt[0] * XROW));
            if (two)
                acc[1] = rx_chunk<W8>(acc[1], st + (je[1] >= 0 ? je[1] : 0) * 64, sw1,
                                      reinterpret_cast<const float *>(xs + jt[1] * XROW));
        } else if (shared_lane) {
            // the shared gate of token `lane`: products first, then the adds
            const float *xr = reinterpret_cast<const float *>(xs + lane * XROW);
            const float *gr = reinterpret_cast<const float *>(st + E * 64);
            float p[KC];
#pragma unroll
            for (int c = 0; c < KC; c += 4) {
                const float4 xv = *reinterpret_cast<const float4 *>(xr + c);
                const float4 gv = *reinterpret_cast<const float4 *>(gr + c);
                p[c] = __fmul_rn(xv.x, gv.x);
                p[c + 1] = __fmul_rn(xv.y, gv.y);
                p[c + 2] = __fmul_rn(xv.z, gv.z);
                p[c + 3] = __fmul_rn(xv.w, gv.w);
            }
            float a = acc[0];
#pragma unroll
            for (int c = 0; c < KC; ++c) a = __fadd_rn(a, p[c]);
            acc[0] = a;
        }
    }
    __syncthreads();
    if (*reinterpret_cast<volatile int *>(s_abort)) return;   // a staged chunk never landed (reported)
    if (routed) {
#pragma unroll
        for (int q = 0; q < RX_MAXJ; ++q) {
            if (je[q] < 0) continue;
            const int t = t0 + jt[q];
            const float v = Ws ? __fmul_rn(acc[q], Ws[je[q]]) : acc[q];
            logits[(size_t)t * ldl + je[q]] = v;
            s_val[tid + q * RX_RW * 32] = v;
        }
    } else if (shared_lane) {
        logits[(size_t)(t0 + lane) * ldl + E] = acc[0];
    }
    __syncthreads();
    // the order check, one warp per token: softmax numerators of the
    // candidates as the select kernel computes them; two of the k + 1 largest
    // that differ but lie within 2^-21 of each other, or a k-th below 2^-100,
    // send the token to the retry pass with every row exact
    for (int tl = warp; tl < ntok; tl += RX_NT / 32) {
        const int nc = s_nc[tl];
        if (nc < 0) continue;
        const bool have = lane < nc;
        float v = have ? s_val[s_off[tl] + lane] : -INFINITY;
        if (have && bias) v = __fadd_rn(v, bias[s_cand[tl * RF_CAPC + lane]]);
        float m = have && v > -1e30f ? v : -1e30f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float ev = have ? omc_expf_glibc(__fsub_rn(v, m)) : -1.f;
        // rank = how many candidates are strictly larger (every lane runs
        // every shuffle: nc is warp-uniform)
        int rank = 0;
        for (int j = 0; j < nc; ++j) rank += __shfl_sync(0xffffffffu, ev, j) > ev ? 1 : 0;
        bool near = false;
        for (int j = 0; j < nc; ++j) {
            const float o = __shfl_sync(0xffffffffu, ev, j);
            const int rj = __shfl_sync(0xffffffffu, rank, j);
            if (have && rank <= K && rj <= K && o != ev) {
                const float big = fmaxf(o, ev), small = fminf(o, ev);
                near |= big <= __fmul_ru(small, 1.000000476837158203125f);   // 1 + 2^-21
            }
        }
        // the k-th numerator: the value of rank k-1
        const bool kth_small = have && rank <= K - 1 && !(ev >= 7.888609052210118e-31f);   // 2^-100
        const bool retry = force_retry > 0 || nc < K || __any_sync(0xffffffffu, near || kth_small);
        if (retry && lane == 0) {
            const int t = t0 + tl, n2 = (E + 3) & ~3;
            const int b = atomicAdd(ctl + 5, n2);
            if (b + n2 > jcap) {
                omc_dev_error(err, OMC_DEVERR_BOUNDS, OMC_SITE_ROUTER, b + n2);
            } else {
                for (int i = 0; i < n2; ++i) jobs2[b + i] = make_int2(t, i < E ? i : -1);
            }
            atomicAdd(ctl + 7, 1);
        }
        if (lane == 0) atomicAdd(ctl + 4, nc + (has_shared ? 1 : 0));
    }
}

// ---- retry chains: one warp per block, 32 jobs (groups of 4 per token) ------
// The tokens retried or taken whole: their rows' exact chains, one per lane,
// each group of four lanes sharing its token's staged row.  Stage: 8 token
// slots and 32 router rows of RF_KC f32 columns, rows padded by 4 floats.
constexpr int RF_KC = 32;
constexpr int RF_ST = 6;
constexpr int RF_LD = RF_KC + 4;
constexpr int RF_STAGE = (8 + 32) * RF_LD;        // floats
constexpr size_t RF_CHAIN_SMEM = (size_t)RF_ST * RF_STAGE * sizeof(float);

__global__ void __launch_bounds__(32) rf_chain_kernel(const float *__restrict__ x, int D, const float *__restrict__ W,
                                                      const float *__restrict__ Ws, const float *__restrict__ sh_gate,
                                                      int E, const int2 *__restrict__ jobs,
                                                      const int *__restrict__ njobs_p, float *__restrict__ logits,
                                                      int ldl, int jcap) {
    extern __shared__ __align__(16) float rsm[];
    const int lane = threadIdx.x, g = lane >> 2;
    // the counter may have passed the capacity (the writers then reported
    // OMC_DEVERR_BOUNDS and wrote nothing past it)
    const int njobs = min(*reinterpret_cast<volatile const int *>(njobs_p), jcap);
    const int nwin = (njobs + 31) >> 5;
    const int nch = (D + RF_KC - 1) / RF_KC;
    for (int win = blockIdx.x; win < nwin; win += gridDim.x) {
        const int j = win * 32 + lane;
        int t = -1, e = -1;
        if (j < njobs) {
            const int2 jb = jobs[j];
            t = jb.x;
            e = jb.y;
        }
        const int tg = __shfl_sync(0xffffffffu, t, g * 4);
        const float *wrow = e >= 0 ? (e < E ? W + (size_t)e * D : sh_gate) : nullptr;
        const float *xrow = tg >= 0 ? x + (size_t)tg * D : nullptr;
        auto stage = [&](int ch) {
            float *st = rsm + (ch % RF_ST) * RF_STAGE;
            const int c0 = ch * RF_KC;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int piece = (lane & 3) * 2 + q, c = c0 + piece * 4;
                const bool ok = xrow && c < D;
                rf_cp16(st + g * RF_LD + piece * 4, ok ? xrow + c : x, ok);
            }
#pragma unroll
            for (int q = 0; q < RF_KC / 4; ++q) {
                const int c = c0 + q * 4;
                const bool ok = wrow && c < D;
                rf_cp16(st + (8 + lane) * RF_LD + q * 4, ok ? wrow + c : x, ok);
            }
        };
#pragma unroll
        for (int s = 0; s < RF_ST - 1; ++s) {
            if (s < nch) stage(s);
            rf_commit();
        }
        float acc = 0.f;
        for (int ch = 0; ch < nch; ++ch) {
            rf_wait<RF_ST - 2>();
            __syncwarp();      // every lane's copies of chunk ch landed; chunk ch-1's stage is free
            if (ch + RF_ST - 1 < nch) stage(ch + RF_ST - 1);
            rf_commit();
            const float *st = rsm + (ch % RF_ST) * RF_STAGE;
            const float *xs = st + g * RF_LD, *wsr = st + (8 + lane) * RF_LD;
#pragma unroll
            for (int c = 0; c < RF_KC; c += 4) {
                const float4 xv = *reinterpret_cast<const float4 *>(xs + c);
                const float4 wv = *reinterpret_cast<const float4 *>(wsr + c);
                acc = __fadd_rn(acc, __fmul_rn(xv.x, wv.x));
                acc = __fadd_rn(acc, __fmul_rn(xv.y, wv.y));
                acc = __fadd_rn(acc, __fmul_rn(xv.z, wv.z));
                acc = __fadd_rn(acc, __fmul_rn(xv.w, wv.w));
            }
        }
        rf_wait<0>();
        __syncwarp();          // the ring is free for the next window
        if (e >= 0) logits[(size_t)t * ldl + e] = (Ws && e < E) ? __fmul_rn(acc, Ws[e]) : acc;
    }
}

__global__ void __launch_bounds__(256) rf_split_rows_kernel(const float *__restrict__ W, long long n, float *__restrict__ dst) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float w = W[i];
        const float h = __half2float(__float2half_rn(w));
        dst[i] = h;
        dst[n + i] = w - h;
    }
}

}  // namespace

int omc_router_exact = 0;
int omc_rf_force_retry = 0;

// 0 (the default): the bounded router for layers with E >= OMC_RF_EMIN from
// T = OMC_RF_TMIN, the exact router otherwise; 1: the exact router for every
// forward (bit-exact routing weights too); 2: the bounded router for every
// eligible layer whatever E (tests of the small-E shapes).
extern "C" int omc_set_router_exact(int mode) {
    if (mode < 0 || mode > 2) return OMC_EINVAL;
    omc_router_exact = mode;
    omc_graphs_invalidate();
    return 0;
}

// Test hook: 1 = every token of a bounded pass is retried with every row exact.
extern "C" int omc_debug_rf_force_retry(int on) {
    if (on != 0 && on != 1) return OMC_EINVAL;
    omc_rf_force_retry = on;
    omc_graphs_invalidate();
    return 0;
}

// dst [2E][D]: the f16 rounding of W's rows (as f32), then the remainders.
extern "C" int omc_launch_rf_split_rows(const float *W, int E, int D, float *dst, cudaStream_t s) {
    const long long n = (long long)E * D;
    if (n <= 0) return OMC_EINVAL;
    rf_split_rows_kernel<<<(int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096), 256, 0, s>>>(W, n, dst);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// Whether a forward of T tokens on L takes the bounded router: the mode (and,
// by default, E >= OMC_RF_EMIN), the layer has its tiles (not GEMMA, D % 8 ==
// 0), T >= OMC_RF_TMIN,
// the workspace holds 2T operand rows, and a block's staging fits.
extern "C" int omc_rf_eligible(const omc_layer_dev *L, int T, const omc_ws *ws) {
    if (omc_router_exact == 1 || (omc_router_exact == 0 && L->E < OMC_RF_EMIN) || !L->rf_tab ||
        L->family == OMC_FAMILY_GEMMA || T < OMC_RF_TMIN || !ws->rf_act ||
        2 * T > ws->rf_R || (L->D % 8) || L->E > 1024 || L->D_pad > 32 * 256)
        return 0;
    const int w8 = L->router_i8 ? 1 : 0;
    if (!L->rf_wc || (L->D % rx_kc(w8)) || (size_t)L->E * 64 > (1u << 20)) return 0;
    return rx_smem_bytes(L->E, w8, L->has_shared && L->sh_gate ? 1 : 0, L->D) <= 220 * 1024;
}

// The bounded router's logits rows (exact for every expert that can be
// selected and for the shared gate, bounded approximations otherwise), xh
// (when non-NULL) the expert GEMMs' f16 token operand.  The caller checked
// eligibility (rf_tab, T >= 16, the workspace's rf buffers).
extern "C" int omc_launch_router_fast(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                                      uint16_t *xh, cudaStream_t s) {
    static int nsm = 0;
    if (!nsm) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return OMC_ECUDA;
    }
    const int E = L->E, D = L->D, M = L->rf_rows;
    if (2 * T > ws->rf_R || (D % 8)) return OMC_EINVAL;
    const int ntiles = (M + OMC_TM - 1) / OMC_TM;
    const int ldl = E + 1;
    // 1. prep
    {
        const long long nw = (long long)T * ((L->D_pad + 255) / 256);
        const int blocks = (int)((nw + 7) / 8 < 4096 ? (nw + 7) / 8 : 4096);
        rf_prep_kernel<<<blocks, 256, 0, s>>>(x, T, D, L->D_pad, ws->rf_R, ws->rf_act, xh, ws->rf_xn,
                                              ws->rf_rowinfo, ws->rf_roww, reinterpret_cast<int4 *>(ws->rf_work),
                                              ws->rf_ctl, ntiles, ws->err);
    }
    // 2. approximate products on the tensor cores
    omc_layer_dev Ld;
    memset(&Ld, 0, sizeof(Ld));
    Ld.family = OMC_FAMILY_OLMOE;
    Ld.D = M;
    Ld.I = D;
    Ld.E = 1;
    Ld.k = 1;
    Ld.D_pad = (M + OMC_KB - 1) / OMC_KB * OMC_KB;
    Ld.I_pad = L->D_pad;
    Ld.D_rows = ntiles * OMC_TM;
    Ld.I_rows = L->D_rows;
    Ld.experts = L->rf_tab;
    int rc = omc_launch_gemm_dense_op(&Ld, ws->rf_act, ws->rf_R, ws->rf_rowinfo, ws->rf_roww, ws->rf_work,
                                      ws->rf_ctl, ws->rf_y, ws->err, s);
    if (rc) return rc;
    // 3. candidates.  coef: see the file comment (u = 2^-24, kappa = 17)
    const double u = 1.0 / 16777216.0;
    const double gam = (double)D * u / (1.0 - (double)D * u);
    double coef = gam + 1.0 / 2097152.0 + 17.0 * (2.0 * u) * ((double)L->D_pad / 16.0 + 1.0) * 1.003 + 4.0 * u;
    coef *= 1.001;
    const float coef_f = nextafterf((float)coef, INFINITY);
    const float *Ws = L->router_i8 ? L->router_s : nullptr;
    const int hs = L->has_shared && L->sh_gate ? 1 : 0;
    const int nv = (E + 31) / 32;
    const bool w8 = L->router_i8 != 0;
    const int smem = rx_smem_bytes(E, w8 ? 1 : 0, hs, D);
    const dim3 gx((T + RX_TB - 1) / RX_TB);
    // 3.-4. candidates and their chains, the order check
#define RFX(NV, W)                                                                                                   \
    do {                                                                                                             \
        static int attr = 0;                                                                                         \
        if (attr < smem) {                                                                                           \
            if (cudaFuncSetAttribute(rf_exact_kernel<NV, W>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=   \
                cudaSuccess)                                                                                         \
                return OMC_ECUDA;                                                                                    \
            attr = smem;                                                                                             \
        }                                                                                                            \
        rf_exact_kernel<NV, W><<<gx, RX_NT, smem, s>>>(                                                              \
            x, T, D, ws->rf_y, M, L->rf_split, coef_f, L->rf_wc, L->rf_wc_stride, Ws, L->sh_gate, E, L->k, hs,       \
            L->rbias,                                                                                                \
            L->rf_wn, ws->rf_xn, (L->D_pad + 255) / 256, ws->logits, ldl, reinterpret_cast<int2 *>(ws->rf_jobs2),     \
            ws->rf_jcap, ws->rf_ctl,                                                                                 \
            omc_rf_force_retry, ws->err);                                                                            \
    } while (0)
#define RFXW(NV) \
    do {         \
        if (w8) RFX(NV, true); \
        else RFX(NV, false);   \
    } while (0)
    if (nv <= 1) RFXW(1);
    else if (nv <= 2) RFXW(2);
    else if (nv <= 4) RFXW(4);
    else if (nv <= 8) RFXW(8);
    else if (nv <= 16) RFXW(16);
    else RFXW(32);
#undef RFXW
#undef RFX
    // 5. tokens retried or taken whole: every row exact
    const long long win_max = ((long long)T * ((E + 4) & ~3) + 31) / 32;
    const int g2 = (int)(win_max < (long long)nsm * 2 ? win_max : (long long)nsm * 2);
    rf_chain_kernel<<<g2, 32, RF_CHAIN_SMEM, s>>>(x, D, L->router, Ws, L->sh_gate, E,
                                                  reinterpret_cast<const int2 *>(ws->rf_jobs2), ws->rf_ctl + 5,
                                                  ws->logits, ldl, ws->rf_jcap);
    omc_g_launches += 3;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}
