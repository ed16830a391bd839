// router.cu -- MoE router on the GPU: logits, softmax, top-k, renormalise.
//
// Bit-exact with the reference CPU router on identical inputs:
//   logits : engines/olmoe.c:74-85 (f32 matmul) / engines/qwen.c:116-121
//            (matmul_q on the int8 router): one sequential fp32 chain per
//            (token, expert), products and sums rounded separately (no FMA),
//            exactly the x86-64 scalar order.  The int8 router is held as its
//            exact f32 values and the row scale applied last (acc*scale).
//   softmax: engines/olmoe.c:170-174 (float running sum) and
//            engines/qwen.c:161-165 (double running sum, divide by float(s)),
//            with omc_expf_glibc, bit-equal to glibc expf.
//   top-k  : engines/olmoe.c:355-362 -- k passes of argmax, strict '>' in
//            ascending id order = (largest p, then lowest id).
//   renorm : engines/olmoe.c:363, engines/qwen.c:476-477 (float sum in
//            selection order, then divide).
//   shared gate: engines/qwen.c:460-461, sigmoid(sum sh_gate[i]*x[i]).
#include "omc_plan.cuh"
#include "omc_select.cuh"

namespace {

// ---- logits -----------------------------------------------------------------
// Block = G x G threads (G = 16 or 8); thread (tg, rg) runs the TT x RR
// chains of tokens tg + Gi and router rows rg + Gj of the block's (G TT) x
// (G RR) tile (strided, so a warp's token rows fall in distinct bank quads
// and its row groups broadcast).  Per four K elements a thread loads TT + RR
// 16-byte vectors and advances 4 TT RR chains: separately rounded products,
// then two chains' adds at a time as one packed add.rn.f32x2.  K
// streams through a 4-stage cp.async ring of KC-element chunks; a partial
// last chunk is zero-filled (adding 0*0 leaves a chain's value unchanged: it
// starts at +0, so it is never -0).  The tile is chosen per launch
// (launch_logits): 2 x 2 chains per thread with 64-element chunks once the
// grid fills the SMs, else one chain per thread with 128-element chunks, so
// that three chunks of chain work cover a chunk's L2 latency.
constexpr int RT_ST = 4;                    // stages (8 measured no faster, and halves occupancy)

template <int G, int TT, int RR, int KC>
constexpr size_t rt_smem() { return (size_t)RT_ST * (G * TT + G * RR) * (KC + 4) * sizeof(float); }
static_assert(rt_smem<16, 4, 4, 32>() <= 200 * 1024 && rt_smem<16, 2, 2, 64>() <= 200 * 1024 &&
                  rt_smem<16, 1, 1, 128>() <= 200 * 1024,
              "router staging");

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc, bool valid) {
    const uint32_t d = smem_u32(smem_dst);
    const int n = valid ? 16 : 0;       // 0 source bytes: the 16 bytes are zero-filled
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Packed IEEE add, two lanes, each rounded to nearest as add.rn.f32.  The
// products stay scalar __fmul_rn: with a packed multiply feeding it, the
// chains came out a few ulps off the reference (as if the product were not
// rounded on its own), so they are kept as two separately rounded multiplies.
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    float2 r;
    asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rc, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rc;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}

// logits[t][j], j < nrows: rows 0..E-1 are the router, row E (when
// has_shared) the shared-expert gate vector.  Every (token, row) value is the
// reference's chain acc = RN(acc + RN(x[i] * w[i])), i ascending.
template <int G, int TT, int RR, int KC>
__global__ void __launch_bounds__(G * G, 2) router_tile_kernel(const float *__restrict__ x, int T, int D,
                                                                  const float *__restrict__ W,
                                                                  const float *__restrict__ Ws, int E,
                                                                  const float *__restrict__ sh_gate, int nrows,
                                                                  float *__restrict__ logits, int ldl,
                                                                  uint16_t *__restrict__ xh, int *err) {
    extern __shared__ __align__(16) float rsm[];
    constexpr int NT = G * G, BT = G * TT, BR = G * RR, LD = KC + 4, STAGE = (BT + BR) * LD;
    const int tid = threadIdx.x, tg = tid % G, rg = tid / G;
    const int t0 = blockIdx.x * BT, r0 = blockIdx.y * BR;
    const int nch = (D + KC - 1) / KC;
    auto load = [&](int ch) {
        float *st = rsm + (size_t)(ch % RT_ST) * STAGE;
        const int c0 = ch * KC;
        for (int i = tid; i < (BT + BR) * (KC / 4); i += NT) {
            const int r = i / (KC / 4), c = (i % (KC / 4)) * 4;
            const float *src;
            bool ok;
            if (r < BT) {
                ok = t0 + r < T;
                src = x + (size_t)(t0 + r) * D + c0 + c;
            } else {
                const int gr = r0 + r - BT;
                ok = gr < nrows;
                src = (gr < E ? W + (size_t)gr * D : sh_gate) + c0 + c;
            }
            ok = ok && c0 + c < D;
            cp_async16(st + r * LD + c, ok ? src : x, ok);
        }
    };
#pragma unroll
    for (int s = 0; s < RT_ST - 1; ++s) {
        if (s < nch) load(s);
        cp_async_commit();
    }
    float acc[TT][RR];
#pragma unroll
    for (int i = 0; i < TT; ++i)
#pragma unroll
        for (int j = 0; j < RR; ++j) acc[i][j] = 0.f;
    for (int ch = 0; ch < nch; ++ch) {
        cp_async_wait<RT_ST - 2>();   // chunk ch has landed (this thread's copies)
        __syncthreads();              // ... everyone's; and chunk ch-1's stage is free
        if (ch + RT_ST - 1 < nch) load(ch + RT_ST - 1);
        cp_async_commit();
        const float *st = rsm + (size_t)(ch % RT_ST) * STAGE;
        if (xh && blockIdx.y == 0) {
            // the f16 token operand of the expert GEMMs (row t of xh = x[t]
            // rounded to f16), written by the first row of blocks; a value
            // outside the f16 range is reported, not clipped silently
            for (int i = tid; i < BT * (KC / 8); i += NT) {
                const int r = i / (KC / 8), c = (i % (KC / 8)) * 8;
                if (t0 + r < T && ch * KC + c < D) {
                    const float *v = st + r * LD + c;
                    bool out = false;
#pragma unroll
                    for (int q = 0; q < 8; ++q) out |= omc_f16_outside(v[q]);
                    if (out) omc_dev_error(err, OMC_DEVERR_RANGE, OMC_SITE_ROUTER, t0 + r);
                    uint4 o;
                    o.x = f32x2_to_f16x2_sat(v[0], v[1]);
                    o.y = f32x2_to_f16x2_sat(v[2], v[3]);
                    o.z = f32x2_to_f16x2_sat(v[4], v[5]);
                    o.w = f32x2_to_f16x2_sat(v[6], v[7]);
                    *reinterpret_cast<uint4 *>(xh + (size_t)(t0 + r) * D + ch * KC + c) = o;
                }
            }
        }
        // operands of the next four K elements are loaded before this
        // four's chain steps, so a shared-memory load's latency is not on
        // the add chain
        float4 xv[TT], wv[RR], xn[TT], wn[RR];
#pragma unroll
        for (int i = 0; i < TT; ++i) xn[i] = *reinterpret_cast<const float4 *>(st + (tg + G * i) * LD);
#pragma unroll
        for (int j = 0; j < RR; ++j) wn[j] = *reinterpret_cast<const float4 *>(st + (BT + rg + G * j) * LD);
        // fully unrolled over the chunk: the next four columns' operands (xn,
        // wn) become renamed registers, not copies
#pragma unroll
        for (int kk = 0; kk < KC; kk += 4) {
#pragma unroll
            for (int i = 0; i < TT; ++i) xv[i] = xn[i];
#pragma unroll
            for (int j = 0; j < RR; ++j) wv[j] = wn[j];
            if (kk + 4 < KC) {
#pragma unroll
                for (int i = 0; i < TT; ++i) xn[i] = *reinterpret_cast<const float4 *>(st + (tg + G * i) * LD + kk + 4);
#pragma unroll
                for (int j = 0; j < RR; ++j)
                    wn[j] = *reinterpret_cast<const float4 *>(st + (BT + rg + G * j) * LD + kk + 4);
            }
#pragma unroll
            for (int sk = 0; sk < 4; ++sk) {
                const float *xs = reinterpret_cast<const float *>(xv);   // xv[i] component sk: xs[4i + sk]
                const float *ws = reinterpret_cast<const float *>(wv);
                if constexpr (RR >= 2) {
#pragma unroll
                    for (int i = 0; i < TT; ++i)
#pragma unroll
                        for (int j = 0; j < RR; j += 2) {
                            const float2 p = make_float2(__fmul_rn(xs[4 * i + sk], ws[4 * j + sk]),
                                                         __fmul_rn(xs[4 * i + sk], ws[4 * (j + 1) + sk]));
                            const float2 r = add2_rn(make_float2(acc[i][j], acc[i][j + 1]), p);
                            acc[i][j] = r.x;
                            acc[i][j + 1] = r.y;
                        }
                } else if constexpr (TT >= 2) {
#pragma unroll
                    for (int i = 0; i < TT; i += 2) {
                        const float2 p = make_float2(__fmul_rn(xs[4 * i + sk], ws[sk]),
                                                     __fmul_rn(xs[4 * (i + 1) + sk], ws[sk]));
                        const float2 r = add2_rn(make_float2(acc[i][0], acc[i + 1][0]), p);
                        acc[i][0] = r.x;
                        acc[i + 1][0] = r.y;
                    }
                } else {
                    acc[0][0] = __fadd_rn(acc[0][0], __fmul_rn(xs[sk], ws[sk]));
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < TT; ++i) {
        const int t = t0 + tg + G * i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < RR; ++j) {
            const int r = r0 + rg + G * j;
            if (r < nrows) logits[(size_t)t * ldl + r] = (Ws && r < E) ? __fmul_rn(acc[i][j], Ws[r]) : acc[i][j];
        }
    }
}

// ---- logits, resident token rows ---------------------------------------------
// Block = 16 tokens x 16 router rows, one chain a thread (thread tid: token
// tid % 16, row tid / 16).  The block's 16 token rows are copied once into
// shared memory by 1-D bulk copies (rows padded by 16 bytes, so that the 16
// rows differ in bank) and its 16 router rows stream through a ring of
// 128-column chunks, each one 8 KB bulk copy of the row-block-major copy rt_w
// (rows rotated by a 16-byte unit each).  Each chunk's products are computed
// ahead of its adds, which keep the reference's order.  Copies complete on
// mbarriers; every wait is bounded.  (The staging of router_tile_kernel, per
// thread cp.async, caps near 15 GB/s per SM on B200; bulk copies do not.)
constexpr int R2_TB = 16, R2_RB = 16, R2_KC = 128, R2_ST = 6;
constexpr int R2_WSTAGE = R2_RB * R2_KC * 4;    // 8 KB
__host__ __device__ constexpr int r2_xrow(int D) { return D * 4 + 16; }
__host__ __device__ constexpr int r2_smem(int D) { return R2_TB * r2_xrow(D) + R2_ST * R2_WSTAGE + (R2_ST + 1) * 8 + 16; }

__global__ void __launch_bounds__(256, 1) router_tile2_kernel(const float *__restrict__ x, int T, int D,
                                                              const float *__restrict__ Wt,
                                                              const float *__restrict__ Ws, int E, int nrows,
                                                              float *__restrict__ logits, int ldl,
                                                              uint16_t *__restrict__ xh, int *err) {
    extern __shared__ __align__(128) unsigned char r2sm[];
    const int XROW = r2_xrow(D);
    unsigned char *xrows = r2sm;
    float *stages = reinterpret_cast<float *>(r2sm + R2_TB * XROW);
    uint64_t *full = reinterpret_cast<uint64_t *>(reinterpret_cast<unsigned char *>(stages) + R2_ST * R2_WSTAGE);
    uint64_t *xbar = full + R2_ST;
    int *s_abort = reinterpret_cast<int *>(xbar + 1);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tg = tid & 15, rg = tid >> 4;
    const int t0 = blockIdx.x * R2_TB, rb = blockIdx.y;
    const int ntok = min(R2_TB, T - t0);
    const int nch = D / R2_KC;
    if (tid == 0) {
        for (int i = 0; i < R2_ST + 1; ++i) mbar_init(&full[i], 1);
        *s_abort = 0;
        fence_barrier_init();
    }
    __syncthreads();
    auto issue = [&](int c) {      // thread 0: chunk c into stage c % ST
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&full[c % R2_ST], (uint32_t)R2_WSTAGE);
        bulk_g2s(reinterpret_cast<unsigned char *>(stages) + (c % R2_ST) * R2_WSTAGE,
                 Wt + (size_t)(rb * nch + c) * R2_RB * R2_KC, (uint32_t)R2_WSTAGE, &full[c % R2_ST]);
    };
    if (warp == 0) {
        if (lane == 0) mbar_arrive_expect_tx(xbar, (uint32_t)(ntok * D * 4));
        __syncwarp();
        if (lane < ntok) bulk_g2s(xrows + lane * XROW, x + (size_t)(t0 + lane) * D, (uint32_t)(D * 4), xbar);
        if (lane == 0)
            for (int c = 0; c < R2_ST - 1 && c < nch; ++c) issue(c);
    }
    if (!mbar_wait(xbar, 0, err, OMC_SITE_ROUTER)) atomicExch(s_abort, 1);
    __syncthreads();
    if (xh && rb == 0 && !*reinterpret_cast<volatile int *>(s_abort)) {
        // the f16 token operand of the expert GEMMs (row t of xh = x[t]
        // rounded to f16), from the resident rows; a value outside the f16
        // range is reported, not clipped silently
        const int n8 = D / 8;
        for (int i = tid; i < ntok * n8; i += 256) {
            const int r = i / n8, c8 = (i - r * n8) * 8;
            const float *v = reinterpret_cast<const float *>(xrows + r * XROW) + c8;
            const float4 a = *reinterpret_cast<const float4 *>(v), b = *reinterpret_cast<const float4 *>(v + 4);
            if (omc_f16_outside(a.x) || omc_f16_outside(a.y) || omc_f16_outside(a.z) || omc_f16_outside(a.w) ||
                omc_f16_outside(b.x) || omc_f16_outside(b.y) || omc_f16_outside(b.z) || omc_f16_outside(b.w))
                omc_dev_error(err, OMC_DEVERR_RANGE, OMC_SITE_ROUTER, t0 + r);
            uint4 o;
            o.x = f32x2_to_f16x2_sat(a.x, a.y);
            o.y = f32x2_to_f16x2_sat(a.z, a.w);
            o.z = f32x2_to_f16x2_sat(b.x, b.y);
            o.w = f32x2_to_f16x2_sat(b.z, b.w);
            *reinterpret_cast<uint4 *>(xh + (size_t)(t0 + r) * D + c8) = o;
        }
    }
    float acc = 0.f;
    const float *xr = reinterpret_cast<const float *>(xrows + tg * XROW);
    for (int c = 0; c < nch; ++c) {
        if (c > 0) __syncthreads();                 // every thread is done with chunk c-1's stage
        if (tid == 0 && c + R2_ST - 1 < nch) issue(c + R2_ST - 1);
        if (!*reinterpret_cast<volatile int *>(s_abort) &&
            !mbar_wait(&full[c % R2_ST], (uint32_t)((c / R2_ST) & 1), err, OMC_SITE_ROUTER))
            atomicExch(s_abort, 1);
        if (*reinterpret_cast<volatile int *>(s_abort)) continue;
        const float *wr = stages + (c % R2_ST) * (R2_RB * R2_KC) + rg * R2_KC;
        const float *xc = xr + c * R2_KC;
#pragma unroll
        for (int h = 0; h < R2_KC; h += 32) {
            float p[32];
#pragma unroll
            for (int q = 0; q < 32; q += 4) {
                const float4 xv = *reinterpret_cast<const float4 *>(xc + h + q);
                const float4 wv = *reinterpret_cast<const float4 *>(wr + ((((h + q) >> 2) + rg) & 31) * 4);
                p[q] = __fmul_rn(xv.x, wv.x);
                p[q + 1] = __fmul_rn(xv.y, wv.y);
                p[q + 2] = __fmul_rn(xv.z, wv.z);
                p[q + 3] = __fmul_rn(xv.w, wv.w);
            }
#pragma unroll
            for (int q = 0; q < 32; ++q) acc = __fadd_rn(acc, p[q]);
        }
    }
    __syncthreads();
    if (*reinterpret_cast<volatile int *>(s_abort)) return;   // a copy never landed (reported)
    const int t = t0 + tg, r = rb * R2_RB + rg;
    if (t < T && r < nrows) logits[(size_t)t * ldl + r] = (Ws && r < E) ? __fmul_rn(acc, Ws[r]) : acc;
}

// rows row0..row0+nr-1 of the row-block-major copy from W [nr][D]
__global__ void __launch_bounds__(256) rt_blocks_kernel(const float *__restrict__ W, int row0, int nr, int D,
                                                        float *__restrict__ dst) {
    const int nch = D / R2_KC;
    const long long n4 = (long long)nr * (D / 4);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const int rr = (int)(i / (D / 4)), u = (int)(i - (long long)rr * (D / 4));   // row, 16-byte unit
        const int row = row0 + rr, c = u / (R2_KC / 4), uc = u - c * (R2_KC / 4);
        const float4 v = *reinterpret_cast<const float4 *>(W + (size_t)rr * D + (size_t)u * 4);
        float *blk = dst + ((size_t)((row / R2_RB) * nch + c) * R2_RB + (row % R2_RB)) * R2_KC;
        *reinterpret_cast<float4 *>(blk + ((uc + row % R2_RB) & 31) * 4) = v;
    }
}

// ---- logits, few tokens --------------------------------------------------------
// Decode-sized batches (T <= 8): one block per 8 router rows stages all of D
// for its rows and the T tokens at once (one memory latency instead of a
// chunk pipeline), then one thread per (token, row) runs the exact chain.
// The chain (D dependent adds) is the floor; the standard kernel would spread
// 8 tokens x 32 rows over a single block and walk D in 16 staged chunks.
constexpr int RS_ROWS = 8;
constexpr int RS_TMAX = 8;

__global__ void __launch_bounds__(256) router_logits_small_kernel(const float *__restrict__ x, int T, int D,
                                                                   const float *__restrict__ W,
                                                                   const float *__restrict__ Ws, int E,
                                                                   const float *__restrict__ sh_gate, int nrows,
                                                                   float *__restrict__ logits, int ldl) {
    extern __shared__ __align__(16) float sm[];     // [T][D+4] tokens, then [RS_ROWS][D+4] rows
    const int LD = D + 4, tid = threadIdx.x;
    const int r0 = blockIdx.x * RS_ROWS;
    float *xs = sm, *wsm = sm + (size_t)T * LD;
    const int q4 = D / 4;
    for (int i = tid; i < (T + RS_ROWS) * q4; i += blockDim.x) {
        const int row = i / q4, c = (i % q4) * 4;
        const float *src;
        float *dst;
        bool ok;
        if (row < T) {
            ok = true;
            src = x + (size_t)row * D + c;
            dst = xs + (size_t)row * LD + c;
        } else {
            const int gr = r0 + row - T;
            ok = gr < nrows;
            src = (gr < E ? W + (size_t)gr * D : sh_gate) + c;
            dst = wsm + (size_t)(row - T) * LD + c;
        }
        cp_async16(dst, ok ? src : x, ok);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    if (tid >= T * RS_ROWS) return;
    const int t = tid / RS_ROWS, r = tid % RS_ROWS, gr = r0 + r;
    const float *xr = xs + (size_t)t * LD, *wr = wsm + (size_t)r * LD;
    float acc = 0.f;
#pragma unroll 8
    for (int c = 0; c < D; c += 4) {
        const float4 xv = *reinterpret_cast<const float4 *>(xr + c);
        const float4 wv = *reinterpret_cast<const float4 *>(wr + c);
        acc = __fadd_rn(acc, __fmul_rn(xv.x, wv.x));
        acc = __fadd_rn(acc, __fmul_rn(xv.y, wv.y));
        acc = __fadd_rn(acc, __fmul_rn(xv.z, wv.z));
        acc = __fadd_rn(acc, __fmul_rn(xv.w, wv.w));
    }
    if (gr < nrows) logits[(size_t)t * ldl + gr] = (Ws && gr < E) ? __fmul_rn(acc, Ws[gr]) : acc;
}

// ---- select: select_token (omc_select.cuh) -------------------------------
__host__ __device__ constexpr int SEL_SMEM_FLOATS(int maxv) { return SEL_WARPS * maxv * 32 > OMC_PLAN_SMEM_INTS ? SEL_WARPS * maxv * 32 : OMC_PLAN_SMEM_INTS; }

template <int SEL_MAXV>
__global__ void __launch_bounds__(SEL_WARPS * 32) router_select_kernel(const float *__restrict__ logits, int ldl, int T,
                                                                       int E, int K, int family, int renorm,
                                                                       int has_shared, const float *__restrict__ pes,
                                                                       const float *__restrict__ bias,
                                                                       int32_t *__restrict__ topk_idx,
                                                                       float *__restrict__ topk_w, float *__restrict__ sg,
                                                                       omc_plan_args plan, int do_plan, int *err) {
    // per-warp softmax rows, reused by the plan in the last block
    __shared__ __align__(16) float sbuf[SEL_SMEM_FLOATS(SEL_MAXV)];
    __shared__ int s_last;
    const int wib = threadIdx.x >> 5;
    const int t = blockIdx.x * SEL_WARPS + wib;
    if (t < T)
        select_token<SEL_MAXV>(logits, ldl, t, E, K, family, renorm, has_shared, pes, bias, topk_idx, topk_w, sg, err,
                               sbuf + wib * SEL_MAXV * 32);
    if (!do_plan) return;
    // count the routed slots per expert here: a slot's rank is its row within
    // the expert's group (arrival order; an expert's rows are independent, so
    // the order changes no value).  Ranks within the block come from
    // shared-memory atomics, then one global atomic per (block, expert) adds
    // the block's count: under skewed routing a hot expert's counter takes one
    // atomic per block instead of one per token.
    __shared__ int s_cnt[OMC_MAX_E], s_gbase[OMC_MAX_E];
    for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
    __syncthreads();
    int my_e = -1, my_local = -1;
    const bool has_slot = t < T && (threadIdx.x & 31) < K;
    if (has_slot) {
        my_e = topk_idx[t * K + (threadIdx.x & 31)];   // this thread's own write in select_token
        if (my_e >= plan.e_lo && my_e < plan.e_hi) my_local = atomicAdd(&s_cnt[my_e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x)
        if (s_cnt[e]) s_gbase[e] = atomicAdd(plan.counts + e, s_cnt[e]);
    __syncthreads();
    if (has_slot) plan.slotrow[t * K + (threadIdx.x & 31)] = my_local >= 0 ? s_gbase[my_e] + my_local : -1;
    // last-block handoff.  The block barrier orders every thread's routing
    // writes before thread 0's gpu-scope fence, which (fences are cumulative)
    // orders them before its count; the block that counts last fences again
    // before its threads read every block's writes.  One fence per block, not
    // one per thread.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(plan.done, 1) == (int)gridDim.x - 1;
        if (s_last) __threadfence();
    }
    __syncthreads();
    if (!s_last) return;
    omc_plan_block(plan, topk_idx, topk_w, err, reinterpret_cast<int *>(sbuf), true);
}

template <int G, int TT, int RR, int KC>
int launch_tile(const omc_layer_dev *L, const float *x, int T, int nrows, float *logits, int ldl, uint16_t *xh,
                int *err, cudaStream_t s) {
    static int attr_done = 0;
    if (!attr_done) {
        if (cudaFuncSetAttribute(router_tile_kernel<G, TT, RR, KC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)rt_smem<G, TT, RR, KC>()) != cudaSuccess)
            return OMC_ECUDA;
        attr_done = 1;
    }
    const dim3 g((T + G * TT - 1) / (G * TT), (nrows + G * RR - 1) / (G * RR));
    router_tile_kernel<G, TT, RR, KC><<<g, G * G, rt_smem<G, TT, RR, KC>(), s>>>(
        x, T, L->D, L->router, L->router_i8 ? L->router_s : nullptr, L->E, L->sh_gate, nrows, logits, ldl, xh, err);
    return 0;
}

// Test hook: a forced tile (G, TT, RR), 0 = automatic.
int g_force_tile = 0;

// The largest tile whose blocks still cover every SM (smaller T: smaller tiles).
int launch_logits(const omc_layer_dev *L, const float *x, int T, int nrows, float *logits, int ldl, uint16_t *xh,
                  int *err, cudaStream_t s) {
    static int nsm = 0;
    if (!nsm) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return OMC_ECUDA;
    }
    auto blocks = [&](int g, int tt, int rr) {
        return (long long)((T + g * tt - 1) / (g * tt)) * ((nrows + g * rr - 1) / (g * rr));
    };
    const long long want = nsm;
    if (!g_force_tile && L->rt_w && r2_smem(L->D) <= 220 * 1024 && nrows <= L->rt_nrb * R2_RB) {
        static int attr2 = 0;
        const int smem = r2_smem(L->D);
        if (attr2 < smem) {
            if (cudaFuncSetAttribute(router_tile2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
                cudaSuccess)
                return OMC_ECUDA;
            attr2 = smem;
        }
        const dim3 g((T + R2_TB - 1) / R2_TB, (nrows + R2_RB - 1) / R2_RB);
        router_tile2_kernel<<<g, 256, smem, s>>>(x, T, L->D, L->rt_w, L->router_i8 ? L->router_s : nullptr, L->E,
                                                 nrows, logits, ldl, xh, err);
        return 0;
    }
    switch (g_force_tile) {
    case 1644: return launch_tile<16, 4, 4, 32>(L, x, T, nrows, logits, ldl, xh, err, s);
    case 1622: return launch_tile<16, 2, 2, 64>(L, x, T, nrows, logits, ldl, xh, err, s);
    case 1611: return launch_tile<16, 1, 1, 128>(L, x, T, nrows, logits, ldl, xh, err, s);
    case 811: return launch_tile<8, 1, 1, 128>(L, x, T, nrows, logits, ldl, xh, err, s);
    default: break;
    }
    // Measured on B200 (logits stage in us, every tile forced; OLMoE D=2048
    // E=64, Gemma D=2816 E=128, Qwen D=2048 E=256+1):
    //                 16x4x4  16x2x2  16x1x1  8x1x1  8x2x2  16x2x1
    //   OLMoE  T=512    137      55      31     35     51      45
    //   OLMoE  T=2048   137      56      84     88     60      63
    //   OLMoE  T=8192   145     158     227    301    172     192
    //   Gemma  T=512    176      72      53     74     58      53
    //   Gemma  T=2048   176     104     156    198    135     144
    //   Gemma  T=8192   292     326     592    768    411     484
    //   Qwen   T=2048   219     148     230    287    174     202
    // Later, with 64-thread blocks of two chains a thread (256 blocks at OLMoE T=512):
    //                 8x2x1   8x1x2  (16x1x1 in the same run)
    //   OLMoE  T=512   39.3    36.3    31.6
    //   OLMoE  T=2048  75.9    72.4    86.8   (16x2x2: 56.9)
    //   Gemma  T=512   51.8    49.8    49.9
    //   Qwen   T=2048 250.4   248.1   233.9   (16x2x2: 148.4)
    // so the bound is each warp's instruction chain (~4.3 cycles an instruction
    // at 2 warps a scheduler), not the SMs a grid covers.
    // (8x2x2, 16x2x1, 8x2x1 and 8x1x2 are not built: never the fastest.  Neither were a
    // lane-per-router-row kernel with broadcast token reads, nor 8-stage
    // staging; ncu on 16x1x1 at T=512: 2 warps per scheduler, ~6 issued
    // instructions per chain step, each waiting ~4.6 cycles on the add chain
    // and shared-memory loads.)
    // A 64 x 64 tile wins once its blocks make one nearly full wave (or
    // enough waves that the last one's tail is small); else 32 x 32 once
    // those fill the SMs; else one chain per thread.
    const long long b44 = blocks(16, 4, 4);
    if (10 * b44 >= 8 * want && (b44 <= want || 10 * b44 >= 16 * want))
        return launch_tile<16, 4, 4, 32>(L, x, T, nrows, logits, ldl, xh, err, s);
    if (10 * blocks(16, 2, 2) >= 8 * want) return launch_tile<16, 2, 2, 64>(L, x, T, nrows, logits, ldl, xh, err, s);
    return launch_tile<16, 1, 1, 128>(L, x, T, nrows, logits, ldl, xh, err, s);
}

}  // namespace

// Forces the router's logits tile for tests (g, tt, rr as one of 16x4x4,
// 16x2x2, 16x1x1, 8x1x1); 0,0,0 = automatic.
extern "C" int omc_debug_router_tile(int g, int tt, int rr) {
    const int code = g * 100 + tt * 10 + rr;
    if (code != 0 && code != 1644 && code != 1622 && code != 1611 && code != 811) return OMC_EINVAL;
    g_force_tile = code;
    omc_graphs_invalidate();
    return 0;
}

extern "C" int omc_launch_router(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                                 int32_t *topk_idx, float *topk_w, const omc_plan_args *plan, cudaStream_t s) {
    if (T <= 0) return 0;
    if (L->E > OMC_MAX_E || L->k > OMC_MAX_K || (L->D & 3)) return OMC_EINVAL;
    static int attr_small = 0;
    const int nrows = L->E + (L->has_shared ? 1 : 0);
    const int ldl = L->E + 1;
    const size_t small_smem = (size_t)(T + RS_ROWS) * (L->D + 4) * sizeof(float);
    if (!plan && T <= RS_TMAX && small_smem <= 200 * 1024) {
        if (!attr_small) {
            if (cudaFuncSetAttribute(router_logits_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024) != cudaSuccess)
                return OMC_ECUDA;
            attr_small = 1;
        }
        router_logits_small_kernel<<<(nrows + RS_ROWS - 1) / RS_ROWS, 256, small_smem, s>>>(
            x, T, L->D, L->router, L->router_i8 ? L->router_s : nullptr, L->E, L->sh_gate, nrows, ws->logits, ldl);
    } else if (omc_rf_eligible(L, T, ws)) {
        // the bounded router: exact chains only where the routing needs them
        const int rc = omc_launch_router_fast(L, x, T, ws, plan ? ws->xh : nullptr, s);
        if (rc) return rc;
    } else {
        // GEMMA's expert operand is not the router's input: prenorm writes it
        const int rc = launch_logits(L, x, T, nrows, ws->logits, ldl,
                                     (plan && L->family != OMC_FAMILY_GEMMA) ? ws->xh : nullptr, ws->err, s);
        if (rc) return rc;
    }
    omc_prof_mark(s, "router_logits");
    const int nv = (L->E + 31) / 32;
    const dim3 g2((T + SEL_WARPS - 1) / SEL_WARPS);
    omc_plan_args pa;
    if (plan) pa = *plan;
    else memset(&pa, 0, sizeof(pa));
#define SEL(NV)                                                                                                    \
    router_select_kernel<NV><<<g2, SEL_WARPS * 32, 0, s>>>(ws->logits, ldl, T, L->E, L->k, L->family, L->renorm, \
                                                         L->has_shared, L->g_pes, L->rbias, topk_idx, topk_w, ws->sg, \
                                                         pa,                                                      \
                                                         plan != nullptr,                                         \
                                                         ws->err)
    if (nv <= 1) SEL(1);
    else if (nv <= 2) SEL(2);
    else if (nv <= 4) SEL(4);
    else if (nv <= 8) SEL(8);
    else if (nv <= 16) SEL(16);
    else SEL(32);
#undef SEL
    omc_g_launches += 2;
    if (plan) {
        const int nfill = T * L->k + (L->has_shared ? T : 0);
        omc_plan_fill_rows<<<(nfill + 255) / 256, 256, 0, s>>>(pa, topk_idx, topk_w);
        omc_g_launches += 1;
    }
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

extern "C" int omc_launch_rt_blocks(const float *W, int row0, int nr, int D, float *dst, cudaStream_t s) {
    if (nr <= 0 || D % R2_KC) return OMC_EINVAL;
    const long long n4 = (long long)nr * (D / 4);
    rt_blocks_kernel<<<(int)((n4 + 255) / 256 < 4096 ? (n4 + 255) / 256 : 4096), 256, 0, s>>>(W, row0, nr, D, dst);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// Evaluates omc_expf_glibc on n inputs: lets the tests compare the device
// restatement with the host's glibc expf bit for bit.
namespace {
__global__ void expf_probe_kernel(const float *__restrict__ x, float *__restrict__ y, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        y[i] = omc_expf_glibc(x[i]);
}
}  // namespace

extern "C" int omc_launch_expf_probe(const float *x, float *y, long long n, cudaStream_t s) {
    expf_probe_kernel<<<1184, 256, 0, s>>>(x, y, n);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}
