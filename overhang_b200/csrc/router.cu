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
// Block = 8 tokens x 32 router rows, 4 warps.  Lane l of warp w owns token
// (l & 7) and rows 8w + 2(l >> 3) + {0, 1}: two chains per thread.  Per four
// K elements a warp reads one 16-byte x vector (8 distinct tokens, one
// wavefront) and two 16-byte row vectors (4 distinct rows each, one wavefront
// each), so shared-memory traffic is 3 wavefronts per 64 chains instead of 5
// per 32 with one row per lane.  K streams through a 4-stage cp.async ring.
constexpr int RL_TOK = 8;                   // tokens per block
constexpr int RL_ROWS = 32;                 // router rows per block
constexpr int RL_THREADS = 128;
constexpr int RL_CH = 128;                  // K elements per stage
constexpr int RL_ST = 4;                    // stages
constexpr int RL_LD = RL_CH + 4;            // padded row: 8 consecutive rows hit 8 distinct bank quads
constexpr int RL_STAGE = (RL_TOK + RL_ROWS) * RL_LD;            // floats per stage
constexpr size_t RL_SMEM = (size_t)RL_ST * RL_STAGE * sizeof(float);   // 84,480 B

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc, bool valid) {
    const uint32_t d = smem_u32(smem_dst);
    const int n = valid ? 16 : 0;       // 0 source bytes: the 16 bytes are zero-filled
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// (a0, a1) = (RN(a0 + b0), RN(a1 + b1)): two independent IEEE single adds in
// one packed instruction; each lane of the pair rounds exactly as add.rn.f32.
__device__ __forceinline__ void add2_rn(float &a0, float &a1, float b0, float b1) {
    asm("{\n\t.reg .b64 ra, rb;\n\t"
        "mov.b64 ra, {%0, %1};\n\t"
        "mov.b64 rb, {%2, %3};\n\t"
        "add.rn.f32x2 ra, ra, rb;\n\t"
        "mov.b64 {%0, %1}, ra;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(b0), "f"(b1));
}

// logits[t][j], j < nrows: rows 0..E-1 are the router, row E (when
// has_shared) the shared-expert gate vector.  Every (token, row) value is the
// reference's chain acc = RN(acc + RN(x[i] * w[i])), i ascending.
__global__ void __launch_bounds__(RL_THREADS) router_logits_kernel(const float *__restrict__ x, int T, int D,
                                                                    const float *__restrict__ W,
                                                                    const float *__restrict__ Ws, int E,
                                                                    const float *__restrict__ sh_gate, int nrows,
                                                                    float *__restrict__ logits, int ldl,
                                                                    uint16_t *__restrict__ xh, int *err) {
    (void)err;
    extern __shared__ __align__(16) float rsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t0 = blockIdx.x * RL_TOK, row0 = blockIdx.y * RL_ROWS;
    const int tok = lane & 7, rl = warp * 8 + (lane >> 3) * 2;   // rows rl, rl+1 of the block
    const int nch = (D + RL_CH - 1) / RL_CH;
    auto load = [&](int ch) {
        float *st = rsm + (size_t)(ch % RL_ST) * RL_STAGE;
        const int c0 = ch * RL_CH;
        // one warp copies one 512-byte row segment per pass (coalesced)
        for (int i = threadIdx.x; i < (RL_TOK + RL_ROWS) * (RL_CH / 4); i += RL_THREADS) {
            const int r = i / (RL_CH / 4), c = (i % (RL_CH / 4)) * 4;
            const float *src;
            bool ok;
            if (r < RL_TOK) {
                ok = t0 + r < T && c0 + c < D;
                src = x + (size_t)(t0 + r) * D + c0 + c;
            } else {
                const int gr = row0 + r - RL_TOK;
                ok = gr < nrows && c0 + c < D;
                src = (gr < E ? W + (size_t)gr * D : sh_gate) + c0 + c;
            }
            cp_async16(st + r * RL_LD + c, ok ? src : x, ok);
        }
    };
#pragma unroll
    for (int s = 0; s < RL_ST - 1; ++s) {
        if (s < nch) load(s);
        cp_async_commit();
    }
    float acc0 = 0.f, acc1 = 0.f;
    for (int ch = 0; ch < nch; ++ch) {
        cp_async_wait<RL_ST - 2>();   // chunk ch has landed (this thread's copies)
        __syncthreads();              // ... everyone's; and chunk ch-1's stage is free
        if (ch + RL_ST - 1 < nch) load(ch + RL_ST - 1);
        cp_async_commit();
        const float *st = rsm + (size_t)(ch % RL_ST) * RL_STAGE;
        if (xh && blockIdx.y == 0) {
            // the f16 token operand of the expert GEMMs (row t of xh = x[t] rounded
            // to f16, saturated): written from the staged chunk by the first
            // column of blocks, 8 values per thread
            const int r = threadIdx.x >> 4, c = (threadIdx.x & 15) * 8, k = ch * RL_CH + c;
            if (t0 + r < T && k < D) {
                const float *v = st + r * RL_LD + c;
                uint4 o;
                o.x = f32x2_to_f16x2_sat(v[0], v[1]);
                o.y = f32x2_to_f16x2_sat(v[2], v[3]);
                o.z = f32x2_to_f16x2_sat(v[4], v[5]);
                o.w = f32x2_to_f16x2_sat(v[6], v[7]);
                *reinterpret_cast<uint4 *>(xh + (size_t)(t0 + r) * D + k) = o;
            }
        }
        const float *xr = st + tok * RL_LD;
        const float *w0 = st + (RL_TOK + rl) * RL_LD, *w1 = w0 + RL_LD;
        const int clen = min(RL_CH, D - ch * RL_CH);     // a multiple of 4
#pragma unroll 8
        for (int c = 0; c < clen; c += 4) {
            const float4 xv = *reinterpret_cast<const float4 *>(xr + c);
            const float4 a = *reinterpret_cast<const float4 *>(w0 + c);
            const float4 b = *reinterpret_cast<const float4 *>(w1 + c);
            add2_rn(acc0, acc1, __fmul_rn(xv.x, a.x), __fmul_rn(xv.x, b.x));
            add2_rn(acc0, acc1, __fmul_rn(xv.y, a.y), __fmul_rn(xv.y, b.y));
            add2_rn(acc0, acc1, __fmul_rn(xv.z, a.z), __fmul_rn(xv.z, b.z));
            add2_rn(acc0, acc1, __fmul_rn(xv.w, a.w), __fmul_rn(xv.w, b.w));
        }
    }
    const int t = t0 + tok, r0 = row0 + rl;
    if (t < T) {
        if (r0 < nrows) logits[(size_t)t * ldl + r0] = (Ws && r0 < E) ? __fmul_rn(acc0, Ws[r0]) : acc0;
        if (r0 + 1 < nrows) logits[(size_t)t * ldl + r0 + 1] = (Ws && r0 + 1 < E) ? __fmul_rn(acc1, Ws[r0 + 1]) : acc1;
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
                                                                       int has_shared, int32_t *__restrict__ topk_idx,
                                                                       float *__restrict__ topk_w, float *__restrict__ sg,
                                                                       omc_plan_args plan, int do_plan, int *err) {
    // per-warp softmax rows, reused by the plan in the last block
    __shared__ __align__(16) float sbuf[SEL_SMEM_FLOATS(SEL_MAXV)];
    __shared__ int s_last;
    const int wib = threadIdx.x >> 5;
    const int t = blockIdx.x * SEL_WARPS + wib;
    if (t < T)
        select_token<SEL_MAXV>(logits, ldl, t, E, K, family, renorm, has_shared, topk_idx, topk_w, sg, err,
                               sbuf + wib * SEL_MAXV * 32);
    if (!do_plan) return;
    // last-block handoff: every block's routing is visible to the block that counts last
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(plan.done, 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    omc_plan_block(plan, topk_idx, topk_w, err, reinterpret_cast<int *>(sbuf));
}

}  // namespace

extern "C" int omc_launch_router(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                                 int32_t *topk_idx, float *topk_w, const omc_plan_args *plan, cudaStream_t s) {
    if (T <= 0) return 0;
    if (L->E > OMC_MAX_E || L->k > OMC_MAX_K || (L->D & 3)) return OMC_EINVAL;
    static int attr_done = 0, attr_small = 0;
    if (!attr_done) {
        if (cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RL_SMEM) !=
            cudaSuccess)
            return OMC_ECUDA;
        attr_done = 1;
    }
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
    } else {
        const dim3 g1((T + RL_TOK - 1) / RL_TOK, (nrows + RL_ROWS - 1) / RL_ROWS);
        router_logits_kernel<<<g1, RL_THREADS, RL_SMEM, s>>>(x, T, L->D, L->router, L->router_i8 ? L->router_s : nullptr,
                                                             L->E, L->sh_gate, nrows, ws->logits, ldl,
                                                             plan ? ws->xh : nullptr, ws->err);
    }
    omc_prof_mark(s, "router_logits");
    const int nv = (L->E + 31) / 32;
    const dim3 g2((T + SEL_WARPS - 1) / SEL_WARPS);
    omc_plan_args pa;
    if (plan) pa = *plan;
    else memset(&pa, 0, sizeof(pa));
#define SEL(NV)                                                                                                    \
    router_select_kernel<NV><<<g2, SEL_WARPS * 32, 0, s>>>(ws->logits, ldl, T, L->E, L->k, L->family, L->renorm, \
                                                         L->has_shared, topk_idx, topk_w, ws->sg, pa, plan != nullptr, \
                                                         ws->err)
    if (nv <= 1) SEL(1);
    else if (nv <= 2) SEL(2);
    else if (nv <= 4) SEL(4);
    else if (nv <= 8) SEL(8);
    else if (nv <= 16) SEL(16);
    else SEL(32);
#undef SEL
    omc_g_launches += 2;
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
