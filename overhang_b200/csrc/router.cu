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

// ---- select -----------------------------------------------------------------
// One warp per token: softmax, top-k, renorm, shared-gate sigmoid.  Lane l
// holds logits l, l+32, ...; order-dependent sums run from a shared-memory
// copy so that their dependent chain is the add latency alone.  With a plan
// (tensor-core forwards) the block that finishes last builds the dispatch
// plan from every token's routing: no per-expert atomics in global memory.
constexpr int SEL_WARPS = 8;

template <int SEL_MAXV>   // ceil(E / 32) rounded up to a power of two
__device__ __forceinline__ void select_token(const float *__restrict__ logits, int ldl, int t, int E, int K,
                                             int family, int renorm, int has_shared,
                                             int32_t *__restrict__ topk_idx, float *__restrict__ topk_w,
                                             float *__restrict__ sg, int *err, float *es) {
    const int lane = threadIdx.x & 31;
    const float *lg = logits + (size_t)t * ldl;
    float v[SEL_MAXV];
    // max, as `if (x[i] > m) m = x[i]` from m = -1e30f
    float m = -1e30f;
#pragma unroll
    for (int j = 0; j < SEL_MAXV; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < E ? lg[i] : -INFINITY;
        if (i < E && v[j] > m) m = v[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // e_i = expf(x_i - m)
    bool tiny = false;
    const float exact_floor = ldexpf(1.0f, (32 - __clz(max(E - 1, 1))) - 30);   // 2^(ceil(log2 E) - 30)
#pragma unroll
    for (int j = 0; j < SEL_MAXV; ++j) {
        const int i = lane + 32 * j;
        if (i < E) {
            v[j] = omc_expf_glibc(__fsub_rn(v[j], m));
            tiny |= v[j] < exact_floor;
            es[i] = v[j];
        }
    }
    __syncwarp();
    float sf;   // the divisor as the reference uses it
    if (family == OMC_FAMILY_QWEN && !__any_sync(0xffffffffu, tiny)) {
        // double running sum.  When every term is >= 2^(ceil(log2 E) - 30) all
        // partial sums are exact in double, so any order gives the
        // reference's value: a butterfly.
        double s = 0.0;
#pragma unroll
        for (int j = 0; j < SEL_MAXV; ++j)
            if (lane + 32 * j < E) s = __dadd_rn(s, (double)v[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        sf = __double2float_rn(s);
    } else if (family == OMC_FAMILY_QWEN) {
        // otherwise the index-order double sum of engines/qwen.c:163, every lane
        double s = 0.0;
        int i = 0;
        for (; i + 4 <= E; i += 4) {
            const float4 q = *reinterpret_cast<const float4 *>(es + i);
            s = __dadd_rn(s, (double)q.x);
            s = __dadd_rn(s, (double)q.y);
            s = __dadd_rn(s, (double)q.z);
            s = __dadd_rn(s, (double)q.w);
        }
        for (; i < E; ++i) s = __dadd_rn(s, (double)es[i]);
        sf = __double2float_rn(s);
    } else {
        // float running sum in index order (engines/olmoe.c:172), every lane
        float s = 0.f;
        int i = 0;
#pragma unroll 4
        for (; i + 4 <= E; i += 4) {
            const float4 q = *reinterpret_cast<const float4 *>(es + i);
            s = __fadd_rn(s, q.x);
            s = __fadd_rn(s, q.y);
            s = __fadd_rn(s, q.z);
            s = __fadd_rn(s, q.w);
        }
        for (; i < E; ++i) s = __fadd_rn(s, es[i]);
        sf = s;
    }
    // probabilities as order keys: p >= 0, so bits(p) + 1 orders like p and
    // 0 marks "not available" (outside E, NaN, or already taken).
    uint32_t key[SEL_MAXV];
    float pv[SEL_MAXV];
#pragma unroll
    for (int j = 0; j < SEL_MAXV; ++j) {
        const int i = lane + 32 * j;
        pv[j] = i < E ? __fdiv_rn(v[j], sf) : 0.f;
        key[j] = (i < E && pv[j] == pv[j]) ? __float_as_uint(pv[j]) + 1u : 0u;
    }
    // top-k: engines/olmoe.c:355-362 -- largest p, ties to the lowest id
    int my_idx = -1;
    float my_val = 0.f;
    for (int kk = 0; kk < K; ++kk) {
        uint32_t bk = 0;
        int bj = 0;
#pragma unroll
        for (int j = 0; j < SEL_MAXV; ++j)
            if (key[j] > bk) { bk = key[j]; bj = j; }      // strict: lowest j (= lowest id) of this lane
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, bk);
        const uint32_t cand = (bk == kmax && kmax != 0u) ? (uint32_t)(lane + 32 * bj) : 0xffffffffu;
        const uint32_t best = __reduce_min_sync(0xffffffffu, cand);
        if (kmax != 0u && (int)(best & 31) == lane) {
#pragma unroll
            for (int j = 0; j < SEL_MAXV; ++j)
                if (j == (int)(best >> 5)) key[j] = 0u;
        }
        if (lane == kk) {
            my_idx = kmax != 0u ? (int)best : -1;
            my_val = __uint_as_float(kmax - 1u);
        }
    }
    // renorm: float sum in selection order, then divide (engines/olmoe.c:363)
    if (renorm || family == OMC_FAMILY_QWEN) {
        float sm = 0.f;
        for (int kk = 0; kk < K; ++kk) sm = __fadd_rn(sm, __shfl_sync(0xffffffffu, my_val, kk));
        my_val = __fdiv_rn(my_val, sm);
    }
    if (lane < K) {
        if (my_idx < 0 || my_idx >= E) omc_dev_error(err, OMC_DEVERR_ROUTE, OMC_SITE_ROUTER, t);
        topk_idx[(size_t)t * K + lane] = my_idx;
        topk_w[(size_t)t * K + lane] = my_val;
    }
    if (has_shared && lane == 0) {
        const float z = lg[E];
        sg[t] = __fdiv_rn(1.f, __fadd_rn(1.f, omc_expf_glibc(-z)));   // engines/qwen.c:158,461
    }
}

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
    static int attr_done = 0;
    if (!attr_done) {
        if (cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RL_SMEM) !=
            cudaSuccess)
            return OMC_ECUDA;
        attr_done = 1;
    }
    const int nrows = L->E + (L->has_shared ? 1 : 0);
    const int ldl = L->E + 1;
    const dim3 g1((T + RL_TOK - 1) / RL_TOK, (nrows + RL_ROWS - 1) / RL_ROWS);
    router_logits_kernel<<<g1, RL_THREADS, RL_SMEM, s>>>(x, T, L->D, L->router, L->router_i8 ? L->router_s : nullptr,
                                                         L->E, L->sh_gate, nrows, ws->logits, ldl,
                                                         plan ? ws->xh : nullptr, ws->err);
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
