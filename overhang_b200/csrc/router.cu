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
#include "omc_common.cuh"

namespace {

constexpr int RT_EXPERTS = 32;   // experts per block (one per lane)
constexpr int RT_WARPS = 4;      // warps per block
constexpr int RT_R = 2;          // tokens per thread: two independent chains fill the FADD latency
constexpr int RT_TOKENS = RT_WARPS * RT_R;
constexpr int RT_CHUNK = 128;    // K elements per pipeline stage
constexpr int RT_STAGES = 4;     // cp.async stages in flight
constexpr int RT_WROW = RT_CHUNK + 4;   // padded smem row (conflict-free float4 reads)
constexpr int RT_STAGE_FLOATS = RT_EXPERTS * RT_WROW + RT_TOKENS * RT_CHUNK;
constexpr size_t RT_SMEM = (size_t)RT_STAGES * RT_STAGE_FLOATS * sizeof(float);

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc, bool valid) {
    const uint32_t d = smem_u32(smem_dst);
    const int n = valid ? 16 : 0;       // 0 source bytes: the 16 bytes are zero-filled
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// logits[t][j], j < nrows: rows 0..E-1 are the router, row E (when
// has_shared) the shared-expert gate vector.  Each thread runs two
// (token, expert) chains side by side, so a warp issues every cycle while
// each chain keeps its own sequential order; the K dimension streams through
// a 4-stage cp.async ring so the chains never wait on memory.
__global__ void __launch_bounds__(RT_WARPS * 32) router_logits_kernel(const float *__restrict__ x, int T, int D,
                                                            const float *__restrict__ W,
                                                            const float *__restrict__ Ws, int E,
                                                            const float *__restrict__ sh_gate, int nrows,
                                                            float *__restrict__ logits, int ldl) {
    extern __shared__ __align__(16) float rsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row0 = blockIdx.y * RT_EXPERTS, t0 = blockIdx.x * RT_TOKENS;
    const int row = row0 + lane, ta = t0 + warp * RT_R;
    const int nchunk = (D + RT_CHUNK - 1) / RT_CHUNK;
    auto load = [&](int chunk) {
        float *st = rsm + (size_t)(chunk % RT_STAGES) * RT_STAGE_FLOATS;
        float *ws = st, *xs = st + RT_EXPERTS * RT_WROW;
        const int c0 = chunk * RT_CHUNK;
        for (int i = threadIdx.x; i < (RT_EXPERTS + RT_TOKENS) * (RT_CHUNK / 4); i += blockDim.x) {
            const int r = i / (RT_CHUNK / 4), c = (i % (RT_CHUNK / 4)) * 4;
            if (r < RT_EXPERTS) {
                const int gr = row0 + r;
                const bool ok = gr < nrows && c0 + c < D;
                const float *src = ok ? ((gr < E) ? W + (size_t)gr * D : sh_gate) + c0 + c : W;
                cp_async16(ws + r * RT_WROW + c, src, ok);
            } else {
                const int tr = r - RT_EXPERTS;
                const bool ok = t0 + tr < T && c0 + c < D;
                cp_async16(xs + tr * RT_CHUNK + c, ok ? x + (size_t)(t0 + tr) * D + c0 + c : x, ok);
            }
        }
    };
#pragma unroll
    for (int sidx = 0; sidx < RT_STAGES - 1; ++sidx) {
        if (sidx < nchunk) load(sidx);
        cp_async_commit();
    }
    float acc0 = 0.f, acc1 = 0.f;
    for (int chunk = 0; chunk < nchunk; ++chunk) {
        if (chunk + RT_STAGES - 1 < nchunk) load(chunk + RT_STAGES - 1);
        cp_async_commit();
        cp_async_wait<RT_STAGES - 1>();
        __syncthreads();
        const float *st = rsm + (size_t)(chunk % RT_STAGES) * RT_STAGE_FLOATS;
        const float *wrow = st + lane * RT_WROW;
        const float *xrow0 = st + RT_EXPERTS * RT_WROW + (warp * RT_R) * RT_CHUNK;
        const float *xrow1 = xrow0 + RT_CHUNK;
        const int clen = min(RT_CHUNK, D - chunk * RT_CHUNK);   // multiple of 4
        // per chain: acc = RN(acc + RN(x*w)) in index order (no contraction)
#pragma unroll 4
        for (int c = 0; c < clen; c += 4) {
            const float4 wv = *reinterpret_cast<const float4 *>(wrow + c);
            const float4 x0 = *reinterpret_cast<const float4 *>(xrow0 + c);
            const float4 x1 = *reinterpret_cast<const float4 *>(xrow1 + c);
            acc0 = __fadd_rn(acc0, __fmul_rn(x0.x, wv.x));
            acc1 = __fadd_rn(acc1, __fmul_rn(x1.x, wv.x));
            acc0 = __fadd_rn(acc0, __fmul_rn(x0.y, wv.y));
            acc1 = __fadd_rn(acc1, __fmul_rn(x1.y, wv.y));
            acc0 = __fadd_rn(acc0, __fmul_rn(x0.z, wv.z));
            acc1 = __fadd_rn(acc1, __fmul_rn(x1.z, wv.z));
            acc0 = __fadd_rn(acc0, __fmul_rn(x0.w, wv.w));
            acc1 = __fadd_rn(acc1, __fmul_rn(x1.w, wv.w));
        }
        __syncthreads();
    }
    if (row < nrows) {
        if (Ws && row < E) {                                // matmul_q: y = acc * scale
            acc0 = __fmul_rn(acc0, Ws[row]);
            acc1 = __fmul_rn(acc1, Ws[row]);
        }
        if (ta < T) logits[(size_t)ta * ldl + row] = acc0;
        if (ta + 1 < T) logits[(size_t)(ta + 1) * ldl + row] = acc1;
    }
}

// One warp per token: softmax, top-k, renorm, shared-gate sigmoid, expert counts.
template <int SEL_MAXV>   // ceil(E / 32) rounded up to a power of two
__global__ void __launch_bounds__(128) router_select_kernel(const float *__restrict__ logits, int ldl, int T,
                                                            int E, int K, int family, int renorm,
                                                            int has_shared, int32_t *__restrict__ topk_idx,
                                                            float *__restrict__ topk_w, float *__restrict__ sg,
                                                            int *__restrict__ counts, int *err) {
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int t = blockIdx.x * 4 + wib;
    if (t >= T) return;
    const float *lg = logits + (size_t)t * ldl;
    const int nv = (E + 31) / 32;
    float v[SEL_MAXV];
    // max, as `if (x[i] > m) m = x[i]` from m = -1e30f
    float m = -1e30f;
#pragma unroll
    for (int j = 0; j < SEL_MAXV; ++j) {
        const int i = lane + 32 * j;
        v[j] = (j < nv && i < E) ? lg[i] : -INFINITY;
        if (j < nv && i < E && v[j] > m) m = v[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // e_i = expf(x_i - m)
    bool tiny = false;
    const float exact_floor = ldexpf(1.0f, (32 - __clz(max(E - 1, 1))) - 30);   // 2^(ceil(log2 E) - 30)
#pragma unroll
    for (int j = 0; j < SEL_MAXV; ++j) {
        const int i = lane + 32 * j;
        if (j < nv && i < E) {
            v[j] = omc_expf_glibc(__fsub_rn(v[j], m));
            tiny |= v[j] < exact_floor;
        }
    }
    __syncwarp();
    float sf;   // the divisor as the reference uses it
    if (family == OMC_FAMILY_QWEN) {
        // double running sum.  When every term is >= 2^(ceil(log2 E) - 30) all
        // partial sums are exact in double, so any order gives the reference's
        // value; otherwise sum sequentially in index order like the CPU.
        double s;
        if (!__any_sync(0xffffffffu, tiny)) {
            s = 0.0;
#pragma unroll
            for (int j = 0; j < SEL_MAXV; ++j) {
                const int i = lane + 32 * j;
                if (j < nv && i < E) s = __dadd_rn(s, (double)v[j]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        } else {
            // every lane runs the same index-order sum; values arrive by shuffle
            s = 0.0;
#pragma unroll
            for (int j = 0; j < SEL_MAXV; ++j) {
                if (j >= nv) break;
                for (int l = 0; l < 32 && 32 * j + l < E; ++l) s = __dadd_rn(s, (double)__shfl_sync(0xffffffffu, v[j], l));
            }
        }
        sf = __double2float_rn(s);
    } else {
        // float running sum in index order (engines/olmoe.c:172); every lane
        // runs the same chain, values arrive by shuffle
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < SEL_MAXV; ++j) {
            if (j >= nv) break;
            for (int l = 0; l < 32 && 32 * j + l < E; ++l) s = __fadd_rn(s, __shfl_sync(0xffffffffu, v[j], l));
        }
        sf = s;
    }
#pragma unroll
    for (int j = 0; j < SEL_MAXV; ++j) v[j] = (j < nv && lane + 32 * j < E) ? __fdiv_rn(v[j], sf) : -INFINITY;
    // top-k: largest probability, ties to the lowest id
    uint32_t taken = 0;
    float val[OMC_MAX_K];
    int idx[OMC_MAX_K];
    for (int kk = 0; kk < K; ++kk) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < SEL_MAXV; ++j) {
            const int i = lane + 32 * j;
            if (j < nv && i < E && !((taken >> j) & 1u) && v[j] > bv) { bv = v[j]; bi = i; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        val[kk] = bv;
        idx[kk] = bi;
    }
    if (lane == 0) {
        if (renorm || family == OMC_FAMILY_QWEN) {
            float sm = 0.f;
            for (int kk = 0; kk < K; ++kk) sm = __fadd_rn(sm, val[kk]);
            for (int kk = 0; kk < K; ++kk) val[kk] = __fdiv_rn(val[kk], sm);
        }
        for (int kk = 0; kk < K; ++kk) {
            if (idx[kk] < 0 || idx[kk] >= E) { omc_dev_error(err, OMC_DEVERR_ROUTE, OMC_SITE_ROUTER, t); continue; }
            topk_idx[(size_t)t * K + kk] = idx[kk];
            topk_w[(size_t)t * K + kk] = val[kk];
            atomicAdd(&counts[idx[kk]], 1);
        }
        if (has_shared) {
            const float z = lg[E];
            sg[t] = __fdiv_rn(1.f, __fadd_rn(1.f, omc_expf_glibc(-z)));   // engines/qwen.c:158,461
        }
    }
}

}  // namespace

extern "C" int omc_launch_router(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                                 int32_t *topk_idx, float *topk_w, cudaStream_t s) {
    if (T <= 0) return 0;
    if (L->E > OMC_MAX_E || L->k > OMC_MAX_K || (L->D & 3)) return OMC_EINVAL;
    static int attr_done = 0;
    if (!attr_done) {
        if (cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RT_SMEM) !=
            cudaSuccess)
            return OMC_ECUDA;
        attr_done = 1;
    }
    const int nrows = L->E + (L->has_shared ? 1 : 0);
    const int ldl = L->E + 1;
    dim3 g1((T + RT_TOKENS - 1) / RT_TOKENS, (nrows + RT_EXPERTS - 1) / RT_EXPERTS);
    router_logits_kernel<<<g1, RT_WARPS * 32, RT_SMEM, s>>>(x, T, L->D, L->router, L->router_i8 ? L->router_s : nullptr, L->E,
                                                  L->sh_gate, nrows, ws->logits, ldl);
    omc_prof_mark(s, "router_logits");
    const int nv = (L->E + 31) / 32;
    const dim3 g2((T + 3) / 4);
#define SEL(NV) router_select_kernel<NV><<<g2, 128, 0, s>>>(ws->logits, ldl, T, L->E, L->k, L->family, L->renorm, \
                                                          L->has_shared, topk_idx, topk_w, ws->sg, ws->counts, ws->err)
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
