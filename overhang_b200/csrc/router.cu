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
constexpr int RT_TOKENS = 8;     // tokens per block (one per warp)
constexpr int RT_CHUNK = 128;    // K elements staged per step

// logits[t][j], j < nrows: rows 0..E-1 are the router, row E (when
// has_shared) the shared-expert gate vector.
__global__ void __launch_bounds__(256) router_logits_kernel(const float *__restrict__ x, int T, int D,
                                                            const float *__restrict__ W,
                                                            const float *__restrict__ Ws, int E,
                                                            const float *__restrict__ sh_gate, int nrows,
                                                            float *__restrict__ logits, int ldl) {
    __shared__ __align__(16) float w_s[RT_EXPERTS][RT_CHUNK + 4];
    __shared__ __align__(16) float x_s[RT_TOKENS][RT_CHUNK];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row0 = blockIdx.y * RT_EXPERTS, t0 = blockIdx.x * RT_TOKENS;
    const int row = row0 + lane, t = t0 + warp;
    float acc = 0.f;
    for (int c0 = 0; c0 < D; c0 += RT_CHUNK) {
        const int clen = min(RT_CHUNK, D - c0);      // D is a multiple of 4
        // stage W rows [row0, row0+32) and x rows [t0, t0+8) for columns [c0, c0+clen)
        for (int i = threadIdx.x; i < RT_EXPERTS * (RT_CHUNK / 4); i += blockDim.x) {
            const int r = i / (RT_CHUNK / 4), c = (i % (RT_CHUNK / 4)) * 4;
            const int gr = row0 + r;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c < clen && gr < nrows) {
                const float *src = (gr < E) ? (W + (size_t)gr * D) : sh_gate;
                v = *reinterpret_cast<const float4 *>(src + c0 + c);
            }
            *reinterpret_cast<float4 *>(&w_s[r][c]) = v;
        }
        for (int i = threadIdx.x; i < RT_TOKENS * (RT_CHUNK / 4); i += blockDim.x) {
            const int r = i / (RT_CHUNK / 4), c = (i % (RT_CHUNK / 4)) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c < clen && t0 + r < T) v = *reinterpret_cast<const float4 *>(x + (size_t)(t0 + r) * D + c0 + c);
            *reinterpret_cast<float4 *>(&x_s[r][c]) = v;
        }
        __syncthreads();
        // one dependent chain per thread: acc = RN(acc + RN(x*w))
        for (int c = 0; c < clen; c += 4) {
            const float4 xv = *reinterpret_cast<const float4 *>(&x_s[warp][c]);
            const float4 wv = *reinterpret_cast<const float4 *>(&w_s[lane][c]);
            acc = __fadd_rn(acc, __fmul_rn(xv.x, wv.x));
            acc = __fadd_rn(acc, __fmul_rn(xv.y, wv.y));
            acc = __fadd_rn(acc, __fmul_rn(xv.z, wv.z));
            acc = __fadd_rn(acc, __fmul_rn(xv.w, wv.w));
        }
        __syncthreads();
    }
    if (t < T && row < nrows) {
        if (Ws && row < E) acc = __fmul_rn(acc, Ws[row]);   // matmul_q: y = acc * scale
        logits[(size_t)t * ldl + row] = acc;
    }
}

// One warp per token: softmax, top-k, renorm, shared-gate sigmoid, expert counts.
constexpr int SEL_MAXV = OMC_MAX_E / 32;

__global__ void __launch_bounds__(128) router_select_kernel(const float *__restrict__ logits, int ldl, int T,
                                                            int E, int K, int family, int renorm,
                                                            int has_shared, int32_t *__restrict__ topk_idx,
                                                            float *__restrict__ topk_w, float *__restrict__ sg,
                                                            int *__restrict__ counts, int *err) {
    __shared__ float e_s[4][OMC_MAX_E];
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
    float *es = e_s[wib];
    bool tiny = false;
    const float exact_floor = ldexpf(1.0f, (32 - __clz(max(E - 1, 1))) - 30);   // 2^(ceil(log2 E) - 30)
#pragma unroll
    for (int j = 0; j < SEL_MAXV; ++j) {
        const int i = lane + 32 * j;
        if (j < nv && i < E) {
            v[j] = omc_expf_glibc(__fsub_rn(v[j], m));
            es[i] = v[j];
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
            s = 0.0;
            if (lane == 0)
                for (int i = 0; i < E; ++i) s = __dadd_rn(s, (double)es[i]);
            s = __shfl_sync(0xffffffffu, s, 0);
        }
        sf = __double2float_rn(s);
    } else {
        // float running sum in index order (engines/olmoe.c:172)
        float s = 0.f;
        if (lane == 0)
            for (int i = 0; i < E; ++i) s = __fadd_rn(s, es[i]);
        sf = __shfl_sync(0xffffffffu, s, 0);
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
    const int nrows = L->E + (L->has_shared ? 1 : 0);
    const int ldl = L->E + 1;
    dim3 g1((T + RT_TOKENS - 1) / RT_TOKENS, (nrows + RT_EXPERTS - 1) / RT_EXPERTS);
    router_logits_kernel<<<g1, 256, 0, s>>>(x, T, L->D, L->router, L->router_i8 ? L->router_s : nullptr, L->E,
                                            L->sh_gate, nrows, ws->logits, ldl);
    router_select_kernel<<<(T + 3) / 4, 128, 0, s>>>(ws->logits, ldl, T, L->E, L->k, L->family, L->renorm,
                                                     L->has_shared, topk_idx, topk_w, ws->sg, ws->counts,
                                                     ws->err);
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
