// ffn_gemv.cu -- expert SwiGLU for few tokens per expert (decode), CUDA cores.
//
// Phase 1 (gemv_gateup_kernel): for every routed slot (token t, choice kk)
// and, for QWEN, every token's shared-expert slot, one block of 128 threads
// computes 128 rows of gate and up over the full hidden size: thread r owns
// row r of the tile and reads its 16-byte int8 chunks straight from the tiled
// slab (a warp reads 512 contiguous bytes per load), dequantises in
// registers (exact), and accumulates in fp32 against x held in shared memory.
// Then h = act(gs*g) * (us*u) as the reference does (engines/olmoe.c:391-393,
// engines/qwen.c:484-485).
//
// Phase 2 (gemv_down_combine_kernel): for every token and 128 output rows,
// each thread computes its row's down projection for all k chosen experts
// (and the shared expert) and combines them in the reference's order, in
// registers: out = [sigmoid gate * shared] + sum_kk w_kk * y_kk
// (engines/olmoe.c:394-397, engines/qwen.c:459-462,486-492).  The combine
// is deterministic and needs no atomics.
#include "omc_common.cuh"

namespace {

__device__ __forceinline__ int4 ldg_nc_v4(const void *p) {
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// acc += sum_j x[j] * q[j] over one 16-byte chunk (16 int8)
__device__ __forceinline__ float dot16(float acc, int4 w, const float *x) {
    float f[16];
    i8x4_to_f32x4((uint32_t)w.x, f[0], f[1], f[2], f[3]);
    i8x4_to_f32x4((uint32_t)w.y, f[4], f[5], f[6], f[7]);
    i8x4_to_f32x4((uint32_t)w.z, f[8], f[9], f[10], f[11]);
    i8x4_to_f32x4((uint32_t)w.w, f[12], f[13], f[14], f[15]);
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float4 xv = x4[j];
        acc = fmaf(xv.x, f[4 * j + 0], acc);
        acc = fmaf(xv.y, f[4 * j + 1], acc);
        acc = fmaf(xv.z, f[4 * j + 2], acc);
        acc = fmaf(xv.w, f[4 * j + 3], acc);
    }
    return acc;
}

// SwiGLU in the family's arithmetic form.
__device__ __forceinline__ float swiglu(int family, float g, float u) {
    const float e = omc_expf_glibc(-g);
    if (family == OMC_FAMILY_QWEN) return __fmul_rn(__fmul_rn(g, __fdiv_rn(1.f, __fadd_rn(1.f, e))), u);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, e)), u);
}

__global__ void __launch_bounds__(128) gemv_gateup_kernel(omc_layer_dev L, const float *__restrict__ x, int T,
                                                          const int32_t *__restrict__ topk_idx,
                                                          float *__restrict__ hbuf, int ldh, int *err) {
    extern __shared__ __align__(16) float xs[];
    const int s = blockIdx.x, ot = blockIdx.y, r = threadIdx.x;
    const int nrouted = T * L.k;
    int t, e, Iw;
    if (s < nrouted) {
        t = s / L.k;
        e = topk_idx[s];
        Iw = L.I;
        if (e < 0 || e >= L.E) {
            if (r == 0) omc_dev_error(err, OMC_DEVERR_ROUTE, OMC_SITE_GEMV, s);
            return;
        }
    } else {
        t = s - nrouted;
        e = L.E;
        Iw = L.Is;
    }
    if (ot * OMC_TM >= Iw) return;
    for (int i = r * 4; i < L.D_pad; i += 128 * 4) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < L.D) v = *reinterpret_cast<const float4 *>(x + (size_t)t * L.D + i);
        *reinterpret_cast<float4 *>(xs + i) = v;
    }
    __syncthreads();
    const omc_expert_ptrs P = L.experts[e];
    const int nkb = L.D_pad / OMC_KB;
    const size_t tile = (size_t)ot * nkb * OMC_PAIR_STRIDE + (size_t)r * 16;   // pair ot: g member 0, u member 1
    const int8_t *gp = P.g + tile, *up = P.u + tile;
    float ag = 0.f, au = 0.f;
#pragma unroll 2
    for (int kb = 0; kb < nkb; ++kb) {
        int4 wg[4], wu[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            wg[c] = ldg_nc_v4(gp + (size_t)kb * OMC_PAIR_STRIDE + c * 2048);
            wu[c] = ldg_nc_v4(up + (size_t)kb * OMC_PAIR_STRIDE + c * 2048);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            ag = dot16(ag, wg[c], xs + kb * OMC_KB + c * 16);
            au = dot16(au, wu[c], xs + kb * OMC_KB + c * 16);
        }
    }
    const int row = ot * OMC_TM + r;
    float h = 0.f;
    if (row < Iw) {
        const float g = __fmul_rn(ag, P.gs[row]);
        const float u = __fmul_rn(au, P.us[row]);
        h = swiglu(L.family, g, u);
    }
    hbuf[(size_t)s * ldh + row] = h;
}

__device__ __forceinline__ float down_dot(const int8_t *dp, const float *h, int nkb) {
    float a = 0.f;
#pragma unroll 2
    for (int kb = 0; kb < nkb; ++kb) {
        int4 w[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) w[c] = ldg_nc_v4(dp + (size_t)kb * OMC_PAIR_STRIDE + c * 2048);
#pragma unroll
        for (int c = 0; c < 4; ++c) a = dot16(a, w[c], h + kb * OMC_KB + c * 16);
    }
    return a;
}

__global__ void __launch_bounds__(128) gemv_down_combine_kernel(omc_layer_dev L, int T,
                                                                const int32_t *__restrict__ topk_idx,
                                                                const float *__restrict__ topk_w,
                                                                const float *__restrict__ sg,
                                                                const float *__restrict__ hbuf, int ldh,
                                                                float *__restrict__ out, int *err) {
    extern __shared__ __align__(16) float hs[];   // [k + 1][ldh]
    const int t = blockIdx.x, dt = blockIdx.y, r = threadIdx.x;
    const int K = L.k, nslots = K + (L.has_shared ? 1 : 0);
    for (int j = 0; j < nslots; ++j) {
        const size_t src = (j < K) ? (size_t)(t * K + j) : (size_t)(T * K + t);
        for (int i = r * 4; i < ldh; i += 128 * 4)
            *reinterpret_cast<float4 *>(hs + (size_t)j * ldh + i) =
                *reinterpret_cast<const float4 *>(hbuf + src * ldh + i);
    }
    __syncthreads();
    const int d = dt * OMC_TM + r;
    float acc = 0.f;
    if (L.has_shared) {
        const omc_expert_ptrs P = L.experts[L.E];
        const int nkb_s = L.Is_pad / OMC_KB;
        const int8_t *dp = P.d + omc_dblk(dt, 0, nkb_s) + (size_t)r * 16;
        const float y = __fmul_rn(down_dot(dp, hs + (size_t)K * ldh, nkb_s), P.ds[d]);
        acc = __fmul_rn(y, sg[t]);                       // out = shared; out *= sigmoid(gate)
    }
    const int nkb = L.I_pad / OMC_KB;
    for (int kk = 0; kk < K; ++kk) {
        const int e = topk_idx[(size_t)t * K + kk];
        if (e < 0 || e >= L.E) {
            if (r == 0) omc_dev_error(err, OMC_DEVERR_ROUTE, OMC_SITE_GEMV, t);
            return;
        }
        const omc_expert_ptrs P = L.experts[e];
        const int8_t *dp = P.d + omc_dblk(dt, 0, nkb) + (size_t)r * 16;
        const float y = __fmul_rn(down_dot(dp, hs + (size_t)kk * ldh, nkb), P.ds[d]);
        acc = __fadd_rn(acc, __fmul_rn(topk_w[(size_t)t * K + kk], y));   // out += w * y
    }
    if (d < L.D) out[(size_t)t * L.D + d] = acc;
}

}  // namespace

extern "C" int omc_launch_gemv_ffn(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                                   const int32_t *topk_idx, const float *topk_w, float *out, cudaStream_t s) {
    if (T <= 0) return 0;
    const int Imax_rows = L->has_shared && L->Is_rows > L->I_rows ? L->Is_rows : L->I_rows;
    const int ldh = Imax_rows;
    const int nslots = T * L->k + (L->has_shared ? T : 0);
    const size_t smem1 = (size_t)L->D_pad * sizeof(float);
    const size_t smem2 = (size_t)(L->k + 1) * ldh * sizeof(float);
    if (smem1 > 200 * 1024 || smem2 > 200 * 1024) return OMC_EUNSUPPORTED;
    static int attr_done = 0;
    if (!attr_done) {
        cudaFuncSetAttribute(gemv_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(gemv_down_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_done = 1;
    }
    dim3 g1(nslots, Imax_rows / OMC_TM);
    gemv_gateup_kernel<<<g1, 128, smem1, s>>>(*L, x, T, topk_idx, ws->hbuf, ldh, ws->err);
    omc_prof_mark(s, "gemv_gateup");
    dim3 g2(T, L->D_rows / OMC_TM);
    gemv_down_combine_kernel<<<g2, 128, smem2, s>>>(*L, T, topk_idx, topk_w, ws->sg, ws->hbuf, ldh, out, ws->err);
    omc_prof_mark(s, "gemv_down_combine");
    omc_g_launches += 2;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}
