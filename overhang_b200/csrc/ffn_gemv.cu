// ffn_gemv.cu -- expert SwiGLU for few tokens per expert (decode), CUDA cores.
//
// Phase 1 (gemv_gateup_kernel): for every routed slot (token t, choice kk)
// and, for QWEN, every token's shared-expert slot, one block of 8 warps
// computes 32 rows of gate and up over the full hidden size: lane l owns row
// l of the group (a warp reads 32 rows' 16-byte chunk, 512 contiguous bytes
// of the tiled slab), the 8 warps split the K blocks and their partial sums
// are added in warp order.  int8 is dequantised exactly in registers and
// accumulated in fp32 against x in shared memory.  Then h = act(gs*g) *
// (us*u) as the reference does (engines/olmoe.c:391-393,
// engines/qwen.c:484-485).  At T=1 this is 256 blocks (OLMoE) instead of one
// 128-row block per slot and tile: enough loads in flight to stream HBM.
//
// Phase 2 (gemv_down_combine_kernel): for every token and 32 output rows,
// warp j computes slot j's down projection (one row per lane), then the
// slots are combined in the reference's order: out = [sigmoid gate *
// shared] + sum_kk w_kk * y_kk (engines/olmoe.c:394-397,
// engines/qwen.c:459-462,486-492).  The combine is deterministic and needs
// no atomics.
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

// SwiGLU in the family's arithmetic form (GEMMA: the GELU-tanh gate).
__device__ __forceinline__ float swiglu(int act, float g, float u) {
    if (act == OMC_ACT_GELU_TANH) return __fmul_rn(omc_gelu_tanh(g), u);   // engines/gemma.c:671
    const float e = omc_expf_glibc(-g);
    if (act == OMC_ACT_SILU_SIG) return __fmul_rn(__fmul_rn(g, __fdiv_rn(1.f, __fadd_rn(1.f, e))), u);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, e)), u);
}

constexpr int GV_WARPS = 8;   // warps per block: they split K, then reduce in a fixed order

// Gate/up for one slot and 32 weight rows: lane l owns row 32*rg + l (a warp
// reads 32 rows' 16-byte chunk: 512 contiguous bytes), warp w takes K blocks
// w, w+8, ...; the 8 partial sums are added in warp order.  Slot s < T*k is
// routed (token s / k, expert topk_idx[s]); s >= T*k is token s - T*k's
// shared expert.
__global__ void __launch_bounds__(GV_WARPS * 32) gemv_gateup_kernel(omc_layer_dev L, const float *__restrict__ x,
                                                                   int T, const int32_t *__restrict__ topk_idx,
                                                                   float *__restrict__ hbuf, int ldh, int *err) {
    extern __shared__ __align__(16) float xs[];            // [D_pad] this token's x, then [8][32][2] partials
    const int s = blockIdx.x, rg = blockIdx.y, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int nrouted = T * L.k;
    int t, e, Iw;
    if (s < nrouted) {
        t = s / L.k;
        e = topk_idx[s];
        Iw = L.I;
        if (e < 0 || e >= L.E) {
            if (threadIdx.x == 0) omc_dev_error(err, OMC_DEVERR_ROUTE, OMC_SITE_GEMV, s);
            return;
        }
    } else {
        t = s - nrouted;
        e = L.E;
        Iw = L.Is;
    }
    if (rg * 32 >= Iw) {
        // rows past the expert's width still feed the down projection (its
        // K runs to I_pad against zero weights): they must hold zeros, not
        // whatever an earlier forward left there
        if (w == 0) hbuf[(size_t)s * ldh + rg * 32 + lane] = 0.f;
        return;
    }
    for (int i = threadIdx.x * 4; i < L.D_pad; i += blockDim.x * 4) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < L.D) v = *reinterpret_cast<const float4 *>(x + (size_t)t * L.D + i);
        *reinterpret_cast<float4 *>(xs + i) = v;
    }
    __syncthreads();
    const omc_expert_ptrs P = L.experts[e];
    const int nkb = L.D_pad / OMC_KB;
    const int row = rg * 32 + lane, tile = row / OMC_TM, r = row % OMC_TM;
    const int8_t *gp = P.g + (size_t)tile * nkb * OMC_PAIR_STRIDE + (size_t)r * 16;   // pair tile: g member 0
    const int8_t *up = P.u + (size_t)tile * nkb * OMC_PAIR_STRIDE + (size_t)r * 16;   // u member 1
    float ag = 0.f, au = 0.f;
#pragma unroll 4
    for (int kb = w; kb < nkb; kb += GV_WARPS) {
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
    float *part = xs + L.D_pad;                              // [GV_WARPS][32][2]
    part[(w * 32 + lane) * 2] = ag;
    part[(w * 32 + lane) * 2 + 1] = au;
    __syncthreads();
    if (w != 0) return;
    ag = 0.f;
    au = 0.f;
    for (int q = 0; q < GV_WARPS; ++q) {
        ag += part[(q * 32 + lane) * 2];
        au += part[(q * 32 + lane) * 2 + 1];
    }
    float h = 0.f;
    if (row < Iw) {
        const float g = __fmul_rn(ag, P.gs[row]);
        const float u = __fmul_rn(au, P.us[row]);
        h = swiglu(L.act, g, u);
    }
    hbuf[(size_t)s * ldh + row] = h;
}

// One slot's down projection for 32 output rows (lane l: row 32*dg + l) over
// K blocks kb0, kb0 + ks, ...; h comes from shared memory.
__device__ __forceinline__ float down_rows(const int8_t *dp, const float *h, int nkb, int kb0, int ks) {
    float a = 0.f;
#pragma unroll 4
    for (int kb = kb0; kb < nkb; kb += ks) {
        int4 q[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) q[c] = ldg_nc_v4(dp + (size_t)kb * OMC_PAIR_STRIDE + c * 2048);
#pragma unroll
        for (int c = 0; c < 4; ++c) a = dot16(a, q[c], h + kb * OMC_KB + c * 16);
    }
    return a;
}

// For token t and 32 output rows: slot j's down projection (slots 0..k-1
// routed in selection order, slot k the shared expert) is split over ks warps
// by K block and their partials added in warp order; then warp 0 combines
// the slots in the reference's order:
// out = [sigmoid gate * shared] + sum_kk w_kk * y_kk.
__global__ void __launch_bounds__(1024) gemv_down_combine_kernel(omc_layer_dev L, int T,
                                                                 const int32_t *__restrict__ topk_idx,
                                                                 const float *__restrict__ topk_w,
                                                                 const float *__restrict__ sg,
                                                                 const float *__restrict__ hbuf, int ldh,
                                                                 float *__restrict__ out, int *err) {
    extern __shared__ __align__(16) float hs[];   // [nsl][ldh] slots' h, then [nsl][ks][32] partial rows
    const int t = blockIdx.x, dg = blockIdx.y, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int K = L.k, nsl = K + (L.has_shared ? 1 : 0), nw = blockDim.x >> 5;
    const int ks = nw >= nsl ? nw / nsl : 1;        // warps per slot
    for (int j = 0; j < nsl; ++j) {
        const size_t src = (j < K) ? (size_t)(t * K + j) : (size_t)(T * K + t);
        for (int i = threadIdx.x * 4; i < ldh; i += blockDim.x * 4)
            *reinterpret_cast<float4 *>(hs + (size_t)j * ldh + i) =
                *reinterpret_cast<const float4 *>(hbuf + src * ldh + i);
    }
    __syncthreads();
    float *ys = hs + (size_t)nsl * ldh;
    const int d = dg * 32 + lane, dt = d / OMC_TM, r = d % OMC_TM;
    for (int u = w; u < nsl * ks; u += nw) {
        const int j = u / ks, q = u % ks;
        const bool shared = j == K;
        const int e = shared ? L.E : topk_idx[(size_t)t * K + j];
        float y = 0.f;
        if (e < 0 || e > L.E) {
            if (lane == 0) omc_dev_error(err, OMC_DEVERR_ROUTE, OMC_SITE_GEMV, t);
        } else if (d < L.D) {
            const omc_expert_ptrs P = L.experts[e];
            const int nkb = (shared ? L.Is_pad : L.I_pad) / OMC_KB;
            const int8_t *dp = P.d + omc_dblk(dt, 0, nkb) + (size_t)r * 16;
            y = down_rows(dp, hs + (size_t)j * ldh, nkb, q, ks);
        }
        ys[u * 32 + lane] = y;
    }
    __syncthreads();
    if (w != 0 || d >= L.D) return;
    // y_j = (sum of its partials, in warp order) * ds (matmul_q: acc * scale)
    auto slot_y = [&](int j) {
        const int e = j == K ? L.E : topk_idx[(size_t)t * K + j];
        float a = 0.f;
        for (int q = 0; q < ks; ++q) a += ys[(j * ks + q) * 32 + lane];
        return (e >= 0 && e <= L.E) ? __fmul_rn(a, L.experts[e].ds[d]) : 0.f;
    };
    float acc = 0.f;
    if (L.has_shared) acc = __fmul_rn(slot_y(K), sg[t]);                      // out = shared; out *= sigmoid(gate)
    for (int kk = 0; kk < K; ++kk) acc = __fadd_rn(acc, __fmul_rn(topk_w[(size_t)t * K + kk], slot_y(kk)));
    out[(size_t)t * L.D + d] = acc;
}

}  // namespace

extern "C" int omc_launch_gemv_ffn(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                                   const int32_t *topk_idx, const float *topk_w, float *out, cudaStream_t s) {
    if (T <= 0) return 0;
    const int Imax_rows = L->has_shared && L->Is_rows > L->I_rows ? L->Is_rows : L->I_rows;
    const int ldh = Imax_rows;
    const int nslots = T * L->k + (L->has_shared ? T : 0);
    const size_t smem1 = (size_t)L->D_pad * sizeof(float) + GV_WARPS * 32 * 2 * sizeof(float);
    const int nsl = L->k + (L->has_shared ? 1 : 0);
    const int nw = nsl < 32 ? (32 / nsl) * nsl : 32;       // warps: ks per slot
    const int ksl = nw >= nsl ? nw / nsl : 1;
    const size_t smem2 = ((size_t)nsl * ldh + (size_t)nsl * ksl * 32) * sizeof(float);
    if (smem1 > 200 * 1024 || smem2 > 200 * 1024) return OMC_EUNSUPPORTED;
    static int attr_done = 0;
    if (!attr_done) {
        cudaFuncSetAttribute(gemv_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(gemv_down_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_done = 1;
    }
    dim3 g1(nslots, Imax_rows / 32);
    gemv_gateup_kernel<<<g1, GV_WARPS * 32, smem1, s>>>(*L, x, T, topk_idx, ws->hbuf, ldh, ws->err);
    omc_prof_mark(s, "gemv_gateup");
    dim3 g2(T, L->D_rows / 32);
    gemv_down_combine_kernel<<<g2, nw * 32, smem2, s>>>(*L, T, topk_idx, topk_w, ws->sg, ws->hbuf, ldh, out, ws->err);
    omc_prof_mark(s, "gemv_down_combine");
    omc_g_launches += 2;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}
