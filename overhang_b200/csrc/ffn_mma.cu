// ffn_mma.cu -- tensor-core (tcgen05) grouped expert SwiGLU for prefill.
//
// Replaces the per-token expert loop of the reference (engines/olmoe.c:386-399,
// engines/qwen.c:480-493) and the Metal per-expert dq_gemm dispatches
// (metal/om_metal.mm:186-229) with four kernels:
//
//   plan    one block: expert row counts -> 16-row padded offsets, and the
//           tile work lists of the two GEMMs (the batch-union of
//           engines/olmoe.c:366-378, on the device)
//   gather  every routed (token, choice) slot -> one f16 row of the
//           activation operand, grouped by expert (+ one row per token for
//           the shared expert); padding rows zeroed
//   gemm<1> per (expert, 128 rows of I, <=128 tokens): gate and up
//           H^T = silu(gs*Wg.X^T) * (us*Wu.X^T), written as the f16 operand of
//   gemm<2> per (expert, 128 rows of D, <=128 tokens): Y^T = ds*Wd.H^T,
//           times the routing weight, into a per-(token, choice) partial
//   combine out = [sigmoid gate * shared] + sum_k partial_k, in the reference's
//           order (engines/olmoe.c:395-397, engines/qwen.c:459-462,492)
//
// GEMM design (one persistent CTA per SM, warp-specialised, 864 threads).
// The expert weights are the MMA's N operand (256 rows per instruction:
// 128 gate + 128 up rows, or two 128-row tiles of the down matrix) and the
// tokens its M (128 rows, padded): a tcgen05.mma costs ~140 cycles whatever
// its N, so N=256 puts 4 KiB of weights through each instruction.
//   warp 26      int8 producer: bulk-copies (no multicast) the two 8 KiB int8
//                weight blocks of each K block into a 6-deep smem ring; the
//                depth covers ~2 us of HBM latency at the streaming rate;
//   warp 0       token producer: bulk-copies the f16 token tile (n rows x
//                128 B, contiguous in the AOL operand) into a 3-deep ring;
//   warps 2..17  dequant, two groups of 256 threads taking alternate K
//                blocks: thread t owns weight row t, converts its 64 int8
//                exactly to f16 and writes them 128B-swizzled into the
//                group's f16 B tile (2-deep ring, one tile per group);
//   warp 1       TMEM allocator + single-thread tcgen05.mma issuer
//                (kind::f16, M=128, N=256, K=16; both operands from smem);
//   warps 18..25 epilogue, one token row per thread (TMEM lane), two warps
//                per lane quarter splitting the 256 columns: SwiGLU or the
//                routing weight, from a double-buffered f32 accumulator
//                ([128 tokens] x [256 weight rows] per buffer, 512 columns).
//
// Every mbarrier wait is bounded (~1 s); on expiry the CTA records
// OMC_DEVERR_TIMEOUT, raises a shared abort flag, and all roles unwind.
#include "omc_common.cuh"

namespace {

constexpr int NMAX = 128;                 // tokens per work item (MMA M)
constexpr int NGRP = 2;                   // dequant groups (alternate K blocks)
constexpr int NDQ = 8;                    // warps per dequant group (256 threads = 256 weight rows)
constexpr int NEPI = 8;                   // epilogue warps: two per TMEM lane quarter
constexpr int SA = 3;                     // token-tile ring
constexpr int SB = NGRP;                  // f16 weight-tile ring: one tile per dequant group
constexpr int SI = 6;                     // int8 ring
constexpr int WARP_DQ0 = 2;
constexpr int WARP_EPI0 = WARP_DQ0 + NGRP * NDQ;              // 18
constexpr int WARP_I8 = WARP_EPI0 + NEPI;                     // 26
constexpr int NTHREADS = (WARP_I8 + 1) * 32;                  // 864
constexpr int W_BYTES = OMC_BLK_BYTES;    // 8 KiB int8 per 128-row weight block per K block
constexpr int A_BYTES = NMAX * 128;       // 16 KiB f16 token tile
constexpr int B_BYTES = 256 * 128;        // 32 KiB f16 weight tile
constexpr uint32_t TMEM_COLS = 512;       // two accumulator buffers of 256 columns

// smem layout (bytes, from a 1024-aligned base)
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + SA * A_BYTES;
constexpr int OFF_I8 = OFF_B + SB * B_BYTES;
constexpr int OFF_SC = OFF_I8 + SI * 2 * W_BYTES;         // [2][256] f32 row scales of the item
constexpr int OFF_BAR = OFF_SC + 2 * 256 * 4;
constexpr int SMEM_BYTES = OFF_BAR + 512 + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "smem budget");

struct WorkItem {
    int g, mt, n0, n;
};

struct GemmArgs {
    omc_layer_dev L;
    const int4 *work;
    const int *nwork;
    const uint16_t *act;       // A operand rows (AOL): x (gemm1) or h (gemm2)
    uint16_t *hout;            // gemm1: h operand out
    float *ypart;              // gemm2: per-slot partials [T][k+1][D]
    const int *rowinfo;        // gemm2: row -> slot
    const float *topk_w;       // gemm2: routing weights [T][k]
    int T, R;                  // tokens, operand rows
    int *err;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, int *err, int site,
                                              volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = omc_globaltimer();
    for (;;) {
        for (int i = 0; i < 128; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (omc_globaltimer() - t0 > OMC_WAIT_LIMIT_NS) {
            omc_dev_error(err, OMC_DEVERR_TIMEOUT, site, (int)parity);
            *abort_flag = 1;
            return false;
        }
    }
}

__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, int *err, int site,
                                          volatile int *abort_flag) {
    return __all_sync(0xffffffffu, wait_or_abort(bar, parity, err, site, abort_flag));
}

__device__ __forceinline__ uint32_t f32x2_to_f16x2_sat(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float swiglu_f(int family, float g, float u) {
    const float e = __expf(-g);
    if (family == OMC_FAMILY_QWEN) return g * __frcp_rn(1.f + e) * u;
    return __fdividef(g, 1.f + e) * u;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16, f32 accumulate.
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The 128-row weight blocks an item multiplies: phase 1 = gate tile mt and up
// tile mt; phase 2 = down tiles 2*mt and 2*mt+1 (the second absent past D_rows).
template <int PHASE>
__device__ __forceinline__ int item_nmat(const omc_layer_dev &L, const WorkItem &it) {
    if (PHASE == 1) return 2;
    return (2 * it.mt + 1) * OMC_TM < L.D_rows ? 2 : 1;
}

template <int PHASE>
struct Ctx {
    const GemmArgs &a;
    __device__ WorkItem item(int idx) const {
        const int4 v = a.work[idx];
        return WorkItem{v.x, v.y, v.z, v.w};
    }
    __device__ bool ok(const WorkItem &it) const {
        const omc_layer_dev &L = a.L;
        if (it.g < 0 || it.g > L.E || (it.g == L.E && !L.has_shared)) return false;
        if (it.n <= 0 || it.n > NMAX || (it.n & 15) || it.n0 < 0 || it.n0 + it.n > a.R || (it.n0 & 15)) return false;
        if (PHASE == 1) return it.mt >= 0 && it.mt * OMC_TM < (it.g == L.E ? L.Is_rows : L.I_rows);
        return it.mt >= 0 && 2 * it.mt * OMC_TM < L.D_rows;
    }
    __device__ int nkb(const WorkItem &it) const {
        if (PHASE == 1) return a.L.D_pad / OMC_KB;
        return (it.g == a.L.E ? a.L.Is_pad : a.L.I_pad) / OMC_KB;
    }
    // first int8 byte of weight block `mat` (0/1) of the item, K block 0
    __device__ const int8_t *wbase(const WorkItem &it, int mat) const {
        const omc_expert_ptrs P = a.L.experts[it.g];
        const int n = nkb(it);
        if (PHASE == 1) return (mat ? P.u : P.g) + (size_t)it.mt * n * W_BYTES;
        return P.d + (size_t)(2 * it.mt + mat) * n * W_BYTES;
    }
};

// Walks this CTA's (item, K block) stages in order.
template <int PHASE>
struct StageIter {
    int idx, kb, nkb, nmat, nitems, stride;
    const int8_t *w0, *w1;
    bool valid;
    __device__ void load_item(const Ctx<PHASE> &c) {
        valid = idx < nitems;
        if (!valid) return;
        const WorkItem it = c.item(idx);
        if (!c.ok(it)) {
            valid = false;
            return;
        }
        nkb = c.nkb(it);
        nmat = item_nmat<PHASE>(c.a.L, it);
        w0 = c.wbase(it, 0);
        w1 = nmat > 1 ? c.wbase(it, 1) : w0;
    }
    __device__ void init(const Ctx<PHASE> &c, int first, int n, int cta_stride) {
        idx = first;
        nitems = n;
        stride = cta_stride;
        kb = 0;
        load_item(c);
    }
    __device__ void step(const Ctx<PHASE> &c) {
        if (!valid) return;
        if (++kb >= nkb) {
            kb = 0;
            idx += stride;
            load_item(c);
        }
    }
};

template <int PHASE>   // 1: gate/up + SwiGLU, 2: down + weighting
__global__ void __launch_bounds__(NTHREADS, 1) moe_gemm_kernel(const GemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *fullA = reinterpret_cast<uint64_t *>(smem + OFF_BAR);   // [SA] token tile landed
    uint64_t *emptyA = fullA + SA;                                    // [SA] its MMAs done
    uint64_t *fullB = emptyA + SA;                                    // [SB] f16 weight tile written
    uint64_t *emptyB = fullB + SB;                                    // [SB] its MMAs done
    uint64_t *fullI = emptyB + SB;                                    // [SI] int8 blocks landed
    uint64_t *emptyI = fullI + SI;                                    // [SI] int8 slot read
    uint64_t *accfull = emptyI + SI;                                  // [2]
    uint64_t *accempty = accfull + 2;                                 // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accempty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Ctx<PHASE> c{a};
    const omc_layer_dev &L = a.L;
    const int nitems = a.nwork[PHASE - 1];

    if (threadIdx.x == 0) {
        for (int i = 0; i < SA; ++i) {
            mbar_init(&fullA[i], 1);
            mbar_init(&emptyA[i], 1);
        }
        for (int i = 0; i < SB; ++i) {
            mbar_init(&fullB[i], NDQ);
            mbar_init(&emptyB[i], 1);
        }
        for (int i = 0; i < SI; ++i) {
            mbar_init(&fullI[i], 1);
            mbar_init(&emptyI[i], NDQ);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accfull[i], 1);
            mbar_init(&accempty[i], NEPI);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ token-tile producer
        if (lane == 0) {
            uint32_t i = 0;
            for (int idx = blockIdx.x; idx < nitems && !*abort_flag; idx += gridDim.x) {
                const WorkItem it = c.item(idx);
                if (!c.ok(it)) {
                    omc_dev_error(a.err, OMC_DEVERR_BOUNDS, OMC_SITE_GEMM_PRODUCER, idx);
                    *abort_flag = 1;
                    break;
                }
                const int nkb = c.nkb(it);
                const uint32_t bytes = (uint32_t)it.n * 128;
                for (int kb = 0; kb < nkb; ++kb, ++i) {
                    const int sa = i % SA;
                    if (!wait_or_abort(&emptyA[sa], ((i / SA) & 1) ^ 1, a.err, OMC_SITE_GEMM_PRODUCER, abort_flag))
                        break;
                    mbar_arrive_expect_tx(&fullA[sa], bytes);
                    const uint8_t *src = reinterpret_cast<const uint8_t *>(a.act) + (size_t)kb * a.R * 128 +
                                         (size_t)it.n0 * 128;
                    bulk_g2s(smem + OFF_A + sa * A_BYTES, src, bytes, &fullA[sa]);
                }
            }
        }
    } else if (warp == WARP_I8) {
        // ------------------------------------------------ int8 weight producer
        if (lane == 0) {
            StageIter<PHASE> it;
            it.init(c, blockIdx.x, nitems, gridDim.x);
            for (uint32_t i = 0; it.valid && !*abort_flag; ++i) {
                const int si = i % SI;
                if (!wait_or_abort(&emptyI[si], ((i / SI) & 1) ^ 1, a.err, OMC_SITE_GEMM_PRODUCER, abort_flag))
                    break;
                mbar_arrive_expect_tx(&fullI[si], it.nmat * W_BYTES);
                uint8_t *dst = smem + OFF_I8 + si * 2 * W_BYTES;
                bulk_g2s(dst, it.w0 + (size_t)it.kb * W_BYTES, W_BYTES, &fullI[si]);
                if (it.nmat > 1) bulk_g2s(dst + W_BYTES, it.w1 + (size_t)it.kb * W_BYTES, W_BYTES, &fullI[si]);
                it.step(c);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t i = 0, ci = 0;
            for (int idx = blockIdx.x; idx < nitems && !*abort_flag; idx += gridDim.x, ++ci) {
                const WorkItem it = c.item(idx);
                if (!c.ok(it)) break;
                const int nkb = c.nkb(it);
                const uint32_t idesc = tc_idesc_f16(NMAX, 128 * item_nmat<PHASE>(L, it));
                const int b = ci & 1;
                if (!wait_or_abort(&accempty[b], ((ci >> 1) & 1) ^ 1, a.err, OMC_SITE_GEMM_MMA, abort_flag)) break;
                tc_fence_after();
                const uint32_t dcol = (uint32_t)b * 256;
                bool ok = true;
                for (int kb = 0; kb < nkb; ++kb, ++i) {
                    const int sa = i % SA, sb = i % SB;
                    ok = wait_or_abort(&fullA[sa], (i / SA) & 1, a.err, OMC_SITE_GEMM_MMA, abort_flag) &&
                         wait_or_abort(&fullB[sb], (i / SB) & 1, a.err, OMC_SITE_GEMM_MMA, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t ad = tc_sdesc_k_sw128(smem_u32(smem + OFF_A + sa * A_BYTES));
                    const uint64_t bd = tc_sdesc_k_sw128(smem_u32(smem + OFF_B + sb * B_BYTES));
#pragma unroll
                    for (int k16 = 0; k16 < 4; ++k16)   // +32 B along K = +2 in the descriptor's 16-byte units
                        tc_mma_ss(tmem + dcol, ad + 2 * k16, bd + 2 * k16, idesc, (kb > 0 || k16 > 0) ? 1u : 0u);
                    tc_commit(&emptyA[sa]);
                    tc_commit(&emptyB[sb]);
                }
                if (!ok) break;
                tc_commit(&accfull[b]);
            }
        }
    } else if (warp < WARP_EPI0) {
        // ------------------------------------------------ dequant: int8 ring -> f16 B tile
        const int dq = warp - WARP_DQ0;
        const int grp = dq / NDQ;                // K blocks i with i % NGRP == grp, B tile `grp`
        const int t = (dq % NDQ) * 32 + lane;    // weight row of the B tile, 0..255
        const int mat = t >> 7, r = t & 127;
        uint8_t *brow = smem + OFF_B + grp * B_BYTES + (uint32_t)(t >> 3) * 1024 + (uint32_t)(t & 7) * 128;
        StageIter<PHASE> pr;
        pr.init(c, blockIdx.x, nitems, gridDim.x);
        for (int j = 0; j < grp; ++j) pr.step(c);
        for (uint32_t i = grp; pr.valid && !*abort_flag; i += NGRP) {
            const int si = i % SI;
            if (!warp_wait(&fullI[si], (i / SI) & 1, a.err, OMC_SITE_GEMM_DEQUANT, abort_flag)) break;
            uint4 f[8];
            const bool active = mat < pr.nmat;
            if (active) {
                const uint8_t *m = smem + OFF_I8 + si * 2 * W_BYTES + mat * W_BYTES;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    const uint4 q = *reinterpret_cast<const uint4 *>(m + (cc * 128 + r) * 16);
                    i8x4_to_f16x4(q.x, f[2 * cc].x, f[2 * cc].y);
                    i8x4_to_f16x4(q.y, f[2 * cc].z, f[2 * cc].w);
                    i8x4_to_f16x4(q.z, f[2 * cc + 1].x, f[2 * cc + 1].y);
                    i8x4_to_f16x4(q.w, f[2 * cc + 1].z, f[2 * cc + 1].w);
                }
            }
            // The slot is released only after the converted values exist: an
            // arrive issued while the ld.shared above is still in flight does
            // not keep the next bulk copy (async proxy) from overwriting the
            // bytes before they are read.
            __syncwarp();
            if (lane == 0) mbar_arrive(&emptyI[si]);
            if (!warp_wait(&emptyB[grp], ((i / NGRP) & 1) ^ 1, a.err, OMC_SITE_GEMM_DEQUANT, abort_flag)) break;
            if (active) {
#pragma unroll
                for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4 *>(brow + ((j ^ (t & 7)) << 4)) = f[j];
            }
            fence_proxy_async_smem();      // generic stores -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&fullB[grp]);
            for (int j = 0; j < NGRP; ++j) pr.step(c);
        }
    } else {
        // ------------------------------------------------ epilogue: one token row per thread
        const int e = warp - WARP_EPI0;          // 0..7
        const int q = warp & 3;                  // TMEM lane quarter
        const int half = e >> 2;                 // which half of the 256 columns
        const int trow = q * 32 + lane;          // token row within the item = TMEM lane
        const uint32_t lane_bits = (uint32_t)(q * 32) << 16;
        uint32_t ci = 0;
        for (int idx = blockIdx.x; idx < nitems && !*abort_flag; idx += gridDim.x, ++ci) {
            const WorkItem it = c.item(idx);
            if (!c.ok(it)) break;
            const int b = ci & 1;
            if (!warp_wait(&accfull[b], (ci >> 1) & 1, a.err, OMC_SITE_GEMM_EPILOGUE, abort_flag)) break;
            tc_fence_after();
            const uint32_t acc = tmem + lane_bits + (uint32_t)b * 256;
            const omc_expert_ptrs P = L.experts[it.g];
            const bool live = trow < it.n;
            const int row = it.n0 + trow;        // operand row of this token slot
            // the item's 256 weight-row scales -> smem (one load round trip per item)
            float *sc = reinterpret_cast<float *>(smem + OFF_SC) + b * 256;
            {
                const int j = e * 32 + lane;     // 0..255
                float v = 0.f;
                if (PHASE == 1) {
                    const int Iw = it.g == L.E ? L.Is : L.I;
                    const int f = it.mt * OMC_TM + (j & 127);
                    if (f < Iw) v = j < 128 ? P.gs[f] : P.us[f];
                } else {
                    const int d = 2 * it.mt * OMC_TM + j;
                    if (d < L.D) v = P.ds[d];
                }
                sc[j] = v;
                asm volatile("bar.sync 1, %0;" ::"n"(NEPI * 32) : "memory");
            }
            if (PHASE == 1) {
                const int Iw = it.g == L.E ? L.Is : L.I;
                const int Iw_pad = it.g == L.E ? L.Is_pad : L.I_pad;
                uint8_t *hrow = reinterpret_cast<uint8_t *>(a.hout) + (size_t)row * 128;
#pragma unroll 1
                for (int j0 = half * 64; j0 < half * 64 + 64; j0 += 16) {
                    const int f0 = it.mt * OMC_TM + j0;              // first feature of the chunk
                    uint32_t gv[16], uv[16];
                    tmem_ld_32x32b_x16(acc + j0, gv);
                    tmem_ld_32x32b_x16(acc + 128 + j0, uv);
                    tc_wait_ld();
                    uint32_t hv[8];
#pragma unroll
                    for (int jj = 0; jj < 16; jj += 2) {
                        const float h0 = f0 + jj < Iw ? swiglu_f(L.family, __uint_as_float(gv[jj]) * sc[j0 + jj],
                                                                  __uint_as_float(uv[jj]) * sc[128 + j0 + jj])
                                                       : 0.f;
                        const float h1 = f0 + jj + 1 < Iw
                                             ? swiglu_f(L.family, __uint_as_float(gv[jj + 1]) * sc[j0 + jj + 1],
                                                        __uint_as_float(uv[jj + 1]) * sc[128 + j0 + jj + 1])
                                             : 0.f;
                        hv[jj >> 1] = f32x2_to_f16x2_sat(h0, h1);
                    }
                    if (live && f0 < Iw_pad) {
                        uint8_t *kbase = hrow + (size_t)(f0 >> 6) * a.R * 128;
                        const int cb = (f0 & 63) >> 3;
                        *reinterpret_cast<uint4 *>(kbase + ((cb ^ (row & 7)) << 4)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                        *reinterpret_cast<uint4 *>(kbase + (((cb + 1) ^ (row & 7)) << 4)) =
                            make_uint4(hv[4], hv[5], hv[6], hv[7]);
                    }
                }
            } else {
                const int K = L.k;
                const int nmat = item_nmat<PHASE>(L, it);
                int slot = -1;
                float w = 1.f;
                if (live) {
                    slot = a.rowinfo[row];
                    if (slot >= 0 && slot < a.T * K) w = a.topk_w[slot];
                }
                float *dst = nullptr;
                if (slot >= 0) {
                    const int tk = slot < a.T * K ? slot / K : slot - a.T * K;
                    const int kk = slot < a.T * K ? slot - tk * K : K;
                    dst = a.ypart + ((size_t)tk * (K + 1) + kk) * L.D;
                }
                const bool shared_row = slot >= a.T * K;
                if (half < nmat) {
#pragma unroll 1
                    for (int j0 = half * 128; j0 < half * 128 + 128; j0 += 16) {
                        const int d0 = 2 * it.mt * OMC_TM + j0;      // first output row of the chunk
                        uint32_t yv[16];
                        tmem_ld_32x32b_x16(acc + j0, yv);
                        tc_wait_ld();
                        float o[16];
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            const float y = __fmul_rn(__uint_as_float(yv[jj]), sc[j0 + jj]);   // matmul_q: acc * scale
                            o[jj] = shared_row ? y : __fmul_rn(w, y);                         // w * hh
                        }
                        if (dst && d0 < L.D) {
#pragma unroll
                            for (int jj = 0; jj < 16; jj += 4)
                                if (d0 + jj < L.D)
                                    *reinterpret_cast<float4 *>(dst + d0 + jj) =
                                        make_float4(o[jj], o[jj + 1], o[jj + 2], o[jj + 3]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accempty[b]);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        tmem_dealloc(tmem, TMEM_COLS);
        tmem_relinquish();
    }
}

// ---------------------------------------------------------------- plan ---
// counts[g]: routed rows of expert g (the router's atomics); the shared
// expert (g = E) gets T rows.  Writes offsets[0..G], the two work lists and
// nwork[0..1]; zeroes fill[].
__global__ void __launch_bounds__(1024) plan_kernel(const int *__restrict__ counts, int E, int has_shared, int T,
                                                    int I_rows, int Is_rows, int D_rows, int R_cap, int cap1,
                                                    int cap2, int *__restrict__ offsets, int *__restrict__ fill,
                                                    int4 *__restrict__ work1, int4 *__restrict__ work2,
                                                    int *__restrict__ nwork, int *err) {
    __shared__ int s_pad[OMC_MAX_E + 1], s_off[OMC_MAX_E + 2], s_w1[OMC_MAX_E + 2], s_w2[OMC_MAX_E + 2];
    const int G = E + (has_shared ? 1 : 0);
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        const int c = g < E ? counts[g] : T;
        const int pad = (c + OMC_ROW_ALIGN - 1) / OMC_ROW_ALIGN * OMC_ROW_ALIGN;
        s_pad[g] = pad;
        const int nch = (pad + NMAX - 1) / NMAX;
        const int mt1 = (g < E ? I_rows : Is_rows) / OMC_TM;
        s_w1[g] = nch * mt1;
        s_w2[g] = nch * ((D_rows / OMC_TM + 1) / 2);
        fill[g] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {   // G <= 1025: a serial scan is a few microseconds
        int o = 0, w1 = 0, w2 = 0;
        for (int g = 0; g < G; ++g) {
            s_off[g] = o;
            o += s_pad[g];
            const int a1 = s_w1[g], a2 = s_w2[g];
            s_w1[g] = w1;
            s_w2[g] = w2;
            w1 += a1;
            w2 += a2;
        }
        s_off[G] = o;
        s_w1[G] = w1;
        s_w2[G] = w2;
        if (o > R_cap || w1 > cap1 || w2 > cap2) {
            omc_dev_error(err, OMC_DEVERR_BOUNDS, OMC_SITE_DISPATCH, o);
            nwork[0] = nwork[1] = 0;
        } else {
            nwork[0] = w1;
            nwork[1] = w2;
        }
        nwork[2] = o;
    }
    __syncthreads();
    const bool okcap = s_off[G] <= R_cap && s_w1[G] <= cap1 && s_w2[G] <= cap2;
    for (int g = threadIdx.x; g <= G; g += blockDim.x) offsets[g] = s_off[g];
    if (!okcap) return;
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        const int pad = s_pad[g];
        if (!pad) continue;
        const int nch = (pad + NMAX - 1) / NMAX;
        const int mt1 = (g < E ? I_rows : Is_rows) / OMC_TM, mt2 = (D_rows / OMC_TM + 1) / 2;
        int p1 = s_w1[g], p2 = s_w2[g];
        for (int c = 0; c < nch; ++c) {
            const int n0 = s_off[g] + c * NMAX;
            const int n = min(NMAX, pad - c * NMAX);
            for (int m = 0; m < mt1; ++m) work1[p1++] = make_int4(g, m, n0, n);
            for (int m = 0; m < mt2; ++m) work2[p2++] = make_int4(g, m, n0, n);
        }
    }
}

// -------------------------------------------------------------- gather ---
// One warp per task: routed slot, shared row, or padding row.
__global__ void __launch_bounds__(256) gather_kernel(const float *__restrict__ x, int T, int D, int D_pad, int K,
                                                     int E, int has_shared, const int32_t *__restrict__ topk_idx,
                                                     const int *__restrict__ counts, const int *__restrict__ offsets,
                                                     int *__restrict__ fill, int *__restrict__ rowinfo,
                                                     uint16_t *__restrict__ xp, int R, int *err) {
    const int task = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int nrouted = T * K, nshared = has_shared ? T : 0;
    const int G = E + (has_shared ? 1 : 0);
    int row = -1, t = -1, info = -1;
    if (task < nrouted) {
        const int e = topk_idx[task];
        if (e < 0 || e >= E) {
            if (lane == 0) omc_dev_error(err, OMC_DEVERR_ROUTE, OMC_SITE_DISPATCH, task);
            return;
        }
        int pos = 0;
        if (lane == 0) pos = atomicAdd(&fill[e], 1);
        pos = __shfl_sync(0xffffffffu, pos, 0);
        row = offsets[e] + pos;
        t = task / K;
        info = task;
    } else if (task < nrouted + nshared) {
        t = task - nrouted;
        row = offsets[E] + t;
        info = nrouted + t;
    } else {
        const int p = task - nrouted - nshared;
        const int g = p / (OMC_ROW_ALIGN - 1), j = p % (OMC_ROW_ALIGN - 1);
        if (g >= G) return;
        const int c = g < E ? counts[g] : T;
        if (offsets[g] + c + j >= offsets[g + 1]) return;
        row = offsets[g] + c + j;
    }
    if (row < 0 || row >= R) {
        if (lane == 0) omc_dev_error(err, OMC_DEVERR_BOUNDS, OMC_SITE_DISPATCH, row);
        return;
    }
    if (lane == 0) rowinfo[row] = info;
    uint8_t *base = reinterpret_cast<uint8_t *>(xp);
    const int nkb = D_pad / 64;
    for (int kb0 = 0; kb0 < nkb; kb0 += 4) {
        const int kb = kb0 + (lane >> 3), c = lane & 7;
        if (kb >= nkb) continue;
        const int k = kb * 64 + c * 8;
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (t >= 0 && k < D) {
            const float4 a = *reinterpret_cast<const float4 *>(x + (size_t)t * D + k);
            const float4 b = *reinterpret_cast<const float4 *>(x + (size_t)t * D + k + 4);
            o.x = f32x2_to_f16x2_sat(a.x, a.y);
            o.y = f32x2_to_f16x2_sat(a.z, a.w);
            o.z = f32x2_to_f16x2_sat(b.x, b.y);
            o.w = f32x2_to_f16x2_sat(b.z, b.w);
        }
        *reinterpret_cast<uint4 *>(base + (size_t)kb * R * 128 + (size_t)row * 128 + ((c ^ (row & 7)) << 4)) = o;
    }
}

// ------------------------------------------------------------- combine ---
__global__ void __launch_bounds__(256) combine_kernel(const float *__restrict__ ypart, const float *__restrict__ sg,
                                                      int T, int D, int K, int has_shared, float *__restrict__ out) {
    const int t = blockIdx.y;
    const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (t >= T || d >= D) return;
    const float *yp = ypart + (size_t)t * (K + 1) * D + d;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (has_shared) {
        const float4 s = *reinterpret_cast<const float4 *>(yp + (size_t)K * D);
        const float gsg = sg[t];
        acc = make_float4(__fmul_rn(s.x, gsg), __fmul_rn(s.y, gsg), __fmul_rn(s.z, gsg), __fmul_rn(s.w, gsg));
    }
    for (int kk = 0; kk < K; ++kk) {
        const float4 p = *reinterpret_cast<const float4 *>(yp + (size_t)kk * D);
        acc.x = __fadd_rn(acc.x, p.x);
        acc.y = __fadd_rn(acc.y, p.y);
        acc.z = __fadd_rn(acc.z, p.z);
        acc.w = __fadd_rn(acc.w, p.w);
    }
    *reinterpret_cast<float4 *>(out + (size_t)t * D + d) = acc;
}

int g_num_sms = 0;

}  // namespace

// Work-list capacity (items of both GEMMs) for an operand of R rows.
extern "C" long long omc_mma_work_items(const omc_layer_dev *L, int R) {
    const int G = L->E + (L->has_shared ? 1 : 0);
    const int Imax_rows = L->has_shared && L->Is_rows > L->I_rows ? L->Is_rows : L->I_rows;
    const long long chunks_max = R / NMAX + G;
    return chunks_max * (Imax_rows / OMC_TM) + chunks_max * ((L->D_rows / OMC_TM + 1) / 2);
}

extern "C" int omc_launch_mma_ffn(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                                  const int32_t *topk_idx, const float *topk_w, float *out, cudaStream_t s) {
    if (T <= 0) return 0;
    if (L->D % 4) return OMC_EUNSUPPORTED;
    static int attr_done = 0;
    if (!attr_done) {
        if (cudaFuncSetAttribute(moe_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
                cudaSuccess ||
            cudaFuncSetAttribute(moe_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
                cudaSuccess)
            return OMC_ECUDA;
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        attr_done = 1;
    }
    const int E = L->E, G = E + (L->has_shared ? 1 : 0);
    const int R = ws->R_cap;
    const int Imax_rows = L->has_shared && L->Is_rows > L->I_rows ? L->Is_rows : L->I_rows;
    const int chunks_max = R / NMAX + G;
    const int cap1 = chunks_max * (Imax_rows / OMC_TM);
    const int cap2 = chunks_max * ((L->D_rows / OMC_TM + 1) / 2);
    int4 *work1 = reinterpret_cast<int4 *>(ws->work);
    int4 *work2 = work1 + cap1;
    plan_kernel<<<1, 1024, 0, s>>>(ws->counts, E, L->has_shared, T, L->I_rows, L->Is_rows, L->D_rows, R, cap1, cap2,
                                   ws->offsets, ws->fill, work1, work2, ws->nwork, ws->err);
    const int ntasks = T * L->k + (L->has_shared ? T : 0) + G * (OMC_ROW_ALIGN - 1);
    gather_kernel<<<(ntasks + 7) / 8, 256, 0, s>>>(x, T, L->D, L->D_pad, L->k, E, L->has_shared, topk_idx, ws->counts,
                                                  ws->offsets, ws->fill, ws->rowinfo, ws->xp, R, ws->err);
    GemmArgs ga;
    ga.L = *L;
    ga.work = work1;
    ga.nwork = ws->nwork;
    ga.act = ws->xp;
    ga.hout = ws->hp;
    ga.ypart = ws->ypart;
    ga.rowinfo = ws->rowinfo;
    ga.topk_w = topk_w;
    ga.T = T;
    ga.R = R;
    ga.err = ws->err;
    const int grid = g_num_sms > 0 ? g_num_sms : 148;
    omc_prof_mark(s, "dispatch");
    moe_gemm_kernel<1><<<grid, NTHREADS, SMEM_BYTES, s>>>(ga);
    omc_prof_mark(s, "gemm_gateup");
    ga.work = work2;
    ga.act = ws->hp;
    moe_gemm_kernel<2><<<grid, NTHREADS, SMEM_BYTES, s>>>(ga);
    omc_prof_mark(s, "gemm_down");
    dim3 gc((L->D / 4 + 255) / 256, T);
    combine_kernel<<<gc, 256, 0, s>>>(ws->ypart, ws->sg, T, L->D, L->k, L->has_shared, out);
    omc_prof_mark(s, "combine");
    omc_g_launches += 5;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}
