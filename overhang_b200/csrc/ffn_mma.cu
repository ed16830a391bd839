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
// GEMM design (one persistent CTA per SM, warp-specialised, 320 threads):
//   warp 0      bulk-copy producer: the int8 weight K-block(s) (8 KiB per
//               matrix, contiguous in the tiled slab) and the f16 token tile
//               (n rows x 128 B, contiguous in the operand) into a smem ring;
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer;
//   warps 2..9  dequant: int8 -> f16 (exact) in registers, written straight
//               into TMEM as the MMA's A operand (tcgen05.st), so the f16
//               weights never round-trip through shared memory; the same
//               warps run the epilogue (tcgen05.ld of the f32 accumulators).
// The weight rows are the MMA's M (=128) and the tokens its N (16..128):
// few tokens per expert still fill the tensor core's M dimension, and the
// per-row int8 scale is one register per epilogue thread.
//
// Every mbarrier wait is bounded (~1 s); on expiry the CTA records
// OMC_DEVERR_TIMEOUT, raises a shared abort flag, and all roles unwind.
#include "omc_common.cuh"

namespace {

constexpr int NMAX = 128;                 // tokens per work item (MMA N)
constexpr int SW = 4;                     // smem ring stages
constexpr int SA = 4;                     // TMEM A stages
constexpr int NTHREADS = 320;
constexpr int W_BYTES = OMC_BLK_BYTES;    // 8 KiB int8 per matrix per stage
constexpr int B_BYTES = NMAX * 128;       // 16 KiB f16 token tile per stage
constexpr uint32_t TMEM_COLS = 512;

// smem layout (bytes, from a 1024-aligned base)
constexpr int OFF_B = 0;                                  // SW x B_BYTES
constexpr int OFF_W = OFF_B + SW * B_BYTES;               // SW x 2 x W_BYTES
constexpr int OFF_BAR = OFF_W + SW * 2 * W_BYTES;         // barriers
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;          // + alignment slack

struct WorkItem {
    int g, mt, n0, n;
};

struct GemmArgs {
    omc_layer_dev L;
    const int4 *work;
    const int *nwork;
    const uint16_t *act;       // B operand rows (AOL): x (gemm1) or h (gemm2)
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

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
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

// Byte offset of element (row, k) in an AOL operand with R rows.
__device__ __forceinline__ size_t aol_off(int R, int row, int k) {
    return (size_t)(k >> 6) * R * 128 + (size_t)row * 128 + ((((k & 63) >> 3) ^ (row & 7)) << 4) + ((k & 7) << 1);
}

template <int PHASE>   // 1: gate/up + SwiGLU, 2: down + weighting
__global__ void __launch_bounds__(NTHREADS, 1) moe_gemm_kernel(const GemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full_w = reinterpret_cast<uint64_t *>(smem + OFF_BAR);   // [SW]
    uint64_t *empty_w = full_w + SW;                                   // [SW]
    uint64_t *afull = empty_w + SW;                                    // [SA]
    uint64_t *aempty = afull + SA;                                     // [SA]
    uint64_t *accfull = aempty + SA;                                   // [1]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accfull + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int NDQ = 8;   // dequant warps

    if (threadIdx.x == 0) {
        for (int i = 0; i < SW; ++i) {
            mbar_init(&full_w[i], 1);
            mbar_init(&empty_w[i], NDQ + 1);
        }
        for (int i = 0; i < SA; ++i) {
            mbar_init(&afull[i], NDQ);
            mbar_init(&aempty[i], 1);
        }
        mbar_init(accfull, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int nitems = a.nwork[PHASE - 1];
    const omc_layer_dev &L = a.L;
    constexpr int NMAT = PHASE == 1 ? 2 : 1;
    // TMEM columns: accumulators at 0 (gate) and NMAX (up) / 0 (down); A stages from 256
    constexpr uint32_t ACOL0 = 256;
    constexpr uint32_t ACOLS_PER_STAGE = 32 * NMAT;

    auto item_at = [&](int idx) -> WorkItem {
        const int4 v = a.work[idx];
        return WorkItem{v.x, v.y, v.z, v.w};
    };
    auto item_ok = [&](const WorkItem &it) -> bool {
        if (it.g < 0 || it.g > L.E || (it.g == L.E && !L.has_shared)) return false;
        if (it.n <= 0 || it.n > NMAX || (it.n & 15) || it.n0 < 0 || it.n0 + it.n > a.R || (it.n0 & 15)) return false;
        const int rows = PHASE == 1 ? (it.g == L.E ? L.Is_rows : L.I_rows) : L.D_rows;
        return it.mt >= 0 && it.mt * OMC_TM < rows;
    };
    auto nkb_of = [&](const WorkItem &it) -> int {
        if (PHASE == 1) return L.D_pad / OMC_KB;
        return (it.g == L.E ? L.Is_pad : L.I_pad) / OMC_KB;
    };

    if (warp == 0) {
        // ------------------------------------------------ producer
        if (lane == 0) {
            uint32_t it_count = 0;
            for (int idx = blockIdx.x; idx < nitems && !*abort_flag; idx += gridDim.x) {
                const WorkItem it = item_at(idx);
                if (!item_ok(it)) {
                    omc_dev_error(a.err, OMC_DEVERR_BOUNDS, OMC_SITE_GEMM_PRODUCER, idx);
                    *abort_flag = 1;
                    break;
                }
                const omc_expert_ptrs P = L.experts[it.g];
                const int nkb = nkb_of(it);
                const int8_t *w0 = PHASE == 1 ? P.g : P.d;
                const int8_t *w1 = P.u;
                const size_t tile = (size_t)it.mt * nkb * W_BYTES;
                const uint32_t bbytes = (uint32_t)it.n * 128;
                for (int kb = 0; kb < nkb; ++kb, ++it_count) {
                    const int s = it_count % SW;
                    const uint32_t ph = (it_count / SW) & 1;
                    if (!wait_or_abort(&empty_w[s], ph ^ 1, a.err, OMC_SITE_GEMM_PRODUCER, abort_flag)) break;
                    mbar_arrive_expect_tx(&full_w[s], NMAT * W_BYTES + bbytes);
                    uint8_t *sw = smem + OFF_W + s * 2 * W_BYTES;
                    bulk_g2s(sw, w0 + tile + (size_t)kb * W_BYTES, W_BYTES, &full_w[s]);
                    if (NMAT == 2) bulk_g2s(sw + W_BYTES, w1 + tile + (size_t)kb * W_BYTES, W_BYTES, &full_w[s]);
                    const uint8_t *src = reinterpret_cast<const uint8_t *>(a.act) + (size_t)kb * a.R * 128 +
                                         (size_t)it.n0 * 128;
                    bulk_g2s(smem + OFF_B + s * B_BYTES, src, bbytes, &full_w[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t it_count = 0, a_count = 0, item_count = 0;
            for (int idx = blockIdx.x; idx < nitems && !*abort_flag; idx += gridDim.x, ++item_count) {
                const WorkItem it = item_at(idx);
                if (!item_ok(it)) break;
                const int nkb = nkb_of(it);
                const uint32_t idesc = tc_idesc_f16(128, it.n);
                bool ok = true;
                for (int kb = 0; kb < nkb && ok; ++kb, ++it_count, ++a_count) {
                    const int s = it_count % SW;
                    const uint32_t ph = (it_count / SW) & 1;
                    const int as = a_count % SA;
                    const uint32_t aph = (a_count / SA) & 1;
                    ok = wait_or_abort(&full_w[s], ph, a.err, OMC_SITE_GEMM_MMA, abort_flag) &&
                         wait_or_abort(&afull[as], aph, a.err, OMC_SITE_GEMM_MMA, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t bsm = smem_u32(smem + OFF_B + s * B_BYTES);
#pragma unroll
                    for (int k16 = 0; k16 < 4; ++k16) {
                        const uint64_t bd = tc_sdesc_k_sw128(bsm + k16 * 32);
                        const uint32_t acc = (kb > 0 || k16 > 0) ? 1u : 0u;
                        const uint32_t acol = ACOL0 + as * ACOLS_PER_STAGE + k16 * 8;
                        tc_mma_ts(tmem + 0, tmem + acol, bd, idesc, acc);
                        if (NMAT == 2) tc_mma_ts(tmem + NMAX, tmem + acol + 32, bd, idesc, acc);
                    }
                    tc_commit(&empty_w[s]);
                    tc_commit(&aempty[as]);
                }
                if (!ok) break;
                tc_commit(accfull);
            }
        }
    } else {
        // ------------------------------------------------ dequant + epilogue (warps 2..9)
        const int dq = warp - 2;                 // 0..7
        const int q = warp & 3;                  // TMEM lane quarter this warp may access
        const int half = dq >> 2;                // 0/1: gate/up (phase 1) or K half (phase 2)
        const int row = q * 32 + lane;           // weight row within the 128-row tile
        const uint32_t lane_bits = (uint32_t)(q * 32) << 16;
        uint32_t it_count = 0, a_count = 0, item_count = 0;
        for (int idx = blockIdx.x; idx < nitems && !*abort_flag; idx += gridDim.x, ++item_count) {
            const WorkItem it = item_at(idx);
            if (!item_ok(it)) break;
            const int nkb = nkb_of(it);
            bool ok = true;
            for (int kb = 0; kb < nkb; ++kb, ++it_count, ++a_count) {
                const int s = it_count % SW;
                const uint32_t ph = (it_count / SW) & 1;
                const int as = a_count % SA;
                const uint32_t aph = (a_count / SA) & 1;
                ok = __all_sync(0xffffffffu, wait_or_abort(&full_w[s], ph, a.err, OMC_SITE_GEMM_DEQUANT, abort_flag));
                if (!ok) break;
                const uint8_t *sw = smem + OFF_W + s * 2 * W_BYTES;
                uint4 raw[4];
                if (PHASE == 1) {
                    const uint8_t *m = sw + half * W_BYTES;
#pragma unroll
                    for (int c = 0; c < 4; ++c) raw[c] = *reinterpret_cast<const uint4 *>(m + (c * 128 + row) * 16);
                } else {
#pragma unroll
                    for (int c = 0; c < 2; ++c)
                        raw[c] = *reinterpret_cast<const uint4 *>(sw + ((2 * half + c) * 128 + row) * 16);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty_w[s]);
                ok = __all_sync(0xffffffffu, wait_or_abort(&aempty[as], aph ^ 1, a.err, OMC_SITE_GEMM_DEQUANT, abort_flag));
                if (!ok) break;
                uint32_t v[32];
                const int nchunk = PHASE == 1 ? 4 : 2;
#pragma unroll
                for (int c = 0; c < nchunk; ++c) {
                    i8x4_to_f16x4(raw[c].x, v[8 * c + 0], v[8 * c + 1]);
                    i8x4_to_f16x4(raw[c].y, v[8 * c + 2], v[8 * c + 3]);
                    i8x4_to_f16x4(raw[c].z, v[8 * c + 4], v[8 * c + 5]);
                    i8x4_to_f16x4(raw[c].w, v[8 * c + 6], v[8 * c + 7]);
                }
                const uint32_t acol = ACOL0 + as * ACOLS_PER_STAGE;
                if (PHASE == 1) {
                    tmem_st_32x32b_x32(tmem + lane_bits + acol + half * 32, *reinterpret_cast<uint32_t(*)[32]>(v));
                } else {
                    tmem_st_32x32b_x16(tmem + lane_bits + acol + half * 16, v);
                }
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[as]);
            }
            if (!ok) break;
            // ---- epilogue of this item
            if (!__all_sync(0xffffffffu, wait_or_abort(accfull, item_count & 1, a.err, OMC_SITE_GEMM_EPILOGUE, abort_flag)))
                break;
            tc_fence_after();
            const omc_expert_ptrs P = L.experts[it.g];
            const int grow = it.mt * OMC_TM + row;            // weight row (I or D index)
            if (PHASE == 1) {
                // rows in [Iw, K-extent of the down GEMM) are written as zeros so
                // the padded K columns of the h operand are finite
                const int Iw = it.g == L.E ? L.Is : L.I;
                const int Iw_pad = it.g == L.E ? L.Is_pad : L.I_pad;
                const float gsc = grow < Iw ? P.gs[grow] : 0.f;
                const float usc = grow < Iw ? P.us[grow] : 0.f;
                for (int c16 = half; c16 < it.n / 16; c16 += 2) {
                    uint32_t gv[16], uv[16];
                    tmem_ld_32x32b_x16(tmem + lane_bits + 0 + c16 * 16, gv);
                    tmem_ld_32x32b_x16(tmem + lane_bits + NMAX + c16 * 16, uv);
                    tc_wait_ld();
                    if (grow < Iw_pad) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            float h = 0.f;
                            if (grow < Iw) {
                                const float g = __uint_as_float(gv[j]) * gsc;
                                const float u = __uint_as_float(uv[j]) * usc;
                                h = swiglu_f(L.family, g, u);
                            }
                            const int r = it.n0 + c16 * 16 + j;
                            const uint32_t hb = f32x2_to_f16x2_sat(h, 0.f) & 0xFFFFu;
                            *reinterpret_cast<uint16_t *>(reinterpret_cast<uint8_t *>(a.hout) + aol_off(a.R, r, grow)) =
                                (uint16_t)hb;
                        }
                    }
                }
            } else {
                const float dsc = grow < L.D ? P.ds[grow] : 0.f;
                const int K = L.k;
                for (int c16 = half; c16 < it.n / 16; c16 += 2) {
                    uint32_t yv[16];
                    tmem_ld_32x32b_x16(tmem + lane_bits + c16 * 16, yv);
                    tc_wait_ld();
                    if (grow < L.D) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int slot = a.rowinfo[it.n0 + c16 * 16 + j];
                            if (slot < 0) continue;
                            const float y = __fmul_rn(__uint_as_float(yv[j]), dsc);   // matmul_q: acc * scale
                            size_t dst;
                            float p;
                            if (slot < a.T * K) {
                                const int t = slot / K, kk = slot - t * K;
                                p = __fmul_rn(a.topk_w[slot], y);                    // w * hh
                                dst = ((size_t)t * (K + 1) + kk) * L.D + grow;
                            } else {
                                const int t = slot - a.T * K;
                                p = y;
                                dst = ((size_t)t * (K + 1) + K) * L.D + grow;
                            }
                            a.ypart[dst] = p;
                        }
                    }
                }
            }
            tc_fence_before();
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
        s_w2[g] = nch * (D_rows / OMC_TM);
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
        const int mt1 = (g < E ? I_rows : Is_rows) / OMC_TM, mt2 = D_rows / OMC_TM;
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
    return chunks_max * (Imax_rows / OMC_TM) + chunks_max * (L->D_rows / OMC_TM);
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
    const int cap2 = chunks_max * (L->D_rows / OMC_TM);
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
