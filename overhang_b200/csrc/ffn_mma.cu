// ffn_mma.cu -- tensor-core (tcgen05) grouped expert SwiGLU for prefill.
//
// Replaces the per-token expert loop of the reference (engines/olmoe.c:386-399,
// engines/qwen.c:480-493) and the Metal per-expert dq_gemm dispatches
// (metal/om_metal.mm:186-229) with four kernels:
//
//   gather  every routed (token, choice) slot -> one f16 row of the
//           activation operand at the row the dispatch plan gave it
//           (omc_plan.cuh, built by the router's last select block),
//           grouped by expert (+ one row per token for the shared expert);
//           padding rows zeroed
//   gemm<1> per (expert, 128 rows of I, <=128 tokens): gate and up
//           H^T = silu(gs*Wg.X^T) * (us*Wu.X^T), written as the f16 operand of
//   gemm<2> per (expert, 128 rows of D, <=128 tokens): Y^T = ds*Wd.H^T,
//           times the routing weight, into a per-(token, choice) partial
//   combine out = [sigmoid gate * shared] + sum_k partial_k, in the reference's
//           order (engines/olmoe.c:395-397, engines/qwen.c:459-462,492)
//
// GEMM design (one persistent CTA per SM, warp-specialised, 864 threads).
// The dequantised expert weights are the MMA's A operand, held in tensor
// memory (M = 128 weight rows per instruction); the tokens are its B operand
// in shared memory (N = the item's 16..128 token rows).  Weights therefore
// never pass through shared memory as f16: per 16 KiB int8 K block the SM's
// shared-memory traffic is the int8 landing + its read (32 KiB), the token
// tile (<= 16 KiB) and the MMA's token reads, instead of also writing and
// re-reading a 32 KiB f16 weight tile.  (tcgen05.mma reads its shared-memory
// operands through the same 128 B/cycle as every other access; with weights
// in TMEM an M=128 N=64 K=16 MMA runs at the full 32-cycle tensor rate.)
//   warp 26      int8 producer: one bulk copy (no multicast) per K block of
//                the item's tile pair, 16 KiB contiguous in the slab's paired
//                layout, into a 6-deep ring, L2 evict-first (every weight
//                byte is read once per forward).  One thread issuing 8 KiB
//                copies tops out near 5.3 TB/s on B200; 16 KiB ones reach
//                ~6.9 TB/s;
//   warps 2..17  dequant, four groups of 4 warps, group g taking the K
//                blocks i with i % 4 == g, so four blocks' latency chains
//                overlap (with two groups of 8 the block period was ~960
//                cycles, set by that chain: token-tile landing, int8 wait,
//                conversion, TMEM stage wait, store).  A group first starts
//                its K block's f16 token tile (n rows x 128 B, contiguous in
//                the AOL operand) into a 5-deep smem ring with per-lane
//                cp.async, L2 evict-last (bulk copies of one SM share a
//                queue: one issued behind the int8 stream waits ~4k cycles
//                even on an L2 hit); then warp w of the group writes weight
//                rows 32*(w%4)..+31 (its TMEM lane quarter) of both tiles
//                (gate/up or down 2mt / 2mt+1), one after the other:
//                64 int8 -> exact f16 -> tcgen05.st into a 3-deep ring of
//                TMEM A stages (64 columns each: 2 tiles x 32);
//   warp 1       TMEM allocator + tcgen05.mma issuer: the warp runs the
//                loop, an elected lane issues (kind::f16, A from TMEM,
//                M=128, N=n, K=16; 8 per K block);
//   warps 18..25 epilogue, one weight row (= TMEM lane) per thread, two
//                warps per lane quarter: SwiGLU into an smem tile that two
//                bulk stores write out as the h operand, or scale x routing
//                weight straight into the per-slot partials.
// Accumulators: two 160-column TMEM slots.  An item of <= 80 tokens uses one
// slot (gate at +0, up at +80), so consecutive items double-buffer; a larger
// item takes both slots.  The epilogue fetches what it needs of an item
// (scales, routing of its rows) before it waits for the accumulator.
//
// Every mbarrier wait is bounded (~1 s); on expiry the CTA records
// OMC_DEVERR_TIMEOUT, raises a shared abort flag, and all roles unwind.
#include "omc_plan.cuh"

namespace {

constexpr int NMAX = OMC_NMAX;            // tokens per work item (MMA N)
constexpr int NGRP = 4;                   // dequant groups (K blocks i with i % NGRP == group)
constexpr int NDQ = 4;                    // warps per dequant group: one per TMEM lane quarter, both tiles
constexpr int GTHREADS = NDQ * 32;        // threads of a group (its token-tile copies)
constexpr int NEPI = 8;                   // epilogue warps: two per TMEM lane quarter
constexpr int SA = 5;                     // token-tile ring (smem)
constexpr int ST = 3;                     // weight A stages (TMEM)
constexpr int SI = 6;                     // int8 ring (smem)
constexpr int WARP_DQ0 = 2;
constexpr int WARP_EPI0 = WARP_DQ0 + NGRP * NDQ;              // 18
constexpr int WARP_I8 = WARP_EPI0 + NEPI;                     // 26
constexpr int NTHREADS = (WARP_I8 + 1) * 32;                  // 864
constexpr int W_BYTES = OMC_BLK_BYTES;    // 8 KiB int8 per 128-row weight block per K block
constexpr int A_BYTES = NMAX * 128;       // 16 KiB f16 token tile
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t ACC_SLOT_COLS = 160;   // accumulator slots at columns 0 and 160
constexpr uint32_t TCOL_A = 320;          // A stages: 320 + 64*stage + 32*tile
constexpr int SMALL_N = 80;               // items up to this many tokens take one slot
static_assert(TCOL_A + ST * 64 <= TMEM_COLS && 2 * ACC_SLOT_COLS <= TCOL_A, "TMEM columns");

// smem layout (bytes, from a 1024-aligned base)
constexpr int OFF_A = 0;
constexpr int OFF_I8 = OFF_A + SA * A_BYTES;
constexpr int OFF_STG = OFF_I8 + SI * 2 * W_BYTES;         // [2 K halves][NMAX rows][128 B] h staging
constexpr int OFF_TAB = OFF_STG + 2 * NMAX * 128;        // [NEPI][NMAX] (ypart row, weight) per epilogue warp
constexpr int OFF_BAR = OFF_TAB + NEPI * NMAX * 8;
constexpr int SMEM_BYTES = OFF_BAR + 512 + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "smem budget");
static_assert(OFF_I8 % 1024 == 0 && OFF_STG % 1024 == 0, "alignment");

struct WorkItem {
    int g, mt, n0, n;
};

struct GemmArgs {
    omc_layer_dev L;
    const int4 *work;
    const int *nwork;
    const uint16_t *act;       // gemm2: h operand rows (AOL, swizzled)
    const uint16_t *xh;        // gemm1: f16 tokens [T][D], gathered per operand row
    uint16_t *hout;            // gemm1: h operand out
    float *ypart;              // gemm2: per-slot partials [T][k+1][D]
    const int *rowinfo;        // row -> slot (-1 padding)
    const float *roww;         // gemm2: row -> routing weight (1 for the shared expert)
    int K, nrouted;            // slots per token and routed slots: a slot s < nrouted is
                               // token s / K, choice s % K; s >= nrouted is token s - nrouted
    int ydirect;               // gemm2: 1 = write row slot of ypart ([slots][D]) instead of
                               // the [T][K+1][D] partials
    int wf16;                  // gemm2: the weights are f16 tiles (omm_dense): one 128-row tile
                               // of 64 f16 columns per 16 KB K block, copied to TMEM as they are
    const int *slot_tok;       // gemm1: token row of each slot (xh row), or NULL: derived
                               // from the slot as above
    int T, R;                  // tokens, operand rows
    int *err;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, int *err, int site,
                                              volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    OmcDeadline dl;
    dl.start();
    for (;;) {
        for (int i = 0; i < 8; ++i)
            if (mbar_try_wait_sleep(bar, parity, 500000u)) return true;   // sleeps up to 0.5 ms per try
        if (*abort_flag) return false;
        if (dl.over()) {
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


__device__ __forceinline__ float swiglu_f(int act, float g, float u) {
    if (act == OMC_ACT_GELU_TANH) return omc_gelu_tanh(g) * u;   // engines/gemma.c:671
    const float e = __expf(-g);
    if (act == OMC_ACT_SILU_SIG) return g * __frcp_rn(1.f + e) * u;
    return __fdividef(g, 1.f + e) * u;
}


// The 128-row weight blocks an item multiplies: phase 1 = gate tile mt and up
// tile mt; phase 2 = down tiles 2*mt and 2*mt+1 (the second absent past D_rows),
// or with f16 weights the one tile mt.
template <int PHASE>
__device__ __forceinline__ int item_nmat(const GemmArgs &a, const WorkItem &it) {
    if (PHASE == 1) return 2;
    if (a.wf16) return 1;
    return (2 * it.mt + 1) * OMC_TM < a.L.D_rows ? 2 : 1;
}
// first output row of tile `half` of a phase-2 item
__device__ __forceinline__ int item_row0(const GemmArgs &a, const WorkItem &it, int half) {
    return (a.wf16 ? it.mt : 2 * it.mt + half) * OMC_TM;
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
        return it.mt >= 0 && (a.wf16 ? it.mt : 2 * it.mt) * OMC_TM < L.D_rows;
    }
    __device__ int nkb(const WorkItem &it) const {
        if (PHASE == 1) return a.L.D_pad / OMC_KB;
        return (it.g == a.L.E ? a.L.Is_pad : a.L.I_pad) / OMC_KB;
    }
    // first int8 byte of the item's tile pair (gate/up of tile mt, or down
    // tiles 2mt and 2mt+1), K block 0; K block kb is OMC_PAIR_STRIDE further
    __device__ const int8_t *pair_base(const WorkItem &it) const {
        const omc_expert_ptrs P = a.L.experts[it.g];
        const size_t off = (size_t)it.mt * nkb(it) * OMC_PAIR_STRIDE;
        return (PHASE == 1 ? P.g : P.d) + off;
    }
};

// Walks this CTA's (item, K block) stages in order.
template <int PHASE>
struct StageIter {
    int idx, kb, nkb, nmat, nitems, stride, n0, n;
    const int8_t *w;
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
        nmat = item_nmat<PHASE>(c.a, it);
        w = c.pair_base(it);
        n0 = it.n0;
        n = it.n;
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

// 16-byte cp.async global -> shared with an L2 cache policy (LSU path).
__device__ __forceinline__ void cp_async16_hint(void *smem_dst, const void *gsrc, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
                 "l"(policy)
                 : "memory");
}
// The same with src_size 0 when !valid: the 16 bytes are zero-filled.
__device__ __forceinline__ void cp_async16_zfill_hint(void *smem_dst, const void *gsrc, bool valid, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(smem_u32(smem_dst)),
                 "l"(gsrc), "r"(valid ? 16 : 0), "l"(policy)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// 16-byte-aligned bulk store shared -> global, tracked by this thread's bulk group.
__device__ __forceinline__ void bulk_s2g(void *gdst, const void *ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(ssrc)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One lane of the (converged) warp, the same each call.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile("{\n\t.reg .pred P1;\n\telect.sync _|P1, 0xffffffff;\n\tselp.b32 %0, 1, 0, P1;\n\t}" : "=r"(pred));
    return pred != 0;
}

// TMEM accumulator columns of an item's weight tile t (both roles agree):
// one slot for <= SMALL_N tokens (tile t at +64t), else one slot per tile.
struct AccSlots {
    uint32_t ctr = 0, u0 = 0, u1 = 0;   // slots taken so far; uses of slot 0 and slot 1
    int nslots = 1, p0 = 0;             // this item: slot count, first slot (second = p0 ^ 1)
    __device__ void begin(int n) {
        nslots = n > SMALL_N ? 2 : 1;
        p0 = (int)(ctr & 1u);
    }
    __device__ int slot(int j) const { return p0 ^ j; }
    __device__ uint32_t col(int t) const {
        return nslots == 1 ? (uint32_t)p0 * ACC_SLOT_COLS + (uint32_t)t * (uint32_t)SMALL_N
                           : (uint32_t)(p0 ^ t) * ACC_SLOT_COLS;
    }
    __device__ uint32_t parity(int j) const { return (slot(j) ? u1 : u0) & 1u; }
    __device__ void end() {
        if (nslots == 2) {
            ++u0;
            ++u1;
        } else if (p0) {
            ++u1;
        } else {
            ++u0;
        }
        ctr += (uint32_t)nslots;
    }
};

template <int PHASE>   // 1: gate/up + SwiGLU, 2: down + weighting
__global__ void __launch_bounds__(NTHREADS, 1) moe_gemm_kernel(const GemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *emptyA = reinterpret_cast<uint64_t *>(smem + OFF_BAR);  // [SA] token slot's MMAs done
    uint64_t *fullI = emptyA + SA;                                    // [SI] int8 blocks landed
    uint64_t *emptyI = fullI + SI;                                    // [SI] int8 slot converted
    uint64_t *fullT = emptyI + SI;                                    // [ST] TMEM weight stage + token tile ready
    uint64_t *emptyT = fullT + ST;                                    // [ST] its MMAs done
    uint64_t *accfull = emptyT + ST;                                  // [2] accumulator slot ready
    uint64_t *accempty = accfull + 2;                                 // [2] accumulator slot drained
    uint64_t *stgfull = accempty + 2;                                 // h staging written (phase 1)
    uint64_t *stgfree = stgfull + 1;                                  // h staging read by its bulk store
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(stgfree + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Ctx<PHASE> c{a};
    const omc_layer_dev &L = a.L;
    const int nitems = a.nwork[PHASE - 1];

    if (threadIdx.x == 0) {
        for (int i = 0; i < SA; ++i) mbar_init(&emptyA[i], 1);
        for (int i = 0; i < SI; ++i) {
            mbar_init(&fullI[i], 1);
            mbar_init(&emptyI[i], NDQ);
        }
        for (int i = 0; i < ST; ++i) {
            mbar_init(&fullT[i], NDQ);
            mbar_init(&emptyT[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accfull[i], 1);
            mbar_init(&accempty[i], NEPI);
        }
        mbar_init(stgfull, NEPI);
        mbar_init(stgfree, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // no role: the token tiles are loaded by the dequant group of their K block
    } else if (warp == WARP_I8) {
        // ------------------------------------------------ int8 weight producer
        if (lane == 0) {
            StageIter<PHASE> it;
            it.init(c, blockIdx.x, nitems, gridDim.x);
            const uint64_t stream = l2_policy_evict_first();
            for (uint32_t i = 0; it.valid && !*abort_flag; ++i) {
                const int si = i % SI;
                if (!wait_or_abort(&emptyI[si], ((i / SI) & 1) ^ 1, a.err, OMC_SITE_GEMM_PRODUCER, abort_flag))
                    break;
                // the pair's K block is one contiguous 16 KiB (8 KiB when the pair has one tile)
                const uint32_t bytes = (PHASE == 2 && a.wf16 ? 2u : (uint32_t)it.nmat) * W_BYTES;
                mbar_arrive_expect_tx(&fullI[si], bytes);
                bulk_g2s_hint(smem + OFF_I8 + si * 2 * W_BYTES, it.w + (size_t)it.kb * OMC_PAIR_STRIDE, bytes,
                              &fullI[si], stream);
                it.step(c);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        // The whole warp runs the loop (operands warp-uniform); one elected
        // lane issues a K block's eight MMAs back to back.  Measured with
        // clock64 stamps (OLMoE T=512): an elect + __syncwarp around every MMA
        // cost ~73 cycles an MMA and made this warp the pipeline's bottleneck
        // (one K block per ~1,020 cycles); one elect per block issues the
        // eight in ~330 cycles, and the block period falls to ~960 cycles,
        // now set by the dequant group.
        uint32_t i = 0;
        AccSlots acc;
        for (int idx = blockIdx.x; idx < nitems && !*abort_flag; idx += gridDim.x) {
            const WorkItem it = c.item(idx);
            if (!c.ok(it)) break;
            const int nkb = c.nkb(it);
            const int nmat = item_nmat<PHASE>(a, it);
            acc.begin(it.n);
            bool ok = true;
            for (int j = 0; j < acc.nslots && ok; ++j)
                ok = warp_wait(&accempty[acc.slot(j)], acc.parity(j) ^ 1u, a.err, OMC_SITE_GEMM_MMA, abort_flag);
            if (!ok) break;
            tc_fence_after();
            const uint32_t idesc = tc_idesc_f16(128, it.n);     // M = weight rows, N = tokens
            const uint32_t d0 = tmem + acc.col(0), d1 = tmem + acc.col(1);
            for (int kb = 0; kb < nkb; ++kb, ++i) {
                const int sa = i % SA, st = i % ST;
                if (!warp_wait(&fullT[st], (i / ST) & 1, a.err, OMC_SITE_GEMM_MMA, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t bd = tc_sdesc_k_sw128(smem_u32(smem + OFF_A + sa * A_BYTES));
                const uint32_t acol = tmem + TCOL_A + (uint32_t)st * 64u;
                // the block's MMAs (K = 16 each: +32 B along K is +2 in the smem
                // descriptor, +8 TMEM columns) from one elected lane, back to back
                if (elect_one()) {
#pragma unroll
                    for (int k16 = 0; k16 < 4; ++k16) {
                        const uint32_t accum = (kb > 0 || k16 > 0) ? 1u : 0u;
                        tc_mma_ts(d0, acol + 8u * k16, bd + 2 * k16, idesc, accum);
                        if (nmat > 1) tc_mma_ts(d1, acol + 32u + 8u * k16, bd + 2 * k16, idesc, accum);
                    }
                }
                __syncwarp();
                if (elect_one()) {
                    tc_commit(&emptyA[sa]);
                    tc_commit(&emptyT[st]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (elect_one())
                for (int j = 0; j < acc.nslots; ++j) tc_commit(&accfull[acc.slot(j)]);
            __syncwarp();
            acc.end();
        }
    } else if (warp < WARP_EPI0) {
        // ------------------------------------------------ dequant: int8 ring -> TMEM A stage
        const int dq = warp - WARP_DQ0;
        const int grp = dq / NDQ;                // K blocks i with i % NGRP == grp
        const int q = warp & 3;                  // this warp's TMEM lane quarter (the group's 4 warps cover all 4)
        const int r = q * 32 + lane;             // weight row within each 128-row tile
        const uint32_t lane_bits = (uint32_t)(q * 32) << 16;
        StageIter<PHASE> pr;
        pr.init(c, blockIdx.x, nitems, gridDim.x);
        for (int j = 0; j < grp; ++j) pr.step(c);
        const int gt = (dq % NDQ) * 32 + lane;   // thread index within the group
        constexpr int XR = NMAX * 8 / GTHREADS;  // token rows this thread copies per tile
        const uint64_t keep = l2_policy_evict_last();
        int xrow_item = -1, xrow[XR];            // gemm1: token of each row this lane copies
#pragma unroll
        for (int u = 0; u < XR; ++u) xrow[u] = -1;
        for (uint32_t i = grp; pr.valid && !*abort_flag; i += NGRP) {
            const int si = i % SI, st = i % ST, sa = i % SA;
            // token tile of this K block: per-lane cp.async (not a bulk copy, which would queue
            // behind the int8 stream's in the SM's copy engine), issued first so that its L2
            // latency overlaps the int8 wait and the conversion
            if (!warp_wait(&emptyA[sa], ((i / SA) & 1) ^ 1, a.err, OMC_SITE_GEMM_DEQUANT, abort_flag)) break;
            {
                uint8_t *dst = smem + OFF_A + sa * A_BYTES;
                if (PHASE == 1) {
                    // gather: operand row j of the item is token xrow[j] of xh (its
                    // routed slot's token, or every token for the shared expert);
                    // padding rows are zero-filled.  Chunk ch = gt + GTHREADS*u of the
                    // tile is row (gt >> 3) + (GTHREADS/8)*u, 16-byte column gt & 7.
                    if (pr.idx != xrow_item) {
                        xrow_item = pr.idx;
#pragma unroll
                        for (int u = 0; u < XR; ++u) {
                            const int j = (gt >> 3) + (GTHREADS / 8) * u;
                            int t = -1;
                            if (j < pr.n) {
                                const int slot = a.rowinfo[pr.n0 + j];
                                t = slot < 0 ? -1
                                             : (a.slot_tok ? a.slot_tok[slot]
                                                           : (slot < a.nrouted ? slot / a.K : slot - a.nrouted));
                            }
                            xrow[u] = t;
                        }
                    }
                    const int c = gt & 7;
                    const uint8_t *xcol = reinterpret_cast<const uint8_t *>(a.xh) + (size_t)pr.kb * 128 + c * 16;
#pragma unroll
                    for (int u = 0; u < XR; ++u) {
                        const int j = (gt >> 3) + (GTHREADS / 8) * u;
                        if (j >= pr.n) break;
                        const bool live = xrow[u] >= 0;
                        const uint8_t *src = live ? xcol + (size_t)xrow[u] * (size_t)L.D * 2 : xcol;
                        cp_async16_zfill_hint(dst + j * 128 + ((c ^ (j & 7)) << 4), src, live, keep);
                    }
                } else {
                    const uint8_t *src = reinterpret_cast<const uint8_t *>(a.act) + (size_t)pr.kb * a.R * 128 +
                                         (size_t)pr.n0 * 128;
                    for (int ch = gt; ch < pr.n * 8; ch += GTHREADS)
                        cp_async16_hint(dst + ch * 16, src + ch * 16, keep);
                }
                cp_async_commit();
            }
            if (!warp_wait(&fullI[si], (i / SI) & 1, a.err, OMC_SITE_GEMM_DEQUANT, abort_flag)) break;
            if (!warp_wait(&emptyT[st], ((i / ST) & 1) ^ 1, a.err, OMC_SITE_GEMM_DEQUANT, abort_flag)) break;
            tc_fence_after();
            // both tiles of the pair, one after the other through the same registers:
            // 64 int8 of row r -> exact f16 -> TMEM columns 32*tile.. of stage st
            const uint8_t *m0 = smem + OFF_I8 + si * 2 * W_BYTES;
            if (PHASE == 2 && a.wf16) {
                // f16 weights: 8 chunks of 8 columns of row r, as they are
                uint32_t v[32];
#pragma unroll
                for (int c8 = 0; c8 < 8; ++c8) {
                    const uint4 hv = *reinterpret_cast<const uint4 *>(m0 + (c8 * 128 + r) * 16);
                    v[4 * c8 + 0] = hv.x;
                    v[4 * c8 + 1] = hv.y;
                    v[4 * c8 + 2] = hv.z;
                    v[4 * c8 + 3] = hv.w;
                }
                tmem_st_32x32b_x32(tmem + lane_bits + TCOL_A + (uint32_t)st * 64u, v);
                tc_wait_st();
            }
            for (int tile = 0; tile < (PHASE == 2 && a.wf16 ? 0 : pr.nmat); ++tile) {   // warp-uniform
                uint32_t v[32];
                const uint8_t *m = m0 + tile * W_BYTES;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {   // 16 int8 of K per chunk -> TMEM columns 8cc..8cc+7
                    const uint4 qv = *reinterpret_cast<const uint4 *>(m + (cc * 128 + r) * 16);
                    i8x4_to_f16x4(qv.x, v[8 * cc + 0], v[8 * cc + 1]);
                    i8x4_to_f16x4(qv.y, v[8 * cc + 2], v[8 * cc + 3]);
                    i8x4_to_f16x4(qv.z, v[8 * cc + 4], v[8 * cc + 5]);
                    i8x4_to_f16x4(qv.w, v[8 * cc + 6], v[8 * cc + 7]);
                }
                tmem_st_32x32b_x32(tmem + lane_bits + TCOL_A + (uint32_t)st * 64u + (uint32_t)tile * 32u, v);
                tc_wait_st();
            }
            // every int8 byte of the slot this warp reads is in TMEM now: release it
            __syncwarp();
            if (lane == 0) mbar_arrive(&emptyI[si]);
            cp_async_wait_all();          // this thread's part of the token tile has landed ...
            fence_proxy_async_smem();     // ... and is visible to the tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&fullT[st]);
            for (int j = 0; j < NGRP; ++j) pr.step(c);
        }
    } else if (warp < WARP_I8) {
        // ------------------------------------------------ epilogue: one weight row per thread
        const int e = warp - WARP_EPI0;          // 0..7
        const int q = warp & 3;                  // TMEM lane quarter
        const int half = e >> 2;                 // phase 1: token chunks of this parity; phase 2: tile
        const int r = q * 32 + lane;             // weight row within the tile = TMEM lane
        const uint32_t lane_bits = (uint32_t)(q * 32) << 16;
        uint8_t *stg = smem + OFF_STG;
        uint32_t ci = 0;
        AccSlots acc;
        int *tab_row = reinterpret_cast<int *>(smem + OFF_TAB + e * NMAX * 8);   // this warp's table
        float *tab_w = reinterpret_cast<float *>(tab_row + NMAX);
        for (int idx = blockIdx.x; idx < nitems && !*abort_flag; idx += gridDim.x, ++ci) {
            const WorkItem it = c.item(idx);
            if (!c.ok(it)) break;
            acc.begin(it.n);
            const omc_expert_ptrs P = L.experts[it.g];
            // fetch what the item needs before waiting for its accumulator
            float sc0 = 0.f, sc1 = 0.f;
            if (PHASE == 1) {
                const int Iw = it.g == L.E ? L.Is : L.I;
                const int f = it.mt * OMC_TM + r;
                if (f < Iw) {
                    sc0 = P.gs[f];
                    sc1 = P.us[f];
                }
            } else {
                const int d = item_row0(a, it, half) + r;
                if (half < item_nmat<PHASE>(a, it) && d < L.D) sc0 = P.ds[d];
                // per token row: its ypart row (token * (k+1) + choice, or the slot
                // itself when ydirect; -1 padding) and weight
                const int K = a.K;
                for (int j = lane; j < it.n; j += 32) {
                    const int slot = a.rowinfo[it.n0 + j];
                    int dst = -1;
                    if (slot >= 0 && a.ydirect) dst = slot;
                    else if (slot >= 0 && slot < a.nrouted) dst = slot / K * (K + 1) + slot % K;
                    else if (slot >= a.nrouted) dst = (slot - a.nrouted) * (K + 1) + K;
                    tab_row[j] = dst;
                    tab_w[j] = a.roww[it.n0 + j];
                }
                __syncwarp();
            }
            bool ok = true;
            for (int j = 0; j < acc.nslots && ok; ++j)
                ok = warp_wait(&accfull[acc.slot(j)], acc.parity(j), a.err, OMC_SITE_GEMM_EPILOGUE, abort_flag);
            if (!ok) break;
            tc_fence_after();
            if (PHASE == 1) {
                const int Iw = it.g == L.E ? L.Is : L.I;
                const int Iw_pad = it.g == L.E ? L.Is_pad : L.I_pad;
                const int f = it.mt * OMC_TM + r;                  // feature of this thread
                // staging of the previous item has been read by its bulk store
                if (!warp_wait(stgfree, (ci & 1) ^ 1, a.err, OMC_SITE_GEMM_EPILOGUE, abort_flag)) break;
                // staging: [64-feature half][token row][128 B, 16-byte chunks XOR-ed with row & 7]
                uint8_t *sbase = stg + (r >> 6) * (NMAX * 128) + (r & 7) * 2;
                const int chunk = (r & 63) >> 3;
                const int nch = it.n >> 4;
#pragma unroll 1
                bool outside = false;                              // an h value past the f16 range
                for (int ch = half; ch < nch; ch += 2) {
                    uint32_t gv[16], uv[16];
                    tmem_ld_32x32b_x16(tmem + lane_bits + acc.col(0) + ch * 16, gv);
                    tmem_ld_32x32b_x16(tmem + lane_bits + acc.col(1) + ch * 16, uv);
                    tc_wait_ld();
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int j = ch * 16 + jj;                // token row within the item
                        const float hv = f < Iw ? swiglu_f(L.act, __uint_as_float(gv[jj]) * sc0,
                                                           __uint_as_float(uv[jj]) * sc1)
                                                : 0.f;
                        outside |= omc_f16_outside(hv);
                        // operand row n0 + j; n0 % 16 == 0, so its swizzle phase is j & 7 = jj & 7
                        *reinterpret_cast<__half *>(sbase + j * 128 + ((chunk ^ (jj & 7)) << 4)) =
                            __float2half_rn(fminf(fmaxf(hv, -65504.f), 65504.f));
                    }
                }
                if (outside) omc_dev_error(a.err, OMC_DEVERR_RANGE, OMC_SITE_GEMM_EPILOGUE, it.g);
                tc_fence_before();
                fence_proxy_async_smem();                          // staging -> visible to the bulk store
                __syncwarp();
                if (lane == 0) {
                    for (int j = 0; j < acc.nslots; ++j) mbar_arrive(&accempty[acc.slot(j)]);
                    mbar_arrive(stgfull);
                }
                if (e == 0) {
                    // one thread writes the two 64-feature halves of the tile's h rows
                    if (!warp_wait(stgfull, ci & 1, a.err, OMC_SITE_GEMM_EPILOGUE, abort_flag)) break;
                    if (lane == 0) {
                        for (int kh = 0; kh < 2; ++kh) {
                            const int f0 = it.mt * OMC_TM + kh * 64;
                            if (f0 >= Iw_pad) break;
                            uint8_t *dst = reinterpret_cast<uint8_t *>(a.hout) +
                                           ((size_t)(f0 >> 6) * a.R + (size_t)it.n0) * 128;
                            bulk_s2g(dst, stg + kh * (NMAX * 128), (uint32_t)it.n * 128);
                        }
                        bulk_commit();
                        bulk_wait_read0();
                        mbar_arrive(stgfree);
                    }
                    __syncwarp();
                }
            } else {
                if (half < item_nmat<PHASE>(a, it)) {
                    const int d = item_row0(a, it, half) + r;       // output row of this thread
                    const uint32_t col = acc.col(half);
#pragma unroll 1
                    for (int ch = 0; ch * 16 < it.n; ++ch) {
                        uint32_t yv[16];
                        tmem_ld_32x32b_x16(tmem + lane_bits + col + ch * 16, yv);
                        tc_wait_ld();
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            const int dst = tab_row[ch * 16 + jj];
                            if (dst < 0 || d >= L.D) continue;
                            // matmul_q: acc * scale; then w * hh (w = 1 for the shared expert)
                            const float y = __fmul_rn(__uint_as_float(yv[jj]), sc0);
                            a.ypart[(size_t)dst * L.D + d] = __fmul_rn(tab_w[ch * 16 + jj], y);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    for (int j = 0; j < acc.nslots; ++j) mbar_arrive(&accempty[acc.slot(j)]);
            }
            acc.end();
        }
        if (PHASE == 1 && e == 0 && lane == 0) bulk_wait0();      // h rows written before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        tmem_dealloc(tmem, TMEM_COLS);
        tmem_relinquish();
    }
}

// -------------------------------------------------- explicit-rows pass ---
// f16 operand rows from f32 rows (saturated), 8 values per thread.
__global__ void __launch_bounds__(256) rows_to_f16_kernel(const float *__restrict__ x, long long n8,
                                                          uint16_t *__restrict__ xh, int *err) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
        const float4 a = reinterpret_cast<const float4 *>(x)[2 * i], b = reinterpret_cast<const float4 *>(x)[2 * i + 1];
        if (err && (omc_f16_outside(a.x) || omc_f16_outside(a.y) || omc_f16_outside(a.z) || omc_f16_outside(a.w) ||
                    omc_f16_outside(b.x) || omc_f16_outside(b.y) || omc_f16_outside(b.z) || omc_f16_outside(b.w)))
            omc_dev_error(err, OMC_DEVERR_RANGE, OMC_SITE_DISPATCH, (int)(i >> 20));
        uint4 o;
        o.x = f32x2_to_f16x2_sat(a.x, a.y);
        o.y = f32x2_to_f16x2_sat(a.z, a.w);
        o.z = f32x2_to_f16x2_sat(b.x, b.y);
        o.w = f32x2_to_f16x2_sat(b.z, b.w);
        reinterpret_cast<uint4 *>(xh)[i] = o;
    }
}

// The dispatch plan of an explicit-rows pass, as one block.
__global__ void __launch_bounds__(1024) plan_rows_kernel(omc_plan_args p, const int32_t *__restrict__ ids,
                                                         const float *__restrict__ w, int *err) {
    __shared__ int smem[OMC_PLAN_SMEM_INTS];
    omc_plan_block(p, ids, w, err, smem);
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

// Dense pass (omm_dense_q): the operand rows are the S input rows in order.
// Writes rowinfo/roww (row r < S is slot r with weight 1, padding rows -1),
// the f16 operand of the down GEMM in the AOL layout (element (r, k) at
// (k/64)*R*128 + r*128 + ((k%64)/8 ^ (r&7))*16 + (k%8)*2; columns >= K and
// rows >= S zero) and the work items (matrix 0, row-tile pair p, 128-row
// chunks of the Sp padded rows).
__global__ void __launch_bounds__(256) dense_prep_kernel(const float *__restrict__ x, int S, int K, int K_pad, int Sp,
                                                         int R, uint16_t *__restrict__ act, int *__restrict__ rowinfo,
                                                         float *__restrict__ roww, int4 *__restrict__ work,
                                                         int *__restrict__ nwork, int npairs, int *err) {
    const int stride = gridDim.x * blockDim.x, tid0 = blockIdx.x * blockDim.x + threadIdx.x;
    for (int r = tid0; r < Sp; r += stride) {
        rowinfo[r] = r < S ? r : -1;
        roww[r] = r < S ? 1.f : 0.f;
    }
    const long long nck = (long long)Sp * (K_pad / 8);
    for (long long i = tid0; i < nck; i += stride) {
        const int r = (int)(i % Sp), kc = (int)(i / Sp), k0 = kc * 8, kb = k0 >> 6, c = (k0 & 63) >> 3;
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (r < S && k0 < K) {
            const float4 a = *reinterpret_cast<const float4 *>(x + (size_t)r * K + k0);
            const float4 b = *reinterpret_cast<const float4 *>(x + (size_t)r * K + k0 + 4);
            if (omc_f16_outside(a.x) || omc_f16_outside(a.y) || omc_f16_outside(a.z) || omc_f16_outside(a.w) ||
                omc_f16_outside(b.x) || omc_f16_outside(b.y) || omc_f16_outside(b.z) || omc_f16_outside(b.w))
                omc_dev_error(err, OMC_DEVERR_RANGE, OMC_SITE_DISPATCH, r);
            o.x = f32x2_to_f16x2_sat(a.x, a.y);
            o.y = f32x2_to_f16x2_sat(a.z, a.w);
            o.z = f32x2_to_f16x2_sat(b.x, b.y);
            o.w = f32x2_to_f16x2_sat(b.z, b.w);
        }
        *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(act) + (size_t)kb * R * 128 + (size_t)r * 128 +
                                   ((c ^ (r & 7)) << 4)) = o;
    }
    if (blockIdx.x == 0) {
        const int nch = (Sp + NMAX - 1) / NMAX;
        for (int j = threadIdx.x; j < nch * npairs; j += blockDim.x) {
            const int ch = j / npairs, p = j - ch * npairs, n0 = ch * NMAX;
            work[j] = make_int4(0, p, n0, min(NMAX, Sp - n0));
        }
        if (threadIdx.x == 0) {
            nwork[0] = 0;
            nwork[1] = nch * npairs;
        }
    }
}

// Once per process: the GEMM's shared-memory attribute and the SM count.
static int gemm_setup() {
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
    return 0;
}

extern "C" int omc_launch_mma_ffn(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                                  const int32_t *topk_idx, const float *topk_w, float *out, cudaStream_t s) {
    if (T <= 0) return 0;
    if (L->D % 4) return OMC_EUNSUPPORTED;
    if (gemm_setup()) return OMC_ECUDA;
    const int R = ws->R_cap;
    omc_plan_args pa;                      // built on the device by the router's last select block
    omc_plan_setup(L, T, ws, &pa);
    const int4 *work1 = reinterpret_cast<const int4 *>(pa.work1), *work2 = reinterpret_cast<const int4 *>(pa.work2);

    GemmArgs ga;
    ga.L = *L;
    ga.work = work1;
    ga.nwork = ws->nwork;
    ga.act = ws->hp;
    ga.xh = ws->xh;
    ga.hout = ws->hp;
    ga.ypart = ws->ypart;
    ga.rowinfo = ws->rowinfo;
    ga.roww = ws->roww;
    ga.K = L->k;
    ga.nrouted = T * L->k;
    ga.ydirect = 0;
    ga.slot_tok = nullptr;
    ga.wf16 = 0;
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
    omc_g_launches += 3;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// Test hook: a smaller operand-row capacity for the dispatch plans that follow
// (0 = the workspace's).  The workspace always has room for every routed row,
// so only this reaches the plan's capacity check, which must end the forward
// with an error status and no out-of-range access.
static int g_plan_rows_limit = 0;

extern "C" int omc_debug_plan_rows(int rows) {
    if (rows < 0) return OMC_EINVAL;
    g_plan_rows_limit = rows;
    omc_graphs_invalidate();
    return 0;
}

extern "C" void omc_plan_setup(const omc_layer_dev *L, int T, const omc_ws *ws, omc_plan_args *pa) {
    const int E = L->E, G = E + (L->has_shared ? 1 : 0);
    const int R = g_plan_rows_limit > 0 && g_plan_rows_limit < ws->R_cap ? g_plan_rows_limit : ws->R_cap;
    const int Imax_rows = L->has_shared && L->Is_rows > L->I_rows ? L->Is_rows : L->I_rows;
    const int chunks_max = R / NMAX + G;
    pa->E = E;
    pa->K = L->k;
    pa->T = T;
    pa->has_shared = L->has_shared;
    pa->rows_mode = 0;
    pa->e_lo = 0;
    pa->e_hi = E;
    pa->I_rows = L->I_rows;
    pa->Is_rows = L->Is_rows;
    pa->D_rows = L->D_rows;
    pa->R_cap = R;
    pa->cap1 = chunks_max * (Imax_rows / OMC_TM);
    pa->cap2 = chunks_max * ((L->D_rows / OMC_TM + 1) / 2);
    pa->counts = ws->counts;
    pa->offsets = ws->offsets;
    pa->nwork = ws->nwork;
    pa->slotrow = ws->slotrow;
    pa->work1 = ws->work;
    pa->work2 = ws->work + 4 * (size_t)pa->cap1;
    pa->done = ws->done;
    pa->rowinfo = ws->rowinfo;
    pa->roww = ws->roww;
}

// Explicit-rows pass (expert parallelism: rows received from other ranks):
// y[r] = w[r] * expert ids[r] (x[r]) for R rows of D f32, through the same
// plan and grouped GEMMs as a forward.  ids must be resident experts
// [e_lo, e_hi), or E for the shared expert.
extern "C" int omc_launch_mma_rows(const omc_layer_dev *L, const float *x, int R, const omc_ws *ws,
                                   const int32_t *ids, const float *w, int e_lo, int e_hi, float *y,
                                   cudaStream_t s) {
    if (R <= 0) return 0;
    if (gemm_setup()) return OMC_ECUDA;
    const long long n8 = (long long)R * L->D / 8;
    if (L->family == OMC_FAMILY_GEMMA) {   // residual rows: the experts' input norm first
        const int rc = omc_launch_gemma_prenorm(L, x, R, nullptr, nullptr, ws->xh, nullptr, ws->err, s);
        if (rc) return rc;
    } else {
        rows_to_f16_kernel<<<(int)((n8 + 255) / 256 < 4096 ? (n8 + 255) / 256 : 4096), 256, 0, s>>>(x, n8, ws->xh,
                                                                                                   ws->err);
    }
    omc_plan_args pa;
    omc_plan_setup(L, R, ws, &pa);
    pa.K = 1;
    pa.rows_mode = 1;
    pa.e_lo = e_lo;
    pa.e_hi = e_hi;
    plan_rows_kernel<<<1, 1024, 0, s>>>(pa, ids, w, ws->err);
    omc_prof_mark(s, "dispatch");
    GemmArgs ga;
    ga.L = *L;
    ga.work = reinterpret_cast<const int4 *>(pa.work1);
    ga.nwork = ws->nwork;
    ga.act = ws->hp;
    ga.xh = ws->xh;
    ga.hout = ws->hp;
    ga.ypart = y;
    ga.rowinfo = ws->rowinfo;
    ga.roww = ws->roww;
    ga.K = 1;
    ga.nrouted = R;
    ga.ydirect = 1;
    ga.slot_tok = nullptr;
    ga.wf16 = 0;
    ga.T = R;
    ga.R = ws->R_cap;
    ga.err = ws->err;
    const int grid = g_num_sms > 0 ? g_num_sms : 148;
    moe_gemm_kernel<1><<<grid, NTHREADS, SMEM_BYTES, s>>>(ga);
    omc_prof_mark(s, "gemm_gateup");
    ga.work = reinterpret_cast<const int4 *>(pa.work2);
    moe_gemm_kernel<2><<<grid, NTHREADS, SMEM_BYTES, s>>>(ga);
    omc_prof_mark(s, "gemm_down");
    omc_g_launches += L->family == OMC_FAMILY_GEMMA ? 3 : 4;   // prenorm counts itself
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// Expert-parallel pass over explicit slots: slot s multiplies operand row
// slot_tok[s] of xh (f16 [rows][D], already converted) by expert slot_e[s]
// (a resident routed expert, or E for the shared expert) and writes
// y[s] = slot_w[s] * expert(x) (rounded as the forward rounds w * y).  The
// slots were counted into their groups already (ws->counts, ws->slotrow,
// one atomic each, by ep_unpack_kernel); this builds the rest of the plan
// (one block), the operand rows, and runs the two grouped GEMMs.
__global__ void __launch_bounds__(1024) plan_counted_kernel(omc_plan_args p, const int32_t *__restrict__ ids,
                                                            const float *__restrict__ w, int *err) {
    __shared__ int smem[OMC_PLAN_SMEM_INTS];
    omc_plan_block(p, ids, w, err, smem, true);
}

extern "C" int omc_launch_mma_slots(const omc_layer_dev *L, const uint16_t *xh, int nslots, const int32_t *slot_tok,
                                    const int32_t *slot_e, const float *slot_w, const omc_ws *ws, int e_lo, int e_hi,
                                    float *y, cudaStream_t s) {
    if (nslots <= 0) return 0;
    if (gemm_setup()) return OMC_ECUDA;
    omc_plan_args pa;
    omc_plan_setup(L, nslots, ws, &pa);
    pa.K = 1;
    pa.rows_mode = 1;
    pa.e_lo = e_lo;
    pa.e_hi = e_hi;
    plan_counted_kernel<<<1, 1024, 0, s>>>(pa, slot_e, slot_w, ws->err);
    omc_plan_fill_rows<<<(nslots + 255) / 256, 256, 0, s>>>(pa, slot_e, slot_w);
    omc_prof_mark(s, "dispatch");
    GemmArgs ga;
    ga.L = *L;
    ga.work = reinterpret_cast<const int4 *>(pa.work1);
    ga.nwork = ws->nwork;
    ga.act = ws->hp;
    ga.xh = xh;
    ga.hout = ws->hp;
    ga.ypart = y;
    ga.rowinfo = ws->rowinfo;
    ga.roww = ws->roww;
    ga.K = 1;
    ga.nrouted = nslots;
    ga.ydirect = 1;
    ga.slot_tok = slot_tok;
    ga.wf16 = 0;
    ga.T = nslots;
    ga.R = ws->R_cap;
    ga.err = ws->err;
    const int grid = g_num_sms > 0 ? g_num_sms : 148;
    moe_gemm_kernel<1><<<grid, NTHREADS, SMEM_BYTES, s>>>(ga);
    omc_prof_mark(s, "gemm_gateup");
    ga.work = reinterpret_cast<const int4 *>(pa.work2);
    moe_gemm_kernel<2><<<grid, NTHREADS, SMEM_BYTES, s>>>(ga);
    omc_prof_mark(s, "gemm_down");
    omc_g_launches += 4;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// ------------------------------------------ job-driven pass (omm_moe) ---
namespace {
// rows[r] = x[pos[r]] (D floats, a multiple of 4).
__global__ void __launch_bounds__(256) gather_rows_kernel(const float *__restrict__ x, const int *__restrict__ pos,
                                                          int R, int S, int D, float *__restrict__ rows, int *err) {
    const int r = blockIdx.y;
    const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (r >= R || d >= D) return;
    const int p = pos[r];
    if (p < 0 || p >= S) {
        if (d == 0) omc_dev_error(err, OMC_DEVERR_BOUNDS, OMC_SITE_DISPATCH, r);
        return;
    }
    *reinterpret_cast<float4 *>(rows + (size_t)r * D + d) = *reinterpret_cast<const float4 *>(x + (size_t)p * D + d);
}

// out[s] += y[list[j]] for j in [off[s], off[s+1]), in that order (the jobs'
// order): each element is one sequential fp32 chain, so the sums are
// deterministic.
__global__ void __launch_bounds__(256) ordered_add_kernel(float *__restrict__ out, const float *__restrict__ y,
                                                          const int *__restrict__ off, const int *__restrict__ list,
                                                          int S, int D) {
    const int s = blockIdx.y;
    const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (s >= S || d >= D) return;
    float4 acc = *reinterpret_cast<const float4 *>(out + (size_t)s * D + d);
    for (int j = off[s]; j < off[s + 1]; ++j) {
        const float4 v = *reinterpret_cast<const float4 *>(y + (size_t)list[j] * D + d);
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    *reinterpret_cast<float4 *>(out + (size_t)s * D + d) = acc;
}
}  // namespace

extern "C" int omc_launch_gather_rows(const float *x, const int *pos, int R, int S, int D, float *rows, int *err,
                                      cudaStream_t s) {
    if (R <= 0) return 0;
    gather_rows_kernel<<<dim3((D / 4 + 255) / 256, R), 256, 0, s>>>(x, pos, R, S, D, rows, err);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

extern "C" int omc_launch_ordered_add(float *out, const float *y, const int *off, const int *list, int S, int D,
                                      cudaStream_t s) {
    if (S <= 0) return 0;
    ordered_add_kernel<<<dim3((D / 4 + 255) / 256, S), 256, 0, s>>>(out, y, off, list, S, D);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// y[S][N] = x[S][K] . (ds * Wd)^T for the one-matrix layer L (its expert 0's
// down matrix, D = N output rows, I = K): the down GEMM with every row its own
// slot (ydirect) and weight 1.  x is f32 [S][K] on the device (K % 64 == 0),
// y f32 [S][N]; the workspace was sized for S rows.
extern "C" int omc_launch_dense_i8(const omc_layer_dev *L, const float *x, int S, const omc_ws *ws, float *y,
                                   cudaStream_t s) {
    if (S <= 0) return 0;
    if (gemm_setup()) return OMC_ECUDA;
    const int Sp = (S + OMC_ROW_ALIGN - 1) / OMC_ROW_ALIGN * OMC_ROW_ALIGN;
    if (Sp > ws->R_cap || (L->I % 64) || L->E != 1) return OMC_EINVAL;
    const int npairs = (L->D_rows / OMC_TM + 1) / 2;
    const long long nck = (long long)Sp * (L->I_pad / 8);
    const int blocks = (int)((nck + 255) / 256 < 2048 ? (nck + 255) / 256 : 2048);
    dense_prep_kernel<<<blocks, 256, 0, s>>>(x, S, L->I, L->I_pad, Sp, ws->R_cap, ws->hp, ws->rowinfo, ws->roww,
                                             reinterpret_cast<int4 *>(ws->work), ws->nwork, npairs, ws->err);
    GemmArgs ga;
    ga.L = *L;
    ga.work = reinterpret_cast<const int4 *>(ws->work);
    ga.nwork = ws->nwork;
    ga.act = ws->hp;
    ga.xh = nullptr;
    ga.hout = ws->hp;
    ga.ypart = y;
    ga.rowinfo = ws->rowinfo;
    ga.roww = ws->roww;
    ga.K = 1;
    ga.nrouted = S;
    ga.ydirect = 1;
    ga.slot_tok = nullptr;
    ga.wf16 = 0;
    ga.T = S;
    ga.R = ws->R_cap;
    ga.err = ws->err;
    const int grid = g_num_sms > 0 ? g_num_sms : 148;
    moe_gemm_kernel<2><<<grid, NTHREADS, SMEM_BYTES, s>>>(ga);
    omc_g_launches += 2;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// f16 weight tiles of a row-major f32 matrix W [N][K] (omm_dense): tile t
// (rows 128t..128t+127), K block kb (64 columns) is 16 KB at
// ((t * nkb + kb) * 16384); inside it, 8-column chunk c of row r sits at
// (c * 128 + r) * 16, so a warp reading 32 consecutive rows' chunk reads 512
// contiguous bytes.  Rounded to nearest; rows >= N and columns >= K are zero;
// a value outside the f16 range is reported (OMC_DEVERR_RANGE).
__global__ void __launch_bounds__(256) f16_tiles_kernel(const float *__restrict__ W, int N, int K, int nkb,
                                                        long long nchunks, uint16_t *__restrict__ dst, int *err) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nchunks;
         i += (long long)gridDim.x * blockDim.x) {
        // i = ((t * nkb + kb) * 8 + c) * 128 + r: consecutive threads write consecutive 16 B
        const int r = (int)(i & 127), c = (int)((i >> 7) & 7);
        const long long tk = i >> 10;
        const int kb = (int)(tk % nkb), t = (int)(tk / nkb);
        const int row = t * OMC_TM + r, k0 = kb * OMC_KB + c * 8;
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (row < N && k0 < K) {
            const float4 a = *reinterpret_cast<const float4 *>(W + (size_t)row * K + k0);
            const float4 b = *reinterpret_cast<const float4 *>(W + (size_t)row * K + k0 + 4);
            if (omc_f16_outside(a.x) || omc_f16_outside(a.y) || omc_f16_outside(a.z) || omc_f16_outside(a.w) ||
                omc_f16_outside(b.x) || omc_f16_outside(b.y) || omc_f16_outside(b.z) || omc_f16_outside(b.w))
                omc_dev_error(err, OMC_DEVERR_RANGE, OMC_SITE_DISPATCH, row);
            o.x = f32x2_to_f16x2_sat(a.x, a.y);
            o.y = f32x2_to_f16x2_sat(a.z, a.w);
            o.z = f32x2_to_f16x2_sat(b.x, b.y);
            o.w = f32x2_to_f16x2_sat(b.z, b.w);
        }
        reinterpret_cast<uint4 *>(dst)[i] = o;
    }
}

extern "C" size_t omc_f16_tiles_bytes(int N, int K) {
    return (size_t)((N + OMC_TM - 1) / OMC_TM) * ((K + OMC_KB - 1) / OMC_KB) * 16384;
}

extern "C" int omc_launch_f16_tiles(const float *W, int N, int K, uint16_t *dst, int *err, cudaStream_t s) {
    if (N <= 0 || K <= 0 || K % 8) return OMC_EINVAL;
    const int nkb = (K + OMC_KB - 1) / OMC_KB;
    const long long nchunks = (long long)omc_f16_tiles_bytes(N, K) / 16;
    const int blocks = (int)((nchunks + 255) / 256 < 8192 ? (nchunks + 255) / 256 : 8192);
    f16_tiles_kernel<<<blocks, 256, 0, s>>>(W, N, K, nkb, nchunks, dst, err);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// y[S][N] = x[S][K] . W^T on the tensor cores with f16 weights (omm_dense):
// L is a one-matrix layer (E = 1, D = N output rows, I = K) whose expert 0
// has d = the f16 tiles (omc_launch_f16_tiles) and ds = N_pad ones; x is f32
// [S][K] on the device (K % 8 == 0), rounded to f16 as the operand; the
// products are summed in f32 (TMEM).  The workspace was sized for S rows.
extern "C" int omc_launch_dense_f16(const omc_layer_dev *L, const float *x, int S, const omc_ws *ws, float *y,
                                    cudaStream_t s) {
    if (S <= 0) return 0;
    if (gemm_setup()) return OMC_ECUDA;
    const int Sp = (S + OMC_ROW_ALIGN - 1) / OMC_ROW_ALIGN * OMC_ROW_ALIGN;
    if (Sp > ws->R_cap || (L->I % 8) || L->E != 1) return OMC_EINVAL;
    const int ntiles = L->D_rows / OMC_TM;
    const long long nck = (long long)Sp * (L->I_pad / 8);
    const int blocks = (int)((nck + 255) / 256 < 2048 ? (nck + 255) / 256 : 2048);
    dense_prep_kernel<<<blocks, 256, 0, s>>>(x, S, L->I, L->I_pad, Sp, ws->R_cap, ws->hp, ws->rowinfo, ws->roww,
                                             reinterpret_cast<int4 *>(ws->work), ws->nwork, ntiles, ws->err);
    GemmArgs ga;
    ga.L = *L;
    ga.work = reinterpret_cast<const int4 *>(ws->work);
    ga.nwork = ws->nwork;
    ga.act = ws->hp;
    ga.xh = nullptr;
    ga.hout = ws->hp;
    ga.ypart = y;
    ga.rowinfo = ws->rowinfo;
    ga.roww = ws->roww;
    ga.K = 1;
    ga.nrouted = S;
    ga.ydirect = 1;
    ga.slot_tok = nullptr;
    ga.wf16 = 1;
    ga.T = S;
    ga.R = ws->R_cap;
    ga.err = ws->err;
    const int grid = g_num_sms > 0 ? g_num_sms : 148;
    moe_gemm_kernel<2><<<grid, NTHREADS, SMEM_BYTES, s>>>(ga);
    omc_g_launches += 2;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// y[r][n] = act row r . W row n (f16 products summed in f32 in tensor memory)
// over an operand that a caller already laid out: act in the AOL layout with
// R rows, rowinfo / roww / the work items / nwork written by that caller (the
// bounded router's prep kernel).  Ld is a one-matrix layer (E = 1, D = the
// output rows, I = K) whose expert 0 has d = f16 tiles and ds = ones.
extern "C" int omc_launch_gemm_dense_op(const omc_layer_dev *Ld, const uint16_t *act, int R, const int *rowinfo,
                                        const float *roww, const int *work, const int *nwork, float *y, int *err,
                                        cudaStream_t s) {
    if (gemm_setup()) return OMC_ECUDA;
    if (Ld->E != 1 || (Ld->I % 8) || (R % OMC_ROW_ALIGN)) return OMC_EINVAL;
    GemmArgs ga;
    ga.L = *Ld;
    ga.work = reinterpret_cast<const int4 *>(work);
    ga.nwork = nwork;
    ga.act = act;
    ga.xh = nullptr;
    ga.hout = nullptr;
    ga.ypart = y;
    ga.rowinfo = rowinfo;
    ga.roww = roww;
    ga.K = 1;
    ga.nrouted = R;
    ga.ydirect = 1;
    ga.slot_tok = nullptr;
    ga.wf16 = 1;
    ga.T = R;
    ga.R = R;
    ga.err = err;
    const int grid = g_num_sms > 0 ? g_num_sms : 148;
    moe_gemm_kernel<2><<<grid, NTHREADS, SMEM_BYTES, s>>>(ga);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// dst[i] = f16(src[i]) (round to nearest, saturated) for n a multiple of 8,
// both 16-byte aligned.
extern "C" int omc_launch_f32_to_f16(const float *src, long long n, uint16_t *dst, cudaStream_t s) {
    if (n <= 0) return 0;
    if (n % 8) return OMC_EINVAL;
    const long long n8 = n / 8;
    rows_to_f16_kernel<<<(int)((n8 + 255) / 256 < 4096 ? (n8 + 255) / 256 : 4096), 256, 0, s>>>(src, n8, dst,
                                                                                                 nullptr);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}
