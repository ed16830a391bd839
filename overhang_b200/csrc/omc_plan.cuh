// omc_plan.cuh -- the dispatch plan of a tensor-core forward, built on the
// device by one block once every token's routing is known.
//
// The reference gathers, per prefill batch, the union of the experts its
// tokens chose and runs each expert over its tokens (engines/olmoe.c:366-378).
// Here that union becomes: per group g (routed expert, or the shared expert
// as group E with every token), its row count, a 16-row-padded row range in
// the activation operand, each routed slot's row inside it, and the work
// items of the two grouped GEMMs.
#pragma once
#include "omc_common.cuh"

// Shared-memory ints the plan needs (four arrays over the groups).
constexpr int OMC_PLAN_SMEM_INTS = 4 * (OMC_MAX_E + 2);

// Run by every thread of one block (any size that is a multiple of 32).
// topk_idx [T][K] must be visible to the block.  smem: OMC_PLAN_SMEM_INTS.
//
// counted = false: the block also counts the routed slots per expert (their
// ranks into p.slotrow) and writes every operand row's slot and weight; one
// block does all of it (the explicit-rows pass).  counted = true: the router's
// select blocks have counted already (p.counts[e] = routed rows of e, every
// slot's rank in p.slotrow, one global atomic per slot), and the rows are
// written afterwards by omc_plan_fill_rows over all slots; the block does the
// scans, the offsets, the work lists and the padding rows.
__device__ inline void omc_plan_block(const omc_plan_args &p, const int32_t *__restrict__ topk_idx,
                                      const float *__restrict__ topk_w, int *err, int *smem, bool counted = false) {
    int *s_cnt = smem, *s_off = s_cnt + (OMC_MAX_E + 2), *s_w1 = s_off + (OMC_MAX_E + 2),
        *s_w2 = s_w1 + (OMC_MAX_E + 2);
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31;
    const int E = p.E, G = E + (p.has_shared ? 1 : 0), nslots = p.T * p.K;
    for (int g = tid; g < G; g += nt) s_cnt[g] = (g < E || p.rows_mode) ? (counted ? __ldcg(p.counts + g) : 0) : p.T;
    __syncthreads();
    // rank of each routed slot within its expert (arrival order; the rows of
    // an expert are independent, so their order does not change any value).
    // Loads go out 8 at a time: one L2 round trip per 8 slots, not per slot.
    // The gather adds the expert's row offset.
    int *__restrict__ rank = p.slotrow;
    for (int base = tid; !counted && base < nslots; base += 8 * nt) {
        int e[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int s = base + u * nt;
            e[u] = s < nslots ? __ldg(topk_idx + s) : 0;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int s = base + u * nt;
            if (s >= nslots) break;
            int pos = -1;
            const bool ok = (e[u] >= p.e_lo && e[u] < p.e_hi) || (p.rows_mode && p.has_shared && e[u] == E);
            if (ok) pos = atomicAdd(&s_cnt[e[u]], 1);
            else omc_dev_error(err, OMC_DEVERR_ROUTE, OMC_SITE_DISPATCH, s);
            rank[s] = pos;
        }
    }
    __syncthreads();
    const int mt2 = (p.D_rows / OMC_TM + 1) / 2;
    for (int g = tid; g < G; g += nt) {
        const int c = s_cnt[g];
        const int pad = (c + OMC_ROW_ALIGN - 1) / OMC_ROW_ALIGN * OMC_ROW_ALIGN;
        const int nch = (pad + OMC_NMAX - 1) / OMC_NMAX;
        p.counts[g] = c;
        s_off[g] = pad;
        s_w1[g] = nch * ((g < E ? p.I_rows : p.Is_rows) / OMC_TM);
        s_w2[g] = nch * mt2;
    }
    __syncthreads();
    // exclusive scans over the groups (one warp, 32 groups per step)
    if (tid < 32) {
        int co = 0, c1 = 0, c2 = 0;
        for (int base = 0; base < G; base += 32) {
            const int g = base + lane;
            const int vo = g < G ? s_off[g] : 0, v1 = g < G ? s_w1[g] : 0, v2 = g < G ? s_w2[g] : 0;
            int io = vo, i1 = v1, i2 = v2;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, io, o), b = __shfl_up_sync(0xffffffffu, i1, o),
                          d = __shfl_up_sync(0xffffffffu, i2, o);
                if (lane >= o) {
                    io += a;
                    i1 += b;
                    i2 += d;
                }
            }
            if (g < G) {
                s_off[g] = co + io - vo;
                s_w1[g] = c1 + i1 - v1;
                s_w2[g] = c2 + i2 - v2;
            }
            co += __shfl_sync(0xffffffffu, io, 31);
            c1 += __shfl_sync(0xffffffffu, i1, 31);
            c2 += __shfl_sync(0xffffffffu, i2, 31);
        }
        if (lane == 0) {
            s_off[G] = co;
            s_w1[G] = c1;
            s_w2[G] = c2;
        }
    }
    __syncthreads();
    const bool okcap = s_off[G] <= p.R_cap && s_w1[G] <= p.cap1 && s_w2[G] <= p.cap2;
    if (tid == 0) {
        if (!okcap) omc_dev_error(err, OMC_DEVERR_BOUNDS, OMC_SITE_DISPATCH, s_off[G]);
        p.nwork[0] = okcap ? s_w1[G] : 0;
        p.nwork[1] = okcap ? s_w2[G] : 0;
        p.nwork[2] = s_off[G];
    }
    for (int g = tid; g <= G; g += nt) p.offsets[g] = s_off[g];
    if (!okcap) return;
    int4 *w1 = reinterpret_cast<int4 *>(p.work1), *w2 = reinterpret_cast<int4 *>(p.work2);
    for (int g = tid; g < G; g += nt) {
        const int pad = s_off[g + 1] - s_off[g];
        if (!pad) continue;
        const int nch = (pad + OMC_NMAX - 1) / OMC_NMAX;
        const int mt1 = (g < E ? p.I_rows : p.Is_rows) / OMC_TM;
        int q1 = s_w1[g], q2 = s_w2[g];
        for (int c = 0; c < nch; ++c) {
            const int n0 = s_off[g] + c * OMC_NMAX, n = min(OMC_NMAX, pad - c * OMC_NMAX);
            for (int m = 0; m < mt1; ++m) w1[q1++] = make_int4(g, m, n0, n);
            for (int m = 0; m < mt2; ++m) w2[q2++] = make_int4(g, m, n0, n);
        }
    }
    // operand rows: routed slot s -> row offsets[e] + rank, with its slot and
    // routing weight (the same thread wrote rank[s] above)
    for (int base = tid; !counted && base < nslots; base += 8 * nt) {
        int e[8], rk[8];
        float w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int s = base + u * nt;
            e[u] = s < nslots ? __ldg(topk_idx + s) : 0;
            w[u] = s < nslots ? __ldg(topk_w + s) : 0.f;
            rk[u] = s < nslots ? rank[s] : -1;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int s = base + u * nt;
            if (s >= nslots || rk[u] < 0) continue;
            const int row = s_off[e[u]] + rk[u];
            p.rowinfo[row] = s;
            p.roww[row] = w[u];
        }
    }
    if (p.has_shared && !p.rows_mode && !counted)   // the shared expert: token t at row offsets[E] + t, weight 1
        for (int t = tid; t < p.T; t += nt) {
            p.rowinfo[s_off[E] + t] = nslots + t;
            p.roww[s_off[E] + t] = 1.f;
        }
    for (int g = tid; g < G; g += nt)        // padding rows of each group
        for (int r = s_off[g] + s_cnt[g]; r < s_off[g + 1]; ++r) {
            p.rowinfo[r] = -1;
            p.roww[r] = 0.f;
        }
}

// The row pass of a counted plan, one thread per routed slot (then one per
// token for the shared expert): row offsets[e] + rank gets the slot and its
// routing weight.  Rows past the capacity are skipped (the plan reported the
// overflow and queued no work).
static __global__ void __launch_bounds__(256) omc_plan_fill_rows(omc_plan_args p, const int32_t *__restrict__ topk_idx,
                                                          const float *__restrict__ topk_w) {
    const int nslots = p.T * p.K, i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < nslots) {
        const int e = topk_idx[i], rk = p.slotrow[i];
        // explicit rows may name the shared expert (group E) themselves
        if (rk < 0 || e < 0 || e > p.E || (e == p.E && !(p.rows_mode && p.has_shared))) return;
        const int row = p.offsets[e] + rk;
        if (row >= p.R_cap) return;
        p.rowinfo[row] = i;
        p.roww[row] = topk_w[i];
    } else if (p.has_shared && !p.rows_mode && i < nslots + p.T) {
        const int t = i - nslots, row = p.offsets[p.E] + t;
        if (row >= p.R_cap) return;
        p.rowinfo[row] = nslots + t;
        p.roww[row] = 1.f;
    }
}
