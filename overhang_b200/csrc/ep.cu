// ep.cu -- device side of the expert-parallel MoE forward (one process per
// GPU, experts split into contiguous ranges; omc_ep.c drives it over NCCL).
//
// The reference runs the whole block on one CPU (engines/olmoe.c:344-402,
// engines/qwen.c:453-495); here its batch union (olmoe.c:366-378) spans ranks:
//
//   ep_layout_kernel   one block: per destination rank, the rows and slots
//                      each home token sends there, block-scanned into the
//                      packed send positions and the return positions of
//                      every routed slot (omc_ep_plan.h defines them)
//   ep_pack_kernel     a warp per token: x -> one f16 row per destination
//                      rank that holds any of its experts (rounded as the
//                      single-GPU tensor-core path rounds it), its meta row,
//                      and the f16 row the home's shared expert reads
//   ep_unpack_kernel   a thread per received row: its slots (operand row,
//                      expert, weight) numbered in the sender's return order,
//                      each counted into its expert's group
//   (then the grouped GEMMs of ffn_mma.cu over those slots)
//   ep_combine_kernel  out = [sigmoid gate * shared] + sum_k partial_k in
//                      selection order, from the returned partials: the
//                      reference's order (olmoe.c:395-397, qwen.c:459-492)
//
// Every product and sum is the single-GPU forward's own operation, so the
// result equals one GPU's tensor-core forward bit for bit.
#include "omc_common.cuh"
#include "omc_ep_plan.h"

namespace {

constexpr int EP_MAXR = OMC_EP_MAX_RANKS;

// Exclusive prefix of v over the block (1024 threads max) and its total.
__device__ int block_excl_scan(int v, int *s_w, int &total) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_w[wid] = x;
    __syncthreads();
    if (wid == 0) {
        int w = lane < nw ? s_w[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        s_w[lane] = w;
    }
    __syncthreads();
    total = s_w[nw - 1];
    const int ex = (wid > 0 ? s_w[wid - 1] : 0) + x - v;
    __syncthreads();   // s_w is reused by the next scan
    return ex;
}

// counts: [0,P) send_rows, [P,2P) send_slots, [2P,3P) send_base, [3P,4P)
// ret_base; pairs: (send_rows[r], send_slots[r]) at 2r, the counts exchange's
// send buffer.  Each thread walks a contiguous run of tokens, so positions
// follow token order exactly as omc_ep_layout_host computes them.
__global__ void __launch_bounds__(1024) ep_layout_kernel(const int32_t *__restrict__ idx, int T, int k, int ne, int P,
                                                          int32_t *__restrict__ tok_pos, int32_t *__restrict__ slot_pos,
                                                          int32_t *__restrict__ counts, int32_t *__restrict__ pairs) {
    __shared__ int s_w[32];
    __shared__ int s_base[2 * EP_MAXR];
    const int nt = blockDim.x, tid = threadIdx.x;
    const int per = (T + nt - 1) / nt;
    const int t0 = min(T, tid * per), t1 = min(T, t0 + per);
    int rows[EP_MAXR], slots[EP_MAXR], cnt[EP_MAXR];
    for (int r = 0; r < P; ++r) rows[r] = slots[r] = 0;
    for (int t = t0; t < t1; ++t) {
        omc_ep_token_counts(idx + (size_t)t * k, k, ne, P, cnt);
        for (int r = 0; r < P; ++r) {
            rows[r] += cnt[r] > 0;
            slots[r] += cnt[r];
        }
    }
    int row_before[EP_MAXR], slot_before[EP_MAXR];
    for (int r = 0; r < P; ++r) {
        int tot_r = 0, tot_s = 0;
        row_before[r] = block_excl_scan(rows[r], s_w, tot_r);
        slot_before[r] = block_excl_scan(slots[r], s_w, tot_s);
        if (tid == 0) {
            counts[r] = tot_r;
            counts[P + r] = tot_s;
            pairs[2 * r] = tot_r;
            pairs[2 * r + 1] = tot_s;
            s_base[r] = tot_r;
            s_base[EP_MAXR + r] = tot_s;
        }
    }
    __syncthreads();
    int send_base[EP_MAXR], ret_base[EP_MAXR];
    int ar = 0, as = 0;
    for (int r = 0; r < P; ++r) {
        send_base[r] = ar;
        ret_base[r] = as;
        ar += s_base[r];
        as += s_base[EP_MAXR + r];
    }
    if (tid == 0)
        for (int r = 0; r < P; ++r) {
            counts[2 * P + r] = send_base[r];
            counts[3 * P + r] = ret_base[r];
        }
    for (int t = t0; t < t1; ++t) {
        const int32_t *it = idx + (size_t)t * k;
        omc_ep_token_counts(it, k, ne, P, cnt);
        omc_ep_token_positions(it, k, ne, P, row_before, slot_before, send_base, ret_base, cnt,
                               tok_pos + (size_t)t * P, slot_pos + (size_t)t * k);
        for (int r = 0; r < P; ++r) {
            row_before[r] += cnt[r] > 0;
            slot_before[r] += cnt[r];
        }
    }
}

// A warp per token: one f16 row per destination (and for the home's shared
// expert), the meta rows.  x rows are D floats (D % 8 == 0).
__global__ void __launch_bounds__(256) ep_pack_kernel(const float *__restrict__ x, const int32_t *__restrict__ idx,
                                                       const float *__restrict__ w, int T, int D, int k, int ne, int P,
                                                       const int32_t *__restrict__ tok_pos,
                                                       const int32_t *__restrict__ slot_pos,
                                                       const int32_t *__restrict__ counts, uint16_t *__restrict__ send_x,
                                                       int32_t *__restrict__ send_meta, uint16_t *__restrict__ home_xh,
                                                       int *err) {
    const int lane = threadIdx.x & 31;
    const int nwarp = gridDim.x * (blockDim.x >> 5);
    const int M = omc_ep_meta_ints(k);
    for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += nwarp) {
        int pos[EP_MAXR];
        for (int r = 0; r < P; ++r) pos[r] = __ldg(tok_pos + (size_t)t * P + r);
        const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)t * D);
        bool outside = false;
        for (int c = lane; c < D / 8; c += 32) {
            const float4 a = __ldg(xr + 2 * c), b = __ldg(xr + 2 * c + 1);
            outside |= omc_f16_outside(a.x) || omc_f16_outside(a.y) || omc_f16_outside(a.z) || omc_f16_outside(a.w) ||
                       omc_f16_outside(b.x) || omc_f16_outside(b.y) || omc_f16_outside(b.z) || omc_f16_outside(b.w);
            uint4 o;
            o.x = f32x2_to_f16x2_sat(a.x, a.y);
            o.y = f32x2_to_f16x2_sat(a.z, a.w);
            o.z = f32x2_to_f16x2_sat(b.x, b.y);
            o.w = f32x2_to_f16x2_sat(b.z, b.w);
            for (int r = 0; r < P; ++r)
                if (pos[r] >= 0) reinterpret_cast<uint4 *>(send_x + (size_t)pos[r] * D)[c] = o;
            if (home_xh) reinterpret_cast<uint4 *>(home_xh + (size_t)t * D)[c] = o;
        }
        if (outside) omc_dev_error(err, OMC_DEVERR_RANGE, OMC_SITE_DISPATCH, t);
        if (lane < P && pos[lane] >= 0) {
            const int r = lane;
            const int32_t *it = idx + (size_t)t * k;
            int first = -1;
            for (int kk = 0; kk < k && first < 0; ++kk)
                if (it[kk] >= 0 && it[kk] / ne == r) first = kk;
            const int slot_in = __ldg(slot_pos + (size_t)t * k + first) - __ldg(counts + 3 * P + r);
            omc_ep_token_meta(it, w + (size_t)t * k, k, ne, r, slot_in, send_meta + (size_t)pos[r] * M);
        }
    }
}

struct EpBases {
    int P;
    int recv_base[EP_MAXR + 1];   // received rows: peer p's at [recv_base[p], recv_base[p+1])
    int slot_base[EP_MAXR + 1];   // their slots
};

// A thread per received row (its slots), then one per home token (its
// shared-expert slot).  Each slot's rank in its expert's group comes from one
// atomic on the plan's counts: an expert's rows are independent, so the
// arrival order changes no value.
__global__ void __launch_bounds__(256) ep_unpack_kernel(const int32_t *__restrict__ meta, int Rr, int k, EpBases b,
                                                         int Thome, int E, int e_lo, int e_hi, int has_shared, int Sr,
                                                         int32_t *__restrict__ slot_tok, int32_t *__restrict__ slot_e,
                                                         float *__restrict__ slot_w, int *__restrict__ counts_e,
                                                         int *__restrict__ slotrow, int *err) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int M = omc_ep_meta_ints(k);
    if (i < Rr) {
        const int p = omc_ep_row_peer(b.recv_base, b.P, i);
        const int32_t *m = meta + (size_t)i * M;
        const int n = m[1], base = b.slot_base[p] + m[0];
        if (n < 0 || n > k || m[0] < 0 || base + n > b.slot_base[p + 1]) {
            omc_dev_error(err, OMC_DEVERR_BOUNDS, OMC_SITE_DISPATCH, i);
            return;
        }
        for (int q = 0; q < n; ++q) {
            const int s = base + q, e = m[2 + q];
            slot_tok[s] = Thome + i;
            slot_e[s] = e;
            slot_w[s] = __int_as_float(m[2 + k + q]);
            if (e >= e_lo && e < e_hi) {
                slotrow[s] = atomicAdd(counts_e + e, 1);
            } else {
                slotrow[s] = -1;
                omc_dev_error(err, OMC_DEVERR_ROUTE, OMC_SITE_DISPATCH, s);
            }
        }
    } else if (has_shared && i - Rr < Thome) {
        const int t = i - Rr, s = Sr + t;
        slot_tok[s] = t;
        slot_e[s] = E;
        slot_w[s] = 1.f;
        slotrow[s] = atomicAdd(counts_e + E, 1);
    }
}

// out[t] = [sg[t] * y_shared[t]] + sum_kk ret[slot_pos[t][kk]], kk ascending:
// the single-GPU combine (combine_kernel in ffn_mma.cu) on the returned rows.
__global__ void __launch_bounds__(256) ep_combine_kernel(const float *__restrict__ ret,
                                                          const int32_t *__restrict__ slot_pos,
                                                          const float *__restrict__ y_shared,
                                                          const float *__restrict__ sg, int T, int D, int k,
                                                          int has_shared, float *__restrict__ out) {
    const int t = blockIdx.y;
    const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (t >= T || d >= D) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (has_shared) {
        const float4 s = *reinterpret_cast<const float4 *>(y_shared + (size_t)t * D + d);
        const float g = sg[t];
        acc = make_float4(__fmul_rn(s.x, g), __fmul_rn(s.y, g), __fmul_rn(s.z, g), __fmul_rn(s.w, g));
    }
    for (int kk = 0; kk < k; ++kk) {
        const int pos = slot_pos[(size_t)t * k + kk];
        if (pos < 0) continue;
        const float4 p = *reinterpret_cast<const float4 *>(ret + (size_t)pos * D + d);
        acc.x = __fadd_rn(acc.x, p.x);
        acc.y = __fadd_rn(acc.y, p.y);
        acc.z = __fadd_rn(acc.z, p.z);
        acc.w = __fadd_rn(acc.w, p.w);
    }
    *reinterpret_cast<float4 *>(out + (size_t)t * D + d) = acc;
}

// Per-rank-sum return (OMC_EP_RANKSUM): one f32 row per received token row,
// the sum of its slots' weighted partials on this rank in selection order.
// A thread per (row, 4 columns).
__global__ void __launch_bounds__(256) ep_ranksum_kernel(const int32_t *__restrict__ meta, int Rr, int k, EpBases b,
                                                          const float *__restrict__ y, int D, float *__restrict__ rows) {
    const int j = blockIdx.y;
    const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (j >= Rr || d >= D) return;
    const int M = omc_ep_meta_ints(k);
    const int p = omc_ep_row_peer(b.recv_base, b.P, j);
    const int32_t *m = meta + (size_t)j * M;
    const int base = b.slot_base[p] + m[0], n = m[1];
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < n; ++q) {
        const float4 v = *reinterpret_cast<const float4 *>(y + (size_t)(base + q) * D + d);
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    *reinterpret_cast<float4 *>(rows + (size_t)j * D + d) = acc;
}

// Home combine of per-rank sums: out = [sg * shared] + the row each rank
// returned, ranks taken in the order their first expert appears in the
// token's selection.
__global__ void __launch_bounds__(256) ep_combine_ranksum_kernel(const float *__restrict__ ret,
                                                                  const int32_t *__restrict__ tok_pos,
                                                                  const int32_t *__restrict__ idx,
                                                                  const float *__restrict__ y_shared,
                                                                  const float *__restrict__ sg, int T, int D, int k,
                                                                  int ne, int P, int has_shared,
                                                                  float *__restrict__ out) {
    const int t = blockIdx.y;
    const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (t >= T || d >= D) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (has_shared) {
        const float4 s = *reinterpret_cast<const float4 *>(y_shared + (size_t)t * D + d);
        const float g = sg[t];
        acc = make_float4(__fmul_rn(s.x, g), __fmul_rn(s.y, g), __fmul_rn(s.z, g), __fmul_rn(s.w, g));
    }
    unsigned seen = 0u;
    for (int kk = 0; kk < k; ++kk) {
        const int e = idx[(size_t)t * k + kk];
        const int r = e >= 0 ? e / ne : -1;
        if (r < 0 || r >= P || (seen >> r & 1u)) continue;
        seen |= 1u << r;
        const int pos = tok_pos[(size_t)t * P + r];
        if (pos < 0) continue;
        const float4 v = *reinterpret_cast<const float4 *>(ret + (size_t)pos * D + d);
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    *reinterpret_cast<float4 *>(out + (size_t)t * D + d) = acc;
}

}  // namespace

extern "C" int omc_launch_ep_layout(const int32_t *idx, int T, int k, int ne, int P, int32_t *tok_pos,
                                    int32_t *slot_pos, int32_t *counts, int32_t *pairs, cudaStream_t s) {
    if (P < 1 || P > EP_MAXR || T < 0) return OMC_EINVAL;
    ep_layout_kernel<<<1, 1024, 0, s>>>(idx, T, k, ne, P, tok_pos, slot_pos, counts, pairs);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

extern "C" int omc_launch_ep_pack(const float *x, const int32_t *idx, const float *w, int T, int D, int k, int ne,
                                  int P, const int32_t *tok_pos, const int32_t *slot_pos, const int32_t *counts,
                                  uint16_t *send_x, int32_t *send_meta, uint16_t *home_xh, int *err, cudaStream_t s) {
    if (T <= 0) return 0;
    if (D % 8 || P > EP_MAXR) return OMC_EINVAL;
    const int blocks = (T + 7) / 8 < 4096 ? (T + 7) / 8 : 4096;
    ep_pack_kernel<<<blocks, 256, 0, s>>>(x, idx, w, T, D, k, ne, P, tok_pos, slot_pos, counts, send_x, send_meta,
                                          home_xh, err);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

extern "C" int omc_launch_ep_unpack(const int32_t *meta, int Rr, int k, int P, const int *recv_base,
                                    const int *slot_base, int Thome, int E, int e_lo, int e_hi, int has_shared, int Sr,
                                    int32_t *slot_tok, int32_t *slot_e, float *slot_w, int *counts_e, int *slotrow,
                                    int *err, cudaStream_t s) {
    if (P > EP_MAXR) return OMC_EINVAL;
    EpBases b;
    b.P = P;
    for (int p = 0; p <= P; ++p) {
        b.recv_base[p] = recv_base[p];
        b.slot_base[p] = slot_base[p];
    }
    const int n = Rr + (has_shared ? Thome : 0);
    if (n <= 0) return 0;
    ep_unpack_kernel<<<(n + 255) / 256, 256, 0, s>>>(meta, Rr, k, b, Thome, E, e_lo, e_hi, has_shared, Sr, slot_tok,
                                                     slot_e, slot_w, counts_e, slotrow, err);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

extern "C" int omc_launch_ep_combine(const float *ret, const int32_t *slot_pos, const float *y_shared, const float *sg,
                                     int T, int D, int k, int has_shared, float *out, cudaStream_t s) {
    if (T <= 0) return 0;
    if (D % 4) return OMC_EINVAL;
    ep_combine_kernel<<<dim3((D / 4 + 255) / 256, T), 256, 0, s>>>(ret, slot_pos, y_shared, sg, T, D, k, has_shared,
                                                                  out);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

extern "C" int omc_launch_ep_ranksum(const int32_t *meta, int Rr, int k, int P, const int *recv_base,
                                     const int *slot_base, const float *y, int D, float *rows, cudaStream_t s) {
    if (Rr <= 0) return 0;
    if (P > EP_MAXR || D % 4) return OMC_EINVAL;
    EpBases b;
    b.P = P;
    for (int p = 0; p <= P; ++p) {
        b.recv_base[p] = recv_base[p];
        b.slot_base[p] = slot_base[p];
    }
    ep_ranksum_kernel<<<dim3((D / 4 + 255) / 256, Rr), 256, 0, s>>>(meta, Rr, k, b, y, D, rows);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

extern "C" int omc_launch_ep_combine_ranksum(const float *ret, const int32_t *tok_pos, const int32_t *idx,
                                             const float *y_shared, const float *sg, int T, int D, int k, int ne,
                                             int P, int has_shared, float *out, cudaStream_t s) {
    if (T <= 0) return 0;
    if (D % 4 || P > 32) return OMC_EINVAL;
    ep_combine_ranksum_kernel<<<dim3((D / 4 + 255) / 256, T), 256, 0, s>>>(ret, tok_pos, idx, y_shared, sg, T, D, k,
                                                                          ne, P, has_shared, out);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}
