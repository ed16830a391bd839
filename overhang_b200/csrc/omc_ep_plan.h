/* omc_ep_plan.h -- index arithmetic of the expert-parallel exchange, shared
 * by the device kernels (ep.cu) and the host versions the tests run
 * (omc_ep.c).  Internal; not part of the public ABI.
 *
 * P ranks split the E routed experts of a layer into contiguous ranges of
 * ne = E/P: expert e lives on rank e / ne.  Every rank brings T "home"
 * tokens with their routing idx[T][k] (selection order) and weights.
 *
 * Dispatch (home -> expert ranks).  A token is sent to rank r once if any of
 * its k experts lives there (one f16 row, whatever the number of its experts
 * on r), with a meta row naming those experts.  Rank r's rows form one block
 * of the packed send buffer, tokens in ascending order:
 *   cnt_r(t)      = #{kk : owner(idx[t][kk]) == r}
 *   send_rows[r]  = #{t : cnt_r(t) > 0}          send_base[r] = sum_{r'<r} send_rows[r']
 *   send_slots[r] = sum_t cnt_r(t)               ret_base[r]  = sum_{r'<r} send_slots[r']
 *   tok_pos[t][r] = send_base[r] + #{t' < t : cnt_r(t') > 0}, or -1 when cnt_r(t) == 0
 * Return (expert ranks -> home).  Every routed slot (t, kk) comes back as one
 * f32 row w_kk * expert(x_t), in the same block order: rank r's block of the
 * home's return buffer holds its slots token by token, kk ascending:
 *   slot_pos[t][kk] = ret_base[r] + sum_{t'<t} cnt_r(t') + #{kk' < kk : owner == r}
 * The meta row of the sent (t, r): [0] slot offset of t's first slot inside
 * r's block, [1] cnt_r(t), [2 .. 2+k) their expert ids in kk order (-1 pad),
 * [2+k .. 2+2k) their weights (float bits).
 *
 * Receiver.  Rows from peer p arrive contiguous at recv_base[p]; their slots
 * are numbered slot_base[p] + meta[0] + i, so the expert rank's slot order
 * per peer is the home's return order for that rank and the y rows of a peer
 * go back as one contiguous block.  The home's own shared-expert slots follow
 * all received ones.
 */
#ifndef OMC_EP_PLAN_H
#define OMC_EP_PLAN_H
#include <stdint.h>

#ifdef __CUDACC__
#define OMC_HD __host__ __device__ __forceinline__
#else
#define OMC_HD static inline
#endif

#define OMC_EP_MAX_RANKS 16

OMC_HD int omc_ep_meta_ints(int k) { return 2 + 2 * k; }

/* cnt[r] = experts of token row `idx` (k of them) on rank r, r < P. */
OMC_HD void omc_ep_token_counts(const int32_t *idx, int k, int ne, int P, int *cnt) {
    for (int r = 0; r < P; ++r) cnt[r] = 0;
    for (int kk = 0; kk < k; ++kk) {
        const int e = idx[kk];
        const int r = e >= 0 ? e / ne : -1;
        if (r >= 0 && r < P) cnt[r]++;
    }
}

/* Positions of one token given the running (per rank) row and slot offsets
 * before it and the block bases: tok_pos[P], slot_pos[k].  A slot whose
 * expert is outside [0, P*ne) gets -1. */
OMC_HD void omc_ep_token_positions(const int32_t *idx, int k, int ne, int P, const int *row_before,
                                   const int *slot_before, const int *send_base, const int *ret_base,
                                   const int *cnt, int32_t *tok_pos, int32_t *slot_pos) {
    int seen[OMC_EP_MAX_RANKS];
    for (int r = 0; r < P; ++r) {
        tok_pos[r] = cnt[r] > 0 ? send_base[r] + row_before[r] : -1;
        seen[r] = 0;
    }
    for (int kk = 0; kk < k; ++kk) {
        const int e = idx[kk];
        const int r = e >= 0 ? e / ne : -1;
        if (r < 0 || r >= P) {
            slot_pos[kk] = -1;
            continue;
        }
        slot_pos[kk] = ret_base[r] + slot_before[r] + seen[r];
        seen[r]++;
    }
}

/* The meta row of token row (idx, w) sent to rank r: see the header. */
OMC_HD void omc_ep_token_meta(const int32_t *idx, const float *w, int k, int ne, int r, int slot_in_block,
                              int32_t *meta) {
    int n = 0;
    for (int kk = 0; kk < k; ++kk) {
        const int e = idx[kk];
        if (e >= 0 && e / ne == r) {
            meta[2 + n] = e;
            union { float f; int32_t i; } u;
            u.f = w[kk];
            meta[2 + k + n] = u.i;
            ++n;
        }
    }
    meta[0] = slot_in_block;
    meta[1] = n;
    for (int j = n; j < k; ++j) {
        meta[2 + j] = -1;
        meta[2 + k + j] = 0;
    }
}

/* Peer of received row j: the p with recv_base[p] <= j < recv_base[p+1]. */
OMC_HD int omc_ep_row_peer(const int *recv_base, int P, int j) {
    int p = 0;
    while (p + 1 < P && recv_base[p + 1] <= j) ++p;
    return p;
}

#ifdef __cplusplus
extern "C" {
#endif
/* Host versions (omc_ep.c), run by the CPU tests on the library's own
 * arithmetic.  counts: [0,P) send_rows, [P,2P) send_slots, [2P,3P)
 * send_base, [3P,4P) ret_base.  meta: one row of omc_ep_meta_ints(k) ints
 * per sent row, at its tok_pos.  Returns the rows sent (sum of send_rows),
 * or -1 on bad arguments. */
int omc_ep_layout_host(const int32_t *idx, const float *w, int T, int k, int E, int P, int32_t *tok_pos,
                       int32_t *slot_pos, int32_t *counts, int32_t *meta);
/* Slots of the received rows: recv_rows[p], recv_slots[p] from peer p (their
 * send_rows / send_slots for this rank); slot_tok[s] = operand row
 * (Thome + received row; the home's shared slots, when has_shared, are
 * s = total received slots + t -> row t), slot_e, slot_w.  Returns the slot
 * count, or -1 when a meta row is inconsistent. */
int omc_ep_unpack_host(const int32_t *meta, const int32_t *recv_rows, const int32_t *recv_slots, int P, int k,
                       int Thome, int E, int has_shared, int32_t *slot_tok, int32_t *slot_e, float *slot_w);
#ifdef __cplusplus
}
#endif

#endif /* OMC_EP_PLAN_H */
