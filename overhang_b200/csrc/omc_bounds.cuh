// omc_bounds.cuh -- the top-k set of one token from intervals on its logits
// (device functions; one warp per token).
//
// Each expert e has an interval [lo_e, hi_e] that holds the logit (bias
// included) the reference's sequential chain produces (engines/olmoe.c:74-85,
// engines/qwen.c:116-121).  The selection (omc_select.cuh) ranks the softmax
// values p_e = RN(expf(v_e - m) / s), or the numerators for Gemma, with ties
// to the lowest id.  p is a non-decreasing function of v, but two logits that
// differ by less than a few units in the last place of the softmax's
// differences may round to the same p, and the id order then decides.  So an
// expert is a candidate when hi_e >= (k-th largest lo) - mu, with mu =
// 2^-19 + 2^-21 (|k-th lo| + |max hi|): a non-candidate's logit is below k
// others' by more than that margin, so its exp value, and its probability,
// are strictly below theirs and it is not selected.  The top-k set is a
// subset of the candidates, and equal to them when there are exactly k.
#pragma once
#include "omc_common.cuh"

// float -> unsigned key in the float order (NaN excluded by the caller)
__device__ __forceinline__ uint32_t omc_ford(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float omc_funord(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// lo/hi hold this lane's experts lane + 32 j (-INFINITY past E; every value
// finite and below 1e30 in magnitude -- the caller checks).  Writes the
// candidates in ascending id order to cand[0 .. min(nc, cap)) and returns nc,
// or -1 when the intervals cannot decide: the k-th lower end is empty, or the
// largest upper end is more than 60 above it (the k-th probability may
// underflow, where the reference's ties are not the interval order's).
template <int MAXV, class C>
__device__ __forceinline__ int omc_topk_candidates(const float (&lo)[MAXV], const float (&hi)[MAXV], int E, int K,
                                                   int cap, C *cand) {
    const int lane = threadIdx.x & 31;
    // the k-th largest lower end: k passes of warp argmax with removal
    uint32_t key[MAXV];
#pragma unroll
    for (int j = 0; j < MAXV; ++j) key[j] = lane + 32 * j < E ? omc_ford(lo[j]) : 0u;
    uint32_t kmax = 0;
    for (int kk = 0; kk < K; ++kk) {
        uint32_t bk = 0;
        int bj = 0;
#pragma unroll
        for (int j = 0; j < MAXV; ++j)
            if (key[j] > bk) { bk = key[j]; bj = j; }
        kmax = __reduce_max_sync(0xffffffffu, bk);
        const uint32_t who = __reduce_min_sync(0xffffffffu, bk == kmax ? (uint32_t)lane : 32u);
        if ((uint32_t)lane == who) {
#pragma unroll
            for (int j = 0; j < MAXV; ++j)
                if (j == bj) key[j] = 0u;
        }
    }
    float mh = -INFINITY;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) mh = fmaxf(mh, hi[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, o));
    const float kth = omc_funord(kmax);
    // margin: a non-candidate's logit is below the k-th by more than two
    // units in the last place of the softmax's differences plus 2^-20, so its
    // exp value, and its probability, are strictly below the k-th
    const float mu = __fadd_ru(1.9073486328125e-6f, __fmul_ru(4.76837158203125e-7f, __fadd_ru(fabsf(kth), fabsf(mh))));
    const float thr = __fsub_rd(kth, mu);
    if (kmax == 0u || __fsub_rd(kth, mh) < -60.f) return -1;
    int nc = 0;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
        const bool c = lane + 32 * j < E && hi[j] >= thr;
        const uint32_t m = __ballot_sync(0xffffffffu, c);
        const int at = nc + __popc(m & ((1u << lane) - 1u));
        if (c && at < cap) cand[at] = (C)(lane + 32 * j);
        nc += __popc(m);
    }
    return nc;
}
