// omc_select.cuh -- one token's routing from its logits (device function),
// shared by the router's select kernel and the fused decode kernel.
//
// Bit-exact with the reference CPU router:
//   softmax: engines/olmoe.c:170-174 (float running sum) and
//            engines/qwen.c:161-165 (double running sum, divide by float(s)),
//            with omc_expf_glibc, bit-equal to glibc expf.
//   top-k  : engines/olmoe.c:355-362 -- k passes of argmax, strict '>' in
//            ascending id order = (largest p, then lowest id).
//   renorm : engines/olmoe.c:363, engines/qwen.c:476-477 (float sum in
//            selection order, then divide).
//   shared gate: engines/qwen.c:460-461, sigmoid(logit row E).
//   bias   : an optional per-expert term added to each routed logit before the
//            softmax (a caller input with no counterpart in the reference: it
//            skews expert load for benchmarks; the oracle adds it the same way).
//   gemma  : engines/gemma.c:463-477 -- the float-sum softmax numerators e_i
//            are ranked themselves (strict '>' from -1: ties to the lowest
//            id), w_k = e_k/sum, renormalised by the float sum of the w_k in
//            selection order, then times per_expert_scale[id].
// Logits are read through L2 (ld.global.cg): they may have been written by
// other blocks of the same kernel.
#pragma once
#include "omc_common.cuh"

// One warp per token: softmax, top-k, renorm, shared-gate sigmoid.  Lane l
// holds logits l, l+32, ...; order-dependent sums run from a shared-memory
// copy so that their dependent chain is the add latency alone.  With a plan
// (tensor-core forwards) the block that finishes last builds the dispatch
// plan from every token's routing: no per-expert atomics in global memory.
constexpr int SEL_WARPS = 8;

template <int SEL_MAXV>   // ceil(E / 32) rounded up to a power of two
__device__ __forceinline__ void select_token(const float *__restrict__ logits, int ldl, int t, int E, int K,
                                             int family, int renorm, int has_shared,
                                             const float *__restrict__ pes, const float *__restrict__ bias,
                                             int32_t *__restrict__ topk_idx, float *__restrict__ topk_w,
                                             float *__restrict__ sg, int *err, float *es) {
    const int lane = threadIdx.x & 31;
    const float *lg = logits + (size_t)t * ldl;
    float v[SEL_MAXV];
    // max, as `if (x[i] > m) m = x[i]` from m = -1e30f
    float m = -1e30f;
#pragma unroll
    for (int j = 0; j < SEL_MAXV; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < E ? __ldcg(lg + i) : -INFINITY;
        if (bias && i < E) v[j] = __fadd_rn(v[j], __ldg(bias + i));   // logit + bias, one f32 add
        if (i < E && v[j] > m) m = v[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // e_i = expf(x_i - m)
    bool tiny = false;
    const float exact_floor = ldexpf(1.0f, (32 - __clz(max(E - 1, 1))) - 30);   // 2^(ceil(log2 E) - 30)
#pragma unroll
    for (int j = 0; j < SEL_MAXV; ++j) {
        const int i = lane + 32 * j;
        if (i < E) {
            v[j] = omc_expf_glibc(__fsub_rn(v[j], m));
            tiny |= v[j] < exact_floor;
            es[i] = v[j];
        }
    }
    __syncwarp();
    float sf;   // the divisor as the reference uses it
    if (family == OMC_FAMILY_QWEN && !__any_sync(0xffffffffu, tiny)) {
        // double running sum.  When every term is >= 2^(ceil(log2 E) - 30) all
        // partial sums are exact in double, so any order gives the
        // reference's value: a butterfly.
        double s = 0.0;
#pragma unroll
        for (int j = 0; j < SEL_MAXV; ++j)
            if (lane + 32 * j < E) s = __dadd_rn(s, (double)v[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        sf = __double2float_rn(s);
    } else if (family == OMC_FAMILY_QWEN) {
        // otherwise the index-order double sum of engines/qwen.c:163, every lane
        double s = 0.0;
        int i = 0;
        for (; i + 4 <= E; i += 4) {
            const float4 q = *reinterpret_cast<const float4 *>(es + i);
            s = __dadd_rn(s, (double)q.x);
            s = __dadd_rn(s, (double)q.y);
            s = __dadd_rn(s, (double)q.z);
            s = __dadd_rn(s, (double)q.w);
        }
        for (; i < E; ++i) s = __dadd_rn(s, (double)es[i]);
        sf = __double2float_rn(s);
    } else {
        // float running sum in index order (engines/olmoe.c:172), every lane
        float s = 0.f;
        int i = 0;
#pragma unroll 4
        for (; i + 4 <= E; i += 4) {
            const float4 q = *reinterpret_cast<const float4 *>(es + i);
            s = __fadd_rn(s, q.x);
            s = __fadd_rn(s, q.y);
            s = __fadd_rn(s, q.z);
            s = __fadd_rn(s, q.w);
        }
        for (; i < E; ++i) s = __fadd_rn(s, es[i]);
        sf = s;
    }
    // probabilities (gemma: the numerators) as order keys: p >= 0, so
    // bits(p) + 1 orders like p and 0 marks "not available" (outside E, NaN,
    // or already taken).
    const bool gemma = family == OMC_FAMILY_GEMMA;
    uint32_t key[SEL_MAXV];
    float pv[SEL_MAXV];
#pragma unroll
    for (int j = 0; j < SEL_MAXV; ++j) {
        const int i = lane + 32 * j;
        pv[j] = i < E ? (gemma ? v[j] : __fdiv_rn(v[j], sf)) : 0.f;
        key[j] = (i < E && pv[j] == pv[j]) ? __float_as_uint(pv[j]) + 1u : 0u;
    }
    // top-k: engines/olmoe.c:355-362 -- largest p, ties to the lowest id
    int my_idx = -1;
    float my_val = 0.f;
    for (int kk = 0; kk < K; ++kk) {
        uint32_t bk = 0;
        int bj = 0;
#pragma unroll
        for (int j = 0; j < SEL_MAXV; ++j)
            if (key[j] > bk) { bk = key[j]; bj = j; }      // strict: lowest j (= lowest id) of this lane
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, bk);
        const uint32_t cand = (bk == kmax && kmax != 0u) ? (uint32_t)(lane + 32 * bj) : 0xffffffffu;
        const uint32_t best = __reduce_min_sync(0xffffffffu, cand);
        if (kmax != 0u && (int)(best & 31) == lane) {
#pragma unroll
            for (int j = 0; j < SEL_MAXV; ++j)
                if (j == (int)(best >> 5)) key[j] = 0u;
        }
        if (lane == kk) {
            my_idx = kmax != 0u ? (int)best : -1;
            my_val = __uint_as_float(kmax - 1u);
        }
    }
    if (gemma) my_val = __fdiv_rn(my_val, sf);   // tw[k] = bv/psum (engines/gemma.c:474)
    // renorm: float sum in selection order, then divide (engines/olmoe.c:363,
    // engines/gemma.c:474,477)
    if (renorm || family == OMC_FAMILY_QWEN || gemma) {
        float sm = 0.f;
        for (int kk = 0; kk < K; ++kk) sm = __fadd_rn(sm, __shfl_sync(0xffffffffu, my_val, kk));
        my_val = __fdiv_rn(my_val, sm);
    }
    if (gemma && lane < K && my_idx >= 0 && my_idx < E) my_val = __fmul_rn(my_val, __ldg(pes + my_idx));
    if (lane < K) {
        if (my_idx < 0 || my_idx >= E) omc_dev_error(err, OMC_DEVERR_ROUTE, OMC_SITE_ROUTER, t);
        topk_idx[(size_t)t * K + lane] = my_idx;
        topk_w[(size_t)t * K + lane] = my_val;
    }
    if (has_shared && lane == 0) {
        const float z = __ldcg(lg + E);
        sg[t] = __fdiv_rn(1.f, __fadd_rn(1.f, omc_expf_glibc(-z)));   // engines/qwen.c:158,461
    }
}

