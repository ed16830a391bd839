// omc_common.cuh -- device helpers shared by the MoE kernels (sm_100a only).
//
//  * omc_dev_error(): first-error-wins report into the library's device error
//    word; every bounded wait reports through it instead of trapping.
//  * omc_expf_glibc(): device restatement of the expf the reference calls.
//  * PTX wrappers: mbarrier, 1-D bulk copy (no multicast), tcgen05.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "omc_internal.h"

#if !defined(__CUDA_ARCH__) || (__CUDA_ARCH__ >= 1000)
#else
#error "overhang_b200 kernels target sm_100a only"
#endif

// ---------------------------------------------------------------- errors --
// err[0] = code (OMC_DEVERR_*), err[1] = site, err[2] = detail.  The first
// writer wins; the host reads it after a synchronise.
__device__ __forceinline__ void omc_dev_error(int *err, int code, int site, int detail) {
    if (err && atomicCAS(err, 0, code) == 0) {
        err[1] = site;
        err[2] = detail;
        __threadfence_system();
    }
}

// Time limit for every wait on a barrier, flag or count: any honest wait
// here is microseconds (one tile); a lost wait ends after ~1 s, reports
// OMC_DEVERR_TIMEOUT and the kernel unwinds instead of hanging.  The limit
// is over only when both clocks agree: %globaltimer (nanoseconds, kept by the
// driver, which may step it) and the SM's own cycle counter (monotonic;
// 1e9 cycles is 0.5 s at 1.965 GHz).  A step of one of them cannot end a
// wait that is still honest.
#define OMC_WAIT_LIMIT_NS 1000000000ull
#define OMC_WAIT_LIMIT_CYCLES 1000000000ll

__device__ __forceinline__ uint64_t omc_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

struct OmcDeadline {
    uint64_t t0;
    long long c0;
    __device__ __forceinline__ void start() {
        t0 = omc_globaltimer();
        c0 = clock64();
    }
    __device__ __forceinline__ bool over() const {
        return omc_globaltimer() - t0 > OMC_WAIT_LIMIT_NS && clock64() - c0 > OMC_WAIT_LIMIT_CYCLES;
    }
};

// ------------------------------------------------------------- gelu_tanh --
// engines/gemma.c:319-321, operation for operation: 0.5f*x*(1 + tanhf(c*(x +
// 0.044715f*x*x*x))).  tanhf is CUDA's (within 2 ulp of the exact value); the
// reference's is libm's, so expert outputs agree within the output tolerance,
// not bit for bit.
__device__ __forceinline__ float omc_gelu_tanh(float x) {
    const float c3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
    const float th = tanhf(__fmul_rn(0.7978845608028654f, __fadd_rn(x, c3)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.f, th));
}

// ------------------------------------------------------------------ expf --
// Device restatement of glibc's expf (glibc >= 2.28, x86-64 FMA build), the
// function the reference's softmax calls (engines/olmoe.c:172,
// engines/qwen.c:163).  The method is the published ARM optimized-routines
// expf (Szabolcs Nagy, 2017): x*32/ln2 = k + r, 2^(k/32) from a 32-entry
// table, 2^(r/32) by a cubic, all in double, rounded once to float.  The
// x86-64 glibc build contracts z*InvLn2N+Shift and the cubic into FMAs; the
// restatement does the same with explicit fma().  Checked equal to the host
// glibc expf on all 2^32 float inputs (tests/test_oracle.py exercises the
// host side; tests/test_router_gpu.py the device side).
__device__ const uint64_t omc_exp2_tab[32] = {
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL,
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL,
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL,
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL,
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL,
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL,
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL,
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL};
// table entry i = bits(2^(i/32)) - (i << 47), computed in 300-bit arithmetic.
// Global memory through the read-only path, not __constant__: lanes index
// it with different i, which the constant cache would serialise.

__device__ __forceinline__ float omc_expf_glibc(float x) {
    const uint32_t ix = __float_as_uint(x);
    const uint32_t abstop = (ix >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) {                         // |x| >= 88 or not finite
        if (ix == 0xff800000u) return 0.0f;         // -inf
        if (abstop >= 0x7f8u) return x + x;         // +inf, nan
        if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double InvLn2N = 0x1.71547652b82fep+0 * 32.0;
    const double Shift = 0x1.8p+52;
    const double C0 = 0x1.c6af84b912394p-5 / 32768.0;   // cubic for 2^(r/32), r in [-1/2,1/2]
    const double C1 = 0x1.ebfce50fac4f3p-3 / 1024.0;
    const double C2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double xd = (double)x;
    double kd = fma(InvLn2N, xd, Shift);
    const uint64_t ki = (uint64_t)__double_as_longlong(kd);
    kd = __dsub_rn(kd, Shift);
    const double r = fma(InvLn2N, xd, -kd);
    uint64_t t = __ldg(&omc_exp2_tab[ki & 31]);
    t += ki << 47;
    const double s = __longlong_as_double((long long)t);
    const double z = fma(C0, r, C1);
    const double r2 = __dmul_rn(r, r);
    double y = fma(C2, r, 1.0);
    y = fma(z, r2, y);
    y = __dmul_rn(y, s);
    return __double2float_rn(y);
}

// ------------------------------------------------------------- mbarrier --
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// As mbar_try_wait, but the thread may sleep in the instruction (up to
// `hint_ns`, woken when the phase completes) instead of returning at once:
// waiting warps then take no issue slots from the warps that do the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (after reporting) when the phase never flips.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    OmcDeadline dl;
    dl.start();
    for (;;) {
        for (int i = 0; i < 256; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (dl.over()) break;
    }
    omc_dev_error(err, OMC_DEVERR_TIMEOUT, site, (int)parity);
    return false;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (no multicast).
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// The tensor-core path's f16 operands: |v| >= 65520 rounds past the largest
// f16 (65504) and would be saturated (NaN is outside too).  Writers check each
// value and report OMC_DEVERR_RANGE instead of clipping silently.
__device__ __forceinline__ bool omc_f16_outside(float v) { return !(fabsf(v) < 65520.f); }

// (lo, hi) -> f16x2, round to nearest, saturated to +-65504.
__device__ __forceinline__ uint32_t f32x2_to_f16x2_sat(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Orders this thread's generic-proxy accesses to shared memory with later
// async-proxy ones (bulk copies, tcgen05.mma operand reads) and vice versa.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// L2 eviction policies for the hinted copies: operands streamed once (the
// expert weights) go first, operands re-read soon after they were written
// (token tiles, h) stay.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// bulk_g2s with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_hint(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// --------------------------------------------------------------- tcgen05 --
// TMEM addresses: bits [31:16] lane, [15:0] column.
__device__ __forceinline__ void tmem_alloc(uint32_t *smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Arrive once on `bar` when all previously issued tcgen05.mma of this thread
// have completed (the CTA's own barrier; no multicast).
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 (A and B both f16), f32 accumulate.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Instruction descriptor, kind::f16: A,B = f16, D = f32, both K-major.
__host__ __device__ constexpr uint32_t tc_idesc_f16(int M, int N) {
    return (1u << 4)                          // D format f32
           | (0u << 7) | (0u << 10)           // A, B format f16
           | ((uint32_t)(N >> 3) << 17)       // N / 8
           | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 B
// (64 f16 along K) in 8-row atoms of 1024 B.  `saddr` is the byte address of
// the first row (atoms 1024-aligned; +32 B per K=16 step inside an atom).
__device__ __forceinline__ uint64_t tc_sdesc_k_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);        // start address
    d |= (uint64_t)1u << 16;                        // leading byte offset (unused for SW128 K-major)
    d |= (uint64_t)(1024u >> 4) << 32;              // stride byte offset: next 8-row atom
    d |= (uint64_t)1u << 46;                        // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;                        // layout: SWIZZLE_128B
    return d;
}

// 32 lanes x 32 columns of 32-bit from registers to TMEM (this warp's lane quarter).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

// 32 lanes x 16 columns of 32-bit from TMEM to registers.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// ------------------------------------------------------- int8 dequant ----
// Four signed int8 packed in w -> two f16x2 (exact: |q| <= 128 fits f16).
// Bias to unsigned (q+128), place each byte under the f16 exponent of 1024
// (0x64XX = 1024 + u), subtract 1152 = 1024 + 128.
__device__ __forceinline__ void i8x4_to_f16x4(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t u = w ^ 0x80808080u;
    uint32_t a = __byte_perm(u, 0x64646464u, 0x5140);
    uint32_t b = __byte_perm(u, 0x64646464u, 0x7362);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    __half2 ha = __hsub2(*reinterpret_cast<__half2 *>(&a), bias);
    __half2 hb = __hsub2(*reinterpret_cast<__half2 *>(&b), bias);
    lo = *reinterpret_cast<uint32_t *>(&ha);
    hi = *reinterpret_cast<uint32_t *>(&hb);
}

// Four signed int8 packed in w -> four f32 (exact), same trick under 2^23.
__device__ __forceinline__ void i8x4_to_f32x4(uint32_t w, float &f0, float &f1, float &f2, float &f3) {
    const uint32_t u = w ^ 0x80808080u;
    const float bias = 8388736.0f;                       // 2^23 + 128
    f0 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)), bias);
    f1 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)), bias);
    f2 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)), bias);
    f3 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)), bias);
}
