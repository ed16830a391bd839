// slab.cu -- re-tiling of uploaded expert weights into the HBM slab layout.
//
// The container tensors arrive row-major (tools/convert_olmoe.py:93-99,
// engines/olmoe.c:237-247); the kernels want the tiled int8 layout described
// in omc_internal.h.  One thread writes one 16-byte chunk of the destination;
// padding rows and columns are written as zeros.
#include "omc_common.cuh"

namespace {

__global__ void relayout_kernel(const int8_t *__restrict__ src, int O, int K, int8_t *__restrict__ dst,
                                int O_pad, int K_pad, int member) {
    const int nkb = K_pad / OMC_KB;
    const long long nchunks = (long long)O_pad * K_pad / 16;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < nchunks;
         idx += (long long)gridDim.x * blockDim.x) {
        const long long blk = idx / 512;
        const int within = (int)(idx % 512);
        const int c = within / OMC_TM, r = within % OMC_TM;
        const int ot = (int)(blk / nkb), kb = (int)(blk % nkb);
        const int row = ot * OMC_TM + r, col = kb * OMC_KB + c * 16;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (row < O) {
            const int8_t *s = src + (size_t)row * K + col;
            if (col + 16 <= K && ((reinterpret_cast<uintptr_t>(s) & 15) == 0)) {
                const int4 v = *reinterpret_cast<const int4 *>(s);
                w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
            } else {
                for (int j = 0; j < 16; ++j) {
                    const uint32_t b = (col + j < K) ? (uint8_t)s[j] : 0u;
                    w[j >> 2] |= b << (8 * (j & 3));
                }
            }
        }
        // paired tiles: member `member` of pair ot, or tiles 2p / 2p+1 of pair p
        const size_t boff = member >= 0 ? ((size_t)ot * nkb + kb) * 2 * OMC_BLK_BYTES + (size_t)member * OMC_BLK_BYTES
                                        : omc_dblk(ot, kb, nkb);
        *reinterpret_cast<int4 *>(dst + boff + (size_t)within * 16) = make_int4(w[0], w[1], w[2], w[3]);
    }
}

__global__ void i8_to_f32_kernel(const int8_t *__restrict__ src, float *__restrict__ dst, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        dst[i] = (float)src[i];
}

}  // namespace

extern "C" int omc_launch_relayout(const int8_t *src, int O, int K, int8_t *dst, int O_pad, int K_pad,
                                   int member, cudaStream_t s) {
    const long long nchunks = (long long)O_pad * K_pad / 16;
    const int grid = (int)((nchunks + 255) / 256 < 65535 ? (nchunks + 255) / 256 : 65535);
    relayout_kernel<<<grid, 256, 0, s>>>(src, O, K, dst, O_pad, K_pad, member);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

extern "C" int omc_launch_i8_to_f32(const int8_t *src, float *dst, long long n, cudaStream_t s) {
    const int grid = (int)((n + 255) / 256 < 65535 ? (n + 255) / 256 : 65535);
    i8_to_f32_kernel<<<grid, 256, 0, s>>>(src, dst, n);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}

// A kernel whose only job is a bounded wait on a flag nothing sets: the
// failure-detection test uses it to check that an expired device wait comes
// back as OMC_ETIMEOUT with the context still usable.
namespace {
__global__ void test_wait_kernel(int *err) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, err, OMC_SITE_TEST_WAIT);   // never completes: times out
    __syncthreads();
}
}  // namespace

extern "C" int omc_launch_test_wait(int *err, cudaStream_t s) {
    test_wait_kernel<<<1, 32, 0, s>>>(err);
    omc_g_launches += 1;
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}
