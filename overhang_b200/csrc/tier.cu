// tier.cu -- the device side of a tiered layer's forward (omc_tier.c).
//
// Launched right after routing, before the expert kernels:
//
// tier_route_kernel (one block): counts this forward's routed slots per
//   expert; updates the hot-store counters (clock += 1; heat[e] += slots,
//   saturating; last[e] = clock for every routed e; every decay_every-th
//   clock halves all heat, include/tier.h:56-58); and lists the routed
//   experts whose table entry is not in the HBM slots, in expert order,
//   pointing entry e at image j of the miss area.
// tier_fetch_kernel (grid): copies each listed expert's home image (mapped
//   pinned host memory, read with plain 16-byte loads) into its miss image.
//
// So the expert kernels, which fetch weights with bulk asynchronous copies,
// only ever read HBM; a non-resident expert crosses the host link once per
// forward that routes to it.  stats = [heat E][last E][clock 1] (uint32);
// list = [count, expert ids...].
#include "omc_common.cuh"

namespace {

struct TierArgs {
    const int32_t *idx;
    int nslots, E, decay_every, miss_cap;
    uint32_t *stats;
    omc_expert_ptrs *tab;
    const char *slots_lo, *slots_hi;   // the HBM slot images
    const char *home;                  // [E] home images (device view of mapped host memory)
    char *miss;                        // [miss_cap] HBM images
    size_t bytes, off_d, off_gs, off_us, off_ds;
    int *list;
    unsigned long long *total;         // misses over all forwards
    int *err;
};

__global__ void __launch_bounds__(1024) tier_route_kernel(TierArgs a) {
    __shared__ uint32_t cnt[OMC_MAX_E];
    const int E = a.E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int s = threadIdx.x; s < a.nslots; s += blockDim.x) {
        const int e = __ldg(a.idx + s);
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1u);
    }
    uint32_t *heat = a.stats, *last = a.stats + E, *clock = a.stats + 2 * E;
    const uint32_t clk = *clock + 1u;
    __syncthreads();   // every thread has read the clock before thread 0 moves it
    const bool decay = a.decay_every > 0 && clk % (uint32_t)a.decay_every == 0;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        uint32_t h = heat[e];
        const uint32_t c = cnt[e];
        if (c) {
            h = h > 0xFFFFFFFFu - c ? 0xFFFFFFFFu : h + c;
            last[e] = clk;
        }
        heat[e] = decay ? h >> 1 : h;
    }
    if (threadIdx.x == 0) *clock = clk;
    // the miss list, in expert order (E <= OMC_MAX_E: one warp scans it)
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        int n = 0;
        for (int base = 0; base < E; base += 32) {
            const int e = base + lane;
            bool miss = false;
            if (e < E && cnt[e]) {
                const char *g = reinterpret_cast<const char *>(a.tab[e].g);
                miss = !(g >= a.slots_lo && g < a.slots_hi);
            }
            const unsigned m = __ballot_sync(0xffffffffu, miss);
            if (miss) {
                const int j = n + __popc(m & ((1u << lane) - 1u));
                if (j < a.miss_cap) {
                    a.list[1 + j] = e;
                    char *img = a.miss + (size_t)j * a.bytes;
                    omc_expert_ptrs p;
                    p.g = reinterpret_cast<const int8_t *>(img);
                    p.u = reinterpret_cast<const int8_t *>(img) + OMC_BLK_BYTES;
                    p.d = reinterpret_cast<const int8_t *>(img + a.off_d);
                    p.gs = reinterpret_cast<const float *>(img + a.off_gs);
                    p.us = reinterpret_cast<const float *>(img + a.off_us);
                    p.ds = reinterpret_cast<const float *>(img + a.off_ds);
                    a.tab[e] = p;
                } else {
                    omc_dev_error(a.err, OMC_DEVERR_BOUNDS, OMC_SITE_DISPATCH, e);
                }
            }
            n += __popc(m);
        }
        if (lane == 0) {
            a.list[0] = min(n, a.miss_cap);
            *a.total += (unsigned long long)min(n, a.miss_cap);
        }
    }
}

// n images of `bytes` (a multiple of 256), image j from home[list[1+j]]:
// 16-byte loads, four in flight per thread, grid-stride.
__global__ void __launch_bounds__(256) tier_fetch_kernel(TierArgs a) {
    const int n = __ldg(a.list);
    if (n <= 0) return;
    const size_t per = a.bytes / 16, total = per * (size_t)n;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < total; i += 4 * stride) {
        int4 v[4];
        size_t dst[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const size_t c = i + u * stride, j = c / per, r = c - j * per;
            const int e = __ldg(a.list + 1 + j);
            v[u] = reinterpret_cast<const int4 *>(a.home + (size_t)e * a.bytes)[r];
            dst[u] = j * per + r;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) reinterpret_cast<int4 *>(a.miss)[dst[u]] = v[u];
    }
    for (; i < total; i += stride) {
        const size_t j = i / per, r = i - j * per;
        const int e = __ldg(a.list + 1 + j);
        reinterpret_cast<int4 *>(a.miss)[j * per + r] = reinterpret_cast<const int4 *>(a.home + (size_t)e * a.bytes)[r];
    }
}

}  // namespace

extern "C" int omc_launch_tier_route(const int32_t *idx, int nslots, int E, uint32_t *stats, int decay_every,
                                     omc_expert_ptrs *tab, const void *slots_lo, const void *slots_hi,
                                     const void *home, void *miss, int miss_cap, const size_t *layout, int *list,
                                     unsigned long long *total, int *err, int grid, cudaStream_t s) {
    if (E <= 0 || E > OMC_MAX_E || nslots < 0 || (layout[0] & 255)) return OMC_EINVAL;
    TierArgs a;
    a.idx = idx;
    a.nslots = nslots;
    a.E = E;
    a.decay_every = decay_every;
    a.miss_cap = miss_cap;
    a.stats = stats;
    a.tab = tab;
    a.slots_lo = static_cast<const char *>(slots_lo);
    a.slots_hi = static_cast<const char *>(slots_hi);
    a.home = static_cast<const char *>(home);
    a.miss = static_cast<char *>(miss);
    a.bytes = layout[0];
    a.off_d = layout[1];
    a.off_gs = layout[2];
    a.off_us = layout[3];
    a.off_ds = layout[4];
    a.list = list;
    a.total = total;
    a.err = err;
    tier_route_kernel<<<1, nslots >= 4096 ? 1024 : 256, 0, s>>>(a);
    omc_g_launches += 1;
    if (miss_cap > 0) {
        tier_fetch_kernel<<<grid, 256, 0, s>>>(a);
        omc_g_launches += 1;
    }
    omc_prof_mark(s, "tier_fetch");
    return cudaGetLastError() == cudaSuccess ? 0 : OMC_ECUDA;
}
