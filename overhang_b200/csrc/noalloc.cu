// noalloc.cu -- scratch for omc_moe_forward_noalloc(), the forward entry that
// allocates nothing.
//
// Every other forward entry grows a per-call workspace with cudaMalloc the
// first time it sees a larger T.  Some callers cannot allow that: an engine
// that reserves all of HBM up front (expert slab, KV cache) and must keep a
// fixed footprint, or a host loop that may not stall in the driver's
// allocator (cudaMalloc/cudaFree can synchronise the device) between tokens.
// For them the workspace of one forward lives in the fixed-size array below
// instead.  Its size is OMC_NOALLOC_SCRATCH_BYTES; every GPU that loads the
// library holds it until the process exits.  Because all calls share it, two
// no-alloc forwards that overlap on the GPU (different streams, no ordering)
// race on it; order them on one stream.
#include "omc_common.cuh"

namespace {
// Name valid only in device code and in cudaGetSymbolAddress: in host code
// this is a host-side stand-in, not a device address.
static __device__ __align__(256) unsigned char omc_noalloc_scratch[OMC_NOALLOC_SCRATCH_BYTES];

void *g_scratch_addr[OMC_MAX_DEVICES];
}  // namespace

// Called by omc_init once for its device, with that device current.
extern "C" int omc_noalloc_setup(int device) {
    if (device < 0 || device >= OMC_MAX_DEVICES) return OMC_EINVAL;
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, omc_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        g_scratch_addr[device] = nullptr;
        return OMC_ECUDA;
    }
    g_scratch_addr[device] = p;
    return OMC_OK;
}

extern "C" void *omc_noalloc_scratch_ptr(int device) {
    if (device < 0 || device >= OMC_MAX_DEVICES) return nullptr;
    return g_scratch_addr[device];
}
