/* omc_ep.c -- expert parallelism: which experts this process holds.
 *
 * A layer's routed experts are split into `world` contiguous ranges
 * (E/world each); the process of rank r holds range r in its slab
 * (the experts of a layer are independent of one another).  The exchange
 * itself -- routed rows to the ranks that hold their experts, weighted rows
 * back, the k-order sum at the token's home rank -- is composed by the
 * caller from omc_moe_route_dev and omc_moe_experts_dev over its own
 * transport (overhang_b200/ep.py does it with torch.distributed over NCCL).
 * Joining an NCCL group from C (a unique id) is not provided. */
#include <string.h>

#include "om_cuda.h"
#include "omc_host.h"

#define G omc_G

int omc_ep_unique_id(void *buf, size_t len) {
    (void)buf;
    (void)len;
    return omc_fail(OMC_EUNSUPPORTED,
                    "omc_ep_unique_id: the library does not own an NCCL group; exchange rows with your own "
                    "transport (overhang_b200.ep uses torch.distributed)");
}

int omc_ep_init(int rank, int world, const void *unique_id) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_ep_init: omc_init not called");
    if (world < 1 || rank < 0 || rank >= world) return omc_fail(OMC_EINVAL, "omc_ep_init: rank %d of %d", rank, world);
    if (unique_id)
        return omc_fail(OMC_EUNSUPPORTED, "omc_ep_init: joining an NCCL group from C is not provided; pass NULL "
                                          "and exchange rows with omc_moe_route_dev/omc_moe_experts_dev");
    for (int i = 0; i < G.nlayers; ++i)
        if (G.layers[i].used)
            return omc_fail(OMC_EINVAL, "omc_ep_init: call before the first omc_layer_init");
    G.ep_rank = rank;
    G.ep_world = world;
    return OMC_OK;
}

int omc_ep_forward(omc_layer *L, const float *x, int T, float *out, int32_t *topk_idx, float *topk_w,
                   cudaStream_t s) {
    (void)L; (void)x; (void)T; (void)out; (void)topk_idx; (void)topk_w; (void)s;
    return omc_fail(OMC_EUNSUPPORTED,
                    "this process holds experts [e0, e0+E/world) only: compose the forward from "
                    "omc_moe_route_dev + exchange + omc_moe_experts_dev (overhang_b200.ep)");
}

void omc_ep_release(void) {}
