/* omc_ep.c -- expert parallelism across GPUs (one process per GPU, NCCL).
 * Placeholder until the all-to-all dispatch/combine lands: joining a group
 * is reported as unsupported so no caller silently runs single-GPU math. */
#include <string.h>

#include "om_cuda.h"
#include "omc_host.h"

int omc_ep_unique_id(void *buf, size_t len) {
    (void)buf;
    (void)len;
    return omc_fail(OMC_EUNSUPPORTED, "omc_ep_unique_id: expert parallelism not built yet");
}

int omc_ep_init(int rank, int world, const void *unique_id) {
    (void)rank;
    (void)world;
    (void)unique_id;
    return omc_fail(OMC_EUNSUPPORTED, "omc_ep_init: expert parallelism not built yet");
}

int omc_ep_forward(omc_layer *L, const float *x, int T, float *out, int32_t *topk_idx, float *topk_w,
                   cudaStream_t s) {
    (void)L; (void)x; (void)T; (void)out; (void)topk_idx; (void)topk_w; (void)s;
    return omc_fail(OMC_EUNSUPPORTED, "expert parallel forward not built yet");
}

void omc_ep_release(void) {}
