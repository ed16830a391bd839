/* omm_shim.c -- the engines' omm_* GPU seam (metal/om_metal.h:14-46) on CUDA.
 * Placeholder: device bring-up and pinned allocation work; the MoE entry
 * returns -3 (unsupported) so the engines keep their CPU path until the
 * job-driven expert pass lands. */
#include <stdlib.h>

#include <cuda_runtime.h>

#include "om_metal.h"
#include "om_cuda.h"
#include "omc_host.h"

int omm_init(void) {
    static int state = -1;
    if (state >= 0) return state;
    const char *dv = getenv("OMC_DEVICE");
    state = omc_init(dv ? atoi(dv) : 0, 0) == OMC_OK ? 1 : 0;
    return state;
}

void *omm_alloc(size_t n) {
    void *p = NULL;
    if (cudaHostAlloc(&p, n ? n : 1, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
        cudaGetLastError();
        return NULL;
    }
    return p;
}

int omm_moe_act(const omm_job *jobs, int nj, const float *x, int S, int D, int I, float *out, int gelu) {
    (void)jobs; (void)nj; (void)x; (void)S; (void)D; (void)I; (void)out; (void)gelu;
    return -3;
}

int omm_moe(const omm_job *jobs, int nj, const float *x, int S, int D, int I, float *out) {
    return omm_moe_act(jobs, nj, x, S, D, I, out, 0);
}

int omm_dense_q(const int8_t *Wq, const float *scales, int N, int K, const float *x, int S, float *out) {
    (void)Wq; (void)scales; (void)N; (void)K; (void)x; (void)S; (void)out;
    return -3;
}

int omm_dense(const float *W, int N, int K, const float *x, int S, float *out) {
    (void)W; (void)N; (void)K; (void)x; (void)S; (void)out;
    return -3;
}
