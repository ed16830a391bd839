// ffn_mma.cu -- tensor-core (tcgen05) grouped expert GEMMs.  Placeholder.
#include "omc_common.cuh"

extern "C" int omc_launch_mma_ffn(const omc_layer_dev *L, const float *x, int T, const omc_ws *ws,
                                  const int32_t *topk_idx, const float *topk_w, float *out, cudaStream_t s) {
    (void)L; (void)x; (void)T; (void)ws; (void)topk_idx; (void)topk_w; (void)out; (void)s;
    return OMC_EUNSUPPORTED;
}
