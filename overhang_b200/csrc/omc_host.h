/* omc_host.h -- host-side state of the runtime (internal). */
#ifndef OMC_HOST_H
#define OMC_HOST_H
#include <cuda_runtime.h>

#include "om_cuda.h"
#include "omc_internal.h"

#ifdef __cplusplus
extern "C" {
#endif

#define OMC_MAX_CHUNKS 512
#define OMC_NSTAGE_EV 12
#define OMC_TIMER_RING 1024          /* stage-timer event pairs kept */

typedef struct {
    int used;
    omc_moe_desc desc;
    omc_layer_dev dev;              /* what kernels receive                 */
    omc_expert_ptrs *h_experts;     /* host copy of the pointer table [E+1] */
    omc_expert_ptrs *d_experts_tab; /* device pointer table [E+1]           */
    unsigned char *have;            /* uploaded flags [E+1]                 */
    int e0, ne;                     /* experts owned by this rank (EP)      */
    int gemma_ready;                /* GEMMA: omc_layer_gemma_norms called  */
    void *tier;                     /* tiered expert store (omc_tier.c)     */
    void *rf_mem;                   /* bounded router's tiles, table, norms */
    void *rt_mem;                   /* exact router's row blocks (dev.rt_w)  */
} omc_layer;

typedef struct {
    float *x, *out, *logits;
    int32_t *topk_idx;
    float *topk_w, *sg;
    int *counts, *rowinfo, *work;
    uint16_t *xh, *hp;
    float *ypart, *hbuf;
    int *slotrow;
    float *xg_r, *xg_e;
    uint16_t *rf_act;               /* bounded router (allocated by omc_ws_ensure) */
    float *rf_y;
    int *rf_misc, *rf_jobs;
} omc_ws_ptrs;

typedef struct {
    int init, device, num_sms;
    cudaStream_t stream;
    int *d_err;
    /* slab */
    size_t slab_budget, slab_used, chunk_used;
    void *chunk[OMC_MAX_CHUNKS];
    size_t chunk_size[OMC_MAX_CHUNKS];
    int nchunk;
    void *staging;
    size_t staging_bytes;
    /* layers */
    omc_layer *layers;
    int nlayers;
    /* workspace */
    omc_ws ws;
    omc_ws_ptrs ws_ptrs;
    size_t ws_bytes[24];
    /* profiling */
    int profiling, prof_valid, prof_nev;
    cudaEvent_t ev[OMC_NSTAGE_EV];
    const char *prof_names[OMC_NSTAGE_EV];
    /* stage timer: one event pair around a named stage of every forward */
    int timer_on, timer_n, timer_created;
    char timer_name[32];
    cudaEvent_t timer_ev[2 * OMC_TIMER_RING];
    int path_override;              /* 0 auto, 1 gemv, 2 mma, 3 fused decode (OMC_FFN_PATH) */
    /* fused decode state: counters (zero between forwards) and pieces */
    int *dec_ctr;
    float *dec_part;
    size_t dec_ctr_n, dec_part_n;
    /* expert parallelism */
    int ep_rank, ep_world;
    void *ep;                       /* omc_ep_state (omc_ep.c)              */
} omc_state;

extern omc_state omc_G;

int omc_fail(int code, const char *fmt, ...);
void *omc_slab_alloc(size_t n, int *on_host);
omc_layer *omc_get_layer(int layer);
int omc_ws_ensure(const omc_layer *L, int T, int host_io);
int omc_ws_ensure_rows(const omc_layer *L, int rows);
/* the same for a workspace other than the library's own (the expert-parallel pass) */
int omc_ws_ensure_rows_in(const omc_layer *L, int rows, omc_ws *ws, omc_ws_ptrs *W, size_t *bytes);
void omc_ws_free_in(omc_ws_ptrs *W, size_t *bytes, int nbytes);
int omc_expert_upload(int D, int D_pad, int D_rows, int I_, int I_pad, int I_rows, const int8_t *g, const float *gs,
                      const int8_t *u, const float *us, const int8_t *d, const float *ds, omc_expert_ptrs *ep,
                      int reuse);
int omc_matrix_upload(const int8_t *q, const float *s, int O, int K, int8_t **dq, const float **ds, int reuse);
int omc_check_device_error(void);
int omc_forward_device(omc_layer *L, const float *x, int T, float *out, int32_t *topk_idx, float *topk_w,
                       cudaStream_t s);

/* tiered expert store (omc_tier.c) */
int omc_tier_upload(omc_layer *L, int e, const int8_t *g, const float *gs, const int8_t *u, const float *us,
                    const int8_t *d, const float *ds);
void omc_tier_free(omc_layer *L);
int omc_tier_before(omc_layer *L, cudaStream_t s);
int omc_tier_route(omc_layer *L, const int32_t *idx, int T, cudaStream_t s);
void omc_tier_release(void);
int omc_tier_after(omc_layer *L, cudaStream_t s);

/* expert parallelism (omc_ep.c) */
int omc_ep_forward(omc_layer *L, const float *x, int T, float *out, int32_t *topk_idx, float *topk_w,
                   cudaStream_t s);
void omc_ep_release(void);

int omc_debug_wait_timeout(void);
int omc_debug_expf(const float *x, float *y, long long n);
int omc_debug_set_path(int path);
int omc_debug_plan_rows(int rows);
int omc_debug_router_tile(int g, int tt, int rr);
int omc_debug_rf_force_retry(int on);
int omc_debug_ws_copy(int which, void *dst, size_t bytes);
int omc_debug_gemma_prenorm(int layer, const float *x, int T, float *xr, float *xe, float *r);
long long omc_debug_container_read(const char *snapshot, const char *name, void *dst, long long cap);

#ifdef __cplusplus
}
#endif
#endif
