/* omc_host.c -- host runtime of the B200 MoE block (C, CUDA runtime API).
 *
 * Owns the device, the library stream, the HBM expert slab, the per-layer
 * weights and the per-forward workspace, and sequences the kernels of one
 * MoE forward:
 *
 *   router (logits -> softmax -> top-k)            engines/olmoe.c:346-364
 *   expert FFN  (tensor-core grouped GEMMs, or      engines/olmoe.c:386-399
 *                CUDA-core GEMV for few tokens)      engines/qwen.c:455-493
 *   weighted combine (fused into the down pass)     engines/olmoe.c:395-397
 *
 * It replaces, in the engines, the per-layer LRU of int8 expert slots
 * (engines/olmoe.c:48-53,250-272) with one HBM slab filled at load time, and
 * the Metal backend's arena (metal/om_metal.mm:14-48) with cudaHostAlloc'd
 * memory for the omm_* seam (omm_shim.c).
 */
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "om_cuda.h"
#include "omc_internal.h"
#include "omc_host.h"

long long omc_g_launches = 0;

omc_state omc_G;
#define G omc_G

static char g_errbuf[512];

/* Generation of everything a forward enqueues (layers, workspace, forced
 * paths): the host entry's replayed forwards are valid for one generation. */
static int g_graph_gen;
void omc_graphs_invalidate(void) { ++g_graph_gen; }
#define graphs_invalidate omc_graphs_invalidate
static void graphs_release(void);
static void async_release(void);

int omc_fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_errbuf, sizeof(g_errbuf), fmt, ap);
    va_end(ap);
    return code;
}

#define CK(call)                                                                                       \
    do {                                                                                               \
        cudaError_t e_ = (call);                                                                       \
        if (e_ != cudaSuccess)                                                                         \
            return omc_fail(e_ == cudaErrorMemoryAllocation ? OMC_ENOMEM : OMC_ECUDA, "%s: %s (%s:%d)", \
                            #call, cudaGetErrorString(e_), __FILE__, __LINE__);                        \
    } while (0)

const char *omc_last_error(void) { return g_errbuf; }

const char *omc_strerror(int st) {
    switch (st) {
    case OMC_OK: return "ok";
    case OMC_EINVAL: return "invalid argument";
    case OMC_ENOMEM: return "out of memory";
    case OMC_ENOINIT: return "not initialised";
    case OMC_ECUDA: return "CUDA error";
    case OMC_EDEVICE: return "device-side error";
    case OMC_ETIMEOUT: return "timeout";
    case OMC_ENCCL: return "NCCL error";
    case OMC_EUNSUPPORTED: return "unsupported";
    case OMC_ERANGE: return "activation outside the f16 operand range";
    default: return "unknown status";
    }
}

const char *omc_version(void) { return "overhang_b200 omc 0.1 (sm_100a)"; }

long long omc_launch_count(int reset) {
    long long n = omc_g_launches;
    if (reset) omc_g_launches = 0;
    return n;
}

/* ---------------------------------------------------------------- slab -- */
/* One budget of HBM for expert weights, handed out in 256-byte aligned
 * pieces from 1 GiB chunks cudaMalloc'd on demand.  Past the budget an
 * upload fails with OMC_ENOMEM: the kernels copy weights with bulk
 * asynchronous copies and are only ever given HBM.  A layer larger than its
 * share of HBM uses the tiered store instead (omc_tier.c), whose host copies
 * reach HBM before any kernel reads them.  *on_host is always 0. */
#define SLAB_CHUNK ((size_t)1 << 30)

void *omc_slab_alloc(size_t n, int *on_host) {
    n = (n + 255) & ~(size_t)255;
    *on_host = 0;
    if (G.slab_used + n > G.slab_budget) return NULL;
    if (!G.nchunk || G.chunk_used + n > G.chunk_size[G.nchunk - 1]) {
        if (G.nchunk == OMC_MAX_CHUNKS) return NULL;
        size_t sz = n > SLAB_CHUNK ? n : SLAB_CHUNK;
        if (sz > G.slab_budget - G.slab_used) sz = G.slab_budget - G.slab_used;
        if (sz < n) return NULL;
        void *p = NULL;
        if (cudaMalloc(&p, sz) != cudaSuccess) {
            cudaGetLastError();
            return NULL;
        }
        G.chunk[G.nchunk] = p;
        G.chunk_size[G.nchunk] = sz;
        G.nchunk++;
        G.chunk_used = 0;
    }
    void *p = (char *)G.chunk[G.nchunk - 1] + G.chunk_used;
    G.chunk_used += n;
    G.slab_used += n;
    return p;
}

static void slab_release(void) {
    for (int i = 0; i < G.nchunk; ++i) cudaFree(G.chunk[i]);
    G.nchunk = 0;
    G.slab_used = G.chunk_used = 0;
}

/* ---------------------------------------------------------------- init -- */
int omc_init(int device, size_t slab_bytes) {
    if (G.init) {
        if (device != G.device) return omc_fail(OMC_EINVAL, "omc_init: already bound to device %d", G.device);
        return OMC_OK;
    }
    int n = 0;
    CK(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return omc_fail(OMC_EINVAL, "omc_init: device %d of %d", device, n);
    CK(cudaSetDevice(device));
    struct cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return omc_fail(OMC_EUNSUPPORTED, "omc_init: %s is sm_%d%d; this build is sm_100a",
                                          prop.name, prop.major, prop.minor);
    G.num_sms = prop.multiProcessorCount;
    CK(cudaStreamCreateWithFlags(&G.stream, cudaStreamNonBlocking));
    CK(cudaMalloc((void **)&G.d_err, 16 * sizeof(int)));
    CK(cudaMemsetAsync(G.d_err, 0, 16 * sizeof(int), G.stream));
    CK(cudaStreamSynchronize(G.stream));
    for (int i = 0; i < OMC_NSTAGE_EV; ++i) CK(cudaEventCreate(&G.ev[i]));
    if (slab_bytes == 0) {
        size_t fr = 0, tot = 0;
        CK(cudaMemGetInfo(&fr, &tot));
        const size_t reserve = (size_t)4 << 30;
        slab_bytes = fr > 2 * reserve ? fr - reserve : fr / 2;
    }
    G.slab_budget = slab_bytes;
    {
        const int rc = omc_noalloc_setup(device);   /* static scratch address, this device */
        if (rc) return omc_fail(rc, "omc_init: cudaGetSymbolAddress of the no-alloc scratch failed");
    }
    G.device = device;
    G.init = 1;
    const char *p = getenv("OMC_FFN_PATH");
    G.path_override = !p ? 0 : (!strcmp(p, "gemv") ? 1 : (!strcmp(p, "mma") ? 2 : (!strcmp(p, "decode") ? 3 : 0)));
    return OMC_OK;
}

static void ws_free(void);
static int dec_ensure(const omc_layer_dev *P);

void omc_shutdown(void) {
    if (!G.init) return;
    cudaSetDevice(G.device);
    cudaDeviceSynchronize();
    graphs_release();
    async_release();
    omc_ep_release();
    omc_tier_release();
    for (int i = 0; i < G.nlayers; ++i) {
        omc_tier_free(&G.layers[i]);
        free(G.layers[i].h_experts);
        cudaFree(G.layers[i].d_experts_tab);
        cudaFree(G.layers[i].rf_mem);
        cudaFree(G.layers[i].rt_mem);
    }
    free(G.layers);
    G.layers = NULL;
    G.nlayers = 0;
    ws_free();
    slab_release();
    cudaFree(G.staging);
    G.staging = NULL;
    G.staging_bytes = 0;
    for (int i = 0; i < OMC_NSTAGE_EV; ++i) cudaEventDestroy(G.ev[i]);
    if (G.timer_created)
        for (int i = 0; i < 2 * OMC_TIMER_RING; ++i) cudaEventDestroy(G.timer_ev[i]);
    cudaFree(G.d_err);
    cudaStreamDestroy(G.stream);
    memset(&G, 0, sizeof(G));
}

/* ---------------------------------------------------------------- layers -- */
omc_layer *omc_get_layer(int layer) {
    if (layer < 0 || layer >= G.nlayers || !G.layers[layer].used) return NULL;
    return &G.layers[layer];
}

static int staging_ensure(size_t n) {
    if (n <= G.staging_bytes) return OMC_OK;
    cudaStreamSynchronize(G.stream);
    cudaFree(G.staging);
    G.staging = NULL;
    G.staging_bytes = 0;
    CK(cudaMalloc(&G.staging, n));
    G.staging_bytes = n;
    return OMC_OK;
}

/* The bounded router's per-layer data (router_fast.cu), one allocation: the
 * f16 tiles of the router rows (int8 routers: their values, exact in f16;
 * f32 routers: the f16 rounding of each row, then the f16 rounding of the
 * remainder, as rows E..2E-1), row scales of 1, the one-matrix pointer table,
 * and each row's ||w||_2 and ||w||_1 from the host rows in double, rounded
 * up.  GEMMA layers (the router reads a normed input), D % 8 != 0, and f32
 * routers with a value outside the f16 range keep the exact router only. */
static int rf_setup(omc_layer *L, const void *router_w) {
    omc_layer_dev *P = &L->dev;
    const int E = P->E, D = P->D;
    P->rf_tab = NULL;
    P->rf_wn = NULL;
    P->rf_wc = NULL;
    P->rf_rows = 0;
    P->rf_split = 0;
    if (P->family == OMC_FAMILY_GEMMA || D % 8 || E <= 0) return OMC_OK;
    float *hn = malloc(sizeof(float) * 2 * (size_t)E);
    if (!hn) return omc_fail(OMC_ENOMEM, "omc_layer_init: host alloc");
    double amax = 0.0;
    for (int e = 0; e < E; ++e) {
        double s2 = 0.0, s1 = 0.0;
        for (int i = 0; i < D; ++i) {
            const double w = P->router_i8 ? (double)((const int8_t *)router_w)[(size_t)e * D + i]
                                          : (double)((const float *)router_w)[(size_t)e * D + i];
            s2 += w * w;
            s1 += fabs(w);
            if (!(fabs(w) <= amax)) amax = fabs(w);   /* NaN sticks */
        }
        hn[e] = nextafterf((float)(sqrt(s2) * (1.0 + 1e-9)), INFINITY);
        hn[E + e] = nextafterf((float)(s1 * (1.0 + 1e-9)), INFINITY);
    }
    if (!P->router_i8 && !(amax < 65000.0)) {
        free(hn);
        return OMC_OK;
    }
    const int M = P->router_i8 ? E : 2 * E;
    const int Mrows = omc_round_up(M, OMC_TM);
    const size_t tb = (omc_f16_tiles_bytes(M, D) + 255) & ~(size_t)255;
    const size_t ob = ((size_t)Mrows * 4 + 255) & ~(size_t)255;
    const size_t nb = ((size_t)E * 2 * 4 + 255) & ~(size_t)255;
    /* chunk-major router rows (rf_wc): 64 bytes per row and chunk */
    const int kce = P->router_i8 ? 64 : 16;
    const size_t q1 = ((size_t)E * D * (P->router_i8 ? 1 : 4) + 255) & ~(size_t)255;   /* one copy */
    const size_t qb = (D % kce) == 0 ? q1 * OMC_RF_NREP : 0;
    unsigned char *hq = qb ? malloc(q1) : NULL;
    if (qb && !hq) {
        free(hn);
        return omc_fail(OMC_ENOMEM, "omc_layer_init: host alloc");
    }
    if (hq) {
        const int nchk = D / kce, esz = P->router_i8 ? 1 : 4;
        for (int c = 0; c < nchk; ++c)
            for (int e = 0; e < E; ++e)
                for (int pc = 0; pc < 4; ++pc) {
                    const int slot = pc ^ ((e >> 1) & 3);
                    const unsigned char *src = (const unsigned char *)router_w +
                                               ((size_t)e * D + (size_t)c * kce + (size_t)pc * (16 / esz)) * esz;
                    memcpy(hq + ((size_t)c * E + e) * 64 + (size_t)slot * 16, src, 16);
                }
    }
    char *mem = NULL;
    float *tmp = NULL, *ones = malloc(sizeof(float) * (size_t)Mrows);
    int rc = OMC_OK;
    if (!ones || cudaMalloc((void **)&mem, tb + ob + nb + 256 + qb) != cudaSuccess ||
        (!P->router_i8 && cudaMalloc((void **)&tmp, (size_t)2 * E * D * 4) != cudaSuccess)) {
        cudaGetLastError();
        rc = omc_fail(OMC_ENOMEM, "omc_layer_init: bounded router tiles");
        goto out;
    }
    for (int i = 0; i < Mrows; ++i) ones[i] = 1.f;
    uint16_t *tiles = (uint16_t *)mem;
    float *d_ones = (float *)(mem + tb), *d_wn = (float *)(mem + tb + ob);
    omc_expert_ptrs tab;
    memset(&tab, 0, sizeof(tab));
    tab.d = (const int8_t *)tiles;
    tab.ds = d_ones;
    omc_expert_ptrs *d_tab = (omc_expert_ptrs *)(mem + tb + ob + nb);
    if (!P->router_i8 && (rc = omc_launch_rf_split_rows(P->router, E, D, tmp, G.stream))) goto out;
    if ((rc = omc_launch_f16_tiles(P->router_i8 ? P->router : tmp, M, D, tiles, G.d_err, G.stream))) goto out;
    if (cudaMemcpyAsync(d_ones, ones, sizeof(float) * (size_t)Mrows, cudaMemcpyHostToDevice, G.stream) ||
        cudaMemcpyAsync(d_wn, hn, sizeof(float) * 2 * (size_t)E, cudaMemcpyHostToDevice, G.stream) ||
        cudaMemcpyAsync(d_tab, &tab, sizeof(tab), cudaMemcpyHostToDevice, G.stream) ||
        (qb && cudaMemcpyAsync(mem + tb + ob + nb + 256, hq, q1, cudaMemcpyHostToDevice, G.stream)) ||
        cudaStreamSynchronize(G.stream)) {
        cudaGetLastError();
        rc = omc_fail(OMC_ECUDA, "omc_layer_init: bounded router upload");
        goto out;
    }
    /* the other copies of the chunk-major rows (see rf_wc) */
    for (int r = 1; qb && r < OMC_RF_NREP; ++r)
        if (cudaMemcpyAsync(mem + tb + ob + nb + 256 + (size_t)r * q1, mem + tb + ob + nb + 256, q1,
                            cudaMemcpyDeviceToDevice, G.stream) != cudaSuccess) {
            cudaGetLastError();
            rc = omc_fail(OMC_ECUDA, "omc_layer_init: bounded router copies");
            goto out;
        }
    if (qb && cudaStreamSynchronize(G.stream) != cudaSuccess) {
        cudaGetLastError();
        rc = omc_fail(OMC_ECUDA, "omc_layer_init: bounded router copies");
        goto out;
    }
    if ((rc = omc_check_device_error())) goto out;
    L->rf_mem = mem;
    mem = NULL;
    P->rf_tab = d_tab;
    P->rf_wn = d_wn;
    P->rf_rows = M;
    P->rf_split = P->router_i8 ? 0 : 1;
    P->rf_wc = qb ? (const unsigned char *)((char *)L->rf_mem + tb + ob + nb + 256) : NULL;
    P->rf_wc_stride = q1;
out:
    cudaFree(mem);
    cudaFree(tmp);
    free(ones);
    free(hn);
    free(hq);
    return rc;
}

int omc_layer_init(int layer, const omc_moe_desc *d, const void *router_w, const float *router_s) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_layer_init: omc_init not called");
    if (layer < 0 || layer > 4096 || !d || !router_w) return omc_fail(OMC_EINVAL, "omc_layer_init: bad arguments");
    if (d->family != OMC_FAMILY_OLMOE && d->family != OMC_FAMILY_QWEN && d->family != OMC_FAMILY_GEMMA)
        return omc_fail(OMC_EINVAL, "omc_layer_init: unknown family %d", d->family);
    if (d->D <= 0 || d->I <= 0 || d->E <= 0 || d->k <= 0 || d->k > d->E || d->k > OMC_MAX_K || d->E > OMC_MAX_E ||
        (d->D % 64) || (d->I % 16))
        return omc_fail(OMC_EINVAL, "omc_layer_init: shape D=%d I=%d E=%d k=%d (D%%64, I%%16, k<=%d, E<=%d)", d->D,
                        d->I, d->E, d->k, OMC_MAX_K, OMC_MAX_E);
    if (d->has_shared && (d->family != OMC_FAMILY_QWEN || d->Is <= 0 || (d->Is % 32)))
        return omc_fail(OMC_EINVAL, "omc_layer_init: shared expert needs QWEN family and Is%%32==0");
    if (d->router_dtype == OMC_ROUTER_I8 && !router_s)
        return omc_fail(OMC_EINVAL, "omc_layer_init: int8 router needs scales");
    if (layer >= G.nlayers) {
        int nn = layer + 1;
        omc_layer *nl = realloc(G.layers, sizeof(omc_layer) * nn);
        if (!nl) return omc_fail(OMC_ENOMEM, "omc_layer_init: host alloc");
        memset(nl + G.nlayers, 0, sizeof(omc_layer) * (nn - G.nlayers));
        G.layers = nl;
        G.nlayers = nn;
    }
    omc_layer *L = &G.layers[layer];
    graphs_invalidate();
    if (L->used) {
        cudaDeviceSynchronize();
        omc_tier_free(L);
        free(L->h_experts);
        cudaFree(L->d_experts_tab);
        cudaFree(L->rf_mem);
        cudaFree(L->rt_mem);
        /* slab space of a re-initialised layer is not reclaimed (bump allocator) */
    }
    memset(L, 0, sizeof(*L));
    L->desc = *d;
    if (d->family == OMC_FAMILY_QWEN || d->family == OMC_FAMILY_GEMMA) L->desc.renorm = 1;
    omc_layer_dev *P = &L->dev;
    P->family = d->family;
    P->act = d->family == OMC_FAMILY_QWEN ? OMC_ACT_SILU_SIG
           : d->family == OMC_FAMILY_GEMMA ? OMC_ACT_GELU_TANH : OMC_ACT_SILU_DIV;
    P->D = d->D; P->I = d->I; P->E = d->E; P->k = d->k;
    P->renorm = L->desc.renorm; P->router_i8 = d->router_dtype == OMC_ROUTER_I8;
    P->has_shared = d->has_shared; P->Is = d->has_shared ? d->Is : 0;
    P->D_pad = omc_round_up(d->D, OMC_KB);
    P->I_pad = omc_round_up(d->I, OMC_KB);
    P->Is_pad = d->has_shared ? omc_round_up(d->Is, OMC_KB) : 0;
    P->D_rows = omc_round_up(d->D, OMC_TM);
    P->I_rows = omc_round_up(d->I, OMC_TM);
    P->Is_rows = d->has_shared ? omc_round_up(d->Is, OMC_TM) : 0;
    /* EP: the experts this rank owns */
    L->e0 = 0;
    L->ne = d->E;
    if (G.ep_world > 1) {
        if (d->E % G.ep_world) return omc_fail(OMC_EINVAL, "omc_layer_init: E=%d not divisible by EP world %d",
                                                d->E, G.ep_world);
        L->ne = d->E / G.ep_world;
        L->e0 = G.ep_rank * L->ne;
    }
    int on_host;
    const size_t rbytes = (size_t)d->E * d->D * sizeof(float);
    float *router = omc_slab_alloc(rbytes, &on_host);
    if (!router) return omc_fail(OMC_ENOMEM, "omc_layer_init: router");
    if (P->router_i8) {
        int rc = staging_ensure((size_t)d->E * d->D);
        if (rc) return rc;
        /* on the library's stream (non-blocking): a plain cudaMemcpy would not
         * wait for an upload's relayout kernel that still reads the staging */
        CK(cudaMemcpyAsync(G.staging, router_w, (size_t)d->E * d->D, cudaMemcpyHostToDevice, G.stream));
        rc = omc_launch_i8_to_f32((const int8_t *)G.staging, router, (long long)d->E * d->D, G.stream);
        if (rc) return omc_fail(rc, "omc_layer_init: router conversion launch");
        float *rs = omc_slab_alloc((size_t)d->E * sizeof(float), &on_host);
        if (!rs) return omc_fail(OMC_ENOMEM, "omc_layer_init: router scales");
        CK(cudaMemcpyAsync(rs, router_s, (size_t)d->E * sizeof(float), cudaMemcpyHostToDevice, G.stream));
        P->router_s = rs;
    } else {
        CK(cudaMemcpyAsync(router, router_w, rbytes, cudaMemcpyHostToDevice, G.stream));
    }
    P->router = router;
    {
        int rc = rf_setup(L, router_w);
        if (rc) return rc;
    }
    /* the exact router's row blocks (the shared gate's row comes with omc_shared_set) */
    P->rt_w = NULL;
    P->rt_nrb = 0;
    if (d->D % 128 == 0) {
        const int nrb = (d->E + (d->has_shared ? 1 : 0) + 15) / 16;
        const size_t bytes = (size_t)nrb * (d->D / 128) * 16 * 128 * 4;
        if (cudaMalloc(&L->rt_mem, bytes) != cudaSuccess) {
            cudaGetLastError();
            return omc_fail(OMC_ENOMEM, "omc_layer_init: router row blocks");
        }
        CK(cudaMemsetAsync(L->rt_mem, 0, bytes, G.stream));
        int rc = omc_launch_rt_blocks(router, 0, d->E, d->D, (float *)L->rt_mem, G.stream);
        if (rc) return omc_fail(rc, "omc_layer_init: router row blocks");
        P->rt_w = (const float *)L->rt_mem;
        P->rt_nrb = nrb;
    }
    L->h_experts = calloc((size_t)d->E + 1, sizeof(omc_expert_ptrs));
    L->have = calloc((size_t)d->E + 1, 1);
    if (!L->h_experts || !L->have) return omc_fail(OMC_ENOMEM, "omc_layer_init: host alloc");
    CK(cudaMalloc((void **)&L->d_experts_tab, sizeof(omc_expert_ptrs) * ((size_t)d->E + 1)));
    CK(cudaMemsetAsync(L->d_experts_tab, 0, sizeof(omc_expert_ptrs) * ((size_t)d->E + 1), G.stream));
    P->experts = L->d_experts_tab;
    L->used = 1;
    CK(cudaStreamSynchronize(G.stream));
    if (G.ep_world <= 1) {
        int rc = dec_ensure(P);
        if (rc) return rc;
    }
    return OMC_OK;
}

int omc_layer_gemma_norms(int layer, float eps, const float *router_scale, const float *per_expert_scale,
                          const float *expert_norm) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_layer_gemma_norms: omc_init not called");
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_layer_gemma_norms: layer %d not initialised", layer);
    if (L->desc.family != OMC_FAMILY_GEMMA)
        return omc_fail(OMC_EINVAL, "omc_layer_gemma_norms: layer %d is not a GEMMA layer", layer);
    if (!router_scale || !per_expert_scale || !(eps >= 0.f))
        return omc_fail(OMC_EINVAL, "omc_layer_gemma_norms: router_scale and per_expert_scale are required, eps >= 0");
    const int D = L->desc.D, E = L->desc.E;
    float *h = malloc(sizeof(float) * (size_t)D);
    if (!h) return omc_fail(OMC_ENOMEM, "omc_layer_gemma_norms: host alloc");
    /* engines/gemma.c:459-460: the float product router.scale[i] * rroot,
     * rroot = 1.f/sqrtf((float)D), which the reference forms per element */
    const float rroot = 1.f / sqrtf((float)D);
    for (int i = 0; i < D; i++) h[i] = router_scale[i] * rroot;
    int on_host;
    float *s2 = omc_slab_alloc((size_t)D * sizeof(float), &on_host);
    float *pes = omc_slab_alloc((size_t)E * sizeof(float), &on_host);
    float *en = expert_norm ? omc_slab_alloc((size_t)D * sizeof(float), &on_host) : NULL;
    if (!s2 || !pes || (expert_norm && !en)) {
        free(h);
        return omc_fail(OMC_ENOMEM, "omc_layer_gemma_norms: slab");
    }
    /* host-to-device copies go on the library's stream: a blocking
     * cudaMemcpy from pageable memory may return before its transfer lands
     * and is not ordered with that (non-blocking) stream's kernels */
    cudaError_t e1 = cudaMemcpyAsync(s2, h, (size_t)D * sizeof(float), cudaMemcpyHostToDevice, G.stream);
    if (e1 == cudaSuccess)
        e1 = cudaMemcpyAsync(pes, per_expert_scale, (size_t)E * sizeof(float), cudaMemcpyHostToDevice, G.stream);
    if (e1 == cudaSuccess && en)
        e1 = cudaMemcpyAsync(en, expert_norm, (size_t)D * sizeof(float), cudaMemcpyHostToDevice, G.stream);
    if (e1 == cudaSuccess) e1 = cudaStreamSynchronize(G.stream);   /* the sources are consumed at return */
    free(h);
    CK(e1);
    graphs_invalidate();
    L->dev.eps = eps;
    L->dev.g_s2 = s2;
    L->dev.g_pes = pes;
    L->dev.g_en = en;
    L->gemma_ready = 1;
    return OMC_OK;
}

/* A per-expert term added to every routed logit before the softmax (bias
 * NULL: none).  Slab space of a replaced bias is not reclaimed. */
int omc_layer_router_bias(int layer, const float *bias) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_layer_router_bias: omc_init not called");
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_layer_router_bias: layer %d not initialised", layer);
    graphs_invalidate();
    if (!bias) {
        L->dev.rbias = NULL;
        return OMC_OK;
    }
    const int E = L->desc.E;
    for (int e = 0; e < E; ++e)
        if (!isfinite(bias[e])) return omc_fail(OMC_EINVAL, "omc_layer_router_bias: bias[%d] is not finite", e);
    int on_host;
    float *b = omc_slab_alloc((size_t)E * sizeof(float), &on_host);
    if (!b) return omc_fail(OMC_ENOMEM, "omc_layer_router_bias: slab");
    CK(cudaMemcpyAsync(b, bias, (size_t)E * sizeof(float), cudaMemcpyHostToDevice, G.stream));
    CK(cudaStreamSynchronize(G.stream));
    L->dev.rbias = b;
    return OMC_OK;
}

/* Upload one row-major int8 matrix [O][K] + scales [O] into slab tiles at
 * dq (paired layout, see omc_expert_ptrs; `member` as in
 * omc_launch_relayout). */
static int upload_matrix(const int8_t *q, const float *s, int O, int K, int O_pad, int K_pad, int8_t *dq, int member,
                         const float **ws, const float *scales_into) {
    int on_host;
    float *dsc = scales_into ? (float *)scales_into : omc_slab_alloc((size_t)O_pad * sizeof(float), &on_host);
    if (!dsc) return omc_fail(OMC_ENOMEM, "expert upload: slab budget exhausted (omc_init slab_bytes; omc_tier_enable for a layer larger than its HBM share)");
    int rc = staging_ensure((size_t)O * K);
    if (rc) return rc;
    CK(cudaMemcpyAsync(G.staging, q, (size_t)O * K, cudaMemcpyHostToDevice, G.stream));
    rc = omc_launch_relayout((const int8_t *)G.staging, O, K, dq, O_pad, K_pad, member, G.stream);
    if (rc) return omc_fail(rc, "expert upload: relayout launch");
    CK(cudaMemsetAsync(dsc, 0, (size_t)O_pad * sizeof(float), G.stream));
    CK(cudaMemcpyAsync(dsc, s, (size_t)O * sizeof(float), cudaMemcpyHostToDevice, G.stream));
    /* the staging buffer is reused by the next matrix */
    CK(cudaStreamSynchronize(G.stream));
    if (ws) *ws = dsc;
    return OMC_OK;
}

/* One expert (g, u [I][D], d [D][I] row-major int8, per-row scales) into the
 * paired tile layout.  reuse != 0: overwrite the buffers ep already points to
 * (same shape); otherwise allocate them from the slab. */
int omc_expert_upload(int D, int D_pad, int D_rows, int I_, int I_pad, int I_rows, const int8_t *g, const float *gs,
                      const int8_t *u, const float *us, const int8_t *d, const float *ds, omc_expert_ptrs *ep,
                      int reuse) {
    int rc, on_host = 0, on_host2 = 0;
    /* g and u interleave as the two members of each tile pair; d's row tiles
     * pair up (an odd last tile leaves its partner's blocks zero) */
    const size_t gu_bytes = (size_t)2 * I_rows * D_pad;
    const size_t d_bytes = (size_t)omc_round_up(D_rows, 2 * OMC_TM) * I_pad;
    int8_t *gu = reuse ? (int8_t *)ep->g : omc_slab_alloc(gu_bytes, &on_host);
    int8_t *dd = reuse ? (int8_t *)ep->d : omc_slab_alloc(d_bytes, &on_host2);
    if (!gu || !dd) return omc_fail(OMC_ENOMEM, "expert upload: slab budget exhausted (omc_init slab_bytes; omc_tier_enable for a layer larger than its HBM share)");
    (void)on_host;
    (void)on_host2;
    CK(cudaMemsetAsync(dd, 0, d_bytes, G.stream));   /* gu is fully written by the two relayouts */
    const float *sg_ = NULL, *su_ = NULL, *sd_ = NULL;
    if ((rc = upload_matrix(g, gs, I_, D, I_rows, D_pad, gu, 0, reuse ? NULL : &sg_, reuse ? ep->gs : NULL))) return rc;
    if ((rc = upload_matrix(u, us, I_, D, I_rows, D_pad, gu, 1, reuse ? NULL : &su_, reuse ? ep->us : NULL))) return rc;
    if ((rc = upload_matrix(d, ds, D, I_, D_rows, I_pad, dd, -1, reuse ? NULL : &sd_, reuse ? ep->ds : NULL))) return rc;
    if (!reuse) {
        ep->gs = sg_;
        ep->us = su_;
        ep->ds = sd_;
    }
    ep->g = gu;
    ep->u = gu + OMC_BLK_BYTES;
    ep->d = dd;
    return OMC_OK;
}

/* One row-major int8 matrix [O][K] + row scales as the down matrix of a
 * one-expert layer (row tiles paired consecutively).  reuse != 0: write into
 * the buffers *dq and *ds already hold (same shape). */
int omc_matrix_upload(const int8_t *q, const float *s, int O, int K, int8_t **dq, const float **ds, int reuse) {
    const int O_rows = omc_round_up(O, OMC_TM), K_pad = omc_round_up(K, OMC_KB);
    const size_t bytes = (size_t)omc_round_up(O_rows, 2 * OMC_TM) * K_pad;
    int on_host = 0, rc;
    int8_t *d = reuse ? *dq : omc_slab_alloc(bytes, &on_host);
    if (!d) return omc_fail(OMC_ENOMEM, "matrix upload: slab budget exhausted (omc_init slab_bytes; omc_tier_enable for a layer larger than its HBM share)");
    (void)on_host;
    CK(cudaMemsetAsync(d, 0, bytes, G.stream));
    const float *sd = NULL;
    if ((rc = upload_matrix(q, s, O, K, O_rows, K_pad, d, -1, reuse ? NULL : &sd, reuse ? *ds : NULL))) return rc;
    if (!reuse) *ds = sd;
    *dq = d;
    return OMC_OK;
}

static int set_expert_slot(omc_layer *L, int slot, int I_, int I_pad, int I_rows, const int8_t *g, const float *gs,
                           const int8_t *u, const float *us, const int8_t *d, const float *ds) {
    const omc_layer_dev *P = &L->dev;
    omc_expert_ptrs ep;
    int rc;
    memset(&ep, 0, sizeof(ep));
    if ((rc = omc_expert_upload(P->D, P->D_pad, P->D_rows, I_, I_pad, I_rows, g, gs, u, us, d, ds, &ep, 0))) return rc;
    L->h_experts[slot] = ep;
    L->have[slot] = 1;
    /* pageable source: staged by the runtime before the call returns */
    CK(cudaMemcpyAsync(L->d_experts_tab + slot, &ep, sizeof(ep), cudaMemcpyHostToDevice, G.stream));
    return OMC_OK;
}

int omc_expert_set(int layer, int e, const int8_t *g, const float *gs, const int8_t *u, const float *us,
                   const int8_t *d, const float *ds) {
    graphs_invalidate();
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_expert_set: layer %d not initialised", layer);
    if (e < 0 || e >= L->desc.E || !g || !gs || !u || !us || !d || !ds)
        return omc_fail(OMC_EINVAL, "omc_expert_set: bad expert %d or null pointer", e);
    if (e < L->e0 || e >= L->e0 + L->ne) return OMC_OK;   /* owned by another EP rank */
    if (L->tier) return omc_tier_upload(L, e, g, gs, u, us, d, ds);
    return set_expert_slot(L, e, L->desc.I, L->dev.I_pad, L->dev.I_rows, g, gs, u, us, d, ds);
}

int omc_experts_set_packed(int layer, const int8_t *g, const float *gs, const int8_t *u, const float *us,
                           const int8_t *d, const float *ds) {
    graphs_invalidate();
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_experts_set_packed: layer %d not initialised", layer);
    const size_t D = L->desc.D, I = L->desc.I;
    for (int e = 0; e < L->desc.E; ++e) {
        int rc = omc_expert_set(layer, e, g + e * I * D, gs + e * I, u + e * I * D, us + e * I, d + e * D * I,
                                ds + e * D);
        if (rc) return rc;
    }
    return OMC_OK;
}

int omc_shared_set(int layer, const int8_t *g, const float *gs, const int8_t *u, const float *us, const int8_t *d,
                   const float *ds, const float *sh_gate) {
    graphs_invalidate();
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_shared_set: layer %d not initialised", layer);
    if (!L->desc.has_shared) return omc_fail(OMC_EINVAL, "omc_shared_set: layer %d has no shared expert", layer);
    if (!g || !gs || !u || !us || !d || !ds || !sh_gate) return omc_fail(OMC_EINVAL, "omc_shared_set: null pointer");
    int on_host;
    float *sgv = omc_slab_alloc((size_t)L->desc.D * sizeof(float), &on_host);
    if (!sgv) return omc_fail(OMC_ENOMEM, "omc_shared_set: gate vector");
    CK(cudaMemcpyAsync(sgv, sh_gate, (size_t)L->desc.D * sizeof(float), cudaMemcpyHostToDevice, G.stream));
    L->dev.sh_gate = sgv;
    if (L->dev.rt_w) {
        /* row E of the exact router's row blocks */
        int rc = omc_launch_rt_blocks(sgv, L->desc.E, 1, L->desc.D, (float *)L->rt_mem, G.stream);
        if (rc) return omc_fail(rc, "omc_shared_set: router row blocks");
    }
    CK(cudaStreamSynchronize(G.stream));
    return set_expert_slot(L, L->desc.E, L->desc.Is, L->dev.Is_pad, L->dev.Is_rows, g, gs, u, us, d, ds);
}

/* ---------------------------------------------------------------- workspace -- */
static void ws_free(void) {
    void **p = (void **)&G.ws_ptrs;
    for (size_t i = 0; i < sizeof(G.ws_ptrs) / sizeof(void *); ++i) {
        cudaFree(p[i]);
        p[i] = NULL;
    }
    memset(&G.ws, 0, sizeof(G.ws));
    memset(G.ws_bytes, 0, sizeof(G.ws_bytes));
    cudaFree(G.dec_ctr);
    cudaFree(G.dec_part);
    G.dec_ctr = NULL;
    G.dec_part = NULL;
    G.dec_ctr_n = G.dec_part_n = 0;
}

/* Grows the fused-decode state to serve layer P (every T <= 8).  New
 * counters start at zero; the kernel leaves them at zero after a forward. */
static int dec_ensure(const omc_layer_dev *P) {
    size_t ci = 0, pf = 0;
    if (omc_decode_state_size(P, G.num_sms, &ci, &pf)) return OMC_OK;   /* layer not served by it */
    if (ci <= G.dec_ctr_n && pf <= G.dec_part_n) return OMC_OK;
    if (ci < G.dec_ctr_n) ci = G.dec_ctr_n;
    if (pf < G.dec_part_n) pf = G.dec_part_n;
    CK(cudaDeviceSynchronize());
    graphs_invalidate();
    cudaFree(G.dec_ctr);
    cudaFree(G.dec_part);
    G.dec_ctr = NULL;
    G.dec_part = NULL;
    G.dec_ctr_n = G.dec_part_n = 0;
    if (cudaMalloc((void **)&G.dec_ctr, ci * sizeof(int)) != cudaSuccess ||
        cudaMalloc((void **)&G.dec_part, pf * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        return omc_fail(OMC_ENOMEM, "decode state: cudaMalloc(%zu ints, %zu floats) failed", ci, pf);
    }
    /* a blocking cudaMemset is not ordered with the library's non-blocking
     * stream: zero on it and wait, so that any stream's launch sees zeros */
    CK(cudaMemsetAsync(G.dec_ctr, 0, ci * sizeof(int), G.stream));
    CK(cudaStreamSynchronize(G.stream));
    G.dec_ctr_n = ci;
    G.dec_part_n = pf;
    return OMC_OK;
}

/* grow-only buffer of a workspace whose sizes are bytes[] */
static int ws_buf_in(size_t *bytes, int slot, void **ptr, size_t need) {
    if (need == 0) need = 256;
    if (bytes[slot] >= need && *ptr) return OMC_OK;
    cudaStreamSynchronize(G.stream);
    cudaDeviceSynchronize();
    graphs_invalidate();
    cudaFree(*ptr);
    *ptr = NULL;
    size_t n = need + need / 4;
    cudaError_t e = cudaMalloc(ptr, n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        bytes[slot] = 0;
        return omc_fail(OMC_ENOMEM, "workspace: cudaMalloc(%zu) failed", n);
    }
    bytes[slot] = n;
    return OMC_OK;
}

/* Workspace for Tz tokens (or explicit rows) with nslots routed slots and
 * nshared implicit shared-expert rows, in (ws, W, bytes): the library's own
 * (G.ws) or another caller's (the expert-parallel pass). */
static int ws_ensure_in(const omc_layer *L, size_t Tz, size_t nslots, size_t nshared, int host_io, omc_ws *ws,
                        omc_ws_ptrs *W, size_t *bytes) {
    const omc_layer_dev *P = &L->dev;
    const size_t D = (size_t)P->D, E = (size_t)P->E, K = (size_t)P->k;
    const size_t Imax_rows = (size_t)(P->Is_rows > P->I_rows ? P->Is_rows : P->I_rows);
    const size_t Imax_pad = (size_t)(P->Is_pad > P->I_pad ? P->Is_pad : P->I_pad);
    const int T = (int)Tz;
    /* activation rows: every routed slot + shared rows + 16-row padding per expert */
    const size_t R = omc_round_up((int)(nslots + nshared + (E + 1) * OMC_ROW_ALIGN), 128);
    int rc = 0;
#define ws_buf(slot, ptr, need) ws_buf_in(bytes, slot, ptr, need)
    if (host_io) {
        if ((rc = ws_buf(0, (void **)&W->x, Tz * D * 4))) return rc;
        if ((rc = ws_buf(1, (void **)&W->out, Tz * D * 4))) return rc;
    }
    if ((rc = ws_buf(2, (void **)&W->logits, Tz * (E + 1) * 4))) return rc;
    if ((rc = ws_buf(3, (void **)&W->topk_idx, Tz * K * 4))) return rc;
    if ((rc = ws_buf(4, (void **)&W->topk_w, Tz * K * 4))) return rc;
    if ((rc = ws_buf(5, (void **)&W->sg, Tz * 4))) return rc;
    if ((rc = ws_buf(6, (void **)&W->counts, (E + 4) * 4 * 3 + 64))) return rc;
    if ((rc = ws_buf(7, (void **)&W->rowinfo, R * 8))) return rc;   /* rowinfo, then roww */
    if ((rc = ws_buf(8, (void **)&W->work, (size_t)omc_mma_work_items(P, (int)R) * 16))) return rc;
    if ((rc = ws_buf(9, (void **)&W->xh, Tz * D * 2))) return rc;
    if ((rc = ws_buf(10, (void **)&W->hp, Imax_pad * R * 2))) return rc;
    if ((rc = ws_buf(11, (void **)&W->ypart, Tz * (K + 1) * D * 4))) return rc;
    if ((rc = ws_buf(12, (void **)&W->hbuf, (Tz * K + Tz) * Imax_rows * 4))) return rc;
    if ((rc = ws_buf(13, (void **)&W->slotrow, (nslots > Tz * K ? nslots : Tz * K) * 4))) return rc;
    if (P->family == OMC_FAMILY_GEMMA) {
        if ((rc = ws_buf(14, (void **)&W->xg_r, Tz * D * 4))) return rc;
        if ((rc = ws_buf(15, (void **)&W->xg_e, Tz * D * 4))) return rc;
    }
#undef ws_buf
    ws->T_cap = T;
    ws->R_cap = (int)R;
    ws->x = W->x;
    ws->out = W->out;
    ws->logits = W->logits;
    ws->topk_idx = W->topk_idx;
    ws->topk_w = W->topk_w;
    ws->sg = W->sg;
    ws->counts = W->counts;
    ws->offsets = W->counts + (E + 4);
    ws->done = W->counts + 2 * (E + 4);
    ws->nwork = W->counts + 3 * (E + 4);
    ws->slotrow = W->slotrow;
    ws->rowinfo = W->rowinfo;
    ws->roww = (float *)(W->rowinfo + R);
    ws->work = W->work;
    ws->xh = W->xh;
    ws->hp = W->hp;
    ws->ypart = W->ypart;
    ws->hbuf = W->hbuf;
    ws->xg_r = P->family == OMC_FAMILY_GEMMA ? W->xg_r : NULL;
    ws->xg_e = P->family == OMC_FAMILY_GEMMA ? W->xg_e : NULL;
    ws->err = G.d_err;
    return OMC_OK;
}

/* The bounded router's buffers in the library's own workspace (the forward
 * entries' prefill calls): the split operand (2T rows), the products, the row
 * map and work items, the per-token state and two job lists of
 * T * roundup(E + 1, 4) chains each (every token taken whole, the bound). */
static int ws_ensure_rf(const omc_layer *L, int T) {
    const omc_layer_dev *P = &L->dev;
    if (!P->rf_tab || T < OMC_RF_TMIN || omc_router_exact == 1 || (omc_router_exact == 0 && P->E < OMC_RF_EMIN))
        return OMC_OK;
    const size_t R = (size_t)omc_round_up(2 * T, 128);
    const size_t nitems = R / 128 * (size_t)((P->rf_rows + OMC_TM - 1) / OMC_TM);
    const size_t jcap = (size_t)T * (size_t)((P->E + 4) & ~3);
    const size_t nseg = (size_t)(P->D_pad + 255) / 256;
    const size_t misc = R * 2 + nitems * 4 + 16 + (size_t)T * 4 + (size_t)T * nseg * 2;   /* ints */
    int rc;
    omc_ws_ptrs *W = &G.ws_ptrs;
    size_t *bytes = G.ws_bytes;
    if ((rc = ws_buf_in(bytes, 16, (void **)&W->rf_act, (size_t)P->D_pad * R * 2))) return rc;
    if ((rc = ws_buf_in(bytes, 17, (void **)&W->rf_y, R * (size_t)P->rf_rows * 4))) return rc;
    if ((rc = ws_buf_in(bytes, 18, (void **)&W->rf_misc, misc * 4))) return rc;
    if ((rc = ws_buf_in(bytes, 19, (void **)&W->rf_jobs, jcap * 2 * 8))) return rc;
    omc_ws *ws = &G.ws;
    ws->rf_R = (int)R;
    ws->rf_act = W->rf_act;
    ws->rf_y = W->rf_y;
    ws->rf_rowinfo = W->rf_misc;
    ws->rf_roww = (float *)(W->rf_misc + R);
    ws->rf_work = W->rf_misc + 2 * R;
    /* every region starts on a multiple of 4 ints: rf_work and rf_tok are
     * read and written as int4 */
    ws->rf_ctl = W->rf_misc + 2 * R + nitems * 4;
    ws->rf_tok = ws->rf_ctl + 16;
    ws->rf_xn = (float *)(ws->rf_tok + (size_t)T * 4);
    ws->rf_jobs = W->rf_jobs;
    ws->rf_jobs2 = W->rf_jobs + jcap * 2;
    ws->rf_jcap = (int)jcap;
    return OMC_OK;
}

/* Counters of the last bounded-router pass on the library's workspace:
 * out[0] chain jobs, out[1] retry jobs, out[2] tokens taken whole from the
 * start, out[3] tokens retried (synchronises the library's stream). */
int omc_router_stats(int *out) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_router_stats: omc_init not called");
    if (!out) return omc_fail(OMC_EINVAL, "omc_router_stats: null pointer");
    memset(out, 0, sizeof(int) * 4);
    if (!G.ws.rf_ctl) return OMC_OK;
    CK(cudaStreamSynchronize(G.stream));
    CK(cudaMemcpy(out, G.ws.rf_ctl + 4, sizeof(int) * 4, cudaMemcpyDeviceToHost));
    return OMC_OK;
}

int omc_decode_stats(int *out, int reset) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_decode_stats: omc_init not called");
    if (!out) return omc_fail(OMC_EINVAL, "omc_decode_stats: null pointer");
    out[0] = out[1] = 0;
    if (!G.dec_ctr) return OMC_OK;
    CK(cudaDeviceSynchronize());   /* the decode may have run on a caller's stream */
    CK(cudaMemcpy(out, G.dec_ctr + OMC_DEC_CTR_STATS, sizeof(int) * 2, cudaMemcpyDeviceToHost));
    if (reset) {
        CK(cudaMemsetAsync(G.dec_ctr + OMC_DEC_CTR_STATS, 0, sizeof(int) * 2, G.stream));
        CK(cudaStreamSynchronize(G.stream));
    }
    return OMC_OK;
}

int omc_ws_ensure(const omc_layer *L, int T, int host_io) {
    const size_t Tz = (size_t)T;
    int rc = ws_ensure_in(L, Tz, Tz * (size_t)L->dev.k, L->dev.has_shared ? Tz : 0, host_io, &G.ws, &G.ws_ptrs,
                          G.ws_bytes);
    if (rc) return rc;
    /* buffers grow only: the pointers set for a larger T serve this one, but
     * rf_R and the job capacity are per call */
    return ws_ensure_rf(L, T);
}

int omc_ws_ensure_rows(const omc_layer *L, int rows) {
    return ws_ensure_in(L, (size_t)rows, (size_t)rows, 0, 0, &G.ws, &G.ws_ptrs, G.ws_bytes);
}

int omc_ws_ensure_rows_in(const omc_layer *L, int rows, omc_ws *ws, omc_ws_ptrs *W, size_t *bytes) {
    return ws_ensure_in(L, (size_t)rows, (size_t)rows, 0, 0, ws, W, bytes);
}

void omc_ws_free_in(omc_ws_ptrs *W, size_t *bytes, int nbytes) {
    void **p = (void **)W;
    for (size_t i = 0; i < sizeof(*W) / sizeof(void *); ++i) {
        cudaFree(p[i]);
        p[i] = NULL;
    }
    memset(bytes, 0, sizeof(size_t) * (size_t)nbytes);
}

/* ---------------------------------------------------------------- errors -- */
int omc_check_device_error(void) {
    int h[4] = {0, 0, 0, 0};
    cudaError_t e = cudaMemcpy(h, G.d_err, sizeof(h), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return omc_fail(OMC_ECUDA, "reading device error word: %s", cudaGetErrorString(e));
    if (!h[0]) return OMC_OK;
    cudaMemsetAsync(G.d_err, 0, sizeof(h), G.stream);
    /* a forward that stopped at a lost wait may leave decode counters set */
    if (G.dec_ctr) cudaMemsetAsync(G.dec_ctr, 0, G.dec_ctr_n * sizeof(int), G.stream);
    cudaStreamSynchronize(G.stream);
    const int st = h[0] == OMC_DEVERR_TIMEOUT ? OMC_ETIMEOUT : h[0] == OMC_DEVERR_RANGE ? OMC_ERANGE : OMC_EDEVICE;
    return omc_fail(st, "device error code %d at site %d (detail %d)", h[0], h[1], h[2]);
}

int omc_sync(void) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_sync: omc_init not called");
    if (G.ep_world > 1) {   /* a peer that left must not hang this wait */
        const int rc = omc_ep_wait();
        if (rc) return rc;
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return omc_fail(OMC_ECUDA, "omc_sync: %s", cudaGetErrorString(e));
    return omc_check_device_error();
}

/* ---------------------------------------------------------------- profiling -- */
int omc_set_profiling(int on) {
    G.profiling = on ? 1 : 0;
    return OMC_OK;
}

int omc_stage_times(float *ms, int n) {
    if (!G.init || !G.prof_valid) return 0;
    cudaEventSynchronize(G.ev[G.prof_nev - 1]);
    int k = 0;
    for (int i = 0; i + 1 < G.prof_nev && k < n; ++i, ++k) {
        float t = 0.f;
        if (cudaEventElapsedTime(&t, G.ev[i], G.ev[i + 1]) != cudaSuccess) {
            cudaGetLastError();
            t = -1.f;
        }
        ms[k] = t;
    }
    return k;
}

const char *omc_stage_name(int i) {
    if (!G.init || i < 0 || i + 1 >= G.prof_nev) return NULL;
    return G.prof_names[i];
}

/* Stage timer.  Every stage boundary of a forward re-records the tentative
 * start event of the current ring slot; the end of the named stage records
 * the slot's end event and moves to the next slot, so slot i keeps the
 * boundary just before the named stage and the one just after it. */
int omc_time_stage(const char *name) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_time_stage: omc_init not called");
    if (!name) {
        G.timer_on = 0;
        return OMC_OK;
    }
    if (strlen(name) >= sizeof(G.timer_name)) return omc_fail(OMC_EINVAL, "omc_time_stage: name too long");
    if (!G.timer_created) {
        for (int i = 0; i < 2 * OMC_TIMER_RING; ++i) CK(cudaEventCreate(&G.timer_ev[i]));
        G.timer_created = 1;
    }
    CK(cudaDeviceSynchronize());   /* no pair of an earlier timing is still pending */
    strcpy(G.timer_name, name);
    G.timer_n = 0;
    G.timer_on = 1;
    return OMC_OK;
}

int omc_stage_timer(float *mean_ms, int *count) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_stage_timer: omc_init not called");
    if (!mean_ms || !count) return omc_fail(OMC_EINVAL, "omc_stage_timer: null output");
    *mean_ms = 0.f;
    *count = 0;
    if (!G.timer_created || G.timer_n == 0) return OMC_OK;
    const int n = G.timer_n;
    const int last = (n - 1) % OMC_TIMER_RING;
    CK(cudaEventSynchronize(G.timer_ev[2 * last + 1]));
    /* once the ring has wrapped, the current slot holds a tentative start */
    const int cur = n % OMC_TIMER_RING;
    double sum = 0.0;
    int k = 0;
    for (int i = 0; i < OMC_TIMER_RING && i < n; ++i) {
        if (n >= OMC_TIMER_RING && i == cur) continue;
        float t = 0.f;
        CK(cudaEventElapsedTime(&t, G.timer_ev[2 * i], G.timer_ev[2 * i + 1]));
        sum += t;
        ++k;
    }
    *mean_ms = k ? (float)(sum / k) : 0.f;
    *count = k;
    return OMC_OK;
}

static void timer_boundary(cudaStream_t s, const char *ended) {
    const int slot = G.timer_n % OMC_TIMER_RING;
    if (ended && !strcmp(ended, G.timer_name)) {
        cudaEventRecord(G.timer_ev[2 * slot + 1], s);
        G.timer_n++;
        cudaEventRecord(G.timer_ev[2 * (G.timer_n % OMC_TIMER_RING)], s);
    } else {
        cudaEventRecord(G.timer_ev[2 * slot], s);
    }
}

static void prof_begin(cudaStream_t s) {
    G.prof_nev = 0;
    if (G.profiling) {
        cudaEventRecord(G.ev[0], s);
        G.prof_nev = 1;
    }
    if (G.timer_on) timer_boundary(s, NULL);
}

/* Ends the stage `name` on stream s (profiling or stage-timer mode only). */
void omc_prof_mark(cudaStream_t s, const char *name) {
    if (G.profiling && G.prof_nev > 0 && G.prof_nev < OMC_NSTAGE_EV) {
        cudaEventRecord(G.ev[G.prof_nev], s);
        G.prof_names[G.prof_nev - 1] = name;
        G.prof_nev++;
    }
    if (G.timer_on) timer_boundary(s, name);
}

/* ---------------------------------------------------------------- forward -- */
static int layer_ready(const omc_layer *L) {
    for (int e = L->e0; e < L->e0 + L->ne; ++e)
        if (!L->have[e]) return omc_fail(OMC_ENOINIT, "forward: expert %d of layer not uploaded", e);
    if (L->desc.has_shared && !L->have[L->desc.E])
        return omc_fail(OMC_ENOINIT, "forward: shared expert not uploaded");
    if (L->desc.family == OMC_FAMILY_GEMMA && !L->gemma_ready)
        return omc_fail(OMC_ENOINIT, "forward: GEMMA layer without omc_layer_gemma_norms");
    return OMC_OK;
}

/* Choose the expert path: tensor-core grouped GEMM from 128 routed slots
 * (or 4 per expert for small E), CUDA-core GEMV below.  Measured on B200
 * (one forward, CUDA-graph replay): OLMoE T=8 112 vs 127 us (GEMV ahead),
 * T=16 194 vs 135 us; Qwen T=16 174 vs 138 us, T=64 552 vs 234 us: the
 * GEMV path reads an expert's weights once per slot, the grouped GEMM once
 * per expert. */
static int g_force_f32;   /* set by omc_moe_forward while it redoes a forward on the f32 path */

static int use_mma(const omc_layer *L, int T) {
    if (g_force_f32 || G.path_override == 1 || G.path_override == 3) return 0;
    if (G.path_override == 2) return 1;
    const long long slots = (long long)T * L->desc.k;
    const long long need = 4LL * L->desc.E < 128 ? 4LL * L->desc.E : 128;
    return slots >= need;
}

/* One forward on workspace `ws` (kernels only: no allocation here). */
static int forward_on_ws(omc_layer *L, const omc_ws *ws, const float *x, int T, float *out, int32_t *topk_idx,
                         float *topk_w, cudaStream_t s) {
    int rc;
    int32_t *idx = topk_idx ? topk_idx : ws->topk_idx;
    float *w = topk_w ? topk_w : ws->topk_w;
    G.prof_valid = 0;
    prof_begin(s);
    const int mma = use_mma(L, T);
    omc_plan_args plan;
    if (mma) {
        /* the per-expert counts (counted by the select blocks) and the
         * select-done counter start at zero: counts, offsets, done are one
         * run of ints in the workspace */
        omc_plan_setup(&L->dev, T, ws, &plan);
        CK(cudaMemsetAsync(ws->counts, 0, (size_t)(ws->done - ws->counts + 1) * sizeof(int), s));
    }
    /* GEMMA: x is the residual; the router and the experts each read their
     * own norm of it (prenorm.cu).  The tensor-core path takes the experts'
     * input as its f16 operand, the CUDA-core paths as f32. */
    const int gemma = L->dev.family == OMC_FAMILY_GEMMA;
    /* decode: the whole block in one launch (decode.cu).  Chosen on its own
     * at T = 1, where it beats the router + GEMV kernels; from T = 2 its
     * CUDA-core dequant-and-dot is the bound and the separate kernels win
     * (measured on B200), so larger T take it only when it is forced.  It
     * takes GEMMA's residual rows as they are and norms them itself. */
    if (!mma && G.ep_world <= 1 && !L->tier && (G.path_override == 3 || (G.path_override == 0 && T == 1)) &&
        omc_decode_supported(&L->dev, T, G.num_sms, G.dec_ctr_n, G.dec_part_n)) {
        if ((rc = omc_launch_decode(&L->dev, x, x, T, ws, G.num_sms, G.dec_ctr, G.dec_part, idx, w, out, s)))
            return omc_fail(rc, "fused decode launch failed (%s)", omc_strerror(rc));
        G.prof_valid = G.profiling;
        return OMC_OK;
    }
    const float *xr = x, *xe = x;
    if (gemma) {
        if ((rc = omc_launch_gemma_prenorm(&L->dev, x, T, ws->xg_r, mma ? NULL : ws->xg_e, mma ? ws->xh : NULL, NULL,
                                           ws->err, s)))
            return omc_fail(rc, "prenorm launch failed");
        xr = ws->xg_r;
        xe = ws->xg_e;
    }
    if (G.path_override == 3) return omc_fail(OMC_EUNSUPPORTED, "fused decode path forced but not available for T=%d", T);
    if ((rc = omc_launch_router(&L->dev, xr, T, ws, idx, w, mma ? &plan : NULL, s)))
        return omc_fail(rc, "router launch failed");
    omc_prof_mark(s, "router_select");
    /* a tiered layer: the routed experts outside HBM are copied in first */
    if ((rc = omc_tier_route(L, idx, T, s))) return omc_fail(rc, "tier fetch launch failed");
    if (mma) {
        rc = omc_launch_mma_ffn(&L->dev, xe, T, ws, idx, w, out, s);
        if (rc == OMC_EUNSUPPORTED && G.path_override != 2) {
            if (gemma && (rc = omc_launch_gemma_prenorm(&L->dev, x, T, NULL, ws->xg_e, NULL, NULL, ws->err, s)))
                return omc_fail(rc, "prenorm launch failed");
            rc = omc_launch_gemv_ffn(&L->dev, xe, T, ws, idx, w, out, s);
        }
    } else {
        rc = omc_launch_gemv_ffn(&L->dev, xe, T, ws, idx, w, out, s);
    }
    if (rc) return omc_fail(rc, "expert FFN launch failed (%s)", omc_strerror(rc));
    G.prof_valid = G.profiling;
    return OMC_OK;
}

int omc_forward_device(omc_layer *L, const float *x, int T, float *out, int32_t *topk_idx, float *topk_w,
                       cudaStream_t s) {
    int rc;
    if ((rc = layer_ready(L))) return rc;
    if ((rc = omc_ws_ensure(L, T, 0))) return rc;
    if (G.ep_world > 1) {
        prof_begin(s);
        return omc_ep_forward(L, x, T, out, topk_idx, topk_w, s);
    }
    return forward_on_ws(L, &G.ws, x, T, out, topk_idx, topk_w, s);
}

/* ---------------------------------------------------- no-alloc forward -- */
/* Lays out one forward's workspace inside the static device scratch
 * (noalloc.cu).  Returns the bytes needed; fills *ws when base is given. */
static size_t noalloc_layout(const omc_layer_dev *P, int T, char *base, omc_ws *ws) {
    const size_t Tz = (size_t)T, D = (size_t)P->D, E = (size_t)P->E, K = (size_t)P->k;
    const size_t Imax_rows = (size_t)(P->Is_rows > P->I_rows ? P->Is_rows : P->I_rows);
    const size_t Imax_pad = (size_t)(P->Is_pad > P->I_pad ? P->Is_pad : P->I_pad);
    const size_t R = (size_t)omc_round_up((int)(Tz * K + (P->has_shared ? Tz : 0) + (E + 1) * OMC_ROW_ALIGN), 128);
    size_t off = 0;
#define TAKE(field, type, bytes)                                     \
    do {                                                             \
        if (base) ws->field = (type)(base + off);                    \
        off += ((size_t)(bytes) + 255) & ~(size_t)255;               \
    } while (0)
    TAKE(logits, float *, Tz * (E + 1) * 4);
    TAKE(topk_idx, int32_t *, Tz * K * 4);
    TAKE(topk_w, float *, Tz * K * 4);
    TAKE(sg, float *, Tz * 4);
    TAKE(counts, int *, (E + 4) * 4 * 3 + 64);
    TAKE(rowinfo, int *, R * 8);   /* rowinfo, then roww */
    TAKE(work, int *, (size_t)omc_mma_work_items(P, (int)R) * 16);
    TAKE(xh, uint16_t *, Tz * D * 2);
    TAKE(hp, uint16_t *, Imax_pad * R * 2);
    TAKE(ypart, float *, Tz * (K + 1) * D * 4);
    TAKE(hbuf, float *, (Tz * K + Tz) * Imax_rows * 4);
    TAKE(slotrow, int *, Tz * K * 4);
    if (P->family == OMC_FAMILY_GEMMA) {
        TAKE(xg_r, float *, Tz * D * 4);
        TAKE(xg_e, float *, Tz * D * 4);
    }
#undef TAKE
    if (base) {
        ws->offsets = ws->counts + (E + 4);
        ws->done = ws->counts + 2 * (E + 4);
        ws->nwork = ws->counts + 3 * (E + 4);
        ws->roww = (float *)(ws->rowinfo + R);
        ws->x = ws->out = NULL;
        ws->T_cap = T;
        ws->R_cap = (int)R;
        ws->err = G.d_err;
    }
    return off;
}

int omc_moe_forward_noalloc(int layer, const float *x, int T, float *out, int32_t *topk_idx, float *topk_w,
                            void *stream) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_moe_forward_noalloc: omc_init not called");
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_moe_forward_noalloc: layer %d not initialised", layer);
    if (T < 0 || (T > 0 && (!x || !out))) return omc_fail(OMC_EINVAL, "omc_moe_forward_noalloc: bad T or pointers");
    if (((uintptr_t)x | (uintptr_t)out) & 15)
        return omc_fail(OMC_EINVAL, "omc_moe_forward_noalloc: x and out must be 16-byte aligned");
    if (G.ep_world > 1)
        return omc_fail(OMC_EUNSUPPORTED, "omc_moe_forward_noalloc: not available with expert parallelism");
    if (T == 0) return OMC_OK;
    int rc;
    if ((rc = layer_ready(L))) return rc;
    const size_t need = noalloc_layout(&L->dev, T, NULL, NULL);
    if (need > OMC_NOALLOC_SCRATCH_BYTES) {
        int lo = 0, hi = T;   /* largest T that fits, for the message */
        while (lo < hi) {
            const int mid = (lo + hi + 1) / 2;
            if (noalloc_layout(&L->dev, mid, NULL, NULL) <= OMC_NOALLOC_SCRATCH_BYTES) lo = mid;
            else hi = mid - 1;
        }
        return omc_fail(OMC_EINVAL,
                        "omc_moe_forward_noalloc: T=%d needs %zu bytes of scratch, the static scratch holds %u; "
                        "at most T=%d for this layer",
                        T, need, (unsigned)OMC_NOALLOC_SCRATCH_BYTES, lo);
    }
    char *base = (char *)omc_noalloc_scratch_ptr(G.device);
    if (!base) return omc_fail(OMC_ENOINIT, "omc_moe_forward_noalloc: scratch address not set up");
    omc_ws ws;
    memset(&ws, 0, sizeof(ws));
    noalloc_layout(&L->dev, T, base, &ws);
    cudaStream_t s = stream ? (cudaStream_t)stream : G.stream;
    if ((rc = omc_tier_before(L, s))) return rc;
    if ((rc = forward_on_ws(L, &ws, x, T, out, topk_idx, topk_w, s))) return rc;
    return omc_tier_after(L, s);
}

int omc_moe_forward_dev(int layer, const float *x, int T, float *out, int32_t *topk_idx, float *topk_w,
                        void *stream) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_moe_forward_dev: omc_init not called");
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_moe_forward_dev: layer %d not initialised", layer);
    if (T < 0 || (T > 0 && (!x || !out))) return omc_fail(OMC_EINVAL, "omc_moe_forward_dev: bad T or pointers");
    if (((uintptr_t)x | (uintptr_t)out) & 15)
        return omc_fail(OMC_EINVAL, "omc_moe_forward_dev: x and out must be 16-byte aligned");
    if (T == 0 && G.ep_world <= 1) return OMC_OK;
    cudaStream_t s = stream ? (cudaStream_t)stream : G.stream;
    int rc;
    if ((rc = omc_tier_before(L, s))) return rc;
    if ((rc = omc_forward_device(L, x, T, out, topk_idx, topk_w, s))) return rc;
    return omc_tier_after(L, s);
}

int omc_moe_route_dev(int layer, const float *x, int T, int32_t *topk_idx, float *topk_w, float *shared_gate,
                      void *stream) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_moe_route_dev: omc_init not called");
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_moe_route_dev: layer %d not initialised", layer);
    if (T < 0 || (T > 0 && (!x || !topk_idx || !topk_w))) return omc_fail(OMC_EINVAL, "omc_moe_route_dev: bad T or pointers");
    if ((uintptr_t)x & 15) return omc_fail(OMC_EINVAL, "omc_moe_route_dev: x must be 16-byte aligned");
    if (T == 0) return OMC_OK;
    int rc;
    if ((rc = omc_ws_ensure(L, T, 0))) return rc;
    if (L->desc.family == OMC_FAMILY_GEMMA && !L->gemma_ready)
        return omc_fail(OMC_ENOINIT, "omc_moe_route_dev: GEMMA layer without omc_layer_gemma_norms");
    cudaStream_t s = stream ? (cudaStream_t)stream : G.stream;
    G.prof_valid = 0;
    if (L->desc.family == OMC_FAMILY_GEMMA) {
        if ((rc = omc_launch_gemma_prenorm(&L->dev, x, T, G.ws.xg_r, NULL, NULL, NULL, G.d_err, s)))
            return omc_fail(rc, "omc_moe_route_dev: prenorm launch failed");
        x = G.ws.xg_r;
    }
    if ((rc = omc_launch_router(&L->dev, x, T, &G.ws, topk_idx, topk_w, NULL, s)))
        return omc_fail(rc, "omc_moe_route_dev: router launch failed");
    if (shared_gate && L->desc.has_shared)
        CK(cudaMemcpyAsync(shared_gate, G.ws.sg, (size_t)T * sizeof(float), cudaMemcpyDeviceToDevice, s));
    return OMC_OK;
}

int omc_moe_experts_dev(int layer, const float *x_rows, int R, const int32_t *expert, const float *weight, float *y,
                        void *stream) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_moe_experts_dev: omc_init not called");
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_moe_experts_dev: layer %d not initialised", layer);
    if (R < 0 || (R > 0 && (!x_rows || !expert || !weight || !y)))
        return omc_fail(OMC_EINVAL, "omc_moe_experts_dev: bad R or pointers");
    if (((uintptr_t)x_rows | (uintptr_t)y) & 15)
        return omc_fail(OMC_EINVAL, "omc_moe_experts_dev: x_rows and y must be 16-byte aligned");
    if (R == 0) return OMC_OK;
    int rc;
    if (L->tier) return omc_fail(OMC_EUNSUPPORTED, "omc_moe_experts_dev: not on a tiered layer");
    for (int e = L->e0; e < L->e0 + L->ne; ++e)
        if (!L->have[e]) return omc_fail(OMC_ENOINIT, "omc_moe_experts_dev: expert %d not uploaded", e);
    if (L->desc.has_shared && !L->have[L->desc.E])
        return omc_fail(OMC_ENOINIT, "omc_moe_experts_dev: shared expert not uploaded");
    if (L->desc.family == OMC_FAMILY_GEMMA && !L->gemma_ready)
        return omc_fail(OMC_ENOINIT, "omc_moe_experts_dev: GEMMA layer without omc_layer_gemma_norms");
    if ((rc = omc_ws_ensure_rows(L, R))) return rc;
    cudaStream_t s = stream ? (cudaStream_t)stream : G.stream;
    G.prof_valid = 0;
    prof_begin(s);
    if ((rc = omc_launch_mma_rows(&L->dev, x_rows, R, &G.ws, expert, weight, L->e0, L->e0 + L->ne, y, s)))
        return omc_fail(rc, "omc_moe_experts_dev: launch failed");
    G.prof_valid = G.profiling;
    return OMC_OK;
}

/* ---------------------------------------------------- replayed forwards -- */
/* The device part of omc_moe_forward for one (layer, T) enqueues the same
 * launches on the same workspace every call.  The first call runs it as is
 * (allocations and one-time kernel attributes happen there); the second
 * captures it in a CUDA graph; from then on the graph is replayed, so a
 * tensor-core forward's six launches and memset cost one graph launch.  A
 * graph is valid for one generation (graphs_invalidate: layer and expert
 * set-up, workspace or decode-state growth, forced paths); profiling, the
 * stage timer and expert parallelism bypass it, and OMC_GRAPHS=0 turns it
 * off. */
#define OMC_NGRAPH 64
typedef struct {
    int layer, T, gen, warm, failed;
    const float *x;         /* the input buffer the graph reads (one graph per staging buffer) */
    cudaGraphExec_t exec;
    long long launches;     /* kernels in one replay */
} omc_fgraph;
static omc_fgraph g_fg[OMC_NGRAPH];
static int g_nfg, g_fg_next;

static void graphs_release(void) {
    for (int i = 0; i < g_nfg; ++i)
        if (g_fg[i].exec) cudaGraphExecDestroy(g_fg[i].exec);
    memset(g_fg, 0, sizeof(g_fg));
    g_nfg = g_fg_next = 0;
}

static int graphs_enabled(void) {
    static int on = -1;
    if (on < 0) {
        const char *e = getenv("OMC_GRAPHS");
        on = !(e && *e == '0');
    }
    return on && !G.profiling && !G.timer_on && G.ep_world <= 1;
}

static int forward_replayed(omc_layer *L, int layer, int T, const float *x, float *out, int32_t *idx, float *w,
                            cudaStream_t s) {
    omc_fgraph *g = NULL;
    for (int i = 0; i < g_nfg; ++i)
        if (g_fg[i].layer == layer && g_fg[i].T == T && g_fg[i].x == x) g = &g_fg[i];
    if (!g) {
        if (g_nfg < OMC_NGRAPH) g = &g_fg[g_nfg++];
        else {
            g = &g_fg[g_fg_next];
            g_fg_next = (g_fg_next + 1) % OMC_NGRAPH;
            if (g->exec) cudaGraphExecDestroy(g->exec);
        }
        memset(g, 0, sizeof(*g));
        g->layer = layer;
        g->T = T;
        g->x = x;
        g->gen = g_graph_gen;
    }
    if (g->gen != g_graph_gen) {
        if (g->exec) cudaGraphExecDestroy(g->exec);
        g->exec = NULL;
        g->warm = g->failed = 0;
        g->gen = g_graph_gen;
    }
    if (g->exec) {
        if (cudaGraphLaunch(g->exec, s) != cudaSuccess) {
            cudaGetLastError();
            return omc_fail(OMC_ECUDA, "forward replay failed");
        }
        omc_g_launches += g->launches;
        return OMC_OK;
    }
    if (!g->warm || g->failed) {
        g->warm = 1;
        return omc_forward_device(L, x, T, out, idx, w, s);
    }
    const long long l0 = omc_g_launches;
    if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        g->failed = 1;
        return omc_forward_device(L, x, T, out, idx, w, s);
    }
    int rc = omc_forward_device(L, x, T, out, idx, w, s);
    cudaGraph_t graph = NULL;
    const cudaError_t ce = cudaStreamEndCapture(s, &graph);
    cudaError_t ie = cudaErrorUnknown;
    if (!rc && ce == cudaSuccess && graph) ie = cudaGraphInstantiate(&g->exec, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    g->launches = omc_g_launches - l0;   /* the kernels one replay launches */
    omc_g_launches = l0;                 /* the capture itself launched nothing */
    if (rc || ce != cudaSuccess || ie != cudaSuccess) {
        cudaGetLastError();
        g->exec = NULL;
        g->failed = 1;
        if (rc) return rc;
        return omc_forward_device(L, x, T, out, idx, w, s);
    }
    if (cudaGraphLaunch(g->exec, s) != cudaSuccess) {
        cudaGetLastError();
        return omc_fail(OMC_ECUDA, "forward replay failed");
    }
    omc_g_launches += g->launches;
    return OMC_OK;
}

int omc_moe_forward(int layer, const float *x, int T, float *out, int32_t *topk_idx, float *topk_w) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_moe_forward: omc_init not called");
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_moe_forward: layer %d not initialised", layer);
    if (T < 0 || (T > 0 && (!x || !out))) return omc_fail(OMC_EINVAL, "omc_moe_forward: bad T or pointers");
    if (T == 0 && G.ep_world <= 1) return OMC_OK;
    int rc;
    if ((rc = omc_ws_ensure(L, T > 0 ? T : 1, 1))) return rc;
    const size_t D = (size_t)L->desc.D, K = (size_t)L->desc.k;
    cudaStream_t s = G.stream;
    if (T > 0) CK(cudaMemcpyAsync(G.ws.x, x, (size_t)T * D * 4, cudaMemcpyHostToDevice, s));
    if ((rc = omc_tier_before(L, s)) ||
        (rc = (T > 0 && graphs_enabled()) ? forward_replayed(L, layer, T, G.ws.x, G.ws.out, G.ws.topk_idx, G.ws.topk_w, s)
                                          : omc_forward_device(L, G.ws.x, T, G.ws.out, G.ws.topk_idx, G.ws.topk_w, s)) ||
        (rc = omc_tier_after(L, s))) {
        cudaStreamSynchronize(s);
        return rc;
    }
    if (G.ep_world > 1 && (rc = omc_ep_wait())) return rc;   /* bounded: a peer may have left */
    for (int pass = 0;; ++pass) {
        if (T > 0) {
            CK(cudaMemcpyAsync(out, G.ws.out, (size_t)T * D * 4, cudaMemcpyDeviceToHost, s));
            if (topk_idx) CK(cudaMemcpyAsync(topk_idx, G.ws.topk_idx, (size_t)T * K * 4, cudaMemcpyDeviceToHost, s));
            if (topk_w) CK(cudaMemcpyAsync(topk_w, G.ws.topk_w, (size_t)T * K * 4, cudaMemcpyDeviceToHost, s));
        }
        CK(cudaStreamSynchronize(s));
        rc = omc_check_device_error();
        /* (an expert-parallel forward is not redone: the other ranks would not
         * take part in the repeated exchange) */
        if (rc != OMC_ERANGE || pass > 0 || T == 0 || G.ep_world > 1) return rc;
        /* an activation outside the tensor-core path's f16 operand range:
         * the same forward again on the CUDA-core path, f32 throughout (the
         * routing is recomputed bit for bit, so only the expert path changes) */
        g_force_f32 = 1;
        rc = omc_forward_device(L, G.ws.x, T, G.ws.out, G.ws.topk_idx, G.ws.topk_w, s);
        g_force_f32 = 0;
        if (rc) {
            cudaStreamSynchronize(s);
            return rc;
        }
    }
}

/* ------------------------------------------------------ pipelined forward -- */
/* omc_moe_forward split into three stream stages so that consecutive calls
 * overlap: the upload of call i+1's x (copy stream), the forward of call i
 * (the library stream, replayed from a CUDA graph per staging slot) and the
 * download of call i-1's results (a second copy stream).  OMC_NASYNC staging
 * slots of device x/out/top-k rotate; events order each slot's reuse. */
#define OMC_NASYNC 3
typedef struct {
    int ready;
    cudaStream_t up, down;
    cudaEvent_t ev_up[OMC_NASYNC], ev_fwd[OMC_NASYNC], ev_down[OMC_NASYNC];
    float *x[OMC_NASYNC], *out[OMC_NASYNC], *w[OMC_NASYNC];
    int32_t *idx[OMC_NASYNC];
    size_t cap_rows[OMC_NASYNC], cap_k[OMC_NASYNC];   /* bytes of x/out, of idx/w */
    long long submitted, waited;                      /* tickets [waited, submitted) are in flight */
} omc_async_state;
static omc_async_state g_as;

static void async_release(void) {
    if (!g_as.ready) return;
    for (int i = 0; i < OMC_NASYNC; ++i) {
        cudaFree(g_as.x[i]);
        cudaFree(g_as.out[i]);
        cudaFree(g_as.idx[i]);
        cudaFree(g_as.w[i]);
        cudaEventDestroy(g_as.ev_up[i]);
        cudaEventDestroy(g_as.ev_fwd[i]);
        cudaEventDestroy(g_as.ev_down[i]);
    }
    cudaStreamDestroy(g_as.up);
    cudaStreamDestroy(g_as.down);
    memset(&g_as, 0, sizeof(g_as));
}

int omc_moe_wait(long long ticket) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_moe_wait: omc_init not called");
    if (!g_as.ready || ticket < g_as.waited) return OMC_OK;
    if (ticket >= g_as.submitted) return omc_fail(OMC_EINVAL, "omc_moe_wait: ticket %lld was not submitted", ticket);
    int rc = OMC_OK;
    for (; g_as.waited <= ticket; ++g_as.waited) {
        const cudaError_t e = cudaEventSynchronize(g_as.ev_down[g_as.waited % OMC_NASYNC]);
        if (e != cudaSuccess && !rc) rc = omc_fail(OMC_ECUDA, "omc_moe_wait: %s", cudaGetErrorString(e));
    }
    if (rc) return rc;
    return omc_check_device_error();
}

int omc_moe_forward_async(int layer, const float *x, int T, float *out, int32_t *topk_idx, float *topk_w,
                          long long *ticket) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_moe_forward_async: omc_init not called");
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_moe_forward_async: layer %d not initialised", layer);
    if (T < 1 || !x || !out || !ticket) return omc_fail(OMC_EINVAL, "omc_moe_forward_async: bad T or pointers");
    if (G.ep_world > 1)
        return omc_fail(OMC_EUNSUPPORTED, "omc_moe_forward_async: expert-parallel layers use omc_moe_forward");
    int rc;
    if (!g_as.ready) {
        CK(cudaStreamCreateWithFlags(&g_as.up, cudaStreamNonBlocking));
        CK(cudaStreamCreateWithFlags(&g_as.down, cudaStreamNonBlocking));
        for (int i = 0; i < OMC_NASYNC; ++i) {
            CK(cudaEventCreateWithFlags(&g_as.ev_up[i], cudaEventDisableTiming));
            CK(cudaEventCreateWithFlags(&g_as.ev_fwd[i], cudaEventDisableTiming));
            CK(cudaEventCreateWithFlags(&g_as.ev_down[i], cudaEventDisableTiming));
        }
        g_as.ready = 1;
    }
    /* a slot is reused after its previous call was waited for */
    if (g_as.submitted - g_as.waited >= OMC_NASYNC && (rc = omc_moe_wait(g_as.submitted - OMC_NASYNC))) return rc;
    const int slot = (int)(g_as.submitted % OMC_NASYNC);
    const size_t D = (size_t)L->desc.D, K = (size_t)L->desc.k;
    const size_t nrow = (size_t)T * D * 4, nk = (size_t)T * K * 4;
    if (g_as.cap_rows[slot] < nrow || g_as.cap_k[slot] < nk) {
        CK(cudaDeviceSynchronize());
        graphs_invalidate();
        cudaFree(g_as.x[slot]);
        cudaFree(g_as.out[slot]);
        cudaFree(g_as.idx[slot]);
        cudaFree(g_as.w[slot]);
        g_as.x[slot] = g_as.out[slot] = g_as.w[slot] = NULL;
        g_as.idx[slot] = NULL;
        g_as.cap_rows[slot] = g_as.cap_k[slot] = 0;
        CK(cudaMalloc((void **)&g_as.x[slot], nrow));
        CK(cudaMalloc((void **)&g_as.out[slot], nrow));
        CK(cudaMalloc((void **)&g_as.idx[slot], nk));
        CK(cudaMalloc((void **)&g_as.w[slot], nk));
        g_as.cap_rows[slot] = nrow;
        g_as.cap_k[slot] = nk;
    }
    if ((rc = omc_ws_ensure(L, T, 0))) return rc;
    cudaStream_t s = G.stream;
    /* upload: after the slot's previous forward has read its x */
    CK(cudaStreamWaitEvent(g_as.up, g_as.ev_fwd[slot], 0));
    CK(cudaMemcpyAsync(g_as.x[slot], x, nrow, cudaMemcpyHostToDevice, g_as.up));
    CK(cudaEventRecord(g_as.ev_up[slot], g_as.up));
    /* forward: after the upload, and after the slot's previous download has read out */
    CK(cudaStreamWaitEvent(s, g_as.ev_up[slot], 0));
    CK(cudaStreamWaitEvent(s, g_as.ev_down[slot], 0));
    if ((rc = omc_tier_before(L, s)) ||
        (rc = graphs_enabled() ? forward_replayed(L, layer, T, g_as.x[slot], g_as.out[slot], g_as.idx[slot], g_as.w[slot], s)
                               : omc_forward_device(L, g_as.x[slot], T, g_as.out[slot], g_as.idx[slot], g_as.w[slot], s)) ||
        (rc = omc_tier_after(L, s)))
        return rc;
    CK(cudaEventRecord(g_as.ev_fwd[slot], s));
    /* download */
    CK(cudaStreamWaitEvent(g_as.down, g_as.ev_fwd[slot], 0));
    CK(cudaMemcpyAsync(out, g_as.out[slot], nrow, cudaMemcpyDeviceToHost, g_as.down));
    if (topk_idx) CK(cudaMemcpyAsync(topk_idx, g_as.idx[slot], nk, cudaMemcpyDeviceToHost, g_as.down));
    if (topk_w) CK(cudaMemcpyAsync(topk_w, g_as.w[slot], nk, cudaMemcpyDeviceToHost, g_as.down));
    CK(cudaEventRecord(g_as.ev_down[slot], g_as.down));
    *ticket = g_as.submitted++;
    return OMC_OK;
}

/* ---------------------------------------------------------------- debug -- */
/* Runs a kernel whose bounded wait can never complete and returns the status
 * the library reports for it (OMC_ETIMEOUT expected), leaving the context
 * usable.  Used by the failure-detection test. */
int omc_debug_wait_timeout(void) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_debug_wait_timeout: omc_init not called");
    int rc = omc_launch_test_wait(G.d_err, G.stream);
    if (rc) return rc;
    CK(cudaStreamSynchronize(G.stream));
    return omc_check_device_error();
}

/* Forces the expert path (0 auto, 1 CUDA-core GEMV, 2 tensor-core grouped
 * GEMM, 3 fused decode); tests use it to run every path on the same inputs. */
int omc_debug_set_path(int path) {
    if (path < 0 || path > 3) return omc_fail(OMC_EINVAL, "omc_debug_set_path: %d", path);
    G.path_override = path;
    graphs_invalidate();
    return OMC_OK;
}

/* Device expf on n host inputs (test hook for the glibc-equality check). */
int omc_debug_expf(const float *x, float *y, long long n) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_debug_expf: omc_init not called");
    if (n <= 0) return OMC_OK;
    float *d = NULL;
    CK(cudaMalloc((void **)&d, (size_t)n * 8));
    CK(cudaMemcpyAsync(d, x, (size_t)n * 4, cudaMemcpyHostToDevice, G.stream));
    int rc = omc_launch_expf_probe(d, d + n, n, G.stream);
    if (!rc) rc = cudaStreamSynchronize(G.stream) == cudaSuccess ? OMC_OK : OMC_ECUDA;
    if (!rc) rc = cudaMemcpy(y, d + n, (size_t)n * 4, cudaMemcpyDeviceToHost) == cudaSuccess ? OMC_OK : OMC_ECUDA;
    cudaFree(d);
    return rc ? omc_fail(rc, "omc_debug_expf failed") : OMC_OK;
}

/* Copies a workspace buffer of the last forward to host memory (debugging):
 * 0 xp, 1 hp, 2 ypart, 3 rowinfo, 4 counts/offsets/done/nwork, 5 logits. */
int omc_debug_ws_copy(int which, void *dst, size_t bytes) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_debug_ws_copy: omc_init not called");
    const void *src = NULL;
    switch (which) {
    case 0: src = G.ws.xh; break;
    case 1: src = G.ws.hp; break;
    case 2: src = G.ws.ypart; break;
    case 3: src = G.ws.rowinfo; break;
    case 4: src = G.ws.counts; break;
    case 5: src = G.ws.logits; break;
    default: return omc_fail(OMC_EINVAL, "omc_debug_ws_copy: buffer %d", which);
    }
    if (!src || bytes > G.ws_bytes[which == 0 ? 9 : which == 1 ? 10 : which == 2 ? 11 : which == 3 ? 7 : which == 4 ? 6 : 2])
        return omc_fail(OMC_EINVAL, "omc_debug_ws_copy: %zu bytes too many", bytes);
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    return OMC_OK;
}

/* GEMMA test hook: the prenorm kernel's outputs for host rows x [T][D]:
 * router input xr, expert input xe [T][D] and the norm factor r [T]. */
int omc_debug_gemma_prenorm(int layer, const float *x, int T, float *xr, float *xe, float *r) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_debug_gemma_prenorm: omc_init not called");
    omc_layer *L = omc_get_layer(layer);
    if (!L || L->desc.family != OMC_FAMILY_GEMMA || !L->gemma_ready)
        return omc_fail(OMC_EINVAL, "omc_debug_gemma_prenorm: layer %d is not a ready GEMMA layer", layer);
    if (T <= 0 || !x || !xr || !xe || !r) return omc_fail(OMC_EINVAL, "omc_debug_gemma_prenorm: bad arguments");
    int rc;
    if ((rc = omc_ws_ensure(L, T, 1))) return rc;
    const size_t n = (size_t)T * L->desc.D * sizeof(float);
    cudaStream_t s = G.stream;
    CK(cudaMemcpyAsync(G.ws.x, x, n, cudaMemcpyHostToDevice, s));
    if ((rc = omc_launch_gemma_prenorm(&L->dev, G.ws.x, T, G.ws.xg_r, G.ws.xg_e, NULL, G.ws.sg, G.d_err, s)))
        return omc_fail(rc, "omc_debug_gemma_prenorm: launch failed");
    CK(cudaMemcpyAsync(xr, G.ws.xg_r, n, cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(xe, G.ws.xg_e, n, cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(r, G.ws.sg, (size_t)T * sizeof(float), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return omc_check_device_error();
}
