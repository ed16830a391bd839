/* omc_tier.c -- tiered expert store: HBM slots for the hot experts, every
 * expert's home copy in mapped pinned host memory, LFRU replacement.
 *
 * The reference keeps experts on disk behind a RAM LRU (expert_get,
 * engines/olmoe.c:250-272) and ships, uncalled, a replacement policy for a
 * smaller hot store above it (include/tier.h:30-58: LFRU score = heat << 8 |
 * recency, the coldest slot swapped for the hottest outsider only past a
 * 25% + 4 margin, heat halved by tier_decay).  On a GPU whose HBM budget
 * does not hold a layer's experts, this file applies that policy:
 *
 *   - home: E expert images in mapped pinned host memory, written once at
 *     upload;
 *   - slots: hbm_slots expert images in HBM, holding the hot experts;
 *   - miss area: HBM images for the routed experts that are not in a slot,
 *     filled from their homes after routing (tier.cu) and shared by every
 *     tiered layer (their forwards run one after another on a stream);
 *   - table: the device pointer table (omc_layer_dev.experts) points a
 *     resident expert at its slot and a routed non-resident one at its miss
 *     image (written on the device by the routing step); entries of experts
 *     that nothing routes point at an HBM placeholder.  Every pointer a
 *     kernel can see is HBM, so the expert kernels are unchanged, and since
 *     they read the table at run time, CUDA graphs of the forward stay valid
 *     across swaps;
 *   - heat: counted per expert on the device by the same routing step
 *     (heat, last, clock);
 *   - decisions: every `interval` forwards the counters are copied to pinned
 *     memory behind an event; the first forward entry that finds the event
 *     complete picks at most one swap (omc_tier_pick, the tier.h rule) and
 *     enqueues it on the forward's stream ahead of its kernels: the evicted
 *     expert's entry -> the placeholder, its slot <- the new expert's home
 *     image (one host-to-device copy), the new expert's entry -> the slot.
 *     Stream order makes every forward see a consistent table; nothing waits
 *     on the host.
 *
 * One image holds [gate/up tiles | down tiles | gs | us | ds], each part
 * 256-byte aligned, so a swap or a miss is one copy. */
#include <stdlib.h>
#include <string.h>

#include "omc_host.h"

#define CK(call)                                                                                       \
    do {                                                                                               \
        cudaError_t e_ = (call);                                                                       \
        if (e_ != cudaSuccess)                                                                         \
            return omc_fail(e_ == cudaErrorMemoryAllocation ? OMC_ENOMEM : OMC_ECUDA, "%s: %s (%s:%d)", \
                            #call, cudaGetErrorString(e_), __FILE__, __LINE__);                        \
    } while (0)

typedef struct omc_tier {
    int nslots, interval, decay_every;
    size_t off_d, off_gs, off_us, off_ds, bytes;   /* image layout */
    char *home;                  /* [E] images, mapped pinned host        */
    char *slots;                 /* [nslots] images, HBM                  */
    char *spare;                 /* one HBM image: upload scratch and the
                                    placeholder of unrouted entries      */
    int *d_list;                 /* [1 + E] miss list (device)            */
    unsigned long long *d_total; /* misses over all forwards (device)     */
    int *pinned;                 /* [nslots] expert in each slot, -1 free */
    int *slot_of;                /* [E] slot of each expert, -1 = home    */
    uint32_t *d_stats;           /* [2E+1] heat, last, clock (device)     */
    uint32_t *snap;              /* [2E+1] pinned copy for decisions      */
    cudaEvent_t ev;
    int pending;                 /* a snapshot copy is in flight          */
    long long calls, swaps;
} omc_tier;

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

/* The miss area, shared by all tiered layers: the largest (E - hbm_slots)
 * images of any of them. */
static char *g_miss;
static size_t g_miss_bytes;

static int miss_ensure(size_t n) {
    if (n <= g_miss_bytes) return OMC_OK;
    CK(cudaDeviceSynchronize());
    cudaFree(g_miss);
    g_miss = NULL;
    g_miss_bytes = 0;
    omc_graphs_invalidate();
    CK(cudaMalloc((void **)&g_miss, n));
    g_miss_bytes = n;
    return OMC_OK;
}

void omc_tier_release(void) {
    cudaFree(g_miss);
    g_miss = NULL;
    g_miss_bytes = 0;
}

/* include/tier.h:30-33: frequency in the high bits, then up to 255 points
 * of recency, so a recent expert never outranks one with more routings. */
static uint64_t tier_score(uint32_t heat, uint32_t last, uint32_t clock) {
    const uint32_t age = clock - last;
    return ((uint64_t)heat << 8) | (age < 255u ? 255u - age : 0u);
}

int omc_tier_pick(const uint32_t *heat, const uint32_t *last, uint32_t clock, int nexpert, const int *pinned, int npin,
                  int *slot, int *eid, long *gain) {
    if (!heat || !last || !pinned || !slot || !eid || !gain || npin < 1 || nexpert < 1) return 0;
    /* coldest resident slot: lowest score, first slot on ties (tier.h:40-43) */
    int cold = 0;
    uint64_t cs = tier_score(heat[pinned[0]], last[pinned[0]], clock);
    for (int z = 1; z < npin; ++z) {
        const uint64_t v = tier_score(heat[pinned[z]], last[pinned[z]], clock);
        if (v < cs) cs = v, cold = z;
    }
    /* hottest expert outside the slots: highest score, lowest id on ties,
     * the first outsider taken even at score 0 (tier.h:44-49) */
    int hot = -1;
    uint64_t hs = 0;
    for (int e = 0; e < nexpert; ++e) {
        int resident = 0;
        for (int z = 0; z < npin && !resident; ++z) resident = pinned[z] == e;
        if (resident) continue;
        const uint64_t v = tier_score(heat[e], last[e], clock);
        if (hot < 0 || v > hs) hs = v, hot = e;
    }
    /* swap only past a quarter of the cold score plus 4 routings (tier.h:51-52) */
    if (hot < 0 || hs <= cs + (cs >> 2) + (4u << 8)) return 0;
    *slot = cold;
    *eid = hot;
    *gain = (long)((hs - cs) >> 8);
    return 1;
}

static omc_tier *tier_of(const omc_layer *L) { return (omc_tier *)L->tier; }

static omc_expert_ptrs image_ptrs(const omc_tier *t, char *base) {
    omc_expert_ptrs p;
    p.g = (const int8_t *)base;
    p.u = (const int8_t *)base + OMC_BLK_BYTES;
    p.d = (const int8_t *)(base + t->off_d);
    p.gs = (const float *)(base + t->off_gs);
    p.us = (const float *)(base + t->off_us);
    p.ds = (const float *)(base + t->off_ds);
    return p;
}

static char *home_of(const omc_tier *t, int e) { return t->home + (size_t)e * t->bytes; }
static char *slot_img(const omc_tier *t, int z) { return t->slots + (size_t)z * t->bytes; }

void omc_tier_free(omc_layer *L) {
    omc_tier *t = tier_of(L);
    if (!t) return;
    if (t->ev) cudaEventDestroy(t->ev);
    cudaFreeHost(t->home);
    cudaFreeHost(t->snap);
    cudaFree(t->slots);
    cudaFree(t->spare);
    cudaFree(t->d_stats);
    cudaFree(t->d_list);
    cudaFree(t->d_total);
    free(t->pinned);
    free(t->slot_of);
    free(t);
    L->tier = NULL;
}

int omc_tier_enable(int layer, int hbm_slots, int interval, int decay_every) {
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_tier_enable: layer %d not initialised", layer);
    const omc_layer_dev *P = &L->dev;
    const int E = P->E;
    if (omc_G.ep_world > 1) return omc_fail(OMC_EUNSUPPORTED, "omc_tier_enable: not with expert parallelism");
    if (hbm_slots < 1 || hbm_slots > E || interval < 0 || decay_every < 0)
        return omc_fail(OMC_EINVAL, "omc_tier_enable: hbm_slots %d (1..%d), interval %d, decay_every %d", hbm_slots, E,
                        interval, decay_every);
    if (L->tier) return omc_fail(OMC_EINVAL, "omc_tier_enable: layer %d is tiered already", layer);
    for (int e = 0; e < E; ++e)
        if (L->have[e]) return omc_fail(OMC_EINVAL, "omc_tier_enable: call it before the layer's experts are uploaded");
    omc_graphs_invalidate();
    omc_tier *t = calloc(1, sizeof(*t));
    if (!t) return omc_fail(OMC_ENOMEM, "omc_tier_enable: host alloc");
    L->tier = t;
    t->nslots = hbm_slots;
    t->interval = interval;
    t->decay_every = decay_every;
    const size_t gu = (size_t)2 * P->I_rows * P->D_pad;
    const size_t dd = (size_t)omc_round_up(P->D_rows, 2 * OMC_TM) * P->I_pad;
    t->off_d = al256(gu);
    t->off_gs = al256(t->off_d + dd);
    t->off_us = al256(t->off_gs + (size_t)P->I_rows * 4);
    t->off_ds = al256(t->off_us + (size_t)P->I_rows * 4);
    t->bytes = al256(t->off_ds + (size_t)P->D_rows * 4);
    t->pinned = malloc(sizeof(int) * (size_t)hbm_slots);
    t->slot_of = malloc(sizeof(int) * (size_t)E);
    if (!t->pinned || !t->slot_of) {
        omc_tier_free(L);
        return omc_fail(OMC_ENOMEM, "omc_tier_enable: host alloc");
    }
    for (int z = 0; z < hbm_slots; ++z) t->pinned[z] = -1;
    for (int e = 0; e < E; ++e) t->slot_of[e] = -1;
    cudaError_t ce = cudaHostAlloc((void **)&t->home, t->bytes * (size_t)E, cudaHostAllocMapped | cudaHostAllocPortable);
    if (ce == cudaSuccess)
        ce = cudaHostAlloc((void **)&t->snap, sizeof(uint32_t) * (2 * (size_t)E + 1), cudaHostAllocDefault);
    if (ce == cudaSuccess) ce = cudaMalloc((void **)&t->slots, t->bytes * (size_t)hbm_slots);
    if (ce == cudaSuccess) ce = cudaMalloc((void **)&t->spare, t->bytes);
    if (ce == cudaSuccess) ce = cudaMalloc((void **)&t->d_stats, sizeof(uint32_t) * (2 * (size_t)E + 1));
    if (ce == cudaSuccess) ce = cudaMalloc((void **)&t->d_list, sizeof(int) * ((size_t)E + 1));
    if (ce == cudaSuccess) ce = cudaMemsetAsync(t->d_list, 0, sizeof(int) * ((size_t)E + 1), omc_G.stream);
    if (ce == cudaSuccess) ce = cudaMalloc((void **)&t->d_total, sizeof(unsigned long long));
    if (ce == cudaSuccess) ce = cudaMemsetAsync(t->d_total, 0, sizeof(unsigned long long), omc_G.stream);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&t->ev, cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(t->d_stats, 0, sizeof(uint32_t) * (2 * (size_t)E + 1), omc_G.stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(omc_G.stream);   /* ordered with, and done before, any forward */
    if (ce != cudaSuccess) {
        cudaGetLastError();
        omc_tier_free(L);
        return omc_fail(ce == cudaErrorMemoryAllocation ? OMC_ENOMEM : OMC_ECUDA, "omc_tier_enable: %s",
                        cudaGetErrorString(ce));
    }
    int rc = miss_ensure(t->bytes * (size_t)(E - hbm_slots));
    if (rc) omc_tier_free(L);
    return rc;
}

/* Expert e of a tiered layer: tiled in HBM (its slot, or the spare image),
 * copied to its home; the first hbm_slots experts uploaded take the slots. */
int omc_tier_upload(omc_layer *L, int e, const int8_t *g, const float *gs, const int8_t *u, const float *us,
                    const int8_t *d, const float *ds) {
    omc_tier *t = tier_of(L);
    const omc_layer_dev *P = &L->dev;
    int z = t->slot_of[e];
    if (z < 0)
        for (int i = 0; i < t->nslots; ++i)
            if (t->pinned[i] < 0) {
                z = i;
                break;
            }
    char *img = z >= 0 ? slot_img(t, z) : t->spare;
    omc_expert_ptrs ep = image_ptrs(t, img);
    int rc = omc_expert_upload(P->D, P->D_pad, P->D_rows, P->I, P->I_pad, P->I_rows, g, gs, u, us, d, ds, &ep, 1);
    if (rc) return rc;
    CK(cudaStreamSynchronize(omc_G.stream));
    CK(cudaMemcpy(home_of(t, e), img, t->bytes, cudaMemcpyDeviceToHost));
    if (z >= 0) {
        t->pinned[z] = e;
        t->slot_of[e] = z;
    }   /* else ep names the placeholder image until a forward routes e */
    L->h_experts[e] = ep;
    L->have[e] = 1;
    CK(cudaMemcpyAsync(L->d_experts_tab + e, &ep, sizeof(ep), cudaMemcpyHostToDevice, omc_G.stream));
    return OMC_OK;
}

/* Enqueue one swap on stream s: slot z's expert leaves HBM, expert h moves
 * into slot z.  The table entries are written from host values the runtime
 * stages at the call (pageable source), each in stream order. */
static int apply_swap(omc_layer *L, int z, int h, cudaStream_t s) {
    omc_tier *t = tier_of(L);
    const int c = t->pinned[z];
    omc_expert_ptrs out = image_ptrs(t, t->spare), in = image_ptrs(t, slot_img(t, z));
    CK(cudaMemcpyAsync(L->d_experts_tab + c, &out, sizeof(out), cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(slot_img(t, z), home_of(t, h), t->bytes, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(L->d_experts_tab + h, &in, sizeof(in), cudaMemcpyHostToDevice, s));
    L->h_experts[c] = out;
    L->h_experts[h] = in;
    t->slot_of[c] = -1;
    t->slot_of[h] = z;
    t->pinned[z] = h;
    t->swaps++;
    return OMC_OK;
}

static int decide(omc_layer *L, const uint32_t *stats, cudaStream_t s, int *eid) {
    omc_tier *t = tier_of(L);
    const int E = L->dev.E;
    int z, h;
    long gain;
    *eid = -1;
    for (int i = 0; i < t->nslots; ++i)
        if (t->pinned[i] < 0) return OMC_OK;   /* slots not all filled yet */
    if (!omc_tier_pick(stats, stats + E, stats[2 * E], E, t->pinned, t->nslots, &z, &h, &gain)) return OMC_OK;
    *eid = h;
    return apply_swap(L, z, h, s);
}

/* A stream being captured into a caller's CUDA graph gets no decisions and
 * no snapshots: they would be frozen into every replay. */
static int capturing(cudaStream_t s) {
    enum cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return cs != cudaStreamCaptureStatusNone;
}

/* Forward entry: apply the decision of a completed snapshot. */
int omc_tier_before(omc_layer *L, cudaStream_t s) {
    omc_tier *t = tier_of(L);
    if (!t || !t->pending || capturing(s)) return OMC_OK;
    const cudaError_t q = cudaEventQuery(t->ev);
    if (q == cudaErrorNotReady) return OMC_OK;
    t->pending = 0;
    if (q != cudaSuccess) return omc_fail(OMC_ECUDA, "tier snapshot: %s", cudaGetErrorString(q));
    int eid;
    return decide(L, t->snap, s, &eid);
}

/* Between routing and the expert kernels of a forward (so CUDA graphs of
 * the forward hold it): counters, miss list, miss images. */
int omc_tier_route(omc_layer *L, const int32_t *idx, int T, cudaStream_t s) {
    omc_tier *t = tier_of(L);
    if (!t || T <= 0) return OMC_OK;
    const int E = L->dev.E;
    const size_t layout[5] = {t->bytes, t->off_d, t->off_gs, t->off_us, t->off_ds};
    return omc_launch_tier_route(idx, T * L->dev.k, E, t->d_stats, t->decay_every, L->d_experts_tab, t->slots,
                                 t->slots + (size_t)t->nslots * t->bytes, t->home, g_miss, E - t->nslots, layout,
                                 t->d_list, t->d_total, omc_G.d_err, 4 * omc_G.num_sms, s);
}

/* Forward exit: every interval-th forward, snapshot the counters. */
int omc_tier_after(omc_layer *L, cudaStream_t s) {
    omc_tier *t = tier_of(L);
    if (!t || capturing(s)) return OMC_OK;
    t->calls++;
    if (!t->interval || t->pending || t->calls % t->interval) return OMC_OK;
    CK(cudaMemcpyAsync(t->snap, t->d_stats, sizeof(uint32_t) * (2 * (size_t)L->dev.E + 1), cudaMemcpyDeviceToHost, s));
    CK(cudaEventRecord(t->ev, s));
    t->pending = 1;
    return OMC_OK;
}

int omc_tier_step(int layer, int *eid) {
    omc_layer *L = omc_get_layer(layer);
    if (!L || !tier_of(L)) return omc_fail(OMC_ENOINIT, "omc_tier_step: layer %d is not tiered", layer);
    omc_tier *t = tier_of(L);
    int h = -1;
    CK(cudaDeviceSynchronize());
    t->pending = 0;
    CK(cudaMemcpy(t->snap, t->d_stats, sizeof(uint32_t) * (2 * (size_t)L->dev.E + 1), cudaMemcpyDeviceToHost));
    int rc = decide(L, t->snap, omc_G.stream, &h);
    if (rc) return rc;
    CK(cudaStreamSynchronize(omc_G.stream));
    if (eid) *eid = h;
    return OMC_OK;
}

int omc_tier_stats(int layer, uint32_t *heat, uint32_t *last, uint32_t *clock, int32_t *slot_expert,
                   long long *swaps, long long *misses) {
    omc_layer *L = omc_get_layer(layer);
    if (!L || !tier_of(L)) return omc_fail(OMC_ENOINIT, "omc_tier_stats: layer %d is not tiered", layer);
    omc_tier *t = tier_of(L);
    const size_t E = (size_t)L->dev.E;
    CK(cudaDeviceSynchronize());
    if (heat) CK(cudaMemcpy(heat, t->d_stats, E * 4, cudaMemcpyDeviceToHost));
    if (last) CK(cudaMemcpy(last, t->d_stats + E, E * 4, cudaMemcpyDeviceToHost));
    if (clock) CK(cudaMemcpy(clock, t->d_stats + 2 * E, 4, cudaMemcpyDeviceToHost));
    if (slot_expert)
        for (int z = 0; z < t->nslots; ++z) slot_expert[z] = t->pinned[z];
    if (swaps) *swaps = t->swaps;
    if (misses) {
        unsigned long long m = 0;
        CK(cudaMemcpy(&m, t->d_total, sizeof(m), cudaMemcpyDeviceToHost));
        *misses = (long long)m;
    }
    return OMC_OK;
}
