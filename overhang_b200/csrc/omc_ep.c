/* omc_ep.c -- expert parallelism: one process per GPU, experts split into
 * contiguous ranges, tokens exchanged over NCCL.
 *
 * A layer's routed experts are independent of one another, so rank r of P
 * holds experts [r*E/P, (r+1)*E/P) in its slab (plus the shared expert) and
 * every rank routes its own ("home") tokens.  One forward (omc_ep_forward):
 *
 *   1. route the home tokens (the single-GPU router: bit-exact top-k)
 *   2. ep_layout_kernel: rows and slots per destination rank, send and
 *      return positions (index arithmetic in omc_ep_plan.h)
 *   3. NCCL: each rank's (rows, slots) counts to every peer; the host reads
 *      them (the one host wait of a forward, bounded: see wait_bounded)
 *   4. ep_pack_kernel: one f16 row per (token, destination rank), deduplicated,
 *      plus its meta row; NCCL grouped send/recv of rows and meta
 *   5. ep_unpack_kernel + the grouped GEMMs (omc_launch_mma_slots): every
 *      received slot's w * expert(x), and the home tokens' shared expert
 *   6. NCCL grouped send/recv of the f32 partials back to their home ranks
 *   7. ep_combine_kernel: the reference's combine order at home
 *
 * The reference has no distributed code; the block it replaces is
 * engines/olmoe.c:344-402 / engines/qwen.c:453-495 on one CPU, and the result
 * equals one GPU's tensor-core forward bit for bit.
 *
 * NCCL is loaded at run time (dlopen of libnccl.so.2: the copy a host
 * framework already loaded, or the system's), so the library links without
 * it and reports OMC_ENCCL when it is missing.  Joining is explicit: rank 0
 * calls omc_ep_unique_id, the caller passes the 128 bytes to every rank by
 * its own means, and each calls omc_ep_init(rank, world, id).  Without an id
 * (NULL) a rank only holds its experts and the caller composes the exchange
 * from omc_moe_route_dev / omc_moe_experts_dev.
 *
 * Failure detection.  Every host wait of an EP forward polls the CUDA event
 * and ncclCommGetAsyncError until a deadline (omc_ep_set_timeout, default
 * 30 s); past it, or on an NCCL error, the communicator is aborted
 * (ncclCommAbort ends its kernels) and the call returns OMC_ETIMEOUT or
 * OMC_ENCCL.  Later EP forwards return OMC_ENCCL until omc_ep_init joins a
 * new group.  No wait on a peer happens inside this library's own kernels.
 */
#include <dlfcn.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <nccl.h>   /* types and constants only: the functions are looked up at run time */

#include "om_cuda.h"
#include "omc_ep_plan.h"
#include "omc_host.h"

#define G omc_G

/* ---------------------------------------------------------------- NCCL -- */
typedef struct {
    void *h;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*GroupStart)(void);
    ncclResult_t (*GroupEnd)(void);
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    const char *(*GetErrorString)(ncclResult_t);
} nccl_api;

static nccl_api N;

static int nccl_load(void) {
    if (N.h) return OMC_OK;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return omc_fail(OMC_ENCCL, "NCCL not found (dlopen libnccl.so.2: %s)", dlerror());
#define SYM(f, name)                                                                      \
    do {                                                                                  \
        *(void **)&N.f = dlsym(h, name);                                                  \
        if (!N.f) return omc_fail(OMC_ENCCL, "NCCL library lacks %s", name);              \
    } while (0)
    SYM(GetUniqueId, "ncclGetUniqueId");
    SYM(CommInitRank, "ncclCommInitRank");
    SYM(CommDestroy, "ncclCommDestroy");
    SYM(CommAbort, "ncclCommAbort");
    SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    SYM(GroupStart, "ncclGroupStart");
    SYM(GroupEnd, "ncclGroupEnd");
    SYM(Send, "ncclSend");
    SYM(Recv, "ncclRecv");
    SYM(GetErrorString, "ncclGetErrorString");
#undef SYM
    N.h = h;
    return OMC_OK;
}

/* ---------------------------------------------------------------- state -- */
typedef struct {
    ncclComm_t comm;
    int have_comm, broken;
    int timeout_ms;
    int combine;                /* OMC_EP_EXACT or OMC_EP_RANKSUM */
    /* grow-only device buffers; sizes in bytes */
    void *buf[16];
    size_t cap[16];
    int *h_cnt;                 /* pinned: own counts [4P], received pairs [2P] */
    /* the expert pass's own workspace: growing it never touches the library's
     * (whose top-k buffers the blocking entry hands to this forward) */
    omc_ws xws;
    omc_ws_ptrs xW;
    size_t xbytes[16];
    cudaEvent_t ev;
    cudaStream_t last_stream;
} omc_ep_state;

enum { B_IDX, B_W, B_SG, B_XE, B_POS, B_SENDX, B_SENDM, B_OPND, B_RECVM, B_STOK, B_SE, B_SW, B_Y, B_RET, B_SMALL,
       B_RSUM };

static omc_ep_state *S(void) {
    if (!G.ep) {
        G.ep = calloc(1, sizeof(omc_ep_state));
        if (G.ep) ((omc_ep_state *)G.ep)->timeout_ms = 30000;
    }
    return (omc_ep_state *)G.ep;
}

static int ep_buf(omc_ep_state *st, int i, size_t need, void **out) {
    if (need == 0) need = 256;
    if (st->cap[i] < need) {
        cudaDeviceSynchronize();
        cudaFree(st->buf[i]);
        st->buf[i] = NULL;
        st->cap[i] = 0;
        const size_t n = need + need / 4;
        if (cudaMalloc(&st->buf[i], n) != cudaSuccess) {
            cudaGetLastError();
            return omc_fail(OMC_ENOMEM, "expert parallelism: cudaMalloc(%zu) failed", n);
        }
        st->cap[i] = n;
    }
    *out = st->buf[i];
    return OMC_OK;
}

static double now_s(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + t.tv_nsec * 1e-9;
}

/* Waits for event ev with the EP deadline, watching the communicator:
 * OMC_OK, or OMC_ETIMEOUT / OMC_ENCCL after aborting it. */
static int wait_bounded(omc_ep_state *st, cudaEvent_t ev, const char *what) {
    const double t0 = now_s();
    for (unsigned it = 0;; ++it) {
        const cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) return OMC_OK;
        if (q != cudaErrorNotReady)
            return omc_fail(OMC_ECUDA, "expert parallelism (%s): %s", what, cudaGetErrorString(q));
        ncclResult_t ae = ncclSuccess;
        if (st->have_comm && N.CommGetAsyncError(st->comm, &ae) == ncclSuccess && ae != ncclSuccess &&
            ae != ncclInProgress) {
            N.CommAbort(st->comm);
            st->have_comm = 0;
            st->broken = 1;
            return omc_fail(OMC_ENCCL, "expert parallelism (%s): NCCL reported %s; communicator aborted", what,
                            N.GetErrorString(ae));
        }
        if ((now_s() - t0) * 1e3 > st->timeout_ms) {
            if (st->have_comm) N.CommAbort(st->comm);
            st->have_comm = 0;
            st->broken = 1;
            return omc_fail(OMC_ETIMEOUT, "expert parallelism (%s): no progress within %d ms (a peer rank left?); "
                                          "communicator aborted", what, st->timeout_ms);
        }
        /* the counts arrive within microseconds when every peer is there:
         * spin for the first 2 ms (a sleep of any length costs tens of us on
         * the forward's critical path), then poll every 50 us */
        if (it > 64 && (now_s() - t0) > 2e-3) usleep(50);
    }
}

#define NCK(call)                                                                                      \
    do {                                                                                               \
        ncclResult_t r_ = (call);                                                                      \
        if (r_ != ncclSuccess) return omc_fail(OMC_ENCCL, "%s: %s", #call, N.GetErrorString(r_));      \
    } while (0)
#define CK(call)                                                                                       \
    do {                                                                                               \
        cudaError_t e_ = (call);                                                                       \
        if (e_ != cudaSuccess) return omc_fail(OMC_ECUDA, "%s: %s", #call, cudaGetErrorString(e_));    \
    } while (0)

/* ---------------------------------------------------------------- ABI -- */
int omc_ep_unique_id(void *buf, size_t len) {
    if (!buf || len < sizeof(ncclUniqueId))
        return omc_fail(OMC_EINVAL, "omc_ep_unique_id: needs a %zu-byte buffer", sizeof(ncclUniqueId));
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId id;
    NCK(N.GetUniqueId(&id));
    memcpy(buf, &id, sizeof(id));
    return OMC_OK;
}

int omc_ep_init(int rank, int world, const void *unique_id) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_ep_init: omc_init not called");
    if (world < 1 || rank < 0 || rank >= world) return omc_fail(OMC_EINVAL, "omc_ep_init: rank %d of %d", rank, world);
    if (world > OMC_EP_MAX_RANKS) return omc_fail(OMC_EINVAL, "omc_ep_init: at most %d ranks", OMC_EP_MAX_RANKS);
    for (int i = 0; i < G.nlayers; ++i)
        if (G.layers[i].used) return omc_fail(OMC_EINVAL, "omc_ep_init: call before the first omc_layer_init");
    omc_ep_state *st = S();
    if (!st) return omc_fail(OMC_ENOMEM, "omc_ep_init: host alloc");
    if (unique_id && world > 1) {
        int rc = nccl_load();
        if (rc) return rc;
        if (st->have_comm) {
            N.CommDestroy(st->comm);
            st->have_comm = 0;
        }
        ncclUniqueId id;
        memcpy(&id, unique_id, sizeof(id));
        CK(cudaSetDevice(G.device));
        NCK(N.CommInitRank(&st->comm, world, id, rank));
        st->have_comm = 1;
        st->broken = 0;
        if (!st->h_cnt) CK(cudaHostAlloc((void **)&st->h_cnt, sizeof(int) * 6 * OMC_EP_MAX_RANKS, cudaHostAllocDefault));
        if (!st->ev) CK(cudaEventCreateWithFlags(&st->ev, cudaEventDisableTiming));
    }
    G.ep_rank = rank;
    G.ep_world = world;
    return OMC_OK;
}

int omc_ep_set_timeout(int timeout_ms) {
    if (timeout_ms <= 0) return omc_fail(OMC_EINVAL, "omc_ep_set_timeout: %d ms", timeout_ms);
    omc_ep_state *st = S();
    if (!st) return omc_fail(OMC_ENOMEM, "omc_ep_set_timeout: host alloc");
    st->timeout_ms = timeout_ms;
    return OMC_OK;
}

int omc_ep_set_combine(int mode) {
    if (mode != OMC_EP_EXACT && mode != OMC_EP_RANKSUM) return omc_fail(OMC_EINVAL, "omc_ep_set_combine: mode %d", mode);
    omc_ep_state *st = S();
    if (!st) return omc_fail(OMC_ENOMEM, "omc_ep_set_combine: host alloc");
    st->combine = mode;
    return OMC_OK;
}

int omc_ep_wait(void) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_ep_wait: omc_init not called");
    omc_ep_state *st = S();
    if (!st || !st->ev || !st->last_stream) return OMC_OK;
    CK(cudaEventRecord(st->ev, st->last_stream));
    int rc = wait_bounded(st, st->ev, "wait");
    if (rc) return rc;
    return omc_check_device_error();
}

/* ---------------------------------------------------------------- forward -- */
int omc_ep_forward(omc_layer *L, const float *x, int T, float *out, int32_t *topk_idx, float *topk_w,
                   cudaStream_t s) {
    omc_ep_state *st = S();
    if (!st) return omc_fail(OMC_ENOMEM, "expert parallelism: host alloc");
    if (st->broken)
        return omc_fail(OMC_ENCCL, "expert parallelism: the communicator was aborted; call omc_ep_init again");
    if (!st->have_comm)
        return omc_fail(OMC_EUNSUPPORTED,
                        "this process holds experts [e0, e0+E/world) only and joined no NCCL group: pass a unique id "
                        "to omc_ep_init, or compose the forward from omc_moe_route_dev + exchange + "
                        "omc_moe_experts_dev");
    if (L->tier) return omc_fail(OMC_EUNSUPPORTED, "expert parallelism: not on a tiered layer");
    const omc_layer_dev *P_ = &L->dev;
    const int P = G.ep_world, me = G.ep_rank, k = P_->k, D = P_->D, E = P_->E, ne = L->ne;
    const int M = omc_ep_meta_ints(k), sh = P_->has_shared, gemma = P_->family == OMC_FAMILY_GEMMA;
    const int Tz = T > 0 ? T : 0;
    const int fan = P < k ? P : k;   /* destinations a token can have */
    int rc;
    st->last_stream = s;
    G.prof_valid = 0;
    /* 1. route the home tokens; what is read after the host wait lives in EP
     * buffers (the shared workspace may be regrown for the expert pass) */
    int32_t *idx = NULL;
    float *w = NULL, *sg = NULL, *xe = NULL;
    int32_t *small = NULL, *pos = NULL;
    if ((rc = ep_buf(st, B_IDX, (size_t)Tz * k * 4, (void **)&idx)) || (rc = ep_buf(st, B_W, (size_t)Tz * k * 4, (void **)&w)) ||
        (rc = ep_buf(st, B_SG, (size_t)Tz * 4, (void **)&sg)) ||
        (rc = ep_buf(st, B_POS, (size_t)Tz * (P + k) * 4, (void **)&pos)) ||
        (rc = ep_buf(st, B_SMALL, sizeof(int) * 8 * OMC_EP_MAX_RANKS, (void **)&small)))
        return rc;
    if (gemma && (rc = ep_buf(st, B_XE, (size_t)Tz * D * 4, (void **)&xe))) return rc;
    int32_t *tok_pos = pos, *slot_pos = pos + (size_t)Tz * P;
    int32_t *counts = small, *pairs_send = small + 4 * P, *pairs_recv = small + 6 * P;
    if (T > 0) {
        if ((rc = omc_ws_ensure(L, T, 0))) return rc;
        omc_ws wsr = G.ws;
        wsr.sg = sg;
        const float *xr = x, *xsrc = x;
        if (gemma) {
            if ((rc = omc_launch_gemma_prenorm(P_, x, T, G.ws.xg_r, xe, NULL, NULL, G.d_err, s)))
                return omc_fail(rc, "expert parallelism: prenorm launch failed");
            xr = G.ws.xg_r;
            xsrc = xe;
        }
        (void)xsrc;
        if ((rc = omc_launch_router(P_, xr, T, &wsr, idx, w, NULL, s))) return omc_fail(rc, "router launch failed");
    }
    /* 2. layout */
    if ((rc = omc_launch_ep_layout(idx, Tz, k, ne, P, tok_pos, slot_pos, counts, pairs_send, s)))
        return omc_fail(rc, "ep layout launch failed");
    /* 3. counts to every peer (NCCL sends to itself too), then to the host */
    NCK(N.GroupStart());
    for (int p = 0; p < P; ++p) {
        NCK(N.Send(pairs_send + 2 * p, 2, ncclInt32, p, st->comm, s));
        NCK(N.Recv(pairs_recv + 2 * p, 2, ncclInt32, p, st->comm, s));
    }
    NCK(N.GroupEnd());
    CK(cudaMemcpyAsync(st->h_cnt, counts, sizeof(int) * 4 * P, cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(st->h_cnt + 4 * P, pairs_recv, sizeof(int) * 2 * P, cudaMemcpyDeviceToHost, s));
    CK(cudaEventRecord(st->ev, s));
    if ((rc = wait_bounded(st, st->ev, "counts"))) return rc;
    const int *hc = st->h_cnt;
    int send_rows[OMC_EP_MAX_RANKS], send_slots[OMC_EP_MAX_RANKS], send_base[OMC_EP_MAX_RANKS],
        ret_base[OMC_EP_MAX_RANKS];
    int recv_base[OMC_EP_MAX_RANKS + 1], slot_base[OMC_EP_MAX_RANKS + 1];
    recv_base[0] = slot_base[0] = 0;
    for (int p = 0; p < P; ++p) {
        send_rows[p] = hc[p];
        send_slots[p] = hc[P + p];
        send_base[p] = hc[2 * P + p];
        ret_base[p] = hc[3 * P + p];
        recv_base[p + 1] = recv_base[p] + hc[4 * P + 2 * p];
        slot_base[p + 1] = slot_base[p] + hc[4 * P + 2 * p + 1];
    }
    const int Rr = recv_base[P], Sr = slot_base[P];
    const int Ntot = Sr + (sh ? Tz : 0);
    size_t sent_slots = 0, sent_rows = 0;
    for (int p = 0; p < P; ++p) {
        sent_slots += (size_t)send_slots[p];
        sent_rows += (size_t)send_rows[p];
    }
    const int ranksum = st->combine == OMC_EP_RANKSUM;
    /* 4. pack and send the rows */
    uint16_t *send_x = NULL, *opnd = NULL;
    int32_t *send_m = NULL, *recv_m = NULL, *slot_tok = NULL, *slot_e = NULL;
    float *slot_w = NULL, *y = NULL, *ret = NULL;
    if ((rc = ep_buf(st, B_SENDX, (size_t)Tz * fan * D * 2, (void **)&send_x)) ||
        (rc = ep_buf(st, B_SENDM, (size_t)Tz * fan * M * 4, (void **)&send_m)) ||
        (rc = ep_buf(st, B_OPND, ((size_t)Tz + Rr) * D * 2, (void **)&opnd)) ||
        (rc = ep_buf(st, B_RECVM, (size_t)Rr * M * 4, (void **)&recv_m)) ||
        (rc = ep_buf(st, B_STOK, (size_t)Ntot * 4, (void **)&slot_tok)) ||
        (rc = ep_buf(st, B_SE, (size_t)Ntot * 4, (void **)&slot_e)) ||
        (rc = ep_buf(st, B_SW, (size_t)Ntot * 4, (void **)&slot_w)) ||
        (rc = ep_buf(st, B_Y, (size_t)Ntot * D * 4, (void **)&y)) ||
        (rc = ep_buf(st, B_RET, (ranksum ? sent_rows : sent_slots) * D * 4, (void **)&ret)))
        return rc;
    float *rsum = NULL;
    if (ranksum && (rc = ep_buf(st, B_RSUM, (size_t)Rr * D * 4, (void **)&rsum))) return rc;
    if (T > 0 && (rc = omc_launch_ep_pack(gemma ? xe : x, idx, w, T, D, k, ne, P, tok_pos, slot_pos, counts, send_x,
                                          send_m, sh ? opnd : NULL, G.d_err, s)))
        return omc_fail(rc, "ep pack launch failed");
    omc_prof_mark(s, "ep_route_pack");
    NCK(N.GroupStart());
    for (int p = 0; p < P; ++p) {
        if (send_rows[p]) {
            NCK(N.Send(send_x + (size_t)send_base[p] * D, (size_t)send_rows[p] * D * 2, ncclUint8, p, st->comm, s));
            NCK(N.Send(send_m + (size_t)send_base[p] * M, (size_t)send_rows[p] * M, ncclInt32, p, st->comm, s));
        }
        const int nr = recv_base[p + 1] - recv_base[p];
        if (nr) {
            NCK(N.Recv(opnd + ((size_t)Tz + recv_base[p]) * D, (size_t)nr * D * 2, ncclUint8, p, st->comm, s));
            NCK(N.Recv(recv_m + (size_t)recv_base[p] * M, (size_t)nr * M, ncclInt32, p, st->comm, s));
        }
    }
    NCK(N.GroupEnd());
    omc_prof_mark(s, "ep_dispatch");
    /* 5. the slots through the local experts (and the home tokens' shared expert) */
    if (Ntot > 0) {
        if ((rc = omc_ws_ensure_rows_in(L, Ntot, &st->xws, &st->xW, st->xbytes))) return rc;
        omc_ws *ws = &st->xws;
        CK(cudaMemsetAsync(ws->counts, 0, (size_t)(ws->done - ws->counts + 1) * sizeof(int), s));
        if ((rc = omc_launch_ep_unpack(recv_m, Rr, k, P, recv_base, slot_base, Tz, E, L->e0, L->e0 + L->ne, sh, Sr,
                                       slot_tok, slot_e, slot_w, ws->counts, ws->slotrow, G.d_err, s)))
            return omc_fail(rc, "ep unpack launch failed");
        if ((rc = omc_launch_mma_slots(P_, opnd, Ntot, slot_tok, slot_e, slot_w, ws, L->e0, L->e0 + L->ne, y, s)))
            return omc_fail(rc, "ep expert pass launch failed (%s)", omc_strerror(rc));
    }
    /* 6. the partials back home: one f32 row per routed slot (exact), or per
     * received token row the sum of its slots here, in selection order */
    if (ranksum && Rr > 0 &&
        (rc = omc_launch_ep_ranksum(recv_m, Rr, k, P, recv_base, slot_base, y, D, rsum, s)))
        return omc_fail(rc, "ep rank-sum launch failed");
    NCK(N.GroupStart());
    for (int p = 0; p < P; ++p) {
        if (ranksum) {
            const int nr = recv_base[p + 1] - recv_base[p];
            if (nr) NCK(N.Send(rsum + (size_t)recv_base[p] * D, (size_t)nr * D, ncclFloat32, p, st->comm, s));
            if (send_rows[p])
                NCK(N.Recv(ret + (size_t)send_base[p] * D, (size_t)send_rows[p] * D, ncclFloat32, p, st->comm, s));
        } else {
            const int ns = slot_base[p + 1] - slot_base[p];
            if (ns) NCK(N.Send(y + (size_t)slot_base[p] * D, (size_t)ns * D, ncclFloat32, p, st->comm, s));
            if (send_slots[p])
                NCK(N.Recv(ret + (size_t)ret_base[p] * D, (size_t)send_slots[p] * D, ncclFloat32, p, st->comm, s));
        }
    }
    NCK(N.GroupEnd());
    omc_prof_mark(s, "ep_return");
    /* 7. combine at home */
    if (T > 0) {
        rc = ranksum ? omc_launch_ep_combine_ranksum(ret, tok_pos, idx, sh ? y + (size_t)Sr * D : NULL, sg, T, D, k,
                                                     ne, P, sh, out, s)
                     : omc_launch_ep_combine(ret, slot_pos, sh ? y + (size_t)Sr * D : NULL, sg, T, D, k, sh, out, s);
        if (rc) return omc_fail(rc, "ep combine launch failed");
        if (topk_idx) CK(cudaMemcpyAsync(topk_idx, idx, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
        if (topk_w) CK(cudaMemcpyAsync(topk_w, w, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
    }
    omc_prof_mark(s, "combine");
    G.prof_valid = G.profiling;
    (void)me;
    return OMC_OK;
}

void omc_ep_release(void) {
    omc_ep_state *st = (omc_ep_state *)G.ep;
    if (!st) return;
    if (st->have_comm) N.CommDestroy(st->comm);
    for (int i = 0; i < 16; ++i) cudaFree(st->buf[i]);
    omc_ws_free_in(&st->xW, st->xbytes, 16);
    if (st->h_cnt) cudaFreeHost(st->h_cnt);
    if (st->ev) cudaEventDestroy(st->ev);
    free(st);
    G.ep = NULL;
}

/* ------------------------------------------------- host versions (tests) -- */
int omc_ep_layout_host(const int32_t *idx, const float *w, int T, int k, int E, int P, int32_t *tok_pos,
                       int32_t *slot_pos, int32_t *counts, int32_t *meta) {
    if (T < 0 || k < 1 || P < 1 || P > OMC_EP_MAX_RANKS || E % P) return -1;
    const int ne = E / P, M = omc_ep_meta_ints(k);
    int cnt[OMC_EP_MAX_RANKS], rows[OMC_EP_MAX_RANKS] = {0}, slots[OMC_EP_MAX_RANKS] = {0};
    for (int t = 0; t < T; ++t) {
        omc_ep_token_counts(idx + (size_t)t * k, k, ne, P, cnt);
        for (int r = 0; r < P; ++r) {
            rows[r] += cnt[r] > 0;
            slots[r] += cnt[r];
        }
    }
    int send_base[OMC_EP_MAX_RANKS], ret_base[OMC_EP_MAX_RANKS], ar = 0, as = 0;
    for (int r = 0; r < P; ++r) {
        send_base[r] = ar;
        ret_base[r] = as;
        ar += rows[r];
        as += slots[r];
        counts[r] = rows[r];
        counts[P + r] = slots[r];
        counts[2 * P + r] = send_base[r];
        counts[3 * P + r] = ret_base[r];
    }
    int row_before[OMC_EP_MAX_RANKS] = {0}, slot_before[OMC_EP_MAX_RANKS] = {0};
    for (int t = 0; t < T; ++t) {
        const int32_t *it = idx + (size_t)t * k;
        omc_ep_token_counts(it, k, ne, P, cnt);
        omc_ep_token_positions(it, k, ne, P, row_before, slot_before, send_base, ret_base, cnt,
                               tok_pos + (size_t)t * P, slot_pos + (size_t)t * k);
        for (int r = 0; r < P; ++r)
            if (cnt[r] > 0 && meta)
                omc_ep_token_meta(it, w + (size_t)t * k, k, ne, r, slot_before[r],
                                  meta + (size_t)tok_pos[(size_t)t * P + r] * M);
        for (int r = 0; r < P; ++r) {
            row_before[r] += cnt[r] > 0;
            slot_before[r] += cnt[r];
        }
    }
    return ar;
}

int omc_ep_unpack_host(const int32_t *meta, const int32_t *recv_rows, const int32_t *recv_slots, int P, int k,
                       int Thome, int E, int has_shared, int32_t *slot_tok, int32_t *slot_e, float *slot_w) {
    if (P < 1 || P > OMC_EP_MAX_RANKS || k < 1) return -1;
    const int M = omc_ep_meta_ints(k);
    int recv_base[OMC_EP_MAX_RANKS + 1], slot_base[OMC_EP_MAX_RANKS + 1];
    recv_base[0] = slot_base[0] = 0;
    for (int p = 0; p < P; ++p) {
        recv_base[p + 1] = recv_base[p] + recv_rows[p];
        slot_base[p + 1] = slot_base[p] + recv_slots[p];
    }
    const int Rr = recv_base[P], Sr = slot_base[P];
    for (int i = 0; i < Rr; ++i) {
        const int p = omc_ep_row_peer(recv_base, P, i);
        const int32_t *m = meta + (size_t)i * M;
        const int n = m[1], base = slot_base[p] + m[0];
        if (n < 0 || n > k || m[0] < 0 || base + n > slot_base[p + 1]) return -1;
        for (int q = 0; q < n; ++q) {
            union { int32_t i; float f; } u;
            u.i = m[2 + k + q];
            slot_tok[base + q] = Thome + i;
            slot_e[base + q] = m[2 + q];
            slot_w[base + q] = u.f;
        }
    }
    if (has_shared)
        for (int t = 0; t < Thome; ++t) {
            slot_tok[Sr + t] = t;
            slot_e[Sr + t] = E;
            slot_w[Sr + t] = 1.f;
        }
    return Sr + (has_shared ? Thome : 0);
}
