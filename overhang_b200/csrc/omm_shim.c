/* omm_shim.c -- the engines' omm_* GPU seam (metal/om_metal.h:14-46) on CUDA.
 *
 * The unmodified engines, built with -DOM_METAL against include/om_metal.h,
 * hand their prefill MoE here (engines/olmoe.c:365-384): routing stays on the
 * CPU, and omm_moe() receives one job per expert that received tokens (the
 * batch union, experts ascending) with that expert's int8 weights, the
 * positions routed to it and their router weights.  The reference backend
 * computes out[pos[r]] += w[r] * SwiGLU_expert(x[pos[r]]) job by job
 * (metal/om_metal.mm:208-296); so does this one, on the tensor-core grouped
 * GEMM of the full forward:
 *
 *   - a job's weights (host memory of the engine's expert slots) are copied
 *     once into HBM in the paired tile layout and looked up by the slot's g
 *     pointer afterwards.  The engine's LRU may load another expert into the
 *     same slot (engines/olmoe.c:263-270); a slot whose three scale vectors
 *     changed is re-uploaded into the same device buffers;
 *   - x is copied in, each job's rows gathered, the jobs run as one
 *     explicit-rows pass (the jobs are the experts of a scratch layer), and
 *     every position's weighted rows are added to out in job order, one
 *     sequential fp32 chain per element, then out is copied back.
 *
 * Status codes are the reference's: 0 done, -1 allocation or device failure
 * (the engine then falls back to its CPU path), -3 a shape this build does
 * not serve (D or I not a multiple of 64, more than 1024 jobs).  gelu = 1 runs
 * the experts with gelu_tanh (engines/gemma.c:319-321), as Gemma's call does.
 * omm_dense_q runs the engine's int8 projections on the tensor-core GEMM,
 * omm_dense its f32 ones through a cached half copy on the same GEMM (below). */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "om_metal.h"
#include "om_cuda.h"
#include "omc_host.h"

#define G omc_G

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

/* ---- identity of the engine's int8 tensors ------------------------------ */
/* The engine refills an expert slot in place when its LRU evicts
 * (engines/olmoe.c:263-270), and the reference's Metal backend reads the slot
 * memory on every call (metal/om_metal.mm:186-229), so a device copy is
 * reused only while the slot's contents are unchanged: the same pointer,
 * bit-equal scales and an equal 64-bit hash of the int8 rows.  The hash runs
 * four XXH64-style lanes (multiply by a 64-bit prime, rotate by 31, multiply)
 * over 32-byte stripes at memory speed; a change that keeps the scales leaves
 * the hash equal with probability 2^-64.  With OMM_TRUST_SLOTS=1 in the
 * environment the pointer and scales alone identify a slot (exact when the
 * engine never evicts: QCACHE >= E). */
static const uint64_t HP1 = 0x9E3779B185EBCA87ull, HP2 = 0xC2B2AE3D27D4EB4Full, HP3 = 0x165667B19E3779F9ull;

static inline uint64_t rotl64(uint64_t v, int r) { return (v << r) | (v >> (64 - r)); }
static inline uint64_t hround(uint64_t acc, uint64_t w) { return rotl64(acc + w * HP2, 31) * HP1; }

static uint64_t omm_hash(const void *p, size_t n, uint64_t seed) {
    const unsigned char *b = (const unsigned char *)p;
    uint64_t a0 = seed + HP1 + HP2, a1 = seed + HP2, a2 = seed, a3 = seed - HP1;
    size_t i = 0;
    for (; i + 32 <= n; i += 32) {
        uint64_t w[4];
        memcpy(w, b + i, 32);
        a0 = hround(a0, w[0]);
        a1 = hround(a1, w[1]);
        a2 = hround(a2, w[2]);
        a3 = hround(a3, w[3]);
    }
    uint64_t h = rotl64(a0, 1) + rotl64(a1, 7) + rotl64(a2, 12) + rotl64(a3, 18) + (uint64_t)n;
    for (; i < n; ++i) h = rotl64(h ^ (b[i] * HP3), 11) * HP1;
    h ^= h >> 33;
    h *= HP2;
    h ^= h >> 29;
    h *= HP3;
    h ^= h >> 32;
    return h;
}

static int trust_slots(void) {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("OMM_TRUST_SLOTS");
        v = e && e[0] == '1';
    }
    return v;
}

/* ---- device copies of the engine's expert slots ------------------------ */
typedef struct {
    const int8_t *hg;            /* the slot's g pointer */
    int D, I;
    float *sc;                   /* host copy of gs | us | ds the device copy was made from */
    uint64_t h;                  /* hash of the g, u, d rows the device copy was made from */
    omc_expert_ptrs dev;
} omm_slot;

static uint64_t slot_hash(const omm_job *j, int D, int I) {
    const size_t n = (size_t)I * D;
    return omm_hash(j->g, n, 1) ^ rotl64(omm_hash(j->u, n, 2), 21) ^ rotl64(omm_hash(j->d, n, 3), 42);
}

static omm_slot *g_slots;
static int g_nslots, g_cap;

static int resolve(const omm_job *j, int D, int I, omc_expert_ptrs *out) {
    const size_t nsc = (size_t)2 * I + D;
    omm_slot *sl = NULL;
    for (int i = 0; i < g_nslots; ++i)
        if (g_slots[i].hg == j->g && g_slots[i].D == D && g_slots[i].I == I) {
            sl = &g_slots[i];
            break;
        }
    const uint64_t h = trust_slots() ? 0 : slot_hash(j, D, I);
    if (sl && !memcmp(sl->sc, j->gs, (size_t)I * 4) && !memcmp(sl->sc + I, j->us, (size_t)I * 4) &&
        !memcmp(sl->sc + 2 * I, j->ds, (size_t)D * 4) && sl->h == h) {
        *out = sl->dev;
        return OMC_OK;
    }
    int reuse = sl != NULL;
    if (!sl) {
        if (g_nslots == g_cap) {
            const int nc = g_cap ? 2 * g_cap : 64;
            omm_slot *ns = realloc(g_slots, sizeof(omm_slot) * (size_t)nc);
            if (!ns) return OMC_ENOMEM;
            g_slots = ns;
            g_cap = nc;
        }
        sl = &g_slots[g_nslots];
        memset(sl, 0, sizeof(*sl));
        sl->sc = malloc(sizeof(float) * nsc);
        if (!sl->sc) return OMC_ENOMEM;
        sl->hg = j->g;
        sl->D = D;
        sl->I = I;
    }
    const int Dr = omc_round_up(D, OMC_TM), Ir = omc_round_up(I, OMC_TM);
    int rc = omc_expert_upload(D, D, Dr, I, I, Ir, j->g, j->gs, j->u, j->us, j->d, j->ds, &sl->dev, reuse);
    if (rc) return rc;
    if (!reuse) ++g_nslots;
    memcpy(sl->sc, j->gs, (size_t)I * 4);
    memcpy(sl->sc + I, j->us, (size_t)I * 4);
    memcpy(sl->sc + 2 * I, j->ds, (size_t)D * 4);
    sl->h = h;
    *out = sl->dev;
    return OMC_OK;
}

/* ---- grow-only device scratch of the job pass -------------------------- */
enum { B_TAB, B_X, B_OUT, B_ROWS, B_Y, B_POS, B_W, B_IDS, B_OFF, B_LIST, NBUF };
static void *g_buf[NBUF];
static size_t g_bytes[NBUF];

static void *scratch(int i, size_t n) {
    if (g_bytes[i] >= n && g_buf[i]) return g_buf[i];
    if (g_buf[i]) cudaFree(g_buf[i]);
    g_buf[i] = NULL;
    g_bytes[i] = 0;
    if (cudaMalloc(&g_buf[i], n ? n : 16) != cudaSuccess) {
        cudaGetLastError();
        return NULL;
    }
    g_bytes[i] = n;
    return g_buf[i];
}

int omm_moe_act(const omm_job *jobs, int nj, const float *x, int S, int D, int I, float *out, int gelu) {
    if (!omm_init()) return -1;
    if (nj <= 0 || S <= 0) return 0;
    if (!jobs || !x || !out || D <= 0 || I <= 0 || D % 64 || I % 64 || nj > OMC_MAX_E) return -3;
    long long Rl = 0;
    for (int j = 0; j < nj; ++j) {
        if (jobs[j].mpos < 0 || (jobs[j].mpos > 0 && (!jobs[j].pos || !jobs[j].w))) return -3;
        for (int r = 0; r < jobs[j].mpos; ++r)
            if (jobs[j].pos[r] < 0 || jobs[j].pos[r] >= S) return -3;
        Rl += jobs[j].mpos;
    }
    if (Rl == 0) return 0;
    if (Rl > (1 << 28)) return -3;
    const int R = (int)Rl;
    cudaSetDevice(G.device);
    cudaStream_t s = G.stream;
    int rc = 0;

    /* the jobs as the experts of a scratch layer */
    omc_expert_ptrs *tab = malloc(sizeof(omc_expert_ptrs) * (size_t)nj);
    int *hpos = malloc(sizeof(int) * (size_t)R), *hids = malloc(sizeof(int) * (size_t)R);
    int *hoff = calloc((size_t)S + 1, sizeof(int)), *hlist = malloc(sizeof(int) * (size_t)R);
    float *hw = malloc(sizeof(float) * (size_t)R);
    if (!tab || !hpos || !hids || !hoff || !hlist || !hw) {
        rc = -1;
        goto done;
    }
    for (int j = 0; j < nj; ++j)
        if (resolve(&jobs[j], D, I, &tab[j])) {
            rc = -1;
            goto done;
        }
    /* rows in job order; per position, its rows in job order */
    for (int j = 0, r = 0; j < nj; ++j)
        for (int q = 0; q < jobs[j].mpos; ++q, ++r) {
            hpos[r] = jobs[j].pos[q];
            hw[r] = jobs[j].w[q];
            hids[r] = j;
            hoff[hpos[r] + 1]++;
        }
    for (int i = 0; i < S; ++i) hoff[i + 1] += hoff[i];
    {
        int *fill = calloc((size_t)S, sizeof(int));
        if (!fill) {
            rc = -1;
            goto done;
        }
        for (int r = 0; r < R; ++r) hlist[hoff[hpos[r]] + fill[hpos[r]]++] = r;
        free(fill);
    }
    omc_layer TL;
    memset(&TL, 0, sizeof(TL));
    TL.desc.family = OMC_FAMILY_OLMOE;         /* SwiGLU g/(1+exp(-g))*u, engines/olmoe.c:393 */
    TL.desc.D = D;
    TL.desc.I = I;
    TL.desc.E = nj;
    TL.desc.k = 1;
    TL.dev.family = OMC_FAMILY_OLMOE;
    /* rows are already the experts' input (the caller normed them);
     * gelu != 0: gelu_tanh(g)*u (engines/gemma.c:319-321 via omm_moe_act,
     * :628), else the SwiGLU of engines/olmoe.c:393 */
    TL.dev.act = gelu ? OMC_ACT_GELU_TANH : OMC_ACT_SILU_DIV;
    TL.dev.D = D;
    TL.dev.I = I;
    TL.dev.E = nj;
    TL.dev.k = 1;
    TL.dev.D_pad = D;
    TL.dev.I_pad = I;
    TL.dev.D_rows = omc_round_up(D, OMC_TM);
    TL.dev.I_rows = omc_round_up(I, OMC_TM);
    TL.e0 = 0;
    TL.ne = nj;
    void *d_tab = scratch(B_TAB, sizeof(omc_expert_ptrs) * (size_t)(nj + 1));
    float *d_x = scratch(B_X, (size_t)S * D * 4), *d_out = scratch(B_OUT, (size_t)S * D * 4);
    float *d_rows = scratch(B_ROWS, (size_t)R * D * 4), *d_y = scratch(B_Y, (size_t)R * D * 4);
    int *d_pos = scratch(B_POS, (size_t)R * 4), *d_ids = scratch(B_IDS, (size_t)R * 4);
    float *d_w = scratch(B_W, (size_t)R * 4);
    int *d_off = scratch(B_OFF, ((size_t)S + 1) * 4), *d_list = scratch(B_LIST, (size_t)R * 4);
    if (!d_tab || !d_x || !d_out || !d_rows || !d_y || !d_pos || !d_ids || !d_w || !d_off || !d_list ||
        omc_ws_ensure_rows(&TL, R)) {
        rc = -1;
        goto done;
    }
    TL.dev.experts = (const omc_expert_ptrs *)d_tab;
    if (cudaMemcpyAsync(d_tab, tab, sizeof(omc_expert_ptrs) * (size_t)nj, cudaMemcpyHostToDevice, s) ||
        cudaMemcpyAsync(d_x, x, (size_t)S * D * 4, cudaMemcpyHostToDevice, s) ||
        cudaMemcpyAsync(d_out, out, (size_t)S * D * 4, cudaMemcpyHostToDevice, s) ||
        cudaMemcpyAsync(d_pos, hpos, (size_t)R * 4, cudaMemcpyHostToDevice, s) ||
        cudaMemcpyAsync(d_ids, hids, (size_t)R * 4, cudaMemcpyHostToDevice, s) ||
        cudaMemcpyAsync(d_w, hw, (size_t)R * 4, cudaMemcpyHostToDevice, s) ||
        cudaMemcpyAsync(d_off, hoff, ((size_t)S + 1) * 4, cudaMemcpyHostToDevice, s) ||
        cudaMemcpyAsync(d_list, hlist, (size_t)R * 4, cudaMemcpyHostToDevice, s)) {
        cudaGetLastError();
        rc = -1;
        goto done;
    }
    if (omc_launch_gather_rows(d_x, d_pos, R, S, D, d_rows, G.d_err, s) ||
        omc_launch_mma_rows(&TL.dev, d_rows, R, &G.ws, d_ids, d_w, 0, nj, d_y, s) ||
        omc_launch_ordered_add(d_out, d_y, d_off, d_list, S, D, s) ||
        cudaMemcpyAsync(out, d_out, (size_t)S * D * 4, cudaMemcpyDeviceToHost, s) || cudaStreamSynchronize(s)) {
        cudaGetLastError();
        rc = -1;
        goto done;
    }
    if (omc_check_device_error()) rc = -1;
done:
    free(tab);
    free(hpos);
    free(hids);
    free(hoff);
    free(hlist);
    free(hw);
    return rc;
}

int omm_moe(const omm_job *jobs, int nj, const float *x, int S, int D, int I, float *out) {
    return omm_moe_act(jobs, nj, x, S, D, I, out, 0);
}

/* ---- dense projections ------------------------------------------------- */
/* omm_dense_q (metal/om_metal.h:38-41): out[S,N] = x[S,K] . dequant(Wq)^T.
 * The engine's int8 matrix (engines/gemma.c:158-175 mat_load, called from
 * mat_apply_b :287-293) is copied once into HBM in the tile layout of the
 * grouped GEMM and found again by its pointer; a matrix whose row scales
 * changed is copied again.  The product runs on the tensor-core down GEMM as
 * a one-matrix layer (tokens in f16, accumulation in f32, the row scale
 * applied to the f32 sum as matmul_q does).  Like the reference backend it
 * takes K % 64 == 0 and N % 32 == 0 and returns -3 otherwise. */
typedef struct {
    const int8_t *hq;            /* the engine's matrix pointer */
    int N, K;
    float *sc;                   /* host copy of the scales the device copy was made from */
    uint64_t h;                  /* hash of the int8 rows it was made from (see omm_hash) */
    int8_t *dq;
    const float *ds;
} omm_dmat;

static omm_dmat *g_dm;
static int g_ndm, g_dmcap;

static int dense_resolve(const int8_t *Wq, const float *scales, int N, int K, omc_expert_ptrs *ep) {
    omm_dmat *m = NULL;
    for (int i = 0; i < g_ndm; ++i)
        if (g_dm[i].hq == Wq && g_dm[i].N == N && g_dm[i].K == K) {
            m = &g_dm[i];
            break;
        }
    const int reuse = m != NULL;
    const uint64_t h = trust_slots() ? 0 : omm_hash(Wq, (size_t)N * K, 4);
    if (!m || memcmp(m->sc, scales, (size_t)N * 4) || m->h != h) {
        if (!m) {
            if (g_ndm == g_dmcap) {
                const int nc = g_dmcap ? 2 * g_dmcap : 64;
                omm_dmat *nm = realloc(g_dm, sizeof(omm_dmat) * (size_t)nc);
                if (!nm) return OMC_ENOMEM;
                g_dm = nm;
                g_dmcap = nc;
            }
            m = &g_dm[g_ndm];
            memset(m, 0, sizeof(*m));
            m->sc = malloc((size_t)N * 4);
            if (!m->sc) return OMC_ENOMEM;
            m->hq = Wq;
            m->N = N;
            m->K = K;
        }
        const int rc = omc_matrix_upload(Wq, scales, N, K, &m->dq, &m->ds, reuse);
        if (rc) return rc;
        memcpy(m->sc, scales, (size_t)N * 4);
        m->h = h;
        if (!reuse) ++g_ndm;
    }
    memset(ep, 0, sizeof(*ep));
    ep->d = m->dq;
    ep->ds = m->ds;
    return OMC_OK;
}

int omm_dense_q(const int8_t *Wq, const float *scales, int N, int K, const float *x, int S, float *out) {
    if (!omm_init()) return -1;
    if (S <= 0) return 0;
    if (!Wq || !scales || !x || !out || N <= 0 || K <= 0 || K % 64 || N % 32) return -3;
    cudaSetDevice(G.device);
    cudaStream_t s = G.stream;
    omc_expert_ptrs tab[2];
    if (dense_resolve(Wq, scales, N, K, &tab[0])) return -1;
    memset(&tab[1], 0, sizeof(tab[1]));
    omc_layer TL;
    memset(&TL, 0, sizeof(TL));
    TL.desc.family = OMC_FAMILY_OLMOE;
    TL.desc.D = N;
    TL.desc.I = K;
    TL.desc.E = 1;
    TL.desc.k = 1;
    TL.dev.family = OMC_FAMILY_OLMOE;
    TL.dev.D = N;
    TL.dev.I = K;
    TL.dev.E = 1;
    TL.dev.k = 1;
    TL.dev.D_pad = omc_round_up(N, OMC_KB);
    TL.dev.I_pad = K;
    TL.dev.D_rows = omc_round_up(N, OMC_TM);
    TL.dev.I_rows = omc_round_up(K, OMC_TM);
    TL.e0 = 0;
    TL.ne = 1;
    void *d_tab = scratch(B_TAB, sizeof(tab));
    float *d_x = scratch(B_X, (size_t)S * K * 4), *d_y = scratch(B_OUT, (size_t)S * N * 4);
    if (!d_tab || !d_x || !d_y || omc_ws_ensure_rows(&TL, S)) return -1;
    TL.dev.experts = (const omc_expert_ptrs *)d_tab;
    if (cudaMemcpyAsync(d_tab, tab, sizeof(tab), cudaMemcpyHostToDevice, s) ||
        cudaMemcpyAsync(d_x, x, (size_t)S * K * 4, cudaMemcpyHostToDevice, s) ||
        omc_launch_dense_i8(&TL.dev, d_x, S, &G.ws, d_y, s) ||
        cudaMemcpyAsync(out, d_y, (size_t)S * N * 4, cudaMemcpyDeviceToHost, s) || cudaStreamSynchronize(s)) {
        cudaGetLastError();
        return -1;
    }
    return omc_check_device_error() ? -1 : 0;
}

/* omm_dense (metal/om_metal.h:43-46): out[S,N] = x[S,K] . W^T with the
 * engine's resident f32 W (engines/olmoe.c:286-292 dense_mm).  As in the
 * reference backend, a half copy of W is made on first use and kept by
 * pointer (here as the tensor-core GEMM's 128-row f16 tiles); x is rounded to
 * half too, and the products are summed in f32 by the library's own
 * tcgen05 GEMM (omc_launch_dense_f16: the down GEMM reading f16 weights into
 * tensor memory as they are).  K % 8 == 0, else -3. */
typedef struct {
    const float *hw;
    int N, K;
    uint16_t *dw;               /* f16 tiles */
    float *ones;                /* [N_pad] row scales of 1 */
} omm_fmat;

static omm_fmat *g_fm;
static int g_nfm, g_fmcap;

int omm_dense(const float *W, int N, int K, const float *x, int S, float *out) {
    if (!omm_init()) return -1;
    if (S <= 0) return 0;
    if (!W || !x || !out || N <= 0 || K <= 0 || K % 8) return -3;
    cudaSetDevice(G.device);
    cudaStream_t s = G.stream;
    omm_fmat *m = NULL;
    for (int i = 0; i < g_nfm; ++i)
        if (g_fm[i].hw == W && g_fm[i].N == N && g_fm[i].K == K) {
            m = &g_fm[i];
            break;
        }
    const int N_rows = omc_round_up(N, OMC_TM);
    if (!m) {
        if (g_nfm == g_fmcap) {
            const int nc = g_fmcap ? 2 * g_fmcap : 64;
            omm_fmat *nm = realloc(g_fm, sizeof(omm_fmat) * (size_t)nc);
            if (!nm) return -1;
            g_fm = nm;
            g_fmcap = nc;
        }
        m = &g_fm[g_nfm];
        memset(m, 0, sizeof(*m));
        const size_t n = (size_t)N * K;
        float *stage = scratch(B_ROWS, n * 4);
        float *h1 = malloc(sizeof(float) * (size_t)N_rows);
        if (!stage || !h1 || cudaMalloc((void **)&m->dw, omc_f16_tiles_bytes(N, K)) != cudaSuccess ||
            cudaMalloc((void **)&m->ones, sizeof(float) * (size_t)N_rows) != cudaSuccess) {
            cudaGetLastError();
            free(h1);
            cudaFree(m->dw);
            return -1;
        }
        for (int i = 0; i < N_rows; ++i) h1[i] = 1.f;
        const int bad = cudaMemcpyAsync(stage, W, n * 4, cudaMemcpyHostToDevice, s) ||
                        cudaMemcpyAsync(m->ones, h1, sizeof(float) * (size_t)N_rows, cudaMemcpyHostToDevice, s) ||
                        omc_launch_f16_tiles(stage, N, K, m->dw, G.d_err, s) || cudaStreamSynchronize(s) ||
                        omc_check_device_error();
        free(h1);
        if (bad) {
            cudaGetLastError();
            cudaFree(m->dw);
            cudaFree(m->ones);
            return -1;
        }
        m->hw = W;
        m->N = N;
        m->K = K;
        ++g_nfm;
    }
    omc_expert_ptrs tab[2];
    memset(tab, 0, sizeof(tab));
    tab[0].d = (const int8_t *)m->dw;
    tab[0].ds = m->ones;
    omc_layer TL;
    memset(&TL, 0, sizeof(TL));
    TL.desc.family = OMC_FAMILY_OLMOE;
    TL.desc.D = N;
    TL.desc.I = K;
    TL.desc.E = 1;
    TL.desc.k = 1;
    TL.dev.family = OMC_FAMILY_OLMOE;
    TL.dev.D = N;
    TL.dev.I = K;
    TL.dev.E = 1;
    TL.dev.k = 1;
    TL.dev.D_pad = omc_round_up(N, OMC_KB);
    TL.dev.I_pad = omc_round_up(K, OMC_KB);
    TL.dev.D_rows = N_rows;
    TL.dev.I_rows = omc_round_up(K, OMC_TM);
    TL.e0 = 0;
    TL.ne = 1;
    void *d_tab = scratch(B_TAB, sizeof(tab));
    float *d_x = scratch(B_X, (size_t)S * K * 4), *d_y = scratch(B_OUT, (size_t)S * N * 4);
    if (!d_tab || !d_x || !d_y || omc_ws_ensure_rows(&TL, S)) return -1;
    TL.dev.experts = (const omc_expert_ptrs *)d_tab;
    if (cudaMemcpyAsync(d_tab, tab, sizeof(tab), cudaMemcpyHostToDevice, s) ||
        cudaMemcpyAsync(d_x, x, (size_t)S * K * 4, cudaMemcpyHostToDevice, s) ||
        omc_launch_dense_f16(&TL.dev, d_x, S, &G.ws, d_y, s) ||
        cudaMemcpyAsync(out, d_y, (size_t)S * N * 4, cudaMemcpyDeviceToHost, s) || cudaStreamSynchronize(s)) {
        cudaGetLastError();
        return -1;
    }
    return omc_check_device_error() ? -1 : 0;
}
