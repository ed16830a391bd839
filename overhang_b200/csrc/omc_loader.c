/* omc_loader.c -- routed experts straight from the engines' int8 container.
 *
 * The engines fill their expert slots one expert at a time from disk
 * (expert_get: engines/olmoe.c:250-272, engines/qwen.c:428-450,
 * engines/gemma.c:335-365): pread of the int8 matrix, pread of its ".qs"
 * scales.  omc_experts_load() does the same reads for a whole layer with
 * several reader threads into pinned staging slots, while the calling thread
 * uploads the finished experts in order (omc_expert_set: copy to HBM and
 * re-tile), so disk, PCIe and the re-tiling overlap.
 *
 * The container is the safetensors layout the converters write
 * (tools/convert_olmoe.py:93-99, tools/convert_gemma.py:386-394): every
 * "*.safetensors" file of the directory is one shard, an 8-byte little-endian
 * header length, a JSON header {name: {"dtype", "shape", "data_offsets"}},
 * then the data.  Matrices are I8 [rows][cols], scales F32 [rows].
 */
#define _GNU_SOURCE
#include <dirent.h>
#include <errno.h>
#include <fcntl.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cuda_runtime.h>

#include "om_cuda.h"
#include "omc_host.h"

#define G omc_G

/* ---- the shard index ---------------------------------------------------- */
typedef struct {
    char *name;
    int file;
    int dtype;          /* 1 = I8, 2 = F32, 0 = other */
    int ndim;
    long long shape[4];
    long long off, nbytes;   /* absolute file offset of the data, size */
} st_ent;

typedef struct {
    int nfiles;
    int *fds;
    st_ent *ents;
    int nents, cap;
    int *hash;          /* open addressing over ents, -1 empty */
    int hcap;
} st_index;

static unsigned long long fnv1a(const char *s) {
    unsigned long long h = 1469598103934665603ULL;
    for (; *s; ++s) h = (h ^ (unsigned char)*s) * 1099511628211ULL;
    return h;
}

/* A minimal reader of the header JSON: objects, arrays, strings, numbers. */
typedef struct {
    const char *p, *end;
} jcur;

static void jws(jcur *c) {
    while (c->p < c->end && (*c->p == ' ' || *c->p == '\n' || *c->p == '\r' || *c->p == '\t')) ++c->p;
}
static int jlit(jcur *c, char ch) {
    jws(c);
    if (c->p < c->end && *c->p == ch) {
        ++c->p;
        return 1;
    }
    return 0;
}
/* a string into buf (escapes kept as the escaped character) */
static int jstr(jcur *c, char *buf, size_t cap) {
    jws(c);
    if (c->p >= c->end || *c->p != '"') return -1;
    ++c->p;
    size_t n = 0;
    while (c->p < c->end && *c->p != '"') {
        char ch = *c->p++;
        if (ch == '\\' && c->p < c->end) ch = *c->p++;
        if (n + 1 < cap) buf[n++] = ch;
    }
    if (c->p >= c->end) return -1;
    ++c->p;
    buf[n] = 0;
    return 0;
}
static int jnum(jcur *c, long long *v) {
    jws(c);
    char *e = NULL;
    *v = strtoll(c->p, &e, 10);
    if (e == c->p) return -1;
    c->p = e;
    return 0;
}
/* skips any value */
static int jskip(jcur *c) {
    jws(c);
    if (c->p >= c->end) return -1;
    if (*c->p == '"') {
        char tmp[8];
        return jstr(c, tmp, sizeof(tmp));
    }
    if (*c->p == '{' || *c->p == '[') {
        const char open = *c->p, close = open == '{' ? '}' : ']';
        ++c->p;
        if (jlit(c, close)) return 0;
        for (;;) {
            if (open == '{') {
                char tmp[8];
                if (jstr(c, tmp, sizeof(tmp)) || !jlit(c, ':')) return -1;
            }
            if (jskip(c)) return -1;
            if (jlit(c, ',')) continue;
            return jlit(c, close) ? 0 : -1;
        }
    }
    while (c->p < c->end && *c->p != ',' && *c->p != '}' && *c->p != ']') ++c->p;
    return 0;
}
static int jints(jcur *c, long long *v, int cap, int *n) {
    if (!jlit(c, '[')) return -1;
    *n = 0;
    if (jlit(c, ']')) return 0;
    for (;;) {
        long long x;
        if (jnum(c, &x)) return -1;
        if (*n < cap) v[*n] = x;
        ++*n;
        if (jlit(c, ',')) continue;
        return jlit(c, ']') ? 0 : -1;
    }
}

static int idx_add(st_index *ix, const st_ent *e) {
    if (ix->nents == ix->cap) {
        const int nc = ix->cap ? 2 * ix->cap : 1024;
        st_ent *ne = realloc(ix->ents, sizeof(st_ent) * (size_t)nc);
        if (!ne) return -1;
        ix->ents = ne;
        ix->cap = nc;
    }
    ix->ents[ix->nents++] = *e;
    return 0;
}

static int parse_header(st_index *ix, int file, const char *h, long long len, long long data0) {
    jcur c = {h, h + len};
    if (!jlit(&c, '{')) return -1;
    if (jlit(&c, '}')) return 0;
    char name[512], key[64], dt[16];
    for (;;) {
        if (jstr(&c, name, sizeof(name)) || !jlit(&c, ':')) return -1;
        if (!strcmp(name, "__metadata__")) {
            if (jskip(&c)) return -1;
        } else {
            st_ent e;
            memset(&e, 0, sizeof(e));
            e.file = file;
            long long offs[2] = {-1, -1};
            int noff = 0;
            if (!jlit(&c, '{')) return -1;
            if (!jlit(&c, '}'))
                for (;;) {
                    if (jstr(&c, key, sizeof(key)) || !jlit(&c, ':')) return -1;
                    if (!strcmp(key, "dtype")) {
                        if (jstr(&c, dt, sizeof(dt))) return -1;
                        e.dtype = !strcmp(dt, "I8") ? 1 : !strcmp(dt, "F32") ? 2 : 0;
                    } else if (!strcmp(key, "shape")) {
                        if (jints(&c, e.shape, 4, &e.ndim)) return -1;
                    } else if (!strcmp(key, "data_offsets")) {
                        if (jints(&c, offs, 2, &noff) || noff != 2) return -1;
                    } else if (jskip(&c)) {
                        return -1;
                    }
                    if (jlit(&c, ',')) continue;
                    if (!jlit(&c, '}')) return -1;
                    break;
                }
            if (offs[0] < 0 || offs[1] < offs[0]) return -1;
            e.off = data0 + offs[0];
            e.nbytes = offs[1] - offs[0];
            e.name = strdup(name);
            if (!e.name || idx_add(ix, &e)) return -1;
        }
        if (jlit(&c, ',')) continue;
        return jlit(&c, '}') ? 0 : -1;
    }
}

static void idx_close(st_index *ix) {
    for (int i = 0; i < ix->nfiles; ++i) close(ix->fds[i]);
    for (int i = 0; i < ix->nents; ++i) free(ix->ents[i].name);
    free(ix->fds);
    free(ix->ents);
    free(ix->hash);
    memset(ix, 0, sizeof(*ix));
}

static int idx_open(st_index *ix, const char *dir) {
    memset(ix, 0, sizeof(*ix));
    DIR *d = opendir(dir);
    if (!d) return omc_fail(OMC_EINVAL, "container: cannot open directory %s (%s)", dir, strerror(errno));
    struct dirent *de;
    int rc = OMC_OK;
    while ((de = readdir(d)) != NULL) {
        const size_t n = strlen(de->d_name);
        if (n < 12 || strcmp(de->d_name + n - 12, ".safetensors")) continue;
        char path[4096];
        snprintf(path, sizeof(path), "%s/%s", dir, de->d_name);
        const int fd = open(path, O_RDONLY);
        if (fd < 0) {
            rc = omc_fail(OMC_EINVAL, "container: cannot open %s", path);
            break;
        }
        unsigned char lb[8];
        if (pread(fd, lb, 8, 0) != 8) {
            close(fd);
            rc = omc_fail(OMC_EINVAL, "container: %s: no header", path);
            break;
        }
        long long hl = 0;
        for (int i = 7; i >= 0; --i) hl = (hl << 8) | lb[i];
        if (hl <= 0 || hl > (1LL << 30)) {
            close(fd);
            rc = omc_fail(OMC_EINVAL, "container: %s: header length %lld", path, hl);
            break;
        }
        char *h = malloc((size_t)hl);
        if (!h || pread(fd, h, (size_t)hl, 8) != (ssize_t)hl) {
            free(h);
            close(fd);
            rc = omc_fail(OMC_EINVAL, "container: %s: short header", path);
            break;
        }
        int *nf = realloc(ix->fds, sizeof(int) * (size_t)(ix->nfiles + 1));
        if (!nf) {
            free(h);
            close(fd);
            rc = omc_fail(OMC_ENOMEM, "container: host alloc");
            break;
        }
        ix->fds = nf;
        ix->fds[ix->nfiles] = fd;
        const int prc = parse_header(ix, ix->nfiles, h, hl, 8 + hl);
        ++ix->nfiles;
        free(h);
        if (prc) {
            rc = omc_fail(OMC_EINVAL, "container: %s: malformed header", path);
            break;
        }
    }
    closedir(d);
    if (rc == OMC_OK && ix->nfiles == 0) rc = omc_fail(OMC_EINVAL, "container: no *.safetensors in %s", dir);
    if (rc == OMC_OK) {
        ix->hcap = 16;
        while (ix->hcap < 2 * ix->nents) ix->hcap *= 2;
        ix->hash = malloc(sizeof(int) * (size_t)ix->hcap);
        if (!ix->hash) rc = omc_fail(OMC_ENOMEM, "container: host alloc");
        else {
            for (int i = 0; i < ix->hcap; ++i) ix->hash[i] = -1;
            for (int i = 0; i < ix->nents; ++i) {
                unsigned long long k = fnv1a(ix->ents[i].name) & (unsigned long long)(ix->hcap - 1);
                while (ix->hash[k] >= 0) k = (k + 1) & (unsigned long long)(ix->hcap - 1);
                ix->hash[k] = i;
            }
        }
    }
    if (rc) idx_close(ix);
    return rc;
}

static const st_ent *idx_find(const st_index *ix, const char *name) {
    unsigned long long k = fnv1a(name) & (unsigned long long)(ix->hcap - 1);
    while (ix->hash[k] >= 0) {
        const st_ent *e = &ix->ents[ix->hash[k]];
        if (!strcmp(e->name, name)) return e;
        k = (k + 1) & (unsigned long long)(ix->hcap - 1);
    }
    return NULL;
}

static int read_full(int fd, void *dst, long long n, long long off) {
    char *p = dst;
    while (n > 0) {
        const ssize_t r = pread(fd, p, (size_t)(n > (1LL << 30) ? (1LL << 30) : n), off);
        if (r <= 0) {
            if (r < 0 && errno == EINTR) continue;
            return -1;
        }
        p += r;
        off += r;
        n -= r;
    }
    return 0;
}

/* One tensor into dst: its dtype and [rows][cols] shape must match. */
static int read_tensor(const st_index *ix, const char *name, int dtype, long long rows, long long cols, void *dst,
                       char *err, size_t errcap) {
    const st_ent *e = idx_find(ix, name);
    if (!e) {
        snprintf(err, errcap, "tensor %s not in the container", name);
        return -1;
    }
    const long long want_elems = rows * (cols > 0 ? cols : 1);
    long long elems = 1;
    for (int i = 0; i < e->ndim; ++i) elems *= e->shape[i];
    const int shape_ok = cols > 0 ? (e->ndim == 2 && e->shape[0] == rows && e->shape[1] == cols)
                                  : (e->ndim == 1 && e->shape[0] == rows);
    if (e->dtype != dtype || !shape_ok || elems != want_elems || e->nbytes != want_elems * (dtype == 1 ? 1 : 4)) {
        snprintf(err, errcap, "tensor %s: dtype or shape differs from the layer", name);
        return -1;
    }
    if (read_full(ix->fds[e->file], dst, e->nbytes, e->off)) {
        snprintf(err, errcap, "tensor %s: read failed", name);
        return -1;
    }
    return 0;
}

/* ---- the loader ----------------------------------------------------------- */
#define LD_SLOTS_PER_THREAD 2

typedef struct {
    int expert;      /* the expert it holds */
    int state;       /* 0 free, 1 being read, 2 ready, 3 failed */
    int turn;        /* the expert index (from e0) it takes next: k, k + nslots, ... */
    unsigned char *buf;
} ld_slot;

typedef struct {
    const st_index *ix;
    int layer, e0, ne, D, I, fused;   /* layer: the container's layer index */
    const char *ng, *nu, *nd;
    int nslots, next;
    ld_slot *slots;
    pthread_mutex_t mu;
    pthread_cond_t cv;
    int stop;
    char err[512];
    size_t gbytes, dbytes;   /* one matrix of g (u) and d */
} ld_job;

static int fmt_name(char *buf, size_t cap, const char *pat, int layer, int e, const char *suffix) {
    const int n = snprintf(buf, cap, pat, layer, e);
    if (n < 0 || (size_t)n >= cap) return -1;
    if (suffix && strlen(buf) + strlen(suffix) + 1 > cap) return -1;
    if (suffix) strcat(buf, suffix);
    return 0;
}

/* one expert into a slot: g | u | d int8, then gs | us | ds f32 */
static int read_expert(ld_job *j, int e, unsigned char *b, char *err, size_t errcap) {
    const long long D = j->D, I = j->I;
    unsigned char *g = b, *u = b + j->gbytes, *d = b + 2 * j->gbytes;
    float *gs = (float *)(b + 2 * j->gbytes + j->dbytes), *us = gs + I, *ds = us + I;
    char nm[512];
    int rc = 0;
    if (j->fused) {   /* gate_up [2I][D]: gate rows then up rows, scales likewise */
        rc |= fmt_name(nm, sizeof(nm), j->ng, j->layer, e, NULL) || read_tensor(j->ix, nm, 1, 2 * I, D, g, err, errcap);
        if (!rc)
            rc |= fmt_name(nm, sizeof(nm), j->ng, j->layer, e, ".qs") ||
                  read_tensor(j->ix, nm, 2, 2 * I, 0, gs, err, errcap);
    } else {
        rc |= fmt_name(nm, sizeof(nm), j->ng, j->layer, e, NULL) || read_tensor(j->ix, nm, 1, I, D, g, err, errcap);
        if (!rc)
            rc |= fmt_name(nm, sizeof(nm), j->ng, j->layer, e, ".qs") ||
                  read_tensor(j->ix, nm, 2, I, 0, gs, err, errcap);
        if (!rc)
            rc |= fmt_name(nm, sizeof(nm), j->nu, j->layer, e, NULL) || read_tensor(j->ix, nm, 1, I, D, u, err, errcap);
        if (!rc)
            rc |= fmt_name(nm, sizeof(nm), j->nu, j->layer, e, ".qs") ||
                  read_tensor(j->ix, nm, 2, I, 0, us, err, errcap);
    }
    if (!rc) rc |= fmt_name(nm, sizeof(nm), j->nd, j->layer, e, NULL) || read_tensor(j->ix, nm, 1, D, I, d, err, errcap);
    if (!rc)
        rc |= fmt_name(nm, sizeof(nm), j->nd, j->layer, e, ".qs") || read_tensor(j->ix, nm, 2, D, 0, ds, err, errcap);
    if (rc && !err[0]) snprintf(err, errcap, "tensor name pattern too long");
    return rc ? -1 : 0;
}

static void *reader(void *arg) {
    ld_job *j = arg;
    char err[512];
    for (;;) {
        pthread_mutex_lock(&j->mu);
        if (j->stop || j->next >= j->ne) {
            pthread_mutex_unlock(&j->mu);
            return NULL;
        }
        const int k = j->next++;
        ld_slot *s = &j->slots[k % j->nslots];
        while (!j->stop && !(s->state == 0 && s->turn == k)) pthread_cond_wait(&j->cv, &j->mu);
        if (j->stop) {
            pthread_mutex_unlock(&j->mu);
            return NULL;
        }
        s->state = 1;
        s->expert = j->e0 + k;
        pthread_mutex_unlock(&j->mu);
        err[0] = 0;
        const int rc = read_expert(j, j->e0 + k, s->buf, err, sizeof(err));
        pthread_mutex_lock(&j->mu);
        s->state = rc ? 3 : 2;
        if (rc && !j->err[0]) snprintf(j->err, sizeof(j->err), "%s", err);
        pthread_cond_broadcast(&j->cv);
        pthread_mutex_unlock(&j->mu);
    }
}

int omc_experts_load(int layer, const char *snapshot, int src_layer, const char *name_g, const char *name_u,
                     const char *name_d, int nthreads) {
    if (!G.init) return omc_fail(OMC_ENOINIT, "omc_experts_load: omc_init not called");
    omc_layer *L = omc_get_layer(layer);
    if (!L) return omc_fail(OMC_ENOINIT, "omc_experts_load: layer %d not initialised", layer);
    if (!snapshot || !name_g || !name_d) return omc_fail(OMC_EINVAL, "omc_experts_load: null argument");
    if (nthreads <= 0) nthreads = 8;
    if (nthreads > 64) nthreads = 64;
    st_index ix;
    int rc = idx_open(&ix, snapshot);
    if (rc) return rc;
    ld_job j;
    memset(&j, 0, sizeof(j));
    j.ix = &ix;
    j.layer = src_layer;
    j.e0 = L->e0;
    j.ne = L->ne;
    j.D = L->desc.D;
    j.I = L->desc.I;
    j.fused = name_u == NULL;
    j.ng = name_g;
    j.nu = name_u;
    j.nd = name_d;
    j.gbytes = (size_t)j.I * j.D;
    j.dbytes = (size_t)j.D * j.I;
    const size_t slot_bytes = 2 * j.gbytes + j.dbytes + sizeof(float) * (2 * (size_t)j.I + j.D);
    if (nthreads > j.ne) nthreads = j.ne > 0 ? j.ne : 1;
    j.nslots = nthreads * LD_SLOTS_PER_THREAD;
    j.slots = calloc((size_t)j.nslots, sizeof(ld_slot));
    pthread_t *th = calloc((size_t)nthreads, sizeof(pthread_t));
    int nstarted = 0;
    pthread_mutex_init(&j.mu, NULL);
    pthread_cond_init(&j.cv, NULL);
    if (!j.slots || !th) rc = omc_fail(OMC_ENOMEM, "omc_experts_load: host alloc");
    for (int i = 0; !rc && i < j.nslots; ++i) {
        j.slots[i].turn = i;
        if (cudaHostAlloc((void **)&j.slots[i].buf, slot_bytes, cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            rc = omc_fail(OMC_ENOMEM, "omc_experts_load: pinned staging (%zu bytes a slot)", slot_bytes);
        }
    }
    for (int i = 0; !rc && i < nthreads; ++i) {
        if (pthread_create(&th[i], NULL, reader, &j)) {
            rc = omc_fail(OMC_ENOMEM, "omc_experts_load: thread start");
            break;
        }
        ++nstarted;
    }
    /* upload in expert order as the slots become ready */
    for (int k = 0; !rc && k < j.ne; ++k) {
        ld_slot *s = &j.slots[k % j.nslots];
        pthread_mutex_lock(&j.mu);
        while (!(s->state >= 2 && s->expert == j.e0 + k)) pthread_cond_wait(&j.cv, &j.mu);
        const int failed = s->state == 3;
        pthread_mutex_unlock(&j.mu);
        if (failed) {
            rc = omc_fail(OMC_EINVAL, "omc_experts_load: %s", j.err);
            break;
        }
        const unsigned char *b = s->buf;
        const int8_t *g = (const int8_t *)b, *u = (const int8_t *)(b + j.gbytes), *d = (const int8_t *)(b + 2 * j.gbytes);
        const float *gs = (const float *)(b + 2 * j.gbytes + j.dbytes), *us = gs + j.I, *ds = us + j.I;
        rc = omc_expert_set(layer, j.e0 + k, g, gs, u, us, d, ds);   /* synchronous: the slot is free after */
        pthread_mutex_lock(&j.mu);
        s->state = 0;
        s->turn = k + j.nslots;
        pthread_cond_broadcast(&j.cv);
        pthread_mutex_unlock(&j.mu);
    }
    pthread_mutex_lock(&j.mu);
    j.stop = 1;
    pthread_cond_broadcast(&j.cv);
    pthread_mutex_unlock(&j.mu);
    for (int i = 0; i < nstarted; ++i) pthread_join(th[i], NULL);
    for (int i = 0; j.slots && i < j.nslots; ++i) cudaFreeHost(j.slots[i].buf);
    free(j.slots);
    free(th);
    pthread_mutex_destroy(&j.mu);
    pthread_cond_destroy(&j.cv);
    idx_close(&ix);
    return rc;
}

/* Reads one tensor of a container into dst (host) without a device: the
 * index and reader behind omc_experts_load, for tests.  Returns its byte
 * count, or a negative status (too small a buffer: OMC_EINVAL). */
long long omc_debug_container_read(const char *snapshot, const char *name, void *dst, long long cap) {
    st_index ix;
    int rc = idx_open(&ix, snapshot);
    if (rc) return rc;
    const st_ent *e = idx_find(&ix, name);
    long long n = OMC_EINVAL;
    if (!e) omc_fail(OMC_EINVAL, "tensor %s not in the container", name);
    else if (e->nbytes > cap) omc_fail(OMC_EINVAL, "buffer too small for %s", name);
    else if (read_full(ix.fds[e->file], dst, e->nbytes, e->off)) omc_fail(OMC_EINVAL, "read of %s failed", name);
    else n = e->nbytes;
    idx_close(&ix);
    return n;
}
