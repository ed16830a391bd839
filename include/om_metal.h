/* om_metal.h -- level-1 drop-in: the engines' existing GPU seam, served by CUDA.
 *
 * The unmodified reference engines reach their GPU backend through these six
 * functions when built with -DOM_METAL (engines/olmoe.c:20-34,286-292,365-384;
 * engines/gemma.c:286-293,611-631).  Compiling them with -DOM_METAL and this
 * directory first on the include path, then linking libomc.so, runs the
 * same engine code with the MoE union on a B200 instead of Metal.
 *
 * The prototypes and the omm_job layout must equal metal/om_metal.h:14-46 so
 * the engines compile unchanged; the behaviour behind them is this library's:
 *
 *   omm_init     metal/om_metal.h:13-14   1 when a CUDA device is ready.
 *   omm_alloc    metal/om_metal.h:16-18   pinned host memory (cudaHostAlloc);
 *                                         expert slots live there, and the
 *                                         library mirrors them into HBM.
 *   omm_moe(_act) metal/om_metal.h:20-36  out[pos] += w*SwiGLU(x[pos]) per job,
 *                                         one device pass for all jobs.  Weights
 *                                         are matched to their HBM copy by slot
 *                                         pointer; a slot whose scale rows
 *                                         changed (LRU refill) is re-uploaded.
 *   omm_dense_q  metal/om_metal.h:38-41   out[S,N] = x[S,K] . dequant(Wq)^T on
 *                                         the tensor-core GEMM; the int8 matrix
 *                                         is copied to HBM once and found by
 *                                         pointer (again if its scales change);
 *                                         K % 64 or N % 32: -3, as the reference.
 *   omm_dense    metal/om_metal.h:43-46   out[S,N] = x[S,K] . W^T: a half copy
 *                                         of the f32 W made on first use (as the
 *                                         reference does), f32 accumulation
 *                                         (cuBLAS); K % 8: -3.
 *
 * Return codes follow metal/om_metal.mm: 0 ok, -1 allocation failure,
 * -2 pointer not from omm_alloc, -3 unsupported shape.
 */
#ifndef OM_METAL_H
#define OM_METAL_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

int omm_init(void);

void *omm_alloc(size_t n);

typedef struct {
    const int8_t *g, *u, *d;        /* int8 [I,D], [I,D], [D,I] from omm_alloc */
    const float  *gs, *us, *ds;     /* per-row scales from omm_alloc          */
    int mpos;                       /* positions routed to this expert        */
    const int    *pos;              /* row indices into x / out  [mpos]       */
    const float  *w;                /* router weights            [mpos]       */
} omm_job;

int omm_moe(const omm_job *jobs, int nj, const float *x, int S, int D, int I, float *out);

/* gelu: 0 = silu (olmoe/qwen), 1 = gelu_tanh (gemma) */
int omm_moe_act(const omm_job *jobs, int nj, const float *x, int S, int D, int I,
                float *out, int gelu);

int omm_dense_q(const int8_t *Wq, const float *scales, int N, int K,
                const float *x, int S, float *out);

int omm_dense(const float *W, int N, int K, const float *x, int S, float *out);

#ifdef __cplusplus
}
#endif
#endif
