"""GPU: the engines' omm_* seam (include/om_metal.h) driven as the unmodified
OLMoE engine drives it: routing on the CPU, then one omm_moe call with one job
per expert that received positions (the batch union of
engines/olmoe.c:366-378, experts ascending, positions ascending).

The seam accumulates out[pos] += w * expert(x[pos]) job by job (the
reference's Metal backend order), so outputs match the reference forward
within the parity tolerance rather than bit for bit."""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close

pytestmark = pytest.mark.gpu


def _jobs(gpu, L, x, slots=None):
    """omm_job array for x routed by the reference; slots[e] = (g, gs, u, us, d, ds) host arrays."""
    import pyoracle as P
    a = L.arrays
    idx, w = P.oracle_route(L, x)
    S, k = idx.shape
    keep, jobs = [], []
    for e in range(L.E):
        sel = [(s, kk) for s in range(S) for kk in range(k) if idx[s, kk] == e]
        if not sel:
            continue
        pos = np.array([s for s, _ in sel], np.int32)
        ww = np.array([w[s, kk] for s, kk in sel], np.float32)
        ws = slots[e] if slots is not None else tuple(np.ascontiguousarray(a[n][e]) for n in ("g", "gs", "u", "us", "d", "ds"))
        keep += [pos, ww, *ws]
        p = lambda v: v.ctypes.data  # noqa: E731
        jobs.append(gpu.OmmJob(p(ws[0]), p(ws[2]), p(ws[4]), p(ws[1]), p(ws[3]), p(ws[5]), len(pos), p(pos), p(ww)))
    arr = (gpu.OmmJob * len(jobs))(*jobs)
    return arr, len(jobs), keep


def test_omm_init_and_alloc(gpu):
    lib = gpu.lib()
    assert lib.omm_init() == 1
    p = lib.omm_alloc(1 << 20)
    assert p


@pytest.mark.parametrize("S", [8, 40])
def test_omm_moe_matches_reference(gpu, oracle, S):
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 16, 4, seed=90)
    x = oracle.normal(91 + S, (S, 256))
    jobs, nj, keep = _jobs(gpu, L, x)
    out = np.zeros((S, 256), np.float32)
    rc = gpu.lib().omm_moe(jobs, nj, x.ctypes.data_as(C.c_void_p), S, 256, 128, out.ctypes.data_as(C.c_void_p))
    assert rc == 0, gpu.last_error()
    ref, _, _ = oracle.oracle_moe(L, x)
    assert_close(out, ref, what=f"omm_moe S={S}")


def test_omm_moe_accumulates_and_follows_slot_reuse(gpu, oracle):
    """out is accumulated into (+=), and an engine slot overwritten in place
    with another expert's weights (the LRU, engines/olmoe.c:263-270) is
    picked up on the next call."""
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 16, 4, seed=92)
    a = L.arrays
    x = oracle.normal(93, (16, 256))
    slots = {e: tuple(np.array(a[n][e]) for n in ("g", "gs", "u", "us", "d", "ds")) for e in range(L.E)}
    base = oracle.normal(94, (16, 256)) * 0.01
    out = base.copy()
    jobs, nj, keep = _jobs(gpu, L, x, slots)
    lib = gpu.lib()
    assert lib.omm_moe(jobs, nj, x.ctypes.data_as(C.c_void_p), 16, 256, 128, out.ctypes.data_as(C.c_void_p)) == 0
    ref, _, _ = oracle.oracle_moe(L, x)
    assert_close(out, base + ref, what="omm_moe accumulate")
    # the engine's slot of expert 3 now holds expert 11 (same host buffers)
    for dst, src in zip(slots[3], slots[11]):
        dst[...] = src
    L2 = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 16, 4, seed=92)
    for n in ("g", "gs", "u", "us", "d", "ds"):
        L2.arrays[n][3] = L2.arrays[n][11]
    out2 = np.zeros((16, 256), np.float32)
    jobs2, nj2, keep2 = _jobs(gpu, L, x, slots)      # routing unchanged (same router)
    assert lib.omm_moe(jobs2, nj2, x.ctypes.data_as(C.c_void_p), 16, 256, 128, out2.ctypes.data_as(C.c_void_p)) == 0
    import pyoracle as P
    idx, w = P.oracle_route(L, x)
    exp = np.zeros((16, 256), np.float32)
    for e in range(L.E):                        # job order: experts ascending
        for s in range(16):
            for kk in range(4):
                if idx[s, kk] == e:
                    y = P.oracle_expert_rows(L2, x[s:s + 1], np.array([e], np.int32))[0]
                    exp[s] = exp[s] + (w[s, kk] * y).astype(np.float32)
    assert_close(out2, exp, what="omm_moe after slot reuse")


def test_omm_moe_slot_refill_with_equal_scales(gpu, oracle):
    """A slot refilled in place with different int8 rows but bit-equal scales
    (what a pointer-and-scales identity would miss): the content hash sees
    the change and the next call uses the new rows."""
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 16, 4, seed=95)
    a = L.arrays
    x = oracle.normal(96, (16, 256))
    slots = {e: tuple(np.array(a[n][e]) for n in ("g", "gs", "u", "us", "d", "ds")) for e in range(L.E)}
    lib = gpu.lib()
    out = np.zeros((16, 256), np.float32)
    jobs, nj, keep = _jobs(gpu, L, x, slots)
    assert lib.omm_moe(jobs, nj, x.ctypes.data_as(C.c_void_p), 16, 256, 128, out.ctypes.data_as(C.c_void_p)) == 0
    # every routed expert's int8 rows negated in place, scales untouched: expert(x) changes
    for e in range(L.E):
        for i in (0, 2, 4):
            slots[e][i][...] = -np.maximum(slots[e][i], -127)
    L2 = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 16, 4, seed=95)
    for e in range(L.E):
        for i, n in ((0, "g"), (2, "u"), (4, "d")):
            L2.arrays[n][e] = slots[e][i]
    out2 = np.zeros((16, 256), np.float32)
    jobs2, nj2, keep2 = _jobs(gpu, L, x, slots)
    assert lib.omm_moe(jobs2, nj2, x.ctypes.data_as(C.c_void_p), 16, 256, 128, out2.ctypes.data_as(C.c_void_p)) == 0
    import pyoracle as P
    idx, w = P.oracle_route(L, x)
    exp = np.zeros((16, 256), np.float32)
    for e in range(L.E):
        for s_ in range(16):
            for kk in range(4):
                if idx[s_, kk] == e:
                    y = P.oracle_expert_rows(L2, x[s_:s_ + 1], np.array([e], np.int32))[0]
                    exp[s_] = exp[s_] + (w[s_, kk] * y).astype(np.float32)
    assert not np.allclose(out2, out), "the refilled rows were not used"
    assert_close(out2, exp, what="omm_moe after an equal-scales refill")


def test_omm_unsupported_shapes_fall_back(gpu):
    lib = gpu.lib()
    x = np.zeros((8, 96), np.float32)
    out = np.zeros((8, 96), np.float32)
    job = (gpu.OmmJob * 1)()
    assert lib.omm_moe_act(job, 1, x.ctypes.data_as(C.c_void_p), 8, 96, 64, out.ctypes.data_as(C.c_void_p), 0) == -3
    # D not a multiple of 64 is refused with gelu too (gelu itself is served:
    # tests/test_gemma_gpu.py::test_omm_moe_act_gelu)
    assert lib.omm_moe_act(job, 1, x.ctypes.data_as(C.c_void_p), 8, 96, 64, out.ctypes.data_as(C.c_void_p), 1) == -3
    assert lib.omm_dense(None, 64, 64, None, 8, None) == -3


# ---- dense projections (metal/om_metal.h:38-46) ------------------------------

def _dense_ref(x, W):
    return (x.astype(np.float64) @ W.astype(np.float64).T).astype(np.float32)


@pytest.mark.parametrize("S,N,K", [(8, 2048, 2048), (40, 1536, 2816), (200, 352, 704)])
def test_omm_dense_q(gpu, oracle, S, N, K):
    """omm_dense_q: out = x . dequant(Wq)^T on the tensor-core GEMM (the int8
    projections of engines/gemma.c:287-293)."""
    q, sc = oracle.quantize_py(oracle.normal(9000 + N, (N, K), 0.02))
    x = oracle.normal(9100 + S, (S, K))
    out = np.full((S, N), np.nan, np.float32)
    lib = gpu.lib()
    rc = lib.omm_dense_q(q.ctypes.data_as(C.c_void_p), sc.ctypes.data_as(C.c_void_p), N, K,
                         x.ctypes.data_as(C.c_void_p), S, out.ctypes.data_as(C.c_void_p))
    assert rc == 0, gpu.last_error()
    assert_close(out, _dense_ref(x, q.astype(np.float32) * sc[:, None]), what=f"omm_dense_q S={S} N={N} K={K}")


def test_omm_dense_q_cache_follows_scales(gpu, oracle):
    """The device copy is found again by pointer; a matrix whose scales changed
    in place is copied again (an engine reusing the buffer)."""
    N, K, S = 256, 512, 16
    q, sc = oracle.quantize_py(oracle.normal(9200, (N, K), 0.02))
    x = oracle.normal(9201, (S, K))
    lib = gpu.lib()
    out = np.zeros((S, N), np.float32)
    call = lambda: lib.omm_dense_q(q.ctypes.data_as(C.c_void_p), sc.ctypes.data_as(C.c_void_p), N, K,  # noqa: E731
                                   x.ctypes.data_as(C.c_void_p), S, out.ctypes.data_as(C.c_void_p))
    assert call() == 0
    first = out.copy()
    assert call() == 0 and np.array_equal(out, first)
    q2, sc2 = oracle.quantize_py(oracle.normal(9202, (N, K), 0.02))
    q[...] = q2
    sc[...] = sc2
    assert call() == 0
    assert_close(out, _dense_ref(x, q.astype(np.float32) * sc[:, None]), what="omm_dense_q after refill")


def test_omm_dense_q_rows_change_scales_equal(gpu, oracle):
    """The int8 rows change in place and the scales do not: copied again."""
    N, K, S = 256, 512, 16
    q, sc = oracle.quantize_py(oracle.normal(9210, (N, K), 0.02))
    x = oracle.normal(9211, (S, K))
    lib = gpu.lib()
    out = np.zeros((S, N), np.float32)
    call = lambda: lib.omm_dense_q(q.ctypes.data_as(C.c_void_p), sc.ctypes.data_as(C.c_void_p), N, K,  # noqa: E731
                                   x.ctypes.data_as(C.c_void_p), S, out.ctypes.data_as(C.c_void_p))
    assert call() == 0
    q[...] = -np.maximum(q, -127)
    assert call() == 0
    assert_close(out, _dense_ref(x, q.astype(np.float32) * sc[:, None]), what="omm_dense_q after a rows-only refill")


def test_omm_dense_q_unsupported(gpu):
    lib = gpu.lib()
    q = np.zeros((64, 96), np.int8)
    sc = np.ones(64, np.float32)
    x = np.zeros((8, 96), np.float32)
    out = np.zeros((8, 64), np.float32)
    args = lambda N, K: (q.ctypes.data_as(C.c_void_p), sc.ctypes.data_as(C.c_void_p), N, K,  # noqa: E731
                         x.ctypes.data_as(C.c_void_p), 8, out.ctypes.data_as(C.c_void_p))
    assert lib.omm_dense_q(*args(64, 96)) == -3      # K % 64
    assert lib.omm_dense_q(*args(48, 64)) == -3      # N % 32


@pytest.mark.parametrize("S,N,K", [(8, 2048, 2048), (64, 512, 1024)])
def test_omm_dense_f32(gpu, oracle, S, N, K):
    """omm_dense: the engine's f32 weights through a cached half copy (the
    attention projections of engines/olmoe.c:286-292)."""
    W = oracle.normal(9300 + N, (N, K), 0.02)
    x = oracle.normal(9301 + S, (S, K))
    out = np.zeros((S, N), np.float32)
    lib = gpu.lib()
    for _ in range(2):        # the second call uses the cached copy
        rc = lib.omm_dense(W.ctypes.data_as(C.c_void_p), N, K, x.ctypes.data_as(C.c_void_p), S,
                           out.ctypes.data_as(C.c_void_p))
        assert rc == 0, gpu.last_error()
        assert_close(out, _dense_ref(x, W), what=f"omm_dense S={S} N={N} K={K}")
