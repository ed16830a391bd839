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
