"""GPU: the GEMMA family -- route_token (engines/gemma.c:455-478) and the
expert union of step_batch (engines/gemma.c:580-685) on the device.

x is the layer's residual row.  The device derives the router input
rms(x)*router.scale*D^-0.5 and the experts' input rms(x)*
pre_feedforward_layernorm_2 (prenorm.cu), routes with the Gemma top-k
(numerators ranked, renormalised, times per_expert_scale) and runs the
experts with gelu_tanh.

Bar:
  * the norm kernel's outputs (router input, expert input, factor r) equal
    the oracle's bit for bit, including rows whose mean square sits on a
    float rounding boundary (the sequential re-sum);
  * routing indices equal the reference's (golden fixtures made by its own
    compiled route_token) and the oracle's; weights equal the oracle's bit
    for bit (correctly rounded factor) and the reference's within 32 ulps
    (its libm powf factor is 1 ulp off on ~0.06% of rows);
  * outputs within the parity tolerance of the reference (fixtures) and of
    the oracle (full Gemma-4-26B-A4B-shaped layer), on every expert path.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close
from gpu_common import GEMMA_GOLDEN, gemma_full, golden, next_layer_id

pytestmark = pytest.mark.gpu

PATHS = ["auto", "gemv", "mma", "decode"]


def _set(gpu, path):
    gpu.set_path({"auto": gpu.PATH_AUTO, "gemv": gpu.PATH_GEMV, "mma": gpu.PATH_MMA,
                  "decode": gpu.PATH_DECODE}[path])


def _ulps(a, b):
    return int(np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64)).max())


def _forward(gpu, m, x, path):
    _set(gpu, path)
    try:
        return m.forward(x)
    finally:
        gpu.set_path(gpu.PATH_AUTO)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("name", GEMMA_GOLDEN)
def test_gemma_golden(gpu, oracle, name, path):
    L, z = golden(name)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    T = z["x"].shape[0] if path != "decode" else min(8, z["x"].shape[0])
    x = np.ascontiguousarray(z["x"][:T])
    out, idx, w = _forward(gpu, m, x, path)
    assert np.array_equal(idx, z["idx_ref"][:T]), "routing differs from the reference"
    assert _ulps(w, z["w_ref"][:T]) <= 32
    oidx, ow = oracle.oracle_route(L, x)            # correctly rounded factor, as the device
    assert np.array_equal(idx, oidx)
    assert np.array_equal(w.view(np.uint32), ow.view(np.uint32))
    assert_close(out, z["out_ref"][:T], what=f"{name} {path}")


def test_prenorm_bitexact(gpu, oracle):
    L = gemma_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    rows = [oracle.normal(7000, (60, L.D), 1.0) * np.float32(s)
            for s in (1.0,)][0]
    rows[1] *= np.float32(1e-3)
    rows[2] *= np.float32(1e4)
    rows[3] = 0.0                                   # r = eps^-0.5
    # mean square exactly halfway between two floats: a = 1 + 2^-12, a*a has
    # 25 significant bits; the kernel must fall back to the index-order sum
    rows[4] = np.float32(1.0 + 2.0 ** -12)
    rows[5] = np.float32(-(1.0 + 2.0 ** -11))
    xr, xe, r = m.debug_prenorm(rows)
    oxr, oxe, orr = oracle.oracle_prenorm(L, rows)
    assert np.array_equal(r.view(np.uint32), orr.view(np.uint32))
    assert np.array_equal(xr.view(np.uint32), oxr.view(np.uint32))
    assert np.array_equal(xe.view(np.uint32), oxe.view(np.uint32))


@pytest.mark.parametrize("T,path", [(1, "auto"), (1, "gemv"), (8, "decode"), (8, "auto"), (64, "auto"),
                                    (64, "gemv"), (64, "mma"), (512, "auto")])
def test_gemma_full_shape(gpu, oracle, T, path):
    L = gemma_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(7100 + T, (T, L.D), 2.0)
    out, idx, w = _forward(gpu, m, x, path)
    ro, ridx, rw = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    assert_close(out, ro, what=f"gemma T={T} {path}")


def test_gemma_repeat_bit_identical(gpu, oracle):
    L = gemma_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    for T in (1, 256):
        x = oracle.normal(7200 + T, (T, L.D))
        first = m.forward(x)[0]
        for _ in range(4):
            assert np.array_equal(m.forward(x)[0].view(np.uint32), first.view(np.uint32))


def test_gemma_route_and_expert_rows(gpu, oracle):
    """The expert-parallel building blocks on a GEMMA layer: omc_moe_route_dev
    takes residual rows, omc_moe_experts_dev residual rows too (it applies the
    experts' input norm), y = w * expert(rows)."""
    import torch
    from gpu_common import route_dev, experts_dev
    L = gemma_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(7300, (48, L.D), 1.5)
    xd = torch.from_numpy(x).cuda()
    idx, w, _ = route_dev(m, xd)
    torch.cuda.synchronize()
    ridx, rw = oracle.oracle_route(L, x)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.array_equal(w.cpu().numpy().view(np.uint32), rw.view(np.uint32))
    rows = x[np.arange(48).repeat(2)]
    ids = np.array([e for t in range(48) for e in ridx[t, :2]], np.int32)
    wt = np.array([v for t in range(48) for v in rw[t, :2]], np.float32)
    y = experts_dev(m, torch.from_numpy(rows).cuda(), torch.from_numpy(ids).cuda(), torch.from_numpy(wt).cuda())
    torch.cuda.synchronize()
    want = oracle.oracle_expert_rows(L, rows, ids) * wt[:, None]
    assert_close(y.cpu().numpy(), want, what="gemma expert rows")


def test_gemma_noalloc(gpu, oracle):
    import torch
    L = gemma_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(7400, (16, L.D))
    xd = torch.from_numpy(x).cuda()
    out = torch.empty_like(xd)
    idx = torch.empty((16, L.k), dtype=torch.int32, device="cuda")
    w = torch.empty((16, L.k), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    gpu.check(gpu.lib().omc_moe_forward_noalloc(m.layer, C.c_void_p(xd.data_ptr()), 16, C.c_void_p(out.data_ptr()),
                                                C.c_void_p(idx.data_ptr()), C.c_void_p(w.data_ptr()),
                                                C.c_void_p(s)), "noalloc")
    torch.cuda.synchronize()
    ro, ridx, rw = oracle.oracle_moe(L, x)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert_close(out.cpu().numpy(), ro, what="gemma noalloc")


def test_gemma_norms_required(gpu, oracle):
    L = oracle.make_layer(oracle.FAMILY_GEMMA, 128, 64, 8, 2, seed=7500)
    a = L.arrays
    m = gpu.MoELayer(next_layer_id(), L.family, L.D, L.I, L.E, L.k, a["router"])
    m.set_experts_packed(a["g"], a["gs"], a["u"], a["us"], a["d"], a["ds"])
    with pytest.raises(gpu.OmcError):
        m.forward(oracle.normal(7501, (2, 128)))
    m.set_gemma_norms(L.eps, a["g_rscale"], a["g_pes"], a["g_enorm"])
    out, idx, _ = m.forward(oracle.normal(7501, (2, 128)))
    assert np.array_equal(idx, oracle.oracle_route(L, oracle.normal(7501, (2, 128)))[0])


@pytest.mark.parametrize("S", [8, 40])
def test_omm_moe_act_gelu(gpu, oracle, S):
    """engines/gemma.c:613-628: the engine routes on the CPU and hands the
    expert union to omm_moe_act(..., gelu=1) with the experts' input rows."""
    L = oracle.make_layer(oracle.FAMILY_GEMMA, 256, 128, 16, 4, seed=7600)
    a = L.arrays
    res = oracle.normal(7601 + S, (S, 256), 2.0)
    _, xe, _ = oracle.oracle_prenorm(L, res)
    idx, w = oracle.oracle_route(L, res)
    jobs, keep, want = [], [], np.zeros((S, 256), np.float32)
    for e in range(L.E):
        sel = [(s, kk) for s in range(S) for kk in range(L.k) if idx[s, kk] == e]
        if not sel:
            continue
        pos = np.array([s for s, _ in sel], np.int32)
        ww = np.array([w[s, kk] for s, kk in sel], np.float32)
        ws = tuple(np.ascontiguousarray(a[n][e]) for n in ("g", "gs", "u", "us", "d", "ds"))
        keep += [pos, ww, *ws]
        p = lambda v: v.ctypes.data  # noqa: E731
        jobs.append(gpu.OmmJob(p(ws[0]), p(ws[2]), p(ws[4]), p(ws[1]), p(ws[3]), p(ws[5]), len(pos), p(pos), p(ww)))
        y = oracle.oracle_expert_rows_act(L, xe[pos], np.full(len(pos), e, np.int32), oracle.ACT_GELU_TANH)
        for r, s in enumerate(pos):
            want[s] += ww[r] * y[r]
    arr = (gpu.OmmJob * len(jobs))(*jobs)
    out = np.zeros((S, 256), np.float32)
    rc = gpu.lib().omm_moe_act(arr, len(jobs), xe.ctypes.data_as(C.c_void_p), S, 256, 128,
                               out.ctypes.data_as(C.c_void_p), 1)
    assert rc == 0, gpu.last_error()
    ref, _, _ = oracle.oracle_moe(L, res)
    assert_close(out, want, what=f"omm_moe_act gelu S={S}")
    assert_close(out, ref, what=f"omm_moe_act gelu vs forward S={S}")
