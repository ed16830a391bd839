"""GPU: parity at the sizes and load shapes the benchmarks measure.

* T = 8192 (OLMoE- and Qwen-shaped layers, both expert paths): at this size
  every expert receives ~1000 (OLMoE) or ~256 (Qwen) rows, so the grouped
  GEMM runs 128-token work items that fill both accumulator slots.  Routing
  (indices and weights) is compared with the oracle for every token, outputs
  on 64 tokens spread over the batch.
* Skewed routing through the router bias (a Zipf(1.1) preference over the
  experts, the skew of the expert-parallel benchmark): one expert is chosen by
  nearly every token, so its group is ~T rows while most others are small.
* The dispatch plan's capacity check: a forward whose rows exceed the plan's
  capacity ends with an error status (no fault), and the next forward is
  correct again.
* Activations outside the f16 operand range of the tensor-core path: the
  device entry reports OMC_ERANGE instead of clipping silently, and the host
  entry recomputes such a forward on the f32 CUDA-core path.

Routing indices are bit-exact throughout, and so are the weights of the exact
router; the bounded router's weights meet conftest.WREL.  Outputs meet max-abs 2e-2 and
max|diff|/max|ref| 1e-2 (conftest.ATOL / RTOL) except where the inputs are
scaled far past N(0, 1), where the absolute error scales with the outputs and
the absolute bar is scaled by max|ref|.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close, assert_weights, RTOL
from gpu_common import next_layer_id, olmoe_full, qwen_full, routing_exact

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["gemv", "mma"])
def path(request, gpu):
    gpu.set_path({"gemv": gpu.PATH_GEMV, "mma": gpu.PATH_MMA}[request.param])
    yield request.param
    gpu.set_path(gpu.PATH_AUTO)


@pytest.fixture(params=["bounded", "exact"])
def router(request, gpu):
    gpu.set_router_mode(gpu.ROUTER_EXACT if request.param == "exact" else gpu.ROUTER_BOUNDED)
    yield request.param
    gpu.set_router_mode(gpu.ROUTER_AUTO)


def _subset(T, n, seed):
    return np.sort(np.random.default_rng(seed).choice(T, n, replace=False))


@pytest.mark.parametrize("family", ["olmoe", "qwen"])
def test_t8192_routing_all_tokens_outputs_subset(gpu, oracle, path, router, family):
    L = olmoe_full() if family == "olmoe" else qwen_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    T = 8192
    x = oracle.normal(9100 + len(family), (T, L.D))
    out, idx, w = m.forward(x)
    ridx, rw = oracle.oracle_route(L, x)
    assert np.array_equal(idx, ridx), "routing indices differ"
    assert_weights(w, rw, router == "exact")
    # every expert is busy: the 128-token items of the grouped GEMM are exercised
    counts = np.bincount(idx.ravel(), minlength=L.E)
    assert counts.min() >= 128, counts.min()
    sub = _subset(T, 64, 9200)
    ro, _, _ = oracle.oracle_moe(L, x[sub])
    assert_close(out[sub], ro, what=f"{family} T=8192 subset/{path}")


@pytest.mark.parametrize("family", ["olmoe", "qwen"])
def test_zipf_skewed_routing(gpu, oracle, path, router, family):
    if family == "olmoe":
        L = oracle.make_layer(oracle.FAMILY_OLMOE, 2048, 1024, 64, 8, seed=1,
                              router_bias=oracle.zipf_bias(64, 1.1, seed=21))
    else:
        L = oracle.make_layer(oracle.FAMILY_QWEN, 2048, 512, 256, 8, seed=2, renorm=1, router_i8=1,
                              has_shared=1, Is=512, router_bias=oracle.zipf_bias(256, 1.1, seed=22))
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    T = 2048
    x = oracle.normal(9300 + L.E, (T, L.D))
    out, idx, w = m.forward(x)
    ridx, rw = oracle.oracle_route(L, x)
    if not np.array_equal(idx, ridx):
        # say whether a second forward of the same input repeats the result
        _, idx2, _ = m.forward(x)
        bad = np.nonzero((idx != ridx).any(axis=1))[0]
        pytest.fail(f"{len(bad)} of {T} rows differ from the oracle (first {bad[:8].tolist()}); "
                    f"a second forward equals the first: {np.array_equal(idx2, idx)}, "
                    f"equals the oracle: {np.array_equal(idx2, ridx)}")
    assert_weights(w, rw, router == "exact")
    counts = np.bincount(idx.ravel(), minlength=L.E)
    # the load is skewed: the hottest expert serves >= 90% of the tokens (a
    # uniform router gives each expert k/E of them: 1/8 for OLMoE, 1/32 for Qwen)
    assert counts.max() >= 0.9 * T, counts.max()
    sub = _subset(T, 64, 9400)
    ro, _, _ = oracle.oracle_moe(L, x[sub])
    assert_close(out[sub], ro, what=f"{family} zipf/{path}")
    # the same layer without the bias routes differently, and the library follows
    m.set_router_bias(None)
    out2, idx2, _ = m.forward(x[sub])
    L.arrays.pop("router_bias")
    ro2, ridx2, _ = oracle.oracle_moe(L, x[sub])
    assert np.array_equal(idx2, ridx2)
    assert not np.array_equal(idx2, idx[sub])
    assert_close(out2, ro2, what=f"{family} bias removed/{path}")


def test_router_bias_decode_and_ties(gpu, oracle):
    """The fused decode kernel adds the bias too; a bias that makes two
    experts tie exactly keeps the lower id first."""
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 16, 4, seed=81)
    x = oracle.normal(82, (4, 256))
    # experts 3 and 9 get the same router row and the same (large) bias: their
    # biased logits are equal for every token, so they tie at the top
    L.arrays["router"][9] = L.arrays["router"][3]
    bias = np.zeros(16, np.float32)
    bias[3] = bias[9] = 4.0
    L.arrays["router_bias"] = bias
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    for p in (gpu.PATH_DECODE, gpu.PATH_GEMV, gpu.PATH_MMA):
        gpu.set_path(p)
        try:
            for T in (1, 4):
                out, idx, w = m.forward(x[:T])
                ro, ridx, rw = oracle.oracle_moe(L, x[:T])
                assert np.array_equal(idx, ridx), (p, T)
                assert (idx[:, 0] == 3).all() and (idx[:, 1] == 9).all()
                assert np.array_equal(w.view(np.uint32), rw.view(np.uint32)), (p, T)
                assert_close(out, ro, what=f"bias path {p} T={T}")
        finally:
            gpu.set_path(gpu.PATH_AUTO)


def test_router_bias_rejects_non_finite(gpu, oracle):
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 128, 64, 8, 2, seed=83)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    b = np.zeros(8, np.float32)
    b[5] = np.inf
    with pytest.raises(gpu.OmcError) as e:
        m.set_router_bias(b)
    assert e.value.status == gpu.EINVAL


def test_plan_capacity_overflow_reports_error(gpu, oracle):
    L = olmoe_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(9500, (48, L.D))
    gpu.set_path(gpu.PATH_MMA)
    try:
        gpu.lib().omc_debug_plan_rows(64)          # 48 tokens x 8 slots need >= 384 rows
        with pytest.raises(gpu.OmcError) as e:
            m.forward(x)
        assert e.value.status == gpu.EDEVICE
        assert "site 21" in gpu.last_error()        # OMC_SITE_DISPATCH: the plan's check
    finally:
        gpu.lib().omc_debug_plan_rows(0)
        gpu.set_path(gpu.PATH_AUTO)
    gpu.set_path(gpu.PATH_MMA)
    try:
        out, idx, _ = m.forward(x)
    finally:
        gpu.set_path(gpu.PATH_AUTO)
    ro, ridx, _ = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert_close(out, ro, what="after the overflow")


def _outliers(oracle, T, D, scale, seed):
    """x ~ N(0,1) with one large entry per token (|x| = scale): the rows a
    model with massive activations feeds its MoE layer."""
    x = oracle.normal(seed, (T, D))
    rng = np.random.default_rng(seed)
    cols = rng.integers(0, D, T)
    x[np.arange(T), cols] = scale * np.where(rng.random(T) < 0.5, -1.0, 1.0)
    return x.astype(np.float32)


def test_large_activations_within_f16_range(gpu, oracle, path):
    """Outliers of 1000 (h stays inside the f16 range): the tensor-core path
    keeps its operands and stays within the relative bar."""
    L = olmoe_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = _outliers(oracle, 64, L.D, 1000.0, 9600)
    out, idx, w = m.forward(x)
    ro, ridx, rw = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert_weights(w, rw, routing_exact(gpu, L, 64))
    assert_close(out, ro, atol=2e-2 * max(1.0, float(np.abs(ro).max())), rtol=RTOL, what=f"outliers 1e3/{path}")


def test_activations_past_f16_range(gpu, oracle):
    """Outliers of 1e5: past the f16 range.  The device entry on the
    tensor-core path reports OMC_ERANGE; the host entry returns the f32
    CUDA-core result, which matches the oracle."""
    import torch
    L = olmoe_full()
    lid = next_layer_id()
    m = gpu.MoELayer.from_oracle_layer(lid, L)
    T = 64
    x = _outliers(oracle, T, L.D, 1.0e5, 9700)
    ro, ridx, rw = oracle.oracle_moe(L, x)
    gpu.set_path(gpu.PATH_MMA)
    try:
        xd = torch.from_numpy(x).cuda()
        od = torch.empty_like(xd)
        torch.cuda.synchronize()
        rc = gpu.lib().omc_moe_forward_dev(lid, C.c_void_p(xd.data_ptr()), T, C.c_void_p(od.data_ptr()), None, None,
                                           None)
        assert rc == 0, gpu.last_error()
        assert gpu.lib().omc_sync() == gpu.ERANGE
        out, idx, w = m.forward(x)                 # host entry: recomputed on the f32 path
    finally:
        gpu.set_path(gpu.PATH_AUTO)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    assert_close(out, ro, atol=2e-2 * max(1.0, float(np.abs(ro).max())), rtol=RTOL, what="outliers 1e5")
    # the next forward of ordinary rows is back on the tensor-core path, unaffected
    x2 = oracle.normal(9800, (64, L.D))
    out2, idx2, _ = m.forward(x2)
    ro2, ridx2, _ = oracle.oracle_moe(L, x2)
    assert np.array_equal(idx2, ridx2)
    assert_close(out2, ro2, what="after the range fallback")
