"""GPU: the bounded router (the default from T = 16).

Approximate logits come from the tensor cores with a proven error interval;
the exact chain of the reference (engines/olmoe.c:74-85, engines/qwen.c:116-121)
runs only for the experts whose interval can reach the top k, plus the shared
gate; a token whose selection order could depend on the approximated rest is
retried with every row exact.  So:

* the indices equal the exact router's and the oracle's bit for bit -- at
  every size, under Zipf-skewed bias, with exactly tied router rows, with
  outlier activations;
* the weights equal the reference's within conftest.WREL (the softmax sum
  includes the approximated logits), and bit for bit when every token is
  retried whole (the retry path's own check);
* the number of exact chains stays near k + 1 per token on ordinary inputs.
"""
import numpy as np
import pytest

from conftest import assert_close, assert_weights
from gpu_common import next_layer_id, olmoe_full, qwen_full

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def bounded_router(gpu):
    """The bounded router whatever E (by default it serves E >= 128 only)."""
    gpu.set_router_mode(gpu.ROUTER_BOUNDED)
    yield
    gpu.set_router_mode(gpu.ROUTER_AUTO)


def _layer(oracle, kind):
    if kind == "olmoe":
        return olmoe_full()
    if kind == "qwen":
        return qwen_full()
    if kind == "olmoe_zipf":
        return oracle.make_layer(oracle.FAMILY_OLMOE, 2048, 1024, 64, 8, seed=1,
                                 router_bias=oracle.zipf_bias(64, 1.1, seed=21))
    return oracle.make_layer(oracle.FAMILY_QWEN, 2048, 512, 256, 8, seed=2, renorm=1, router_i8=1,
                             has_shared=1, Is=512, router_bias=oracle.zipf_bias(256, 1.1, seed=22))


def _both(gpu, m, x):
    gpu.set_router_mode(gpu.ROUTER_EXACT)
    try:
        exact = m.forward(x)
    finally:
        gpu.set_router_mode(gpu.ROUTER_BOUNDED)
    bounded = m.forward(x)
    return exact, bounded, gpu.router_stats()


@pytest.mark.parametrize("kind", ["olmoe", "qwen", "olmoe_zipf", "qwen_zipf"])
@pytest.mark.parametrize("T", [16, 100, 1000, 4096])
def test_bounded_equals_exact_and_oracle(gpu, oracle, kind, T):
    L = _layer(oracle, kind)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(12000 + T + L.E, (T, L.D))
    (eo, ei, ew), (bo, bi, bw), st = _both(gpu, m, x)
    assert np.array_equal(bi, ei), "bounded indices differ from the exact router's"
    assert_weights(bw, ew, False, "bounded vs exact weights")
    assert_close(bo, eo, what=f"{kind} T={T} bounded vs exact")
    sub = np.arange(0, T, max(1, T // 48))
    ridx, rw = oracle.oracle_route(L, x[sub])
    assert np.array_equal(bi[sub], ridx)
    assert_weights(bw[sub], rw, False, "bounded vs oracle weights")
    # cost: about k + 1 chains a token (k candidates, a few more near the
    # boundary, the shared gate, padding to groups of 4); nothing taken whole
    assert st["whole_tokens"] == 0, st
    assert st["jobs"] <= 16 * T, st
    assert st["retried_tokens"] <= max(2, T // 100), st


@pytest.mark.parametrize("kind", ["olmoe", "qwen_zipf"])
def test_forced_retry_is_bit_exact(gpu, oracle, kind):
    """Every token retried whole: the logits rows are all exact, so the weights
    equal the exact router's bit for bit."""
    L = _layer(oracle, kind)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    T = 300
    x = oracle.normal(12500, (T, L.D))
    gpu.debug_rf_force_retry(True)
    try:
        (eo, ei, ew), (bo, bi, bw), st = _both(gpu, m, x)
    finally:
        gpu.debug_rf_force_retry(False)
    assert st["retried_tokens"] == T, st
    assert np.array_equal(bi, ei)
    assert_weights(bw, ew, True, "retried weights")
    assert np.array_equal(bo.view(np.uint32), eo.view(np.uint32))


def test_tied_router_rows(gpu, oracle):
    """Half of the router rows duplicate the other half: exact ties at every
    rank, the lower id first.  Tied experts are candidates together."""
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 64, 16, 6, seed=31)
    r = L.arrays["router"]
    r[8:] = r[:8]
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(32, (200, 256))
    _, idx, w = m.forward(x)
    ridx, rw = oracle.oracle_route(L, x)
    assert np.array_equal(idx, ridx)
    assert_weights(w, rw, False)


def test_near_ties_are_retried(gpu, oracle):
    """Two router rows equal but for one element, moved by 1.5e-7: for each
    token the two logits differ by |x_17| * 1.5e-7, a few units in the last
    place of the logit or less (a change of one ulp of the weight would be
    absorbed by the chain's rounding: an exact tie).  Those near-ties are
    retried with every row exact, and the order equals the reference's."""
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 64, 16, 4, seed=33)
    r = L.arrays["router"]
    r[9] = r[2]
    r[9, 17] = np.float32(r[2, 17] + np.float32(1.5e-7))
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(34, (256, 256))
    _, idx, w = m.forward(x)
    st = gpu.router_stats()
    ridx, rw = oracle.oracle_route(L, x)
    assert np.array_equal(idx, ridx)
    assert_weights(w, rw, False)
    assert st["retried_tokens"] > 0, st


def test_outlier_tokens_are_taken_whole(gpu, oracle):
    """Tokens with an entry past the f16 range cannot be split into f16 parts:
    the routing-only entry (no f16 expert operand) takes them whole, the rest
    bounded; indices equal the oracle's, and the whole tokens' weights are
    bit-exact."""
    import torch
    from gpu_common import route_dev
    L = olmoe_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    T = 64
    x = oracle.normal(12600, (T, L.D))
    big = np.arange(0, T, 4)
    x[big, 5] = 1.0e5
    xd = torch.from_numpy(x).cuda()
    idx, w, _ = route_dev(m, xd)
    st = gpu.router_stats()                    # synchronises the library's stream
    idx, w = idx.cpu().numpy(), w.cpu().numpy()
    ridx, rw = oracle.oracle_route(L, x)
    assert np.array_equal(idx, ridx)
    assert st["whole_tokens"] == len(big), st
    assert_weights(w[big], rw[big], True, "whole tokens' weights")
    assert_weights(w, rw, False)


def test_small_models_and_shared_gate(gpu, oracle):
    """E = 8, k = 2 (the tiny converted models' shape) with a shared expert:
    the shared gate is always an exact chain."""
    L = oracle.make_layer(oracle.FAMILY_QWEN, 64, 32, 8, 2, seed=35, renorm=1, router_i8=1, has_shared=1, Is=32)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(36, (40, 64))
    (eo, ei, ew), (bo, bi, bw), st = _both(gpu, m, x)
    assert np.array_equal(bi, ei)
    assert_weights(bw, ew, False)
    assert_close(bo, eo, what="tiny qwen bounded vs exact")
    ro, ridx, rw = oracle.oracle_moe(L, x)
    assert np.array_equal(bi, ridx)
    assert_close(bo, ro, what="tiny qwen vs oracle")
