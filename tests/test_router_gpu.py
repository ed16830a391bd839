"""GPU: the exact router is bit-exact with the reference (indices AND weights).

The device computes the logits as one sequential fp32 chain per (token,
expert), the softmax with a restatement of glibc expf and the reference's
summation order, and top-k with the lower-id tie rule, so the routing is
compared with ``==`` (no tolerance).  Every test here runs with the exact
router (omc_set_router_exact(1)); the bounded router, the default from
T = 16, is checked in test_router_bounded_gpu.py."""
import ctypes as C

import numpy as np
import pytest

from gpu_common import golden, GOLDEN_NAMES, next_layer_id, olmoe_full, qwen_full

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def exact_router(gpu):
    gpu.set_router_exact(True)
    yield
    gpu.set_router_exact(False)


def test_device_expf_equals_glibc(gpu, oracle):
    # strided sweep over all float bit patterns plus a dense band of softmax arguments
    bits = np.arange(0, 1 << 32, 257, dtype=np.uint64).astype(np.uint32)
    xs = np.concatenate([bits.view(np.float32), np.linspace(-30, 0, 1 << 20, dtype=np.float32)])
    xs = np.ascontiguousarray(xs)
    ys = np.empty_like(xs)
    rc = gpu.lib().omc_debug_expf(xs.ctypes.data_as(C.c_void_p), ys.ctypes.data_as(C.c_void_p), xs.size)
    assert rc == 0, gpu.last_error()
    ref = oracle.glibc_expf(xs)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(ys), nan)
    assert np.array_equal(ys[~nan].view(np.uint32), ref[~nan].view(np.uint32))


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_routing_golden_bitexact(gpu, name):
    L, z = golden(name)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    _, idx, w = m.forward(z["x"])
    assert np.array_equal(idx, z["idx_ref"])
    assert np.array_equal(w.view(np.uint32), z["w_ref"].view(np.uint32))


@pytest.mark.parametrize("T", [1, 7, 512])
def test_routing_olmoe_full_bitexact(gpu, oracle, T):
    L = olmoe_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(9000 + T, (T, L.D))
    _, idx, w = m.forward(x)
    ridx, rw = oracle.oracle_route(L, x)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))


@pytest.mark.parametrize("T", [1, 300])
def test_routing_qwen_full_bitexact(gpu, oracle, T):
    L = qwen_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(9100 + T, (T, L.D))
    _, idx, w = m.forward(x)
    ridx, rw = oracle.oracle_route(L, x)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))


def test_int8_router_after_queued_uploads(gpu, oracle):
    """Layers built back to back: each upload leaves expert copies and
    relayouts queued on the library's stream while the next layer's int8
    router goes through the same staging buffer.  The router must be the
    layer's own (a router built from another upload's bytes routes nearly
    every token differently)."""
    L = qwen_full()
    x = oracle.normal(9150, (64, L.D))
    ridx, rw = oracle.oracle_route(L, x)
    for _ in range(3):
        m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
        _, idx, w = m.forward(x)
        assert np.array_equal(idx, ridx)
        assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))


def test_routing_ties_many(gpu, oracle):
    """Half of the router rows duplicate the other half: every token sees
    exactly tied probabilities; the reference keeps the lower expert id."""
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 64, 16, 6, seed=31)
    r = L.arrays["router"]
    r[8:] = r[:8]
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(31, (64, 256))
    _, idx, w = m.forward(x)
    ridx, rw = oracle.oracle_route(L, x)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))


@pytest.mark.parametrize("tile", [(16, 4, 4), (16, 2, 2), (16, 1, 1), (8, 1, 1)])
@pytest.mark.parametrize("kind,T", [("olmoe", 96), ("qwen", 70)])
def test_every_logits_tile_bitexact(gpu, oracle, tile, kind, T):
    """Each register tile of the logits kernel (the launch picks one by T x E)
    keeps every chain's order: routing equal to the oracle's with `==`.  T is
    a multiple of no tile, so the token tail is exercised too; Qwen adds the
    int8 router and the shared-gate row."""
    L = olmoe_full() if kind == "olmoe" else qwen_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(9500 + T, (T, L.D))
    gpu.set_router_tile(*tile)
    try:
        _, idx, w = m.forward(x)
    finally:
        gpu.set_router_tile()
    ridx, rw = oracle.oracle_route(L, x)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
