"""GPU: the fused decode forward (one cooperative launch for T <= 8).

Same bar as the other paths: routing (indices and weights) bit-exact, outputs
within the parity tolerance of the reference's golden outputs and of the
oracle, repeated forwards bit-identical.  Shapes cover the full OLMoE and
Qwen layers at every T from 1 to 8, the golden fixtures (first 8 tokens: a
token's output depends on that token alone), and padded shapes whose row
tiles do not pair up evenly.
"""
import numpy as np
import pytest

from conftest import assert_close
from gpu_common import golden, GOLDEN_NAMES, next_layer_id, olmoe_full, qwen_full

pytestmark = pytest.mark.gpu


@pytest.fixture
def decode(gpu):
    gpu.set_path(gpu.PATH_DECODE)
    yield
    gpu.set_path(gpu.PATH_AUTO)


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_golden_first_tokens(gpu, decode, name):
    L, z = golden(name)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    T = min(8, z["x"].shape[0], 64 // L.k)
    out, idx, w = m.forward(np.ascontiguousarray(z["x"][:T]))
    assert np.array_equal(idx, z["idx_ref"][:T])
    assert np.array_equal(w.view(np.uint32), z["w_ref"][:T].view(np.uint32))
    assert_close(out, z["out_ref"][:T], what=f"{name} decode")


@pytest.mark.parametrize("T", [1, 2, 3, 5, 8])
def test_olmoe_full_decode(gpu, oracle, decode, T):
    L = olmoe_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(8000 + T, (T, L.D))
    out, idx, w = m.forward(x)
    ro, ridx, rw = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    assert_close(out, ro, what=f"olmoe decode T={T}")


@pytest.mark.parametrize("T", [1, 4, 8])
def test_qwen_full_decode(gpu, oracle, decode, T):
    L = qwen_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(8100 + T, (T, L.D))
    out, idx, w = m.forward(x)
    ro, ridx, rw = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    assert_close(out, ro, what=f"qwen decode T={T}")


@pytest.mark.parametrize("T", [1, 8])
def test_decode_repeat_bit_identical(gpu, oracle, decode, T):
    """Pieces are summed in CTA order and the per-launch tag and counters
    reset themselves: sixteen back-to-back forwards agree bit for bit."""
    L = qwen_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(8200 + T, (T, L.D))
    first = m.forward(x)[0]
    for _ in range(15):
        assert np.array_equal(m.forward(x)[0].view(np.uint32), first.view(np.uint32)), "not deterministic"


def test_decode_alternates_with_other_paths(gpu, oracle):
    """Decode forwards between GEMM and GEMV forwards of other layers (the
    state is shared by every layer) stay exact."""
    Lo, Lq = olmoe_full(), qwen_full()
    mo = gpu.MoELayer.from_oracle_layer(next_layer_id(), Lo)
    mq = gpu.MoELayer.from_oracle_layer(next_layer_id(), Lq)
    x1 = oracle.normal(8300, (1, Lo.D))
    x8 = oracle.normal(8301, (64, Lq.D))
    ro, ridx, _ = oracle.oracle_moe(Lo, x1)
    for i in range(3):
        out, idx, _ = mo.forward(x1)            # auto: the fused decode at T=1
        assert np.array_equal(idx, ridx)
        assert_close(out, ro, what=f"olmoe decode, round {i}")
        mq.forward(x8)                          # auto: another path
        mq.forward(x8[:1])                      # auto: decode on the other layer


@pytest.mark.parametrize("D,I,E,k,T", [(320, 96, 24, 3, 7), (192, 160, 8, 8, 8), (256, 64, 40, 1, 1)])
def test_padded_shapes(gpu, oracle, decode, D, I, E, k, T):
    """D not a multiple of 256 (a row-tile pair with one tile), I not a
    multiple of 64, k = E (every expert), k = 1."""
    L = oracle.make_layer(oracle.FAMILY_OLMOE, D, I, E, k, seed=D + I + E, renorm=1)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(D + T, (T, D))
    out, idx, _ = m.forward(x)
    ro, ridx, _ = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert_close(out, ro, what=f"padded D={D} I={I} E={E} k={k}")


def test_qwen_padded_shared(gpu, oracle, decode):
    L = oracle.make_layer(oracle.FAMILY_QWEN, 320, 96, 16, 4, seed=77, renorm=1, router_i8=1, has_shared=1, Is=160)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(78, (6, 320))
    out, idx, _ = m.forward(x)
    ro, ridx, _ = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert_close(out, ro, what="qwen padded shared")


def test_decode_refuses_large_T(gpu, oracle, decode):
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 128, 64, 8, 2, seed=79)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    with pytest.raises(Exception):
        m.forward(oracle.normal(80, (9, 128)))


def _early_vs_waiting(gpu, m, x):
    gpu.decode_stats(reset=True)
    gpu.debug_decode_early(False)
    try:
        waited = m.forward(x)
        st_wait = gpu.decode_stats(reset=True)
    finally:
        gpu.debug_decode_early(True)
    early = m.forward(x)
    st_early = gpu.decode_stats(reset=True)
    return waited, early, st_wait, st_early


@pytest.mark.parametrize("kind", ["olmoe", "qwen"])
@pytest.mark.parametrize("T", [1, 2, 8])
def test_early_start_is_bit_identical(gpu, oracle, decode, kind, T):
    """The kernel streams as soon as the logit intervals decide every
    token's top-k set; the exact chains and the selection finish beside the
    stream and the combine takes the reference's weights and order from
    them.  So the forward equals the one that waits for the selection, bit
    for bit, and the oracle's routing."""
    L = olmoe_full() if kind == "olmoe" else qwen_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(8400 + T, (T, L.D))
    (wo, wi, ww), (eo, ei, ew), st_wait, st_early = _early_vs_waiting(gpu, m, x)
    assert st_wait == {"early": 0, "waited": 1}, st_wait
    assert st_early["early"] + st_early["waited"] == 1, st_early
    assert np.array_equal(ei, wi)
    assert np.array_equal(ew.view(np.uint32), ww.view(np.uint32))
    assert np.array_equal(eo.view(np.uint32), wo.view(np.uint32))
    ro, ridx, rw = oracle.oracle_moe(L, x)
    assert np.array_equal(ei, ridx)
    assert np.array_equal(ew.view(np.uint32), rw.view(np.uint32))
    assert_close(eo, ro, what=f"{kind} early decode T={T}")


def test_early_start_decides_most_tokens(gpu, oracle, decode):
    """Ordinary inputs: the intervals decide the set in nearly every forward."""
    L = olmoe_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    gpu.decode_stats(reset=True)
    for i in range(40):
        m.forward(oracle.normal(8500 + i, (1, L.D)))
    st = gpu.decode_stats(reset=True)
    assert st["early"] + st["waited"] == 40, st
    assert st["early"] >= 36, st


def test_tied_rows_wait_for_the_selection(gpu, oracle, decode):
    """Router rows 8.. duplicate rows 0..: every expert is tied with another,
    so whenever a tied pair straddles the k-th place the intervals cannot
    decide and the kernel waits for the exact selection (lower id first).
    Routing equals the oracle's either way."""
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 64, 16, 5, seed=41)
    r = L.arrays["router"]
    r[8:] = r[:8]
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    gpu.decode_stats(reset=True)
    for i in range(12):
        x = oracle.normal(8600 + i, (1, 256))
        out, idx, w = m.forward(x)
        ro, ridx, rw = oracle.oracle_moe(L, x)
        assert np.array_equal(idx, ridx)
        assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
        assert_close(out, ro, what=f"tied rows decode {i}")
    st = gpu.decode_stats(reset=True)
    assert st["waited"] == 12, st      # k = 5 is odd: a tied pair always straddles it
