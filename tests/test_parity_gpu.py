"""GPU: the MoE block's outputs match the reference.

* golden fixtures (outputs of the reference's own compiled moe()/moe_step()):
  routing bit-exact, outputs within max-abs 2e-2 and max|diff|/max|ref| 1e-2;
* full OLMoE- and Qwen-shaped layers against the C restatement (oracle) at
  token counts the oracle finishes in seconds;
* at the benchmark's full size (T=512 OLMoE), size-independent properties:
  determinism, token-permutation equivariance, and agreement with the
  oracle on a random subset of tokens;
* edge cases the reference handles: T=1, odd T, k=1, the tied router.

Each case runs on both expert paths (CUDA-core GEMV and tensor-core grouped
GEMM) where the shape allows.
"""
import numpy as np
import pytest

from conftest import assert_close, assert_weights
from gpu_common import golden, GOLDEN_NAMES, next_layer_id, olmoe_full, qwen_full, routing_exact

pytestmark = pytest.mark.gpu

PATHS = ["gemv", "mma"]


@pytest.fixture(params=PATHS)
def path(request, gpu):
    p = {"gemv": gpu.PATH_GEMV, "mma": gpu.PATH_MMA}[request.param]
    gpu.set_path(p)
    yield request.param
    gpu.set_path(gpu.PATH_AUTO)


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_golden_parity(gpu, path, name):
    L, z = golden(name)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    out, idx, w = m.forward(z["x"])
    assert np.array_equal(idx, z["idx_ref"])
    assert_weights(w, z["w_ref"], routing_exact(gpu, L, z["x"].shape[0]))
    assert_close(out, z["out_ref"], what=f"{name}/{path}")


@pytest.mark.parametrize("T", [1, 5, 64])
def test_olmoe_full_shape_parity(gpu, oracle, path, T):
    L = olmoe_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(7000 + T, (T, L.D))
    out, idx, w = m.forward(x)
    ro, ridx, rw = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert_close(out, ro, what=f"olmoe T={T}/{path}")


@pytest.mark.parametrize("T", [1, 5, 200])
def test_repeat_is_bit_identical(gpu, oracle, path, T):
    """Eight forwards of the same input give bit-identical outputs.  A race
    between the pipeline's producer and consumer roles shows up here first:
    at small T each CTA streams many K blocks through the rings while the
    epilogue has little to do."""
    L = olmoe_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(7300 + T, (T, L.D))
    first = m.forward(x)[0]
    for _ in range(7):
        assert np.array_equal(m.forward(x)[0].view(np.uint32), first.view(np.uint32)), "not deterministic"


@pytest.mark.parametrize("T", [1, 48])
def test_qwen_full_shape_parity(gpu, oracle, path, T):
    L = qwen_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(7100 + T, (T, L.D))
    out, idx, w = m.forward(x)
    ro, ridx, rw = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert_close(out, ro, what=f"qwen T={T}/{path}")


def test_olmoe_bench_size_properties(gpu, oracle, path):
    """T=512 (the benchmark workload): deterministic, permutation-equivariant,
    and equal to the oracle on 48 random tokens."""
    L = olmoe_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    T = 512
    x = oracle.normal(4242, (T, L.D))
    o1, i1, w1 = m.forward(x)
    o2, i2, w2 = m.forward(x)
    assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32)), "not deterministic"
    perm = np.random.default_rng(5).permutation(T)
    o3, i3, _ = m.forward(x[perm])
    assert np.array_equal(i3, i1[perm])
    assert np.array_equal(o3.view(np.uint32), o1[perm].view(np.uint32)), "not permutation-equivariant"
    sub = np.sort(np.random.default_rng(6).choice(T, 48, replace=False))
    ro, ridx, _ = oracle.oracle_moe(L, x[sub])
    assert np.array_equal(i1[sub], ridx)
    assert_close(o1[sub], ro, what=f"olmoe T=512 subset/{path}")


def test_qwen_prefill_size_subset(gpu, oracle, path):
    L = qwen_full()
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    T = 2048
    x = oracle.normal(4343, (T, L.D))
    out, idx, _ = m.forward(x)
    sub = np.sort(np.random.default_rng(7).choice(T, 24, replace=False))
    ro, ridx, _ = oracle.oracle_moe(L, x[sub])
    assert np.array_equal(idx[sub], ridx)
    assert_close(out[sub], ro, what=f"qwen T=2048 subset/{path}")


@pytest.mark.parametrize("k", [1, 2])
def test_small_k_and_odd_T(gpu, oracle, path, k):
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 16, k, seed=50 + k, renorm=1)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(60 + k, (37, 256))
    out, idx, _ = m.forward(x)
    ro, ridx, _ = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert_close(out, ro, what=f"k={k}/{path}")


def test_zero_tokens_is_noop(gpu, oracle):
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 128, 64, 8, 2, seed=70)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    out, idx, w = m.forward(np.zeros((0, 128), np.float32))
    assert out.shape == (0, 128)
