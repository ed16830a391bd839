"""GPU: greedy tokens of the OLMoE engine with its MoE layer on the GPU are
identical to the reference engine's on the CPU (random-init model).

A smaller model than the C0 configuration (2 layers, vocab 4096) keeps the
suite short; every layer has the full OLMoE-shaped MoE (D 2048, 64 experts,
top-8, I 1024).  The 32-token prompt runs the prefill through the library
(routing, dispatch, experts, combine on the GPU) and every generated token
the decode path.  Both expert paths for the prompt are checked: the default
(tensor-core grouped GEMM with f16 operands) and the CUDA-core path with f32
activations.  The full C0 run is `python tests/e2e_olmoe.py`.
"""
import os

import pytest

import e2e_olmoe as E2E

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def snapshot(tmp_path_factory):
    if not (os.path.exists(E2E.REF_ENGINE) and os.path.exists(E2E.OMC_ENGINE)):
        pytest.skip("engine builds missing (oracle/_ref/olmoe, olmoe_omc): run the build")
    d = str(tmp_path_factory.mktemp("olmoe_e2e"))
    E2E.make_snapshot(os.path.join(d, "snap"), layers=2, vocab=4096)
    return d


@pytest.mark.parametrize("path", [None, "gemv"])
def test_greedy_tokens_identical(snapshot, path):
    # the engine processes initialise the library themselves (their own slab)
    r = E2E.compare(layers=2, vocab=4096, n_prompt=32, n_new=16, path=path, workdir=snapshot)
    assert r["identical"], f"first difference at token {r['first_difference']}: {r['cpu_tokens']} vs {r['gpu_tokens']}"


def test_greedy_tokens_tiered(snapshot):
    """The hooked engine with OMC_TIER_SLOTS=16: each layer keeps 16 of its 64
    experts in HBM and copies the others in when routed (omc_tier_enable);
    the greedy tokens still equal the CPU engine's."""
    r = E2E.compare(layers=2, vocab=4096, n_prompt=32, n_new=16, path=None, workdir=snapshot,
                    env_extra={"OMC_TIER_SLOTS": "16", "OMC_TIER_DECAY": "64"})
    assert r["identical"], f"first difference at token {r['first_difference']}: {r['cpu_tokens']} vs {r['gpu_tokens']}"


def test_greedy_tokens_level1_seam(snapshot):
    """The unmodified engine built with -DOM_METAL against include/om_metal.h:
    its prefill attention projections (omm_dense, half copies of the f32
    weights, as the reference backend makes them) and MoE union (omm_moe) run
    on the GPU."""
    if not os.path.exists(E2E.METAL_ENGINE):
        pytest.skip("oracle/_ref/olmoe_metal not built")
    r = E2E.compare(layers=2, vocab=4096, n_prompt=32, n_new=16, path=None, workdir=snapshot, level=1)
    assert r["identical"], f"first difference at token {r['first_difference']}: {r['cpu_tokens']} vs {r['gpu_tokens']}"


def test_gemma_greedy_tokens_identical(tmp_path):
    """The Gemma engine (int8 container, stream mode) with its routing and
    expert union on the GPU (include/omc_gemma_hook.h) gives the CPU engine's
    greedy tokens (prefill batched, then token-by-token decode)."""
    import e2e_gemma as G
    if not (os.path.exists(G.REF_ENGINE) and os.path.exists(G.OMC_ENGINE)):
        pytest.skip("engine builds missing (oracle/_ref/gemma, gemma_omc): run the build")
    r = G.compare(layers=4, vocab=4096, n_prompt=24, n_new=16, workdir=str(tmp_path))
    assert r["identical"], f"first difference at token {r['first_difference']}: {r['cpu_tokens']} vs {r['gpu_tokens']}"


def test_qwen_tiny_int8_greedy_tokens(tmp_path):
    """The reference's tiny Qwen fixture converted by its own converter (int8
    stream mode, tests/golden/qwen_tiny_i8): the engine with moe_step on the
    GPU (include/omc_qwen_hook.h) gives the CPU engine's greedy tokens, which
    are the reference's recorded ones (oracle/ref_qwen.json)."""
    import e2e_qwen as Q
    if not (os.path.exists(Q.REF_ENGINE) and os.path.exists(Q.OMC_ENGINE)):
        pytest.skip("engine builds missing (oracle/_ref/qwen, qwen_omc): run the build")
    r = Q.compare(model="tiny", workdir=str(tmp_path))
    assert r["identical"], f"first difference at token {r['first_difference']}: {r['cpu_tokens']} vs {r['gpu_tokens']}"
    assert r["gpu_equals_reference_fixture"], (r["gpu_tokens"], r["reference_tokens"])


def test_qwen_shaped_greedy_tokens(tmp_path):
    """A random-init Qwen3.6-35B-A3B-shaped model (4 layers: three gated
    DeltaNet, one full attention; 256 experts top-8 + shared expert, int8
    container): the hooked engine's greedy tokens equal the CPU engine's."""
    import e2e_qwen as Q
    if not (os.path.exists(Q.REF_ENGINE) and os.path.exists(Q.OMC_ENGINE)):
        pytest.skip("engine builds missing (oracle/_ref/qwen, qwen_omc): run the build")
    r = Q.compare(model="shaped", layers=4, vocab=4096, n_prompt=16, n_new=16, workdir=str(tmp_path))
    assert r["identical"], f"first difference at token {r['first_difference']}: {r['cpu_tokens']} vs {r['gpu_tokens']}"
