"""GPU: omc_experts_load uploads a layer's experts straight from the int8
container (the per-expert tensors the converters write), with the same
result as uploading the arrays: forward parity against the oracle for the
OLMoE naming (gate/up/down + .qs) and Gemma's fused gate_up, and a full-size
OLMoE layer's load throughput."""
import os
import time

import numpy as np
import pytest

from conftest import assert_close
from e2e_olmoe import SafetensorsWriter
from gpu_common import next_layer_id

pytestmark = pytest.mark.gpu

OLMOE_NAMES = ("model.layers.%d.mlp.experts.%d.gate_proj.weight", "model.layers.%d.mlp.experts.%d.up_proj.weight",
               "model.layers.%d.mlp.experts.%d.down_proj.weight")
GEMMA_NAMES = ("model.layers.%d.experts.%d.gate_up_proj", None, "model.layers.%d.experts.%d.down_proj")


def write_container(path, L, layer, names, shards=2):
    """The layer's experts as container tensors, spread over `shards` files."""
    a = L.arrays
    per = []
    for e in range(L.E):
        if names[1] is None:
            per.append([(names[0] % (layer, e), np.ascontiguousarray(np.concatenate([a["g"][e], a["u"][e]]))),
                        (names[0] % (layer, e) + ".qs", np.ascontiguousarray(np.concatenate([a["gs"][e], a["us"][e]])))])
        else:
            per.append([(names[0] % (layer, e), a["g"][e]), (names[0] % (layer, e) + ".qs", a["gs"][e]),
                        (names[1] % (layer, e), a["u"][e]), (names[1] % (layer, e) + ".qs", a["us"][e])])
        per[-1] += [(names[2] % (layer, e), a["d"][e]), (names[2] % (layer, e) + ".qs", a["ds"][e])]
    os.makedirs(path, exist_ok=True)
    for sh in range(shards):
        ts = [t for e in range(sh, L.E, shards) for t in per[e]]
        wr = SafetensorsWriter(os.path.join(path, f"model-{sh:05d}.safetensors"),
                               [(n, v.dtype, v.shape) for n, v in ts])
        for n, v in ts:
            wr.put(n, np.ascontiguousarray(v))
        wr.close()


def _layer_from_router(gpu, L):
    a = L.arrays
    m = gpu.MoELayer(next_layer_id(), L.family, L.D, L.I, L.E, L.k, a["router"], a.get("router_s"), L.renorm)
    if L.family == gpu.FAMILY_GEMMA:
        m.set_gemma_norms(L.eps, a["g_rscale"], a["g_pes"], a.get("g_enorm"))
    return m


@pytest.mark.parametrize("family", ["olmoe", "gemma"])
def test_load_matches_oracle(gpu, oracle, tmp_path, family):
    if family == "olmoe":
        L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 16, 4, seed=61)
        names = OLMOE_NAMES
    else:
        L = oracle.make_layer(oracle.FAMILY_GEMMA, 256, 64, 16, 4, seed=62, router_i8=1)
        names = GEMMA_NAMES
    m = _layer_from_router(gpu, L)
    write_container(str(tmp_path), L, 3, names)
    m.load_experts(str(tmp_path), 3, names[0], names[1], names[2], 4)
    x = oracle.normal(63, (48, 256), 2.0 if family == "gemma" else 1.0)
    out, idx, _ = m.forward(x)
    ro, ridx, _ = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert_close(out, ro, what=f"{family} loaded from the container")


def test_load_refuses_missing_and_mismatched(gpu, oracle, tmp_path):
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 8, 2, seed=64)
    m = _layer_from_router(gpu, L)
    write_container(str(tmp_path), L, 0, OLMOE_NAMES)
    with pytest.raises(gpu.OmcError):          # layer 1's tensors are not there
        m.load_experts(str(tmp_path), 1, *OLMOE_NAMES)
    with pytest.raises(gpu.OmcError):          # shapes that differ from the layer: down read as gate
        m.load_experts(str(tmp_path), 0, OLMOE_NAMES[2], OLMOE_NAMES[1], OLMOE_NAMES[0])


def test_load_full_olmoe_layer_throughput(gpu, oracle, tmp_path):
    """A full OLMoE layer (64 experts x 6.3 MB) from the page cache: correct,
    and its load rate is reported."""
    L = oracle.olmoe_layer(65)
    m = _layer_from_router(gpu, L)
    write_container(str(tmp_path), L, 0, OLMOE_NAMES, shards=4)
    t0 = time.perf_counter()
    m.load_experts(str(tmp_path), 0, *OLMOE_NAMES, 8)
    dt = time.perf_counter() - t0
    nbytes = L.E * (3 * L.D * L.I + 4 * (2 * L.I + L.D))
    print(f"\nfull OLMoE layer: {nbytes / 1e6:.0f} MB in {dt * 1e3:.0f} ms = {nbytes / dt / 1e9:.2f} GB/s")
    x = oracle.normal(66, (8, L.D))
    out, idx, _ = m.forward(x)
    ro, ridx, _ = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert_close(out, ro, what="full OLMoE layer loaded from the container")
