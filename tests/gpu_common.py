"""Helpers shared by the GPU tests (layer ids, cached seeded layers)."""
import functools
import itertools
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_ids = itertools.count(100)


def next_layer_id() -> int:
    return next(_ids)


@functools.lru_cache(maxsize=None)
def olmoe_full(seed=1):
    import pyoracle
    return pyoracle.olmoe_layer(seed)


@functools.lru_cache(maxsize=None)
def qwen_full(seed=2):
    import pyoracle
    return pyoracle.qwen_layer(seed)


@functools.lru_cache(maxsize=None)
def gemma_full(seed=3):
    import pyoracle
    return pyoracle.gemma_layer(seed)


def golden(name):
    import pyoracle
    z = np.load(os.path.join(ROOT, "tests", "golden", f"golden_{name}.npz"))
    fam, D, I, E, k, renorm, r_i8, has_sh, Is = (int(v) for v in z["meta"])
    L = pyoracle.Layer(fam, D, I, E, k, renorm, r_i8, has_sh, Is)
    for n in ("router", "router_s", "g", "u", "d", "gs", "us", "ds", "sh_g", "sh_u", "sh_d",
              "sh_gs", "sh_us", "sh_ds", "sh_gate", "g_rscale", "g_pes", "g_enorm"):
        if n in z.files:
            L.arrays[n] = np.ascontiguousarray(z[n])
    if "eps" in z.files:
        L.eps = float(z["eps"][0])      # oracle in the device's (correctly rounded) mode
    return L, z


GOLDEN_NAMES = ["olmoe_small", "olmoe_renorm", "olmoe_ties", "qwen_small", "qwen_tiny_l0",
                "qwen_tiny_l3"]
GEMMA_GOLDEN = ["gemma_small", "gemma_i8", "gemma_ties", "gemma_tiny_l0", "gemma_tiny_l5"]
