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


def routing_exact(gpu, L, T) -> bool:
    """True when a forward of T tokens on layer L takes the exact router (its
    weights bit-equal the reference's): exact mode, T < 16, a GEMMA layer, or
    (in the default mode) fewer than 128 experts."""
    import pyoracle
    mode = gpu.router_mode()
    return (mode == gpu.ROUTER_EXACT or T < 16 or L.family == pyoracle.FAMILY_GEMMA
            or (mode == gpu.ROUTER_AUTO and L.E < 128))


def route_dev(m, xd):
    """omc_moe_route_dev on device tensor xd [T, D]: (idx, w, shared gate or None)."""
    import ctypes as C
    import torch
    import overhang_b200 as ob
    T = xd.shape[0]
    idx = torch.empty((T, m.k), dtype=torch.int32, device=xd.device)
    w = torch.empty((T, m.k), dtype=torch.float32, device=xd.device)
    sg = torch.empty(T, dtype=torch.float32, device=xd.device) if m.has_shared else None
    s = torch.cuda.current_stream(xd.device).cuda_stream
    ob.check(ob.lib().omc_moe_route_dev(m.layer, C.c_void_p(xd.data_ptr()), T, C.c_void_p(idx.data_ptr()),
                                        C.c_void_p(w.data_ptr()), C.c_void_p(sg.data_ptr() if sg is not None else None),
                                        C.c_void_p(s)), "omc_moe_route_dev")
    return idx, w, sg


def experts_dev(m, rows, ids, w):
    """omc_moe_experts_dev: y [R, D] = w[r] * expert ids[r] (rows[r]) on device tensors."""
    import ctypes as C
    import torch
    import overhang_b200 as ob
    R = rows.shape[0]
    y = torch.empty((R, m.D), dtype=torch.float32, device=rows.device)
    rows, ids, w = rows.contiguous(), ids.to(torch.int32).contiguous(), w.to(torch.float32).contiguous()
    s = torch.cuda.current_stream(rows.device).cuda_stream
    ob.check(ob.lib().omc_moe_experts_dev(m.layer, C.c_void_p(rows.data_ptr()), R, C.c_void_p(ids.data_ptr()),
                                          C.c_void_p(w.data_ptr()), C.c_void_p(y.data_ptr()), C.c_void_p(s)),
             "omc_moe_experts_dev")
    return y
