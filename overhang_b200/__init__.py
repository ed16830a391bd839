"""overhang_b200 -- B200-native MoE block for the overhang engines.

The product is the C-ABI library ``libomc.so`` (include/om_cuda.h, and the
engines' own GPU seam include/om_metal.h).  This module is its Python face:
ctypes prototypes plus a small ``MoELayer`` wrapper mirroring the engines'
per-layer MoE call (``moe()`` in engines/olmoe.c:344, ``moe_step()`` in
engines/qwen.c:453).  There is no Python or CPU fallback: if the library is
missing or a call fails, an ``OmcError`` is raised.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libomc.so")

FAMILY_OLMOE, FAMILY_QWEN, FAMILY_GEMMA = 0, 1, 2
ROUTER_F32, ROUTER_I8 = 0, 1

OK, EINVAL, ENOMEM, ENOINIT, ECUDA, EDEVICE, ETIMEOUT, ENCCL, EUNSUPPORTED, ERANGE = 0, -1, -2, -3, -4, -5, -6, -7, -8, -9


class OmcError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


class MoEDesc(C.Structure):
    """omc_moe_desc (include/om_cuda.h)."""
    _fields_ = [(n, C.c_int) for n in
                ("family", "D", "I", "E", "k", "renorm", "router_dtype", "has_shared", "Is")]


class OmmJob(C.Structure):
    """omm_job (include/om_metal.h; same layout as metal/om_metal.h:21-27)."""
    _fields_ = [("g", C.c_void_p), ("u", C.c_void_p), ("d", C.c_void_p),
                ("gs", C.c_void_p), ("us", C.c_void_p), ("ds", C.c_void_p),
                ("mpos", C.c_int), ("pos", C.c_void_p), ("w", C.c_void_p)]


# every symbol include/*.h declares, with its ctypes signature
_vp, _i, _sz = C.c_void_p, C.c_int, C.c_size_t
SIGNATURES = {
    "omc_init": (_i, [_i, _sz]),
    "omc_shutdown": (None, []),
    "omc_layer_init": (_i, [_i, C.POINTER(MoEDesc), _vp, _vp]),
    "omc_layer_gemma_norms": (_i, [_i, C.c_float, _vp, _vp, _vp]),
    "omc_layer_router_bias": (_i, [_i, _vp]),
    "omc_expert_set": (_i, [_i, _i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "omc_experts_set_packed": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "omc_experts_load": (_i, [_i, C.c_char_p, _i, C.c_char_p, C.c_char_p, C.c_char_p, _i]),
    "omc_shared_set": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "omc_tier_enable": (_i, [_i, _i, _i, _i]),
    "omc_tier_step": (_i, [_i, _vp]),
    "omc_tier_stats": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "omc_tier_pick": (_i, [_vp, _vp, C.c_uint32, _i, _vp, _i, _vp, _vp, _vp]),
    "omc_moe_forward": (_i, [_i, _vp, _i, _vp, _vp, _vp]),
    "omc_moe_forward_dev": (_i, [_i, _vp, _i, _vp, _vp, _vp, _vp]),
    "omc_moe_forward_async": (_i, [_i, _vp, _i, _vp, _vp, _vp, C.POINTER(C.c_longlong)]),
    "omc_moe_wait": (_i, [C.c_longlong]),
    "omc_moe_forward_noalloc": (_i, [_i, _vp, _i, _vp, _vp, _vp, _vp]),
    "omc_moe_route_dev": (_i, [_i, _vp, _i, _vp, _vp, _vp, _vp]),
    "omc_moe_experts_dev": (_i, [_i, _vp, _i, _vp, _vp, _vp, _vp]),
    "omc_sync": (_i, []),
    "omc_ep_init": (_i, [_i, _i, _vp]),
    "omc_ep_unique_id": (_i, [_vp, _sz]),
    "omc_ep_set_timeout": (_i, [_i]),
    "omc_ep_set_combine": (_i, [_i]),
    "omc_ep_wait": (_i, []),
    "omc_ep_layout_host": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "omc_ep_unpack_host": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "omc_strerror": (C.c_char_p, [_i]),
    "omc_last_error": (C.c_char_p, []),
    "omc_set_profiling": (_i, [_i]),
    "omc_stage_times": (_i, [C.POINTER(C.c_float), _i]),
    "omc_stage_name": (C.c_char_p, [_i]),
    "omc_time_stage": (_i, [C.c_char_p]),
    "omc_stage_timer": (_i, [C.POINTER(C.c_float), C.POINTER(_i)]),
    "omc_launch_count": (C.c_longlong, [_i]),
    "omc_version": (C.c_char_p, []),
    "omc_set_router_exact": (_i, [_i]),
    "omc_router_stats": (_i, [C.POINTER(_i)]),
    "omm_init": (_i, []),
    "omm_alloc": (_vp, [_sz]),
    "omm_moe": (_i, [C.POINTER(OmmJob), _i, _vp, _i, _i, _i, _vp]),
    "omm_moe_act": (_i, [C.POINTER(OmmJob), _i, _vp, _i, _i, _i, _vp, _i]),
    "omm_dense_q": (_i, [_vp, _vp, _i, _i, _vp, _i, _vp]),
    "omm_dense": (_i, [_vp, _i, _i, _vp, _i, _vp]),
    # not in the public headers: failure-detection test hook
    "omc_debug_wait_timeout": (_i, []),
    "omc_debug_expf": (_i, [_vp, _vp, C.c_longlong]),
    "omc_debug_set_path": (_i, [_i]),
    "omc_debug_plan_rows": (_i, [_i]),
    "omc_debug_router_tile": (_i, [_i, _i, _i]),
    "omc_debug_rf_force_retry": (_i, [_i]),
    "omc_decode_stats": (_i, [C.POINTER(_i), _i]),
    "omc_debug_decode_early": (_i, [_i]),
    "omc_debug_ws_copy": (_i, [_i, _vp, _sz]),
    "omc_debug_gemma_prenorm": (_i, [_i, _vp, _i, _vp, _vp, _vp]),
    "omc_debug_container_read": (C.c_longlong, [C.c_char_p, C.c_char_p, _vp, C.c_longlong]),
}

PATH_AUTO, PATH_GEMV, PATH_MMA, PATH_DECODE = 0, 1, 2, 3


def set_path(path: int) -> None:
    """Force the expert path (tests): PATH_AUTO, PATH_GEMV, PATH_MMA or PATH_DECODE
    (the fused decode forward, T <= 8)."""
    check(lib().omc_debug_set_path(path), "omc_debug_set_path")


ROUTER_TILES = [(16, 4, 4), (16, 2, 2), (16, 1, 1), (8, 1, 1)]


def set_router_tile(g: int = 0, tt: int = 0, rr: int = 0) -> None:
    """Force the router logits tile (tests): one of ROUTER_TILES, or 0,0,0 = automatic."""
    check(lib().omc_debug_router_tile(g, tt, rr), "omc_debug_router_tile")

ROUTER_AUTO, ROUTER_EXACT, ROUTER_BOUNDED = 0, 1, 2
_router_mode = ROUTER_AUTO


def set_router_mode(mode: int) -> None:
    """Router of the forwards with T >= 16: ROUTER_AUTO (the default: the
    bounded router -- indices bit-exact, weights within a few ulps of the
    reference's -- for layers of >= 128 experts, the exact one below),
    ROUTER_EXACT (the exact chain for every (token, expert): weights bit-exact
    too) or ROUTER_BOUNDED (the bounded router whatever E)."""
    global _router_mode
    check(lib().omc_set_router_exact(mode), "omc_set_router_exact")
    _router_mode = mode


def set_router_exact(on: bool) -> None:
    set_router_mode(ROUTER_EXACT if on else ROUTER_AUTO)


def router_mode() -> int:
    return _router_mode


def router_exact() -> bool:
    return _router_mode == ROUTER_EXACT


def router_stats() -> dict:
    """Counters of the last bounded-router pass (synchronises the library's stream)."""
    out = (C.c_int * 4)()
    check(lib().omc_router_stats(out), "omc_router_stats")
    return {"jobs": out[0], "retry_jobs": out[1], "whole_tokens": out[2], "retried_tokens": out[3]}


def debug_rf_force_retry(on: bool) -> None:
    """Test hook: every token of a bounded pass is retried with every row exact."""
    check(lib().omc_debug_rf_force_retry(1 if on else 0), "omc_debug_rf_force_retry")


def decode_stats(reset: bool = False) -> dict:
    """Fused decode forwards whose top-k sets the logit intervals decided
    ("early") and forwards that waited for the exact selection ("waited")."""
    out = (C.c_int * 2)()
    check(lib().omc_decode_stats(out, 1 if reset else 0), "omc_decode_stats")
    return {"early": out[0], "waited": out[1]}


def debug_decode_early(on: bool) -> None:
    """Test hook: False = the fused decode waits for the exact selection
    before streaming (the output is the same bit for bit)."""
    check(lib().omc_debug_decode_early(1 if on else 0), "omc_debug_decode_early")


_lib = None


def lib() -> C.CDLL:
    """Load the in-tree libomc.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OmcError(ENOINIT, f"{LIB_PATH} missing: run `python -m overhang_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().omc_last_error().decode()


def check(rc: int, what: str) -> None:
    if rc != OK:
        raise OmcError(rc, f"{what}: {lib().omc_strerror(rc).decode()}: {last_error()}")


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def tier_pick(heat, last, clock: int, pinned):
    """The library's hot-store replacement rule (omc_tier_pick, no device
    needed): (slot, expert, gain) of the swap it would make, or None."""
    heat, last = np.ascontiguousarray(heat, np.uint32), np.ascontiguousarray(last, np.uint32)
    pinned = np.ascontiguousarray(pinned, np.int32)
    s, e, g = C.c_int(-1), C.c_int(-1), C.c_long(0)
    rc = lib().omc_tier_pick(_p(heat), _p(last), clock & 0xFFFFFFFF, heat.size, _p(pinned), pinned.size,
                             C.byref(s), C.byref(e), C.byref(g))
    return (s.value, e.value, g.value) if rc else None


def init(device: int = 0, slab_bytes: int = 0) -> None:
    check(lib().omc_init(device, slab_bytes), "omc_init")


def shutdown() -> None:
    lib().omc_shutdown()


def sync() -> None:
    check(lib().omc_sync(), "omc_sync")


def launch_count(reset: bool = False) -> int:
    return int(lib().omc_launch_count(1 if reset else 0))


def stage_times(n: int = 12):
    """[(stage name, ms)] of the last forward run with profiling on."""
    buf = (C.c_float * n)()
    k = lib().omc_stage_times(buf, n)
    return [(lib().omc_stage_name(i).decode(), buf[i]) for i in range(k)]


def set_profiling(on: bool) -> None:
    lib().omc_set_profiling(1 if on else 0)


def ep_unique_id() -> bytes:
    """A new NCCL unique id (128 bytes) for ep_init, made on rank 0."""
    buf = C.create_string_buffer(128)
    check(lib().omc_ep_unique_id(buf, 128), "omc_ep_unique_id")
    return buf.raw


def ep_init(rank: int, world: int, unique_id: bytes = None) -> None:
    """Hold routed experts [rank*E/world, (rank+1)*E/world) of every layer
    created afterwards; with unique_id (ep_unique_id() of rank 0) the ranks
    join one NCCL group and every forward runs expert-parallel."""
    uid = None if unique_id is None else C.create_string_buffer(bytes(unique_id), 128)
    check(lib().omc_ep_init(rank, world, uid), "omc_ep_init")


EP_EXACT, EP_RANKSUM = 0, 1


def ep_set_combine(mode: int) -> None:
    """EP_EXACT (bit-equal to one GPU) or EP_RANKSUM (one row per token and rank back)."""
    check(lib().omc_ep_set_combine(mode), "omc_ep_set_combine")


def ep_set_timeout(ms: int) -> None:
    check(lib().omc_ep_set_timeout(ms), "omc_ep_set_timeout")


def time_stage(name) -> None:
    """Time stage `name` ("gemm_gateup", ...) in every following forward with
    one CUDA-event pair on its stream; None stops."""
    check(lib().omc_time_stage(None if name is None else name.encode()), "omc_time_stage")


def stage_timer():
    """(mean ms, forwards averaged) of the stage given to time_stage."""
    ms, n = C.c_float(0.0), C.c_int(0)
    check(lib().omc_stage_timer(C.byref(ms), C.byref(n)), "omc_stage_timer")
    return float(ms.value), int(n.value)


class MoELayer:
    """One MoE layer resident on the GPU.

    ``forward(x)`` is the drop-in for the engines' per-layer MoE call: x is
    the post-norm activation [T, D] f32, the result is out [T, D] f32 plus the
    routing (topk_idx [T, k] int32, topk_w [T, k] f32) in selection order.
    """

    def __init__(self, layer: int, family: int, D: int, I: int, E: int, k: int, router,
                 router_s=None, renorm: int = 0, has_shared: int = 0, Is: int = 0):
        self.layer = layer
        r_i8 = router.dtype == np.int8
        self.desc = MoEDesc(family, D, I, E, k, renorm, ROUTER_I8 if r_i8 else ROUTER_F32,
                            has_shared, Is)
        self._keep = [np.ascontiguousarray(router)]
        rs = None if router_s is None else np.ascontiguousarray(router_s, np.float32)
        check(lib().omc_layer_init(layer, C.byref(self.desc), _p(self._keep[0]), _p(rs)),
              "omc_layer_init")

    D = property(lambda self: self.desc.D)
    E = property(lambda self: self.desc.E)
    k = property(lambda self: self.desc.k)
    has_shared = property(lambda self: self.desc.has_shared)

    @classmethod
    def from_oracle_layer(cls, layer: int, L, tier=None) -> "MoELayer":
        """Upload a seeded layer built by oracle.pyoracle.make_layer (tests/bench).
        tier = (hbm_slots, interval, decay_every): a tiered layer (omc_tier_enable)."""
        a = L.arrays
        m = cls(layer, L.family, L.D, L.I, L.E, L.k, a["router"], a.get("router_s"),
                L.renorm, L.has_shared, L.Is)
        if tier is not None:
            m.tier_enable(*tier)
        if L.family == FAMILY_GEMMA:
            m.set_gemma_norms(L.eps, a["g_rscale"], a["g_pes"], a.get("g_enorm"))
        if a.get("router_bias") is not None:
            m.set_router_bias(a["router_bias"])
        m.set_experts_packed(a["g"], a["gs"], a["u"], a["us"], a["d"], a["ds"])
        if L.has_shared:
            m.set_shared(a["sh_g"], a["sh_gs"], a["sh_u"], a["sh_us"], a["sh_d"], a["sh_ds"],
                         a["sh_gate"])
        return m

    def set_gemma_norms(self, eps: float, router_scale, per_expert_scale, expert_norm=None) -> None:
        """GEMMA: router.scale [D], per_expert_scale [E], pre_feedforward_layernorm_2 [D]."""
        arrs = [None if v is None else np.ascontiguousarray(v, np.float32)
                for v in (router_scale, per_expert_scale, expert_norm)]
        self._keep += [v for v in arrs if v is not None]
        check(lib().omc_layer_gemma_norms(self.layer, float(eps), *[_p(v) for v in arrs]),
              "omc_layer_gemma_norms")

    def set_router_bias(self, bias) -> None:
        """bias [E] added to every router logit before the softmax (None removes it)."""
        b = None if bias is None else np.ascontiguousarray(bias, np.float32).reshape(self.desc.E)
        if b is not None:
            self._keep.append(b)
        check(lib().omc_layer_router_bias(self.layer, _p(b)), "omc_layer_router_bias")

    def debug_prenorm(self, x: np.ndarray):
        """GEMMA: (router input, expert input, norm factor) from the device kernel."""
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        xr = np.empty((T, self.desc.D), np.float32)
        xe = np.empty((T, self.desc.D), np.float32)
        r = np.empty(T, np.float32)
        check(lib().omc_debug_gemma_prenorm(self.layer, _p(x), T, _p(xr), _p(xe), _p(r)),
              "omc_debug_gemma_prenorm")
        return xr, xe, r

    def tier_enable(self, hbm_slots: int, interval: int = 1, decay_every: int = 0) -> None:
        """Tiered expert store: hbm_slots experts in HBM, the rest read from
        pinned host memory; LFRU swaps every `interval` forwards."""
        check(lib().omc_tier_enable(self.layer, hbm_slots, interval, decay_every), "omc_tier_enable")

    def tier_step(self) -> int:
        """Apply at most one swap now; the expert moved into HBM, or -1."""
        e = C.c_int(-1)
        check(lib().omc_tier_step(self.layer, C.byref(e)), "omc_tier_step")
        return e.value

    def tier_stats(self, hbm_slots: int):
        """(heat [E], last [E], clock, expert per HBM slot, swaps, misses)."""
        E = self.desc.E
        heat, last = np.empty(E, np.uint32), np.empty(E, np.uint32)
        clock, swaps, misses = C.c_uint32(0), C.c_longlong(0), C.c_longlong(0)
        slots = np.empty(hbm_slots, np.int32)
        check(lib().omc_tier_stats(self.layer, _p(heat), _p(last), C.byref(clock), _p(slots), C.byref(swaps),
                                   C.byref(misses)), "omc_tier_stats")
        return heat, last, clock.value, slots, swaps.value, misses.value

    def load_experts(self, snapshot: str, src_layer: int, name_g: str, name_u, name_d: str,
                     nthreads: int = 0) -> None:
        """Upload this layer's experts from an int8 container directory
        (omc_experts_load): printf name patterns taking (src_layer, expert);
        name_u None = name_g is the fused gate_up."""
        check(lib().omc_experts_load(self.layer, snapshot.encode(), src_layer, name_g.encode(),
                                     None if name_u is None else name_u.encode(), name_d.encode(), nthreads),
              "omc_experts_load")

    def set_experts_packed(self, g, gs, u, us, d, ds) -> None:
        arrs = [np.ascontiguousarray(v) for v in (g, gs, u, us, d, ds)]
        check(lib().omc_experts_set_packed(self.layer, *[_p(v) for v in arrs]),
              "omc_experts_set_packed")

    def set_expert(self, e: int, g, gs, u, us, d, ds) -> None:
        arrs = [np.ascontiguousarray(v) for v in (g, gs, u, us, d, ds)]
        check(lib().omc_expert_set(self.layer, e, *[_p(v) for v in arrs]), "omc_expert_set")

    def set_shared(self, g, gs, u, us, d, ds, sh_gate) -> None:
        arrs = [np.ascontiguousarray(v) for v in (g, gs, u, us, d, ds, sh_gate)]
        check(lib().omc_shared_set(self.layer, *[_p(v) for v in arrs]), "omc_shared_set")

    def forward(self, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        out = np.empty((T, self.desc.D), np.float32)
        idx = np.empty((T, self.desc.k), np.int32)
        w = np.empty((T, self.desc.k), np.float32)
        check(lib().omc_moe_forward(self.layer, _p(x), T, _p(out), _p(idx), _p(w)),
              "omc_moe_forward")
        return out, idx, w

    def forward_dev(self, x_ptr: int, T: int, out_ptr: int, idx_ptr: int = 0, w_ptr: int = 0,
                    stream: int = 0) -> None:
        check(lib().omc_moe_forward_dev(self.layer, C.c_void_p(x_ptr), T, C.c_void_p(out_ptr),
                                        C.c_void_p(idx_ptr or None), C.c_void_p(w_ptr or None),
                                        C.c_void_p(stream or None)),
              "omc_moe_forward_dev")
