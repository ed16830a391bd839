"""ctypes access to the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and the cpu_baseline / reference leg
of ``bench.py`` import this module, and only as the checker or the timed CPU
baseline.  The product library (``overhang_b200/libomc.so``) never loads it.

Two checkers live here:

* ``liboracle.so``: the C restatement in ``moe_oracle.c`` (always built);
* ``_ref/libref_olmoe.so`` / ``_ref/libref_qwen.so`` / ``_ref/libref_gemma.so``:
  the reference engines' own ``moe()`` (engines/olmoe.c:344-402),
  ``moe_step()`` (engines/qwen.c:453-495) and ``route_token()`` with the
  expert union (engines/gemma.c:455-478, :580-685), compiled from the
  reference sources by ``oracle/Makefile`` (present wherever they were built
  and shipped).

It also generates the seeded synthetic layers used by tests and bench: weights
N(0, 0.02) through the converters' per-row int8 rule
(tools/convert_olmoe.py:32-38), activations N(0, 1).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
FAMILY_OLMOE, FAMILY_QWEN, FAMILY_GEMMA = 0, 1, 2
RSQRT_CR, RSQRT_LIBM = 0, 1

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


class OrcDesc(C.Structure):
    _fields_ = [(n, C.c_int) for n in
                ("family", "D", "I", "E", "k", "renorm", "router_i8", "has_shared", "Is")] + \
               [("eps", C.c_float), ("rsqrt_mode", C.c_int)]


class OrcWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in
                ("router", "router_s", "g", "u", "d", "gs", "us", "ds",
                 "sh_g", "sh_u", "sh_d", "sh_gs", "sh_us", "sh_ds", "sh_gate",
                 "g_rscale", "g_pes", "g_enorm", "router_bias")]


_lib = None
_ref = {}


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"oracle not built: {path} (run make -C oracle)")
        L = C.CDLL(path)
        L.orc_moe.restype = C.c_int
        L.orc_moe.argtypes = [C.POINTER(OrcDesc), C.POINTER(OrcWeights), _f32p, C.c_int,
                              _f32p, C.c_void_p, C.c_void_p]
        L.orc_route.restype = C.c_int
        L.orc_route.argtypes = [C.POINTER(OrcDesc), C.POINTER(OrcWeights), _f32p, C.c_int,
                                C.c_void_p, C.c_void_p]
        L.orc_shared_gate.restype = C.c_int
        L.orc_shared_gate.argtypes = [C.POINTER(OrcDesc), C.POINTER(OrcWeights), _f32p, C.c_int, _f32p]
        L.orc_expert_rows.restype = C.c_int
        L.orc_expert_rows.argtypes = [C.POINTER(OrcDesc), C.POINTER(OrcWeights), _f32p, C.c_int,
                                      C.c_void_p, _f32p]
        L.orc_expert_rows_act.restype = C.c_int
        L.orc_expert_rows_act.argtypes = [C.POINTER(OrcDesc), C.POINTER(OrcWeights), _f32p, C.c_int,
                                          C.c_void_p, C.c_int, _f32p]
        L.orc_gemma_prenorm.restype = C.c_int
        L.orc_gemma_prenorm.argtypes = [C.POINTER(OrcDesc), C.POINTER(OrcWeights), _f32p, C.c_int,
                                        _f32p, _f32p, _f32p]
        L.orc_quantize_rows_py.argtypes = [_f32p, C.c_int, C.c_int, _i8p, _f32p]
        L.orc_quantize_rows_c.argtypes = [_f32p, C.c_int, C.c_int, _i8p, _f32p]
        L.orc_fill_normal.argtypes = [C.c_uint64, _f32p, C.c_int64, C.c_float]
        L.orc_expf.restype = C.c_float
        L.orc_expf.argtypes = [C.c_float]
        L.orc_expf_array.argtypes = [_f32p, _f32p, C.c_int64]
        _lib = L
    return _lib


def ref_root():
    """The reference sources (for fixture generation and harness builds):
    $REF_ROOT, or a directory named `reference` beside this repository; None
    when neither holds engines/olmoe.c."""
    cands = [os.environ.get("REF_ROOT"), os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")]
    for c in cands:
        if c and os.path.exists(os.path.join(c, "engines", "olmoe.c")):
            return os.path.abspath(c)
    return None


def ref_lib(name: str):
    """The compiled reference (``olmoe``, ``qwen`` or ``gemma``), or None if not built."""
    if name not in _ref:
        path = os.path.join(HERE, "_ref", f"libref_{name}.so")
        _ref[name] = C.CDLL(path) if os.path.exists(path) else None
    return _ref[name]


def ref_available() -> bool:
    return ref_lib("olmoe") is not None and ref_lib("qwen") is not None and ref_lib("gemma") is not None


def normal(seed: int, shape, sigma: float = 1.0) -> np.ndarray:
    a = np.empty(int(np.prod(shape)), np.float32)
    lib().orc_fill_normal(seed & 0xFFFFFFFFFFFFFFFF, a, a.size, sigma)
    return a.reshape(shape)


def glibc_expf(x: np.ndarray) -> np.ndarray:
    """The host's glibc expf, elementwise (what the reference's softmax calls)."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_expf_array(x.ravel(), y.ravel(), x.size)
    return y


def quantize_py(w: np.ndarray):
    w = np.ascontiguousarray(w, np.float32)
    O, I = w.shape
    q = np.empty((O, I), np.int8)
    s = np.empty(O, np.float32)
    lib().orc_quantize_rows_py(w, O, I, q, s)
    return q, s


def quantize_c(w: np.ndarray):
    w = np.ascontiguousarray(w, np.float32)
    O, I = w.shape
    q = np.empty((O, I), np.int8)
    s = np.empty(O, np.float32)
    lib().orc_quantize_rows_c(w, O, I, q, s)
    return q, s


@dataclass
class Layer:
    """One seeded MoE layer in the packed expert-major layout."""
    family: int
    D: int
    I: int
    E: int
    k: int
    renorm: int = 0
    router_i8: int = 0
    has_shared: int = 0
    Is: int = 0
    arrays: dict = field(default_factory=dict)
    eps: float = 1e-6          # gemma: rms_norm_eps
    rsqrt_mode: int = RSQRT_CR  # gemma: RSQRT_CR (the device's value) or RSQRT_LIBM (powf)

    def desc(self) -> OrcDesc:
        return OrcDesc(self.family, self.D, self.I, self.E, self.k, self.renorm,
                       self.router_i8, self.has_shared, self.Is, self.eps, self.rsqrt_mode)

    def weights(self) -> OrcWeights:
        a = self.arrays

        def p(n):
            v = a.get(n)
            return None if v is None else v.ctypes.data

        return OrcWeights(p("router"), p("router_s"), p("g"), p("u"), p("d"), p("gs"),
                          p("us"), p("ds"), p("sh_g"), p("sh_u"), p("sh_d"), p("sh_gs"),
                          p("sh_us"), p("sh_ds"), p("sh_gate"), p("g_rscale"), p("g_pes"),
                          p("g_enorm"), p("router_bias"))


def make_layer(family: int, D: int, I: int, E: int, k: int, seed: int, *, renorm: int = 0,
               router_i8: int = 0, has_shared: int = 0, Is: int = 0,
               sigma: float = 0.02, router_bias=None, eps: float = 1e-6) -> Layer:
    """Seeded random layer.  Experts: N(0, sigma) quantised per row with the
    converter rule.  Router: f32 N(0, sigma), or (router_i8) quantised with the
    engine's load-time rule as qwen.c does in stream mode (qwen.c:283-288).
    The shared expert is quantised the same way (qwen.c:285-287); sh_gate
    stays f32 (qwen.c:282).

    GEMMA: the router is N(0, 1) (its input is unit-RMS scaled by D^-0.5, so
    logits have unit spread), int8 with the converter rule when router_i8
    (tools/convert_gemma.py:31-40 quantises router.proj); router.scale,
    per_expert_scale and pre_feedforward_layernorm_2 are 1 + N(0, 0.1)."""
    L = Layer(family, D, I, E, k, renorm, router_i8, has_shared, Is, eps=eps)
    a = L.arrays
    if router_bias is not None:
        a["router_bias"] = np.ascontiguousarray(router_bias, np.float32).reshape(E)
    g = np.empty((E, I, D), np.int8); u = np.empty((E, I, D), np.int8)
    d = np.empty((E, D, I), np.int8)
    gs = np.empty((E, I), np.float32); us = np.empty((E, I), np.float32)
    ds = np.empty((E, D), np.float32)
    base = seed * 1000003
    for e in range(E):
        g[e], gs[e] = quantize_py(normal(base + 3 * e + 1, (I, D), sigma))
        u[e], us[e] = quantize_py(normal(base + 3 * e + 2, (I, D), sigma))
        d[e], ds[e] = quantize_py(normal(base + 3 * e + 3, (D, I), sigma))
    a.update(g=g, u=u, d=d, gs=gs, us=us, ds=ds)
    if family == FAMILY_GEMMA:
        rw = normal(base + 7, (E, D), 1.0)
        if router_i8:
            a["router"], a["router_s"] = quantize_py(rw)
        else:
            a["router"] = rw
        a["g_rscale"] = 1.0 + normal(base + 15, (D,), 0.1)
        a["g_pes"] = 1.0 + normal(base + 16, (E,), 0.1)
        a["g_enorm"] = 1.0 + normal(base + 17, (D,), 0.1)
        return L
    rw = normal(base + 7, (E, D), sigma)
    if router_i8:
        a["router"], a["router_s"] = quantize_c(rw)
    else:
        a["router"] = rw
    if has_shared:
        a["sh_g"], a["sh_gs"] = quantize_c(normal(base + 11, (Is, D), sigma))
        a["sh_u"], a["sh_us"] = quantize_c(normal(base + 12, (Is, D), sigma))
        a["sh_d"], a["sh_ds"] = quantize_c(normal(base + 13, (D, Is), sigma))
        a["sh_gate"] = normal(base + 14, (D,), sigma)
    return L


def zipf_bias(E: int, s: float = 1.1, seed: int = 11) -> np.ndarray:
    """Router bias for a Zipf(s) skew over the experts: bias_e = -s*ln(rank_e),
    rank a seeded permutation of 1..E (a harness input; the reference has no
    bias term).  Added to the logits, it multiplies expert e's softmax weight
    by rank_e^-s."""
    rank = np.random.default_rng(seed).permutation(E) + 1
    return (-s * np.log(rank.astype(np.float64))).astype(np.float32)


def olmoe_layer(seed: int = 1, D=2048, I=1024, E=64, k=8, renorm=0) -> Layer:
    return make_layer(FAMILY_OLMOE, D, I, E, k, seed, renorm=renorm)


def qwen_layer(seed: int = 2, D=2048, I=512, E=256, k=8, Is=512, router_i8=1) -> Layer:
    return make_layer(FAMILY_QWEN, D, I, E, k, seed, renorm=1, router_i8=router_i8,
                      has_shared=1, Is=Is)


def gemma_layer(seed: int = 3, D=2816, I=704, E=128, k=8, router_i8=1) -> Layer:
    """Gemma-4-26B-A4B-shaped MoE layer (hidden 2816, 128 experts, top-8,
    moe_intermediate 704), int8 router as the converter writes it."""
    return make_layer(FAMILY_GEMMA, D, I, E, k, seed, router_i8=router_i8)


def oracle_prenorm(L: Layer, x: np.ndarray):
    """GEMMA: (router input xr [T,D], expert input xe [T,D], norm factor r [T])."""
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    xr = np.empty((T, L.D), np.float32)
    xe = np.empty((T, L.D), np.float32)
    r = np.empty(T, np.float32)
    d, ww = L.desc(), L.weights()
    if lib().orc_gemma_prenorm(C.byref(d), C.byref(ww), x, T, xr, xe, r):
        raise ValueError("orc_gemma_prenorm rejected the descriptor")
    return xr, xe, r


def oracle_moe(L: Layer, x: np.ndarray):
    """(out [T,D], topk_idx [T,k], topk_w [T,k]) from the C restatement."""
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    out = np.empty((T, L.D), np.float32)
    idx = np.empty((T, L.k), np.int32)
    w = np.empty((T, L.k), np.float32)
    d, ww = L.desc(), L.weights()
    rc = lib().orc_moe(C.byref(d), C.byref(ww), x, T, out, idx.ctypes.data, w.ctypes.data)
    if rc:
        raise ValueError("orc_moe rejected the descriptor")
    return out, idx, w


def oracle_expert_rows(L: Layer, x: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """y [R,D]: expert ids[r] (E = the shared expert) applied to x[r], unweighted."""
    x = np.ascontiguousarray(x, np.float32)
    ids = np.ascontiguousarray(ids, np.int32)
    y = np.empty((x.shape[0], L.D), np.float32)
    d, ww = L.desc(), L.weights()
    if lib().orc_expert_rows(C.byref(d), C.byref(ww), x, x.shape[0], ids.ctypes.data, y):
        raise ValueError("orc_expert_rows rejected the descriptor or an id")
    return y


ACT_SILU_DIV, ACT_SILU_SIG, ACT_GELU_TANH = 0, 1, 2


def oracle_expert_rows_act(L: Layer, x: np.ndarray, ids: np.ndarray, act: int) -> np.ndarray:
    """y [R,D]: routed expert ids[r] on row x[r] as given, activation `act`."""
    x = np.ascontiguousarray(x, np.float32)
    ids = np.ascontiguousarray(ids, np.int32)
    y = np.empty((x.shape[0], L.D), np.float32)
    d, ww = L.desc(), L.weights()
    if lib().orc_expert_rows_act(C.byref(d), C.byref(ww), x, x.shape[0], ids.ctypes.data, act, y):
        raise ValueError("orc_expert_rows_act rejected the descriptor, an id or act")
    return y


def oracle_shared_gate(L: Layer, x: np.ndarray) -> np.ndarray:
    """sg [T]: the shared expert's sigmoid gate."""
    x = np.ascontiguousarray(x, np.float32)
    sg = np.empty(x.shape[0], np.float32)
    d, ww = L.desc(), L.weights()
    if lib().orc_shared_gate(C.byref(d), C.byref(ww), x, x.shape[0], sg):
        raise ValueError("orc_shared_gate rejected the descriptor")
    return sg


def oracle_route(L: Layer, x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    idx = np.empty((T, L.k), np.int32)
    w = np.empty((T, L.k), np.float32)
    d, ww = L.desc(), L.weights()
    if lib().orc_route(C.byref(d), C.byref(ww), x, T, idx.ctypes.data, w.ctypes.data):
        raise ValueError("orc_route rejected the descriptor")
    return idx, w


def reference_moe(L: Layer, x: np.ndarray) -> np.ndarray:
    """out [T,D] from the reference's own compiled moe()/moe_step()."""
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    out = np.zeros((T, L.D), np.float32)
    a = L.arrays
    vp = lambda n: a[n].ctypes.data_as(C.c_void_p)  # noqa: E731
    if L.family == FAMILY_GEMMA:
        R = ref_lib("gemma")
        if R is None:
            raise RuntimeError("oracle/_ref not built")
        if "_gate_up" not in a:      # the container's fused gate_up layout, built once
            a["_gate_up"] = np.ascontiguousarray(np.concatenate([a["g"], a["u"]], axis=1))     # [E, 2I, D]
            a["_gate_up_s"] = np.ascontiguousarray(np.concatenate([a["gs"], a["us"]], axis=1))  # [E, 2I]
        gq, gsc = a["_gate_up"], a["_gate_up_s"]
        rs = a.get("router_s")
        rc = R.ref_gemma_moe(C.c_int(L.D), C.c_int(L.E), C.c_int(L.k), C.c_int(L.I), C.c_float(L.eps),
                             C.c_int(L.router_i8), vp("router"),
                             None if rs is None else rs.ctypes.data_as(C.c_void_p),
                             vp("g_rscale"), vp("g_pes"), vp("g_enorm"),
                             gq.ctypes.data_as(C.c_void_p), gsc.ctypes.data_as(C.c_void_p),
                             vp("d"), vp("ds"), x.ctypes.data_as(C.c_void_p), C.c_int(T),
                             out.ctypes.data_as(C.c_void_p))
    elif L.family == FAMILY_OLMOE:
        R = ref_lib("olmoe")
        if R is None:
            raise RuntimeError("oracle/_ref not built")
        assert not L.router_i8
        rc = R.ref_olmoe_moe(C.c_int(L.D), C.c_int(L.E), C.c_int(L.k), C.c_int(L.I),
                             C.c_int(L.renorm), x.ctypes.data_as(C.c_void_p), C.c_int(T),
                             vp("router"), vp("g"), vp("gs"), vp("u"), vp("us"), vp("d"),
                             vp("ds"), out.ctypes.data_as(C.c_void_p))
    else:
        R = ref_lib("qwen")
        if R is None:
            raise RuntimeError("oracle/_ref not built")
        assert L.router_i8 and L.has_shared
        rc = R.ref_qwen_moe(C.c_int(L.D), C.c_int(L.E), C.c_int(L.k), C.c_int(L.I),
                            C.c_int(L.Is), vp("router"), vp("router_s"), vp("sh_g"),
                            vp("sh_gs"), vp("sh_u"), vp("sh_us"), vp("sh_d"), vp("sh_ds"),
                            vp("sh_gate"), vp("g"), vp("gs"), vp("u"), vp("us"), vp("d"),
                            vp("ds"), x.ctypes.data_as(C.c_void_p), C.c_int(T),
                            out.ctypes.data_as(C.c_void_p))
    if rc:
        raise RuntimeError("reference harness failed")
    return out


def reference_route(L: Layer, x: np.ndarray):
    """GEMMA: (topk_idx [T,k], topk_w [T,k]) from the reference's own compiled
    route_token (engines/gemma.c:455-478)."""
    assert L.family == FAMILY_GEMMA
    R = ref_lib("gemma")
    if R is None:
        raise RuntimeError("oracle/_ref not built")
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    idx = np.empty((T, L.k), np.int32)
    w = np.empty((T, L.k), np.float32)
    a = L.arrays
    rs = a.get("router_s")
    vp = lambda n: a[n].ctypes.data_as(C.c_void_p)  # noqa: E731
    rc = R.ref_gemma_route(C.c_int(L.D), C.c_int(L.E), C.c_int(L.k), C.c_float(L.eps), C.c_int(L.router_i8),
                           vp("router"), None if rs is None else rs.ctypes.data_as(C.c_void_p),
                           vp("g_rscale"), vp("g_pes"), x.ctypes.data_as(C.c_void_p), C.c_int(T),
                           idx.ctypes.data_as(C.c_void_p), w.ctypes.data_as(C.c_void_p))
    if rc:
        raise RuntimeError("reference harness failed")
    return idx, w


# ------------------------------------------------------------- hot store --
# include/tier.h restated (moe_oracle.c) and, when built, the reference's own
# functions (_ref/libref_tier.so).  `pinned` names the expert in each HBM
# slot; a pick returns (slot, eid, gain) or None.

_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def _tier_bind(L, prefix):
    lfru = getattr(L, prefix + "pick_lfru")
    lfru.restype = C.c_int
    lfru.argtypes = [_u32p, _u32p, C.c_uint32, C.c_int, _i32p, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int),
                     C.POINTER(C.c_long)]
    heat = getattr(L, prefix + ("pick_heat" if prefix == "orc_tier_" else "pick_swap"))
    heat.restype = C.c_int
    heat.argtypes = [_u32p, C.c_int, _i32p, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_long)]
    score = getattr(L, prefix + ("score" if prefix == "orc_tier_" else "lfru_score"))
    score.restype = C.c_uint64
    score.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32]
    getattr(L, prefix + "decay").argtypes = [_u32p, C.c_int]
    return lfru, heat, score, getattr(L, prefix + "decay")


class Tier:
    """The four tier.h functions from one library (the restatement or the
    reference build)."""

    def __init__(self, which: str = "oracle"):
        if which == "oracle":
            L = lib()
            self.lfru, self.heat, self.score_fn, self.decay_fn = _tier_bind(L, "orc_tier_")
            L.orc_tier_account.argtypes = [_i32p, C.c_int, C.c_int, _u32p, _u32p, C.POINTER(C.c_uint32), C.c_int]
            self._account = L.orc_tier_account
        else:
            R = ref_lib("tier")
            if R is None:
                raise RuntimeError("reference tier.h harness not built (oracle/_ref/libref_tier.so)")
            self.lfru, self.heat, self.score_fn, self.decay_fn = _tier_bind(R, "ref_tier_")
            self._account = None

    @staticmethod
    def _out(rc, slot, eid, gain):
        return (slot.value, eid.value, gain.value) if rc else None

    def pick_lfru(self, heat, last, clock, pinned):
        heat, last = np.ascontiguousarray(heat, np.uint32), np.ascontiguousarray(last, np.uint32)
        pinned = np.ascontiguousarray(pinned, np.int32)
        s, e, g = C.c_int(-1), C.c_int(-1), C.c_long(0)
        rc = self.lfru(heat, last, clock & 0xFFFFFFFF, heat.size, pinned, pinned.size, C.byref(s), C.byref(e),
                       C.byref(g))
        return self._out(rc, s, e, g)

    def pick_heat(self, heat, pinned):
        heat, pinned = np.ascontiguousarray(heat, np.uint32), np.ascontiguousarray(pinned, np.int32)
        s, e, g = C.c_int(-1), C.c_int(-1), C.c_long(0)
        rc = self.heat(heat, heat.size, pinned, pinned.size, C.byref(s), C.byref(e), C.byref(g))
        return self._out(rc, s, e, g)

    def score(self, heat, last, clock):
        return int(self.score_fn(heat & 0xFFFFFFFF, last & 0xFFFFFFFF, clock & 0xFFFFFFFF))

    def decay(self, heat):
        h = np.array(heat, np.uint32)
        self.decay_fn(h, h.size)
        return h

    def account(self, topk_idx, nexpert, heat, last, clock, decay_every=0):
        """One forward's routing into (heat, last, clock); returns the new triple."""
        idx = np.ascontiguousarray(topk_idx, np.int32).ravel()
        h, l = np.array(heat, np.uint32), np.array(last, np.uint32)
        c = C.c_uint32(clock)
        self._account(idx, idx.size, nexpert, h, l, C.byref(c), decay_every)
        return h, l, c.value
