"""Generate the golden MoE fixtures from the REFERENCE itself.

Run in a container that has the reference sources (oracle/_ref built by
``make -C oracle``; the tiny fixture model under REF_ROOT/oracle/qwen_tiny):

    python tests/golden/make_golden.py

Each ``golden_*.npz`` holds the layer (int8 experts + scales, router,
shared expert), the input x, and ``out_ref`` -- the output of the reference's
own compiled moe() (engines/olmoe.c:344-402) or moe_step()
(engines/qwen.c:453-495) on those inputs.  ``idx_ref``/``w_ref`` are the
routing of the C restatement (oracle/moe_oracle.c), recorded only after its
out matched out_ref bit for bit.  The fixtures pin the oracle where the
reference cannot be built, and the GPU path against the reference directly.

Cases:
  olmoe_small   D=128 I=64 E=8 k=2, softmax top-k, no renorm
  olmoe_renorm  D=128 I=96 E=12 k=3, norm_topk_prob=1
  olmoe_ties    D=128 I=64 E=8 k=3, router rows duplicated -> exactly tied
                probabilities, which the reference breaks by lower expert id
  qwen_small    D=128 I=64 E=16 k=4 Is=64, int8 router, shared expert
  qwen_tiny_l0 / qwen_tiny_l3
                the reference's own test model (oracle/qwen_tiny,
                tools/make_qwen_oracle.py) layers 0 and 3, quantised the way
                stream mode runs it: experts with the converter rule
                (tools/convert_qwen.py:23-27), router and shared expert with
                the engine's load-time rule (engines/qwen.c:124-138,283-288)
  gemma_small   D=128 I=64 E=16 k=4, f32 router; x is the residual row
  gemma_i8      D=128 I=32 E=24 k=8, int8 router (tools/convert_gemma.py:31-40)
  gemma_ties    D=128 I=64 E=8 k=3, router rows duplicated -> tied softmax
                numerators, broken by lower expert id (engines/gemma.c:468-475)
  gemma_tiny_l0 / gemma_tiny_l5
                the reference's own Gemma fixture (oracle/gemma_tiny,
                tools/make_gemma_oracle.py) layers 0 and 5: its f32 router,
                router.scale, per_expert_scale and pre_feedforward_layernorm_2;
                its fused gate_up / down experts quantised with the converter
                rule (tools/convert_gemma.py:35-40)
For Gemma the oracle runs with the reference's powf (RSQRT_LIBM) so that it
is bit-identical to the reference; ``eps`` holds rms_norm_eps.

``tier_cases.npz`` holds hot-store policy cases (include/tier.h, compiled
from the reference as oracle/_ref/libref_tier.so): heat/last/clock/pinned
inputs, including exact ties, margins on and one past the hysteresis bound,
clock wrap-around and 32-bit heat overflow, with the results of the
reference's tier_pick_lfru, tier_pick_swap, tier_lfru_score and tier_decay.
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import pyoracle as P  # noqa: E402

REF_ROOT = P.ref_root()
if REF_ROOT is None:
    sys.exit("the reference sources are needed: set REF_ROOT")


def bits_equal(a, b):
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def save(name, L, x, out_ref, extra=None):
    o, idx, w = P.oracle_moe(L, x)
    assert bits_equal(o, out_ref), f"{name}: oracle differs from the reference"
    meta = np.array([L.family, L.D, L.I, L.E, L.k, L.renorm, L.router_i8, L.has_shared, L.Is],
                    np.int32)
    arrays = {k: v for k, v in L.arrays.items() if not k.startswith("_")}
    arrays.update(meta=meta, x=x, out_ref=out_ref, idx_ref=idx, w_ref=w)
    if L.family == P.FAMILY_GEMMA:
        ridx, rw = P.reference_route(L, x)
        assert np.array_equal(ridx, idx) and bits_equal(rw, w), f"{name}: routing differs"
        arrays.update(eps=np.array([L.eps], np.float32))
    if extra:
        arrays.update(extra)
    np.savez_compressed(os.path.join(HERE, f"golden_{name}.npz"), **arrays)
    print(f"{name}: T={x.shape[0]} max|out|={np.abs(out_ref).max():.4f} idx[0]={idx[0]}")


def tiny_layer(li):
    R = P.ref_lib("qwen")
    snap = os.path.join(REF_ROOT, "oracle", "qwen_tiny").encode()
    R.ref_qwen_tiny_load(C.c_char_p(snap))
    dims = (C.c_int * 7)()
    R.ref_qwen_tiny_dims(dims)
    D, E, K, MI, SI = dims[0], dims[1], dims[2], dims[3], dims[4]
    f = lambda *s: np.zeros(s, np.float32)  # noqa: E731
    gate, shg, shu, shd, shgate = f(E, D), f(SI, D), f(SI, D), f(D, SI), f(D)
    eg, eu, ed = f(E, MI, D), f(E, MI, D), f(E, D, MI)
    vp = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    rc = R.ref_qwen_tiny_weights(C.c_int(li), vp(gate), vp(shg), vp(shu), vp(shd), vp(shgate),
                                 vp(eg), vp(eu), vp(ed))
    assert rc == 0
    L = P.Layer(P.FAMILY_QWEN, D, MI, E, K, 1, 1, 1, SI)
    a = L.arrays
    a["router"], a["router_s"] = P.quantize_c(gate)
    a["sh_g"], a["sh_gs"] = P.quantize_c(shg)
    a["sh_u"], a["sh_us"] = P.quantize_c(shu)
    a["sh_d"], a["sh_ds"] = P.quantize_c(shd)
    a["sh_gate"] = shgate
    q = [P.quantize_py(m) for m in eg]
    a["g"], a["gs"] = np.stack([t[0] for t in q]), np.stack([t[1] for t in q])
    q = [P.quantize_py(m) for m in eu]
    a["u"], a["us"] = np.stack([t[0] for t in q]), np.stack([t[1] for t in q])
    q = [P.quantize_py(m) for m in ed]
    a["d"], a["ds"] = np.stack([t[0] for t in q]), np.stack([t[1] for t in q])
    # the reference's own f32-resident moe_step on the same x (information only)
    return L, R


def gemma_tiny_layer(li):
    R = P.ref_lib("gemma")
    snap = os.path.join(REF_ROOT, "oracle", "gemma_tiny").encode()
    R.ref_gemma_tiny_load(C.c_char_p(snap))
    dims = (C.c_int * 6)()
    eps = C.c_float()
    R.ref_gemma_tiny_dims(dims, C.byref(eps))
    D, E, K, MI = dims[0], dims[1], dims[2], dims[3]
    assert dims[5] == 0, "gemma_tiny is expected f32-resident"
    f = lambda *s: np.zeros(s, np.float32)  # noqa: E731
    router, rscale, pes, enorm = f(E, D), f(D), f(E), f(D)
    eg, ed = f(E, 2 * MI, D), f(E, D, MI)
    vp = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    rc = R.ref_gemma_tiny_weights(C.c_int(li), vp(router), vp(rscale), vp(pes), vp(enorm), vp(eg), vp(ed))
    assert rc == 0, rc
    L = P.Layer(P.FAMILY_GEMMA, D, MI, E, K, 1, 0, 0, 0, eps=eps.value, rsqrt_mode=P.RSQRT_LIBM)
    a = L.arrays
    a["router"], a["g_rscale"], a["g_pes"], a["g_enorm"] = router, rscale, pes, enorm
    # the converter quantises the fused gate_up rows [2MI, D] as one matrix
    q = [P.quantize_py(m) for m in eg]
    gq, gsc = np.stack([t[0] for t in q]), np.stack([t[1] for t in q])
    a["g"], a["u"] = np.ascontiguousarray(gq[:, :MI]), np.ascontiguousarray(gq[:, MI:])
    a["gs"], a["us"] = np.ascontiguousarray(gsc[:, :MI]), np.ascontiguousarray(gsc[:, MI:])
    q = [P.quantize_py(m) for m in ed]
    a["d"], a["ds"] = np.stack([t[0] for t in q]), np.stack([t[1] for t in q])
    return L, R


def gemma_cases():
    L = P.make_layer(P.FAMILY_GEMMA, 128, 64, 16, 4, seed=201)
    L.rsqrt_mode = P.RSQRT_LIBM
    x = P.normal(2001, (12, 128), 3.0)
    save("gemma_small", L, x, P.reference_moe(L, x))

    L = P.make_layer(P.FAMILY_GEMMA, 128, 32, 24, 8, seed=202, router_i8=1)
    L.rsqrt_mode = P.RSQRT_LIBM
    x = P.normal(2002, (10, 128), 0.5)
    save("gemma_i8", L, x, P.reference_moe(L, x))

    L = P.make_layer(P.FAMILY_GEMMA, 128, 64, 8, 3, seed=203)
    L.rsqrt_mode = P.RSQRT_LIBM
    r = L.arrays["router"]
    r[5] = r[2]
    r[6] = r[1]
    x = P.normal(2003, (16, 128))
    out = P.reference_moe(L, x)
    _, idx, w = P.oracle_moe(L, x)
    ties = sum(int(idx[t, j] in (1, 2) and idx[t, j + 1] in (5, 6)) for t in range(16) for j in range(2))
    assert ties > 0, "tie case produced no tied selections"
    save("gemma_ties", L, x, out)

    for li in (0, 5):
        L, R = gemma_tiny_layer(li)
        x = P.normal(2100 + li, (8, L.D), 2.0)
        out = P.reference_moe(L, x)
        ti = np.zeros((8, L.k), np.int32)
        tw = np.zeros((8, L.k), np.float32)
        R.ref_gemma_tiny_route(C.c_int(li), x.ctypes.data_as(C.c_void_p), C.c_int(8),
                               ti.ctypes.data_as(C.c_void_p), tw.ctypes.data_as(C.c_void_p))
        ridx, rw = P.reference_route(L, x)
        assert np.array_equal(ti, ridx) and bits_equal(tw, rw), "fixture routing differs from its arrays"
        save(f"gemma_tiny_l{li}", L, x, out)


def main():
    assert P.ref_available(), "build oracle/_ref first (make -C oracle)"
    L = P.make_layer(P.FAMILY_OLMOE, 128, 64, 8, 2, seed=101)
    x = P.normal(1001, (12, 128))
    save("olmoe_small", L, x, P.reference_moe(L, x))

    L = P.make_layer(P.FAMILY_OLMOE, 128, 96, 12, 3, seed=102, renorm=1)
    x = P.normal(1002, (9, 128))
    save("olmoe_renorm", L, x, P.reference_moe(L, x))

    L = P.make_layer(P.FAMILY_OLMOE, 128, 64, 8, 3, seed=103)
    r = L.arrays["router"]
    r[5] = r[2]
    r[6] = r[1]
    x = P.normal(1003, (16, 128))
    out = P.reference_moe(L, x)
    _, idx, w = P.oracle_moe(L, x)
    ties = sum(int(w[t, j] == w[t, j + 1]) for t in range(16) for j in range(2))
    assert ties > 0, "tie case produced no tied selections"
    save("olmoe_ties", L, x, out)

    L = P.make_layer(P.FAMILY_QWEN, 128, 64, 16, 4, seed=104, renorm=1, router_i8=1,
                     has_shared=1, Is=64)
    x = P.normal(1004, (10, 128))
    save("qwen_small", L, x, P.reference_moe(L, x))

    for li in (0, 3):
        L, R = tiny_layer(li)
        x = P.normal(1100 + li, (8, L.D))
        out = P.reference_moe(L, x)
        f32 = np.zeros_like(out)
        R.ref_qwen_tiny_moe(C.c_int(li), x.ctypes.data_as(C.c_void_p), C.c_int(x.shape[0]),
                            f32.ctypes.data_as(C.c_void_p))
        save(f"qwen_tiny_l{li}", L, x, out, {"out_ref_f32_resident": f32})

    gemma_cases()
    tier_cases()


def tier_cases(n=480, emax=64):
    """Policy cases through the reference's own tier.h functions."""
    R = P.Tier("ref")
    rng = np.random.default_rng(2024)
    H = np.zeros((n, emax), np.uint32)
    La = np.zeros((n, emax), np.uint32)
    PIN = np.full((n, emax), -1, np.int32)
    E_, NP, CLK = np.zeros(n, np.int32), np.zeros(n, np.int32), np.zeros(n, np.uint32)
    for c in range(n):
        E = int(rng.integers(1, emax + 1))
        npin = int(rng.integers(1, E + 1))
        kind = c % 8
        hi = [4, 64, 1 << 12, 1 << 24, 2**32 - 1, 16, 1 << 10, 3][kind]
        heat = rng.integers(0, hi, E, dtype=np.uint64).astype(np.uint32)
        clock = int(rng.integers(0, 2**32)) if kind != 5 else int(rng.integers(0, 300))
        last = ((clock - rng.integers(0, 600, E)) & 0xFFFFFFFF).astype(np.uint32)
        if kind == 5:                       # last recorded before a clock wrap-around
            last[: E // 2] = (2**32 - rng.integers(1, 50, E // 2)).astype(np.uint32)
        pinned = rng.choice(E, npin, replace=False).astype(np.int32)
        if kind == 2:                       # exact ties
            heat[:] = heat[0]
            last[:] = last[0]
        if kind == 3 and npin < E:          # hottest outsider on, or one past, the margin
            cold = int(pinned[0])
            heat[pinned] = np.maximum(heat[pinned], heat[cold])
            last[pinned] = clock
            out = [e for e in range(E) if e not in set(pinned.tolist())]
            cs = R.score(int(heat[cold]), int(last[cold]), clock)
            bound = cs + (cs >> 2) + (4 << 8) + (c // 8) % 2
            heat[out] = 0
            heat[out[0]] = bound >> 8
            last[out[0]] = (clock - (255 - (bound & 255))) & 0xFFFFFFFF
        H[c, :E], La[c, :E], PIN[c, :npin] = heat, last, pinned
        E_[c], NP[c], CLK[c] = E, npin, clock
    res_l = np.full((n, 4), -1, np.int64)
    res_h = np.full((n, 4), -1, np.int64)
    scores = np.zeros((n, emax), np.uint64)
    decayed = np.zeros((n, emax), np.uint32)
    for c in range(n):
        E, npin = int(E_[c]), int(NP[c])
        a = R.pick_lfru(H[c, :E], La[c, :E], int(CLK[c]), PIN[c, :npin])
        b = R.pick_heat(H[c, :E], PIN[c, :npin])
        res_l[c] = (1, *a) if a else (0, -1, -1, 0)
        res_h[c] = (1, *b) if b else (0, -1, -1, 0)
        scores[c, :E] = [R.score(int(H[c, e]), int(La[c, e]), int(CLK[c])) for e in range(E)]
        decayed[c, :E] = R.decay(H[c, :E])
    np.savez_compressed(os.path.join(HERE, "tier_cases.npz"), heat=H, last=La, pinned=PIN, E=E_, npin=NP,
                        clock=CLK, lfru=res_l, swap=res_h, score=scores, decay=decayed)


if __name__ == "__main__":
    main()
