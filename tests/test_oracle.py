"""CPU: the oracle (C restatement) against the reference.

1. against the golden fixtures made by the reference's own compiled code
   (tests/golden/make_golden.py) -- runs everywhere;
2. against the reference compiled from its sources (oracle/_ref) on fresh
   seeded inputs -- wherever oracle/_ref was built;
3. the reference's own token oracles (oracle/qwen_tiny + ref_qwen.json,
   oracle/gemma_tiny + ref_gemma.json), run through the same reference
   build, still say 20/20;
4. the device expf restatement's host twin equals glibc expf bit for bit;
5. Gemma's router norm: the oracle with the reference's powf is the
   reference bit for bit; with the correctly rounded factor the device uses,
   routing indices are the same and weights move by a few ulps on the rows
   whose factor differs.
"""
import glob
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "golden_*.npz")))


def load_golden(oracle, path):
    z = np.load(path)
    fam, D, I, E, k, renorm, r_i8, has_sh, Is = (int(v) for v in z["meta"])
    L = oracle.Layer(fam, D, I, E, k, renorm, r_i8, has_sh, Is)
    for name in ("router", "router_s", "g", "u", "d", "gs", "us", "ds", "sh_g", "sh_u", "sh_d",
                 "sh_gs", "sh_us", "sh_ds", "sh_gate", "g_rscale", "g_pes", "g_enorm"):
        if name in z.files:
            L.arrays[name] = np.ascontiguousarray(z[name])
    if "eps" in z.files:
        L.eps = float(z["eps"][0])
        L.rsqrt_mode = oracle.RSQRT_LIBM     # the fixtures hold the reference's own outputs
    return L, z


def test_golden_fixtures_present():
    names = {os.path.basename(p) for p in GOLDEN}
    for want in ("olmoe_small", "olmoe_renorm", "olmoe_ties", "qwen_small", "qwen_tiny_l0",
                 "qwen_tiny_l3", "gemma_small", "gemma_i8", "gemma_ties", "gemma_tiny_l0",
                 "gemma_tiny_l5"):
        assert f"golden_{want}.npz" in names


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[7:-4] for p in GOLDEN])
def test_oracle_matches_reference_golden(oracle, path):
    L, z = load_golden(oracle, path)
    out, idx, w = oracle.oracle_moe(L, z["x"])
    assert np.array_equal(out.view(np.uint32), z["out_ref"].view(np.uint32))
    assert np.array_equal(idx, z["idx_ref"])
    assert np.array_equal(w.view(np.uint32), z["w_ref"].view(np.uint32))
    ridx, rw = oracle.oracle_route(L, z["x"])
    assert np.array_equal(ridx, idx) and np.array_equal(rw, w)


@pytest.mark.parametrize("name", ["olmoe_ties", "gemma_ties"])
def test_tie_break_lower_expert_id(oracle, name):
    L, z = load_golden(oracle, os.path.join(ROOT, "tests", "golden", f"golden_{name}.npz"))
    idx, w = z["idx_ref"], z["w_ref"]
    # gemma scales each weight by its expert's per_expert_scale: compare the
    # weights before that factor
    pre = w / L.arrays["g_pes"][idx] if "g_pes" in L.arrays else w
    n = 0
    for t in range(idx.shape[0]):
        for j in range(idx.shape[1] - 1):
            if pre[t, j] == pre[t, j + 1]:
                assert idx[t, j] < idx[t, j + 1]
                n += 1
    assert n > 0


needs_ref = pytest.mark.skipif(
    not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libref_olmoe.so")),
    reason="oracle/_ref not built here")


@needs_ref
@pytest.mark.parametrize("case", ["f32", "i8"])
def test_gemma_oracle_bitexact_vs_reference_build(oracle, case):
    """route_token and the expert union of engines/gemma.c against the
    oracle with the reference's powf: routing and output bit for bit."""
    L = oracle.make_layer(oracle.FAMILY_GEMMA, 256, 96, 32, 8, seed=31 + (case == "i8"),
                          router_i8=int(case == "i8"))
    L.rsqrt_mode = oracle.RSQRT_LIBM
    x = oracle.normal(600, (40, L.D), 1.5)
    out, idx, w = oracle.oracle_moe(L, x)
    ridx, rw = oracle.reference_route(L, x)
    assert np.array_equal(idx, ridx)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    ref = oracle.reference_moe(L, x)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_gemma_rsqrt_modes(oracle):
    """Correctly rounded factor (device) against libm powf (reference) over
    20000 residual rows: identical routing indices; weights identical on every
    row whose factor agrees, within 32 ulps on the others."""
    L = oracle.make_layer(oracle.FAMILY_GEMMA, 256, 32, 64, 8, seed=41, router_i8=1)
    x = oracle.normal(601, (20000, L.D), 2.0)
    L.rsqrt_mode = oracle.RSQRT_LIBM
    _, _, rl = oracle.oracle_prenorm(L, x)
    il, wl = oracle.oracle_route(L, x)
    L.rsqrt_mode = oracle.RSQRT_CR
    _, _, rc = oracle.oracle_prenorm(L, x)
    ic, wc = oracle.oracle_route(L, x)
    same_r = rl.view(np.uint32) == rc.view(np.uint32)
    assert np.array_equal(il, ic)
    assert np.array_equal(wl[same_r].view(np.uint32), wc[same_r].view(np.uint32))
    assert np.all(np.abs(rl.view(np.int32) - rc.view(np.int32)) <= 1)
    ulps = np.abs(wl.view(np.int32).astype(np.int64) - wc.view(np.int32).astype(np.int64))
    assert ulps.max() <= 32


def test_gemma_rsqrt_check():
    """oracle/rsqrt_check: the device's factor formula equals the long double
    value rounded to float on every 7th positive float."""
    exe = os.path.join(ROOT, "oracle", "rsqrt_check")
    if not os.path.exists(exe):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "rsqrt_check"], check=True,
                       capture_output=True)
    p = subprocess.run([exe, "7"], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0 and " 0 double/long-double mismatches" in p.stdout, p.stdout + p.stderr


@needs_ref
@pytest.mark.parametrize("case", ["olmoe", "olmoe_renorm", "qwen", "olmoe_full_T3"])
def test_oracle_bitexact_vs_reference_build(oracle, case):
    if case == "olmoe":
        L = oracle.olmoe_layer(11, D=256, I=128, E=16, k=4)
        T = 33
    elif case == "olmoe_renorm":
        L = oracle.olmoe_layer(12, D=192, I=96, E=10, k=3, renorm=1)
        T = 17
    elif case == "qwen":
        L = oracle.qwen_layer(13, D=256, I=64, E=32, k=8, Is=96)
        T = 21
    else:
        L = oracle.olmoe_layer(14)          # full OLMoE shape
        T = 3
    x = oracle.normal(500 + T, (T, L.D))
    out, _, _ = oracle.oracle_moe(L, x)
    ref = oracle.reference_moe(L, x)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("model", ["qwen", "gemma"])
def test_reference_token_oracle_through_harness_build(oracle, model):
    """The reference's own known-answer tests (Makefile:37-41) still pass with
    the reference compiled by oracle/Makefile: the build is faithful."""
    ref_root = oracle.ref_root()
    snap = os.path.join(ref_root or "", "oracle", f"{model}_tiny")
    if ref_root is None or not os.path.isdir(snap):
        pytest.skip("reference sources not present")
    exe = os.path.join(ROOT, "oracle", "_ref", model)
    p = subprocess.run([exe, os.path.join(ref_root, "oracle", f"ref_{model}.json")],
                       env=dict(os.environ, SNAP=snap), capture_output=True, text=True, timeout=120)
    assert p.returncode == 0 and "20/20 EXACT" in p.stdout


def test_glibc_expf_restatement_exhaustive_sample():
    """oracle/expf_check: the restated expf equals glibc on every 7th float
    bit pattern (all 2^32 with stride 1; ~6 s on 8 cores)."""
    exe = os.path.join(ROOT, "oracle", "expf_check")
    if not os.path.exists(exe):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "expf_check"], check=True,
                       capture_output=True)
    p = subprocess.run([exe, "7"], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout + p.stderr
    assert " 0 mismatches" in p.stdout


def test_quantizer_rules(oracle):
    w = oracle.normal(77, (16, 64), 0.02)
    q, s = oracle.quantize_py(w)
    amax = np.abs(w).max(axis=1)
    np.testing.assert_array_equal(s, (np.maximum(amax, np.float32(1e-12)) / np.float32(127.0)).astype(np.float32))
    np.testing.assert_array_equal(q, np.clip(np.round(w / s[:, None]), -128, 127).astype(np.int8))
    q2, s2 = oracle.quantize_c(w)
    assert np.abs(q2.astype(int) - q.astype(int)).max() <= 1
