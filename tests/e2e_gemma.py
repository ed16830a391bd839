"""End-to-end Gemma greedy generation: the reference engine on the CPU against
the same engine with its MoE block on the GPU (test infrastructure).

A seeded random-init Gemma-4-style snapshot is written in the engine's int8
container format (config.json + safetensors, the layout tools/convert_gemma.py
writes and engines/gemma.c:381-437 loads): f32 embeddings, norms, attention
and dense-MLP matrices; router.proj as int8 + .qs; per-expert
experts.E.gate_up_proj [2I,D] and down_proj [D,I] as int8 + .qs (so the
engine runs in stream mode, engines/gemma.c:385).  Matrices are N(0, 0.02)
from the oracle's generator, int8 ones quantised with the converter rule
(tools/convert_gemma.py:35-40, oracle `quantize_py`); norm weights,
router.scale and per_expert_scale are 1 + N(0, 0.1); layer_scalar is 1.

Two builds of the unmodified engines/gemma.c generate greedily from the same
prompt (main, engines/gemma.c:875-929: a batched teacher-forcing pass, then a
batched prefill and token-by-token decode):
  oracle/_ref/gemma       the reference, all host cores (OpenMP)
  oracle/_ref/gemma_omc   the same engine with the routing + expert union of
                          every step on the GPU (include/omc_gemma_hook.h)
and their greedy tokens are compared.

CLI:  python tests/e2e_gemma.py [--layers 4 --new 16]  prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import shutil
import subprocess
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, HERE)
from e2e_olmoe import SafetensorsWriter, _oracle, _seed, prompt_ids  # noqa: E402

REF_ENGINE = os.path.join(ROOT, "oracle", "_ref", "gemma")
OMC_ENGINE = os.path.join(ROOT, "oracle", "_ref", "gemma_omc")

# a small Gemma-4-shaped model: sliding layers with a full-attention last layer
D, NH, NKV, HD, NGKV, GHD = 256, 4, 2, 64, 1, 128
E, K, MI, INTER = 16, 4, 64, 128


def layer_types(layers):
    return ["full_attention" if (i + 1) % 4 == 0 else "sliding_attention" for i in range(layers)]


def make_snapshot(snap: str, layers: int, vocab: int, seed: int = 4242) -> None:
    P = _oracle()
    os.makedirs(snap, exist_ok=True)
    cfg = {"architectures": ["Gemma4ForCausalLM"], "hidden_size": D, "num_hidden_layers": layers,
           "num_attention_heads": NH, "num_key_value_heads": NKV, "head_dim": HD,
           "num_global_key_value_heads": NGKV, "global_head_dim": GHD, "num_experts": E,
           "top_k_experts": K, "moe_intermediate_size": MI, "intermediate_size": INTER,
           "vocab_size": vocab, "sliding_window": 8, "rms_norm_eps": 1e-6, "final_logit_softcapping": 30.0,
           "rope_parameters": {"full_attention": {"partial_rotary_factor": 0.25, "rope_theta": 1000000.0},
                               "sliding_attention": {"rope_theta": 10000.0}},
           "layer_types": layer_types(layers), "eos_token_id": -1}
    with open(os.path.join(snap, "config.json"), "w") as f:
        json.dump(cfg, f)
    specs, vals = [], {}

    def mat(name, shape, idx):
        specs.append((name, np.float32, shape))
        vals[name] = ("n", _seed(seed, -2, idx), shape, 0.02)

    def norm(name, n, idx):
        specs.append((name, np.float32, (n,)))
        vals[name] = ("one", _seed(seed, -3, idx), (n,), 0.1)

    def i8(name, shape, idx):
        specs.append((name, np.int8, shape))
        specs.append((name + ".qs", np.float32, (shape[0],)))
        vals[name] = ("q", _seed(seed, -4, idx), shape, 0.02)

    n = 0
    mat("model.embed_tokens.weight", (vocab, D), n); n += 1
    norm("model.norm.weight", D, n); n += 1
    for li, lt in enumerate(layer_types(layers)):
        full = lt == "full_attention"
        hd, nkv = (GHD, NGKV) if full else (HD, NKV)
        p = f"model.layers.{li}."
        for nm in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                   "post_feedforward_layernorm", "post_feedforward_layernorm_1", "post_feedforward_layernorm_2",
                   "pre_feedforward_layernorm_2"):
            norm(p + nm + ".weight", D, n); n += 1
        specs.append((p + "layer_scalar", np.float32, (1,)))
        vals[p + "layer_scalar"] = ("const", 1.0)
        mat(p + "self_attn.q_proj.weight", (NH * hd, D), n); n += 1
        norm(p + "self_attn.q_norm.weight", hd, n); n += 1
        mat(p + "self_attn.k_proj.weight", (nkv * hd, D), n); n += 1
        norm(p + "self_attn.k_norm.weight", hd, n); n += 1
        if not full:
            mat(p + "self_attn.v_proj.weight", (nkv * hd, D), n); n += 1
        mat(p + "self_attn.o_proj.weight", (D, NH * hd), n); n += 1
        mat(p + "mlp.gate_proj.weight", (INTER, D), n); n += 1
        mat(p + "mlp.up_proj.weight", (INTER, D), n); n += 1
        mat(p + "mlp.down_proj.weight", (D, INTER), n); n += 1
        specs.append((p + "router.proj.weight", np.int8, (E, D)))
        specs.append((p + "router.proj.weight.qs", np.float32, (E,)))
        vals[p + "router.proj.weight"] = ("q", _seed(seed, -5, n), (E, D), 1.0); n += 1
        norm(p + "router.scale", D, n); n += 1
        norm(p + "router.per_expert_scale", E, n); n += 1
        for e in range(E):
            i8(f"{p}experts.{e}.gate_up_proj", (2 * MI, D), n); n += 1
            i8(f"{p}experts.{e}.down_proj", (D, MI), n); n += 1
    wr = SafetensorsWriter(os.path.join(snap, "model-00000.safetensors"), specs)
    for name, dt, shape in specs:
        if name.endswith(".qs"):
            continue
        v = vals[name]
        if v[0] == "n":
            wr.put(name, P.normal(v[1], v[2], v[3]))
        elif v[0] == "one":
            wr.put(name, (1.0 + P.normal(v[1], v[2], v[3])).astype(np.float32))
        elif v[0] == "const":
            wr.put(name, np.full(shape, v[1], np.float32))
        else:
            q, s = P.quantize_py(P.normal(v[1], v[2], v[3]))
            wr.put(name, q)
            wr.put(name + ".qs", s)
    wr.close()


def run_engine(binary: str, snap: str, prompt: list, n_new: int, timeout=1800):
    """Runs the engine's batched teacher-forcing pass and greedy generation;
    returns (new tokens, seconds, log).  The reference file holds the prompt
    and zeros as "expected" continuation, so the engine's own match count is
    meaningless here (it exits 1); its generated tokens are what is compared."""
    with tempfile.TemporaryDirectory() as td:
        ref = os.path.join(td, "ref.json")
        with open(ref, "w") as f:
            json.dump({"prompt_ids": prompt, "full_ids": prompt + [0] * n_new, "tf_argmax": []}, f)
        t0 = time.perf_counter()
        p = subprocess.run([binary, ref], env=dict(os.environ, SNAP=snap), capture_output=True, text=True,
                           timeout=timeout)
        dt = time.perf_counter() - t0
    log = p.stdout + p.stderr
    if p.returncode not in (0, 1):
        raise RuntimeError(f"{binary} exited {p.returncode}:\n{log[-3000:]}")
    m = re.search(r"^engine +: ([0-9 ]+)", p.stdout, re.M)
    if not m or "int8 streaming" not in p.stdout:
        raise RuntimeError(f"unexpected output of {binary}:\n{log[-3000:]}")
    return [int(t) for t in m.group(1).split()], dt, log


def compare(layers: int, vocab: int, n_prompt: int, n_new: int, workdir: str | None = None):
    own = workdir is None
    workdir = workdir or tempfile.mkdtemp(prefix="gemma_e2e_")
    snap = os.path.join(workdir, "snap")
    try:
        if not os.path.exists(os.path.join(snap, "config.json")):
            make_snapshot(snap, layers, vocab)
        prompt = prompt_ids(vocab, n_prompt, seed=11)
        cpu, t_cpu, _ = run_engine(REF_ENGINE, snap, prompt, n_new)
        gpu, t_gpu, _ = run_engine(OMC_ENGINE, snap, prompt, n_new)
        first = next((i for i, (a, b) in enumerate(zip(cpu, gpu)) if a != b), None)
        return {"model": "gemma-shaped random init", "layers": layers, "vocab": vocab, "D": D, "experts": E,
                "top_k": K, "moe_intermediate": MI, "prompt_tokens": n_prompt, "new_tokens": n_new,
                "cpu_tokens": cpu, "gpu_tokens": gpu, "matching": sum(a == b for a, b in zip(cpu, gpu)),
                "identical": cpu == gpu, "first_difference": first,
                "seconds": {"cpu_engine": round(t_cpu, 1), "gpu_engine": round(t_gpu, 1)}}
    finally:
        if own:
            shutil.rmtree(workdir, ignore_errors=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--vocab", type=int, default=4096)
    ap.add_argument("--prompt", type=int, default=24)
    ap.add_argument("--new", type=int, default=16)
    ap.add_argument("--workdir", default=None)
    a = ap.parse_args()
    print(json.dumps(compare(a.layers, a.vocab, a.prompt, a.new, a.workdir)), flush=True)


if __name__ == "__main__":
    main()
