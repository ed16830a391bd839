"""End-to-end Qwen greedy generation: the reference engine on the CPU against
the same engine with its MoE layer on the GPU (test infrastructure).

Two models, both in the engine's int8 container (stream mode,
engines/qwen.c:215-218: routed experts as int8 rows + f32 ".qs" scales,
everything else f32):

* the reference's own tiny fixture model (oracle/qwen_tiny) converted by the
  reference's converter (tools/convert_qwen.py), committed as
  tests/golden/qwen_tiny_i8/ by tests/golden/make_qwen_tiny_i8.py together
  with the reference's prompt and greedy tokens (oracle/ref_qwen.json);
* a seeded random-init Qwen3.6-35B-A3B-shaped model (hidden 2048, 256 routed
  experts top-8 of FFN 512, a shared expert of FFN 512 behind its sigmoid
  gate; gated-DeltaNet layers with a full-attention layer every fourth),
  written here: matrices N(0, 0.02) from the oracle's generator, expert
  matrices quantised with the converter rule (tools/convert_qwen.py:22-26,
  oracle `quantize_py`), norm weights 0 (the engine's rmsnorm scales by
  1 + w, engines/qwen.c:147-151), A_log and dt_bias 0.

Two builds of the unmodified engines/qwen.c generate greedily from the same
prompt (main, engines/qwen.c:606-648: the prompt token by token, then greedy
decoding; every token goes through moe_step):
  oracle/_ref/qwen       the reference, all host cores (OpenMP)
  oracle/_ref/qwen_omc   the same engine with moe_step hooked to libomc
                         (include/omc_qwen_hook.h): the whole MoE block of
                         every token on the GPU
and their tokens are compared.

CLI:  python tests/e2e_qwen.py [--model tiny|shaped] [--layers 4 --new 16]
prints one JSON line.
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

REF_ENGINE = os.path.join(ROOT, "oracle", "_ref", "qwen")
OMC_ENGINE = os.path.join(ROOT, "oracle", "_ref", "qwen_omc")
TINY = os.path.join(HERE, "golden", "qwen_tiny_i8")

# Qwen3.6-35B-A3B-shaped dimensions (fewer layers and a smaller vocabulary)
SHAPED = dict(hidden_size=2048, num_attention_heads=16, num_key_value_heads=2, head_dim=256,
              linear_num_key_heads=16, linear_num_value_heads=32, linear_key_head_dim=128,
              linear_value_head_dim=128, linear_conv_kernel_dim=4, num_experts=256, num_experts_per_tok=8,
              moe_intermediate_size=512, shared_expert_intermediate_size=512, full_attention_interval=4,
              partial_rotary_factor=0.25, rms_norm_eps=1e-6)


def _specs(cfg: dict, layer: int):
    D = cfg["hidden_size"]
    p = f"model.layers.{layer}."
    f32, i8 = np.float32, np.int8
    s = [(p + "input_layernorm.weight", f32, (D,)), (p + "post_attention_layernorm.weight", f32, (D,))]
    if (layer + 1) % cfg["full_attention_interval"] == 0:
        H, KV, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
        s += [(p + "self_attn.q_proj.weight", f32, (H * hd * 2, D)), (p + "self_attn.k_proj.weight", f32, (KV * hd, D)),
              (p + "self_attn.v_proj.weight", f32, (KV * hd, D)), (p + "self_attn.o_proj.weight", f32, (D, H * hd)),
              (p + "self_attn.q_norm.weight", f32, (hd,)), (p + "self_attn.k_norm.weight", f32, (hd,))]
    else:
        kh, vh = cfg["linear_num_key_heads"], cfg["linear_num_value_heads"]
        kd, vd, ck = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"], cfg["linear_conv_kernel_dim"]
        conv = 2 * kh * kd + vh * vd
        q = p + "linear_attn."
        s += [(q + "in_proj_qkv.weight", f32, (conv, D)), (q + "in_proj_z.weight", f32, (vh * vd, D)),
              (q + "in_proj_b.weight", f32, (vh, D)), (q + "in_proj_a.weight", f32, (vh, D)),
              (q + "conv1d.weight", f32, (conv, 1, ck)), (q + "A_log", f32, (vh,)), (q + "dt_bias", f32, (vh,)),
              (q + "norm.weight", f32, (vd,)), (q + "out_proj.weight", f32, (D, vh * vd))]
    E, I, Is = cfg["num_experts"], cfg["moe_intermediate_size"], cfg["shared_expert_intermediate_size"]
    s += [(p + "mlp.gate.weight", f32, (E, D)), (p + "mlp.shared_expert.gate_proj.weight", f32, (Is, D)),
          (p + "mlp.shared_expert.up_proj.weight", f32, (Is, D)),
          (p + "mlp.shared_expert.down_proj.weight", f32, (D, Is)),
          (p + "mlp.shared_expert_gate.weight", f32, (1, D))]
    for e in range(E):
        for nm, shape in (("gate_proj", (I, D)), ("up_proj", (I, D)), ("down_proj", (D, I))):
            w = p + f"mlp.experts.{e}.{nm}.weight"
            s += [(w, i8, shape), (w + ".qs", f32, (shape[0],))]
    return s


def make_shaped_snapshot(snap: str, layers: int, vocab: int, seed: int = 3131) -> None:
    """Writes the random-init Qwen-shaped int8 container into `snap`."""
    P = _oracle()
    os.makedirs(snap, exist_ok=True)
    cfg = dict(SHAPED, architectures=["Qwen3_5MoeForCausalLM"], num_hidden_layers=layers, vocab_size=vocab,
               rope_parameters={"rope_theta": 10000000, "partial_rotary_factor": SHAPED["partial_rotary_factor"]})
    with open(os.path.join(snap, "config.json"), "w") as f:
        json.dump(cfg, f)
    D = cfg["hidden_size"]
    wr = SafetensorsWriter(os.path.join(snap, "model-00000.safetensors"),
                           [("model.embed_tokens.weight", np.float32, (vocab, D)),
                            ("lm_head.weight", np.float32, (vocab, D)),
                            ("model.norm.weight", np.float32, (D,))])
    wr.put("model.embed_tokens.weight", P.normal(_seed(seed, -1, 0), (vocab, D), 0.02))
    wr.put("lm_head.weight", P.normal(_seed(seed, -1, 1), (vocab, D), 0.02))
    wr.put("model.norm.weight", np.zeros(D, np.float32))
    wr.close()
    for li in range(layers):
        specs = _specs(cfg, li)
        wr = SafetensorsWriter(os.path.join(snap, f"model-{li + 1:05d}.safetensors"), specs)
        for idx, (name, dt, shape) in enumerate(specs):
            if name.endswith(".qs"):
                continue                   # written with its matrix
            if "norm" in name or name.endswith("A_log") or name.endswith("dt_bias"):
                wr.put(name, np.zeros(shape, np.float32))
            elif np.dtype(dt) == np.float32:
                wr.put(name, P.normal(_seed(seed, li, idx), shape, 0.02))
            else:
                q, s = P.quantize_py(P.normal(_seed(seed, li, idx), shape, 0.02))
                wr.put(name, q)
                wr.put(name + ".qs", s)
        wr.close()


def run_engine(binary: str, snap: str, prompt: list, n_new: int, env_extra=None, timeout=1800):
    """The engine's greedy generation (its validation main); returns (new tokens, seconds, log)."""
    with tempfile.TemporaryDirectory() as td:
        ref = os.path.join(td, "ref.json")
        with open(ref, "w") as f:
            json.dump({"prompt_ids": prompt, "full_ids": prompt + [0] * n_new}, f)
        env = dict(os.environ, SNAP=snap)
        env.update(env_extra or {})
        t0 = time.perf_counter()
        p = subprocess.run([binary, ref], env=env, capture_output=True, text=True, timeout=timeout, cwd=td)
        dt = time.perf_counter() - t0
    log = p.stdout + p.stderr
    m = re.search(r"engine   : ([0-9 ]+)", p.stdout)
    if not m:
        raise RuntimeError(f"no token line in the output of {binary} (exit {p.returncode}):\n{log[-3000:]}")
    toks = [int(t) for t in m.group(1).split()]
    if len(toks) != n_new:
        raise RuntimeError(f"{binary} gave {len(toks)} of {n_new} tokens:\n{log[-3000:]}")
    return toks, dt, log


def compare(model: str = "shaped", layers: int = 4, vocab: int = 4096, n_prompt: int = 16, n_new: int = 16,
            workdir: str | None = None, env_extra: dict | None = None):
    """Runs the CPU engine and the hooked one on the same snapshot and prompt."""
    own = workdir is None
    workdir = workdir or tempfile.mkdtemp(prefix="qwen_e2e_")
    try:
        t0 = time.perf_counter()
        if model == "tiny":
            snap = TINY
            ref = json.load(open(os.path.join(TINY, "ref_qwen.json")))
            prompt = list(ref["prompt_ids"])
            n_new = len(ref["full_ids"]) - len(prompt)
            expected = list(ref["full_ids"][len(prompt):])
        else:
            snap = os.path.join(workdir, "snap")
            if not os.path.exists(os.path.join(snap, "config.json")):
                make_shaped_snapshot(snap, layers, vocab)
            prompt = prompt_ids(vocab, n_prompt, seed=17)
            expected = None
        t_gen = time.perf_counter() - t0
        cpu, t_cpu, _ = run_engine(REF_ENGINE, snap, prompt, n_new)
        gpu, t_gpu, _ = run_engine(OMC_ENGINE, snap, prompt, n_new, env_extra)
        first_diff = next((i for i, (a, b) in enumerate(zip(cpu, gpu)) if a != b), None)
        r = {"model": model, "layers": layers if model != "tiny" else 8, "prompt_tokens": len(prompt),
             "new_tokens": n_new, "prompt": prompt, "cpu_tokens": cpu, "gpu_tokens": gpu,
             "matching": sum(a == b for a, b in zip(cpu, gpu)), "identical": cpu == gpu,
             "first_difference": first_diff,
             "seconds": {"snapshot": round(t_gen, 1), "cpu_engine": round(t_cpu, 1), "gpu_engine": round(t_gpu, 1)},
             "cpu_threads": os.cpu_count()}
        if expected is not None:
            r["reference_tokens"] = expected
            r["gpu_equals_reference_fixture"] = gpu == expected
        return r
    finally:
        if own:
            shutil.rmtree(workdir, ignore_errors=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="shaped", choices=["tiny", "shaped"])
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--vocab", type=int, default=4096)
    ap.add_argument("--prompt", type=int, default=16)
    ap.add_argument("--new", type=int, default=16)
    ap.add_argument("--workdir", default=None, help="reuse a snapshot directory (kept)")
    a = ap.parse_args()
    print(json.dumps(compare(a.model, a.layers, a.vocab, a.prompt, a.new, a.workdir)), flush=True)


if __name__ == "__main__":
    main()
