"""End-to-end OLMoE greedy generation: the reference engine on the CPU against
the same engine with its MoE layer on the GPU (test infrastructure).

A seeded random-init OLMoE snapshot is written in the engine's own container
format (config.json + safetensors: f32 dense tensors, int8 expert rows with
f32 `.qs` row scales, the container fast path of engines/olmoe.c:237-247).
Weights are N(0, 0.02) from the oracle's SplitMix64/Box-Muller generator;
expert matrices are quantised with the converter rule
(tools/convert_olmoe.py:32-38, oracle `quantize_py`); norms are ones.

Then two builds of the unmodified engines/olmoe.c generate greedily from the
same prompt (engines/olmoe.c:429-451, main :548-586):
  oracle/_ref/olmoe       the reference, all host cores (OpenMP)
  oracle/_ref/olmoe_omc   the same engine with moe() hooked to libomc
                          (include/omc_engine_hook.h): level 2, the whole
                          MoE block on the GPU at every step
  oracle/_ref/olmoe_metal the unmodified engine built for its own GPU seam
                          (-DOM_METAL, include/om_metal.h): level 1, the
                          prefill's attention projections (omm_dense) and
                          MoE union (omm_moe) on the GPU, decode on the CPU
and their tokens are compared.  The engine's expert cache is given every
expert of a layer (no LRU eviction).

CLI (the C0 configuration: 16 layers, vocab 50304, 32 prompt + 64 new):
    python tests/e2e_olmoe.py --layers 16 --vocab 50304 --new 64 [--path gemv]
prints one JSON line.  The pytest in test_e2e_gpu.py runs a smaller model.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
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
REF_ENGINE = os.path.join(ROOT, "oracle", "_ref", "olmoe")
OMC_ENGINE = os.path.join(ROOT, "oracle", "_ref", "olmoe_omc")
METAL_ENGINE = os.path.join(ROOT, "oracle", "_ref", "olmoe_metal")

# OLMoE-1B-7B shape (the C0 configuration)
D, NH, E, K, I = 2048, 16, 64, 8, 1024


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle
    return pyoracle


class SafetensorsWriter:
    """Writes tensors whose shapes and dtypes are declared up front, one at a
    time, so a layer never has to be held in memory whole."""

    def __init__(self, path: str, specs):
        self.f = open(path, "wb")
        self.specs = list(specs)          # [(name, dtype, shape)]
        header, off = {}, 0
        for name, dt, shape in self.specs:
            n = int(np.prod(shape)) * np.dtype(dt).itemsize
            header[name] = {"dtype": {np.dtype(np.float32): "F32", np.dtype(np.int8): "I8"}[np.dtype(dt)],
                            "shape": list(shape), "data_offsets": [off, off + n]}
            off += n
        h = json.dumps(header).encode()
        h += b" " * ((8 - len(h) % 8) % 8)
        self.f.write(len(h).to_bytes(8, "little"))
        self.f.write(h)
        self.i = 0

    def put(self, name: str, a: np.ndarray):
        want = self.specs[self.i]
        assert name == want[0] and a.dtype == np.dtype(want[1]) and tuple(a.shape) == tuple(want[2]), name
        self.f.write(np.ascontiguousarray(a).tobytes())
        self.i += 1

    def close(self):
        assert self.i == len(self.specs)
        self.f.close()


def _seed(base: int, layer: int, idx: int) -> int:
    return (base * 1_000_003 + (layer + 1) * 10_007 + idx) & 0xFFFFFFFFFFFF


def _write_layer(args):
    snap, layer, seed = args
    P = _oracle()
    p = f"model.layers.{layer}."
    specs = [(p + "input_layernorm.weight", np.float32, (D,)),
             (p + "post_attention_layernorm.weight", np.float32, (D,))]
    for nm in ("q", "k", "v", "o"):
        specs.append((p + f"self_attn.{nm}_proj.weight", np.float32, (D, D)))
    specs += [(p + "self_attn.q_norm.weight", np.float32, (D,)),
              (p + "self_attn.k_norm.weight", np.float32, (D,)),
              (p + "mlp.gate.weight", np.float32, (E, D))]
    for e in range(E):
        for nm, shape in (("gate_proj", (I, D)), ("up_proj", (I, D)), ("down_proj", (D, I))):
            w = p + f"mlp.experts.{e}.{nm}.weight"
            specs += [(w, np.int8, shape), (w + ".qs", np.float32, (shape[0],))]
    wr = SafetensorsWriter(os.path.join(snap, f"model-{layer + 1:05d}.safetensors"), specs)
    idx = 0
    ones = np.ones(D, np.float32)
    for name, dt, shape in specs:
        if name.endswith(".qs"):
            continue                      # written with its matrix
        if "layernorm" in name or name.endswith("_norm.weight"):
            wr.put(name, ones)
        elif np.dtype(dt) == np.float32:
            wr.put(name, P.normal(_seed(seed, layer, idx), shape, 0.02))
        else:
            q, s = P.quantize_py(P.normal(_seed(seed, layer, idx), shape, 0.02))
            wr.put(name, q)
            wr.put(name + ".qs", s)
        idx += 1
    wr.close()
    return layer


def make_snapshot(snap: str, layers: int, vocab: int, seed: int = 2024, workers: int = 0) -> None:
    """Writes the random-init OLMoE snapshot into directory `snap`."""
    P = _oracle()
    os.makedirs(snap, exist_ok=True)
    cfg = {"hidden_size": D, "num_hidden_layers": layers, "num_attention_heads": NH,
           "num_key_value_heads": NH, "num_experts": E, "num_experts_per_tok": K,
           "intermediate_size": I, "vocab_size": vocab, "rope_theta": 10000.0,
           "rms_norm_eps": 1e-5, "norm_topk_prob": False, "eos_token_id": -1}
    with open(os.path.join(snap, "config.json"), "w") as f:
        json.dump(cfg, f)
    wr = SafetensorsWriter(os.path.join(snap, "model-00000.safetensors"),
                           [("model.embed_tokens.weight", np.float32, (vocab, D)),
                            ("lm_head.weight", np.float32, (vocab, D)),
                            ("model.norm.weight", np.float32, (D,))])
    wr.put("model.embed_tokens.weight", P.normal(_seed(seed, -1, 0), (vocab, D), 0.02))
    wr.put("lm_head.weight", P.normal(_seed(seed, -1, 1), (vocab, D), 0.02))
    wr.put("model.norm.weight", np.ones(D, np.float32))
    wr.close()
    workers = workers or min(layers, os.cpu_count() or 4, 16)
    jobs = [(snap, li, seed) for li in range(layers)]
    if workers > 1:
        with mp.get_context("spawn").Pool(workers) as pool:
            for _ in pool.imap_unordered(_write_layer, jobs):
                pass
    else:
        for j in jobs:
            _write_layer(j)


def prompt_ids(vocab: int, n: int, seed: int = 7) -> list:
    """n token ids uniform in [0, vocab) (numpy PCG64, seed recorded here)."""
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def run_engine(binary: str, snap: str, prompt: list, n_new: int, env_extra=None, timeout=3600):
    """Runs the engine's greedy generation; returns (new tokens, seconds, log)."""
    with tempfile.TemporaryDirectory() as td:
        ref = os.path.join(td, "ref.json")
        with open(ref, "w") as f:
            json.dump({"prompt_ids": prompt, "full_ids": prompt + [0] * n_new}, f)
        env = dict(os.environ, SNAP=snap)
        env.update(env_extra or {})
        t0 = time.perf_counter()
        p = subprocess.run([binary, str(E), "8", ref], env=env, capture_output=True, text=True, timeout=timeout)
        dt = time.perf_counter() - t0
    log = p.stdout + p.stderr
    if p.returncode != 0:
        raise RuntimeError(f"{binary} exited {p.returncode}:\n{log[-3000:]}")
    m = re.search(r"C engine : ([0-9 ]+)", p.stdout)
    if not m:
        raise RuntimeError(f"no token line in the output of {binary}:\n{log[-3000:]}")
    return [int(t) for t in m.group(1).split()], dt, log


def compare(layers: int, vocab: int, n_prompt: int, n_new: int, path: str | None, workdir: str | None = None,
            level: int = 2, env_extra: dict | None = None):
    """Builds the snapshot, runs the CPU engine and the GPU one (level 2: the
    moe() hook; level 1: the engine's own omm_* seam), returns the result dict."""
    own = workdir is None
    workdir = workdir or tempfile.mkdtemp(prefix="olmoe_e2e_")
    snap = os.path.join(workdir, "snap")
    try:
        t0 = time.perf_counter()
        if not os.path.exists(os.path.join(snap, "config.json")):
            make_snapshot(snap, layers, vocab)
        t_gen = time.perf_counter() - t0
        prompt = prompt_ids(vocab, n_prompt)
        cpu, t_cpu, _ = run_engine(REF_ENGINE, snap, prompt, n_new)
        env = {"OMC_FFN_PATH": path} if path else {}
        env.update(env_extra or {})
        gpu, t_gpu, log = run_engine(OMC_ENGINE if level == 2 else METAL_ENGINE, snap, prompt, n_new, env)
        first_diff = next((i for i, (a, b) in enumerate(zip(cpu, gpu)) if a != b), None)
        return {"layers": layers, "vocab": vocab, "prompt_tokens": n_prompt, "new_tokens": n_new,
                "level": level, "expert_path": path or "auto", "prompt": prompt, "cpu_tokens": cpu, "gpu_tokens": gpu,
                "matching": sum(a == b for a, b in zip(cpu, gpu)), "identical": cpu == gpu,
                "first_difference": first_diff, "seconds": {"snapshot": round(t_gen, 1),
                                                            "cpu_engine": round(t_cpu, 1),
                                                            "gpu_engine": round(t_gpu, 1)},
                "cpu_threads": os.cpu_count()}
    finally:
        if own:
            shutil.rmtree(workdir, ignore_errors=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--vocab", type=int, default=50304)
    ap.add_argument("--prompt", type=int, default=32)
    ap.add_argument("--new", type=int, default=64)
    ap.add_argument("--path", default=None, choices=[None, "gemv", "mma"])
    ap.add_argument("--workdir", default=None, help="reuse a snapshot directory (kept)")
    ap.add_argument("--level", type=int, default=2, choices=[1, 2],
                    help="2: the moe() hook (olmoe_omc); 1: the engine's omm_* seam (olmoe_metal)")
    a = ap.parse_args()
    print(json.dumps(compare(a.layers, a.vocab, a.prompt, a.new, a.path, a.workdir, a.level)), flush=True)


if __name__ == "__main__":
    main()
