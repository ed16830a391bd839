"""Writes tests/golden/qwen_tiny_i8/: the reference's tiny Qwen fixture model
(oracle/qwen_tiny) in the int8 container, made by the reference's own
converter (tools/convert_qwen.py: routed experts as int8 rows + ".qs" f32
row scales, everything else as it was), plus the reference's prompt and
greedy tokens for it (oracle/ref_qwen.json).  The Qwen engine runs such a
snapshot in stream mode (engines/qwen.c:215-218), the mode whose MoE layer
include/omc_qwen_hook.h moves to the GPU.

Needs the reference sources (REF_ROOT, or a directory named `reference`
beside this repository) and torch + safetensors, which the converter imports.
Run once; the GPU test compares the hooked engine's tokens with these.

    python tests/golden/make_qwen_tiny_i8.py
"""
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import pyoracle as P  # noqa: E402

OUT = os.path.join(HERE, "qwen_tiny_i8")


def main():
    ref = P.ref_root()
    if ref is None:
        sys.exit("the reference sources are needed: set REF_ROOT")
    with tempfile.TemporaryDirectory() as td:
        conv = os.path.join(td, "out")
        subprocess.run([sys.executable, os.path.join(ref, "tools", "convert_qwen.py"),
                        "--model", os.path.join(ref, "oracle", "qwen_tiny"), "--out", conv], check=True)
        os.makedirs(OUT, exist_ok=True)
        for f in ("config.json", "generation_config.json", "model.safetensors"):
            shutil.copyfile(os.path.join(conv, f), os.path.join(OUT, f))
    shutil.copyfile(os.path.join(ref, "oracle", "ref_qwen.json"), os.path.join(OUT, "ref_qwen.json"))
    # the CPU engine reproduces the reference's tokens on the converted model
    exe = os.path.join(ROOT, "oracle", "_ref", "qwen")
    if os.path.exists(exe):
        p = subprocess.run([exe, os.path.join(OUT, "ref_qwen.json")], env=dict(os.environ, SNAP=OUT),
                           capture_output=True, text=True, timeout=300)
        print(p.stdout.strip().splitlines()[-1])
        if "EXACT" not in p.stdout:
            sys.exit("the CPU engine does not reproduce ref_qwen.json on the converted model")
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
