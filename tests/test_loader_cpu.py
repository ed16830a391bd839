"""CPU: the container index and reader behind omc_experts_load (the
safetensors shards the converters write, tools/convert_olmoe.py:93-99):
tensors come back byte for byte from every shard, whatever the header holds
besides them; a missing name or a too-small buffer is refused."""
import ctypes as C
import json
import os

import numpy as np

from e2e_olmoe import SafetensorsWriter


def _write(path, tensors, metadata=None):
    wr = SafetensorsWriter(path, [(n, a.dtype, a.shape) for n, a in tensors])
    for n, a in tensors:
        wr.put(n, a)
    wr.close()
    if metadata is not None:   # rewrite the header with a __metadata__ entry in front
        raw = open(path, "rb").read()
        hl = int.from_bytes(raw[:8], "little")
        h = json.loads(raw[8:8 + hl])
        h2 = {"__metadata__": metadata}
        h2.update(h)
        hb = json.dumps(h2).encode()
        hb += b" " * ((8 - len(hb) % 8) % 8)
        open(path, "wb").write(len(hb).to_bytes(8, "little") + hb + raw[8 + hl:])


def test_container_read_across_shards(omc_lib, oracle, tmp_path):
    rng = np.random.default_rng(3)
    a = rng.integers(-128, 128, (96, 64), dtype=np.int8)
    s = oracle.normal(1, (96,), 0.01)
    b = rng.integers(-128, 128, (64, 96), dtype=np.int8)
    _write(str(tmp_path / "model-00001.safetensors"),
           [("model.layers.0.mlp.experts.0.gate_proj.weight", a),
            ("model.layers.0.mlp.experts.0.gate_proj.weight.qs", s)], metadata={"format": "pt"})
    _write(str(tmp_path / "model-00002.safetensors"), [("model.layers.0.mlp.experts.0.down_proj.weight", b)])
    (tmp_path / "config.json").write_text("{}")
    lib = omc_lib.lib()
    for name, want in (("model.layers.0.mlp.experts.0.gate_proj.weight", a),
                       ("model.layers.0.mlp.experts.0.gate_proj.weight.qs", s),
                       ("model.layers.0.mlp.experts.0.down_proj.weight", b)):
        buf = np.zeros(want.nbytes, np.uint8)
        n = lib.omc_debug_container_read(str(tmp_path).encode(), name.encode(), buf.ctypes.data_as(C.c_void_p),
                                         buf.size)
        assert n == want.nbytes, omc_lib.last_error()
        assert np.array_equal(buf, np.frombuffer(want.tobytes(), np.uint8))
    buf = np.zeros(16, np.uint8)
    assert lib.omc_debug_container_read(str(tmp_path).encode(), b"no.such.tensor", buf.ctypes.data_as(C.c_void_p),
                                        16) == omc_lib.EINVAL
    assert lib.omc_debug_container_read(str(tmp_path).encode(), b"model.layers.0.mlp.experts.0.down_proj.weight",
                                        buf.ctypes.data_as(C.c_void_p), 16) == omc_lib.EINVAL
    assert lib.omc_debug_container_read(str(tmp_path / "missing").encode(), b"x", buf.ctypes.data_as(C.c_void_p),
                                        16) == omc_lib.EINVAL
