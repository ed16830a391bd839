"""GPU: omc_moe_forward_noalloc, the forward entry that allocates nothing.

Callers that cannot allocate device memory per call (an engine with its HBM
budget fixed up front, or a serving loop that may not stall in the allocator
between tokens) use this entry; its workspace is a fixed static device array
instead of cudaMalloc'd memory.  Its output must equal the regular device
entry's, within the tests' tolerance, on two calls in a row (the second call
runs on the array the first one left behind).  This file is named so pytest
collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close, assert_weights
from gpu_common import next_layer_id, routing_exact

pytestmark = pytest.mark.gpu


def _run(gpu, lib_fn, layer, x_dev, out_dev, idx_dev, w_dev, stream):
    rc = lib_fn(layer, C.c_void_p(x_dev.data_ptr()), x_dev.shape[0], C.c_void_p(out_dev.data_ptr()),
                C.c_void_p(idx_dev.data_ptr()), C.c_void_p(w_dev.data_ptr()), C.c_void_p(stream))
    assert rc == 0, gpu.last_error()


@pytest.mark.parametrize("case", ["olmoe_T160", "qwen_T48", "olmoe_T3", "olmoe_T1", "qwen_T1"])
def test_noalloc_matches_device_entry_twice(gpu, oracle, case):
    """T=1 takes the fused decode kernel, whose routing and pieces then live in
    the static array too; it is also checked against the oracle."""
    import torch
    T = int(case.split("T")[1])
    if case.startswith("olmoe"):
        L = oracle.make_layer(oracle.FAMILY_OLMOE, 2048, 1024, 64, 8, seed=61)
    else:
        L = oracle.make_layer(oracle.FAMILY_QWEN, 2048, 512, 256, 8, seed=62, renorm=1, router_i8=1,
                              has_shared=1, Is=512)
    lid = next_layer_id()
    gpu.MoELayer.from_oracle_layer(lid, L)
    lib = gpu.lib()
    x = torch.from_numpy(oracle.normal(6100 + T, (T, L.D))).cuda()
    stream = torch.cuda.Stream()
    outs = {}
    for name, fn in (("dev", lib.omc_moe_forward_dev), ("noalloc1", lib.omc_moe_forward_noalloc),
                     ("noalloc2", lib.omc_moe_forward_noalloc)):
        out = torch.full((T, L.D), float("nan"), device="cuda")
        idx = torch.full((T, L.k), -1, dtype=torch.int32, device="cuda")
        w = torch.zeros((T, L.k), device="cuda")
        _run(gpu, fn, lid, x, out, idx, w, stream.cuda_stream)
        stream.synchronize()
        gpu.sync()
        outs[name] = (out.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy())
    ref_out, ref_idx, ref_w = outs["dev"]
    for name in ("noalloc1", "noalloc2"):
        o, i, w = outs[name]
        assert np.array_equal(i, ref_idx), name
        # the no-alloc entry always takes the exact router; the device entry
        # the bounded one from T = 16
        assert_weights(w, ref_w, routing_exact(gpu, L, T), name)
        assert_close(o, ref_out, what=name)
    if T == 1:
        ro, ridx, rw = oracle.oracle_moe(L, x.cpu().numpy())
        o, i, w = outs["noalloc2"]
        assert np.array_equal(i, ridx)
        assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
        assert_close(o, ro, what=f"{case} vs oracle")


@pytest.mark.parametrize("family,limit", [("olmoe", 238), ("qwen", 273)])
def test_noalloc_limit_is_exact(gpu, oracle, family, limit):
    """The largest T the static array holds is the one the header and the docs
    quote: T=limit runs, T=limit+1 is rejected with that bound."""
    import torch
    if family == "olmoe":
        L = oracle.make_layer(oracle.FAMILY_OLMOE, 2048, 1024, 64, 8, seed=64)
    else:
        L = oracle.make_layer(oracle.FAMILY_QWEN, 2048, 512, 256, 8, seed=65, renorm=1, router_i8=1,
                              has_shared=1, Is=512)
    lid = next_layer_id()
    gpu.MoELayer.from_oracle_layer(lid, L)
    x = torch.from_numpy(oracle.normal(6300, (limit + 1, L.D))).cuda()
    out = torch.zeros((limit + 1, L.D), device="cuda")
    fn = gpu.lib().omc_moe_forward_noalloc
    rc = fn(lid, C.c_void_p(x.data_ptr()), limit, C.c_void_p(out.data_ptr()), None, None, None)
    assert rc == 0, gpu.last_error()
    gpu.sync()
    rc = fn(lid, C.c_void_p(x.data_ptr()), limit + 1, C.c_void_p(out.data_ptr()), None, None, None)
    assert rc == gpu.EINVAL
    assert f"at most T={limit} " in gpu.last_error()


def test_noalloc_rejects_T_beyond_scratch(gpu, oracle):
    import torch
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 2048, 1024, 64, 8, seed=63)
    lid = next_layer_id()
    gpu.MoELayer.from_oracle_layer(lid, L)
    T = 4096
    x = torch.zeros((T, L.D), device="cuda")
    out = torch.zeros((T, L.D), device="cuda")
    rc = gpu.lib().omc_moe_forward_noalloc(lid, C.c_void_p(x.data_ptr()), T, C.c_void_p(out.data_ptr()),
                                           None, None, None)
    assert rc == gpu.EINVAL
    msg = gpu.last_error()
    assert "at most T=" in msg and "static scratch" in msg
