"""GPU failure detection without faulting the GPU.

A device wait that can never complete (an mbarrier nothing arrives on) must
end on its own time limit, come back to the host as OMC_ETIMEOUT, and leave
the context usable.  Bad arguments come back as OMC_EINVAL, never as a
device fault."""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close
from gpu_common import next_layer_id

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(gpu, oracle):
    rc = gpu.lib().omc_debug_wait_timeout()
    assert rc == gpu.ETIMEOUT, gpu.last_error()
    assert "site 90" in gpu.last_error()
    # the context still works
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 128, 64, 8, 2, seed=80)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    x = oracle.normal(81, (4, 128))
    out, idx, _ = m.forward(x)
    ro, ridx, _ = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert_close(out, ro)
    gpu.sync()


def test_invalid_arguments_are_rejected(gpu, oracle):
    lib = gpu.lib()
    d = gpu.MoEDesc(0, 100, 64, 8, 2, 0, 0, 0, 0)          # D not a multiple of 64
    r = np.zeros((8, 100), np.float32)
    assert lib.omc_layer_init(next_layer_id(), C.byref(d), r.ctypes.data_as(C.c_void_p), None) == gpu.EINVAL
    d = gpu.MoEDesc(0, 128, 64, 8, 9, 0, 0, 0, 0)          # k > E
    r = np.zeros((8, 128), np.float32)
    assert lib.omc_layer_init(next_layer_id(), C.byref(d), r.ctypes.data_as(C.c_void_p), None) == gpu.EINVAL
    assert lib.omc_moe_forward(99999, None, 1, None, None, None) == gpu.ENOINIT


def test_forward_before_experts_uploaded(gpu):
    lid = next_layer_id()
    d = gpu.MoEDesc(0, 128, 64, 8, 2, 0, 0, 0, 0)
    r = np.zeros((8, 128), np.float32)
    assert gpu.lib().omc_layer_init(lid, C.byref(d), r.ctypes.data_as(C.c_void_p), None) == 0
    x = np.zeros((2, 128), np.float32)
    out = np.zeros((2, 128), np.float32)
    rc = gpu.lib().omc_moe_forward(lid, x.ctypes.data_as(C.c_void_p), 2, out.ctypes.data_as(C.c_void_p),
                                   None, None)
    assert rc == gpu.ENOINIT


def test_misaligned_device_pointers_are_rejected(gpu, oracle):
    """The device entries move x and out rows with 16-byte bulk copies and
    vector stores: a pointer off a 16-byte boundary is refused on the host
    (OMC_EINVAL) before anything is launched."""
    import torch
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 128, 64, 8, 2, seed=82)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    buf = torch.zeros(4 * 128 + 4, dtype=torch.float32, device="cuda")
    out = torch.zeros(4 * 128 + 4, dtype=torch.float32, device="cuda")
    lib = gpu.lib()
    for fn in (lib.omc_moe_forward_dev, lib.omc_moe_forward_noalloc):
        rc = fn(m.layer, C.c_void_p(buf.data_ptr() + 4), 4, C.c_void_p(out.data_ptr()), None, None, None)
        assert rc == gpu.EINVAL, gpu.last_error()
        assert "16-byte aligned" in gpu.last_error()
        rc = fn(m.layer, C.c_void_p(buf.data_ptr()), 4, C.c_void_p(out.data_ptr() + 8), None, None, None)
        assert rc == gpu.EINVAL
    gpu.sync()
