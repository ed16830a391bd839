"""CPU: the C-ABI library loads and exports every symbol include/*.h declares,
and its host-side argument checks answer without a GPU."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("om_cuda.h", "om_metal.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**\s*\b(om[cm]_[a-z0-9_]+)\s*\(",
                             src, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_the_boundary():
    names = declared_functions()
    for want in ("omc_init", "omc_layer_init", "omc_expert_set", "omc_moe_forward",
                 "omc_moe_forward_dev", "omc_ep_init", "omm_init", "omm_alloc", "omm_moe",
                 "omm_moe_act", "omm_dense_q", "omm_dense"):
        assert want in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_symbol(omc_lib, name):
    L = C.CDLL(omc_lib.LIB_PATH)
    assert hasattr(L, name), f"libomc.so does not export {name}"


def test_python_binding_covers_header(omc_lib):
    for name in declared_functions():
        assert name in omc_lib.SIGNATURES


def test_host_checks_without_gpu(omc_lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    lib = omc_lib.lib()
    assert lib.omc_strerror(omc_lib.ETIMEOUT) == b"timeout"
    assert lib.omc_layer_init(0, None, None, None) == omc_lib.ENOINIT
    assert lib.omc_moe_forward(0, None, 1, None, None, None) == omc_lib.ENOINIT
    assert lib.omc_init(0, 0) != omc_lib.OK          # no device here
    assert lib.omc_last_error()
