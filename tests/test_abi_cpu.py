"""CPU: the C-ABI libraries load and export every symbol include/moe_cuda.h
and include/moe_host.h declare; host-side error paths (no GPU here)."""
import os
import re

import pytest

import moe_cuda as mc

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "moe_cuda.h")


def declared(hdr=HDR):
    src = open(hdr).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "typedef")))


def test_header_lists_expected_entry_points():
    assert set(declared()) == set(mc.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = mc.lib()
    for name in declared():
        assert hasattr(lib, name), name


def test_host_driver_exports_every_declared_symbol():
    import moe_host as mh
    names = declared(os.path.join(os.path.dirname(HDR), "moe_host.h"))
    assert set(names) == set(mh.EXPORTS)
    lib = mh.lib()
    for name in names:
        assert hasattr(lib, name), name


def test_model_surface_exports_every_declared_symbol():
    import moe_host as mh
    names = declared(os.path.join(os.path.dirname(HDR), "moe_model.h"))
    assert set(names) == set(mh.MODEL_EXPORTS)
    lib = mh.lib()
    for name in names:
        assert hasattr(lib, name), name


def test_calls_before_init_fail_loudly():
    import numpy as np
    lib = mc.lib()
    rc = lib.moe_cuda_free_layer(123)
    assert rc != 0
    x = np.zeros((1, 16), np.float32)
    with pytest.raises(mc.MoeError):
        mc.check(lib.moe_ffn(0, mc._p(x), mc._p(x), 1, None, None, mc.HOST_PTRS, None))


def test_bad_ep_group_rejected():
    lib = mc.lib()
    assert lib.moe_cuda_init(0, 2, 5, None) == mc.MOE_ERR_INVALID
    assert b"expert-parallel" in lib.moe_cuda_last_error()
