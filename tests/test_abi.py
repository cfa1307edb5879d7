"""CPU tests of the C-ABI library: it builds, loads, exports every symbol that
include/*.h declares, and rejects bad arguments before touching the device."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", src, flags=re.M):
            name = m.group(1)
            if name not in ("if", "for", "while", "defined", "sizeof"):
                names.add(name)
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from kandiga_b200 import _native, build
    build()
    return _native.load()


def test_header_declares_entry_points():
    names = declared_functions()
    assert "bakan_cpu_expert_init" in names and "kq_moe_decode" in names
    assert len(names) >= 20


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_table_covers_header():
    from kandiga_b200 import _native
    assert set(declared_functions()) <= set(_native.SIGNATURES)


def test_argument_validation_without_device(lib):
    from kandiga_b200 import _native as N
    h = ctypes.c_void_p()
    assert lib.kq_table_create(None, ctypes.byref(h)) == 1
    d = N.kq_table_desc(1, 8, 2048, 512, 5, 64, 0, 0)  # 5-bit: unsupported
    assert lib.kq_table_create(ctypes.byref(d), ctypes.byref(h)) == 6
    d = N.kq_table_desc(1, 8, 2048, 500, 3, 64, 0, 0)  # inter not a multiple of 64
    assert lib.kq_table_create(ctypes.byref(d), ctypes.byref(h)) == 1
    assert lib.kq_router_topk(None, 1, 2000, 8, None, None, None) == 1  # E > 1024
    assert lib.kq_router_topk(None, 0, 256, 8, None, None, None) == 0   # empty input
    assert lib.kq_moe_decode(None, 0, None, 0, 1, None, None, None, 8, None, None, 0, None, None, 0,
                             None) == 1
    assert lib.kq_qmat_create(100, 512, 3, 0, 0, ctypes.byref(h)) == 1  # rows % 16
    m = (ctypes.c_float * 4)()
    assert lib.kq_tq_create(0, 2, 1, 4, m, m, ctypes.byref(h)) == 1     # head_dim 0
    assert lib.kq_tq_create(200, 2, 1, 4, m, m, ctypes.byref(h)) == 6   # head_dim above 128
    assert lib.kq_ep_create(0, 9, 16, 1024, 8, 0, ctypes.byref(h)) == 1  # more ranks than KQ_EP_MAX_RANKS
    assert lib.kq_ep_create(2, 2, 16, 1024, 8, 0, ctypes.byref(h)) == 1  # rank outside the group
    assert lib.kq_ep_buffer_bytes(2, 16, 1024, 8) > 2 * 2 * 16 * 1024 * 2
    assert lib.bakan_cpu_expert_num_layers(None) == 0
    assert lib.bakan_cpu_expert_mlp_f16(None, 0, None, None, 8, None) == -1


def test_integration_guide_lists_every_entry_point():
    """INTEGRATION.md's appendix gives the ctypes signature of every bound entry point."""
    from kandiga_b200 import _native
    guide = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    missing = [n for n in _native.SIGNATURES if f"\n{n}: " not in guide]
    assert not missing, missing


def test_product_package_does_not_import_oracle():
    for py in glob.glob(os.path.join(ROOT, "kandiga_b200", "**", "*.py"), recursive=True):
        src = open(py).read()
        assert "oracle" not in re.findall(r"^\s*(?:from|import)\s+(\w+)", src, flags=re.M), py
