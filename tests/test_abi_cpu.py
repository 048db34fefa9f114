"""The C-ABI library loads without a GPU and exports every symbol its
headers declare; device acquisition fails with the reference's
AdapterUnavailable when no GPU is visible."""
import ctypes
import os
import re

import pytest

from hephaestus_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include", "heph")
    for f in os.listdir(inc):
        text = open(os.path.join(inc, f)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(heph_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_headers_declare_entry_points():
    names = declared_symbols()
    assert "heph_reduce_full" in names and "heph_scan_axis" in names
    assert len(names) >= 50


@pytest.mark.parametrize("name", declared_symbols())
def test_symbol_exported(name):
    assert hasattr(N.lib, name), f"{name} declared in include/heph but not exported"


def test_binding_table_covers_headers():
    bound = {n for n, _, _ in N.SIGNATURES}
    assert set(declared_symbols()) == bound


def test_library_targets_sm100a_only():
    # The build recipe compiles for exactly one architecture.
    import importlib.util
    spec = importlib.util.spec_from_file_location("_b", os.path.join(ROOT, "hephaestus_b200", "build.py"))
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_no_gpu_is_adapter_unavailable():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    h = ctypes.c_void_p()
    assert N.lib.heph_device_open(0, ctypes.byref(h)) == N.ADAPTER_UNAVAILABLE
    n = ctypes.c_int(-1)
    assert N.lib.heph_device_count(ctypes.byref(n)) == N.OK and n.value == 0


def test_status_names_are_reference_prefixes():
    # HephaestusError Display strings, core error.rs:10-52
    assert N.lib.heph_status_name(N.DISPATCH_FAILED) == b"kernel dispatch failed"
    assert N.lib.heph_status_name(N.TRANSFER_FAILED) == b"device transfer failed"
    assert N.lib.heph_dtype_size(N.F64) == 8 and N.lib.heph_dtype_size(N.U32) == 4
