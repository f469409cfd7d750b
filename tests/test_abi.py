"""The C ABI without a GPU: the product library loads, exports every entry
point include/maxim_b200.h declares, and reports a missing device as an error
status (never a CPU fallback)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "maxim_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mx_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_executor_boundary():
    syms = declared_symbols()
    for s in ["mx_driver_ready", "mx_gpu_new", "mx_gpu_run", "mx_gpu_begin", "mx_gpu_step_op", "mx_gpu_read_buf",
              "mx_gpu_read_arena", "mx_gpu_set_timeline", "mx_gpu_timeline", "mx_gpu_get_stats", "mx_gpu_free",
              "mx_last_error"]:
        assert s in syms


def test_library_exports_every_declared_symbol(mx):
    lib = ctypes.CDLL(mx.lib()._name)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_the_header(mx):
    assert set(declared_symbols()) <= set(mx.exported_symbols())


def test_no_device_is_an_error_not_a_fallback(mx):
    if mx.device_count() > 0:
        pytest.skip("a CUDA device is visible")
    with pytest.raises(mx.MaximError):
        mx.driver_ready()
    plan = mx.Plan(variant="S-1", h=64, w=64)
    with pytest.raises(mx.MaximError):
        mx.Gpu(plan)
