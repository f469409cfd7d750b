"""The C ABI without a GPU: the product library loads, exports every entry
point include/maxim_b200.h declares, and reports a missing device as an error
status (never a CPU fallback)."""
import ctypes
import os
import re
import subprocess

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


RUST_TYPES = {"i32": 4, "i64": 8, "f32": 4, "usize": 8}


def rust_struct(name):
    """Field names and byte sizes of a `#[repr(C)]` struct as INTEGRATION.md
    declares it for the Rust crate."""
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    m = re.search(r"pub struct %s \{(.*?)\}" % name, text, flags=re.S)
    assert m, name
    fields = []
    for fname, ftype in re.findall(r"pub (\w+):\s*([^,]+?)\s*(?:,|$)", m.group(1)):
        ftype = ftype.strip()
        arr = re.match(r"\[u8;\s*(\d+)\]", ftype)
        if arr:
            fields.append((fname, int(arr.group(1)), 1))
        elif ftype in RUST_TYPES:
            fields.append((fname, RUST_TYPES[ftype], RUST_TYPES[ftype]))
        else:
            fields.append((fname, 8, 8))  # pointers and nested 8-byte-aligned structs
    return fields


def rust_layout(fields):
    off, out, align = 0, [], 1
    for name, size, al in fields:
        off = (off + al - 1) // al * al
        out.append((name, off))
        off += size
        align = max(align, al)
    return out, (off + align - 1) // align * align


def c_layout(tmp_path, struct, fields):
    """sizeof and offsetof each field of a C struct from include/maxim_b200.h,
    as gcc lays it out."""
    src = tmp_path / "layout.c"
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "maxim_b200.h"', "int main(void) {",
             '  printf("%%zu\\n", sizeof(%s));' % struct]
    lines += ['  printf("%%zu\\n", offsetof(%s, %s));' % (struct, f) for f in fields]
    lines += ["  return 0;", "}"]
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    return vals[0], vals[1:]


@pytest.mark.parametrize("rust,c", [("MxGpuStats", "mx_gpu_stats"), ("MxOp", "mx_op"), ("MxBuf", "mx_buf")])
def test_integration_rust_structs_match_the_c_abi(tmp_path, rust, c):
    """The Rust declarations a maintainer copies from INTEGRATION.md must have
    the C structs' exact fields, offsets and size: the library writes whole
    structs (mx_gpu_get_stats memsets sizeof(mx_gpu_stats) bytes)."""
    fields = rust_struct(rust)
    names = [f[0] for f in fields]
    layout, size = rust_layout(fields)
    c_size, c_offs = c_layout(tmp_path, c, names)
    assert size == c_size, (rust, size, c_size)
    assert [o for _, o in layout] == c_offs


def test_binding_stats_struct_matches_the_c_abi(mx, tmp_path):
    names = [f[0] for f in mx._native.mx_gpu_stats._fields_]
    c_size, c_offs = c_layout(tmp_path, "mx_gpu_stats", names)
    assert ctypes.sizeof(mx._native.mx_gpu_stats) == c_size
    assert [getattr(mx._native.mx_gpu_stats, n).offset for n in names] == c_offs
