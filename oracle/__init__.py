"""TEST INFRASTRUCTURE: the CPU oracle (a C++ restatement of the reference's
src/exec_cpu.rs, see oracle/exec_cpu.cpp). Only tests/, the smoke check and
bench.py's CPU-baseline and reference arms may use it, and only as the checker
or the timed CPU baseline - never as part of the product path.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libmaxim_oracle.so")
_lib = None


def _abi():
    # The ABI's ctypes declarations (pure Python: importing them maps no library).
    import importlib
    return importlib.import_module("maxim-rs_b200._native")


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("%s is missing: run `python maxim-rs_b200/build.py`" % LIB_PATH)
        A = _abi()
        L = ctypes.CDLL(LIB_PATH)
        vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
        sigs = {
            "mxo_run": (ctypes.c_int, [vp, vp, ctypes.c_int]),
            "mxo_run_range": (ctypes.c_int, [vp, vp, i32, i32, ctypes.c_int]),
            "mxo_run_bf16_storage": (ctypes.c_int, [vp, vp, ctypes.c_int]),
            "mxo_last_error": (sz, [ctypes.c_char_p, sz]),
            "mxo_param_spec": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, sz, ctypes.POINTER(sz)]),
            "mxo_weights_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(vp)]),
            "mxo_weights_free": (None, [vp]),
            "mxo_plan_build": (ctypes.c_int, [vp, i32, i32, ctypes.c_int, ctypes.POINTER(vp)]),
            "mxo_plan_free": (None, [vp]),
            "mxo_plan_view": (ctypes.POINTER(A.mx_plan), [vp]),
            "mxo_preprocess": (ctypes.c_int, [ctypes.POINTER(A.mx_image), i32, ctypes.POINTER(A.mx_image),
                                              ctypes.POINTER(i32), ctypes.POINTER(i32)]),
            "mxo_image_free": (None, [ctypes.POINTER(A.mx_image)]),
        }
        for name, (res, args) in sigs.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _lib = L
    return _lib


def _check(rc, what):
    if rc != 0:
        buf = ctypes.create_string_buffer(4096)
        lib().mxo_last_error(buf, len(buf))
        raise RuntimeError("%s: %s" % (what, buf.value.decode(errors="replace")))


def param_spec(variant):
    """[(name, shape)] of a `variant` checkpoint, from the oracle's own builder."""
    need = ctypes.c_size_t()
    _check(lib().mxo_param_spec(variant.encode(), None, 0, ctypes.byref(need)), "param spec")
    buf = ctypes.create_string_buffer(need.value)
    _check(lib().mxo_param_spec(variant.encode(), buf, need.value, None), "param spec")
    out = []
    for line in buf.value.decode().splitlines():
        name, shape = line.split("\t")
        out.append((name, tuple(int(x) for x in shape.split(","))))
    return out


class HostPlan:
    """A plan built by the oracle library's own copy of the plan builder, for
    CPU-only runs that must not map the GPU product library. It has the
    attributes `run` / `take` / `output` use (view, arena_len, input, output,
    buf, off)."""

    def __init__(self, checkpoint_path, h, w, dumps=False):
        self._w = ctypes.c_void_p()
        _check(lib().mxo_weights_open(os.fsencode(checkpoint_path), ctypes.byref(self._w)), checkpoint_path)
        self._h = ctypes.c_void_p()
        _check(lib().mxo_plan_build(self._w, h, w, int(dumps), ctypes.byref(self._h)), "plan")
        self.view = lib().mxo_plan_view(self._h)
        v = self.view.contents
        self.n_ops, self.n_bufs, self.arena_len = v.n_ops, v.n_bufs, v.arena_len
        self.input, self.output = v.input, v.output
        self.shape = (v.shape.c, v.shape.h, v.shape.w)

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                lib().mxo_plan_free(self._h)
                self._h = None
            if getattr(self, "_w", None):
                lib().mxo_weights_free(self._w)
                self._w = None
        except Exception:  # interpreter shutdown: the module's globals may already be gone
            pass

    def buf(self, i):
        b = self.view.contents.bufs[i]
        return (b.c, b.h, b.w)

    def off(self, i):
        return self.view.contents.offs[i]

    def ops(self):
        v = self.view.contents
        return [v.ops[i] for i in range(v.n_ops)]


def preprocess(a, factor=64):
    """`image::preprocess` (src/image.rs:171-207) through the oracle library."""
    A = _abi()
    a = np.ascontiguousarray(a, dtype=np.float32)
    img = A.mx_image(a.shape[0], a.shape[1], a.shape[2], a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    out = A.mx_image()
    eh, ew = ctypes.c_int32(), ctypes.c_int32()
    _check(lib().mxo_preprocess(ctypes.byref(img), factor, ctypes.byref(out), ctypes.byref(eh), ctypes.byref(ew)),
           "preprocess")
    r = np.ctypeslib.as_array(out.data, shape=(out.c, out.h, out.w)).copy()
    lib().mxo_image_free(ctypes.byref(out))
    return r, (eh.value, ew.value)


def new_arena(plan, image):
    """A zeroed arena with `image` ([3][H][W]) placed at the plan's input buffer."""
    arena = np.zeros(plan.arena_len, np.float32)
    o = plan.off(plan.input)
    x = np.ascontiguousarray(image, np.float32).reshape(-1)
    arena[o:o + x.size] = x
    return arena


def run(plan, image, threads=0, arena=None):
    """Run the whole plan on the CPU; returns the arena."""
    if arena is None:
        arena = new_arena(plan, image)
    rc = lib().mxo_run(ctypes.cast(plan.view, ctypes.c_void_p), arena.ctypes.data_as(ctypes.c_void_p), threads)
    if rc != 0:
        raise RuntimeError("oracle run failed (%d)" % rc)
    return arena


def run_range(plan, arena, first, last, threads=0):
    rc = lib().mxo_run_range(ctypes.cast(plan.view, ctypes.c_void_p), arena.ctypes.data_as(ctypes.c_void_p),
                             first, last, threads)
    if rc != 0:
        raise RuntimeError("oracle run_range failed (%d)" % rc)
    return arena


def take(plan, arena, buf_id):
    """Buffer `buf_id` as [c][h][w] from a CPU arena."""
    c, h, w = plan.buf(buf_id)
    o = plan.off(buf_id)
    return arena[o:o + c * h * w].reshape(c, h, w).copy()


def output(plan, image, threads=0):
    return take(plan, run(plan, image, threads), plan.output)


def output_bf16_storage(plan, image, threads=0):
    """The plan's output with every activation rounded to bfloat16 as it is
    written (a what-if for bf16 activation storage, not the reference)."""
    arena = new_arena(plan, image)
    rc = lib().mxo_run_bf16_storage(ctypes.cast(plan.view, ctypes.c_void_p), arena.ctypes.data_as(ctypes.c_void_p),
                                    threads)
    if rc != 0:
        raise RuntimeError("oracle bf16-storage run failed (%d)" % rc)
    return take(plan, arena, plan.output)
