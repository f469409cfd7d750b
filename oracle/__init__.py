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


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("%s is missing: run `python maxim-rs_b200/build.py`" % LIB_PATH)
        L = ctypes.CDLL(LIB_PATH)
        L.mxo_run.restype = ctypes.c_int
        L.mxo_run.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.mxo_run_range.restype = ctypes.c_int
        L.mxo_run_range.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int]
        _lib = L
    return _lib


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
