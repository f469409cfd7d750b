"""ctypes binding of libmaxim_b200.so (declared in include/maxim_b200.h).

The library is the product: the GPU executor behind the reference's
`exec_gpu::Gpu` interface (src/exec_gpu.rs:48-357) and the C++ restatement of
the reference's host contract (weights, config, plan builder, image pipeline).
This module only marshals arguments; it performs no computation of its own.
Loading fails loudly when the library has not been built.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmaxim_b200.so")

MX_OK = 0
OP_NAMES = ["copy", "add", "mul", "gate_apply", "gelu", "lrelu", "sigmoid", "chan_ln", "chan_mean", "chan_scale",
            "conv1x1", "conv3x3", "conv4x4s2", "convt2x2", "gate_mm", "block_perm", "resize", "down_s"]


class mx_op(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("dst", ctypes.c_int32), ("src", ctypes.c_int32),
                ("src2", ctypes.c_int32), ("tmp", ctypes.c_int32), ("w", ctypes.c_int32), ("wt", ctypes.c_int32),
                ("bias", ctypes.c_int32), ("scale", ctypes.c_int32), ("n", ctypes.c_int64),
                ("c", ctypes.c_int32), ("c_in", ctypes.c_int32), ("c_out", ctypes.c_int32), ("h", ctypes.c_int32),
                ("wd", ctypes.c_int32), ("oh", ctypes.c_int32), ("ow", ctypes.c_int32),
                ("pad_top", ctypes.c_int32), ("pad_left", ctypes.c_int32), ("outer", ctypes.c_int32),
                ("inner", ctypes.c_int32), ("mode", ctypes.c_int32), ("gh", ctypes.c_int32), ("gw", ctypes.c_int32),
                ("fh", ctypes.c_int32), ("fw", ctypes.c_int32), ("swap", ctypes.c_int32),
                ("forward", ctypes.c_int32), ("stride", ctypes.c_int32), ("off", ctypes.c_int32),
                ("hin", ctypes.c_int32), ("win", ctypes.c_int32), ("hout", ctypes.c_int32),
                ("wout", ctypes.c_int32), ("hw", ctypes.c_int64), ("slope", ctypes.c_float)]


class mx_buf(ctypes.Structure):
    _fields_ = [("c", ctypes.c_int64), ("h", ctypes.c_int64), ("w", ctypes.c_int64)]


class mx_plan(ctypes.Structure):
    _fields_ = [("n_bufs", ctypes.c_int32), ("bufs", ctypes.POINTER(mx_buf)), ("offs", ctypes.POINTER(ctypes.c_int64)),
                ("alias_parent", ctypes.POINTER(ctypes.c_int32)), ("alias_delta", ctypes.POINTER(ctypes.c_int64)),
                ("n_ops", ctypes.c_int32), ("ops", ctypes.POINTER(mx_op)), ("n_weights", ctypes.c_int32),
                ("weights", ctypes.POINTER(ctypes.POINTER(ctypes.c_float))),
                ("weight_lens", ctypes.POINTER(ctypes.c_int64)), ("arena_len", ctypes.c_int64),
                ("input", ctypes.c_int32), ("output", ctypes.c_int32), ("shape", mx_buf)]


class mx_gpu_stats(ctypes.Structure):
    _fields_ = [("device_name", ctypes.c_char * 128), ("arena_bytes", ctypes.c_int64),
                ("weight_bytes", ctypes.c_int64), ("pool_bytes", ctypes.c_int64), ("ops", ctypes.c_int64),
                ("kernels", ctypes.c_int64), ("steps", ctypes.c_int64), ("ops_fused", ctypes.c_int64),
                ("perms_dropped", ctypes.c_int64), ("pass_arena_bytes", ctypes.c_int64)]


class mx_build_info(ctypes.Structure):
    _fields_ = [("layouts_loaded", ctypes.c_int64), ("layouts_derived", ctypes.c_int64),
                ("cache_saved", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("seconds_cache_read", ctypes.c_double), ("seconds_steps", ctypes.c_double),
                ("seconds_device", ctypes.c_double), ("seconds_cache_write", ctypes.c_double)]


class mx_batch_worker(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("state", ctypes.c_int32), ("error_code", ctypes.c_int32),
                ("images_done", ctypes.c_int32), ("seconds", ctypes.c_double), ("error", ctypes.c_char * 256)]


class mx_batch_config(ctypes.Structure):
    _fields_ = [("plan", ctypes.POINTER(mx_plan)), ("device_mem_budget", ctypes.c_int64)]


EXEC_OPEN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p))
EXEC_RUN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_float),
                            ctypes.POINTER(ctypes.c_float))
EXEC_CLOSE = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_void_p)


class mx_batch_executor(ctypes.Structure):
    _fields_ = [("ctx", ctypes.c_void_p), ("open", EXEC_OPEN), ("run", EXEC_RUN), ("close", EXEC_CLOSE)]


class mx_image(ctypes.Structure):
    _fields_ = [("c", ctypes.c_int32), ("h", ctypes.c_int32), ("w", ctypes.c_int32),
                ("data", ctypes.POINTER(ctypes.c_float))]


class mx_image8(ctypes.Structure):
    _fields_ = [("c", ctypes.c_int32), ("h", ctypes.c_int32), ("w", ctypes.c_int32),
                ("data", ctypes.POINTER(ctypes.c_uint8))]


class MaximError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


_lib = None

_SIGS = {
    "mx_last_error": (ctypes.c_size_t, [ctypes.c_char_p, ctypes.c_size_t]),
    "mx_driver_ready": (ctypes.c_int, []),
    "mx_device_count": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "mx_gpu_new": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(mx_plan), ctypes.POINTER(ctypes.c_void_p)]),
    "mx_gpu_free": (None, [ctypes.c_void_p]),
    "mx_gpu_new_cached": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(mx_plan), ctypes.c_int64, ctypes.c_char_p,
                                         ctypes.POINTER(ctypes.c_void_p)]),
    "mx_gpu_save_weight_cache": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p]),
    "mx_gpu_build_info": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(mx_build_info)]),
    "mx_gpu_run": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "mx_gpu_upload_input": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "mx_gpu_enqueue": (ctypes.c_int, [ctypes.c_void_p]),
    "mx_gpu_download_output": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "mx_gpu_sync": (ctypes.c_int, [ctypes.c_void_p]),
    "mx_gpu_poll": (ctypes.c_int, [ctypes.c_void_p]),
    "mx_gpu_stream": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "mx_gpu_upload_rgb8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32]),
    "mx_gpu_download_rgb8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "mx_gpu_run_rgb8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_int32, ctypes.c_void_p]),
    "mx_gpu_upload_input_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "mx_gpu_download_output_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "mx_gpu_begin": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "mx_gpu_step_op": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32]),
    "mx_gpu_read_buf": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64]),
    "mx_gpu_read_into": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64]),
    "mx_gpu_read_arena": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]),
    "mx_gpu_set_timeline": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "mx_gpu_timeline": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                       ctypes.POINTER(ctypes.c_float)]),
    "mx_gpu_timeline_kernels": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32]),
    "mx_gpu_get_stats": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(mx_gpu_stats)]),
    "mx_gpu_schedule": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32]),
    "mx_plan_schedule": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(mx_gpu_stats), ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_int32]),
    "mx_channel_mean_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int64,
                                               ctypes.c_void_p, ctypes.c_void_p]),
    "mx_gpu_new_budget": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(mx_plan), ctypes.c_int64,
                                         ctypes.POINTER(ctypes.c_void_p)]),
    "mx_batch_new": (ctypes.c_int, [ctypes.POINTER(mx_batch_config), ctypes.POINTER(ctypes.c_int32), ctypes.c_int32,
                                    ctypes.POINTER(mx_batch_executor), ctypes.POINTER(ctypes.c_void_p)]),
    "mx_batch_run": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p),
                                    ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_int32)]),
    "mx_batch_run_png": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_char_p),
                                        ctypes.POINTER(ctypes.c_char_p), ctypes.c_int32,
                                        ctypes.POINTER(ctypes.c_int32)]),
    "mx_batch_worker_count": (ctypes.c_int32, [ctypes.c_void_p]),
    "mx_batch_workers": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(mx_batch_worker), ctypes.c_int32]),
    "mx_batch_free": (None, [ctypes.c_void_p]),
    "mx_weights_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "mx_weights_free": (None, [ctypes.c_void_p]),
    "mx_weights_variant": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]),
    "mx_param_spec": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t,
                                     ctypes.POINTER(ctypes.c_size_t)]),
    "mx_plan_build": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int,
                                     ctypes.POINTER(ctypes.c_void_p)]),
    "mx_plan_build_variant": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int,
                                             ctypes.POINTER(ctypes.c_void_p)]),
    "mx_plan_free": (None, [ctypes.c_void_p]),
    "mx_plan_view": (ctypes.POINTER(mx_plan), [ctypes.c_void_p]),
    "mx_plan_dump_count": (ctypes.c_int32, [ctypes.c_void_p]),
    "mx_plan_dump": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_char_p, ctypes.c_size_t,
                                    ctypes.POINTER(ctypes.c_int32)]),
    "mx_plan_label": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_char_p, ctypes.c_size_t]),
    "mx_image_free": (None, [ctypes.POINTER(mx_image)]),
    "mx_png_read": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(mx_image)]),
    "mx_png_read_mem": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(mx_image)]),
    "mx_png_write": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(mx_image)]),
    "mx_preprocess": (ctypes.c_int, [ctypes.POINTER(mx_image), ctypes.c_int32, ctypes.POINTER(mx_image),
                                     ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]),
    "mx_crop_out": (ctypes.c_int, [ctypes.POINTER(mx_image), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                   ctypes.c_int32, ctypes.POINTER(mx_image)]),
    "mx_pad_geometry": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32] +
                        [ctypes.POINTER(ctypes.c_int32)] * 4),
    "mx_image8_free": (None, [ctypes.POINTER(mx_image8)]),
    "mx_png_size_mem": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int32),
                                       ctypes.POINTER(ctypes.c_int32)]),
    "mx_png_read_rgb8_mem": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(mx_image8)]),
    "mx_png_write_rgb8": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(mx_image8)]),
}


def lib():
    """The loaded library. Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("%s is missing: run `python maxim-rs_b200/build.py` (or __graft_entry__.build())"
                               % LIB_PATH)
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    """The ABI's entry point names (what include/maxim_b200.h declares)."""
    return sorted(_SIGS)


def last_error():
    buf = ctypes.create_string_buffer(4096)
    lib().mx_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc, what=""):
    if rc != MX_OK:
        raise MaximError(rc, (what + ": " if what else "") + last_error())


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class Weights:
    """`Weights::open` (src/weights.rs:37-41): a converted checkpoint, variant derived from the file."""

    def __init__(self, path):
        self._h = ctypes.c_void_p()
        check(lib().mx_weights_open(os.fsencode(path), ctypes.byref(self._h)), path)
        buf = ctypes.create_string_buffer(16)
        check(lib().mx_weights_variant(self._h, buf, 16))
        self.variant = buf.value.decode()

    def __del__(self):
        if getattr(self, "_h", None):
            lib().mx_weights_free(self._h)
            self._h = None


def param_spec(variant):
    """[(name, shape)] a checkpoint of `variant` holds, in the builder's request order."""
    need = ctypes.c_size_t()
    check(lib().mx_param_spec(variant.encode(), None, 0, ctypes.byref(need)))
    buf = ctypes.create_string_buffer(need.value)
    check(lib().mx_param_spec(variant.encode(), buf, need.value, None))
    out = []
    for line in buf.value.decode().splitlines():
        name, shape = line.split("\t")
        out.append((name, tuple(int(x) for x in shape.split(","))))
    return out


class Plan:
    """`model::Plan` (src/model.rs:1237-1272) for one padded input shape."""

    def __init__(self, weights=None, h=0, w=0, dumps=False, variant=None):
        self._h = ctypes.c_void_p()
        self._weights = weights
        if weights is not None:
            check(lib().mx_plan_build(weights._h, h, w, int(dumps), ctypes.byref(self._h)), "plan")
        else:
            check(lib().mx_plan_build_variant(variant.encode(), h, w, int(dumps), ctypes.byref(self._h)), "plan")
        self.view = lib().mx_plan_view(self._h)
        v = self.view.contents
        self.n_ops, self.n_bufs, self.n_weights = v.n_ops, v.n_bufs, v.n_weights
        self.arena_len, self.input, self.output = v.arena_len, v.input, v.output
        self.shape = (v.shape.c, v.shape.h, v.shape.w)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().mx_plan_free(self._h)
            self._h = None

    @property
    def arena_bytes(self):
        return self.arena_len * 4

    def buf(self, i):
        b = self.view.contents.bufs[i]
        return (b.c, b.h, b.w)

    def off(self, i):
        return self.view.contents.offs[i]

    def alias(self, i):
        v = self.view.contents
        p = v.alias_parent[i]
        return None if p < 0 else (p, v.alias_delta[i])

    def op(self, i):
        return self.view.contents.ops[i]

    def ops(self):
        v = self.view.contents
        return [v.ops[i] for i in range(v.n_ops)]

    def label(self, i):
        buf = ctypes.create_string_buffer(128)
        check(lib().mx_plan_label(self._h, i, buf, 128))
        return buf.value.decode()

    def dumps(self):
        out = []
        for i in range(lib().mx_plan_dump_count(self._h)):
            buf = ctypes.create_string_buffer(256)
            bid = ctypes.c_int32()
            check(lib().mx_plan_dump(self._h, i, buf, 256, ctypes.byref(bid)))
            out.append((buf.value.decode(), bid.value))
        return out

    def weight_bytes(self):
        v = self.view.contents
        return sum(v.weight_lens[i] for i in range(v.n_weights)) * 4

    def weight(self, i):
        v = self.view.contents
        n = v.weight_lens[i]
        return np.ctypeslib.as_array(v.weights[i], shape=(n,)).copy() if n else np.zeros(0, np.float32)


def driver_ready():
    """`exec_gpu::driver_ready` (src/exec_gpu.rs:81-83)."""
    check(lib().mx_driver_ready(), "cuda")


def device_count():
    n = ctypes.c_int()
    rc = lib().mx_device_count(ctypes.byref(n))
    return n.value if rc == MX_OK else 0


class Gpu:
    """`exec_gpu::Gpu` (src/exec_gpu.rs:48-357) on one device, over the C ABI."""

    def __init__(self, plan, device=0, weight_cache=None, mem_budget=0):
        """weight_cache: path of a converted-weights cache file
        (`mx_gpu_new_cached`): layouts found there are loaded, the rest
        derived and the file written."""
        self.plan = plan
        self._h = ctypes.c_void_p()
        if weight_cache is None and not mem_budget:
            check(lib().mx_gpu_new(device, plan.view, ctypes.byref(self._h)), "gpu")
        else:
            check(lib().mx_gpu_new_cached(device, plan.view, mem_budget,
                                          None if weight_cache is None else os.fsencode(weight_cache),
                                          ctypes.byref(self._h)), "gpu")
        c, h, w = plan.buf(plan.input)
        self.in_len = c * h * w
        c, h, w = plan.buf(plan.output)
        self.out_shape = (c, h, w)

    def close(self):
        if getattr(self, "_h", None):
            lib().mx_gpu_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def run(self, image, out=None):
        x = np.ascontiguousarray(image, dtype=np.float32).reshape(-1)
        if x.size != self.in_len:
            raise ValueError("input has %d values, the plan's input buffer %d" % (x.size, self.in_len))
        if out is None:
            out = np.empty(self.out_shape, np.float32)
        check(lib().mx_gpu_run(self._h, _ptr(x), _ptr(out)), "run")
        return out

    def build_info(self):
        """`mx_gpu_build_info` as a dict: layouts loaded / derived, whether the
        cache was saved, and the construction phases' seconds."""
        b = mx_build_info()
        check(lib().mx_gpu_build_info(self._h, ctypes.byref(b)))
        return {f: getattr(b, f) for f, _ in b._fields_ if f != "reserved"}

    def weight_cache_info(self):
        """(loaded, derived, saved): how the executor's weight layouts were obtained."""
        b = self.build_info()
        return b["layouts_loaded"], b["layouts_derived"], b["cache_saved"]

    def save_weight_cache(self, path):
        check(lib().mx_gpu_save_weight_cache(self._h, os.fsencode(path)), str(path))

    def run_rgb8(self, rgb, factor=64, out=None):
        """The image path with its per-pixel steps on the device: h x w x 3 uint8
        in, the restored h x w x 3 uint8 out (`mx_gpu_run_rgb8`)."""
        x = np.ascontiguousarray(rgb, dtype=np.uint8)
        if x.ndim != 3 or x.shape[2] != 3:
            raise ValueError("expected h x w x 3 uint8 samples, got shape %s" % (x.shape,))
        if out is None:
            out = np.empty(x.shape, np.uint8)
        check(lib().mx_gpu_run_rgb8(self._h, _ptr(x), x.shape[0], x.shape[1], factor, _ptr(out)), "run_rgb8")
        return out

    def upload_rgb8(self, rgb, factor=64):
        x = np.ascontiguousarray(rgb, dtype=np.uint8)
        check(lib().mx_gpu_upload_rgb8(self._h, _ptr(x), x.shape[0], x.shape[1], factor), "upload_rgb8")
        self._rgb_keep = x  # the copy from pageable memory may still be reading it

    def download_rgb8(self, out):
        check(lib().mx_gpu_download_rgb8(self._h, _ptr(out)), "download_rgb8")

    def upload_input(self, image):
        x = np.ascontiguousarray(image, dtype=np.float32).reshape(-1)
        check(lib().mx_gpu_upload_input(self._h, _ptr(x)), "upload")

    def enqueue(self):
        check(lib().mx_gpu_enqueue(self._h), "enqueue")

    def download_output(self, out):
        check(lib().mx_gpu_download_output(self._h, _ptr(out)), "download")

    def stream(self):
        """The handle's cudaStream_t as an integer (for torch.cuda.ExternalStream)."""
        s = ctypes.c_void_p()
        check(lib().mx_gpu_stream(self._h, ctypes.byref(s)), "stream")
        return s.value or 0

    def upload_input_device(self, dev_ptr):
        """Copy the input from device memory (an integer address on this device)."""
        check(lib().mx_gpu_upload_input_device(self._h, ctypes.c_void_p(dev_ptr)), "upload (device)")

    def download_output_device(self, dev_ptr):
        check(lib().mx_gpu_download_output_device(self._h, ctypes.c_void_p(dev_ptr)), "download (device)")

    def sync(self):
        check(lib().mx_gpu_sync(self._h), "sync")

    def begin(self, image):
        x = np.ascontiguousarray(image, dtype=np.float32).reshape(-1)
        check(lib().mx_gpu_begin(self._h, _ptr(x)), "begin")

    def step_op(self, i):
        check(lib().mx_gpu_step_op(self._h, i), "step_op %d" % i)

    def read_buf(self, i):
        c, h, w = self.plan.buf(i)
        out = np.empty((c, h, w), np.float32)
        check(lib().mx_gpu_read_buf(self._h, i, _ptr(out), out.size), "read_buf")
        return out

    def read_into(self, off, n):
        """`Gpu::read_into`: n floats of the plan-layout arena from element off."""
        out = np.empty(n, np.float32)
        check(lib().mx_gpu_read_into(self._h, off, _ptr(out), n), "read_into")
        return out

    def read_arena(self):
        """`Gpu::read_arena`: the whole arena in the plan's layout."""
        out = np.empty(self.plan.arena_len, np.float32)
        check(lib().mx_gpu_read_arena(self._h, _ptr(out), out.size), "read_arena")
        return out

    def set_timeline(self, on):
        check(lib().mx_gpu_set_timeline(self._h, int(on)))

    def timeline(self):
        per = np.zeros(self.plan.n_ops, np.float32)
        tot = ctypes.c_float()
        check(lib().mx_gpu_timeline(self._h, _ptr(per), self.plan.n_ops, ctypes.byref(tot)), "timeline")
        return per, tot.value

    def timeline_kernels(self):
        """`Timeline::kernels_per_op` of the last timed pass."""
        k = np.zeros(self.plan.n_ops, np.int32)
        check(lib().mx_gpu_timeline_kernels(self._h, _ptr(k), self.plan.n_ops), "timeline kernels")
        return k

    def stats(self):
        s = mx_gpu_stats()
        check(lib().mx_gpu_get_stats(self._h, ctypes.byref(s)))
        return _stats_dict(s)

    def schedule(self, flags=False):
        """Per plan op, the op whose scheduled step carries it out (-1: removed);
        with flags=True also the per-op SCHED_* flags."""
        out = np.zeros(self.plan.n_ops, np.int32)
        fl = np.zeros(self.plan.n_ops, np.int32)
        check(lib().mx_gpu_schedule(self._h, _ptr(out), _ptr(fl), self.plan.n_ops), "schedule")
        return (out, fl) if flags else out


class Batch:
    """`mx_batch_*`: independent images round-robin over devices, one worker
    thread and executor handle per device, with the runner's failure
    handling (a device that cannot be built is left out; a worker that fails
    is retired and its unfinished images go to the others).

    By default the executor is this library's GPU executor for `plan`. A
    Python `executor` may replace it: an object with `in_len` / `out_len`
    (floats per image) and `open(device) -> handle`, `run(handle, x, y)`
    (x, y float32 arrays; raise to fail) and `close(handle)`."""

    def __init__(self, plan=None, devices=(0,), mem_budget=0, executor=None):
        self._h = ctypes.c_void_p()
        self.plan = plan
        self._py = executor
        cfg = mx_batch_config(plan.view if plan is not None else None, int(mem_budget))
        devs = (ctypes.c_int32 * len(devices))(*devices)
        ex = None
        if executor is not None:
            import itertools
            import threading
            self._handles, self._keys, self._mu = {}, itertools.count(1), threading.Lock()
            ex = mx_batch_executor(None, EXEC_OPEN(self._open), EXEC_RUN(self._run), EXEC_CLOSE(self._close))
            self._ex = ex  # the callbacks must outlive the batch
            self.in_len, self.out_len = executor.in_len, executor.out_len
        else:
            c, h, w = plan.buf(plan.input)
            self.in_len = c * h * w
            self.out_shape = plan.buf(plan.output)
            self.out_len = int(np.prod(self.out_shape))
        check(lib().mx_batch_new(ctypes.byref(cfg), devs, len(devices), ctypes.byref(ex) if ex else None,
                                 ctypes.byref(self._h)), "batch")

    # Python-executor trampolines (run on the runner's worker threads).
    def _open(self, ctx, device, handle):
        try:
            h = self._py.open(int(device))
        except Exception:
            return -1
        with self._mu:
            key = next(self._keys)
            self._handles[key] = h
        handle[0] = key
        return 0

    def _run(self, ctx, handle, x, y):
        try:
            xa = np.ctypeslib.as_array(x, shape=(self.in_len,))
            ya = np.ctypeslib.as_array(y, shape=(self.out_len,))
            self._py.run(self._handles[handle], xa, ya)
        except Exception:
            return -1
        return 0

    def _close(self, ctx, handle):
        try:
            self._py.close(self._handles.pop(handle))
        except Exception:
            pass

    def close(self):
        if getattr(self, "_h", None):
            lib().mx_batch_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def run(self, images, outs=None, raise_on_error=True):
        """Restore every image; returns (outputs, per-image status codes)."""
        xs = [np.ascontiguousarray(im, dtype=np.float32).reshape(-1) for im in images]
        for x in xs:
            if x.size != self.in_len:
                raise ValueError("an image has %d values, the batch's input %d" % (x.size, self.in_len))
        if outs is None:
            shape = getattr(self, "out_shape", (self.out_len,))
            outs = [np.empty(shape, np.float32) for _ in xs]
        n = len(xs)
        ip = (ctypes.c_void_p * n)(*[x.ctypes.data for x in xs])
        op = (ctypes.c_void_p * n)(*[o.ctypes.data for o in outs])
        st = (ctypes.c_int32 * n)()
        rc = lib().mx_batch_run(self._h, n, ip, op, st)
        status = [int(v) for v in st]
        if rc != MX_OK and raise_on_error:
            raise MaximError(rc, "batch: " + last_error())
        return outs, status

    def run_png(self, in_paths, out_paths, factor=64, raise_on_error=True):
        """`mx_batch_run_png`: PNG files in, PNG files out over the device-side
        image path; returns the per-image status codes."""
        n = len(in_paths)
        if len(out_paths) != n:
            raise ValueError("in_paths and out_paths differ in length")
        ip = (ctypes.c_char_p * n)(*[os.fsencode(p) for p in in_paths])
        op = (ctypes.c_char_p * n)(*[os.fsencode(p) for p in out_paths])
        st = (ctypes.c_int32 * n)()
        rc = lib().mx_batch_run_png(self._h, n, ip, op, factor, st)
        status = [int(v) for v in st]
        if rc != MX_OK and raise_on_error:
            raise MaximError(rc, "batch: " + last_error())
        return status

    def workers(self):
        n = lib().mx_batch_worker_count(self._h)
        arr = (mx_batch_worker * n)()
        check(lib().mx_batch_workers(self._h, arr, n), "batch workers")
        return [{"device": w.device, "state": "ready" if w.state == 0 else "failed", "error_code": w.error_code,
                 "images_done": w.images_done, "seconds": w.seconds, "error": w.error.decode(errors="replace")}
                for w in arr]


def _stats_dict(s):
    return {"device_name": s.device_name.decode(), "arena_bytes": s.arena_bytes, "weight_bytes": s.weight_bytes,
            "pool_bytes": s.pool_bytes, "ops": s.ops, "kernels": s.kernels, "steps": s.steps,
            "ops_fused": s.ops_fused, "perms_dropped": s.perms_dropped, "pass_arena_bytes": s.pass_arena_bytes}


SCHED_STATS_ONLY, SCHED_LN_ON_LOAD, SCHED_LN_IN_EPILOGUE, SCHED_LN_INPUT_UNSTORED = 1, 2, 4, 8


def plan_schedule(plan, flags=False):
    """`mx_plan_schedule`: the executor's schedule of a plan, worked out on the
    host: (stats dict, per-op primary op array[, per-op SCHED_* flags])."""
    s = mx_gpu_stats()
    out = np.zeros(plan.n_ops, np.int32)
    fl = np.zeros(plan.n_ops, np.int32)
    check(lib().mx_plan_schedule(ctypes.cast(plan.view, ctypes.c_void_p), ctypes.byref(s), _ptr(out), _ptr(fl),
                                 plan.n_ops), "plan schedule")
    return (_stats_dict(s), out, fl) if flags else (_stats_dict(s), out)


def channel_mean_noalloc(x_ptr, npix, c, pixel_stride, out_ptr, stream=0):
    """`mx_channel_mean_noalloc`: the channel mean of an NHWC tensor already in
    device memory (integer device addresses), using no allocation."""
    check(lib().mx_channel_mean_noalloc(ctypes.c_void_p(x_ptr), npix, c, pixel_stride, ctypes.c_void_p(out_ptr),
                                        ctypes.c_void_p(stream)), "channel mean (no allocation)")


def _image_to_np(img):
    a = np.ctypeslib.as_array(img.data, shape=(img.c, img.h, img.w)).copy()
    lib().mx_image_free(ctypes.byref(img))
    return a


def _np_to_image(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    img = mx_image(a.shape[0], a.shape[1], a.shape[2], a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return img, a


def png_read(path):
    img = mx_image()
    check(lib().mx_png_read(os.fsencode(path), ctypes.byref(img)), str(path))
    return _image_to_np(img)


def png_read_bytes(data):
    img = mx_image()
    check(lib().mx_png_read_mem(data, len(data), ctypes.byref(img)), "png")
    return _image_to_np(img)


def png_write(path, a):
    img, keep = _np_to_image(a)
    check(lib().mx_png_write(os.fsencode(path), ctypes.byref(img)), str(path))


def preprocess(a, factor=64):
    """`image::preprocess` (src/image.rs:171-207) -> (padded, (even_h, even_w))."""
    img, keep = _np_to_image(a)
    out = mx_image()
    eh, ew = ctypes.c_int32(), ctypes.c_int32()
    check(lib().mx_preprocess(ctypes.byref(img), factor, ctypes.byref(out), ctypes.byref(eh), ctypes.byref(ew)),
          "preprocess")
    return _image_to_np(out), (eh.value, ew.value)


def crop_out(a, orig_h, orig_w, even_h, even_w):
    img, keep = _np_to_image(a)
    out = mx_image()
    check(lib().mx_crop_out(ctypes.byref(img), orig_h, orig_w, even_h, even_w, ctypes.byref(out)), "crop")
    return _image_to_np(out)


def pad_geometry(h, w, factor=64):
    """`mx_pad_geometry` -> ((padded_h, padded_w), (even_h, even_w))."""
    v = [ctypes.c_int32() for _ in range(4)]
    check(lib().mx_pad_geometry(h, w, factor, *[ctypes.byref(x) for x in v]), "pad_geometry")
    return (v[0].value, v[1].value), (v[2].value, v[3].value)


def png_size(data):
    """Height and width from a PNG's IHDR chunk."""
    h, w = ctypes.c_int32(), ctypes.c_int32()
    check(lib().mx_png_size_mem(data, len(data), ctypes.byref(h), ctypes.byref(w)), "png")
    return h.value, w.value


def png_read_rgb8_bytes(data):
    """A PNG's 8-bit samples as h x w x 3 uint8 (gray expanded to RGB)."""
    img = mx_image8()
    check(lib().mx_png_read_rgb8_mem(data, len(data), ctypes.byref(img)), "png")
    a = np.ctypeslib.as_array(img.data, shape=(img.h, img.w, img.c)).copy()
    lib().mx_image8_free(ctypes.byref(img))
    return a


def png_write_rgb8(path, a):
    a = np.ascontiguousarray(a, dtype=np.uint8)
    img = mx_image8(3, a.shape[0], a.shape[1], a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
    check(lib().mx_png_write_rgb8(os.fsencode(path), ctypes.byref(img)), str(path))
