"""Seeded synthetic checkpoints and inputs.

No MAXIM checkpoint or dataset is available offline, so every run of this
build uses random-init weights of the real architecture and seeded synthetic
images with the shapes and value distributions of the benchmark configurations.

Checkpoints are written in the reference converter's safetensors layout
(tools/convert.py:88-126): an 8-byte header length, a JSON header with sorted
keys and a `__metadata__` block, the tensor bytes in sorted-name order. The
parameter inventory comes from the library's own builder (`param_spec`), so a
synthetic checkpoint holds exactly the tensors the plan asks for.

Weight init (names visited in sorted order, one numpy PCG64 stream per seed):
  */kernel  standard_normal(shape) * sqrt(2 / fan_in) * gain, fan_in = prod(shape[:-1])
  */bias    0          */scale  1        (LayerNorm gamma / beta = 1 / 0)
`gain` 1.0 is He-normal; the network diverges to |y| ~ 1e7 under it, so 0.5 is
the companion init whose outputs stay O(1). `rich=True` also draws nonzero
biases and LayerNorm affine terms, which the plain init leaves at 0 and 1 and
which therefore need their own parity coverage.
"""
import json
import math
import os

import numpy as np

from . import _native


def make_params(variant, seed, gain=1.0, rich=False, dense_std=None, spec=None):
    """{name: float32 array} for every tensor `variant` needs. `spec` is the
    parameter inventory [(name, shape)]; by default the library's builder's."""
    spec = dict(spec if spec is not None else _native.param_spec(variant))
    rng = np.random.default_rng(seed)
    out = {}
    for name in sorted(spec):
        shape = spec[name]
        if name.endswith("/scale"):
            a = np.ones(shape, np.float32)
            if rich:
                a = (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
        elif name.endswith("/bias"):
            a = np.zeros(shape, np.float32)
            if rich:
                a = (0.1 * rng.standard_normal(shape)).astype(np.float32)
        else:
            if dense_std is not None:
                a = (dense_std * rng.standard_normal(shape)).astype(np.float32)
            else:
                fan_in = int(np.prod(shape[:-1]))
                a = (gain * rng.standard_normal(shape) * math.sqrt(2.0 / fan_in)).astype(np.float32)
        out[name] = a
    return out


def write_safetensors(path, params, variant, task="synthetic"):
    names = sorted(params)
    header = {"__metadata__": {"format": "maxim", "task": task, "variant": variant,
                               "tensor_count": str(len(names)),
                               "source": "seeded random init (maxim-rs_b200.synth)"}}
    off = 0
    for k in names:
        a = np.ascontiguousarray(params[k], dtype=np.float32)
        header[k] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
    blob = json.dumps(header, separators=(",", ":"), sort_keys=True).encode()
    blob += b" " * ((-(8 + len(blob))) % 8)
    # A temporary of this process's own, renamed into place: processes that
    # write the same checkpoint at once (ranks on one box) each rename a
    # complete file, and the last rename wins with identical bytes.
    tmp = "%s.tmp%d" % (path, os.getpid())
    with open(tmp, "wb") as f:
        f.write(len(blob).to_bytes(8, "little"))
        f.write(blob)
        for k in names:
            f.write(np.ascontiguousarray(params[k], dtype=np.float32).tobytes())
    os.replace(tmp, path)
    return path


def checkpoint(path, variant, seed, gain=1.0, rich=False, spec=None):
    """Write (or reuse) a synthetic checkpoint and return its path."""
    if not os.path.exists(path):
        write_safetensors(path, make_params(variant, seed, gain, rich, spec=spec), variant)
    return path


def _bilinear_up(a, oh, ow):
    """Half-pixel bilinear upsampling of a [h][w] grid (align_corners=False)."""
    ih, iw = a.shape

    def axis(n_in, n_out):
        src = (np.arange(n_out) + 0.5) * (n_in / n_out) - 0.5
        src = np.clip(src, 0, None)
        i0 = np.minimum(np.floor(src).astype(np.int64), n_in - 1)
        i1 = np.minimum(i0 + 1, n_in - 1)
        return i0, i1, (src - i0).astype(np.float64)

    y0, y1, fy = axis(ih, oh)
    x0, x1, fx = axis(iw, ow)
    top = a[y0][:, x0] * (1 - fx) + a[y0][:, x1] * fx
    bot = a[y1][:, x0] * (1 - fx) + a[y1][:, x1] * fx
    return top * (1 - fy)[:, None] + bot * fy[:, None]


def image_uniform(rng, h, w):
    """[3][h][w] pixels i.i.d. U[0,1)."""
    return rng.random((3, h, w), dtype=np.float32)


def image_smooth_noisy(rng, h, w):
    """A bilinear-upsampled 8x8 U[0,1) grid per channel plus N(0, (25/255)^2), clipped (config 2)."""
    out = np.empty((3, h, w), np.float32)
    for c in range(3):
        g = rng.random((8, 8))
        out[c] = _bilinear_up(g, h, w)
    out += rng.standard_normal((3, h, w)) * (25.0 / 255.0)
    return np.clip(out, 0.0, 1.0).astype(np.float32)


def image_dark(rng, h, w):
    """U[0,0.25) plus Poisson-like noise with std 0.02*sqrt(v), clipped (config 4)."""
    v = rng.random((3, h, w)) * 0.25
    v = v + rng.standard_normal((3, h, w)) * 0.02 * np.sqrt(v)
    return np.clip(v, 0.0, 1.0).astype(np.float32)


def input_rng(seed):
    """The input stream of a configuration: distinct from its weight stream."""
    return np.random.default_rng([seed, 1])
