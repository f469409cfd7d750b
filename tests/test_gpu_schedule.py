"""The executor's schedule on the GPU: the fused pass (GEMM epilogues, copy
forwarding, block permutations replaced by gating through 5-D tensor maps,
re-packed arena) must compute exactly what the same executor computes op by
op, and still meet the parity bars against the CPU oracle.

The unfused reference here is the same library with MAXIM_NO_FUSE set, which
keeps the plan's op list (one step per op, blocked gating buffers, every
Copy) and only re-packs the arena. Every value is produced by the same
arithmetic in the same order either way, so the outputs are compared for
bit equality.
"""
import os

import numpy as np
import pytest

from conftest import lsb_fraction, psnr

pytestmark = pytest.mark.gpu


def _unfused(mx, plan):
    os.environ["MAXIM_NO_FUSE"] = "1"
    try:
        return mx.Gpu(plan)
    finally:
        del os.environ["MAXIM_NO_FUSE"]


@pytest.mark.parametrize("variant,h,w,gain,rich", [
    ("S-2", 64, 128, 1.0, True),    # every op kind, nonzero biases and LayerNorm affine
    ("S-3", 256, 320, 0.5, False),  # multi-tile, grid and block gating at three scales
    ("S-1", 128, 192, 1.0, True),
])
def test_fused_pass_is_bit_identical(variant, h, w, gain, rich, mx, synth, oracle, checkpoint):
    wts = mx.Weights(checkpoint(variant, 7, gain, rich))
    img = synth.image_smooth_noisy(synth.input_rng(7), h, w)
    plan = mx.Plan(wts, h, w)
    fused = mx.Gpu(plan)
    st = fused.stats()
    assert st["ops_fused"] > 0 and st["perms_dropped"] > 0, st
    assert st["steps"] < st["ops"]
    sched = fused.schedule()
    kinds = [op.kind for op in plan.ops()]
    assert all(sched[i] >= 0 or kinds[i] in (15, 0) for i in range(len(kinds))), \
        "only block permutations and copies are removed"
    out = fused.run(img)
    ref = _unfused(mx, plan)
    assert ref.stats()["ops_fused"] == 0
    base = ref.run(img)
    diff = np.abs(out.astype(np.float64) - base)
    assert np.array_equal(out, base), "fused and unfused passes differ: max %.3e at %s" % (
        diff.max(), np.unravel_index(diff.argmax(), diff.shape))
    cpu = oracle.output(plan, img)
    assert psnr(cpu, out) >= 50.0
    assert lsb_fraction(cpu, out) >= 0.999


def test_fused_pass_repeats_and_survives_the_op_walk(mx, synth, checkpoint):
    """The op-by-op walk uses the plan's own offsets in the same arena: a pass
    after a walk, and a walk after a pass, both still give their own answers."""
    wts = mx.Weights(checkpoint("S-2", 3, 1.0, True))
    img = synth.image_uniform(synth.input_rng(3), 64, 64)
    plan = mx.Plan(wts, 64, 64)
    gpu = mx.Gpu(plan)
    first = gpu.run(img)
    gpu.begin(img)
    for i in range(plan.n_ops):
        gpu.step_op(i)
    walked = gpu.read_buf(plan.output)
    second = gpu.run(img)
    assert np.array_equal(first, second)
    assert psnr(walked, first) >= 50.0
