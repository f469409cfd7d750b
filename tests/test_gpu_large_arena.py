"""BASELINE config 4 on the GPU: MAXIM-3S on one 2048x2048 dark image, a
7.4 GB arena, the largest the benchmark runs (its latency is part of the
metric). Byte offsets into the arena pass 2^31 here and at no smaller size,
so this is where an offset computed in 32 bits would show.

The CPU oracle would take minutes at this size, so the check is the
executor against itself. The fused pass re-packs the arena, so every buffer
sits at a different offset than in the op-by-op pass (MAXIM_NO_FUSE), which
keeps the plan's own packing. The two must agree bit for bit, as at the
smaller sizes where both are checked against the oracle.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_config4_2048_fused_and_op_by_op_agree(mx, synth, checkpoint):
    wts = mx.Weights(checkpoint("S-3", 3, 1.0, False))
    img = synth.image_dark(synth.input_rng(3), 2048, 2048)
    padded, _ = mx.preprocess(img, 64)
    plan = mx.Plan(wts, padded.shape[1], padded.shape[2])
    fused = mx.Gpu(plan)
    st = fused.stats()
    assert st["arena_bytes"] > 2**31 and st["pass_arena_bytes"] > 2**31, st
    out = fused.run(padded)
    again = fused.run(padded)
    fused.close()
    assert np.isfinite(out).all()
    assert np.array_equal(out, again), "two fused passes differ"
    os.environ["MAXIM_NO_FUSE"] = "1"
    try:
        ref = mx.Gpu(plan)
    finally:
        del os.environ["MAXIM_NO_FUSE"]
    base = ref.run(padded)
    ref.close()
    diff = np.abs(out.astype(np.float64) - base)
    assert np.array_equal(out, base), "fused and op-by-op passes differ: max %.3e at %s" % (
        diff.max(), np.unravel_index(diff.argmax(), diff.shape))
