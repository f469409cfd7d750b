"""The batch runner (mx_batch_*) on the GPU executor: results equal to the
single-image executor's bit for bit, two workers sharing one device, and the
memory-budget refusal (a device whose pass would exceed its budget is left
out; with no device left the batch is refused with the numbers)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def small(mx, synth, checkpoint, n=5):
    plan = mx.Plan(mx.Weights(checkpoint("S-1", 3, 0.5)), 64, 128)
    imgs = [synth.image_uniform(synth.input_rng(20 + i), 64, 128) for i in range(n)]
    return plan, imgs


def test_batch_matches_the_executor(mx, synth, checkpoint):
    plan, imgs = small(mx, synth, checkpoint)
    g = mx.Gpu(plan)
    want = [g.run(x) for x in imgs]
    g.close()
    n = max(1, mx.device_count())
    b = mx.Batch(plan, devices=tuple(range(n)))
    outs, st = b.run(imgs)
    assert st == [0] * len(imgs)
    for o, w in zip(outs, want):
        assert np.array_equal(o, w)
    ws = b.workers()
    assert sum(w["images_done"] for w in ws) == len(imgs)
    assert all(w["state"] == "ready" for w in ws)
    b.close()


def test_two_workers_on_one_device(mx, synth, checkpoint):
    plan, imgs = small(mx, synth, checkpoint, 4)
    g = mx.Gpu(plan)
    want = [g.run(x) for x in imgs]
    g.close()
    b = mx.Batch(plan, devices=(0, 0))
    outs, st = b.run(imgs)
    assert st == [0] * 4
    assert all(np.array_equal(o, w) for o, w in zip(outs, want))
    assert [w["images_done"] for w in b.workers()] == [2, 2]


def test_memory_budget_refusal(mx, synth, checkpoint):
    plan, imgs = small(mx, synth, checkpoint, 1)
    with pytest.raises(mx.MaximError, match="(?s)not enough device memory.*budget"):
        mx.Batch(plan, devices=(0,), mem_budget=1 << 20)
    # The executor itself, with the same budget.
    import ctypes
    h = ctypes.c_void_p()
    rc = mx.lib().mx_gpu_new_budget(0, plan.view, 1 << 20, ctypes.byref(h))
    assert rc == -4 and "budget" in mx._native.last_error()
