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


def test_png_batch_over_the_device_image_path(mx, checkpoint, tmp_path):
    """mx_batch_run_png: PNG files in and out, two workers on one device,
    images of two sizes that pad to the same plan; an unreadable file, a
    broken PNG and an image too small to pad fail alone, the rest are written
    and equal the single-image device path's output."""
    plan = mx.Plan(mx.Weights(checkpoint("S-1", 3, 0.5)), 64, 128)
    rng = np.random.default_rng(7)
    sizes = [(45, 70), (50, 80), (45, 70), (64, 128), (50, 80)]
    imgs = [rng.integers(0, 256, (h, w, 3), dtype=np.uint8) for h, w in sizes]
    ins, outs = [], []
    for k, im in enumerate(imgs):
        ins.append(str(tmp_path / ("in%d.png" % k)))
        outs.append(str(tmp_path / ("out%d.png" % k)))
        mx.png_write_rgb8(ins[-1], im)
    bad = [str(tmp_path / "missing.png"), str(tmp_path / "broken.png"), str(tmp_path / "tiny.png")]
    (tmp_path / "broken.png").write_bytes(b"\x89PNG\r\n\x1a\n" + b"\x00" * 40)
    mx.png_write_rgb8(bad[2], np.zeros((16, 16, 3), np.uint8))
    order = [0, 5, 1, 2, 6, 3, 7, 4]  # the failing ones between good ones
    all_in = ins + bad
    all_out = outs + [str(tmp_path / ("bad%d.png" % k)) for k in range(3)]
    g = mx.Gpu(plan)
    want = [g.run_rgb8(im) for im in imgs]
    g.close()
    b = mx.Batch(plan, devices=(0, 0))
    st = b.run_png([all_in[i] for i in order], [all_out[i] for i in order], raise_on_error=False)
    good = [st[j] for j, i in enumerate(order) if i < 5]
    failed = [st[j] for j, i in enumerate(order) if i >= 5]
    assert good == [0] * 5 and all(s != 0 for s in failed)
    for k in range(5):
        assert np.array_equal(mx.png_read_rgb8_bytes(open(outs[k], "rb").read()), want[k])
    assert sum(w["images_done"] for w in b.workers()) == 5
    assert all(w["state"] == "ready" for w in b.workers())
    with pytest.raises(mx.MaximError, match="were not restored"):
        b.run_png([bad[0]], [all_out[5]])
    b.close()
