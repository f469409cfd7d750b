"""The image steps either side of the pass, on the device (mx_gpu_run_rgb8):
8-bit RGB in, divide by 255, even reflect, centred reflect pad to a multiple
of 64, the pass, centred crop, clamp and round half up to 8 bits out
(src/image.rs:40-104, 171-246; the CLI's path, src/main.rs:467-504).

The checker is the host pipeline (mx_preprocess, pinned to the reference's
own PyTorch preprocessing by tests/test_image.py) and numpy's reflect pad and
float32 arithmetic; the bar is bit equality."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def reflect_pad_np(x, factor):
    """The published pipeline in numpy: reflect (no edge repeat) to an even
    shape at the bottom / right, then centred to the next multiple of
    `factor` (strictly above when not already a multiple)."""
    _, h, w = x.shape
    x = np.pad(x, ((0, 0), (0, h % 2), (0, w % 2)), mode="reflect")
    _, eh, ew = x.shape
    hp = ((eh + factor) // factor) * factor if eh % factor else eh
    wp = ((ew + factor) // factor) * factor if ew % factor else ew
    t, l = (hp - eh) // 2, (wp - ew) // 2
    return np.pad(x, ((0, 0), (t, t), (l, l)), mode="reflect"), (eh, ew)


def quantize_np(a):
    return np.floor(np.clip(a, 0, 1) * np.float32(255) + np.float32(0.5)).astype(np.uint8)


@pytest.mark.parametrize("h,w", [(97, 131), (45, 70), (64, 64), (200, 23 * 2 + 1)])
def test_device_image_path_is_the_host_pipeline(mx, checkpoint, h, w):
    ckpt = checkpoint("S-1", 5, 0.5)
    rgb = np.random.default_rng(h * 1000 + w).integers(0, 256, (h, w, 3), dtype=np.uint8)
    x = rgb.transpose(2, 0, 1).astype(np.float32) / np.float32(255.0)
    padded, (eh, ew) = mx.preprocess(x, 64)
    want_pad, even = reflect_pad_np(x, 64)
    assert even == (eh, ew) and np.array_equal(padded, want_pad)
    gpu = mx.Gpu(mx.Plan(mx.Weights(ckpt), padded.shape[1], padded.shape[2]))
    try:
        out8 = gpu.run_rgb8(rgb)
        # the device's padded input, as the plan's input buffer
        assert np.array_equal(gpu.read_buf(gpu.plan.input), padded)
        ref = gpu.run(padded)
        want = quantize_np(mx.crop_out(ref, h, w, eh, ew)).transpose(1, 2, 0)
        assert out8.shape == (h, w, 3) and np.array_equal(out8, want)
        # again, through the split form, into a reused buffer
        again = np.zeros_like(out8)
        gpu.upload_rgb8(rgb)
        gpu.enqueue()
        gpu.download_rgb8(again)
        gpu.sync()
        assert np.array_equal(again, out8)
    finally:
        gpu.close()


def test_device_image_path_refusals(mx, checkpoint):
    ckpt = checkpoint("S-1", 5, 0.5)
    gpu = mx.Gpu(mx.Plan(mx.Weights(ckpt), 64, 128))
    try:
        with pytest.raises(mx.MaximError, match="too small"):
            gpu.run_rgb8(np.zeros((16, 16, 3), np.uint8))
        with pytest.raises(mx.MaximError, match="pads to"):
            gpu.run_rgb8(np.zeros((100, 100, 3), np.uint8))
        with pytest.raises(mx.MaximError, match="no image was uploaded"):
            gpu.download_rgb8(np.zeros((45, 70, 3), np.uint8))
        # the handle still works after the refusals
        rgb = np.random.default_rng(1).integers(0, 256, (45, 70, 3), dtype=np.uint8)
        assert gpu.run_rgb8(rgb).shape == (45, 70, 3)
    finally:
        gpu.close()
