"""The image pipeline (a C++ restatement of src/image.rs): the reference's
padding tests (tests/padding.rs:41-81), its preprocess against the reference's
own PyTorch pipeline (golden fixture), the crop, and PNG I/O against PIL."""
import io

import numpy as np
import pytest

from conftest import golden


def rgb(h, w):
    return (np.arange(3 * h * w) % 251).astype(np.float32).reshape(3, h, w) / np.float32(251.0)


def test_a_sixteen_pixel_image_is_refused_with_the_numbers(mx):
    with pytest.raises(mx.MaximError) as e:
        mx.preprocess(rgb(16, 16), 64)
    m = str(e.value)
    assert "too small" in m
    assert "height is 16 pixels" in m
    assert "24 pixels of padding a side" in m
    assert "at least 22 pixels" in m


def test_one_axis_over_the_line_is_refused_by_name(mx):
    with pytest.raises(mx.MaximError) as e:
        mx.preprocess(rgb(64, 16), 64)
    assert "width is 16 pixels" in str(e.value)
    assert "the height is 16" not in str(e.value)


def test_a_square_over_the_boundary_pads_to_one_factor_block(mx):
    p, even = mx.preprocess(rgb(32, 32), 64)
    assert p.shape == (3, 64, 64) and even == (32, 32)


def test_the_boundary_itself_is_accepted(mx):
    p, _ = mx.preprocess(rgb(22, 22), 64)
    assert p.shape == (3, 64, 64)


def test_an_odd_size_is_made_even_first_and_still_pads(mx):
    p, even = mx.preprocess(rgb(33, 33), 64)
    assert even == (34, 34) and p.shape == (3, 64, 64)


def test_preprocess_matches_the_reference_pipeline(mx):
    z = golden("preprocess")
    i = 0
    while "in%d" % i in z.files:
        p, even = mx.preprocess(z["in%d" % i], 64)
        assert tuple(even) == tuple(z["even%d" % i])
        assert np.array_equal(p, z["out%d" % i])
        i += 1
    assert i >= 5


def test_crop_inverts_the_padding(mx):
    a = rgb(37, 53)
    p, (eh, ew) = mx.preprocess(a, 64)
    back = mx.crop_out(p, 37, 53, eh, ew)
    assert np.array_equal(back, a)


def test_png_round_trip_and_pil_agreement(mx, tmp_path):
    from PIL import Image
    rng = np.random.default_rng(3)
    a = rng.random((3, 29, 41), dtype=np.float32)
    path = str(tmp_path / "x.png")
    mx.png_write(path, a)
    # what we wrote, as PIL reads it: clamp then round half up
    pil = np.asarray(Image.open(path).convert("RGB")).transpose(2, 0, 1).astype(np.int32)
    expect = np.floor(np.clip(a, 0, 1) * np.float32(255) + np.float32(0.5)).astype(np.int32)
    assert np.array_equal(pil, expect)
    back = mx.png_read(path)
    assert np.array_equal(np.round(back * 255).astype(np.int32), expect)


@pytest.mark.parametrize("mode", ["RGB", "RGBA", "L", "LA"])
def test_png_read_matches_pil(mx, mode):
    from PIL import Image
    rng = np.random.default_rng(4)
    chans = {"RGB": 3, "RGBA": 4, "L": 1, "LA": 2}[mode]
    arr = rng.integers(0, 256, (17, 23, chans), dtype=np.uint8)
    img = Image.fromarray(arr[..., 0] if chans == 1 else arr, mode)
    buf = io.BytesIO()
    img.save(buf, "PNG")
    got = mx.png_read_bytes(buf.getvalue())
    want = np.asarray(img.convert("RGB")).transpose(2, 0, 1).astype(np.float32) / np.float32(255.0)
    assert np.array_equal(got, want)


def test_png_rejects_indexed(mx):
    from PIL import Image
    img = Image.fromarray(np.zeros((8, 8), np.uint8), "L").convert("P")
    buf = io.BytesIO()
    img.save(buf, "PNG")
    with pytest.raises(mx.MaximError, match="indexed PNG"):
        mx.png_read_bytes(buf.getvalue())


# ---- the 8-bit side: what the device-side pipeline (mx_gpu_run_rgb8) takes and gives

@pytest.mark.parametrize("h,w", [(22, 22), (33, 97), (64, 64), (65, 130), (853, 1280), (400, 600), (1362, 2048),
                                 (41, 300)])
@pytest.mark.parametrize("factor", [64, 32, 8])
def test_pad_geometry_is_preprocess_without_pixels(mx, h, w, factor):
    p, even = mx.preprocess(np.zeros((3, h, w), np.float32), factor)
    (ph, pw), even2 = mx.pad_geometry(h, w, factor)
    assert (ph, pw) == p.shape[1:] and even2 == tuple(even)


@pytest.mark.parametrize("h,w", [(16, 16), (64, 16), (20, 200)])
def test_pad_geometry_refuses_what_preprocess_refuses(mx, h, w):
    with pytest.raises(mx.MaximError) as a:
        mx.preprocess(np.zeros((3, h, w), np.float32), 64)
    with pytest.raises(mx.MaximError) as b:
        mx.pad_geometry(h, w, 64)
    assert str(a.value).split(": ", 1)[-1] == str(b.value).split(": ", 1)[-1]


@pytest.mark.parametrize("mode", ["RGB", "RGBA", "L", "LA"])
def test_png_rgb8_decode_matches_pil_and_the_float_reader(mx, mode):
    from PIL import Image
    rng = np.random.default_rng(5)
    chans = {"RGB": 3, "RGBA": 4, "L": 1, "LA": 2}[mode]
    arr = rng.integers(0, 256, (19, 27, chans), dtype=np.uint8)
    img = Image.fromarray(arr[..., 0] if chans == 1 else arr, mode)
    buf = io.BytesIO()
    img.save(buf, "PNG")
    data = buf.getvalue()
    got = mx.png_read_rgb8_bytes(data)
    assert got.dtype == np.uint8 and np.array_equal(got, np.asarray(img.convert("RGB")))
    assert mx.png_size(data) == (19, 27)
    # the float reader is exactly these samples divided by 255
    f = mx.png_read_bytes(data)
    assert np.array_equal(f, got.transpose(2, 0, 1).astype(np.float32) / np.float32(255.0))


def test_png_rgb8_write_round_trip(mx, tmp_path):
    from PIL import Image
    a = np.random.default_rng(6).integers(0, 256, (23, 31, 3), dtype=np.uint8)
    path = str(tmp_path / "x8.png")
    mx.png_write_rgb8(path, a)
    assert np.array_equal(np.asarray(Image.open(path).convert("RGB")), a)
    # the float writer quantises to the same file contents
    path2 = str(tmp_path / "xf.png")
    mx.png_write(path2, a.transpose(2, 0, 1).astype(np.float32) / np.float32(255.0))
    assert open(path, "rb").read() == open(path2, "rb").read()


def test_png_size_refuses_non_png(mx):
    with pytest.raises(mx.MaximError, match="not a PNG"):
        mx.png_size(b"GIF89a....................")
