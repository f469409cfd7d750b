"""The `maxim` CLI (src/main.rs): PNG in, pad to 64, GPU pass, crop, PNG out."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT

CLI = os.path.join(ROOT, "maxim-rs_b200", "maxim")


def test_cli_refuses_cpu_and_missing_model():
    r = subprocess.run([CLI, "--device", "cpu", "-m", "x"], capture_output=True, text=True)
    assert r.returncode == 1 and "GPU only" in r.stderr
    r = subprocess.run([CLI, "-i", "x.png"], capture_output=True, text=True)
    assert r.returncode == 2 and "--model is required" in r.stderr


@pytest.mark.gpu
def test_cli_matches_the_library_pipeline(mx, synth, checkpoint, tmp_path):
    ckpt = checkpoint("S-1", 5, 0.5)
    img = synth.image_uniform(synth.input_rng(5), 45, 70)
    src, dst = str(tmp_path / "in.png"), str(tmp_path / "out.png")
    mx.png_write(src, img)
    r = subprocess.run([CLI, "-m", ckpt, "-i", src, "-o", dst, "-q"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    got = mx.png_read(dst)
    x = mx.png_read(src)
    padded, (eh, ew) = mx.preprocess(x, 64)
    out = mx.Gpu(mx.Plan(mx.Weights(ckpt), padded.shape[1], padded.shape[2])).run(padded)
    want = np.floor(np.clip(mx.crop_out(out, 45, 70, eh, ew), 0, 1) * np.float32(255) + np.float32(0.5))
    assert got.shape == (3, 45, 70)
    assert np.array_equal(np.round(got * 255), want)


@pytest.mark.gpu
def test_cli_batch_mode(mx, synth, checkpoint, tmp_path):
    """`--batch in out`: every PNG restored through the batch runner (two
    shapes, so two plans), a broken PNG reported and skipped with exit
    status 1, the others written and equal to the single-image CLI's."""
    ckpt = checkpoint("S-1", 5, 0.5)
    src, dst = tmp_path / "in", tmp_path / "out"
    src.mkdir()
    dst.mkdir()
    shapes = [(45, 70), (64, 64), (45, 70)]
    for k, (h, w) in enumerate(shapes):
        mx.png_write(str(src / ("img%d.png" % k)), synth.image_uniform(synth.input_rng(10 + k), h, w))
    (src / "broken.png").write_bytes(b"\x89PNG\r\n\x1a\nnot really")
    r = subprocess.run([CLI, "-m", ckpt, "--batch", str(src), str(dst), "--devices", "0"], capture_output=True,
                       text=True)
    assert r.returncode == 1, r.stderr
    assert "broken.png" in r.stderr and "wrote 3 image(s)" in r.stderr
    for k in range(3):
        one = str(tmp_path / ("one%d.png" % k))
        r1 = subprocess.run([CLI, "-m", ckpt, "-i", str(src / ("img%d.png" % k)), "-o", one, "-q"],
                            capture_output=True, text=True)
        assert r1.returncode == 0, r1.stderr
        assert np.array_equal(mx.png_read(one), mx.png_read(str(dst / ("img%d.png" % k))))
