"""Shared fixtures. `gpu`-marked tests need a CUDA device (B200); the rest run
on CPU only and never launch a kernel."""
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")
    # Incremental native build; a no-op when the shipped libraries are current.
    build = importlib.import_module("maxim-rs_b200.build")
    build.build()


@pytest.fixture(scope="session")
def mx():
    return importlib.import_module("maxim-rs_b200")


@pytest.fixture(scope="session")
def synth():
    return importlib.import_module("maxim-rs_b200.synth")


@pytest.fixture(scope="session")
def oracle():
    return importlib.import_module("oracle")


@pytest.fixture(scope="session")
def ckpt_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("ckpt")


@pytest.fixture(scope="session")
def checkpoint(ckpt_dir, synth):
    """checkpoint(variant, seed, gain=1.0, rich=False) -> path of a synthetic checkpoint."""

    def make(variant, seed, gain=1.0, rich=False):
        path = os.path.join(str(ckpt_dir), "%s_%d_%g_%d.safetensors" % (variant, seed, gain, int(rich)))
        return synth.checkpoint(path, variant, seed, gain, rich)

    return make


def golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


GOLDEN_CASES = ["s2_64_he", "s2_64_rich", "s3_64x128", "m1_64"]


def psnr(ref, got, peak=None):
    ref = np.asarray(ref, np.float64)
    err = np.asarray(got, np.float64) - ref
    mse = float((err ** 2).mean())
    if peak is None:
        peak = float(np.abs(ref).max())
    return float("inf") if mse == 0 else 10.0 * np.log10(peak * peak / mse)


def rel_rms(ref, got):
    ref = np.asarray(ref, np.float64)
    err = np.asarray(got, np.float64) - ref
    return float(np.sqrt((err ** 2).mean()) / max(np.sqrt((ref ** 2).mean()), 1e-30))


def to_u8(a):
    """The reference's PNG write: clamp to [0,1], then round half up (src/image.rs:97-98)."""
    a = np.clip(np.asarray(a, np.float32), 0.0, 1.0)
    return np.floor(a * np.float32(255.0) + np.float32(0.5)).astype(np.int32)


def lsb_fraction(ref, got):
    """Fraction of 8-bit output pixels within 1 LSB of the reference's."""
    return float((np.abs(to_u8(ref) - to_u8(got)) <= 1).mean())
