"""The GELU the CUDA kernels evaluate (csrc/gpu_common.cuh, gelu_f):
max(x, 0) - u * 2^(-x^2 log2(e) / 2) * R(u), u = min(|x|, 5.6), R a fitted
polynomial. This restates that evaluation step by step in numpy fp32 (the
exponential exactly rounded; the device's ex2.approx adds at most about 2 ulp
to the one factor it produces) and bounds its error against the erf form of
GELU in double precision, which src/exec_cpu.rs computes in fp32. The
coefficients are read from the kernel source, so the test follows any refit."""
import os
import re

import numpy as np
import pytest

scipy_special = pytest.importorskip("scipy.special")

SRC = os.path.join(os.path.dirname(__file__), "..", "maxim-rs_b200", "csrc", "gpu_common.cuh")


def coefficients():
    text = open(SRC).read()
    m = re.search(r"kGeluR\[(\d+)\]\s*=\s*\{([^}]*)\}", text)
    assert m, "kGeluR not found in gpu_common.cuh"
    vals = [np.float32(v.strip().rstrip("f")) for v in m.group(2).split(",") if v.strip()]
    assert len(vals) == int(m.group(1))
    return vals


def fma32(a, b, c):
    # a*b is exact in double for fp32 inputs; one rounding of the sum to fp32.
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def gelu_device(x, c):
    x = x.astype(np.float32)
    u = np.minimum(np.abs(x), np.float32(5.6))
    p = np.full_like(x, c[-1])
    for k in range(len(c) - 2, -1, -1):
        p = fma32(p, u, np.full_like(x, c[k]))
    with np.errstate(over="ignore"):
        a = (x * np.float32(-0.72134752)).astype(np.float32)
        a = (a * x).astype(np.float32)
    e = np.exp2(a.astype(np.float64)).astype(np.float32)
    s = (u * e).astype(np.float32)
    return fma32(-s, p, np.maximum(x, np.float32(0)))


def gelu_exact(x):
    x = x.astype(np.float64)
    return 0.5 * x * (1.0 + scipy_special.erf(x / np.sqrt(2.0)))


def test_gelu_polynomial_error_bound():
    c = coefficients()
    xs = np.concatenate([
        np.linspace(-12, 12, 1_200_001, dtype=np.float64),
        np.linspace(-1e-3, 1e-3, 100_001, dtype=np.float64),
        np.array([5.6, -5.6, 5.6000001, 100.0, -100.0, 1e30, -1e30, 0.0, -0.0]),
    ]).astype(np.float32)
    got = gelu_device(xs, c).astype(np.float64)
    ref = gelu_exact(xs)
    err = np.abs(got - ref)
    ulp_x = np.spacing(np.maximum(np.abs(xs), np.float32(1e-30))).astype(np.float64)
    # Within 1.5 ulp of |x| everywhere (the erf form loses that much to the
    # rounding of 1 + erf for x < 0) ...
    assert (err / ulp_x).max() <= 1.5
    # ... and within 3 ulp of the result where the result is not tiny against
    # x (x > -0.7). The worst case, near x = -0.3, is fp32 rounding in the
    # product u * e * R, not the fit: a degree-13 fit still shows 2.2 ulp.
    big = np.abs(ref) >= 0.25 * np.abs(xs.astype(np.float64))
    ulp_g = np.spacing(np.abs(ref[big]).astype(np.float32)).astype(np.float64)
    assert (err[big] / ulp_g).max() <= 3.0


def test_gelu_polynomial_special_values():
    c = coefficients()
    x = np.array([np.inf, -np.inf, np.nan, 0.0], dtype=np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        g = gelu_device(x, c)
    assert g[0] == np.inf and g[1] == 0.0 and np.isnan(g[2]) and g[3] == 0.0


def paired_coefficients():
    text = open(SRC).read()
    m = re.search(r"kGeluRw\[(\d+)\]\s*=\s*\{([^}]*)\}", text)
    assert m, "kGeluRw not found in gpu_common.cuh"
    return [np.float32(v.strip().rstrip("f")) for v in m.group(2).split(",") if v.strip()]


def gelu_device_paired(x, cw):
    """gelu_f2's evaluation: Horner over w = -min(|x|, 5.6) with kGeluRw."""
    x = x.astype(np.float32)
    w = np.maximum(-np.abs(x), np.float32(-5.6))
    p = np.full_like(x, cw[-1])
    for k in range(len(cw) - 2, -1, -1):
        p = fma32(p, w, np.full_like(x, cw[k]))
    with np.errstate(over="ignore"):
        a = (x * np.float32(-0.72134752)).astype(np.float32)
        a = (a * x).astype(np.float32)
    e = np.exp2(a.astype(np.float64)).astype(np.float32)
    s = (w * e).astype(np.float32)
    return fma32(s, p, np.maximum(x, np.float32(0)))


def test_paired_gelu_is_bit_identical_to_the_scalar_one():
    """The epilogue's paired GELU (gelu_f2) must give exactly gelu_f's bits,
    so a fused GELU step still equals the unfused op bit for bit."""
    c, cw = coefficients(), paired_coefficients()
    assert len(c) == len(cw)
    for k in range(len(c)):
        assert cw[k] == np.float32((-1) ** k) * c[k], k
    xs = np.concatenate([np.linspace(-12, 12, 600_001, dtype=np.float64),
                         np.array([5.6, -5.6, 0.0, -0.0, 1e30, -1e30, 3e-39, -3e-39])]).astype(np.float32)
    a, b = gelu_device(xs, c), gelu_device_paired(xs, cw)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
