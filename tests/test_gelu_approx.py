"""The GEGLU epilogue's erf (Abramowitz & Stegun 7.1.26), evaluated on the host.

The GEMM kernel computes gelu(x) = relu(x) - |x| * erfc(|x| / sqrt(2)) / 2 with
erfc from A&S 7.1.26 (|error| <= 1.5e-7).  This restates that arithmetic in
float64 and float32 with the kernel's constants and checks it against the exact
erf GELU of the reference (src/tensor.cpp:96-98): the approximation stays far
below one bf16 rounding step (2^-9 relative) over the range activations take.
"""
import math

import numpy as np

P = 0.3275911
A = (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def gelu_as(x, dtype):
    x = np.asarray(x, dtype)
    ax = np.abs(x)
    t = dtype(1) / (dtype(1) + dtype(P / math.sqrt(2.0)) * ax)
    p = dtype(0)
    for a in reversed(A):
        p = (p + dtype(a)) * t  # Horner: t (a1 + t (a2 + ... + t a5))
    tail = dtype(0.5) * p * np.exp2(-(x * x) * dtype(0.5 / math.log(2.0)))  # 1 - Phi(|x|)
    return np.maximum(x, dtype(0)) - ax * tail


def gelu_exact(x):
    return np.array([0.5 * v * (1.0 + math.erf(v / math.sqrt(2.0))) for v in x])


def test_erf_bound_float64():
    x = np.linspace(-12.0, 12.0, 20001)
    err = np.abs(gelu_as(x, np.float64) - gelu_exact(x))
    # |x| * |erfc error| / 2 with |erfc error| <= 1.5e-7
    assert np.all(err <= 0.5 * 1.5e-7 * np.abs(x) + 1e-15)


def test_float32_far_below_bf16_step():
    x = np.linspace(-10.0, 10.0, 40001)
    got = gelu_as(x.astype(np.float32), np.float32).astype(np.float64)
    want = gelu_exact(x)
    rel = np.abs(got - want) / np.maximum(np.abs(want), 1.0)
    assert rel.max() < 2.0 ** -9 / 64


def gelu_tanh(x, dtype):
    """The tanh form the e4m3-output GEGLU epilogue (SJ_PREC_FP8_TENSOR) uses,
    with its constants, in the given precision (tanh itself exact here; the
    kernel's tanh.approx.f32 adds ~2^-11 relative to the tanh)."""
    x = np.asarray(x, dtype)
    k0 = dtype(0.7978845608028654)
    k1 = dtype(0.044715) * k0
    inner = x * (x * x * k1 + k0)
    h = dtype(0.5) * x
    return h * np.tanh(inner) + h


def test_tanh_form_within_e4m3_rounding():
    """The tanh form's distance from the erf GELU: at most 4.8e-4 absolute,
    and below 1/64 of |gelu(x)| (a quarter of e4m3's relative rounding step
    of 2^-4) wherever |gelu(x)| >= 0.05."""
    x = np.linspace(-12.0, 12.0, 48001)
    want = gelu_exact(x)
    got = gelu_tanh(x, np.float64)
    err = np.abs(got - want)
    assert err.max() <= 4.8e-4
    big = np.abs(want) >= 0.05
    assert np.all(err[big] <= np.abs(want[big]) / 64)
