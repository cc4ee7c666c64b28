"""The GEMM epilogue's GELU / GELU' pair (gelu_and_grad2 in
flodl_b200/csrc/kernels/sm100_ptx.cuh: erf after Abramowitz & Stegun 7.1.26,
sharing its exponential with GELU'), restated in float32 numpy and checked
against the exact erf forms."""
import math

import numpy as np


def _gelu_pair(x):
    x = x.astype(np.float32)
    kp = np.float32(0.3275911 * 0.70710678118654752)
    a = [np.float32(c) for c in (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)]
    t = (np.float32(1) / (np.abs(x) * kp + np.float32(1))).astype(np.float32)
    poly = a[4] * t + a[3]
    for c in (a[2], a[1], a[0]):
        poly = (poly * t + c).astype(np.float32)
    poly = (poly * t).astype(np.float32)
    e = np.exp2((x * (x * np.float32(-0.72134752044448170))).astype(np.float32)).astype(np.float32)
    h = (poly * e * np.float32(-0.5) + np.float32(0.5)).astype(np.float32)
    cdf = (np.copysign(h, x) + np.float32(0.5)).astype(np.float32)
    g = x * cdf
    d = (x * e) * np.float32(0.39894228040143268) + cdf
    return g.astype(np.float32), d.astype(np.float32)


def test_gelu_pair_matches_exact_erf_forms():
    x = np.concatenate([np.linspace(-12, 12, 200001), np.array([0.0, -0.0, 1e-30, -1e-30])])
    g, d = _gelu_pair(x)
    erf = np.vectorize(math.erf)
    phi = 0.5 * (1 + erf(x / math.sqrt(2)))
    g_ref = x * phi
    d_ref = phi + x * np.exp(-0.5 * x * x) / math.sqrt(2 * math.pi)
    assert np.max(np.abs(g - g_ref)) < 2e-6
    assert np.max(np.abs(d - d_ref)) < 2e-6
