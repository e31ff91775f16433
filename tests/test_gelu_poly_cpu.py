"""The division-free normal CDF of the GELU epilogues (``norm_cdf_poly`` in
csrc/common.cuh), evaluated here in fp32 exactly as the kernel does (clamp,
shift, Horner), against torch.erf in fp64: max |error| <= 1e-5 on [-10, 10]."""
import re
from pathlib import Path

import numpy as np
import torch

SRC = Path(__file__).resolve().parents[1] / "csrc" / "common.cuh"


def _coeffs():
    body = SRC.read_text().split("float norm_cdf_poly(float x) {", 1)[1].split("}", 1)[0]
    clamp = float(re.search(r"fmaxf\(x, -([0-9.]+)f\)", body).group(1))
    scale = float(re.search(r"fmaf\(xc \* xc, ([0-9.]+)f, -1\.0f\)", body).group(1))
    first = re.search(r"float r = fmaf\((-?[0-9.e-]+)f, t, (-?[0-9.e-]+)f\)", body)
    rest = re.findall(r"r = fmaf\(r, t, (-?[0-9.e-]+)f\)", body)
    hi_to_lo = [float(first.group(1)), float(first.group(2))] + [float(v) for v in rest]
    return clamp, scale, hi_to_lo


def _cdf_f32(x):
    clamp, scale, ks = _coeffs()
    x = x.astype(np.float32)
    xc = np.clip(x, np.float32(-clamp), np.float32(clamp))
    t = (xc * xc * np.float32(scale) - np.float32(1)).astype(np.float32)
    r = np.full_like(t, np.float32(ks[0]))
    for k in ks[1:]:
        r = (r * t + np.float32(k)).astype(np.float32)
    p = (np.float32(0.5) + xc * r).astype(np.float32)
    return np.where(np.abs(x) < np.float32(clamp), p, (x > 0).astype(np.float32))


def test_norm_cdf_poly_error_bound():
    _, _, ks = _coeffs()
    assert len(ks) == 10                                   # degree 9
    x = np.linspace(-10, 10, 2_000_001)
    ref = (0.5 * (1 + torch.erf(torch.from_numpy(x) / np.sqrt(2.0)))).numpy()
    err = np.abs(_cdf_f32(x).astype(np.float64) - ref)
    assert err.max() <= 1e-5, err.max()
    gelu_err = np.abs(x * _cdf_f32(x) - x * ref)[np.abs(x) <= 10]
    assert gelu_err.max() <= 3e-5, gelu_err.max()


def test_norm_cdf_poly_is_bounded_with_exact_tails():
    x = np.linspace(-60, 60, 200_001)
    y = _cdf_f32(x)
    assert (y >= -1e-5).all() and (y <= 1 + 1e-5).all()
    assert (y[x <= -4.5] == 0).all() and (y[x >= 4.5] == 1).all()
