"""The division-free normal CDF of the GELU epilogues (``norm_cdf_poly`` /
``norm_cdf_poly2`` in csrc/common.cuh), evaluated here in fp32 exactly as the
kernel does (t held at 1 beyond the fitted range, Horner, saturating final
FMA), against torch.erf in fp64: max |error| <= 1e-5 everywhere, exactly 0 / 1
in the tails."""
import re
from pathlib import Path

import numpy as np
import torch

SRC = Path(__file__).resolve().parents[1] / "csrc" / "common.cuh"


def _coeffs():
    text = SRC.read_text()
    scale = float(re.search(r"#define PD_CDF_T_SCALE ([0-9.e-]+)f", text).group(1))
    body = text.split("#define PD_CDF_HORNER", 1)[1].split("#define PD_ID", 1)[0]
    first = re.search(r"R = FMA\(K\((-?[0-9.e-]+)f\), T, K\((-?[0-9.e-]+)f\)\)", body)
    rest = re.findall(r"R = FMA\(R, T, K\((-?[0-9.e-]+)f\)\)", body)
    return scale, [float(first.group(1)), float(first.group(2))] + [float(v) for v in rest]


def _cdf_f32(x):
    scale, ks = _coeffs()
    x = x.astype(np.float32)
    t = np.minimum((x * x * np.float32(scale) - np.float32(1)).astype(np.float32), np.float32(1))
    r = np.full_like(t, np.float32(ks[0]))
    for k in ks[1:]:
        r = (r * t + np.float32(k)).astype(np.float32)
    return np.clip((np.float32(0.5) + x * r).astype(np.float32), 0, 1)


def test_norm_cdf_poly_error_bound():
    _, ks = _coeffs()
    assert len(ks) == 10                                   # degree 9
    x = np.linspace(-10, 10, 2_000_001)
    ref = (0.5 * (1 + torch.erf(torch.from_numpy(x) / np.sqrt(2.0)))).numpy()
    err = np.abs(_cdf_f32(x).astype(np.float64) - ref)
    assert err.max() <= 1e-5, err.max()
    gelu_err = np.abs(x * _cdf_f32(x) - x * ref)
    assert gelu_err.max() <= 3e-5, gelu_err.max()


def test_norm_cdf_poly_tails_are_exact():
    x = np.concatenate([np.linspace(4.5, 60, 100_001), np.array([1e3, 1e6, 3e38])])
    assert (_cdf_f32(x) == 1).all() and (_cdf_f32(-x) == 0).all()
    y = _cdf_f32(np.linspace(-6, 6, 200_001))
    assert (y >= 0).all() and (y <= 1).all()
