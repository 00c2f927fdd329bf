"""Error bound of the FMA-pipe exponential used by the selection kernel.

`exp2_poly_x2` (csrc/common.cuh) evaluates 2^x as 2^n * q(f) with n = rint(x)
and a quartic q on [-0.5, 0.5]. The selection kernel computes a quarter of its
exponentials this way, so its energies stay well inside the 1e-5 relative band
in which the parity rules allow a block to flip only if the relative error of
one exponential is far below 1e-5. This test reads the coefficients from the
shipped header and evaluates the same float32 operation sequence on the CPU.
"""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np

HEADER = Path(__file__).resolve().parents[1] / "flashprefillv2-mlx_b200" / "csrc" / "common.cuh"


def _coefficients() -> list[float]:
    text = HEADER.read_text()
    body = text[text.index("exp2_poly_x2(float2 x) {"):]
    body = body[: body.index("\n}\n")]
    # make_float2(c, c) pairs in Horner order: highest degree first
    found = re.findall(r"make_float2\(([0-9.]+)f, \1f\)", body)
    coeffs = [float(v) for v in found if v not in ("12582912.", "12582912")]
    coeffs = [c for c in coeffs if c != 12582912.0]
    assert len(coeffs) == 5, coeffs
    return coeffs


def _fma32(a, b, c):
    return (a.astype(np.float64) * b + c).astype(np.float32)


def _poly_exp2(x: np.ndarray, coeffs: list[float]) -> np.ndarray:
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    n = (t - magic).astype(np.float32)
    f = _fma32(n, np.float32(-1.0), x)
    c4, c3, c2, c1, c0 = (np.float32(c) for c in coeffs)
    p = _fma32(np.full_like(f, c4), f, c3)
    p = _fma32(p, f, c2)
    p = _fma32(p, f, c1)
    p = _fma32(p, f, c0)
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    return bits.view(np.float32)


def test_exp2_poly_relative_error_bound():
    coeffs = _coefficients()
    x = np.concatenate([
        np.linspace(-125.0, 16.0, 2_000_001, dtype=np.float64),
        -np.logspace(-8, 2, 2001),
        np.array([0.0, -0.5, 0.5, -1.5, 15.5]),
    ]).astype(np.float32)
    got = _poly_exp2(x, coeffs).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got / ref - 1.0)
    assert rel.max() < 3e-6, rel.max()


def test_exp2_poly_clamps_without_sign_or_exponent_wrap():
    coeffs = _coefficients()
    x = np.array([-1e30, -3.0e38, -200.0, -127.0, -126.0], dtype=np.float32)
    got = _poly_exp2(x, coeffs)
    assert np.all(got >= 0.0) and np.all(got < 2.0 ** -124)


def test_coefficients_are_the_minimax_relative_error_fit():
    """The shipped coefficients are the Remez (minimax relative error) quartic for
    2^f on [-0.5, 0.5] (tests/exp2_poly_fit.py), to float32-level agreement."""
    from tests.exp2_poly_fit import float32_coefficients, remez_exp2

    _, levelled = remez_exp2()
    assert levelled < 2.7e-6
    fitted = np.array(float32_coefficients())
    shipped = np.array(_coefficients())
    assert np.allclose(fitted, shipped, rtol=2e-5, atol=0.0), (fitted, shipped)
