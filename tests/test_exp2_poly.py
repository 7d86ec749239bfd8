"""The forward kernel's FMA-pipe exponential (``exp2_poly`` in
``csrc/ring_fwd.cuh``, variant 2): its coefficients are the ones the Remez
exchange in ``tests/gen_exp2_poly.py`` derives, and the device steps, emulated
in float32 here, stay within 1e-4 relative error of 2**x on (-126, 0] (the
bf16 P it feeds is rounded to 2**-9) and give exactly 0 at or below -126 and
for masked keys (-inf), as ``ex2.approx.ftz`` does."""

import importlib.util
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "hcp_vllm_plugin_b200", "csrc")


def _header_coeffs():
    src = open(os.path.join(CSRC, "ring_fwd.cuh")).read()
    m = re.search(r"kC0 = ([0-9.]+)f, kC1 = ([0-9.]+)f, kC2 = ([0-9.]+)f, kC3 = ([0-9.]+)f", src)
    assert m, "exp2_poly coefficients not found"
    return [np.float32(float(v)) for v in m.groups()]


def _fma32(a, b, c):
    # one rounding, as the device's fmaf
    return (a.astype(np.float64) * b + c).astype(np.float32)


def exp2_poly(x):
    """The device steps of exp2_poly in float32."""
    c0, c1, c2, c3 = _header_coeffs()
    magic = np.float32(12582912.0)
    x = np.asarray(x, np.float32)
    xc = np.maximum(x, np.float32(-126.0))
    t = (xc + magic).astype(np.float32)
    f = (xc - (t - magic).astype(np.float32)).astype(np.float32)
    p = _fma32(_fma32(_fma32(np.full_like(f, c3), f, c2), f, c1), f, c0)
    bits = p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)
    r = (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return np.where(x > -126.0, r, np.float32(0.0))


def test_coefficients_are_the_remez_solution():
    spec = importlib.util.spec_from_file_location("gen_exp2_poly", os.path.join(ROOT, "tests", "gen_exp2_poly.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    c, err = gen.remez_exp2()
    assert err < 8e-5
    np.testing.assert_array_equal(np.float32(c), np.array(_header_coeffs(), np.float32))


def test_relative_error_and_underflow():
    x = np.concatenate([np.linspace(-125.9, 0.0, 2_000_001, dtype=np.float32),
                        np.float32([0.0, -0.5, 0.5 - 1.0, -1.0, -7.25, -125.5])])
    got = exp2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() < 1e-4, rel.max()
    low = np.float32([-126.0, -126.5, -200.0, -np.inf])
    assert np.all(exp2_poly(low) == 0.0)
    assert abs(float(exp2_poly(np.float32([0.0]))[0]) - 1.0) < 1e-4
