"""CPU check of the software exp2 used for part of the softmax exponentials
(blackwell_b200/csrc/softmax_math.cuh: ex2_poly2), evaluated step by step in
IEEE float32 with numpy, against the float64 exp2."""
import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parent.parent / "blackwell_b200" / "csrc" / "softmax_math.cuh"


def _coeffs():
    text = SRC.read_text()
    return [np.float32(float(re.search(rf"kExpA{i} = ([0-9.e+-]+)f", text).group(1))) for i in (1, 2, 3)]


def ex2_poly(x):
    a1, a2, a3 = _coeffs()
    f32 = np.float32
    x = np.maximum(x.astype(f32), f32(-126))
    t = (x + f32(12582912.0)).astype(f32)
    j = (t - f32(12582912.0)).astype(f32)
    f = (x - j).astype(f32)
    p = (f * a3 + a2).astype(f32)
    p = (p * f + a1).astype(f32)
    p = (p * f + f32(1)).astype(f32)
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_bound():
    x = np.linspace(-125.0, 8.0, 400001).astype(np.float32)
    got = ex2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert rel.max() < 1.1e-4          # well below the bf16 step (3.9e-3) of P


def test_underflow_and_masked_inputs_give_tiny_non_negative():
    x = np.array([-np.inf, -1e30, -500.0, -126.4, -130.0], dtype=np.float32)
    y = ex2_poly(x)
    assert np.all(y >= 0) and np.all(y < 2e-38)
