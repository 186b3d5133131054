"""CPU restatement of the kernels' FMA-pipe exp2 (fa_sm100.cuh: exp2_poly2), checked in
float32 over its whole input range.

The kernel evaluates part of each softmax row's 2^x (x <= 0, or up to the rescale threshold above
the running max) without the MUFU unit: x is clamped at -125, n = round(x) comes from adding
1.5 * 2^23, f = x - n lies in [-1/2, 1/2], 2^f is a degree-3 polynomial and n is added to the
result's exponent field.  The coefficients and the clamp are read from the kernel source, so this
test follows the code.  Bound: relative error <= 1e-4 (half an fp16 ulp is 2.4e-4), every result
finite and normal."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                   "fused-attention_b200", "csrc", "fa_sm100.cuh")


def _kernel_constants():
    text = open(SRC).read()
    body = text[text.index("exp2_poly2(uint64_t x2)"):]
    body = body[:body.index("\n}\n")]
    clamp = float(re.search(r"fmaxf\(f2lo\(x2\), (-?[0-9.]+)f\)", body).group(1))
    coeffs = [float(c) for c in re.findall(r"f2\((-?[0-9.]+)f, \1f\)", body) if float(c) != 12582912.0]
    # ffma2 order in the source: c3*f + c2, then *f + c1, then *f + c0
    return clamp, coeffs


def exp2_poly(x, clamp, coeffs):
    """The kernel's bit arithmetic in float32."""
    c3, c2, c1, c0 = (np.float32(c) for c in coeffs)
    xc = np.maximum(x.astype(np.float32), np.float32(clamp))
    magic = np.float32(12582912.0)
    j = (xc + magic).astype(np.float32)
    n = (j - magic).astype(np.float32)
    f = (xc - n).astype(np.float32)
    p = (c3 * f + c2).astype(np.float32)
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    bits = (p.view(np.uint32).astype(np.uint64) + ((j.view(np.uint32).astype(np.uint64) << 23) & 0xFFFFFFFF))
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32), xc


def test_kernel_polynomial_constants_are_found():
    clamp, coeffs = _kernel_constants()
    assert clamp == -125.0
    assert len(coeffs) == 4


def test_exp2_polynomial_accuracy_over_the_input_range():
    clamp, coeffs = _kernel_constants()
    x = np.concatenate([np.linspace(-200.0, 8.0, 800001), np.array([-125.0, -124.5, -0.5, 0.0, 0.5, 7.99])])
    got, xc = exp2_poly(x.astype(np.float32), clamp, coeffs)
    ref = np.exp2(xc.astype(np.float64))
    assert np.isfinite(got).all()
    assert (got > 0).all() and (np.abs(got) >= np.finfo(np.float32).tiny).all()  # normal numbers
    assert float((np.abs(got - ref) / ref).max()) <= 1e-4
    # masked scores (-inf) clamp to 2^-125: negligible next to the row's largest term, which is 1
    m, _ = exp2_poly(np.array([-np.inf], np.float32), clamp, coeffs)
    assert 0 < float(m[0]) < 2.0 ** -124
