"""Fit the polynomial the softmax kernels use to evaluate 2^x on the FMA pipe.

Method: range reduction x = n + f with n = rint(x), f in [-1/2, 1/2], so 2^x = 2^n * 2^f; 2^n is
applied by adding n to the float's exponent field, and 2^f is approximated by
    p(f) = c0 + c1 f + c2 f^2 + ... + cd f^d
whose coefficients minimise the maximum RELATIVE error |p(f) / 2^f - 1| over [-1/2, 1/2]
(Remez exchange with weight 2^-f).  The kernels clamp x at -126 first: with p(f) >= 2^-1/2 the
rebuilt exponent then never goes below 0.
The coefficients are then rounded to float32 and the error is re-measured in float32 Horner
arithmetic (what the kernel does).

    python fused-attention_b200/csrc/fit_exp2_poly.py          # prints coefficients and errors
"""
import numpy as np


def remez(deg, iters=40):
    lo, hi = -0.5, 0.5
    # initial reference: Chebyshev extrema, deg + 2 points (deg + 1 coefficients + error level)
    m = deg + 2
    x = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * np.arange(m)[::-1] / (m - 1))
    grid = np.linspace(lo, hi, 200001)
    c = None
    for _ in range(iters):
        # sum c_k x^k / 2^x - 1 = (-1)^i E   ->   sum c_k x^k - (-1)^i E 2^x = 2^x
        A = np.zeros((m, m))
        for k in range(deg + 1):
            A[:, k] = x ** k
        A[:, deg + 1] = -((-1.0) ** np.arange(m)) * 2.0 ** x
        sol = np.linalg.solve(A, 2.0 ** x)
        c = sol[:deg + 1]
        err = sum(c[k] * grid ** k for k in range(deg + 1)) / 2.0 ** grid - 1.0
        # new reference: the extremum of each sign-alternating segment
        sign = np.sign(err)
        idx = np.flatnonzero(np.diff(sign) != 0)
        bounds = np.concatenate(([0], idx + 1, [len(grid)]))
        ext = [s + np.argmax(np.abs(err[s:e])) for s, e in zip(bounds[:-1], bounds[1:])]
        if len(ext) >= m:
            # keep the m largest-|err| points in order, preserving alternation
            ext = sorted(sorted(ext, key=lambda i: -abs(err[i]))[:m])
            x = grid[ext]
    return c, float(np.abs(err).max())


def f32_error(c):
    """Max relative error of the float32 kernel arithmetic over a dense set of x in [-127, 8]."""
    xs = np.linspace(-125.0, 8.0, 2000001).astype(np.float32)
    t = (xs + np.float32(12582912.0)).astype(np.float32)
    n = (t - np.float32(12582912.0)).astype(np.float32)
    f = (xs - n).astype(np.float32)
    p = np.float32(c[-1])
    for ck in c[-2::-1]:
        p = (p * f + np.float32(ck)).astype(np.float32)
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    got = bits.view(np.float32).astype(np.float64)
    ref = np.exp2(xs.astype(np.float64))
    return float(np.abs(got / ref - 1.0).max())


if __name__ == "__main__":
    for deg in (3, 4):
        c, e = remez(deg)
        c32 = [float(np.float32(v)) for v in c]
        print(f"degree {deg}: minimax relative error {e:.3e}; float32 kernel error {f32_error(c32):.3e}")
        print("   coefficients c0..c%d: %s" % (deg, ", ".join(f"{v:.9e}f" for v in c32)))
