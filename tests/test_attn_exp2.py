"""The FMA-pipe exponential of the attention kernel (exp2_fma2 in
hexkernels_b200/csrc/attn_tc.cu): its coefficients are the relative-minimax
degree-3 fit of 2^f on [-1/2, 1/2] (Remez exchange, recomputed here), and
the float32 evaluation with the Cody-Waite style range reduction stays within
7.6e-5 relative error of exp2 over the exponents the kernel feeds it."""
import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parent.parent / "hexkernels_b200" / "csrc" / "attn_tc.cu"


def kernel_coeffs():
    text = SRC.read_text()
    return [float(re.search(rf"kExp2C{i} = ([0-9.e+-]+)f", text).group(1)) for i in range(4)]


def remez_exp2(deg=3, lo=-0.5, hi=0.5, iters=30):
    """Relative-error minimax polynomial for 2^x on [lo, hi] (Remez exchange
    on a dense grid); returns c0..c_deg and the levelled error."""
    n = deg + 2
    xs = np.cos(np.pi * np.arange(n) / (n - 1))[::-1] * (hi - lo) / 2 + (hi + lo) / 2
    grid = np.linspace(lo, hi, 200001)
    for _ in range(iters):
        A = np.zeros((n, n))
        for i, x in enumerate(xs):
            A[i, :deg + 1] = x ** np.arange(deg + 1)
            A[i, deg + 1] = (-1) ** i * np.exp2(x)
        sol = np.linalg.solve(A, np.exp2(xs))
        c, lev = sol[:deg + 1], sol[deg + 1]
        err = (np.polyval(c[::-1], grid) - np.exp2(grid)) / np.exp2(grid)
        sign = np.sign(err)
        segs = np.split(np.arange(grid.size), np.flatnonzero(np.diff(sign) != 0) + 1)
        ext = [seg[np.argmax(np.abs(err[seg]))] for seg in segs]
        if len(ext) != n:
            ext = sorted(sorted(ext, key=lambda i: -abs(err[i]))[:n])
        xs = grid[ext]
    return c, abs(lev)


def f32(v):
    return np.asarray(v, np.float64).astype(np.float32)


def fma32(a, b, c):
    # single rounding of a*b + c: the product of two float32 is exact in float64
    return f32(a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64))


def exp2_fma2_emulated(x, c):
    """exp2_fma2 step by step in float32 arithmetic."""
    c0, c1, c2, c3 = (np.float32(v) for v in c)
    x = np.maximum(f32(x), np.float32(-125.0))
    t = f32(x + np.float32(12582912.0))
    nf = f32(t - np.float32(12582912.0))
    fr = fma32(nf, np.full_like(nf, -1.0), x)
    p = fma32(np.full_like(fr, c3), fr, np.full_like(fr, c2))
    p = fma32(p, fr, np.full_like(fr, c1))
    p = fma32(p, fr, np.full_like(fr, c0))
    bits = p.view(np.int32).astype(np.int64) + ((t.view(np.uint32).astype(np.int64) << 23) & 0xFFFFFFFF)
    bits = ((bits + 2**31) % 2**32) - 2**31
    return bits.astype(np.int32).view(np.float32)


def test_coefficients_are_the_remez_fit():
    c, lev = remez_exp2()
    assert lev < 7.6e-5
    np.testing.assert_allclose(kernel_coeffs(), c, rtol=2e-6, atol=0)


def test_float32_evaluation_error_bound():
    c = kernel_coeffs()
    # the kernel's exponents: s * scale * log2e - m_ref <= 8 (lazy rescale), and
    # anything below -125 is clamped (those P are zero in fp16)
    x = np.concatenate([np.linspace(-125, 8.5, 2_000_003), np.arange(-125, 9, dtype=np.float64)])
    got = exp2_fma2_emulated(x, c).astype(np.float64)
    exact = np.exp2(f32(x).astype(np.float64))
    rel = np.abs(got - exact) / exact
    assert rel.max() < 7.6e-5, rel.max()
