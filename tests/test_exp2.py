"""The prefill softmax's exponentials, evaluated on the GPU on dense input grids.

The tcgen05 kernel computes P = 2^x with two routines (csrc/common.cuh): the
MUFU's ex2.approx.ftz.f32 for most columns and, for a few columns per row, a
polynomial on the FMA pipe (f2_exp2_poly: x = n + f with n = round(x), 2^f by
a fitted degree-3 minimax polynomial, 2^n added to the exponent field). Here
both are checked against float64 2^x on the host and against CUDA's exp2f:
relative error <= 7.5e-5 for the polynomial on [-125.99, 8] (the kernel only
evaluates x <= 8: the running max it subtracts is at most 8 behind), and a
clamp below -126 (and for -inf, which masked scores become) to a value under
2^-125, i.e. 0 once P is rounded to fp16.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

POLY_REL = 7.5e-5   # the polynomial's stated bound
MUFU_REL = 2e-6     # ex2.approx.ftz.f32 on normal results (a loose bound)


def grid():
    dense = np.linspace(-125.99, 8.0, 1 << 22, dtype=np.float64)
    # Around every integer and half-integer: the range reduction's switch points.
    k = np.arange(-125, 9, dtype=np.float64)
    off = np.linspace(-0.5, 0.5, 4097)
    near = (k[:, None] + off[None, :]).ravel()
    near = near[(near >= -125.99) & (near <= 8.0)]
    return np.concatenate([dense, near]).astype(np.float32)


def run(ext, x_np):
    x = torch.from_numpy(x_np).cuda()
    poly, mufu, lib = (t.cpu().numpy() for t in ext.selftest_exp2(x))
    return poly, mufu, lib


def test_polynomial_relative_error(ext):
    x = grid()
    poly, mufu, lib = run(ext, x)
    true = np.exp2(x.astype(np.float64))
    rel_poly = np.abs(poly.astype(np.float64) - true) / true
    rel_lib = np.abs(poly.astype(np.float64) - lib) / lib
    assert rel_poly.max() <= POLY_REL, (rel_poly.max(), x[rel_poly.argmax()])
    assert rel_lib.max() <= POLY_REL + 1e-6, (rel_lib.max(), x[rel_lib.argmax()])
    # The MUFU path, on the same grid where its results are normal (x >= -126).
    rel_mufu = np.abs(mufu.astype(np.float64) - true) / true
    assert rel_mufu.max() <= MUFU_REL, (rel_mufu.max(), x[rel_mufu.argmax()])


def test_polynomial_clamp_below_minus_126(ext):
    x = np.concatenate([np.linspace(-200.0, -126.0, 100001), [-np.inf, -1e30, -126.0]])
    x = x.astype(np.float32)
    poly, mufu, _ = run(ext, x)
    assert np.all(poly > 0) and np.all(poly <= 2.0 ** -125), poly.max()
    # Both routines give 0 after the fp16 rounding of P.
    assert np.all(torch.from_numpy(poly).half().numpy() == 0)
    assert np.all(torch.from_numpy(mufu).half().numpy() == 0)


def test_polynomial_at_exact_powers(ext):
    """At integers f = 0 and 2^x = c0 * 2^n: within the bound, never above 1 at 0."""
    x = np.arange(-125, 9, dtype=np.float32)
    poly, _, _ = run(ext, x)
    true = np.exp2(x.astype(np.float64))
    assert np.all(np.abs(poly - true) / true <= POLY_REL)
    assert poly[x == 0][0] <= 1.0


def test_odd_length_input(ext):
    """The kernel evaluates pairs; an odd count handles its last element alone."""
    x = np.array([0.5, -3.25, 7.0], dtype=np.float32)
    poly, mufu, lib = run(ext, x)
    assert np.allclose(poly, np.exp2(x), rtol=POLY_REL, atol=0)
    assert np.allclose(lib, np.exp2(x), rtol=1e-6, atol=0)
