"""Accuracy of the kernels' FMA-pipe exponentials (exp2_poly, exp2_poly2 in csrc/nva_ptx.cuh; the softmax of the
single-tile prefill kernel puts a quarter of its weights through exp2_poly2).  Their method: a Cody-Waite split
x = n + f (n = rint(x), f in [-1/2, 1/2]), 2^f from a degree-3 polynomial fitted for minimal relative error (7.48e-5
in exact arithmetic), 2^n added into the exponent field; inputs below -126 are clamped there.  Checked on the GPU
against float64 2^x over the softmax's range (every 2^-12 step of [-125.5, 8] plus random points), at the bottom of
the range and the clamp, and beside CUDA's own exp2f on the same inputs.  At the bottom, where n = -126 and
2^f's polynomial comes out below 1 (x within ~1e-4 above -126, and the clamped inputs), the exponent-field add
yields a subnormal whose relative error is up to 1.5e-4 (absolute error below 2^-138): softmax weights of that size
add nothing to a row sum of at least 1."""
import ctypes
import os
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import exp2_build  # noqa: E402

pytestmark = pytest.mark.gpu

BOUND = 7.6e-5    # the fit's 7.48e-5 plus float32 rounding of the polynomial's evaluation


def _run(x_np):
    lib = ctypes.CDLL(exp2_build.build())
    x = torch.from_numpy(x_np.astype(np.float32)).cuda()
    outs = [torch.empty_like(x) for _ in range(3)]
    rc = lib.exp2_check(ctypes.c_void_p(x.data_ptr()), ctypes.c_int(x.numel()), *(ctypes.c_void_p(o.data_ptr())
                        for o in outs), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    return [o.cpu().numpy().astype(np.float64) for o in outs]


def test_exp2_poly_relative_error_over_softmax_range(cuda):
    grid = np.arange(-125.5, 8.0, 2.0 ** -12)
    rnd = np.random.default_rng(0).uniform(-125.5, 8.0, 1 << 20)
    x = np.concatenate([grid, rnd]).astype(np.float32)
    poly, poly2, ref = _run(x)
    exact = np.exp2(x.astype(np.float64))
    err1 = np.abs(poly / exact - 1).max()
    err2 = np.abs(poly2 / exact - 1).max()
    err_cuda = np.abs(ref / exact - 1).max()
    print(f"max relative error: exp2_poly {err1:.3e}, exp2_poly2 {err2:.3e}, CUDA exp2f {err_cuda:.3e}")
    assert err1 <= BOUND and err2 <= BOUND
    # the two forms implement the same arithmetic (the pair form with packed f32x2 instructions)
    assert np.array_equal(poly, poly2)


def test_exp2_poly_integers_bottom_and_clamp(cuda):
    """Integer inputs hit f = 0 (p(0) = 0.99993): the exponent-field add gives p(0) * 2^n exactly down to -125.
    Over [-127, -125.5] (the bottom of the range and clamped inputs) the absolute error stays below 2^-138, and
    every input below -126 gives the value at -126 (never 0, inf or a wrapped exponent)."""
    n = np.arange(-125, 9, dtype=np.float32)
    bottom = np.linspace(-127.0, -125.5, 4097, dtype=np.float32)
    clamped = np.array([-126.4, -127.0, -200.0, -1e30, -126.0], dtype=np.float32)
    poly, poly2, _ = _run(np.concatenate([n, bottom, clamped]))
    p0 = np.float32(0.9999280572)
    k = len(n)
    assert np.array_equal(poly[:k], (p0 * np.exp2(n.astype(np.float64))).astype(np.float32).astype(np.float64))
    assert np.array_equal(poly2[:k], poly[:k])
    exact = np.exp2(np.maximum(bottom.astype(np.float64), -126.0))
    assert np.abs(poly2[k:k + len(bottom)] - exact).max() < 2.0 ** -138
    c = poly2[k + len(bottom):]
    assert np.all(c == c[-1]) and abs(c[-1] / 2.0 ** -126 - 1) < 1.5e-4, c
