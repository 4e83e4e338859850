"""The FMA-pipe exponential of the attention forward (``ex2_fma2`` in
``scope_b200/csrc/tc_ptx.cuh``): Cody-Waite reduction for base 2 plus a
degree-3 minimax polynomial for 2^f on [-1/2, 1/2].

CPU: the constants in the header are the ones the generator fits, and their
float32 evaluation stays inside the stated 7.5e-5 relative error bound.
GPU: the device function itself against exp2 in float64, over the range the
softmax feeds it (scaled scores minus the running max: at most 8, down to
-inf for masked entries).
"""
import importlib.util
import os
import re

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "..", "scope_b200", "csrc")
BOUND = 7.5e-5


def _gen():
    spec = importlib.util.spec_from_file_location("gen_exp2_poly", os.path.join(CSRC, "gen_exp2_poly.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _header_coeffs():
    src = open(os.path.join(CSRC, "tc_ptx.cuh")).read()
    body = src[src.index("ex2_fma2"):]
    return [float(re.search(rf"C{j} = ([0-9.e+-]+)f", body).group(1)) for j in range(4)]


def test_constants_match_generator():
    g = _gen()
    c = g.remez_rel(3).astype(np.float32)
    hc = np.array(_header_coeffs(), dtype=np.float32)
    assert np.array_equal(c, hc), (c, hc)


def test_float32_evaluation_within_bound():
    g = _gen()
    c32 = np.array(_header_coeffs(), dtype=np.float32)
    xs = np.linspace(-125.0, 8.0, 2_000_001).astype(np.float32)
    got = g.eval_f32(c32, xs).astype(np.float64)
    ref = np.exp2(xs.astype(np.float64))
    assert (np.abs(got - ref) / ref).max() < BOUND


@pytest.mark.gpu
def test_device_exp2_fma_against_exp2():
    from scope_b200 import _lib
    torch.manual_seed(0)
    x = torch.cat([torch.linspace(-125.0, 8.0, 1_000_001), torch.rand(1_000_000) * -30.0,
                   torch.tensor([0.0, -0.5, 0.5, 8.0, -125.0, -126.5, -1000.0, float("-inf")])]).float().cuda()
    y = torch.empty_like(x)
    st = _lib.lib().scope_selftest_exp2_fma(x.data_ptr(), y.data_ptr(), x.numel(),
                                            torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "scope_selftest_exp2_fma")
    torch.cuda.synchronize()
    xd, yd = x.double(), y.double()
    inr = xd >= -125.0
    ref = torch.exp2(xd[inr])
    assert ((yd[inr] - ref).abs() / ref).max().item() < BOUND
    # below the clamp (and -inf, a masked score) the result is 2^-125 to the same
    # bound (the polynomial's value at f = 0 times 2^-125), not 0
    assert ((yd[~inr] - 2.0 ** -125).abs() / 2.0 ** -125).max().item() < BOUND
