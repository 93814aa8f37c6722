"""The CPU oracle against the reference's golden data (no GPU).

The oracle (oracle/s2s_oracle.cpp) restates swin2sr-rs src/cpu.rs. It is pinned
here to (a) the published PyTorch network through the SW2F fixtures made by
tests/golden/make_golden.py, and (b) the reference's own bicubic golden vectors
(tests/bicubic.rs:38-58, tol 2e-5).
"""
import math

import numpy as np
import pytest

from s2s_testlib import GOLDEN, TOL, adjust, golden_cases, load_fixture, oracle, pkg


@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: c["name"])
def test_oracle_matches_published_network(case):
    O, P = oracle(), pkg()
    h, w, s, win, x, y, aux = load_fixture(case["name"])
    wt = P.weights.Weights.seeded(case["task"], case["wseed"], case["perturb"])
    out, oaux = O.forward(wt, h, w, adjust(wt, x))
    # An exact transcription lands near 1e-6 (README.md:23 of the reference); the
    # gate is the reference's fixture tolerance.
    assert np.abs(out - y).max() < 2e-5, np.abs(out - y).max()
    assert np.abs(out - y).max() < TOL
    if aux is not None:
        assert oaux is not None and np.abs(oaux - aux).max() < 2e-5


def test_oracle_bicubic_matches_reference_golden_vectors():
    O = oracle()
    x = np.load(GOLDEN / "bicubic_in_40x32.npy")
    want = np.load(GOLDEN / "bicubic_out_148x116.npy")
    assert x.shape == (1, 1, 40, 32) and want.shape == (1, 1, 148, 116)
    got = O.bicubic(x[0], 148, 116)
    assert np.abs(got - want[0]).max() < 2e-5


def test_fast_exp_is_sqrt2_times_exp_on_the_softmax_domain():
    # src/cpu.rs:1095-1120 as written evaluates 2^(t + 0.5) for t = x log2(e) <= 0:
    # a constant sqrt(2) that cancels in the softmax normalisation.
    O = oracle()
    for x in [0.0, -0.3, -1.0, -2.7, -10.0, -50.0]:
        got = O.fast_exp(x)
        want = math.sqrt(2.0) * math.exp(x)
        assert abs(got - want) <= 2e-5 * want, (x, got, want)
    assert O.fast_exp(-95.0) == 0.0


def test_oracle_pad_reflect_matches_plan():
    O, P = oracle(), pkg()
    rng = np.random.default_rng(0)
    x = rng.random((3, 13, 21)).astype(np.float32)
    pl = P.plan.Plan.new(13, 21, 8, 3)
    a = O.pad_reflect(x, pl.hp, pl.wp)
    b = P.plan.pad_reflect(x, 13, 21, pl.hp, pl.wp)
    assert a.shape == (3, 16, 24) and np.array_equal(a, b)
    # whole-plane mirror: the added columns mirror the FIRST columns read backwards
    assert np.array_equal(a[:, :13, 21], x[:, :, 20])


def test_oracle_layer_norm_is_one_pass():
    O = oracle()
    rng = np.random.default_rng(1)
    x = rng.standard_normal((180, 50)).astype(np.float32)
    g = rng.standard_normal(180).astype(np.float32)
    b = rng.standard_normal(180).astype(np.float32)
    y = O.layer_norm(x, g, b)
    m = x.astype(np.float64).mean(0)
    v = x.astype(np.float64).var(0)
    ref = (x - m) / np.sqrt(v + 1e-5) * g[:, None] + b[:, None]
    assert np.abs(y - ref).max() < 1e-4
