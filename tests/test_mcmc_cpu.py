"""The MCMC refine oracle (Trainer.cpp:1195-1435) on the CPU.

Pins: the restated mt19937_64 against the C++ standard's known answer and against the reference
toolchain's std::mt19937_64; the restated refine against the reference's own Trainer::mcmc_refine
(compiled from the reference tree into oracle/_ref) on random clouds, bit for bit; and the
reference's McmcStrategyTests scenarios (relocation index flow, Adam surgery convention, growth
trajectory and schedule) restated on the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from oracle import McmcOracle

from helpers import mcmc_cloud as _cloud, mcmc_random_cloud as _random_cloud


def _needs_ref():
    if not oracle.ref_available():
        pytest.skip("oracle/_ref (the reference's own CPU code) not built here")


def _sigmoid(x):
    x = np.float32(x)
    return np.float32(1) / (np.float32(1) + np.exp(-x))


def test_mt64_known_answer():
    """[rand.predef]: the 10000th output of a default-constructed (seed 5489) mt19937_64."""
    g = McmcOracle(5489)
    for _ in range(9999):
        g.next()
    assert g.next() == 9981545732273789042


def test_mt64_matches_reference_toolchain():
    _needs_ref()
    for seed in (0, 42, 20260711, 2**64 - 1):
        g = McmcOracle(seed)
        mine = np.array([g.next() for _ in range(1000)], np.uint64)
        assert np.array_equal(mine, oracle.ref_mt64_outputs(seed, 1000)), seed


def test_multinomial_never_picks_zero_weight_and_follows_weights():
    g = McmcOracle(7)
    w = np.array([0.0, 1.0, 0.0, 3.0, 0.0], np.float32)
    s = g.multinomial(w, 20000)
    assert set(np.unique(s)) <= {1, 3}
    frac = float((s == 3).mean())
    assert abs(frac - 0.75) < 0.02
    with pytest.raises(ValueError):
        g.multinomial(np.array([1.0, np.nan], np.float32), 3)
    with pytest.raises(ValueError):
        g.multinomial(np.zeros(4, np.float32), 3)


@pytest.mark.parametrize("n,cap,sh,refines", [(600, 1000, 3, 4), (2000, 2050, 1, 3), (300, 300, 0, 2)])
def test_refine_matches_reference_trainer_bitwise(n, cap, sh, refines):
    """The restated refine == the reference's Trainer::mcmc_refine on its CPU backend: the same
    index lists, counts, parameters and moments, bit for bit, over several refines."""
    _needs_ref()
    rng = np.random.default_rng(100 + n)
    P, M, V = _random_cloud(rng, n, cap, sh)
    Pr, Mr, Vr = [x.copy() for x in P], [x.copy() for x in M], [x.copy() for x in V]
    ref = oracle.ref_trainer_mcmc_refine(Pr, Mr, Vr, sh, n, cap, 0.005, 1234, refines)
    g = McmcOracle(1234)
    count, dead, src, added = n, [], [], []
    for r in range(refines):
        out = g.refine(P, M, V, count, cap)
        count = out["count"]
        assert count == ref["stats"][r, 0]
        assert len(out["relocated_dead"]) == ref["stats"][r, 1]
        assert len(out["added_src"]) == ref["stats"][r, 2]
        dead.append(out["relocated_dead"])
        src.append(out["relocation_src"])
        added.append(out["added_src"])
    assert np.array_equal(np.concatenate(dead), ref["relocated_dead"])
    assert np.array_equal(np.concatenate(src), ref["relocation_src"])
    assert np.array_equal(np.concatenate(added), ref["added_src"])
    assert ref["stats"][0, 1] > 0 and ref["stats"][:, 2].sum() > 0 or cap == n  # non-vacuous
    for g_ in range(6):
        assert np.array_equal(P[g_].view(np.uint32), Pr[g_].view(np.uint32)), ("params", g_)
        assert np.array_equal(M[g_].view(np.uint32), Mr[g_].view(np.uint32)), ("exp_avg", g_)
        assert np.array_equal(V[g_].view(np.uint32), Vr[g_].view(np.uint32)), ("exp_avg_sq", g_)


def test_relocates_dead_to_eq9_scenario():
    """McmcStrategyTests (a): one alive (0.9), three dead -> every dead row copies source 0, whose
    opacity becomes 1 - (1 - 0.9)^(1/4)."""
    P = _cloud([0.9, 0.004, 0.002, 0.0049], 4)
    before = [x.copy() for x in P]
    M = [np.zeros_like(x) for x in P]
    V = [np.zeros_like(x) for x in P]
    out = McmcOracle(42).refine(P, M, V, 4, 4)
    assert out["relocated_dead"].tolist() == [1, 2, 3]
    assert out["relocation_src"].tolist() == [0, 0, 0]
    assert out["added_src"].size == 0 and out["count"] == 4
    o0 = float(_sigmoid(before[3][0, 0]))
    expect = 1.0 - (1.0 - o0) ** 0.25
    for i in range(4):
        assert abs(float(_sigmoid(P[3][i, 0])) - expect) <= 1e-5 * expect + 1e-6
    for i in range(1, 4):
        for g in range(6):
            assert np.array_equal(P[g][i].view(np.uint32), P[g][0].view(np.uint32))
    for g in (0, 1, 4, 5):  # the source keeps everything but opacity and scale
        assert np.array_equal(P[g][0], before[g][0])


def test_adam_surgery_follows_gsplat_scenarios():
    """McmcStrategyTests (b): relocate zeroes the SOURCE rows' moments and keeps the dead rows';
    add zeroes the NEW rows' moments and keeps the sources'."""
    P = _cloud([0.9, 0.004, 0.002, 0.0049], 4)
    M = [np.full_like(x, 7.0) for x in P]
    V = [np.full_like(x, 3.0) for x in P]
    out = McmcOracle().refine(P, M, V, 4, 4)
    assert out["relocation_src"].tolist() == [0, 0, 0]
    for g in range(6):
        assert (M[g][0] == 0).all() and (V[g][0] == 0).all()
        assert (M[g][1:4] == 7).all() and (V[g][1:4] == 3).all()

    P = _cloud([0.7, 0.3], 3)
    snap = [x.copy() for x in P]
    M = [np.full_like(x, 7.0) for x in P]
    V = [np.full_like(x, 3.0) for x in P]
    out = McmcOracle().refine(P, M, V, 2, 3)
    assert out["relocated_dead"].size == 0 and out["count"] == 3 and out["added_src"].size == 1
    s = int(out["added_src"][0])
    o_s = float(_sigmoid(snap[3][s, 0]))
    assert abs(float(_sigmoid(P[3][s, 0])) - (1 - (1 - o_s) ** 0.5)) <= 1e-5
    assert np.array_equal(P[3][2], P[3][s]) and np.array_equal(P[2][2], P[2][s])
    for g in (0, 1, 4, 5):
        assert np.array_equal(P[g][2], snap[g][s])
    other = 1 - s
    assert np.array_equal(P[3][other], snap[3][other]) and np.array_equal(P[2][other], snap[2][other])
    for g in range(6):
        assert (M[g][:2] == 7).all() and (V[g][:2] == 3).all()
        assert (M[g][2] == 0).all() and (V[g][2] == 0).all()


def test_growth_trajectory_is_capped():
    """McmcStrategyTests (c): ceil(21 N / 20) growth, 16 -> ... -> 24 (cap)."""
    P = _cloud([0.5] * 16, 24)
    M = [np.zeros_like(x) for x in P]
    V = [np.zeros_like(x) for x in P]
    g = McmcOracle()
    count = 16
    for want in (17, 18, 19, 20, 21, 23, 24, 24, 24):
        out = g.refine(P, M, V, count, 24)
        assert out["count"] == want and len(out["added_src"]) == want - count
        count = want


def test_refine_schedule_matches_reference():
    """mcmc_refine_due (Trainer.cpp:1262-1270) at total 3000: start 50, stop 2500, every 10."""
    from splatx_cuda.mcmc import McmcOptions, refine_due
    m = McmcOptions(enabled=True)
    for it, want in ((0, False), (50, False), (55, False), (60, True), (2490, True), (2500, False),
                     (2510, False)):
        assert refine_due(m, it, 3000) == want, it
    assert not refine_due(McmcOptions(enabled=False), 60, 3000)
    # 7000 iterations, every 100/7000
    m = McmcOptions(enabled=True, refine_every_ratio=100.0 / 7000.0)
    assert refine_due(m, 200, 7000) and not refine_due(m, 150, 7000)


def test_rng_state_text_layout():
    """The state text is 312 words plus the position, as libstdc++ writes the engine."""
    g = McmcOracle(42)
    t = g.state_text().split()
    assert len(t) == 313 and t[-1] == "312" and t[0] == "42"
