"""The device-resident MCMC refine (sxcuda_executor_mcmc_refine) against the refine oracle, which
is pinned bit for bit to the reference's own Trainer::mcmc_refine.

Bars: the index lists (dead rows, relocation sources, add sources) and counts exact; moments exact
(zeroed rows, untouched rows); parameters within 1e-5 relative (the relocation kernel's float
pow on the device against the host's); copied rows bit-identical to their sources.
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import assert_trajectory_close, mcmc_cloud, mcmc_random_cloud

pytestmark = pytest.mark.gpu


def _executor(cap, sh):
    from splatx_cuda.executor import TrainStepExecutor
    return TrainStepExecutor(cap, sh)


def _upload(ex, P, M, V, rows):
    ex.upload_params([np.ascontiguousarray(x) for x in P], [np.ascontiguousarray(x) for x in M],
                     [np.ascontiguousarray(x) for x in V], rows)


def _download(ex, like, rows):
    P = [np.zeros_like(x) for x in like]
    M = [np.zeros_like(x) for x in like]
    V = [np.zeros_like(x) for x in like]
    ex.download_params(P, M, V, rows)
    return P, M, V


def _close(a, b, what):
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    bad = ~(np.abs(a64 - b64) <= 1e-6 + 1e-5 * np.abs(b64))
    assert not bad.any(), f"{what}: {int(bad.sum())} elements off, e.g. {a64[bad][:4]} vs {b64[bad][:4]}"


@pytest.mark.parametrize("n,cap,sh,refines", [(5000, 6000, 3, 3), (20000, 20500, 1, 2), (777, 777, 0, 2)])
def test_refine_matches_oracle(n, cap, sh, refines):
    from oracle import McmcOracle
    rng = np.random.default_rng(7 + n)
    P, M, V = mcmc_random_cloud(rng, n, cap, sh)
    ex = _executor(cap, sh)
    _upload(ex, P, M, V, cap)
    ex.mcmc_seed(99)
    g = McmcOracle(99)
    count = n
    for _ in range(refines):
        want = g.refine(P, M, V, count, cap)
        got = ex.mcmc_refine(count, cap)
        assert got["count"] == want["count"]
        for k in ("relocated_dead", "relocation_src", "added_src"):
            assert np.array_equal(got[k], want[k]), k
        count = got["count"]
    assert ex.mcmc_rng_state() == g.state_text()
    Pd, Md, Vd = _download(ex, P, cap)
    for k in range(6):
        if P[k].size == 0:
            continue
        _close(Pd[k], P[k], ("params", k))
        assert np.array_equal(Md[k], M[k]), ("exp_avg", k)
        assert np.array_equal(Vd[k], V[k]), ("exp_avg_sq", k)
    ex.close()


def test_copied_rows_are_bitwise_copies_and_sources_relocated():
    """McmcStrategyTests (a) on the device: one alive row, three dead."""
    P = mcmc_cloud([0.9, 0.004, 0.002, 0.0049], 4)
    before = [x.copy() for x in P]
    Z = [np.zeros_like(x) for x in P]
    ex = _executor(4, 1)
    _upload(ex, P, Z, Z, 4)
    out = ex.mcmc_refine(4, 4)
    assert out["relocated_dead"].tolist() == [1, 2, 3]
    assert out["relocation_src"].tolist() == [0, 0, 0]
    assert out["count"] == 4 and out["added_src"].size == 0
    Pd, _, _ = _download(ex, P, 4)
    o0 = 1.0 / (1.0 + np.exp(-np.float64(before[3][0, 0])))
    expect = 1.0 - (1.0 - o0) ** 0.25
    for i in range(4):
        assert abs(1.0 / (1.0 + np.exp(-np.float64(Pd[3][i, 0]))) - expect) <= 1e-5 * expect + 1e-6
    for i in range(1, 4):
        for g in range(6):
            assert np.array_equal(Pd[g][i].view(np.uint32), Pd[g][0].view(np.uint32)), (i, g)
    for g in (0, 1, 4, 5):
        assert np.array_equal(Pd[g][0], before[g][0])
    ex.close()


def test_adam_surgery_convention_on_device():
    """McmcStrategyTests (b): relocate zeroes the sources' moments, add zeroes the new rows'."""
    P = mcmc_cloud([0.9, 0.004, 0.002, 0.0049], 4)
    M = [np.full_like(x, 7.0) for x in P]
    V = [np.full_like(x, 3.0) for x in P]
    ex = _executor(4, 1)
    _upload(ex, P, M, V, 4)
    ex.mcmc_refine(4, 4)
    _, Md, Vd = _download(ex, P, 4)
    for g in range(6):
        assert (Md[g][0] == 0).all() and (Vd[g][0] == 0).all()
        assert (Md[g][1:4] == 7).all() and (Vd[g][1:4] == 3).all()
    ex.close()

    P = mcmc_cloud([0.7, 0.3], 3)
    M = [np.full_like(x, 7.0) for x in P]
    V = [np.full_like(x, 3.0) for x in P]
    ex = _executor(3, 1)
    _upload(ex, P, M, V, 3)  # the tail row's moments are dirty on purpose
    out = ex.mcmc_refine(2, 3)
    assert out["count"] == 3 and out["added_src"].size == 1 and out["relocated_dead"].size == 0
    s = int(out["added_src"][0])
    Pd, Md, Vd = _download(ex, P, 3)
    for g in range(6):
        assert np.array_equal(Pd[g][2].view(np.uint32), Pd[g][s].view(np.uint32))
        assert (Md[g][:2] == 7).all() and (Vd[g][:2] == 3).all()
        assert (Md[g][2] == 0).all() and (Vd[g][2] == 0).all()
    ex.close()


def test_growth_trajectory_and_errors():
    P = mcmc_cloud([0.5] * 16, 24)
    Z = [np.zeros_like(x) for x in P]
    ex = _executor(24, 1)
    _upload(ex, P, Z, Z, 24)
    count = 16
    for want in (17, 18, 19, 20, 21, 23, 24, 24, 24):
        out = ex.mcmc_refine(count, 24)
        assert out["count"] == want and out["n_added"] == want - count
        count = want
    with pytest.raises(Exception):
        ex.mcmc_refine(24, 25)  # cap_max beyond the arena
    with pytest.raises(Exception):
        ex.mcmc_refine(24, 20)  # cap_max below count
    with pytest.raises(Exception):
        ex.mcmc_refine(24, 24, min_opacity=1.5)
    ex.close()


def test_rng_state_round_trip():
    """A restored engine state continues the same draws (checkpoint/resume of the refine)."""
    rng = np.random.default_rng(3)
    P, M, V = mcmc_random_cloud(rng, 3000, 4000, 1)
    a, b = _executor(4000, 1), _executor(4000, 1)
    for ex in (a, b):
        _upload(ex, P, M, V, 4000)
    a.mcmc_seed(5)
    a.mcmc_refine(3000, 4000)
    b.set_mcmc_rng_state(a.mcmc_rng_state())
    b_out = b.mcmc_refine(3000, 4000)
    a2 = _executor(4000, 1)
    _upload(a2, P, M, V, 4000)
    a2.set_mcmc_rng_state(a.mcmc_rng_state())
    a2_out = a2.mcmc_refine(3000, 4000)
    for k in ("relocated_dead", "relocation_src", "added_src"):
        assert np.array_equal(a2_out[k], b_out[k])
    with pytest.raises(Exception):
        b.set_mcmc_rng_state("not a state")
    for ex in (a, b, a2):
        ex.close()


def test_inject_noise_matches_oracle_perturb():
    import oracle
    rng = np.random.default_rng(11)
    n = 10000
    P, M, V = mcmc_random_cloud(rng, n, n, 1)
    ex = _executor(n, 1)
    _upload(ex, P, M, V, n)
    ex.inject_noise(n, seed=42, offset=17, noise_scale=0.08)
    Pd, _, _ = _download(ex, P, n)
    ob = oracle.OracleBackend()
    noise = ob.rng_normal_f32(42, 17, n * 3)
    pos = P[0].copy()
    ob.mcmc_perturb_positions(pos, P[1], P[2], P[3], noise, 0.08)
    moved = np.abs(pos - P[0]).max()
    assert moved > 0
    assert np.abs(Pd[0].astype(np.float64) - pos).max() <= 1e-5 * max(1.0, np.abs(pos).max())
    for g in range(1, 6):
        assert np.array_equal(Pd[g], P[g])
    ex.close()


def test_training_with_refine_follows_host_path():
    """Steps, a refine, then steps on the grown count: the executor against the oracle's host
    round trip (host_step + the refine oracle), as the reference trainer orders them."""
    import torch
    import oracle
    from oracle import McmcOracle
    from splatx_cuda.scene import small_scene
    n, cap, sh = 4096, 4400, 1
    scene, cam = small_scene(seed=23, n=n, sh_degree=sh)
    dims = [3, 4, 3, 1, 3, 9]
    P = [np.zeros((cap, d), np.float32) for d in dims]
    for g, x in enumerate(scene.groups()):
        P[g][:n] = np.asarray(x, np.float32).reshape(n, -1)
    P[3][:n:9, 0] = -7.0  # some dead rows
    M = [np.zeros_like(x) for x in P]
    V = [np.zeros_like(x) for x in P]
    gt = np.random.default_rng(1).uniform(0, 1, cam.width * cam.height * 3).astype(np.float32)
    lr = [1.6e-4, 1e-3, 5e-3, 5e-2, 2.5e-3, 2.5e-3 / 20]
    ex = _executor(cap, sh)
    _upload(ex, P, M, V, cap)
    gt_dev = torch.from_numpy(gt).cuda()
    g = McmcOracle(42)
    count = n
    for it in range(6):
        ex.step_async(cam.viewmat, cam.K, cam.width, cam.height, gt_dev.data_ptr(), count,
                      degrees_to_use=sh, lr=lr)
        ex.last_result()
        oracle.host_step([x[:count] for x in P], cam, gt, sh, degrees_to_use=sh, lr=lr,
                         exp_avg=[x[:count] for x in M], exp_avg_sq=[x[:count] for x in V])
        if it == 2:
            want = g.refine(P, M, V, count, cap)
            got = ex.mcmc_refine(count, cap)
            assert got["count"] == want["count"] > count
            assert np.array_equal(got["relocated_dead"], want["relocated_dead"])
            count = got["count"]
    Pd, _, _ = _download(ex, P, cap)
    for k in range(6):
        assert_trajectory_close(Pd[k][:count], P[k][:count], ("params", k), v_ref=V[k][:count],
                                lr=lr[k], steps=6)
    ex.close()
