"""SXCK checkpoints of the resident arena against the reference's own save/load
(Checkpoint.cpp compiled into oracle/_ref): files written from the device read back exactly in
the reference, the reference's files load exactly into the device arena, fp16 files are
byte-identical to the reference's (device half conversion, sqrt compression, clamp), and the
fingerprint and shape checks reject mismatches."""
from __future__ import annotations

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

CFG = {"sh_degree": 2, "factor": 0, "test_split": 0, "total_iters": 7000, "mcmc_enabled": 1,
       "antialiased": 0, "cap_max": 900, "mcmc_seed": 42, "scene_scale": 9.5, "ssim_weight": 0.2}


def _needs_ref():
    if not oracle.ref_available():
        pytest.skip("oracle/_ref (the reference's own CPU code) not available")


def _arrays(n, deg=2, seed=0, extreme=False):
    rng = np.random.default_rng(seed)
    dims = [3, 4, 3, 1, 3, ((deg + 1) ** 2 - 1) * 3]
    P = [rng.normal(0, 1, (n, d)).astype(np.float32) for d in dims]
    M = [rng.normal(0, 1e-3, (n, d)).astype(np.float32) for d in dims]
    V = [(10.0 ** rng.uniform(-17, -5, (n, d))).astype(np.float32) for d in dims]
    if extreme:  # beyond half's range, and moments that underflow
        P[0][:4, 0] = [7e4, -9e5, 65504.0, 65520.0]
        V[5][:5] = 1e-20
    return P, M, V


def _executor(cap, deg, P=None, M=None, V=None):
    from splatx_cuda.executor import TrainStepExecutor
    ex = TrainStepExecutor(cap, deg)
    if P is not None:
        n = P[0].shape[0]
        pad = lambda xs: [np.concatenate([x, np.zeros((cap - n, x.shape[1]), np.float32)]) for x in xs]
        ex.upload_params(pad(P), pad(M), pad(V), cap)
    return ex


def _download(ex, cap, deg):
    dims = [3, 4, 3, 1, 3, ((deg + 1) ** 2 - 1) * 3]
    P = [np.zeros((cap, d), np.float32) for d in dims]
    M = [np.zeros_like(x) for x in P]
    V = [np.zeros_like(x) for x in P]
    ex.download_params(P, M, V, cap)
    return P, M, V


def _rng_text():
    from oracle import McmcOracle
    g = McmcOracle(7)
    for _ in range(1000):
        g.next()
    return g.state_text()


def test_device_save_reads_back_in_the_reference(tmp_path):
    _needs_ref()
    n, cap = 700, 900
    P, M, V = _arrays(n, seed=1)
    ex = _executor(cap, 2, P, M, V)
    ex.set_mcmc_rng_state(_rng_text())
    ex.save_checkpoint(CFG, 1234, n, tmp_path / "a.sxck")
    ref = oracle.ref_checkpoint_load(tmp_path / "a.sxck", [x.shape[1] for x in P])
    assert ref["iter"] == 1234 and ref["count"] == n and ref["rng"] == _rng_text()
    assert ref["config"] == pytest.approx(CFG)
    for g in range(6):
        for a, b in ((ref["P"][g], P[g]), (ref["M"][g], M[g]), (ref["V"][g], V[g])):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), g
    ex.close()


def test_reference_file_loads_into_the_arena(tmp_path):
    _needs_ref()
    n, cap = 600, 900
    P, M, V = _arrays(n, seed=2)
    oracle.ref_checkpoint_save(CFG, 77, P, M, V, tmp_path / "r.sxck", rng=_rng_text())
    junk = _arrays(cap, seed=3)
    ex = _executor(cap, 2, *junk)  # a dirty arena: the load zeroes the tail
    h = ex.load_checkpoint(tmp_path / "r.sxck", current=CFG)
    assert h["iter"] == 77 and h["alive_count"] == n and not h["fp16"]
    assert ex.mcmc_rng_state() == _rng_text()
    Pd, Md, Vd = _download(ex, cap, 2)
    for g in range(6):
        for a, b in ((Pd[g], P[g]), (Md[g], M[g]), (Vd[g], V[g])):
            assert np.array_equal(a[:n].view(np.uint32), b.view(np.uint32)), g
            assert not a[n:].any()
    ex.close()


def test_fp16_files_match_the_reference_bytes_and_decoding(tmp_path):
    _needs_ref()
    n, cap = 500, 512
    P, M, V = _arrays(n, seed=4, extreme=True)
    ex = _executor(cap, 2, P, M, V)
    ex.save_checkpoint(CFG, 5, n, tmp_path / "ours16.sxck", fp16=True)
    oracle.ref_checkpoint_save(CFG, 5, P, M, V, tmp_path / "ref16.sxck", fp16=True,
                               rng=ex.mcmc_rng_state())
    assert (tmp_path / "ours16.sxck").read_bytes() == (tmp_path / "ref16.sxck").read_bytes()
    ex2 = _executor(cap, 2)
    h = ex2.load_checkpoint(tmp_path / "ref16.sxck")
    assert h["fp16"]
    ref = oracle.ref_checkpoint_load(tmp_path / "ref16.sxck", [x.shape[1] for x in P])
    Pd, Md, Vd = _download(ex2, cap, 2)
    for g in range(6):
        for a, b in ((Pd[g], ref["P"][g]), (Md[g], ref["M"][g]), (Vd[g], ref["V"][g])):
            assert np.array_equal(a[:n].view(np.uint32), b.view(np.uint32)), g
    assert (Md[5][:5] == 0).all() and (Vd[5][:5] == 0).all()  # paired zeroing
    assert Pd[0][0, 0] == 65504.0 and Pd[0][1, 0] == -65504.0
    for e in (ex, ex2):
        e.close()


def test_load_rejections(tmp_path):
    n, cap = 300, 400
    P, M, V = _arrays(n, seed=5)
    ex = _executor(cap, 2, P, M, V)
    ex.save_checkpoint(CFG, 9, n, tmp_path / "c.sxck")
    with pytest.raises(RuntimeError, match="total_iters"):
        ex.load_checkpoint(tmp_path / "c.sxck", current=dict(CFG, total_iters=30000))
    with pytest.raises(Exception, match="SH degree"):
        _executor(cap, 3).load_checkpoint(tmp_path / "c.sxck")
    with pytest.raises(Exception, match="more rows"):
        _executor(200, 2).load_checkpoint(tmp_path / "c.sxck")
    with pytest.raises(Exception):
        ex.save_checkpoint(dict(CFG, sh_degree=3), 9, n, tmp_path / "d.sxck")
    with pytest.raises(Exception):
        ex.save_checkpoint(CFG, 9, cap + 1, tmp_path / "d.sxck")
    assert not (tmp_path / "d.sxck").exists() and not (tmp_path / "d.sxck.tmp").exists()
    ex.close()


@pytest.mark.parametrize("fp16", [False, True])
def test_failed_load_leaves_the_arena_untouched(tmp_path, fp16):
    """A truncated or padded checkpoint is refused before the arena is written: the executor keeps
    its parameters and both moments (the reference loads into a separate snapshot, so a failed
    load leaves its trainer as it was)."""
    n, cap = 300, 400
    P, M, V = _arrays(n, seed=8)
    ex = _executor(cap, 2, P, M, V)
    good = tmp_path / "c.sxck"
    ex.save_checkpoint(CFG, 9, n, good, fp16=fp16)
    body = good.read_bytes()
    P2, M2, V2 = _arrays(n, seed=9)
    other = _executor(cap, 2, P2, M2, V2)
    before = _download(other, cap, 2)
    for name, data in (("short", body[:-6]), ("half", body[: len(body) // 2]),
                       ("long", body + b"\0" * 8)):
        bad = tmp_path / f"{name}.sxck"
        bad.write_bytes(data)
        with pytest.raises(RuntimeError, match="truncated or corrupt|trailing"):
            other.load_checkpoint(bad)
        after = _download(other, cap, 2)
        for a, b in zip(before, after):
            for x, y in zip(a, b):
                assert np.array_equal(x, y), name
    other.load_checkpoint(good)  # a good file still loads afterwards
    loaded = _download(other, cap, 2)
    want = _download(ex, cap, 2)[0][0][:n]
    if fp16:  # the file holds half values (round to nearest even)
        want = want.astype(np.float16).astype(np.float32)
    assert np.array_equal(loaded[0][0][:n], want)
    ex.close()
    other.close()


def test_resume_continues_training(tmp_path):
    """Save mid-run, load into a fresh executor: the next steps from the loaded arena follow the
    uninterrupted run within the trajectory tolerance (the backward's float atomics)."""
    import torch
    from helpers import assert_trajectory_close
    from splatx_cuda.scene import small_scene
    scene, cam = small_scene(seed=8, n=2048, sh_degree=1)
    n = scene.count
    P = [np.ascontiguousarray(g.reshape(n, -1)).copy() for g in scene.groups()]
    Z = [np.zeros_like(x) for x in P]
    lr = [1.6e-4, 1e-3, 5e-3, 5e-2, 2.5e-3, 2.5e-3 / 20]
    gt = torch.from_numpy(np.random.default_rng(2).uniform(0, 1, cam.width * cam.height * 3)
                          .astype(np.float32)).cuda()
    cfg = dict(CFG, sh_degree=1, cap_max=n)

    def steps(ex, k):
        for _ in range(k):
            ex.step_async(cam.viewmat, cam.K, cam.width, cam.height, gt.data_ptr(), n,
                          degrees_to_use=1, lr=lr)
        ex.last_result()

    a = _executor(n, 1, P, Z, Z)
    steps(a, 3)
    a.save_checkpoint(cfg, 3, n, tmp_path / "mid.sxck")
    steps(a, 2)
    b = _executor(n, 1)
    assert b.load_checkpoint(tmp_path / "mid.sxck", current=cfg)["iter"] == 3
    steps(b, 2)
    Pa, _, Va = _download(a, n, 1)
    Pb, _, _ = _download(b, n, 1)
    for g in range(6):
        assert_trajectory_close(Pb[g], Pa[g], ("params", g), v_ref=Va[g], lr=lr[g], steps=5)
    a.close()
    b.close()
