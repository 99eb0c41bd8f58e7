"""View-parallel training on the GPU: the executor's accumulate + apply path.

One view accumulated and applied over all rows must equal the fused resident step (same
gradients, same Adam, regularisers added once); two accumulated views must hold the sum of the
two single-view gradient sets."""
from __future__ import annotations

import numpy as np
import pytest

from helpers import assert_step_close, assert_trajectory_close

pytestmark = pytest.mark.gpu

LR = [1.6e-4, 1e-3, 5e-3, 5e-2, 2.5e-3, 2.5e-3 / 20]


def _setup(n=4096, sh=3, seed=31):
    import torch
    from splatx_cuda.scene import small_scene
    scene, cam = small_scene(seed=seed, n=n, sh_degree=sh)
    P = [np.ascontiguousarray(g.reshape(n, -1)).copy() for g in scene.groups()]
    gts = [torch.from_numpy(np.random.default_rng(seed + k).uniform(0, 1, cam.width * cam.height * 3)
                            .astype(np.float32)).cuda() for k in range(2)]
    return scene, cam, P, gts


def _download(ex, P, n):
    G = [np.zeros_like(x) for x in P]
    ex.download_params(G, [np.zeros_like(x) for x in P], [np.zeros_like(x) for x in P], n)
    return G


def test_accumulate_apply_one_view_equals_fused_step():
    from splatx_cuda.executor import TrainStepExecutor
    scene, cam, P, gts = _setup()
    n, sh = scene.count, scene.sh_degree
    Z = [np.zeros_like(x) for x in P]
    kw = dict(opacity_reg_w=0.01 / n, scale_reg_w=0.01 / (n * 3))
    fused = TrainStepExecutor(n, sh)
    fused.upload_params(P, Z, Z, n)
    fused.step_async(cam.viewmat, cam.K, cam.width, cam.height, gts[0].data_ptr(), n,
                     degrees_to_use=sh, lr=LR, **kw)
    fused.last_result()
    acc = TrainStepExecutor(n, sh)
    acc.upload_params(P, Z, Z, n)
    acc.step_accumulate(cam.viewmat, cam.K, cam.width, cam.height, gts[0].data_ptr(), n, sh)
    padded = acc.resident_buffers()["padded_rows"]
    acc.apply_grads(0, padded, n, 1, LR, **kw)
    acc.last_result()
    a, b = _download(fused, P, n), _download(acc, P, n)
    for g in range(6):
        assert_step_close(b[g], a[g], ("params", g))
    fused.close()
    acc.close()


def test_two_views_accumulate_to_their_sum():
    """The gradient buffers after two accumulated views equal the sum of each view's buffer
    alone (what apply_grads divides by n_views)."""
    import torch
    from splatx_cuda.executor import TrainStepExecutor
    from splatx_cuda.scene import Camera
    scene, cam, P, gts = _setup(seed=33)
    n, sh = scene.count, scene.sh_degree
    vm2 = cam.viewmat.copy()
    vm2[3] += 0.3  # the same camera shifted sideways: an overlapping second view
    cams = [cam, Camera(vm2, cam.K, cam.width, cam.height)]
    Z = [np.zeros_like(x) for x in P]
    ex = TrainStepExecutor(n, sh)
    ex.upload_params(P, Z, Z, n)
    bufs = ex.resident_buffers()
    from splatx_cuda.parallel import device_tensor
    grads = []
    for k, c in enumerate(cams):  # each view's gradient alone
        ex.clear_grads()
        ex.step_accumulate(c.viewmat, c.K, c.width, c.height, gts[k].data_ptr(), n, sh)
        ex.last_result()
        grads.append([device_tensor(bufs["grads"][g], bufs["padded_rows"] * d, 0).clone()
                      for g, d in enumerate(bufs["dims"]) if d])
    ex.clear_grads()
    for k, c in enumerate(cams):  # both together
        ex.step_accumulate(c.viewmat, c.K, c.width, c.height, gts[k].data_ptr(), n, sh)
    ex.last_result()
    both = [device_tensor(bufs["grads"][g], bufs["padded_rows"] * d, 0).clone()
            for g, d in enumerate(bufs["dims"]) if d]
    for g in range(len(both)):
        s = grads[0][g] + grads[1][g]
        scale = float(s.abs().max()) + 1e-30
        assert float((both[g] - s).abs().max()) <= 1e-4 * scale, g
    ex.close()
    torch.cuda.synchronize()


def test_exchange_apply_single_rank_equals_apply_grads():
    """The fused peer-exchange kernel with one rank (no peers) is apply_grads bit for bit, on the
    same accumulated gradients (the raster backward's float atomics make two accumulations differ
    in the last bits, so both updates start from one snapshot)."""
    import torch
    from splatx_cuda.executor import TrainStepExecutor
    from splatx_cuda.parallel import device_tensor
    scene, cam, P, gts = _setup(seed=35)
    n, sh = scene.count, scene.sh_degree
    rng = np.random.default_rng(5)
    M = [rng.normal(0, 1e-3, x.shape).astype(np.float32) for x in P]
    V = [rng.uniform(0, 1e-6, x.shape).astype(np.float32) for x in P]
    kw = dict(opacity_reg_w=0.01 / n, scale_reg_w=0.01 / (n * 3), inject_noise=True,
              noise_seed=42, noise_offset=3, noise_scale=0.05)
    ex = TrainStepExecutor(n, sh)
    ex.upload_params(P, M, V, n)
    bufs = ex.resident_buffers()
    padded = bufs["padded_rows"]
    for k in range(2):
        ex.step_accumulate(cam.viewmat, cam.K, cam.width, cam.height, gts[k].data_ptr(), n, sh)
    ex.last_result()
    views = [device_tensor(bufs["grads"][g], padded * d, 0) for g, d in enumerate(bufs["dims"]) if d]
    views.append(device_tensor(bufs["visibility"], padded, 0))
    snap = [t.clone() for t in views]
    ex.apply_grads(0, padded, n, 2, LR, **kw)
    ex.last_result()
    Pa, Ma, Va = _download_all(ex, P, n)
    ex.upload_params(P, M, V, n)
    for t, s_ in zip(views, snap):
        t.copy_(s_)
    torch.cuda.synchronize()
    ex.open_peers(0, 1, [ex.peer_handles()])
    ex.exchange_apply(0, padded, n, 2, LR, **kw)
    ex.clear_grads()
    ex.last_result()
    Pb, Mb, Vb = _download_all(ex, P, n)
    for g in range(6):
        for a, b, what in ((Pa, Pb, "params"), (Ma, Mb, "exp_avg"), (Va, Vb, "exp_avg_sq")):
            assert np.array_equal(a[g].view(np.uint32), b[g].view(np.uint32)), (what, g)
    assert all(float(t.abs().max()) == 0.0 for t in views)  # accumulators cleared
    ex.close()


def _download_all(ex, like, n):
    P = [np.zeros_like(x) for x in like]
    M = [np.zeros_like(x) for x in like]
    V = [np.zeros_like(x) for x in like]
    ex.download_params(P, M, V, n)
    return P, M, V


def test_open_peers_rejects_bad_layouts():
    from splatx_cuda.executor import TrainStepExecutor
    a, b = TrainStepExecutor(4096, 1), TrainStepExecutor(8192, 1)
    with pytest.raises(Exception):
        a.open_peers(0, 2, [a.peer_handles(), b.peer_handles()])  # different arenas
    with pytest.raises(Exception):
        a.open_peers(0, 9, [a.peer_handles()] * 9)  # more than 8 ranks
    with pytest.raises(Exception):
        a.exchange_apply(0, 32, 10, 1, LR)  # peers never opened
    a.close()
    b.close()


@pytest.mark.parametrize("chunks", [1, 3, 4])
def test_step_exchange_single_rank_equals_accumulate_then_exchange(chunks):
    """The overlapped step (chunked backward, device barriers, exchange per chunk on a second
    stream) with one rank equals step_accumulate + exchange_apply + clear_grads over two steps,
    within the trajectory tolerance (the raster backward's float atomics differ between two runs
    in the last bits); the barrier epochs advance. The accumulators keep the last step's sums,
    and the next accumulating view writes them (zeros where it sees nothing) instead of adding:
    what a freshly cleared executor with the same parameters accumulates."""
    from splatx_cuda.executor import TrainStepExecutor
    from splatx_cuda.parallel import device_tensor
    scene, cam, P, gts = _setup(seed=37)
    n, sh = scene.count, scene.sh_degree
    rng = np.random.default_rng(6)
    M = [rng.normal(0, 1e-3, x.shape).astype(np.float32) for x in P]
    V = [rng.uniform(0, 1e-6, x.shape).astype(np.float32) for x in P]
    kw = dict(opacity_reg_w=0.01 / n, scale_reg_w=0.01 / (n * 3), inject_noise=True,
              noise_seed=42, noise_offset=3, noise_scale=0.05)
    a, b = TrainStepExecutor(n, sh), TrainStepExecutor(n, sh)
    for ex in (a, b):
        ex.upload_params(P, M, V, n)
        ex.open_peers(0, 1, [ex.peer_handles()])
    padded = a.resident_buffers()["padded_rows"]
    for k in range(2):
        a.step_accumulate(cam.viewmat, cam.K, cam.width, cam.height, gts[k].data_ptr(), n, sh)
        a.exchange_apply(0, padded, n, 1, LR, **kw)
        a.clear_grads()
        b.step_exchange(cam.viewmat, cam.K, cam.width, cam.height, gts[k].data_ptr(), n, sh,
                        0, padded, 1, LR, chunks=chunks, **kw)
    a.last_result()
    b.last_result()
    Pa, Ma, Va = _download_all(a, P, n)
    Pb, Mb, Vb = _download_all(b, P, n)
    for g in range(6):
        assert_trajectory_close(Pb[g], Pa[g], ("params", g), v_ref=Va[g], lr=LR[g], steps=2)
        assert_trajectory_close(Mb[g], Ma[g], ("exp_avg", g))
        assert_trajectory_close(Vb[g], Va[g], ("exp_avg_sq", g))
    # a view after the exchange: written, not added — the same as a cleared executor's view
    view = (cam.viewmat, cam.K, cam.width, cam.height, gts[0].data_ptr(), n, sh)
    b.step_accumulate(*view)
    c = TrainStepExecutor(n, sh)
    c.upload_params(Pb, Mb, Vb, n)
    c.step_accumulate(*view)
    b.last_result()
    c.last_result()

    def acc_of(ex):
        bufs = ex.resident_buffers()
        t = [device_tensor(bufs["grads"][g], padded * d, 0).cpu().numpy()
             for g, d in enumerate(bufs["dims"]) if d]
        return t, device_tensor(bufs["visibility"], padded, 0).cpu().numpy()

    (gb, vb), (gc, vc) = acc_of(b), acc_of(c)
    assert np.array_equal(vb[:n], vc[:n]) and 0 < vb[:n].sum() < n
    for x, y in zip(gb, gc):
        assert_step_close(x, y, "accumulated gradients after an exchange")
    c.close()
    # per step: one barrier per chunk (fewer chunks than tiles here) and the closing one
    import ctypes
    from splatx_cuda import _native
    h = _native.SxPeerHandles()
    ctypes.memmove(ctypes.byref(h), b.peer_handles(), ctypes.sizeof(h))
    assert h.barrier_epoch == 2 * (chunks + 1)
    a.close()
    b.close()


def test_step_exchange_rejections():
    from splatx_cuda.executor import TrainStepExecutor
    scene, cam, P, gts = _setup(n=2048, sh=1, seed=39)
    n, sh = scene.count, scene.sh_degree
    Z = [np.zeros_like(x) for x in P]
    a, b = TrainStepExecutor(n, sh), TrainStepExecutor(n, sh)
    a.upload_params(P, Z, Z, n)
    padded = a.resident_buffers()["padded_rows"]
    args = (cam.viewmat, cam.K, cam.width, cam.height, gts[0].data_ptr(), n, sh)
    with pytest.raises(Exception, match="open_peers"):
        a.step_exchange(*args, 0, padded, 1, LR)
    a.open_peers(0, 1, [a.peer_handles()])
    for bad in (0, 9):
        with pytest.raises(Exception, match="chunks"):
            a.step_exchange(*args, 0, padded, 1, LR, chunks=bad)
    with pytest.raises(Exception, match="owner rows"):
        a.step_exchange(*args, 32, padded, 1, LR)
    a.set_profiling(True)  # the profiled overlapped step reports its timeline
    a.step_exchange(*args, 0, padded, 1, LR, chunks=2)
    a.set_profiling(False)
    tl = dict(a.exchange_timeline())
    assert tl["start"] == 0.0
    assert 0 < tl["raster_bwd_end"] <= tl["bwd_chunk0_end"] <= tl["bwd_chunk1_end"]
    assert tl["bwd_chunk0_end"] <= tl["barrier0_end"] <= tl["exchange0_end"] <= tl["exchange1_end"]
    assert tl["exchange1_end"] <= tl["closing_barrier_end"] <= tl["clear_end"]
    a.segment_times()
    a.last_result()
    # a's executor has taken barriers, b's none: their epochs disagree
    with pytest.raises(Exception, match="peer barriers"):
        a.open_peers(0, 2, [a.peer_handles(), b.peer_handles()])
    a.close()
    b.close()


def test_device_barrier_wait_is_bounded():
    """A peer that never signals (a flag array nothing writes): the device barrier's bounded wait
    runs out after about a second, reports the "peer barrier" status bit, and the context stays
    usable; with one rank the barrier passes at once."""
    import time
    import torch
    from splatx_cuda.parallel import peer_barrier_selftest
    assert peer_barrier_selftest(0, 1) == 0
    t0 = time.time()
    assert peer_barrier_selftest(0, 2) == 2
    assert time.time() - t0 < 60
    x = torch.ones(4, device="cuda")
    assert float(x.sum()) == 4.0


def test_exchange_after_a_timed_out_barrier_changes_nothing():
    """What an overlapped step enqueues after a device barrier — the owner-row exchange — runs
    only when the barrier completed: after a wait that ran out the parameters and moments stay as
    they were (a late peer's gradients may be missing from the sum)."""
    import torch
    from splatx_cuda.parallel import peer_exchange_selftest
    assert peer_exchange_selftest(0, 1) == (0, True)
    assert peer_exchange_selftest(0, 2) == (2, False)
    x = torch.ones(4, device="cuda")
    assert float(x.sum()) == 4.0
