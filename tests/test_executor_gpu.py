"""Resident executor vs the host round-trip path (both on the GPU kernels).

Mirrors splatx-metal's host-vs-resident contrast gate (Sources/SplatXTests/TrainerTests.cpp:
1720-1750): exact n_isects, per-step loss |d| <= 1e-6 + 1e-4 |L|, first render rel_l2 <= 1e-5 and
parameters rel_l2 <= 1e-4 after five steps.
"""
import numpy as np
import pytest

from helpers import assert_step_close, assert_trajectory_close, rel_l2
from hostpath import HostState, host_step

pytestmark = pytest.mark.gpu

LR = [1.6e-4, 1e-3, 5e-3, 5e-2, 2.5e-3, 2.5e-3 / 20]


def _target(scene, cam, seed=99):
    from splatx_cuda.executor import TrainStepExecutor
    rng = np.random.default_rng(seed)
    hidden = [g.copy() for g in scene.groups()]
    hidden[0] = hidden[0] + rng.normal(0, 0.05, hidden[0].shape).astype(np.float32)
    ex = TrainStepExecutor(scene.count, scene.sh_degree, ssim_weight=0.2)
    z = [np.zeros_like(g) for g in hidden]
    ex.upload_params([np.ascontiguousarray(g.reshape(scene.count, -1)) for g in hidden],
                     [np.ascontiguousarray(a.reshape(scene.count, -1)) for a in z],
                     [np.ascontiguousarray(a.reshape(scene.count, -1)) for a in z], scene.count)
    _, _, img = ex.step(cam.viewmat, cam.K, cam.width, cam.height, None, scene.count,
                        degrees_to_use=scene.sh_degree, forward_only=True, want_render=True)
    ex.close()
    return img


@pytest.mark.parametrize("sh_degree,ssim_weight,aa", [(0, 0.2, False), (1, 0.0, False),
                                                      (3, 0.2, False), (1, 0.2, True)])
def test_resident_matches_host_path(backend, sh_degree, ssim_weight, aa):
    from splatx_cuda.executor import TrainStepExecutor
    from splatx_cuda.scene import small_scene
    scene, cam = small_scene(seed=1, n=3000, sh_degree=sh_degree)
    gt = _target(scene, cam)
    cfg = dict(ssim_weight=ssim_weight, lr=LR, degrees_to_use=sh_degree, antialiased=aa,
               opacity_reg=0.01, scale_reg=0.01)
    host = HostState(scene)
    ex = TrainStepExecutor(scene.count, sh_degree, ssim_weight=ssim_weight, antialiased=aa)
    ex.upload_params(host.p, host.m, host.v, scene.count)
    N = scene.count
    for it in range(5):
        h = host_step(backend, host, cam, gt, cfg, it)
        loss, n_isects, render = ex.step(cam.viewmat, cam.K, cam.width, cam.height, gt, N,
                                         degrees_to_use=sh_degree, lr=LR, opacity_reg_w=0.01 / N,
                                         scale_reg_w=0.01 / (N * 3), want_render=(it == 0))
        assert n_isects == h["n_isects"], (it, n_isects, h["n_isects"])
        assert abs(loss - h["loss"]) <= 1e-6 + 1e-4 * abs(h["loss"]), (it, loss, h["loss"])
        if it == 0:
            assert rel_l2(render, h["render"], h["render"]) <= 1e-5
            p1 = [np.zeros_like(a) for a in host.p]
            ex.download_params(p1, [np.zeros_like(a) for a in p1], [np.zeros_like(a) for a in p1], N)
            for g in range(6):
                if host.p[g].size:
                    assert_step_close(p1[g], host.p[g], ("step-1 params", g))
    p = [np.zeros_like(a) for a in host.p]
    m = [np.zeros_like(a) for a in host.m]
    v = [np.zeros_like(a) for a in host.v]
    ex.download_params(p, m, v, N)
    for g in range(6):
        if host.p[g].size:
            assert_trajectory_close(p[g], host.p[g], ("params", g), v_ref=host.v[g], lr=LR[g], steps=5)
    ex.close()


def test_resident_noise_matches_host_path(backend):
    from splatx_cuda.executor import TrainStepExecutor
    from splatx_cuda.scene import small_scene
    scene, cam = small_scene(seed=2, n=2048, sh_degree=0)
    gt = _target(scene, cam)
    cfg = dict(ssim_weight=0.2, lr=LR, degrees_to_use=0, inject_noise=True, noise_seed=42,
               noise_scale=1.6e-4 * 5e5)
    host = HostState(scene)
    ex = TrainStepExecutor(scene.count, 0, ssim_weight=0.2)
    ex.upload_params(host.p, host.m, host.v, scene.count)
    for it in range(3):
        host_step(backend, host, cam, gt, cfg, it)
        ex.step(cam.viewmat, cam.K, cam.width, cam.height, gt, scene.count, lr=LR,
                inject_noise=True, noise_seed=42, noise_offset=it, noise_scale=1.6e-4 * 5e5)
    p = [np.zeros_like(a) for a in host.p]
    ex.download_params(p, [np.zeros_like(a) for a in p], [np.zeros_like(a) for a in p], scene.count)
    assert_trajectory_close(p[0], host.p[0], "means", v_ref=host.v[0], lr=LR[0], steps=3)
    ex.close()


def test_executor_capacity_growth_replays_step(backend):
    """A step that overflows the intersection capacity is replayed, not half-applied."""
    from splatx_cuda.executor import TrainStepExecutor
    from splatx_cuda.scene import small_scene
    scene, cam = small_scene(seed=3, n=20000, sh_degree=0)
    gt = np.full(cam.width * cam.height * 3, 0.5, np.float32)
    host = HostState(scene)
    a = TrainStepExecutor(scene.count, 0)
    a.upload_params(host.p, host.m, host.v, scene.count)
    la, na, _ = a.step(cam.viewmat, cam.K, cam.width, cam.height, gt, scene.count, lr=LR)
    b = TrainStepExecutor(scene.count, 0)
    b.upload_params(host.p, host.m, host.v, scene.count)
    b.reserve_isects(na + 10)  # no growth needed
    lb, nb, _ = b.step(cam.viewmat, cam.K, cam.width, cam.height, gt, scene.count, lr=LR)
    assert na == nb and na > 65536 and abs(la - lb) <= 1e-6 + 1e-5 * abs(la)
    a.close()
    b.close()


def test_executor_rejects_bad_inputs():
    from splatx_cuda.executor import TrainStepExecutor
    with pytest.raises(ValueError):
        TrainStepExecutor(0, 3)
    ex = TrainStepExecutor(16, 0)
    with pytest.raises(ValueError):
        ex.step(np.eye(4, dtype=np.float32).ravel(), np.eye(3, dtype=np.float32).ravel(), 8, 8,
                np.zeros(8 * 8 * 3, np.float32), 17)
    ex.close()


def test_graph_replay_follows_changing_cameras(backend):
    """Steps of one shape replay captured CUDA graphs (from the second step on); the camera,
    learning rates and noise live in a device parameter block, so alternating cameras must give
    the host path's losses and intersection counts step by step."""
    from splatx_cuda.executor import TrainStepExecutor
    from splatx_cuda.scene import Camera, small_scene
    scene, cam = small_scene(seed=5, n=3000, sh_degree=1)
    vm2 = cam.viewmat.copy()
    vm2[3] += 0.25
    cams = [cam, Camera(vm2, cam.K, cam.width, cam.height)]
    gts = [_target(scene, c) for c in cams]
    cfg = dict(ssim_weight=0.2, lr=LR, degrees_to_use=1, antialiased=False)
    host = HostState(scene)
    ex = TrainStepExecutor(scene.count, 1, ssim_weight=0.2)
    ex.upload_params(host.p, host.m, host.v, scene.count)
    for it in range(6):
        c, gt = cams[it % 2], gts[it % 2]
        h = host_step(backend, host, c, gt, cfg, it)
        loss, n_isects, _ = ex.step(c.viewmat, c.K, c.width, c.height, gt, scene.count,
                                    degrees_to_use=1, lr=LR)
        assert n_isects == h["n_isects"], (it, n_isects, h["n_isects"])
        assert abs(loss - h["loss"]) <= 1e-6 + 1e-4 * abs(h["loss"]), (it, loss, h["loss"])
    p = [np.zeros_like(a) for a in host.p]
    ex.download_params(p, [np.zeros_like(a) for a in p], [np.zeros_like(a) for a in p], scene.count)
    for g in range(6):
        if host.p[g].size:
            assert_trajectory_close(p[g], host.p[g], ("params", g), v_ref=host.v[g], lr=LR[g],
                                    steps=6)
    ex.close()
