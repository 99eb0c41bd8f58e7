"""A reduced MCMC training run (config 3's recipe at small scale) on the device-resident trainer
against the same run on the CPU oracle at matched seed: the alive count follows the same growth,
the early losses agree, and the held-out PSNR of the two trajectories agrees (chaotic divergence
of individual Gaussians is expected once sampling decisions differ by a last-bit change; the image
quality must not)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _cams(n, width, height, seed=0, offset=0.0):
    from splatx_cuda.scene import Camera, ring_camera
    f = 1150.0 * width / 1297.0
    K = np.array([f, 0, width / 2, 0, f, height / 2, 0, 0, 1], np.float32)
    out = []
    for i in range(n):
        c = ring_camera(i, n, width, height, seed=seed) if offset == 0.0 else None
        if c is None:  # held-out views between the training views
            c = ring_camera(i, n, width, height, seed=seed + 7)
            vm = c.viewmat.reshape(4, 4).astype(np.float64)
            a = 2 * np.pi * offset / n
            rot_t = np.array([[np.cos(a), 0, -np.sin(a), 0], [0, 1, 0, 0], [np.sin(a), 0, np.cos(a), 0],
                              [0, 0, 0, 1]])
            c = Camera((vm @ rot_t).astype(np.float32).ravel(), K, width, height)
        out.append(Camera(c.viewmat, K, width, height))
    return out


def test_reduced_mcmc_run_matches_oracle_psnr():
    import oracle
    from splatx_cuda.executor import TrainStepExecutor
    from splatx_cuda.scene import large_scene
    from splatx_cuda.trainer import (ResidentTrainer, TrainConfig, init_splats, mcmc_presets,
                                     psnr, scene_scale_from_cameras)
    sh, W, H = 1, 96, 96
    hidden, _ = large_scene(seed=1, n=6000, sh_degree=sh)
    HP = [np.ascontiguousarray(g.reshape(6000, -1)).copy() for g in hidden.groups()]
    train = _cams(12, W, H)
    held = _cams(3, W, H, offset=0.5)
    render_hidden = lambda c: oracle.host_step(HP, c, None, sh, forward_only=True,
                                               want_render=True)["render"]
    gts = [render_hidden(c) for c in train]
    gts_held = [render_hidden(c) for c in held]

    cfg = TrainConfig(total_iters=150)
    init_op, init_scale = mcmc_presets(cfg)
    cfg.mcmc.cap_max = 3000
    cfg.mcmc.refine_every_ratio = 10.0 / 150.0
    cfg.scene_scale = scene_scale_from_cameras([c.viewmat for c in train])
    rgb = np.clip((hidden.sh0.reshape(-1, 3) * 0.28209479 + 0.5) * 255, 0, 255).astype(np.uint8)
    init = init_splats(hidden.means.reshape(-1, 3), rgb, 1500, init_op, init_scale, sh)
    n0, cap = init[0].shape[0], cfg.mcmc.cap_max
    dims = [x.shape[1] for x in init]
    P = [np.zeros((cap, d), np.float32) for d in dims]
    for g in range(6):
        P[g][:n0] = init[g]
    M = [np.zeros_like(x) for x in P]
    V = [np.zeros_like(x) for x in P]
    order = list(np.random.default_rng(0).permutation(len(train)))

    ex = TrainStepExecutor(cap, sh)
    ex.upload_params(P, M, V, cap)
    tr = ResidentTrainer(ex, n0, sh, cfg)
    psnr0 = np.mean([psnr(tr.render(c), g) for c, g in zip(held, gts_held)])
    gpu_losses, counts = [], []
    for it in range(cfg.total_iters):
        v = order[it % len(order)]
        loss, _ = tr.step(it, train[v], 0, gt_host=gts[v])
        gpu_losses.append(loss)
        counts.append(tr.count)
    psnr_gpu = np.mean([psnr(tr.render(c), g) for c, g in zip(held, gts_held)])

    count_cpu, cpu_losses = oracle.host_mcmc_trajectory(P, M, V, n0, train, gts, cfg, sh,
                                                        cfg.total_iters, order)
    psnr_cpu = np.mean([psnr(oracle.host_step([x[:count_cpu] for x in P], c, None, sh,
                                              forward_only=True, want_render=True)["render"], g)
                        for c, g in zip(held, gts_held)])
    ex.close()

    assert counts[-1] == count_cpu > n0  # the same capped growth
    for a, b in zip(gpu_losses[:5], cpu_losses[:5]):  # before any refine: the same steps
        assert abs(a - b) <= 1e-4 * abs(b) + 1e-6
    assert psnr_gpu > psnr0 + 1.0, (psnr0, psnr_gpu)  # training improves the held-out views
    assert abs(psnr_gpu - psnr_cpu) < 0.5, (psnr_gpu, psnr_cpu)
