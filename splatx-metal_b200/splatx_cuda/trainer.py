"""Host mirror of the reference trainer's resident loop (Trainer::step_resident,
Sources/SplatXCore/Trainer.cpp:916-967) over the CUDA executor, MCMC included.

Per iteration, as the reference orders it:
  * the learning rates of the iteration (means decayed 0.01^(iter/total) and scaled by the scene
    scale, Trainer.cpp:496-500), the SH degree of the ramp (:502-508) and the regulariser weights
    reg/N and reg/(3N) (:934-941);
  * on a non-refine MCMC iteration the noise is fused into the step (seed, offset = iter, scale =
    means lr x noise_lr, :944-950);
  * on a refine iteration the step runs without noise, then the refine (relocate + add) and the
    noise on the grown count (:959-967) — here the refine runs on the device-resident arena
    instead of the reference's download / host mutation / upload.

The initial cloud follows init_splats (Trainer.cpp:270-330): seed points subsampled with stride
M/N, sh0 from the seed colours, identity rotations, opacity logit(init_opacity), isotropic
log-scales log(mean 3-NN distance x init_scale).
"""
from __future__ import annotations

import dataclasses

import numpy as np

from .mcmc import McmcOptions, means_lr_at, noise_scale_at, refine_due

SH_C0 = 0.28209479177387814


@dataclasses.dataclass
class TrainConfig:
    """The fields of TrainConfig (Trainer.h:206-260) the resident loop uses."""
    total_iters: int = 300
    scene_scale: float = 1.0
    lr_means: float = 1.6e-4
    lr_scales: float = 5e-3
    lr_quats: float = 1e-3
    lr_opacities: float = 5e-2
    lr_sh0: float = 2.5e-3
    lr_shN: float = 2.5e-3 / 20.0
    sh_degree_interval_ratio: float = 1.0 / 30.0
    opacity_reg: float = 0.0
    scale_reg: float = 0.0
    ssim_weight: float = 0.2
    mcmc: McmcOptions = dataclasses.field(default_factory=McmcOptions)


def mcmc_presets(cfg: TrainConfig) -> tuple[float, float]:
    """apply_mcmc_presets (Trainer.cpp:564-570): returns (init_opacity, init_scale) and sets the
    regularisers and MCMC on."""
    cfg.opacity_reg = 0.01
    cfg.scale_reg = 0.01
    cfg.mcmc.enabled = True
    return 0.5, 0.1


def scene_scale_from_cameras(viewmats) -> float:
    """scene_scale_from_cameras (Trainer.cpp:470-494): 1.1 x the largest distance of a camera
    centre from the centres' mean (1 for fewer than two cameras), in double with the reference's
    summation order, rounded to float."""
    import math
    vms = [np.asarray(v, np.float32).ravel() for v in viewmats]
    n = len(vms)
    if n < 2:
        return 1.0
    pos = []
    for vm in vms:
        v = [float(x) for x in vm]
        pos.append([-(v[0 * 4 + i] * v[0 * 4 + 3] + v[1 * 4 + i] * v[1 * 4 + 3] +
                      v[2 * 4 + i] * v[2 * 4 + 3]) for i in range(3)])
    c = [0.0, 0.0, 0.0]
    for p in pos:
        for i in range(3):
            c[i] += p[i]
    c = [x / n for x in c]
    best = 0.0
    for p in pos:
        dx, dy, dz = p[0] - c[0], p[1] - c[1], p[2] - c[2]
        best = max(best, math.sqrt(dx * dx + dy * dy + dz * dz))
    return float(np.float32(best * 1.1)) if best > 0.0 else 1.0


def sh_degree_at(cfg: TrainConfig, it: int, sh_degree: int) -> int:
    """sh_degree_at (Trainer.cpp:502-508)."""
    if sh_degree <= 0 or it < 0:
        return 0
    interval = max(1, int(np.float32(cfg.total_iters) * np.float32(cfg.sh_degree_interval_ratio)))
    return min(it // interval, sh_degree)


def knn3_mean_dists(pts: np.ndarray) -> np.ndarray:
    """knn3_mean_dists (Trainer.cpp:84-268): the mean distance to each point's k = min(3, n-1)
    nearest other points, with the reference's float arithmetic — squared distances
    dx*dx + dy*dy + dz*dz of float differences, the k smallest in ascending order, their float
    square roots summed in that order and divided by k. A k-d tree proposes 8 candidates per point
    (in double); the float distances decide among them."""
    from scipy.spatial import cKDTree
    p = np.asarray(pts, np.float32).reshape(-1, 3)
    n = p.shape[0]
    k = min(3, n - 1)
    if k <= 0:
        return np.zeros(n, np.float32)
    cand = min(8, n - 1)
    _, idx = cKDTree(p.astype(np.float64)).query(p.astype(np.float64), k=cand + 1)
    idx = idx.reshape(n, cand + 1)
    d = p[idx] - p[:, None, :]                                   # float32 differences
    d2 = (d[..., 0] * d[..., 0] + d[..., 1] * d[..., 1]) + d[..., 2] * d[..., 2]
    d2 = np.where(idx == np.arange(n)[:, None], np.float32(np.inf), d2)  # not the point itself
    best = np.sort(d2, axis=1)[:, :k]
    acc = np.zeros(n, np.float32)
    for t in range(k):
        acc = (acc + np.sqrt(best[:, t])).astype(np.float32)
    return (acc / np.float32(k)).astype(np.float32)


def init_splats(seed_points, seed_rgb, n_max: int, init_opacity: float, init_scale: float,
                sh_degree: int) -> list[np.ndarray]:
    """init_splats (Trainer.cpp:270-330) -> the six groups [N, dims] in the D3 order."""
    pts = np.asarray(seed_points, np.float32).reshape(-1, 3)
    rgb = np.asarray(seed_rgb).reshape(-1, 3)
    M = pts.shape[0]
    N = min(M, int(n_max))
    src = (np.arange(N, dtype=np.int64) * M) // N
    means = pts[src].copy()
    sh0 = ((rgb[src].astype(np.float32) * np.float32(1.0 / 255.0) - np.float32(0.5))
           / np.float32(SH_C0)).astype(np.float32)
    quats = np.zeros((N, 4), np.float32)
    quats[:, 0] = 1.0
    from ._libm import logf, logf_array
    p = np.float32(init_opacity)
    opac = np.full((N, 1), logf(np.float32(p / (np.float32(1) - p))), np.float32)
    mean_d = knn3_mean_dists(means)
    log_s = logf_array((np.maximum(mean_d, np.float32(1e-6)) * np.float32(init_scale)).astype(np.float32))
    scales = np.repeat(log_s[:, None], 3, axis=1)
    K = (sh_degree + 1) ** 2
    shN = np.zeros((N, (K - 1) * 3), np.float32)
    return [means, quats, scales, opac, sh0, shN]


class ResidentTrainer:
    """Trainer::step_resident over a TrainStepExecutor whose arena holds cfg.mcmc.cap_max rows
    (or the initial count without MCMC)."""

    def __init__(self, executor, count: int, sh_degree: int, cfg: TrainConfig):
        self.ex, self.count, self.sh_degree, self.cfg = executor, int(count), sh_degree, cfg
        if cfg.mcmc.enabled:
            executor.mcmc_seed(cfg.mcmc.seed)
        self.last_refine = None

    def lr(self, it: int) -> list[float]:
        c = self.cfg
        return [means_lr_at(c.lr_means, c.scene_scale, it, c.total_iters), c.lr_quats, c.lr_scales,
                c.lr_opacities, c.lr_sh0, c.lr_shN]

    def step(self, it: int, cam, gt_device_ptr: int, sync: bool = False, gt_host=None):
        """One iteration; returns (loss, n_isects) with ``sync`` (a read-back), else None."""
        c, m = self.cfg, self.cfg.mcmc
        n = self.count
        refine = m.enabled and refine_due(m, it, c.total_iters)
        noise = m.enabled and not refine
        ns = noise_scale_at(m, c.lr_means, c.scene_scale, it, c.total_iters) if m.enabled else 0.0
        kw = dict(degrees_to_use=sh_degree_at(c, it, self.sh_degree), lr=self.lr(it),
                  opacity_reg_w=float(np.float32(c.opacity_reg) / np.float32(n)) if c.opacity_reg > 0 else 0.0,
                  scale_reg_w=float(np.float32(c.scale_reg) / np.float32(n * 3)) if c.scale_reg > 0 else 0.0,
                  inject_noise=noise, noise_seed=m.seed, noise_offset=it, noise_scale=ns)
        out = None
        if gt_host is not None:
            loss, nis, _ = self.ex.step(cam.viewmat, cam.K, cam.width, cam.height, gt_host, n, **kw)
            out = (loss, nis)
        else:
            self.ex.step_async(cam.viewmat, cam.K, cam.width, cam.height, gt_device_ptr, n, **kw)
            if sync:
                loss, nis, _ = self.ex.last_result()
                out = (loss, nis)
        if refine:
            self.last_refine = self.ex.mcmc_refine(n, m.cap_max, m.min_opacity, want_lists=False)
            self.count = self.last_refine["count"]
            self.ex.inject_noise(self.count, m.seed, it, ns)
        return out

    def render(self, cam, degree=None):
        """Forward-only render of the current cloud (host image [H*W*3])."""
        _, _, img = self.ex.step(cam.viewmat, cam.K, cam.width, cam.height, None, self.count,
                                 degrees_to_use=self.sh_degree if degree is None else degree,
                                 forward_only=True, want_render=True)
        return img


def psnr(img, ref) -> float:
    """PSNR of an image against a reference in [0, 1] (renders clipped to [0, 1])."""
    a = np.clip(np.asarray(img, np.float64), 0.0, 1.0)
    b = np.clip(np.asarray(ref, np.float64), 0.0, 1.0)
    mse = float(np.mean((a - b) ** 2))
    return float("inf") if mse == 0 else -10.0 * np.log10(mse)
