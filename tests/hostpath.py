"""The host round-trip training step, composed from per-kernel backend calls.

A restatement of splatx-metal's ``Trainer::step`` host path (Sources/SplatXCore/Trainer.cpp:
716-832 forward_pass, :974-1131 step): activations -> projection -> SH + post-op -> AccuTile
intersection -> stable sort -> offsets -> raster fwd -> L1 (+SSIM) -> raster bwd -> relu mask ->
SH bwd -> projection bwd -> v_means += v_dirs -> activation chains + regularisers -> Adam x6 ->
(MCMC) noise. The reference keeps this path as the parity oracle of its resident executor; here it
runs over any object with the KernelBackend method names (the GPU CudaBackend), and the test
contrasts it with the resident executor exactly as TrainerTests.cpp:1720-1750 does.
Element-wise glue is float32 numpy.
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


class HostState:
    def __init__(self, scene):
        self.p = [np.array(g, np.float32, copy=True).reshape(scene.count, -1) for g in scene.groups()]
        self.m = [np.zeros_like(g) for g in self.p]
        self.v = [np.zeros_like(g) for g in self.p]
        self.sh_degree = scene.sh_degree

    @property
    def count(self):
        return self.p[0].shape[0]


def campos(vm):
    vm = np.asarray(vm, np.float32).reshape(4, 4)
    out = np.zeros(3, np.float32)
    for i in range(3):
        out[i] = -(f32(vm[0, i] * vm[0, 3]) + f32(vm[1, i] * vm[1, 3]) + f32(vm[2, i] * vm[2, 3]))
    return out


def host_step(be, st: HostState, cam, gt, cfg: dict, it: int = 0, forward_only=False):
    N = st.count
    K = (st.sh_degree + 1) ** 2
    deg = cfg.get("degrees_to_use", st.sh_degree)
    lam = cfg.get("ssim_weight", 0.2)
    aa = cfg.get("antialiased", False)
    means, quats, lsc, logit, sh0, shN = st.p
    s_lin = np.exp(lsc).astype(np.float32)
    sig = (f32(1.0) / (f32(1.0) + np.exp(-logit).astype(np.float32))).astype(np.float32).ravel()
    W, H = cam.width, cam.height
    common = dict(width=W, height=H, eps2d=cfg.get("eps2d", 0.3), near_plane=0.01, far_plane=1e10,
                  radius_clip=0.0, calc_compensations=aa)
    proj = be.projection_fused_fwd(means, cam.viewmat, cam.K, quats=quats, scales=s_lin,
                                   opacities=sig, **common)
    raster_op = sig * proj.compensations if aa else sig
    valid = ((proj.radii.reshape(-1, 2) > 0).all(axis=1)).astype(np.uint8)
    dirs = (means - campos(cam.viewmat)).astype(np.float32)
    coeffs = np.concatenate([sh0.reshape(N, 1, 3), shN.reshape(N, K - 1, 3)], axis=1)
    colors = be.sh_fwd(dirs, coeffs, deg, 1, N, K, 3, masks=valid).colors
    pre = colors + f32(0.5)
    relu = (pre > 0).astype(np.float32)
    colors = np.maximum(pre, f32(0.0))
    tw, th = (W + 15) // 16, (H + 15) // 16
    isect = be.isect_tiles(proj.means2d, proj.radii, proj.depths, 1, N, 16, tw, th,
                           conics=proj.conics, opacities=raster_op)
    srt = be.sort_isect(isect.isect_ids, isect.flatten_ids, 32 + isect.tile_n_bits + isect.image_n_bits)
    offsets = be.isect_offset_encode(srt.keys_sorted, isect.n_isects, 1, tw, th)
    rargs = dict(means2d=proj.means2d, conics=proj.conics, colors=colors, opacities=raster_op,
                 isect_offsets=offsets, flatten_ids=srt.values_sorted, I=1, N=N,
                 n_isects=isect.n_isects, image_width=W, image_height=H, tile_size=16,
                 tile_width=tw, tile_height=th)
    ras = be.rasterize_fwd(**rargs)
    out = {"render": ras.render_colors, "n_isects": isect.n_isects}
    if forward_only:
        return out
    r = ras.render_colors
    g = np.asarray(gt, np.float32).ravel()
    d = (r - g).astype(np.float32)
    n = d.size
    l1 = float(np.float32(np.abs(d.astype(np.float64)).sum() / n))
    gval = f32(1.0) / f32(n)
    v = np.where(d > 0, gval, np.where(d < 0, -gval, f32(0))).astype(np.float32)
    loss = l1
    if lam > 0:
        so = be.ssim_fwd(r, g, 1, H, W, 3, need_coeffs=True)
        v_dssim = be.ssim_bwd(r, g, 1, H, W, 3, so.coeff_mu, so.coeff_sigma, so.coeff_cross, v_loss=lam)
        v = (f32(1.0 - lam) * v + v_dssim).astype(np.float32)
        loss = float(f32(1.0 - lam) * f32(l1) + f32(lam) * (f32(1.0) - f32(so.ssim)))
    out["loss"] = loss
    rg = be.rasterize_bwd(**rargs, render_alphas=ras.render_alphas, last_ids=ras.last_ids,
                          v_render_colors=v, v_render_alphas=np.zeros(W * H, np.float32))
    v_colors = (rg.v_colors * relu.ravel()).astype(np.float32)
    sg = be.sh_bwd(dirs, coeffs, v_colors, deg, 1, N, K, 3, masks=valid, compute_v_dirs=True)
    v_op = rg.v_opacities.astype(np.float32)
    extra = {}
    if aa:
        v_comp = (v_op * sig).astype(np.float32)
        v_op = (v_op * proj.compensations).astype(np.float32)
        extra = dict(compensations=proj.compensations, v_compensations=v_comp)
    pg = be.projection_fused_bwd(means, cam.viewmat, cam.K, radii=proj.radii, conics=proj.conics,
                                 v_means2d=rg.v_means2d, v_depths=np.zeros(N, np.float32),
                                 v_conics=rg.v_conics, quats=quats, scales=s_lin, **extra, **common)
    v_means = (pg.v_means + sg.v_dirs).astype(np.float32)
    v_scales = (pg.v_scales * s_lin.ravel()).astype(np.float32)
    v_opc = (v_op * (sig * (f32(1) - sig))).astype(np.float32)
    orw, srw = cfg.get("opacity_reg", 0.0), cfg.get("scale_reg", 0.0)
    if orw > 0:
        v_opc = (v_opc + f32(orw / N) * sig * (f32(1) - sig)).astype(np.float32)
    if srw > 0:
        v_scales = (v_scales + f32(srw / (N * 3)) * s_lin.ravel()).astype(np.float32)
    vco = sg.v_coeffs.reshape(N, K, 3)
    grads = [v_means, pg.v_quats, v_scales, v_opc, vco[:, 0, :].copy(), vco[:, 1:, :].copy()]
    lrs = cfg["lr"]
    for gi in range(6):
        if st.p[gi].size == 0:
            continue
        be.fused_adam(st.p[gi], grads[gi].reshape(st.p[gi].shape), st.m[gi], st.v[gi], valid=valid,
                      n_gauss=N, lr=lrs[gi], b1=0.9, b2=0.999, eps=1e-15)
    if cfg.get("inject_noise"):
        noise = be.rng_normal_f32(cfg["noise_seed"], it, N * 3)
        be.mcmc_perturb_positions(st.p[0], st.p[1], st.p[2], st.p[3], noise, cfg["noise_scale"])
    return out
