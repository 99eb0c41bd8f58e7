"""CudaBackend — the host-side mirror of splatx-metal's ``KernelBackend`` for the B200 library.

Method names, argument meaning and error behaviour follow
``Sources/SplatXCore/include/splatx/KernelBackend.h:396-509``: inputs are host arrays (numpy),
outputs are fresh host arrays (the reference returns ``std::vector``), contract violations raise
``ValueError`` (``std::invalid_argument``) and device failures ``RuntimeError``. Every method runs
the sm_100a kernels of libsplatx_cuda.so through the C-ABI (include/splatx_cuda.h); torch is used
only to hold device memory and to name the current CUDA stream.
"""
from __future__ import annotations

import ctypes as C
from types import SimpleNamespace

import numpy as np
import torch

from . import _native as _nat
from ._native import check

_TORCH = {np.float32: torch.float32, np.int32: torch.int32, np.int64: torch.int64,
          np.uint8: torch.uint8, np.uint64: torch.int64, np.uint32: torch.int32,
          np.float64: torch.float64}


def _dt(dtype):
    return _TORCH[np.dtype(dtype).type]


class _Dev:
    """Keeps device copies alive for the duration of one call."""

    def __init__(self, device):
        self.device = device
        self.keep = []

    def up(self, arr, dtype=np.float32):
        if arr is None:
            return None
        a = np.ascontiguousarray(np.asarray(arr, dtype=dtype))
        view = a.view(np.int64) if a.dtype == np.uint64 else (a.view(np.int32) if a.dtype == np.uint32 else a)
        t = torch.from_numpy(view.copy()).to(self.device)
        self.keep.append(t)
        return t

    def empty(self, n, dtype=np.float32, zero=True):
        n = max(int(n), 0)
        t = (torch.zeros if zero else torch.empty)(max(n, 1), dtype=_dt(dtype), device=self.device)
        self.keep.append(t)
        return t

    @staticmethod
    def ptr(t):
        return None if t is None else C.c_void_p(t.data_ptr())

    @staticmethod
    def host(t, n, dtype=np.float32):
        a = t[: int(n)].cpu().numpy()
        return a.view(np.dtype(dtype)) if np.dtype(dtype).itemsize == a.itemsize else a.astype(dtype)


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


class CudaBackend:
    """B200 implementation of the KernelBackend verification surface (37 kernel entry points)."""

    def __init__(self, device: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("CudaBackend requires a CUDA device (no CPU fallback)")
        self.device = torch.device("cuda", device)
        _nat.lib()  # load now: a missing library fails here, loudly

    def name(self) -> str:
        return "cuda-sm100a"

    # ------------------------------------------------------------------ Adam
    def fused_adam(self, param, grad, exp_avg, exp_avg_sq, valid=None, n_gauss=None,
                   lr=0.0, b1=0.9, b2=0.999, eps=1e-8):
        """In place on the given float32 arrays (AdamInputs, KernelBackend.h:18-27)."""
        d = _Dev(self.device)
        n = int(np.asarray(param).size)
        tp, tg, tm, tv = d.up(param), d.up(grad), d.up(exp_avg), d.up(exp_avg_sq)
        tval = d.up(valid, np.uint8)
        a = _nat.SxAdamInputs(d.ptr(tp), d.ptr(tg), d.ptr(tm), d.ptr(tv), d.ptr(tval), n,
                           int(n_gauss if n_gauss is not None else n), lr, b1, b2, eps)
        check(_nat.lib().sxcuda_fused_adam(C.byref(a), _stream()))
        for t, arr in ((tp, param), (tm, exp_avg), (tv, exp_avg_sq)):
            arr[...] = t.cpu().numpy().reshape(np.shape(arr))

    # ------------------------------------------------------------------ projection
    def _proj_in(self, d, means, quats, scales, covars, opacities, viewmats, Ks, width, height,
                 eps2d, near_plane, far_plane, radius_clip, camera_model, calc_compensations):
        means = np.asarray(means, np.float32)
        Nn = means.size // 3
        C_ = np.asarray(viewmats).size // 16
        ins = _nat.SxProjectionFusedInputs(
            d.ptr(d.up(means)), d.ptr(d.up(covars)), d.ptr(d.up(quats)), d.ptr(d.up(scales)),
            d.ptr(d.up(opacities)), d.ptr(d.up(viewmats)), d.ptr(d.up(Ks)), Nn, C_, width, height,
            eps2d, near_plane, far_plane, radius_clip, camera_model, int(bool(calc_compensations)))
        return ins, Nn, C_

    def projection_fused_fwd(self, means, viewmats, Ks, width, height, quats=None, scales=None,
                             covars=None, opacities=None, eps2d=0.3, near_plane=0.01,
                             far_plane=1e10, radius_clip=0.0, camera_model=0,
                             calc_compensations=False):
        d = _Dev(self.device)
        ins, Nn, C_ = self._proj_in(d, means, quats, scales, covars, opacities, viewmats, Ks,
                                    width, height, eps2d, near_plane, far_plane, radius_clip,
                                    camera_model, calc_compensations)
        CN = Nn * C_
        radii, m2, dep, con = d.empty(CN * 2, np.int32), d.empty(CN * 2), d.empty(CN), d.empty(CN * 3)
        comp = d.empty(CN) if calc_compensations else None
        out = _nat.SxProjectionFusedOutputs(d.ptr(radii), d.ptr(m2), d.ptr(dep), d.ptr(con), d.ptr(comp))
        check(_nat.lib().sxcuda_projection_fused_fwd(C.byref(ins), C.byref(out), _stream()))
        return SimpleNamespace(radii=d.host(radii, CN * 2, np.int32), means2d=d.host(m2, CN * 2),
                               depths=d.host(dep, CN), conics=d.host(con, CN * 3),
                               compensations=d.host(comp, CN) if comp is not None else np.zeros(0, np.float32))

    def projection_fused_bwd(self, means, viewmats, Ks, width, height, radii, conics, v_means2d,
                             v_depths, v_conics, quats=None, scales=None, covars=None,
                             opacities=None, compensations=None, v_compensations=None,
                             viewmats_grad=False, eps2d=0.3, near_plane=0.01, far_plane=1e10,
                             radius_clip=0.0, camera_model=0, calc_compensations=False):
        d = _Dev(self.device)
        ins, Nn, C_ = self._proj_in(d, means, quats, scales, covars, opacities, viewmats, Ks,
                                    width, height, eps2d, near_plane, far_plane, radius_clip,
                                    camera_model, calc_compensations)
        g = _nat.SxProjectionFusedGradsIn(
            d.ptr(d.up(radii, np.int32)), d.ptr(d.up(conics)), d.ptr(d.up(compensations)),
            d.ptr(d.up(v_means2d)), d.ptr(d.up(v_depths)), d.ptr(d.up(v_conics)),
            d.ptr(d.up(v_compensations)), int(bool(viewmats_grad)))
        vm = d.empty(Nn * 3)
        vc = d.empty(Nn * 6) if covars is not None else None
        vq = d.empty(Nn * 4) if covars is None else None
        vs = d.empty(Nn * 3) if covars is None else None
        vv = d.empty(C_ * 16) if viewmats_grad else None
        out = _nat.SxProjectionFusedGrads(d.ptr(vm), d.ptr(vc), d.ptr(vq), d.ptr(vs), d.ptr(vv))
        check(_nat.lib().sxcuda_projection_fused_bwd(C.byref(ins), C.byref(g), C.byref(out), _stream()))
        e = np.zeros(0, np.float32)
        return SimpleNamespace(
            v_means=d.host(vm, Nn * 3), v_covars=d.host(vc, Nn * 6) if vc is not None else e,
            v_quats=d.host(vq, Nn * 4) if vq is not None else e,
            v_scales=d.host(vs, Nn * 3) if vs is not None else e,
            v_viewmats=d.host(vv, C_ * 16) if vv is not None else e)

    # ------------------------------------------------------------------ SH
    def _sh_in(self, d, dirs, coeffs, masks, degrees_to_use, B, N_, K, D, compute_v_dirs=False):
        return _nat.SxShInputs(d.ptr(d.up(dirs)), d.ptr(d.up(coeffs)), d.ptr(d.up(masks, np.uint8)),
                            degrees_to_use, B, N_, K, D, int(bool(compute_v_dirs)))

    def sh_fwd(self, dirs, coeffs, degrees_to_use, B, N, K, D=3, masks=None):
        d = _Dev(self.device)
        ins = self._sh_in(d, dirs, coeffs, masks, degrees_to_use, B, N, K, D)
        colors = d.empty(B * N * D)
        check(_nat.lib().sxcuda_sh_fwd(C.byref(ins), d.ptr(colors), _stream()))
        return SimpleNamespace(colors=d.host(colors, B * N * D))

    def sh_bwd(self, dirs, coeffs, v_colors, degrees_to_use, B, N, K, D=3, masks=None,
               compute_v_dirs=False):
        d = _Dev(self.device)
        ins = self._sh_in(d, dirs, coeffs, masks, degrees_to_use, B, N, K, D, compute_v_dirs)
        vco = d.empty(N * K * D)
        vdi = d.empty(B * N * 3) if compute_v_dirs else None
        check(_nat.lib().sxcuda_sh_bwd(C.byref(ins), d.ptr(d.up(v_colors)), d.ptr(vco),
                                                  d.ptr(vdi), _stream()))
        return SimpleNamespace(v_coeffs=d.host(vco, N * K * D),
                               v_dirs=d.host(vdi, B * N * 3) if vdi is not None else np.zeros(0, np.float32))

    # ------------------------------------------------------------------ intersection / sort
    def isect_tiles(self, means2d, radii, depths, I, N, tile_size, tile_width, tile_height,
                    conics=None, opacities=None):
        d = _Dev(self.device)
        L = _nat.lib()
        ins = _nat.SxIsectTilesInputs(
            d.ptr(d.up(means2d)), d.ptr(d.up(radii, np.int32)), d.ptr(d.up(depths)),
            d.ptr(d.up(conics)), d.ptr(d.up(opacities)), I, N, tile_size, tile_width, tile_height)
        n = I * N
        tiles = d.empty(n, np.int32)
        cum = d.empty(n, np.int64)
        nbytes = C.c_size_t(0)
        n_isects = C.c_int64(0)
        check(L.sxcuda_isect_tile_count(C.byref(ins), d.ptr(tiles), d.ptr(cum), C.byref(n_isects),
                                        None, C.byref(nbytes), _stream()))
        ws = d.empty(nbytes.value, np.uint8, zero=False)
        check(L.sxcuda_isect_tile_count(C.byref(ins), d.ptr(tiles), d.ptr(cum), C.byref(n_isects),
                                        d.ptr(ws), C.byref(nbytes), _stream()))
        ni = n_isects.value
        ids = d.empty(ni, np.int64)
        fl = d.empty(ni, np.int32)
        check(L.sxcuda_isect_tile_emit(C.byref(ins), d.ptr(cum), d.ptr(ids), d.ptr(fl), _stream()))
        tb = L.sxcuda_bits_for_count(tile_width * tile_height)
        return SimpleNamespace(tiles_per_gauss=d.host(tiles, n, np.int32),
                               isect_ids=d.host(ids, ni, np.uint64), flatten_ids=d.host(fl, ni, np.int32),
                               n_isects=ni, tile_n_bits=tb, image_n_bits=L.sxcuda_bits_for_count(I))

    def prefix_scan_i64(self, values):
        d = _Dev(self.device)
        L = _nat.lib()
        v = np.asarray(values, np.int32)
        n = v.size
        tin, tout = d.up(v, np.int32), d.empty(n, np.int64)
        nbytes = C.c_size_t(0)
        check(L.sxcuda_prefix_scan_i64(d.ptr(tin), d.ptr(tout), n, None, C.byref(nbytes), _stream()))
        ws = d.empty(nbytes.value, np.uint8, zero=False)
        check(L.sxcuda_prefix_scan_i64(d.ptr(tin), d.ptr(tout), n, d.ptr(ws), C.byref(nbytes), _stream()))
        return d.host(tout, n, np.int64)

    def sort_isect(self, keys, values, key_n_bits=64):
        d = _Dev(self.device)
        L = _nat.lib()
        k = np.asarray(keys, np.uint64)
        n = k.size
        tk, tv = d.up(k, np.uint64), d.up(values, np.int32)
        ok, ov = d.empty(n, np.int64), d.empty(n, np.int32)
        nbytes = C.c_size_t(0)
        check(L.sxcuda_sort_isect(d.ptr(tk), d.ptr(tv), d.ptr(ok), d.ptr(ov), n, key_n_bits, None,
                                  C.byref(nbytes), _stream()))
        ws = d.empty(nbytes.value, np.uint8, zero=False)
        check(L.sxcuda_sort_isect(d.ptr(tk), d.ptr(tv), d.ptr(ok), d.ptr(ov), n, key_n_bits,
                                  d.ptr(ws), C.byref(nbytes), _stream()))
        return SimpleNamespace(keys_sorted=d.host(ok, n, np.uint64), values_sorted=d.host(ov, n, np.int32))

    def isect_offset_encode(self, isect_ids, n_isects, I, tile_width, tile_height):
        d = _Dev(self.device)
        total = I * tile_width * tile_height
        off = d.empty(total, np.int32)
        check(_nat.lib().sxcuda_isect_offset_encode(
            d.ptr(d.up(isect_ids, np.uint64)), n_isects, I, tile_width, tile_height, d.ptr(off),
            _stream()))
        return d.host(off, total, np.int32)

    # ------------------------------------------------------------------ raster
    def _raster_in(self, d, means2d, conics, colors, opacities, isect_offsets, flatten_ids, I, N_,
                   n_isects, image_width, image_height, tile_size, tile_width, tile_height,
                   backgrounds=None, masks=None):
        return _nat.SxRasterizeFwdInputs(
            d.ptr(d.up(means2d)), d.ptr(d.up(conics)), d.ptr(d.up(colors)), d.ptr(d.up(opacities)),
            d.ptr(d.up(backgrounds)), d.ptr(d.up(masks, np.uint8)),
            d.ptr(d.up(isect_offsets, np.int32)), d.ptr(d.up(flatten_ids, np.int32)), I, N_,
            n_isects, image_width, image_height, tile_size, tile_width, tile_height)

    def rasterize_fwd(self, means2d, conics, colors, opacities, isect_offsets, flatten_ids, I, N,
                      n_isects, image_width, image_height, tile_size, tile_width, tile_height,
                      backgrounds=None, masks=None):
        d = _Dev(self.device)
        ins = self._raster_in(d, means2d, conics, colors, opacities, isect_offsets, flatten_ids, I,
                              N, n_isects, image_width, image_height, tile_size, tile_width,
                              tile_height, backgrounds, masks)
        px = I * image_width * image_height
        rc, ra, li = d.empty(px * 3), d.empty(px), d.empty(px, np.int32)
        check(_nat.lib().sxcuda_rasterize_fwd(C.byref(ins), d.ptr(rc), d.ptr(ra), d.ptr(li),
                                                        _stream()))
        return SimpleNamespace(render_colors=d.host(rc, px * 3), render_alphas=d.host(ra, px),
                               last_ids=d.host(li, px, np.int32))

    def rasterize_bwd(self, means2d, conics, colors, opacities, isect_offsets, flatten_ids, I, N,
                      n_isects, image_width, image_height, tile_size, tile_width, tile_height,
                      render_alphas, last_ids, v_render_colors, v_render_alphas,
                      backgrounds=None, masks=None, absgrad=False):
        d = _Dev(self.device)
        ins = self._raster_in(d, means2d, conics, colors, opacities, isect_offsets, flatten_ids, I,
                              N, n_isects, image_width, image_height, tile_size, tile_width,
                              tile_height, backgrounds, masks)
        g = _nat.SxRasterizeBwdGradsIn(
            d.ptr(d.up(render_alphas)), d.ptr(d.up(last_ids, np.int32)),
            d.ptr(d.up(v_render_colors)), d.ptr(d.up(v_render_alphas)), int(bool(absgrad)))
        IN = I * N
        vm, vc, vo, vp_ = d.empty(IN * 2), d.empty(IN * 3), d.empty(IN * 3), d.empty(IN)
        va = d.empty(IN * 2) if absgrad else None
        out = _nat.SxRasterizeBwdGrads(d.ptr(vm), d.ptr(vc), d.ptr(vo), d.ptr(vp_), d.ptr(va))
        check(_nat.lib().sxcuda_rasterize_bwd(C.byref(ins), C.byref(g), C.byref(out), _stream()))
        return SimpleNamespace(v_means2d=d.host(vm, IN * 2), v_conics=d.host(vc, IN * 3),
                               v_colors=d.host(vo, IN * 3), v_opacities=d.host(vp_, IN),
                               v_means2d_abs=d.host(va, IN * 2) if va is not None else np.zeros(0, np.float32))

    # ------------------------------------------------------------------ RNG / MCMC
    def rng_normal_f32(self, seed, offset, count):
        d = _Dev(self.device)
        out = d.empty(count)
        check(_nat.lib().sxcuda_rng_normal_f32(seed, offset, count, d.ptr(out), _stream()))
        return d.host(out, count)

    def rng_philox_u32(self, seed, offset, count):
        d = _Dev(self.device)
        out = d.empty(count, np.int32)
        check(_nat.lib().sxcuda_rng_philox_u32(seed, offset, count, d.ptr(out), _stream()))
        return d.host(out, count, np.uint32)

    def mcmc_relocation(self, opacities, scales, ratios, binoms, n_max=51, min_opacity=0.005):
        d = _Dev(self.device)
        n = np.asarray(opacities).size
        ins = _nat.SxRelocationInputs(
            d.ptr(d.up(opacities)), d.ptr(d.up(scales)), d.ptr(d.up(ratios, np.int32)),
            d.ptr(d.up(binoms)), n, n_max, min_opacity)
        no, ns = d.empty(n), d.empty(n * 3)
        check(_nat.lib().sxcuda_mcmc_relocation(C.byref(ins), d.ptr(no), d.ptr(ns), _stream()))
        return SimpleNamespace(new_opacities=d.host(no, n), new_scales=d.host(ns, n * 3))

    def mcmc_perturb_positions(self, positions, quats, scales_log, opacities_logit, noise,
                               noise_scale, t=0.005, k=100.0):
        """Updates ``positions`` in place (PerturbInputs, KernelBackend.h:265-275)."""
        d = _Dev(self.device)
        n = np.asarray(opacities_logit).size
        tp = d.up(positions)
        ins = _nat.SxPerturbInputs(
            d.ptr(tp), d.ptr(d.up(quats)), d.ptr(d.up(scales_log)), d.ptr(d.up(opacities_logit)),
            d.ptr(d.up(noise)), n, noise_scale, t, k)
        check(_nat.lib().sxcuda_mcmc_perturb_positions(C.byref(ins), _stream()))
        positions[...] = tp.cpu().numpy().reshape(np.shape(positions))

    # ------------------------------------------------------------------ SSIM
    def ssim_fwd(self, img1, img2, I, H, W, C_=3, need_coeffs=False):
        d = _Dev(self.device)
        L = _nat.lib()
        ins = _nat.SxSsimInputs(d.ptr(d.up(img1)), d.ptr(d.up(img2)), I, H, W, C_,
                                          int(bool(need_coeffs)))
        m = I * max(H - 10, 0) * max(W - 10, 0) * C_
        mp = d.empty(m)
        cm, cs, cc = (d.empty(m), d.empty(m), d.empty(m)) if need_coeffs else (None, None, None)
        mean = d.empty(1, np.float64)
        nbytes = C.c_size_t(0)
        check(L.sxcuda_ssim_fwd(C.byref(ins), d.ptr(mp), d.ptr(cm), d.ptr(cs), d.ptr(cc), d.ptr(mean),
                                None, C.byref(nbytes), _stream()))
        ws = d.empty(nbytes.value, np.uint8, zero=False)
        check(L.sxcuda_ssim_fwd(C.byref(ins), d.ptr(mp), d.ptr(cm), d.ptr(cs), d.ptr(cc), d.ptr(mean),
                                d.ptr(ws), C.byref(nbytes), _stream()))
        e = np.zeros(0, np.float32)
        return SimpleNamespace(ssim=float(mean.cpu().numpy()[0]), ssim_map=d.host(mp, m),
                               coeff_mu=d.host(cm, m) if cm is not None else e,
                               coeff_sigma=d.host(cs, m) if cs is not None else e,
                               coeff_cross=d.host(cc, m) if cc is not None else e)

    def ssim_bwd(self, img1, img2, I, H, W, C_, coeff_mu, coeff_sigma, coeff_cross, v_loss=1.0):
        d = _Dev(self.device)
        ins = _nat.SxSsimInputs(d.ptr(d.up(img1)), d.ptr(d.up(img2)), I, H, W, C_, 1)
        g = _nat.SxSsimGradsIn(d.ptr(d.up(coeff_mu)), d.ptr(d.up(coeff_sigma)),
                                         d.ptr(d.up(coeff_cross)), v_loss)
        n = I * H * W * C_
        out = d.empty(n)
        check(_nat.lib().sxcuda_ssim_bwd(C.byref(ins), C.byref(g), d.ptr(out), _stream()))
        return d.host(out, n)

    # ------------------------------------------------------------------ executor
    def make_train_step_executor(self, **desc):
        from .executor import TrainStepExecutor
        return TrainStepExecutor(device=self.device.index or 0, **desc)


def make_binoms_lut(n_max: int = 51) -> np.ndarray:
    lut = np.zeros(n_max * n_max, np.float32)
    check(_nat.lib().sxcuda_make_binoms_lut(n_max, lut.ctypes.data_as(C.c_void_p)))
    return lut
