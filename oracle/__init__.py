"""CPU oracle of the 3DGS training step — TEST INFRASTRUCTURE.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference arm may import
this package, and only as the checker or the timed CPU reference; nothing in the product path
(splatx-metal_b200/) uses it.

``OracleBackend`` exposes the reference's KernelBackend method names over the plain-C restatement
(liboracle.so, sx_oracle.c); ``RefBackend`` the same names over the reference's own CPU kernels
(oracle/_ref/libsplatx_ref.so, built from the reference tree by ``make ref`` where that tree
exists). Their results are numpy arrays, like splatx_cuda.backend.CudaBackend's, so a test can run
the same comparison over all three.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib
import subprocess
from types import SimpleNamespace

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libsplatx_ref.so"


def reference_tree(explicit=None):
    """The reference checkout: `explicit`, else $SPLATX_REFERENCE; None when neither names a tree
    that holds the reference's CPU sources."""
    root = explicit if explicit is not None else os.environ.get("SPLATX_REFERENCE")
    if not root:
        return None
    root = pathlib.Path(root)
    return root if (root / "Sources" / "SplatXCore" / "CpuKernels.cpp").exists() else None


def build(force: bool = False, reference=None) -> None:
    """Compile liboracle.so, and oracle/_ref when a reference tree is given (argument or
    $SPLATX_REFERENCE) and present."""
    args = ["make", "-C", str(HERE)] + (["-B"] if force else [])
    subprocess.run(args, check=True, capture_output=True)
    tree = reference_tree(reference)
    if tree is not None:
        jobs = f"-j{min(16, os.cpu_count() or 1)}"
        subprocess.run(args + [jobs, "ref", "ref-tests", f"REF={tree}"], check=True,
                       capture_output=True)


def available() -> bool:
    return LIB.exists()


def ref_available() -> bool:
    return REF_LIB.exists()


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            raise RuntimeError(f"{LIB} missing: run `make -C oracle`")
        _lib = C.CDLL(str(LIB))
        _lib.sxo_isect_count.restype = C.c_int64
        _lib.sxo_ssim_fwd.restype = C.c_double
        _lib.sxo_bits_for_count.restype = C.c_uint32
        for name in ("sxo_sort_isect", "sxo_mcmc_relocation", "sxo_train_step", "sxo_set_threads",
                     "sxo_multinomial", "sxo_mcmc_refine"):
            getattr(_lib, name).restype = C.c_int32
        _lib.sxo_mt64_next.restype = C.c_uint64
        _lib.sxo_train_loss.restype = C.c_float
    return _lib


def set_threads(n: int) -> int:
    """OpenMP threads for the oracle's parallel loops; returns the effective count."""
    return int(lib().sxo_set_threads(C.c_int32(int(n))))


def ref_lib():
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise RuntimeError(f"{REF_LIB} missing: run `make -C oracle ref` where the reference exists")
        _ref = C.CDLL(str(REF_LIB))
        _ref.sxr_last_error.restype = C.c_char_p
    return _ref


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype=np.float32):
    return None if a is None else np.ascontiguousarray(np.asarray(a, dtype))


I64, U32, F32, U64, I32, D64 = C.c_int64, C.c_uint32, C.c_float, C.c_uint64, C.c_int32, C.c_double


class OracleBackend:
    """KernelBackend method names over the C restatement (sx_oracle.c)."""

    def name(self):
        return "cpu-oracle"

    def fused_adam(self, param, grad, exp_avg, exp_avg_sq, valid=None, n_gauss=None, lr=0.0,
                   b1=0.9, b2=0.999, eps=1e-8):
        n = param.size
        g = _c(grad)
        v8 = _c(valid, np.uint8)
        lib().sxo_fused_adam(_p(param), _p(g), _p(exp_avg), _p(exp_avg_sq), _p(v8), I64(n),
                             I64(n_gauss if n_gauss is not None else n), F32(lr), F32(b1),
                             F32(b2), F32(eps))

    def projection_fused_fwd(self, means, viewmats, Ks, width, height, quats=None, scales=None,
                             covars=None, opacities=None, eps2d=0.3, near_plane=0.01,
                             far_plane=1e10, radius_clip=0.0, camera_model=0,
                             calc_compensations=False):
        m, q, s, cv, o = _c(means), _c(quats), _c(scales), _c(covars), _c(opacities)
        vm, K = _c(viewmats), _c(Ks)
        N, Cn = m.size // 3, vm.size // 16
        out = SimpleNamespace(radii=np.zeros(Cn * N * 2, np.int32), means2d=np.zeros(Cn * N * 2, np.float32),
                              depths=np.zeros(Cn * N, np.float32), conics=np.zeros(Cn * N * 3, np.float32),
                              compensations=np.zeros(Cn * N if calc_compensations else 0, np.float32))
        lib().sxo_projection_fused_fwd(_p(m), _p(cv), _p(q), _p(s), _p(o), _p(vm), _p(K), I64(N),
                                       I64(Cn), I32(width), I32(height), F32(eps2d),
                                       F32(near_plane), F32(far_plane), F32(radius_clip),
                                       I32(int(bool(calc_compensations))), _p(out.radii),
                                       _p(out.means2d), _p(out.depths), _p(out.conics),
                                       _p(out.compensations) if calc_compensations else None)
        return out

    def projection_fused_bwd(self, means, viewmats, Ks, width, height, radii, conics, v_means2d,
                             v_depths, v_conics, quats=None, scales=None, covars=None,
                             opacities=None, compensations=None, v_compensations=None,
                             viewmats_grad=False, eps2d=0.3, **_):
        m, q, s, cv = _c(means), _c(quats), _c(scales), _c(covars)
        vm, K = _c(viewmats), _c(Ks)
        N, Cn = m.size // 3, vm.size // 16
        vmean = np.zeros(N * 3, np.float32)
        vcov = np.zeros(N * 6, np.float32) if covars is not None else np.zeros(0, np.float32)
        vq = np.zeros(N * 4 if covars is None else 0, np.float32)
        vs = np.zeros(N * 3 if covars is None else 0, np.float32)
        vv = np.zeros(Cn * 16 if viewmats_grad else 0, np.float32)
        lib().sxo_projection_fused_bwd(
            _p(m), _p(cv), _p(q), _p(s), _p(vm), _p(K), I64(N), I64(Cn), I32(width), I32(height),
            F32(eps2d), _p(_c(radii, np.int32)), _p(_c(conics)), _p(_c(compensations)),
            _p(_c(v_means2d)), _p(_c(v_depths)), _p(_c(v_conics)), _p(_c(v_compensations)),
            _p(vmean), _p(vcov) if covars is not None else None, _p(vq) if covars is None else None,
            _p(vs) if covars is None else None, _p(vv) if viewmats_grad else None)
        return SimpleNamespace(v_means=vmean, v_covars=vcov, v_quats=vq, v_scales=vs, v_viewmats=vv)

    def sh_fwd(self, dirs, coeffs, degrees_to_use, B, N, K, D=3, masks=None):
        colors = np.zeros(B * N * D, np.float32)
        lib().sxo_sh_fwd(_p(_c(dirs)), _p(_c(coeffs)), _p(_c(masks, np.uint8)), U32(degrees_to_use),
                         I64(B), I64(N), I64(K), U32(D), _p(colors))
        return SimpleNamespace(colors=colors)

    def sh_bwd(self, dirs, coeffs, v_colors, degrees_to_use, B, N, K, D=3, masks=None,
               compute_v_dirs=False):
        vco = np.zeros(N * K * D, np.float32)
        vd = np.zeros(B * N * 3, np.float32) if compute_v_dirs else np.zeros(0, np.float32)
        lib().sxo_sh_bwd(_p(_c(dirs)), _p(_c(coeffs)), _p(_c(masks, np.uint8)), U32(degrees_to_use),
                         I64(B), I64(N), I64(K), U32(D), _p(_c(v_colors)), _p(vco),
                         _p(vd) if compute_v_dirs else None)
        return SimpleNamespace(v_coeffs=vco, v_dirs=vd)

    def isect_tiles(self, means2d, radii, depths, I, N, tile_size, tile_width, tile_height,
                    conics=None, opacities=None):
        m2, r, d = _c(means2d), _c(radii, np.int32), _c(depths)
        cn, op = _c(conics), _c(opacities)
        tiles = np.zeros(I * N, np.int32)
        n = int(lib().sxo_isect_count(_p(m2), _p(r), _p(cn), _p(op), I64(I * N), U32(tile_size),
                                      U32(tile_width), U32(tile_height), _p(tiles)))
        ids = np.zeros(n, np.uint64)
        fl = np.zeros(n, np.int32)
        lib().sxo_isect_emit(_p(m2), _p(r), _p(d), _p(cn), _p(op), I64(I), I64(N), U32(tile_size),
                             U32(tile_width), U32(tile_height), _p(tiles), _p(ids), _p(fl))
        L = lib()
        return SimpleNamespace(tiles_per_gauss=tiles, isect_ids=ids, flatten_ids=fl, n_isects=n,
                               tile_n_bits=L.sxo_bits_for_count(I64(tile_width * tile_height)),
                               image_n_bits=L.sxo_bits_for_count(I64(I)))

    def prefix_scan_i64(self, values):
        return np.cumsum(np.asarray(values, np.int32), dtype=np.int64)

    def sort_isect(self, keys, values, key_n_bits=64):
        k, v = _c(keys, np.uint64), _c(values, np.int32)
        ko, vo = np.zeros_like(k), np.zeros_like(v)
        if lib().sxo_sort_isect(_p(k), _p(v), I64(k.size), U32(key_n_bits), _p(ko), _p(vo)) != 0:
            raise ValueError("sort_isect: key has bits above key_n_bits")
        return SimpleNamespace(keys_sorted=ko, values_sorted=vo)

    def isect_offset_encode(self, isect_ids, n_isects, I, tile_width, tile_height):
        off = np.zeros(I * tile_width * tile_height, np.int32)
        lib().sxo_isect_offset_encode(_p(_c(isect_ids, np.uint64)), I64(n_isects), I64(I),
                                      U32(tile_width), U32(tile_height), _p(off))
        return off

    def _ras(self, means2d, conics, colors, opacities, isect_offsets, flatten_ids, backgrounds,
             masks):
        return [_c(means2d), _c(conics), _c(colors), _c(opacities), _c(backgrounds),
                _c(masks, np.uint8), _c(isect_offsets, np.int32), _c(flatten_ids, np.int32)]

    def rasterize_fwd(self, means2d, conics, colors, opacities, isect_offsets, flatten_ids, I, N,
                      n_isects, image_width, image_height, tile_size, tile_width, tile_height,
                      backgrounds=None, masks=None):
        a = self._ras(means2d, conics, colors, opacities, isect_offsets, flatten_ids, backgrounds, masks)
        px = I * image_width * image_height
        rc, ra, li = np.zeros(px * 3, np.float32), np.zeros(px, np.float32), np.zeros(px, np.int32)
        lib().sxo_rasterize_fwd(*map(_p, a), I64(I), I64(N), I64(n_isects), U32(image_width),
                                U32(image_height), U32(tile_size), U32(tile_width),
                                U32(tile_height), _p(rc), _p(ra), _p(li))
        return SimpleNamespace(render_colors=rc, render_alphas=ra, last_ids=li)

    def rasterize_bwd(self, means2d, conics, colors, opacities, isect_offsets, flatten_ids, I, N,
                      n_isects, image_width, image_height, tile_size, tile_width, tile_height,
                      render_alphas, last_ids, v_render_colors, v_render_alphas,
                      backgrounds=None, masks=None, absgrad=False):
        a = self._ras(means2d, conics, colors, opacities, isect_offsets, flatten_ids, backgrounds, masks)
        IN = I * N
        vm, vc, vo, vp = (np.zeros(IN * 2, np.float32), np.zeros(IN * 3, np.float32),
                          np.zeros(IN * 3, np.float32), np.zeros(IN, np.float32))
        va = np.zeros(IN * 2 if absgrad else 0, np.float32)
        lib().sxo_rasterize_bwd(*map(_p, a), I64(I), I64(N), I64(n_isects), U32(image_width),
                                U32(image_height), U32(tile_size), U32(tile_width),
                                U32(tile_height), _p(_c(render_alphas)), _p(_c(last_ids, np.int32)),
                                _p(_c(v_render_colors)), _p(_c(v_render_alphas)), _p(vm), _p(vc),
                                _p(vo), _p(vp), _p(va) if absgrad else None)
        return SimpleNamespace(v_means2d=vm, v_conics=vc, v_colors=vo, v_opacities=vp, v_means2d_abs=va)

    def rng_normal_f32(self, seed, offset, count):
        out = np.zeros(count, np.float32)
        lib().sxo_rng_normal_f32(U64(seed), U64(offset), I64(count), _p(out))
        return out

    def rng_philox_u32(self, seed, offset, count):
        out = np.zeros(count, np.uint32)
        lib().sxo_rng_philox_u32(U64(seed), U64(offset), I64(count), _p(out))
        return out

    def philox4x32_10(self, ctr, key):
        c = np.asarray(ctr, np.uint32)
        k = np.asarray(key, np.uint32)
        out = np.zeros(4, np.uint32)
        lib().sxo_philox4x32_10(_p(c), _p(k), _p(out))
        return out

    def mcmc_relocation(self, opacities, scales, ratios, binoms, n_max=51, min_opacity=0.005):
        o = _c(opacities)
        no, ns = np.zeros(o.size, np.float32), np.zeros(o.size * 3, np.float32)
        if lib().sxo_mcmc_relocation(_p(o), _p(_c(scales)), _p(_c(ratios, np.int32)), _p(_c(binoms)),
                                     I64(o.size), I32(n_max), F32(min_opacity), _p(no), _p(ns)) != 0:
            raise ValueError("mcmc_relocation: ratio outside [1, n_max]")
        return SimpleNamespace(new_opacities=no, new_scales=ns)

    def mcmc_perturb_positions(self, positions, quats, scales_log, opacities_logit, noise,
                               noise_scale, t=0.005, k=100.0):
        n = np.asarray(opacities_logit).size
        lib().sxo_mcmc_perturb_positions(_p(positions), _p(_c(quats)), _p(_c(scales_log)),
                                         _p(_c(opacities_logit)), _p(_c(noise)), I64(n),
                                         F32(noise_scale), F32(t), F32(k))

    def ssim_fwd(self, img1, img2, I, H, W, C_=3, need_coeffs=False):
        m = I * (H - 10) * (W - 10) * C_
        mp = np.zeros(m, np.float32)
        cm, cs, cc = (np.zeros(m, np.float32) for _ in range(3))
        s = lib().sxo_ssim_fwd(_p(_c(img1)), _p(_c(img2)), I64(I), I64(H), I64(W), I64(C_),
                               I32(int(bool(need_coeffs))), _p(mp), _p(cm), _p(cs), _p(cc))
        e = np.zeros(0, np.float32)
        return SimpleNamespace(ssim=float(s), ssim_map=mp, coeff_mu=cm if need_coeffs else e,
                               coeff_sigma=cs if need_coeffs else e, coeff_cross=cc if need_coeffs else e)

    def ssim_bwd(self, img1, img2, I, H, W, C_, coeff_mu, coeff_sigma, coeff_cross, v_loss=1.0):
        out = np.zeros(I * H * W * C_, np.float32)
        lib().sxo_ssim_bwd(_p(_c(img1)), _p(_c(img2)), I64(I), I64(H), I64(W), I64(C_),
                           _p(_c(coeff_mu)), _p(_c(coeff_sigma)), _p(_c(coeff_cross)), F32(v_loss),
                           _p(out))
        return out


class RefBackend:
    """The same method names over the reference's own CPU kernels (oracle/_ref, ref_shim.cpp)."""

    def _ok(self, rc):
        if rc != 0:
            raise ValueError(ref_lib().sxr_last_error().decode())

    def fused_adam(self, param, grad, exp_avg, exp_avg_sq, valid=None, n_gauss=None, lr=0.0,
                   b1=0.9, b2=0.999, eps=1e-8):
        n = param.size
        self._ok(ref_lib().sxr_fused_adam(_p(param), _p(_c(grad)), _p(exp_avg), _p(exp_avg_sq),
                                          _p(_c(valid, np.uint8)), I64(n),
                                          I64(n_gauss if n_gauss is not None else n), F32(lr),
                                          F32(b1), F32(b2), F32(eps)))

    def projection_fused_fwd(self, means, viewmats, Ks, width, height, quats=None, scales=None,
                             covars=None, opacities=None, eps2d=0.3, near_plane=0.01,
                             far_plane=1e10, radius_clip=0.0, camera_model=0,
                             calc_compensations=False):
        m, vm = _c(means), _c(viewmats)
        N, Cn = m.size // 3, vm.size // 16
        out = SimpleNamespace(radii=np.zeros(Cn * N * 2, np.int32), means2d=np.zeros(Cn * N * 2, np.float32),
                              depths=np.zeros(Cn * N, np.float32), conics=np.zeros(Cn * N * 3, np.float32),
                              compensations=np.zeros(Cn * N if calc_compensations else 0, np.float32))
        self._ok(ref_lib().sxr_projection_fused_fwd(
            _p(m), _p(_c(covars)), _p(_c(quats)), _p(_c(scales)), _p(_c(opacities)), _p(vm),
            _p(_c(Ks)), I64(N), I64(Cn), I32(width), I32(height), F32(eps2d), F32(near_plane),
            F32(far_plane), F32(radius_clip), I32(int(bool(calc_compensations))), _p(out.radii),
            _p(out.means2d), _p(out.depths), _p(out.conics),
            _p(out.compensations) if calc_compensations else None))
        return out

    def sh_fwd(self, dirs, coeffs, degrees_to_use, B, N, K, D=3, masks=None):
        colors = np.zeros(B * N * D, np.float32)
        self._ok(ref_lib().sxr_sh_fwd(_p(_c(dirs)), _p(_c(coeffs)), _p(_c(masks, np.uint8)),
                                      U32(degrees_to_use), I64(B), I64(N), I64(K), U32(D), _p(colors)))
        return SimpleNamespace(colors=colors)

    def isect_tiles(self, means2d, radii, depths, I, N, tile_size, tile_width, tile_height,
                    conics=None, opacities=None):
        a = [_c(means2d), _c(radii, np.int32), _c(depths), _c(conics), _c(opacities)]
        tiles = np.zeros(I * N, np.int32)
        n = C.c_int64()
        args = [*map(_p, a), I64(I), I64(N), U32(tile_size), U32(tile_width), U32(tile_height), _p(tiles)]
        self._ok(ref_lib().sxr_isect_tiles(*args, None, None, I64(0), C.byref(n)))
        ids, fl = np.zeros(n.value, np.uint64), np.zeros(n.value, np.int32)
        self._ok(ref_lib().sxr_isect_tiles(*args, _p(ids), _p(fl), I64(n.value), C.byref(n)))
        return SimpleNamespace(tiles_per_gauss=tiles, isect_ids=ids, flatten_ids=fl, n_isects=n.value,
                               tile_n_bits=lib().sxo_bits_for_count(I64(tile_width * tile_height)),
                               image_n_bits=lib().sxo_bits_for_count(I64(I)))

    def sort_isect(self, keys, values, key_n_bits=64):
        k, v = _c(keys, np.uint64), _c(values, np.int32)
        ko, vo = np.zeros_like(k), np.zeros_like(v)
        self._ok(ref_lib().sxr_sort_isect(_p(k), _p(v), I64(k.size), U32(key_n_bits), _p(ko), _p(vo)))
        return SimpleNamespace(keys_sorted=ko, values_sorted=vo)

    def isect_offset_encode(self, isect_ids, n_isects, I, tile_width, tile_height):
        off = np.zeros(I * tile_width * tile_height, np.int32)
        self._ok(ref_lib().sxr_isect_offset_encode(_p(_c(isect_ids, np.uint64)), I64(n_isects), I64(I),
                                                   U32(tile_width), U32(tile_height), _p(off)))
        return off

    def rasterize_fwd(self, means2d, conics, colors, opacities, isect_offsets, flatten_ids, I, N,
                      n_isects, image_width, image_height, tile_size, tile_width, tile_height,
                      backgrounds=None, masks=None):
        px = I * image_width * image_height
        rc, ra, li = np.zeros(px * 3, np.float32), np.zeros(px, np.float32), np.zeros(px, np.int32)
        self._ok(ref_lib().sxr_rasterize_fwd(
            _p(_c(means2d)), _p(_c(conics)), _p(_c(colors)), _p(_c(opacities)), _p(_c(backgrounds)),
            _p(_c(isect_offsets, np.int32)), _p(_c(flatten_ids, np.int32)), I64(I), I64(N),
            I64(n_isects), U32(image_width), U32(image_height), U32(tile_size), U32(tile_width),
            U32(tile_height), _p(rc), _p(ra), _p(li)))
        return SimpleNamespace(render_colors=rc, render_alphas=ra, last_ids=li)

    def ssim_fwd(self, img1, img2, I, H, W, C_=3, need_coeffs=False):
        m = I * (H - 10) * (W - 10) * C_
        mp, cm, cs, cc = (np.zeros(m, np.float32) for _ in range(4))
        mean = C.c_double()
        self._ok(ref_lib().sxr_ssim_fwd(_p(_c(img1)), _p(_c(img2)), I64(I), I64(H), I64(W), I64(C_),
                                        I32(int(bool(need_coeffs))), _p(mp), _p(cm), _p(cs), _p(cc),
                                        C.byref(mean)))
        return SimpleNamespace(ssim=mean.value, ssim_map=mp, coeff_mu=cm, coeff_sigma=cs, coeff_cross=cc)

    def rng_philox_u32(self, seed, offset, count):
        out = np.zeros(count, np.uint32)
        self._ok(ref_lib().sxr_rng_philox_u32(U64(seed), U64(offset), I64(count), _p(out)))
        return out

    def rng_normal_f32(self, seed, offset, count):
        out = np.zeros(count, np.float32)
        self._ok(ref_lib().sxr_rng_normal_f32(U64(seed), U64(offset), I64(count), _p(out)))
        return out

    def mcmc_relocation(self, opacities, scales, ratios, binoms, n_max=51, min_opacity=0.005):
        o = _c(opacities)
        no, ns = np.zeros(o.size, np.float32), np.zeros(o.size * 3, np.float32)
        self._ok(ref_lib().sxr_mcmc_relocation(_p(o), _p(_c(scales)), _p(_c(ratios, np.int32)),
                                               _p(_c(binoms)), I64(o.size), I32(n_max),
                                               F32(min_opacity), _p(no), _p(ns)))
        return SimpleNamespace(new_opacities=no, new_scales=ns)

    def mcmc_perturb_positions(self, positions, quats, scales_log, opacities_logit, noise,
                               noise_scale, t=0.005, k=100.0):
        n = np.asarray(opacities_logit).size
        self._ok(ref_lib().sxr_mcmc_perturb_positions(_p(positions), _p(_c(quats)), _p(_c(scales_log)),
                                                      _p(_c(opacities_logit)), _p(_c(noise)), I64(n),
                                                      F32(noise_scale), F32(t), F32(k)))


class _Mt64(C.Structure):
    _fields_ = [("x", C.c_uint64 * 312), ("i", C.c_int32)]


class _McmcResult(C.Structure):
    _fields_ = [("count", C.c_int64), ("n_relocated", C.c_int64), ("n_added", C.c_int64)]


class McmcOracle:
    """The reference's MCMC refine host logic (Trainer.cpp:1195-1435) over numpy arrays, with its
    own mt19937_64 state (seeded like McmcOptions::seed, default 42)."""

    def __init__(self, seed: int = 42):
        self._g = _Mt64()
        self.seed(seed)

    def seed(self, seed: int):
        lib().sxo_mt64_seed(C.byref(self._g), C.c_uint64(int(seed)))

    def next(self) -> int:
        return int(lib().sxo_mt64_next(C.byref(self._g)))

    def state_text(self) -> str:
        """The engine as libstdc++ writes ``os << std::mt19937_64``: the 312 words, then the
        position."""
        return " ".join(str(int(v)) for v in self._g.x) + " " + str(int(self._g.i))

    def multinomial(self, weights, n_samples: int) -> np.ndarray:
        w = _c(weights)
        out = np.zeros(max(int(n_samples), 1), np.int64)
        rc = lib().sxo_multinomial(_p(w), I64(w.size), I64(int(n_samples)), C.byref(self._g), _p(out))
        if rc != 0:
            raise ValueError("multinomial: bad weights")
        return out[:int(n_samples)]

    def refine(self, params, exp_avg, exp_avg_sq, count: int, cap_max: int,
               min_opacity: float = 0.005) -> dict:
        """One refine in place on six [arena_rows, dims] float32 arrays per set (rows >= cap_max)."""
        dims = np.array([a.shape[1] if a.ndim == 2 else 0 for a in params], np.int64)
        for arrs in (params, exp_avg, exp_avg_sq):
            for a in arrs:
                assert a.dtype == np.float32 and a.flags.c_contiguous
        ptrs = [(C.c_void_p * 6)(*[a.ctypes.data for a in arrs]) for arrs in (params, exp_avg, exp_avg_sq)]
        lists = [np.zeros(max(int(cap_max), 1), np.int64) for _ in range(3)]
        res = _McmcResult()
        rc = lib().sxo_mcmc_refine(C.byref(self._g), ptrs[0], ptrs[1], ptrs[2], _p(dims),
                                   I64(int(count)), I64(int(cap_max)), F32(min_opacity),
                                   _p(lists[0]), _p(lists[1]), _p(lists[2]), C.byref(res))
        if rc != 0:
            raise ValueError("mcmc_refine: contract violation")
        return {"count": int(res.count), "relocated_dead": lists[0][:res.n_relocated].copy(),
                "relocation_src": lists[1][:res.n_relocated].copy(),
                "added_src": lists[2][:res.n_added].copy()}


def ref_mt64_outputs(seed: int, n: int) -> np.ndarray:
    """The first n outputs of the reference toolchain's std::mt19937_64(seed) (oracle/_ref)."""
    out = np.zeros(n, np.uint64)
    rc = ref_lib().sxr_mt64_outputs(C.c_uint64(int(seed)), I64(n), _p(out))
    if rc != 0:
        raise ValueError(ref_lib().sxr_last_error().decode())
    return out


def ref_trainer_mcmc_refine(params, exp_avg, exp_avg_sq, sh_degree: int, count: int, cap_max: int,
                            min_opacity: float, seed: int, n_refines: int) -> dict:
    """The reference's own Trainer::mcmc_refine on its CPU backend, n_refines times (in place on
    six [cap_max, dims] float32 arrays per set)."""
    ptrs = [(C.c_void_p * 6)(*[a.ctypes.data for a in arrs]) for arrs in (params, exp_avg, exp_avg_sq)]
    stats = np.zeros(3 * n_refines, np.int64)
    cap = int(cap_max) * max(n_refines, 1)
    lists = [np.zeros(cap, np.int64) for _ in range(3)]
    rc = ref_lib().sxr_trainer_mcmc_refine(ptrs[0], ptrs[1], ptrs[2], I32(sh_degree), I64(count),
                                           I64(cap_max), F32(min_opacity), C.c_uint64(int(seed)),
                                           I32(n_refines), _p(stats), _p(lists[0]), _p(lists[1]),
                                           _p(lists[2]), I64(cap))
    if rc != 0:
        raise ValueError(ref_lib().sxr_last_error().decode())
    st = stats.reshape(n_refines, 3)
    nd, na = int(st[:, 1].sum()), int(st[:, 2].sum())
    return {"stats": st, "relocated_dead": lists[0][:nd], "relocation_src": lists[1][:nd],
            "added_src": lists[2][:na]}


def make_binoms_lut(n_max=51):
    lut = np.zeros(n_max * n_max, np.float32)
    lib().sxo_make_binoms_lut(I32(n_max), _p(lut))
    return lut


class _StepConfig(C.Structure):
    _fields_ = [("sh_degree", C.c_int32), ("degrees_to_use", C.c_uint32), ("lr", C.c_float * 6),
                ("b1", C.c_float), ("b2", C.c_float), ("eps", C.c_float), ("eps2d", C.c_float),
                ("near_plane", C.c_float), ("far_plane", C.c_float), ("radius_clip", C.c_float),
                ("ssim_weight", C.c_float), ("antialiased", C.c_int32), ("opacity_reg", C.c_float),
                ("scale_reg", C.c_float), ("inject_noise", C.c_int32), ("noise_seed", C.c_uint64),
                ("noise_offset", C.c_uint64), ("noise_scale", C.c_float), ("forward_only", C.c_int32)]


def host_step(params, cam, gt, sh_degree, degrees_to_use=None, lr=(0,) * 6, exp_avg=None,
              exp_avg_sq=None, ssim_weight=0.2, antialiased=False, opacity_reg=0.0, scale_reg=0.0,
              inject_noise=False, noise_seed=0, noise_offset=0, noise_scale=0.0,
              forward_only=False, want_render=False, b1=0.9, b2=0.999, eps=1e-15):
    """One Trainer::step host round trip on the CPU (in place on params / moments when given)."""
    n = params[0].shape[0] if params[0].ndim == 2 else params[0].size // 3
    if exp_avg is None:
        exp_avg = [np.zeros_like(p) for p in params]
    if exp_avg_sq is None:
        exp_avg_sq = [np.zeros_like(p) for p in params]
    arr = lambda xs: (C.c_void_p * 6)(*[x.ctypes.data if x.size else None for x in xs])
    cfg = _StepConfig(sh_degree, degrees_to_use if degrees_to_use is not None else sh_degree,
                      (C.c_float * 6)(*lr), b1, b2, eps, 0.3, 0.01, 1e10, 0.0, ssim_weight,
                      int(antialiased), opacity_reg, scale_reg, int(inject_noise), noise_seed,
                      noise_offset, noise_scale, int(forward_only))
    loss, nis = C.c_float(), C.c_int64()
    render = np.zeros(cam.width * cam.height * 3, np.float32) if want_render else None
    gt_a = _c(gt) if gt is not None else None
    rc = lib().sxo_train_step(arr(params), arr(exp_avg), arr(exp_avg_sq), I64(n), _p(_c(cam.viewmat)),
                              _p(_c(cam.K)), I32(cam.width), I32(cam.height), _p(gt_a), C.byref(cfg),
                              C.byref(loss), C.byref(nis), _p(render))
    if rc != 0:
        raise ValueError("oracle host_step: contract violation")
    return {"loss": float(loss.value), "n_isects": int(nis.value), "render": render}


def train_activations(log_scales, logits):
    """(exp(log-scales), sigmoid(logits)) with the float expf of Trainer::step's host path."""
    ls, lg = _c(log_scales), _c(logits)
    n = lg.size
    s = np.zeros(n * 3, np.float32)
    o = np.zeros(n, np.float32)
    lib().sxo_train_activations(_p(ls), _p(lg), I64(n), _p(s), _p(o))
    return s, o


def train_loss(render, gt, width, height, ssim_weight=0.2):
    """The host loss of Trainer::step on a given render: (loss, v_render) with v_render the
    gradient with respect to the render (L1 sign term + SSIM term)."""
    r, g = _c(render), _c(gt)
    v = np.zeros(int(width) * int(height) * 3, np.float32)
    loss = lib().sxo_train_loss(_p(r), _p(g), I32(height), I32(width), F32(ssim_weight), _p(v))
    return float(loss), v


def host_mcmc_trajectory(P, M, V, count, cams, gts, cfg, sh_degree, iters, view_order):
    """The reference trainer's host loop with MCMC (Trainer::step host path + mcmc_refine +
    mcmc_inject_noise, Trainer.cpp:1100-1131 and :1273-1420) on the C oracle, in place on the
    [cap, dims] arenas P / M / V. ``cfg`` is a splatx_cuda.trainer.TrainConfig (schedules only);
    returns the alive count after ``iters`` iterations and the per-iteration losses."""
    from splatx_cuda.mcmc import means_lr_at, noise_scale_at, refine_due
    from splatx_cuda.trainer import sh_degree_at
    m = cfg.mcmc
    g = McmcOracle(m.seed)
    ob = OracleBackend()
    losses = []
    for it in range(iters):
        v = view_order[it % len(view_order)]
        n = count
        refine = m.enabled and refine_due(m, it, cfg.total_iters)
        ns = noise_scale_at(m, cfg.lr_means, cfg.scene_scale, it, cfg.total_iters) if m.enabled else 0.0
        lr = [means_lr_at(cfg.lr_means, cfg.scene_scale, it, cfg.total_iters), cfg.lr_quats,
              cfg.lr_scales, cfg.lr_opacities, cfg.lr_sh0, cfg.lr_shN]
        r = host_step([x[:n] for x in P], cams[v], gts[v], sh_degree,
                      degrees_to_use=sh_degree_at(cfg, it, sh_degree), lr=lr,
                      exp_avg=[x[:n] for x in M], exp_avg_sq=[x[:n] for x in V],
                      ssim_weight=cfg.ssim_weight, opacity_reg=cfg.opacity_reg,
                      scale_reg=cfg.scale_reg, inject_noise=m.enabled and not refine,
                      noise_seed=m.seed, noise_offset=it, noise_scale=ns)
        losses.append(r["loss"])
        if refine:
            count = g.refine(P, M, V, n, m.cap_max, m.min_opacity)["count"]
            noise = ob.rng_normal_f32(m.seed, it, count * 3)
            ob.mcmc_perturb_positions(P[0][:count], P[1][:count], P[2][:count], P[3][:count],
                                      noise, ns)
    return count, losses


# ---- the reference's PLY IO, export filter and eval metrics (PlyIO.cpp, Trainer.cpp) ----
def _ref_cloud_ptrs(c):
    return [c[f].ctypes.data_as(C.c_void_p) for f in ("means", "scales", "quats", "opacities", "sh0", "shN")]


def ref_ply_write(c, path, pad_sh_full=True):
    L = ref_lib()
    rc = L.sxr_ply_write(I64(c["count"]), I32(c["sh_degree"]), *_ref_cloud_ptrs(c),
                         str(path).encode(), I32(int(bool(pad_sh_full))))
    if rc != 0:
        raise ValueError(L.sxr_last_error().decode())


def ref_ply_read(path):
    from splatx_cuda.io import empty_cloud
    L = ref_lib()
    n, d = C.c_int64(), C.c_int32()
    if L.sxr_ply_info(str(path).encode(), C.byref(n), C.byref(d)) != 0:
        raise ValueError(L.sxr_last_error().decode())
    c = empty_cloud(n.value, d.value)
    if L.sxr_ply_read(str(path).encode(), *_ref_cloud_ptrs(c)) != 0:
        raise ValueError(L.sxr_last_error().decode())
    return c


def ref_filter_for_export(c, min_opacity=0.005):
    L = ref_lib()
    w = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in c.items()}
    st = np.zeros(4, np.int64)
    if L.sxr_filter_for_export(I64(w["count"]), I32(w["sh_degree"]), *_ref_cloud_ptrs(w),
                               F32(min_opacity), _p(st)) != 0:
        raise ValueError(L.sxr_last_error().decode())
    k = int(st[3])
    out = {"count": k, "sh_degree": w["sh_degree"]}
    for f in ("means", "scales", "quats", "opacities", "sh0", "shN"):
        out[f] = np.ascontiguousarray(w[f][:k])
    return out, {"input": int(st[0]), "removed_nonfinite": int(st[1]),
                 "removed_low_opacity": int(st[2]), "kept": int(st[3])}


def ref_psnr(a, b):
    L = ref_lib()
    a, b = _c(a), _c(b)
    out = C.c_float()
    if L.sxr_psnr(_p(a), _p(b), I64(a.size), C.byref(out)) != 0:
        raise ValueError(L.sxr_last_error().decode())
    return float(out.value)


def ref_color_correct(img, ref):
    L = ref_lib()
    img, ref = _c(img), _c(ref)
    out = np.zeros_like(img)
    if L.sxr_color_correct(_p(img), _p(ref), I64(img.size), _p(out)) != 0:
        raise ValueError(L.sxr_last_error().decode())
    return out


def eval_metrics(render, gt, H, W):
    """The reference's eval of one view (TrainC.cpp:653-696) restated in numpy (double sums) with
    the oracle's SSIM: (psnr, cc_psnr, ssim, cc_ssim) of the clamped render."""
    r = np.clip(np.asarray(render, np.float32).reshape(-1), 0.0, 1.0)
    g = np.asarray(gt, np.float32).reshape(-1)

    def psnr(a, b):
        mse = float(np.sum((a.astype(np.float64) - b.astype(np.float64)) ** 2)) / a.size
        return float(np.float32(10.0 * np.log10(1.0 / mse))) if mse > 0 else float("inf")

    n_px = r.size // 3
    cc = np.empty_like(r)
    for c in range(3):
        rc, mc = g[c::3].astype(np.float64), r[c::3].astype(np.float64)
        ref_mean, img_mean = rc.sum() / n_px, mc.sum() / n_px
        var_ref = max((rc * rc).sum() / n_px - ref_mean * ref_mean, 1e-8)
        a = ((rc * mc).sum() / n_px - ref_mean * img_mean) / var_ref
        b = img_mean - a * ref_mean
        if abs(a) < 1e-8:
            a = 1.0
        cc[c::3] = np.clip((mc - b) / a, 0.0, 1.0).astype(np.float32)
    ob = OracleBackend()
    s1 = ob.ssim_fwd(r, g, 1, H, W).ssim if H >= 11 and W >= 11 else float("nan")
    s2 = ob.ssim_fwd(cc, g, 1, H, W).ssim if H >= 11 and W >= 11 else float("nan")
    return psnr(r, g), psnr(cc, g), s1, s2


# ---- the reference's SXCK checkpoint files (Checkpoint.cpp) ----
def _ck_arrays(cfg):
    ci = np.array([cfg.get("sh_degree", 3), cfg.get("factor", 0), cfg.get("test_split", 0),
                   cfg.get("total_iters", 0), cfg.get("mcmc_enabled", 0), cfg.get("antialiased", 0)],
                  np.int32)
    cl = np.array([cfg.get("cap_max", 0), np.int64(np.uint64(cfg.get("mcmc_seed", 0)))], np.int64)
    cf = np.array([cfg.get("scene_scale", 1.0), cfg.get("ssim_weight", 0.0)], np.float32)
    return ci, cl, cf


def ref_checkpoint_save(cfg, it, P, M, V, path, fp16=False, rng=""):
    L = ref_lib()
    ci, cl, cf = _ck_arrays(cfg)
    arr = lambda xs: (C.c_void_p * 6)(*[x.ctypes.data for x in xs])
    n = P[0].shape[0]
    rc = L.sxr_checkpoint_save(_p(ci), _p(cl), _p(cf), I32(it), I64(n), arr(P), arr(M), arr(V),
                               rng.encode(), str(path).encode(), I32(int(bool(fp16))))
    if rc != 0:
        raise ValueError(L.sxr_last_error().decode())


def ref_checkpoint_load(path, dims):
    L = ref_lib()
    ci, cl, cf = np.zeros(6, np.int32), np.zeros(2, np.int64), np.zeros(2, np.float32)
    it, n, rl = C.c_int32(), C.c_int64(), C.c_int64()
    if L.sxr_checkpoint_load(str(path).encode(), _p(ci), _p(cl), _p(cf), C.byref(it), C.byref(n),
                             None, None, None, None, I64(0), C.byref(rl)) != 0:
        raise ValueError(L.sxr_last_error().decode())
    P = [np.zeros((n.value, d), np.float32) for d in dims]
    M = [np.zeros_like(x) for x in P]
    V = [np.zeros_like(x) for x in P]
    rng = C.create_string_buffer(rl.value + 1)
    arr = lambda xs: (C.c_void_p * 6)(*[x.ctypes.data for x in xs])
    if L.sxr_checkpoint_load(str(path).encode(), _p(ci), _p(cl), _p(cf), C.byref(it), C.byref(n),
                             arr(P), arr(M), arr(V), rng, I64(rl.value + 1), C.byref(rl)) != 0:
        raise ValueError(L.sxr_last_error().decode())
    cfg = {"sh_degree": int(ci[0]), "factor": int(ci[1]), "test_split": int(ci[2]),
           "total_iters": int(ci[3]), "mcmc_enabled": int(ci[4]), "antialiased": int(ci[5]),
           "cap_max": int(cl[0]), "mcmc_seed": int(np.uint64(cl[1])), "scene_scale": float(cf[0]),
           "ssim_weight": float(cf[1])}
    return {"config": cfg, "iter": it.value, "count": n.value, "P": P, "M": M, "V": V,
            "rng": rng.raw[:rl.value].decode()}


def ref_checkpoint_verify(saved, current):
    L = ref_lib()
    a, b = _ck_arrays(saved), _ck_arrays(current)
    if L.sxr_checkpoint_verify(*[_p(x) for x in a], *[_p(x) for x in b]) != 0:
        raise ValueError(L.sxr_last_error().decode())


def ref_spz_write(c, path, min_opacity=0.005, antialiased=False):
    L = ref_lib()
    st = np.zeros(4, np.int64)
    if L.sxr_spz_write(I64(c["count"]), I32(c["sh_degree"]), *_ref_cloud_ptrs(c), str(path).encode(),
                       F32(min_opacity), I32(int(bool(antialiased))), _p(st)) != 0:
        raise ValueError(L.sxr_last_error().decode())
    return {"input": int(st[0]), "removed_nonfinite": int(st[1]),
            "removed_low_opacity": int(st[2]), "kept": int(st[3])}


def ref_spz_read(path):
    from splatx_cuda.io import empty_cloud
    L = ref_lib()
    n, d, aa = C.c_int64(), C.c_int32(), C.c_int32()
    if L.sxr_spz_info(str(path).encode(), C.byref(n), C.byref(d), C.byref(aa)) != 0:
        raise ValueError(L.sxr_last_error().decode())
    c = empty_cloud(n.value, d.value)
    if L.sxr_spz_read(str(path).encode(), *_ref_cloud_ptrs(c)) != 0:
        raise ValueError(L.sxr_last_error().decode())
    c["antialiased"] = bool(aa.value)
    return c
