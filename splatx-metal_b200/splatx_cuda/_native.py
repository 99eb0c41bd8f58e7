"""ctypes bindings of include/splatx_cuda.h (the C-ABI of libsplatx_cuda.so).

Loading fails loudly when the shared library is missing — there is no CPU fallback. Error codes
map to the reference's exception types: SXCUDA_EINVAL -> ValueError (std::invalid_argument),
SXCUDA_ERUNTIME -> RuntimeError (std::runtime_error).
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib

from .build import lib_path as _lib_path

SXCUDA_OK, SXCUDA_EINVAL, SXCUDA_ERUNTIME = 0, 1, 2

c_float_p = C.POINTER(C.c_float)
c_int32_p = C.POINTER(C.c_int32)
c_int64_p = C.POINTER(C.c_int64)
c_uint32_p = C.POINTER(C.c_uint32)
c_uint64_p = C.POINTER(C.c_uint64)
c_uint8_p = C.POINTER(C.c_uint8)
c_double_p = C.POINTER(C.c_double)
c_size_p = C.POINTER(C.c_size_t)
vp = C.c_void_p


class SxTrainStepExecutorDesc(C.Structure):
    _fields_ = [("arena_rows", C.c_int64), ("sh_degree", C.c_int32), ("eps2d", C.c_float),
                ("near_plane", C.c_float), ("far_plane", C.c_float), ("radius_clip", C.c_float),
                ("b1", C.c_float), ("b2", C.c_float), ("eps", C.c_float),
                ("ssim_weight", C.c_float), ("antialiased", C.c_int32)]


class SxResidentParamSync(C.Structure):
    _fields_ = [("params", vp * 6), ("exp_avg", vp * 6), ("exp_avg_sq", vp * 6),
                ("rows", C.c_int64)]


class SxResidentStepInputs(C.Structure):
    _fields_ = [("viewmat", vp), ("K", vp), ("width", C.c_int32), ("height", C.c_int32),
                ("gt_rgb", vp), ("count", C.c_int64), ("degrees_to_use", C.c_uint32),
                ("lr", C.c_float * 6), ("opacity_reg_w", C.c_float), ("scale_reg_w", C.c_float),
                ("forward_only", C.c_int32), ("want_render", C.c_int32),
                ("inject_noise", C.c_int32), ("noise_seed", C.c_uint64),
                ("noise_offset", C.c_uint64), ("noise_scale", C.c_float),
                ("gt_on_device", C.c_int32)]


class SxResidentStepOutputs(C.Structure):
    _fields_ = [("loss", C.c_float), ("n_isects", C.c_int64), ("render_colors", vp)]


class SxApplyGradsInputs(C.Structure):
    _fields_ = [("row_begin", C.c_int64), ("row_end", C.c_int64), ("count", C.c_int64),
                ("n_views", C.c_int32), ("lr", C.c_float * 6), ("opacity_reg_w", C.c_float),
                ("scale_reg_w", C.c_float), ("inject_noise", C.c_int32),
                ("noise_seed", C.c_uint64), ("noise_offset", C.c_uint64),
                ("noise_scale", C.c_float)]


class SxResidentBuffers(C.Structure):
    _fields_ = [("params", vp * 6), ("grads", vp * 6), ("visibility", vp),
                ("dims", C.c_int64 * 6), ("padded_rows", C.c_int64)]


class SxExecutorGaussianTrace(C.Structure):
    _fields_ = [("valid", vp), ("means2d", vp), ("conics", vp), ("opacities", vp), ("colors", vp),
                ("tiles_per_gauss", vp), ("depth_keys", vp), ("depth_order", vp)]


class SxAdamInputs(C.Structure):
    _fields_ = [("param", vp), ("grad", vp), ("exp_avg", vp), ("exp_avg_sq", vp), ("valid", vp),
                ("n_elems", C.c_int64), ("n_gauss", C.c_int64), ("lr", C.c_float),
                ("b1", C.c_float), ("b2", C.c_float), ("eps", C.c_float)]


class SxProjectionFusedInputs(C.Structure):
    _fields_ = [("means", vp), ("covars", vp), ("quats", vp), ("scales", vp), ("opacities", vp),
                ("viewmats", vp), ("Ks", vp), ("N", C.c_int64), ("C", C.c_int64),
                ("width", C.c_int32), ("height", C.c_int32), ("eps2d", C.c_float),
                ("near_plane", C.c_float), ("far_plane", C.c_float), ("radius_clip", C.c_float),
                ("camera_model", C.c_uint32), ("calc_compensations", C.c_int32)]


class SxProjectionFusedOutputs(C.Structure):
    _fields_ = [("radii", vp), ("means2d", vp), ("depths", vp), ("conics", vp),
                ("compensations", vp)]


class SxProjectionFusedGradsIn(C.Structure):
    _fields_ = [("radii", vp), ("conics", vp), ("compensations", vp), ("v_means2d", vp),
                ("v_depths", vp), ("v_conics", vp), ("v_compensations", vp),
                ("viewmats_grad", C.c_int32)]


class SxProjectionFusedGrads(C.Structure):
    _fields_ = [("v_means", vp), ("v_covars", vp), ("v_quats", vp), ("v_scales", vp),
                ("v_viewmats", vp)]


class SxShInputs(C.Structure):
    _fields_ = [("dirs", vp), ("coeffs", vp), ("masks", vp), ("degrees_to_use", C.c_uint32),
                ("B", C.c_int64), ("N", C.c_int64), ("K", C.c_int64), ("D", C.c_uint32),
                ("compute_v_dirs", C.c_int32)]


class SxIsectTilesInputs(C.Structure):
    _fields_ = [("means2d", vp), ("radii", vp), ("depths", vp), ("conics", vp), ("opacities", vp),
                ("I", C.c_int64), ("N", C.c_int64), ("tile_size", C.c_uint32),
                ("tile_width", C.c_uint32), ("tile_height", C.c_uint32)]


class SxRasterizeFwdInputs(C.Structure):
    _fields_ = [("means2d", vp), ("conics", vp), ("colors", vp), ("opacities", vp),
                ("backgrounds", vp), ("masks", vp), ("isect_offsets", vp), ("flatten_ids", vp),
                ("I", C.c_int64), ("N", C.c_int64), ("n_isects", C.c_int64),
                ("image_width", C.c_uint32), ("image_height", C.c_uint32),
                ("tile_size", C.c_uint32), ("tile_width", C.c_uint32),
                ("tile_height", C.c_uint32)]


class SxRasterizeBwdGradsIn(C.Structure):
    _fields_ = [("render_alphas", vp), ("last_ids", vp), ("v_render_colors", vp),
                ("v_render_alphas", vp), ("absgrad", C.c_int32)]


class SxRasterizeBwdGrads(C.Structure):
    _fields_ = [("v_means2d", vp), ("v_conics", vp), ("v_colors", vp), ("v_opacities", vp),
                ("v_means2d_abs", vp)]


class SxEvalResult(C.Structure):
    _fields_ = [("psnr", C.c_double), ("cc_psnr", C.c_double), ("ssim", C.c_double),
                ("cc_ssim", C.c_double)]


class SxCloud(C.Structure):
    _fields_ = [("count", C.c_int64), ("sh_degree", C.c_int32), ("means", vp), ("scales", vp),
                ("quats", vp), ("opacities", vp), ("sh0", vp), ("shN", vp)]


class SxExportFilterStats(C.Structure):
    _fields_ = [("input", C.c_int64), ("removed_nonfinite", C.c_int64),
                ("removed_low_opacity", C.c_int64), ("kept", C.c_int64)]


class SxRenderSessionArgs(C.Structure):
    _fields_ = [("ply_path", C.c_char_p), ("antialiased", C.c_int32), ("sh_degree", C.c_int32),
                ("device", C.c_int32)]


class SxCheckpointConfig(C.Structure):
    _fields_ = [("sh_degree", C.c_int32), ("factor", C.c_int32), ("test_split", C.c_int32),
                ("total_iters", C.c_int32), ("mcmc_enabled", C.c_uint8), ("antialiased", C.c_uint8),
                ("cap_max", C.c_int64), ("mcmc_seed", C.c_uint64), ("scene_scale", C.c_float),
                ("ssim_weight", C.c_float)]


class SxCheckpointHeader(C.Structure):
    _fields_ = [("config", SxCheckpointConfig), ("iter", C.c_int32), ("alive_count", C.c_int64),
                ("fp16", C.c_int32), ("version", C.c_uint32)]


class SxPeerHandles(C.Structure):
    _fields_ = [("handle", (C.c_ubyte * 64) * 14), ("padded_rows", C.c_int64),
                ("sh_degree", C.c_int32), ("barrier_epoch", C.c_uint32)]


class SxMcmcRefineInputs(C.Structure):
    _fields_ = [("count", C.c_int64), ("cap_max", C.c_int64), ("min_opacity", C.c_float)]


class SxMcmcRefineResult(C.Structure):
    _fields_ = [("count", C.c_int64), ("n_relocated", C.c_int64), ("n_added", C.c_int64),
                ("relocated_dead", vp), ("relocation_src", vp), ("added_src", vp),
                ("list_capacity", C.c_int64)]


class SxRelocationInputs(C.Structure):
    _fields_ = [("opacities", vp), ("scales", vp), ("ratios", vp), ("binoms", vp),
                ("N", C.c_int64), ("n_max", C.c_int32), ("min_opacity", C.c_float)]


class SxPerturbInputs(C.Structure):
    _fields_ = [("positions", vp), ("quats", vp), ("scales_log", vp), ("opacities_logit", vp),
                ("noise", vp), ("N", C.c_int64), ("noise_scale", C.c_float), ("t", C.c_float),
                ("k", C.c_float)]


class SxSsimInputs(C.Structure):
    _fields_ = [("img1", vp), ("img2", vp), ("I", C.c_int64), ("H", C.c_int64), ("W", C.c_int64),
                ("C", C.c_int64), ("need_coeffs", C.c_int32)]


class SxSsimGradsIn(C.Structure):
    _fields_ = [("coeff_mu", vp), ("coeff_sigma", vp), ("coeff_cross", vp), ("v_loss", C.c_float)]


P = C.POINTER
_SIGNATURES = {
    "sxcuda_last_error": (C.c_char_p, []),
    "sxcuda_abi_version": (C.c_int32, []),
    "sxcuda_bits_for_count": (C.c_uint32, [C.c_int64]),
    "sxcuda_make_binoms_lut": (C.c_int32, [C.c_int32, vp]),
    "sxcuda_executor_create": (C.c_int32, [P(SxTrainStepExecutorDesc), C.c_int32, P(vp)]),
    "sxcuda_executor_destroy": (None, [vp]),
    "sxcuda_executor_upload_params": (C.c_int32, [vp, P(SxResidentParamSync)]),
    "sxcuda_executor_download_params": (C.c_int32, [vp, P(SxResidentParamSync)]),
    "sxcuda_executor_step": (C.c_int32, [vp, P(SxResidentStepInputs), P(SxResidentStepOutputs)]),
    "sxcuda_executor_step_async": (C.c_int32, [vp, P(SxResidentStepInputs)]),
    "sxcuda_executor_step_accumulate": (C.c_int32, [vp, P(SxResidentStepInputs)]),
    "sxcuda_executor_apply_grads": (C.c_int32, [vp, P(SxApplyGradsInputs)]),
    "sxcuda_executor_clear_grads": (C.c_int32, [vp]),
    "sxcuda_executor_resident_buffers": (C.c_int32, [vp, P(SxResidentBuffers)]),
    "sxcuda_executor_read_gaussians": (C.c_int32, [vp, P(SxExecutorGaussianTrace), c_int64_p]),
    "sxcuda_executor_read_isects": (C.c_int32, [vp, vp, C.c_int64, vp, C.c_int64, c_int64_p,
                                                c_int64_p]),
    "sxcuda_executor_read_images": (C.c_int32, [vp, vp, vp, vp, vp]),
    "sxcuda_executor_peer_handles": (C.c_int32, [vp, P(SxPeerHandles)]),
    "sxcuda_colmap_open": (C.c_int32, [C.c_char_p, C.c_char_p, P(vp)]),
    "sxcuda_colmap_close": (None, [vp]),
    "sxcuda_colmap_counts": (C.c_int32, [vp, c_int64_p, c_int64_p]),
    "sxcuda_colmap_cameras": (C.c_int32, [vp, vp, vp, vp, vp]),
    "sxcuda_colmap_image_path": (C.c_int32, [vp, C.c_int64, C.c_char_p, C.c_int64, c_int64_p]),
    "sxcuda_colmap_seed": (C.c_int32, [vp, vp, vp]),
    "sxcuda_checkpoint_verify_config": (C.c_int32, [P(SxCheckpointConfig), P(SxCheckpointConfig)]),
    "sxcuda_checkpoint_info": (C.c_int32, [C.c_char_p, P(SxCheckpointHeader)]),
    "sxcuda_executor_save_checkpoint": (C.c_int32, [vp, P(SxCheckpointConfig), C.c_int32, C.c_int64,
                                                    C.c_char_p, C.c_int32]),
    "sxcuda_executor_load_checkpoint": (C.c_int32, [vp, C.c_char_p, P(SxCheckpointConfig),
                                                    P(SxCheckpointHeader)]),
    "sxcuda_executor_eval_view": (C.c_int32, [vp, P(SxResidentStepInputs), P(SxEvalResult)]),
    "sxcuda_executor_render_rgba8": (C.c_int32, [vp, P(SxResidentStepInputs), vp]),
    "sxcuda_executor_export_ply": (C.c_int32, [vp, C.c_int64, C.c_char_p, C.c_float, C.c_int32,
                                               P(SxExportFilterStats)]),
    "sxcuda_ply_write": (C.c_int32, [P(SxCloud), C.c_char_p, C.c_int32]),
    "sxcuda_spz_write": (C.c_int32, [P(SxCloud), C.c_char_p, C.c_float, C.c_int32, P(SxExportFilterStats)]),
    "sxcuda_spz_info": (C.c_int32, [C.c_char_p, c_int64_p, c_int32_p, c_int32_p]),
    "sxcuda_spz_read": (C.c_int32, [C.c_char_p, P(SxCloud)]),
    "sxcuda_executor_export_spz": (C.c_int32, [vp, C.c_int64, C.c_char_p, C.c_float, C.c_int32,
                                               P(SxExportFilterStats)]),
    "sxcuda_ply_info": (C.c_int32, [C.c_char_p, c_int64_p, c_int32_p]),
    "sxcuda_ply_read": (C.c_int32, [C.c_char_p, P(SxCloud)]),
    "sxcuda_filter_for_export": (C.c_int32, [P(SxCloud), C.c_float, vp, P(SxExportFilterStats)]),
    "sxcuda_render_session_open": (vp, [P(SxRenderSessionArgs), C.c_char_p, C.c_int32]),
    "sxcuda_render_session_frame": (C.c_int32, [vp, vp, C.c_float, C.c_float, C.c_float, C.c_float,
                                                C.c_int32, C.c_int32, vp, C.c_char_p, C.c_int32]),
    "sxcuda_render_session_close": (None, [vp]),
    "sxcuda_executor_open_peers": (C.c_int32, [vp, C.c_int32, C.c_int32, P(SxPeerHandles)]),
    "sxcuda_executor_exchange_apply": (C.c_int32, [vp, P(SxApplyGradsInputs)]),
    "sxcuda_executor_step_exchange": (C.c_int32, [vp, P(SxResidentStepInputs),
                                                  P(SxApplyGradsInputs), C.c_int32]),
    "sxcuda_executor_mcmc_seed": (C.c_int32, [vp, C.c_uint64]),
    "sxcuda_executor_mcmc_rng_state": (C.c_int32, [vp, C.c_char_p, C.c_int64, c_int64_p]),
    "sxcuda_executor_mcmc_set_rng_state": (C.c_int32, [vp, C.c_char_p, C.c_int64]),
    "sxcuda_executor_mcmc_refine": (C.c_int32, [vp, P(SxMcmcRefineInputs), P(SxMcmcRefineResult)]),
    "sxcuda_executor_inject_noise": (C.c_int32, [vp, C.c_int64, C.c_uint64, C.c_uint64, C.c_float]),
    "sxcuda_executor_last_result": (C.c_int32, [vp, c_float_p, c_int64_p, c_int64_p]),
    "sxcuda_executor_reserve_isects": (C.c_int32, [vp, C.c_int64]),
    "sxcuda_executor_stream": (vp, [vp]),
    "sxcuda_executor_last_launch_count": (C.c_int64, [vp]),
    "sxcuda_executor_set_profiling": (C.c_int32, [vp, C.c_int32]),
    "sxcuda_executor_segment_times": (C.c_int32, [vp, C.POINTER(C.c_char_p), c_float_p, C.c_int32, c_int32_p]),
    "sxcuda_executor_exchange_timeline": (C.c_int32, [vp, C.POINTER(C.c_char_p), c_float_p, C.c_int32,
                                                      c_int32_p]),
    "sxcuda_executor_set_pair_counting": (C.c_int32, [vp, C.c_int32]),
    "sxcuda_executor_set_tile_lists": (C.c_int32, [vp, C.c_int32]),
    "sxcuda_executor_bin_stats": (C.c_int32, [vp, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "sxcuda_peer_barrier_selftest": (C.c_int32, [C.c_int32, C.c_int32, C.POINTER(C.c_uint32)]),
    "sxcuda_peer_exchange_selftest": (C.c_int32, [C.c_int32, C.c_int32, C.POINTER(C.c_uint32),
                                                  c_int32_p]),
    "sxcuda_executor_raster_pairs": (C.c_int32, [vp, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "sxcuda_fused_adam": (C.c_int32, [P(SxAdamInputs), vp]),
    "sxcuda_projection_fused_fwd": (C.c_int32, [P(SxProjectionFusedInputs), P(SxProjectionFusedOutputs), vp]),
    "sxcuda_projection_fused_bwd": (C.c_int32, [P(SxProjectionFusedInputs), P(SxProjectionFusedGradsIn),
                                                P(SxProjectionFusedGrads), vp]),
    "sxcuda_sh_fwd": (C.c_int32, [P(SxShInputs), vp, vp]),
    "sxcuda_sh_bwd": (C.c_int32, [P(SxShInputs), vp, vp, vp, vp]),
    "sxcuda_isect_tile_count": (C.c_int32, [P(SxIsectTilesInputs), vp, vp, c_int64_p, vp, c_size_p, vp]),
    "sxcuda_isect_tile_emit": (C.c_int32, [P(SxIsectTilesInputs), vp, vp, vp, vp]),
    "sxcuda_prefix_scan_i64": (C.c_int32, [vp, vp, C.c_int64, vp, c_size_p, vp]),
    "sxcuda_prefix_scan_i64_noalloc": (C.c_int32, [vp, vp, C.c_int64, vp]),
    "sxcuda_sort_isect": (C.c_int32, [vp, vp, vp, vp, C.c_int64, C.c_uint32, vp, c_size_p, vp]),
    "sxcuda_isect_offset_encode": (C.c_int32, [vp, C.c_int64, C.c_int64, C.c_uint32, C.c_uint32, vp, vp]),
    "sxcuda_rasterize_fwd": (C.c_int32, [P(SxRasterizeFwdInputs), vp, vp, vp, vp]),
    "sxcuda_rasterize_bwd": (C.c_int32, [P(SxRasterizeFwdInputs), P(SxRasterizeBwdGradsIn),
                                         P(SxRasterizeBwdGrads), vp]),
    "sxcuda_rng_normal_f32": (C.c_int32, [C.c_uint64, C.c_uint64, C.c_int64, vp, vp]),
    "sxcuda_rng_philox_u32": (C.c_int32, [C.c_uint64, C.c_uint64, C.c_int64, vp, vp]),
    "sxcuda_mcmc_relocation": (C.c_int32, [P(SxRelocationInputs), vp, vp, vp]),
    "sxcuda_mcmc_perturb_positions": (C.c_int32, [P(SxPerturbInputs), vp]),
    "sxcuda_ssim_fwd": (C.c_int32, [P(SxSsimInputs), vp, vp, vp, vp, vp, vp, c_size_p, vp]),
    "sxcuda_ssim_bwd": (C.c_int32, [P(SxSsimInputs), P(SxSsimGradsIn), vp, vp]),
}

_lib = None


def library_path() -> pathlib.Path:
    return pathlib.Path(os.environ.get("SPLATX_CUDA_LIB", str(_lib_path())))


def lib():
    """The loaded libsplatx_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"libsplatx_cuda.so not found at {path}: build it with "
                "`python splatx-metal_b200/splatx_cuda/build.py` (there is no CPU fallback)")
        L = C.CDLL(str(path))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(code: int) -> None:
    """Raise the exception the reference would throw for a non-zero status."""
    if code == SXCUDA_OK:
        return
    msg = lib().sxcuda_last_error().decode(errors="replace")
    if code == SXCUDA_EINVAL:
        raise ValueError(msg)
    raise RuntimeError(msg)


def declared_symbols(header: pathlib.Path | None = None) -> list[str]:
    """Function names declared in include/splatx_cuda.h."""
    import re
    if header is None:
        header = pathlib.Path(__file__).resolve().parents[2] / "include" / "splatx_cuda.h"
    text = header.read_text()
    return sorted(set(re.findall(r"\b(sxcuda_[a-z0-9_]+)\s*\(", text)))
