"""TrainStepExecutor — host mirror of splatx-metal's resident step executor
(``TrainStepExecutor``, ``Sources/SplatXCore/include/splatx/KernelBackend.h:338-392``).

Parameters use the reference's D3 group order: 0 means[3], 1 quats[4], 2 scales[3] (log),
3 opacities[1] (logit), 4 sh0[3], 5 shN[(K-1)*3]. ``upload_params`` / ``download_params`` take six
float32 host arrays of ``rows`` rows each for params, exp_avg and exp_avg_sq; ``step`` takes the
camera and a host ground-truth image and returns ``(loss, n_isects, render_or_None)``.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as _nat
from ._native import check


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, np.float32))


class TrainStepExecutor:
    def __init__(self, arena_rows: int, sh_degree: int = 3, eps2d: float = 0.3,
                 near_plane: float = 0.01, far_plane: float = 1e10, radius_clip: float = 0.0,
                 b1: float = 0.9, b2: float = 0.999, eps: float = 1e-15, ssim_weight: float = 0.2,
                 antialiased: bool = False, device: int = 0):
        self.K = (sh_degree + 1) ** 2
        self.dims = [3, 4, 3, 1, 3, (self.K - 1) * 3]
        self.arena_rows = int(arena_rows)
        desc = _nat.SxTrainStepExecutorDesc(int(arena_rows), int(sh_degree), eps2d, near_plane,
                                            far_plane, radius_clip, b1, b2, eps, ssim_weight,
                                            int(bool(antialiased)))
        h = C.c_void_p()
        check(_nat.lib().sxcuda_executor_create(C.byref(desc), int(device), C.byref(h)))
        self._h = h
        self._keep = []

    def close(self):
        if getattr(self, "_h", None) and self._h.value:
            _nat.lib().sxcuda_executor_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _sync_struct(self, params, exp_avg, exp_avg_sq, rows):
        s = _nat.SxResidentParamSync()
        s.rows = int(rows)
        for g in range(6):
            if self.dims[g] == 0:
                continue
            for field, arrs in (("params", params), ("exp_avg", exp_avg), ("exp_avg_sq", exp_avg_sq)):
                a = arrs[g]
                if a.dtype != np.float32 or not a.flags.c_contiguous:
                    raise ValueError("sync arrays must be C-contiguous float32")
                if a.size < rows * self.dims[g]:
                    raise ValueError(f"group {g}: array holds fewer than rows*{self.dims[g]} floats")
                getattr(s, field)[g] = a.ctypes.data
        return s

    def upload_params(self, params, exp_avg, exp_avg_sq, rows):
        s = self._sync_struct(params, exp_avg, exp_avg_sq, rows)
        check(_nat.lib().sxcuda_executor_upload_params(self._h, C.byref(s)))

    def download_params(self, params, exp_avg, exp_avg_sq, rows):
        s = self._sync_struct(params, exp_avg, exp_avg_sq, rows)
        check(_nat.lib().sxcuda_executor_download_params(self._h, C.byref(s)))

    def _inputs(self, viewmat, K, width, height, gt_ptr, count, degrees_to_use, lr, opacity_reg_w,
                scale_reg_w, forward_only, want_render, inject_noise, noise_seed, noise_offset,
                noise_scale, gt_on_device):
        vm, Km = _f32(viewmat), _f32(K)
        self._keep = [vm, Km]
        lr6 = (C.c_float * 6)(*[float(x) for x in (list(lr) + [0.0] * 6)[:6]])
        return _nat.SxResidentStepInputs(
            vm.ctypes.data, Km.ctypes.data, int(width), int(height), gt_ptr, int(count),
            int(degrees_to_use), lr6, float(opacity_reg_w), float(scale_reg_w), int(bool(forward_only)),
            int(bool(want_render)), int(bool(inject_noise)), int(noise_seed), int(noise_offset),
            float(noise_scale), int(bool(gt_on_device)))

    def step(self, viewmat, K, width, height, gt_rgb=None, count=None, degrees_to_use=0,
             lr=(0,) * 6, opacity_reg_w=0.0, scale_reg_w=0.0, forward_only=False,
             want_render=False, inject_noise=False, noise_seed=0, noise_offset=0, noise_scale=0.0):
        """One synchronous step with a HOST ground-truth image (the reference's contract)."""
        gt = None if gt_rgb is None else _f32(gt_rgb)
        ins = self._inputs(viewmat, K, width, height, None if gt is None else gt.ctypes.data,
                           count if count is not None else self.arena_rows, degrees_to_use, lr,
                           opacity_reg_w, scale_reg_w, forward_only, want_render, inject_noise,
                           noise_seed, noise_offset, noise_scale, False)
        render = np.empty(int(width) * int(height) * 3, np.float32) if want_render else None
        out = _nat.SxResidentStepOutputs(0.0, 0, None if render is None else render.ctypes.data)
        check(_nat.lib().sxcuda_executor_step(self._h, C.byref(ins), C.byref(out)))
        return float(out.loss), int(out.n_isects), render

    def step_async(self, viewmat, K, width, height, gt_device_ptr, count, degrees_to_use=0,
                   lr=(0,) * 6, opacity_reg_w=0.0, scale_reg_w=0.0, inject_noise=False,
                   noise_seed=0, noise_offset=0, noise_scale=0.0):
        """Enqueue one step whose ground truth already lives in device memory."""
        ins = self._inputs(viewmat, K, width, height, int(gt_device_ptr), count, degrees_to_use, lr,
                           opacity_reg_w, scale_reg_w, False, False, inject_noise, noise_seed,
                           noise_offset, noise_scale, True)
        check(_nat.lib().sxcuda_executor_step_async(self._h, C.byref(ins)))

    # ---- view-parallel training (no reference counterpart): accumulate, exchange, apply
    def step_accumulate(self, viewmat, K, width, height, gt_device_ptr, count, degrees_to_use=0):
        """Enqueue forward + backward of one view, adding its gradients to the gradient buffers."""
        ins = self._inputs(viewmat, K, width, height, int(gt_device_ptr), count, degrees_to_use,
                           (0,) * 6, 0.0, 0.0, False, False, False, 0, 0, 0.0, True)
        check(_nat.lib().sxcuda_executor_step_accumulate(self._h, C.byref(ins)))

    def step_accumulate_host(self, viewmat, K, width, height, gt_rgb, count, degrees_to_use=0):
        """As step_accumulate with a HOST ground-truth image (copied on the executor's copy
        stream while the forward runs)."""
        gt = _f32(gt_rgb)
        self._keep_gt = gt
        ins = self._inputs(viewmat, K, width, height, gt.ctypes.data, count, degrees_to_use,
                           (0,) * 6, 0.0, 0.0, False, False, False, 0, 0, 0.0, False)
        check(_nat.lib().sxcuda_executor_step_accumulate(self._h, C.byref(ins)))

    def apply_grads(self, row_begin, row_end, count, n_views, lr, opacity_reg_w=0.0,
                    scale_reg_w=0.0, inject_noise=False, noise_seed=0, noise_offset=0,
                    noise_scale=0.0):
        """Enqueue Adam on rows [row_begin, row_end) from the accumulated gradients."""
        lr6 = (C.c_float * 6)(*[float(x) for x in (list(lr) + [0.0] * 6)[:6]])
        a = _nat.SxApplyGradsInputs(int(row_begin), int(row_end), int(count), int(n_views), lr6,
                                    float(opacity_reg_w), float(scale_reg_w),
                                    int(bool(inject_noise)), int(noise_seed), int(noise_offset),
                                    float(noise_scale))
        check(_nat.lib().sxcuda_executor_apply_grads(self._h, C.byref(a)))

    # ---- evaluation, frames and export ----
    def eval_view(self, viewmat, K, width, height, gt_rgb, count, degrees_to_use=0) -> dict:
        """The training eval of one view (TrainC.cpp:653-696) on the device: psnr, cc_psnr, ssim,
        cc_ssim of the clamped render against ``gt_rgb`` (a host array or a device pointer)."""
        on_dev = isinstance(gt_rgb, int)
        gt = None if on_dev else _f32(gt_rgb)
        ptr = gt_rgb if on_dev else gt.ctypes.data
        ins = self._inputs(viewmat, K, width, height, ptr, count, degrees_to_use, (0,) * 6, 0.0, 0.0,
                           True, False, False, 0, 0, 0.0, on_dev)
        r = _nat.SxEvalResult()
        check(_nat.lib().sxcuda_executor_eval_view(self._h, C.byref(ins), C.byref(r)))
        return {"psnr": r.psnr, "cc_psnr": r.cc_psnr, "ssim": r.ssim, "cc_ssim": r.cc_ssim}

    def render_rgba8(self, viewmat, K, width, height, count, degrees_to_use=0) -> np.ndarray:
        """Forward-only render quantised to RGBA8 on the device: uint8 [H, W, 4]."""
        ins = self._inputs(viewmat, K, width, height, None, count, degrees_to_use, (0,) * 6, 0.0,
                           0.0, True, False, False, 0, 0, 0.0, False)
        out = np.empty((int(height), int(width), 4), np.uint8)
        check(_nat.lib().sxcuda_executor_render_rgba8(self._h, C.byref(ins), out.ctypes.data))
        return out

    def export_ply(self, count, path, min_opacity=0.005, pad_sh_full=True) -> dict:
        """Download rows [0, count), apply the export filter and write an INRIA PLY."""
        st = _nat.SxExportFilterStats()
        check(_nat.lib().sxcuda_executor_export_ply(self._h, int(count), str(path).encode(),
                                                    float(min_opacity), int(bool(pad_sh_full)),
                                                    C.byref(st)))
        return {"input": st.input, "removed_nonfinite": st.removed_nonfinite,
                "removed_low_opacity": st.removed_low_opacity, "kept": st.kept}

    def export_spz(self, count, path, min_opacity=0.005, antialiased=False) -> dict:
        """Download rows [0, count), apply the export filter and write an SPZ v3 file."""
        st = _nat.SxExportFilterStats()
        check(_nat.lib().sxcuda_executor_export_spz(self._h, int(count), str(path).encode(),
                                                    float(min_opacity), int(bool(antialiased)),
                                                    C.byref(st)))
        return {"input": st.input, "removed_nonfinite": st.removed_nonfinite,
                "removed_low_opacity": st.removed_low_opacity, "kept": st.kept}

    # ---- SXCK checkpoints (Checkpoint.h) ----
    def save_checkpoint(self, config: dict, iter: int, count: int, path, fp16: bool = False):
        """save_checkpoint_file of rows [0, count) at step ``iter`` (config: CheckpointConfig)."""
        c = checkpoint_config(config)
        check(_nat.lib().sxcuda_executor_save_checkpoint(self._h, C.byref(c), int(iter), int(count),
                                                         str(path).encode(), int(bool(fp16))))

    def load_checkpoint(self, path, current: dict | None = None) -> dict:
        """load_checkpoint_file into the arena; verifies the fingerprint against ``current``."""
        h = _nat.SxCheckpointHeader()
        cur = checkpoint_config(current) if current is not None else None
        check(_nat.lib().sxcuda_executor_load_checkpoint(self._h, str(path).encode(),
                                                         C.byref(cur) if cur is not None else None,
                                                         C.byref(h)))
        return _header_dict(h)

    # ---- the exchange fused over peer memory (CUDA IPC) ----
    def peer_handles(self) -> bytes:
        """This executor's IPC handles (grads, visibility, params) as bytes to share with peers."""
        h = _nat.SxPeerHandles()
        check(_nat.lib().sxcuda_executor_peer_handles(self._h, C.byref(h)))
        return bytes(h)

    def open_peers(self, rank: int, world: int, handles: list):
        """Map every other rank's buffers (handles[r] from that rank's ``peer_handles``)."""
        arr = (_nat.SxPeerHandles * world)()
        for r, b in enumerate(handles):
            C.memmove(C.byref(arr[r]), b, C.sizeof(_nat.SxPeerHandles))
        check(_nat.lib().sxcuda_executor_open_peers(self._h, int(rank), int(world), arr))

    def exchange_apply(self, row_begin, row_end, count, n_views, lr, opacity_reg_w=0.0,
                       scale_reg_w=0.0, inject_noise=False, noise_seed=0, noise_offset=0,
                       noise_scale=0.0):
        """Enqueue the fused reduce + Adam + broadcast of the owner rows over peer memory."""
        lr6 = (C.c_float * 6)(*[float(x) for x in (list(lr) + [0.0] * 6)[:6]])
        a = _nat.SxApplyGradsInputs(int(row_begin), int(row_end), int(count), int(n_views), lr6,
                                    float(opacity_reg_w), float(scale_reg_w),
                                    int(bool(inject_noise)), int(noise_seed), int(noise_offset),
                                    float(noise_scale))
        check(_nat.lib().sxcuda_executor_exchange_apply(self._h, C.byref(a)))

    def step_exchange(self, viewmat, K, width, height, gt, count, degrees_to_use,
                      row_begin, row_end, n_views, lr, chunks=4, opacity_reg_w=0.0,
                      scale_reg_w=0.0, inject_noise=False, noise_seed=0, noise_offset=0,
                      noise_scale=0.0):
        """The last view of a view-parallel step with the exchange overlapped (after
        ``open_peers``): forward + backward of the view accumulate, the per-Gaussian backward
        runs in ``chunks`` row chunks, and each chunk's owner-row exchange (device barrier over
        peer memory, reduce, Adam, store into every replica) runs on a second stream while the
        next chunk's backward runs; a closing device barrier precedes zeroing the accumulators.
        ``gt``: a device pointer (int) or a host array (copied on the executor's copy stream
        while the forward runs)."""
        on_dev = isinstance(gt, int)
        if not on_dev:
            gt = _f32(gt)
            self._keep_gt = gt
        ins = self._inputs(viewmat, K, width, height, gt if on_dev else gt.ctypes.data, count,
                           degrees_to_use, (0,) * 6, 0.0, 0.0, False, False, False, 0, 0, 0.0,
                           on_dev)
        lr6 = (C.c_float * 6)(*[float(x) for x in (list(lr) + [0.0] * 6)[:6]])
        a = _nat.SxApplyGradsInputs(int(row_begin), int(row_end), int(count), int(n_views), lr6,
                                    float(opacity_reg_w), float(scale_reg_w),
                                    int(bool(inject_noise)), int(noise_seed), int(noise_offset),
                                    float(noise_scale))
        check(_nat.lib().sxcuda_executor_step_exchange(self._h, C.byref(ins), C.byref(a),
                                                       int(chunks)))

    def clear_grads(self):
        check(_nat.lib().sxcuda_executor_clear_grads(self._h))

    def resident_buffers(self) -> dict:
        """Device pointers of the resident arena: params[6], grads[6], visibility, dims, padded."""
        b = _nat.SxResidentBuffers()
        check(_nat.lib().sxcuda_executor_resident_buffers(self._h, C.byref(b)))
        return {"params": [int(b.params[g] or 0) for g in range(6)],
                "grads": [int(b.grads[g] or 0) for g in range(6)],
                "visibility": int(b.visibility or 0), "dims": [int(b.dims[g]) for g in range(6)],
                "padded_rows": int(b.padded_rows)}

    # ---- MCMC refine on the resident arena (Trainer::mcmc_refine, Trainer.cpp:1273-1435) ----
    def mcmc_seed(self, seed: int):
        """Seed the refine's mt19937_64 (Trainer.cpp:713; 42 until called)."""
        check(_nat.lib().sxcuda_executor_mcmc_seed(self._h, int(seed)))

    def mcmc_rng_state(self) -> str:
        """The refine engine's state as ``os << std::mt19937_64`` text (the checkpoint field)."""
        n = C.c_int64()
        check(_nat.lib().sxcuda_executor_mcmc_rng_state(self._h, None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value)
        check(_nat.lib().sxcuda_executor_mcmc_rng_state(self._h, buf, n.value, C.byref(n)))
        return buf.raw[:n.value].decode()

    def set_mcmc_rng_state(self, text: str):
        b = text.encode()
        check(_nat.lib().sxcuda_executor_mcmc_set_rng_state(self._h, b, len(b)))

    def mcmc_refine(self, count: int, cap_max: int, min_opacity: float = 0.005,
                    want_lists: bool = True) -> dict:
        """Relocate the dead rows, then grow to min(cap_max, ceil(1.05 count)); synchronous.

        Returns ``count`` (alive rows afterwards) and, with ``want_lists``, the reference's
        McmcRefineResult lists ``relocated_dead``, ``relocation_src``, ``added_src``."""
        ins = _nat.SxMcmcRefineInputs(int(count), int(cap_max), float(min_opacity))
        res = _nat.SxMcmcRefineResult()
        lists = None
        if want_lists:
            cap = max(int(cap_max), 1)
            lists = [np.zeros(cap, np.int64) for _ in range(3)]
            res.relocated_dead, res.relocation_src, res.added_src = (x.ctypes.data for x in lists)
            res.list_capacity = cap
        check(_nat.lib().sxcuda_executor_mcmc_refine(self._h, C.byref(ins), C.byref(res)))
        out = {"count": int(res.count), "n_relocated": int(res.n_relocated),
               "n_added": int(res.n_added)}
        if lists is not None:
            out["relocated_dead"] = lists[0][:res.n_relocated].copy()
            out["relocation_src"] = lists[1][:res.n_relocated].copy()
            out["added_src"] = lists[2][:res.n_added].copy()
        return out

    def inject_noise(self, count: int, seed: int, offset: int, noise_scale: float):
        """MCMC position noise on rows [0, count) outside a step (asynchronous)."""
        check(_nat.lib().sxcuda_executor_inject_noise(self._h, int(count), int(seed), int(offset),
                                                      float(noise_scale)))

    def last_result(self):
        loss, n, ov = C.c_float(), C.c_int64(), C.c_int64()
        check(_nat.lib().sxcuda_executor_last_result(self._h, C.byref(loss), C.byref(n), C.byref(ov)))
        return float(loss.value), int(n.value), int(ov.value)

    def reserve_isects(self, n: int):
        check(_nat.lib().sxcuda_executor_reserve_isects(self._h, int(n)))

    def stream_handle(self) -> int:
        return int(_nat.lib().sxcuda_executor_stream(self._h) or 0)

    def set_profiling(self, on: bool = True):
        check(_nat.lib().sxcuda_executor_set_profiling(self._h, int(bool(on))))

    def segment_times(self) -> dict:
        """Milliseconds per segment of the last profiled step, in execution order."""
        cap = 32
        names = (C.c_char_p * cap)()
        ms = (C.c_float * cap)()
        n = C.c_int32()
        check(_nat.lib().sxcuda_executor_segment_times(self._h, names, ms, cap, C.byref(n)))
        return {names[i].decode(): float(ms[i]) for i in range(n.value)}

    def set_pair_counting(self, on: bool = True):
        """Count the raster kernels' (pixel, Gaussian) pair evaluations in the following steps."""
        check(_nat.lib().sxcuda_executor_set_pair_counting(self._h, int(bool(on))))

    def set_tile_lists(self, mode: int = 0):
        """0: supertile binning where the tile grid allows (default); 1: the (tile, Gaussian) pair
        sort. Both build the same tile-sorted intersection list."""
        check(_nat.lib().sxcuda_executor_set_tile_lists(self._h, int(mode)))

    def bin_stats(self) -> tuple:
        """(entries, supertiles) of the last step's supertile binning; (0, 0) after a pair sort."""
        e, st = C.c_int64(), C.c_int64()
        check(_nat.lib().sxcuda_executor_bin_stats(self._h, C.byref(e), C.byref(st)))
        return int(e.value), int(st.value)

    def raster_pairs(self) -> tuple:
        """(forward pairs, backward pairs) of the last counted step."""
        f, b = C.c_int64(), C.c_int64()
        check(_nat.lib().sxcuda_executor_raster_pairs(self._h, C.byref(f), C.byref(b)))
        return int(f.value), int(b.value)

    def exchange_timeline(self) -> list:
        """(event, ms from the step's start) of the last profiled step_exchange: the backward
        chunks on the executor's stream, the barriers and exchanges on the exchange stream."""
        cap = 64
        names = (C.c_char_p * cap)()
        ms = (C.c_float * cap)()
        n = C.c_int32()
        check(_nat.lib().sxcuda_executor_exchange_timeline(self._h, names, ms, cap, C.byref(n)))
        return [(names[i].decode(), round(float(ms[i]), 4)) for i in range(n.value)]

    def last_launch_count(self) -> int:
        return int(_nat.lib().sxcuda_executor_last_launch_count(self._h))

    # ---- the last step's intermediate tensors (parity checks against the host path) ----
    def read_gaussians(self) -> dict:
        """Per-Gaussian forward outputs of the last step (valid, means2d, conics, raster opacity,
        colours, AccuTile tile counts, depth keys, depth order) as host arrays."""
        cnt = C.c_int64()
        check(_nat.lib().sxcuda_executor_read_gaussians(self._h, C.byref(_nat.SxExecutorGaussianTrace()),
                                                        C.byref(cnt)))
        n = int(cnt.value)
        out = {"valid": np.zeros(n, np.uint8), "means2d": np.zeros((n, 2), np.float32),
               "conics": np.zeros((n, 3), np.float32), "opacities": np.zeros(n, np.float32),
               "colors": np.zeros((n, 3), np.float32), "tiles_per_gauss": np.zeros(n, np.int32),
               "depth_keys": np.zeros(n, np.uint32), "depth_order": np.zeros(n, np.int32)}
        t = _nat.SxExecutorGaussianTrace(*[out[k].ctypes.data for k in (
            "valid", "means2d", "conics", "opacities", "colors", "tiles_per_gauss", "depth_keys",
            "depth_order")])
        check(_nat.lib().sxcuda_executor_read_gaussians(self._h, C.byref(t), C.byref(cnt)))
        return out

    def read_isects(self) -> dict:
        """The last step's tile-sorted flatten_ids and per-tile start offsets."""
        n, nt = C.c_int64(), C.c_int64()
        lib = _nat.lib()
        lib.sxcuda_executor_read_isects(self._h, None, 0, None, 0, C.byref(n), C.byref(nt))
        ids = np.zeros(max(n.value, 1), np.int32)
        offs = np.zeros(max(nt.value, 1), np.int32)
        check(lib.sxcuda_executor_read_isects(self._h, ids.ctypes.data, ids.size, offs.ctypes.data,
                                              offs.size, C.byref(n), C.byref(nt)))
        return {"n_isects": int(n.value), "flatten_ids": ids[: n.value], "offsets": offs[: nt.value]}

    def read_images(self, width: int, height: int) -> dict:
        """The last step's render [H,W,3], alpha [H,W], last_ids [H,W] and v_render [H,W,3]."""
        hw = int(width) * int(height)
        out = {"render": np.zeros(hw * 3, np.float32), "alpha": np.zeros(hw, np.float32),
               "last_ids": np.zeros(hw, np.int32), "v_render": np.zeros(hw * 3, np.float32)}
        check(_nat.lib().sxcuda_executor_read_images(
            self._h, *[out[k].ctypes.data for k in ("render", "alpha", "last_ids", "v_render")]))
        return out


CHECKPOINT_FIELDS = ("sh_degree", "factor", "test_split", "total_iters", "mcmc_enabled",
                     "antialiased", "cap_max", "mcmc_seed", "scene_scale", "ssim_weight")


def checkpoint_config(d: dict) -> _nat.SxCheckpointConfig:
    """A CheckpointConfig (Checkpoint.h:84-95) from a dict; missing fields take the defaults."""
    base = {"sh_degree": 3, "factor": 0, "test_split": 0, "total_iters": 0, "mcmc_enabled": 0,
            "antialiased": 0, "cap_max": 0, "mcmc_seed": 0, "scene_scale": 1.0, "ssim_weight": 0.0}
    base.update(d or {})
    return _nat.SxCheckpointConfig(*[base[k] for k in CHECKPOINT_FIELDS])


def _header_dict(h) -> dict:
    cfg = {k: getattr(h.config, k) for k in CHECKPOINT_FIELDS}
    return {"config": cfg, "iter": int(h.iter), "alive_count": int(h.alive_count),
            "fp16": bool(h.fp16), "version": int(h.version)}


def checkpoint_info(path) -> dict:
    """load_checkpoint_header (Checkpoint.h:145)."""
    h = _nat.SxCheckpointHeader()
    check(_nat.lib().sxcuda_checkpoint_info(str(path).encode(), C.byref(h)))
    return _header_dict(h)


def verify_checkpoint_config(saved: dict, current: dict):
    """verify_checkpoint_config (Checkpoint.h:127): raises naming the mismatched field."""
    a, b = checkpoint_config(saved), checkpoint_config(current)
    check(_nat.lib().sxcuda_checkpoint_verify_config(C.byref(a), C.byref(b)))
