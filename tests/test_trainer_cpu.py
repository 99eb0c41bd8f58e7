"""The resident trainer's host arithmetic against the reference's own Trainer.cpp functions
(oracle/_ref): means_lr_at, sh_degree_at, scene_scale_from_cameras and init_splats, bit for bit."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import oracle
from splatx_cuda.mcmc import means_lr_at
from splatx_cuda.scene import ring_camera
from splatx_cuda.trainer import TrainConfig, init_splats, scene_scale_from_cameras, sh_degree_at


@pytest.fixture(scope="module")
def ref():
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built here")
    L = oracle.ref_lib()
    L.sxr_means_lr_at.restype = C.c_float
    L.sxr_means_lr_at.argtypes = [C.c_int, C.c_float, C.c_float, C.c_int]
    L.sxr_sh_degree_at.restype = C.c_uint32
    L.sxr_sh_degree_at.argtypes = [C.c_int, C.c_float, C.c_int, C.c_int]
    L.sxr_scene_scale.restype = C.c_float
    L.sxr_scene_scale.argtypes = [C.c_void_p, C.c_int64]
    return L


def test_schedules_match_reference(ref):
    for total in (300, 7000, 30000):
        for it in (0, 1, 17, total // 3, total - 1, total):
            for scale in (1.0, 11.37):
                assert means_lr_at(1.6e-4, scale, it, total) == ref.sxr_means_lr_at(total, 1.6e-4, scale, it)
            cfg = TrainConfig(total_iters=total)
            for deg in (0, 1, 3):
                assert sh_degree_at(cfg, it, deg) == ref.sxr_sh_degree_at(total, cfg.sh_degree_interval_ratio, it, deg)


def test_scene_scale_matches_reference(ref):
    for n in (1, 2, 37, 185):
        vms = np.stack([ring_camera(i, n, seed=3).viewmat for i in range(n)]).astype(np.float32)
        assert scene_scale_from_cameras(list(vms)) == ref.sxr_scene_scale(vms.ctypes.data, n)


@pytest.mark.parametrize("M,N", [(5000, 5000), (20000, 3000), (2, 2), (1, 1)])
def test_init_splats_matches_reference(ref, M, N):
    rng = np.random.default_rng(M + N)
    pts = rng.normal(0, 2, (M, 3)).astype(np.float32)
    if M > 10:
        pts[5] = pts[4]  # a duplicate point: a zero distance
    rgb = rng.integers(0, 256, (M, 3), dtype=np.uint8)
    ours = init_splats(pts, rgb, N, 0.5, 0.1, 3)
    n = ours[0].shape[0]
    out = [np.zeros((n, 3), np.float32), np.zeros((n, 3), np.float32), np.zeros((n, 4), np.float32),
           np.zeros(n, np.float32), np.zeros((n, 3), np.float32), np.zeros((n, 45), np.float32)]
    rc = ref.sxr_init_splats(pts.ctypes.data_as(C.c_void_p), rgb.ctypes.data_as(C.c_void_p),
                             C.c_int64(M), C.c_int64(N), C.c_float(0.5), C.c_float(0.1), C.c_int(3),
                             *[o.ctypes.data_as(C.c_void_p) for o in out])
    assert rc == 0
    means, scales, quats, op, sh0, shN = out
    for a, b, f in ((ours[0], means, "means"), (ours[1], quats, "quats"), (ours[2], scales, "scales"),
                    (ours[3].ravel(), op, "opacities"), (ours[4], sh0, "sh0"), (ours[5], shN, "shN")):
        assert np.array_equal(np.asarray(a, np.float32).view(np.uint32), b.view(np.uint32)), f
