"""Device evaluation, RGBA frames, PLY export from the resident arena and the render session
(TrainC.cpp:653-696 and :1440-1584, PlyIO.cpp) on the GPU.

Bars: the eval metrics equal the reference's eval arithmetic (numpy restatement pinned to the
reference's psnr / color_correct_affine on the CPU, oracle SSIM) evaluated on the same render,
within 1e-5 relative; frames equal the host quantisation of the float render bit for bit; the
export equals the host filter of the uploaded rows bit for bit; a session renders what the
executor renders for the same cloud."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _scene(n=3000, sh=2, seed=13):
    from splatx_cuda.scene import small_scene
    scene, cam = small_scene(seed=seed, n=n, sh_degree=sh)
    P = [np.ascontiguousarray(g.reshape(n, -1)).copy() for g in scene.groups()]
    return scene, cam, P


def _executor(P, n, sh):
    from splatx_cuda.executor import TrainStepExecutor
    ex = TrainStepExecutor(n, sh)
    Z = [np.zeros_like(x) for x in P]
    ex.upload_params(P, Z, Z, n)
    return ex


def _quantise(rgb):
    v = np.asarray(rgb, np.float32).copy()
    v[~(v > 0)] = 0.0
    v[v > 1] = 1.0
    q = np.rint((v * np.float32(255.0)).astype(np.float32)).astype(np.uint8)
    out = np.full(q.shape[:-1] + (4,), 255, np.uint8)
    out[..., :3] = q
    return out


def test_eval_view_matches_reference_arithmetic():
    import oracle
    scene, cam, P = _scene()
    n, sh = scene.count, scene.sh_degree
    ex = _executor(P, n, sh)
    _, _, render = ex.step(cam.viewmat, cam.K, cam.width, cam.height, None, n, degrees_to_use=sh,
                           forward_only=True, want_render=True)
    gt = np.clip(render * 0.9 + 0.05 + np.random.default_rng(1).normal(0, 0.03, render.size),
                 0, 1).astype(np.float32)
    got = ex.eval_view(cam.viewmat, cam.K, cam.width, cam.height, gt, n, sh)
    want = oracle.eval_metrics(render, gt, cam.height, cam.width)
    for k, w in zip(("psnr", "cc_psnr", "ssim", "cc_ssim"), want):
        assert abs(got[k] - w) <= 1e-5 * abs(w), (k, got[k], w)
    import torch
    gt_dev = torch.from_numpy(gt).cuda()  # a device target gives the same numbers
    got2 = ex.eval_view(cam.viewmat, cam.K, cam.width, cam.height, gt_dev.data_ptr(), n, sh)
    assert got2 == got
    small = ex.eval_view(cam.viewmat, [40, 0, 5, 0, 40, 5, 0, 0, 1], 10, 10,
                         np.zeros(300, np.float32), n, sh)
    assert np.isnan(small["ssim"]) and np.isnan(small["cc_ssim"])  # SSIM needs 11x11
    ex.close()


def test_rgba8_frames_quantise_the_float_render():
    scene, cam, P = _scene(seed=14)
    n, sh = scene.count, scene.sh_degree
    ex = _executor(P, n, sh)
    for (w, h) in ((cam.width, cam.height), (97, 61)):
        K = np.array([300 * w / 256, 0, w / 2, 0, 300 * w / 256, h / 2, 0, 0, 1], np.float32)
        _, _, render = ex.step(cam.viewmat, K, w, h, None, n, degrees_to_use=sh, forward_only=True,
                               want_render=True)
        frame = ex.render_rgba8(cam.viewmat, K, w, h, n, sh)
        assert frame.shape == (h, w, 4)
        assert np.array_equal(frame, _quantise(render.reshape(h, w, 3)))
    ex.close()


def test_export_ply_equals_host_filter(tmp_path):
    from splatx_cuda import io as sio
    scene, cam, P = _scene(seed=15)
    n, sh = scene.count, scene.sh_degree
    P[3][::5, 0] = -7.0  # dead rows
    ex = _executor(P, n, sh)
    st = ex.export_ply(n, tmp_path / "out.ply")
    host, hst = sio.filter_for_export(sio.from_groups(P, sh))
    assert st == hst and st["removed_low_opacity"] >= n // 5
    back = sio.read_ply(tmp_path / "out.ply")  # padded to degree 3 for viewers
    assert back["count"] == host["count"] and back["sh_degree"] == 3
    for f in ("means", "scales", "quats", "opacities", "sh0"):
        assert np.array_equal(back[f], host[f]), f
    K = (sh + 1) ** 2 - 1
    assert np.array_equal(back["shN"][:, :K], host["shN"]) and not back["shN"][:, K:].any()
    ex.close()


def test_render_session_renders_the_executor_frames(tmp_path):
    from splatx_cuda import io as sio
    from splatx_cuda.render import RenderSession
    scene, cam, P = _scene(seed=16, sh=3)
    n = scene.count
    sio.write_ply(sio.from_groups(P, 3), tmp_path / "s.ply", pad_sh_full=False)
    ex = _executor(P, n, 3)
    fx, fy, cx, cy = (float(cam.K[i]) for i in (0, 4, 2, 5))
    with RenderSession(tmp_path / "s.ply") as s:
        f1 = s.frame(cam.viewmat, fx, fy, cx, cy, cam.width, cam.height)
        assert np.array_equal(f1, ex.render_rgba8(cam.viewmat, cam.K, cam.width, cam.height, n, 3))
        f2 = s.frame(cam.viewmat, fx, fy, cx, cy, cam.width, cam.height)
        assert np.array_equal(f1, f2)  # the same camera renders bit-identically
        f3 = s.frame(cam.viewmat, fx / 2, fy / 2, 40, 30, 80, 60)  # another size
        assert f3.shape == (60, 80, 4)
        with pytest.raises(ValueError):
            s.frame(cam.viewmat, -1.0, fy, cx, cy, 64, 64)
        with pytest.raises(ValueError):
            s.frame(cam.viewmat, fx, fy, cx, cy, 0, 64)
    ex.close()
    # a capped SH degree renders the truncated cloud
    Pt = [x.copy() for x in P]
    Pt[5] = np.ascontiguousarray(P[5].reshape(n, 15, 3)[:, :3].reshape(n, 9))
    ext = _executor(Pt, n, 1)
    with RenderSession(tmp_path / "s.ply", sh_degree=1) as s:
        assert np.array_equal(s.frame(cam.viewmat, fx, fy, cx, cy, cam.width, cam.height),
                              ext.render_rgba8(cam.viewmat, cam.K, cam.width, cam.height, n, 1))
    ext.close()
    with pytest.raises(RuntimeError):
        RenderSession(tmp_path / "missing.ply")
    sio.write_ply(sio.from_groups([x[:, :] for x in Pt], 1), tmp_path / "d1.ply", pad_sh_full=False)
    with pytest.raises(RuntimeError, match="exceeds"):
        RenderSession(tmp_path / "d1.ply", sh_degree=2)


def test_images_decode_on_the_device(tmp_path):
    """JPEG decodes on the GPU (nvJPEG) agree with the host decoder within the decoders' IDCT
    differences (a 4:4:4 file: chroma upsampling of subsampled files differs between decoders by
    design); PNG goes through the host decoder exactly; downsampling matches."""
    from PIL import Image
    from splatx_cuda.dataset import load_image, load_image_device
    rng = np.random.default_rng(5)
    a = (np.clip(rng.normal(128, 40, (64, 96, 3)), 0, 255)).astype(np.uint8)
    Image.fromarray(a).save(tmp_path / "a.jpg", quality=95, subsampling=0)
    Image.fromarray(a).save(tmp_path / "a.png")
    d = load_image_device(tmp_path / "a.jpg").cpu().numpy()
    h = load_image(tmp_path / "a.jpg")
    assert d.shape == h.shape == (64, 96, 3)
    assert np.abs(d - h).max() <= 6.0 / 255.0 and np.abs(d - h).mean() < 1.0 / 255.0
    assert np.array_equal(load_image_device(tmp_path / "a.png").cpu().numpy(), load_image(tmp_path / "a.png"))
    assert np.abs(load_image_device(tmp_path / "a.png", 2).cpu().numpy() -
                  load_image(tmp_path / "a.png", 2)).max() < 1e-6


def test_export_spz_equals_host_writer(tmp_path):
    from splatx_cuda import io as sio
    scene, cam, P = _scene(seed=17, sh=3)
    n = scene.count
    P[3][::4, 0] = -7.0
    ex = _executor(P, n, 3)
    st = ex.export_spz(n, tmp_path / "dev.spz", antialiased=True)
    hst = sio.write_spz(sio.from_groups(P, 3), tmp_path / "host.spz", antialiased=True)
    assert st == hst
    assert (tmp_path / "dev.spz").read_bytes() == (tmp_path / "host.spz").read_bytes()
    ex.close()


def test_raster_pair_counting():
    """The counting raster variants change no result, and count exactly: one Gaussian is
    evaluated once by every pixel of every tile it intersects in the forward; the backward
    replays it for the pixels it reached (plus the non-contributing pixels of the tile whose
    list starts at index 0, since "no contributor" is stored as last id 0)."""
    from splatx_cuda.executor import TrainStepExecutor
    scene, cam, P = _scene(seed=18, sh=1)
    n = scene.count
    ex = _executor(P, n, 1)
    _, _, plain = ex.step(cam.viewmat, cam.K, cam.width, cam.height, None, n, degrees_to_use=1,
                          forward_only=True, want_render=True)
    ex.set_pair_counting(True)
    _, _, counted = ex.step(cam.viewmat, cam.K, cam.width, cam.height, None, n, degrees_to_use=1,
                            forward_only=True, want_render=True)
    fwd, bwd = ex.raster_pairs()
    ex.set_pair_counting(False)
    assert np.array_equal(plain.view(np.uint32), counted.view(np.uint32))
    assert 0 < fwd and bwd == 0  # a forward-only step has no replay
    ex.close()

    # one Gaussian 5 units in front of an identity camera, 64x64 pixels (whole tiles)
    P1 = [np.array([[0.1, -0.2, 5.0]], np.float32), np.array([[1, 0, 0, 0]], np.float32),
          np.log(np.full((1, 3), 0.1, np.float32)), np.array([[2.0]], np.float32),
          np.full((1, 3), 0.4, np.float32), np.zeros((1, 0), np.float32)]
    ex = _executor(P1, 1, 0)
    vm = np.eye(4, dtype=np.float32).ravel()
    K = np.array([100, 0, 32, 0, 100, 32, 0, 0, 1], np.float32)
    gt = np.full(64 * 64 * 3, 0.5, np.float32)
    ex.set_pair_counting(True)
    loss, n_isects, render = ex.step(vm, K, 64, 64, gt, 1, degrees_to_use=0, want_render=True)
    fwd, bwd = ex.raster_pairs()
    ex.set_pair_counting(False)
    reached = int((render.reshape(64 * 64, 3)[:, 0] > 0).sum())
    assert n_isects >= 2 and loss > 0 and reached > 0
    assert fwd == 256 * n_isects
    assert reached <= bwd <= reached + 256
    ex.close()
