"""Training input from a COLMAP dataset (load_colmap_bundle + training_input_from_colmap,
Sources/SplatXCore/ColmapLoader.cpp and TrainingInput.cpp; resolve_images_dir,
TrainingInput.h:29-41) over libsplatx_cuda's host loader, plus ground-truth images.

Images decode to float32 RGB in [0, 1] (u8 times the float 1/255, the reference's ImageIO
convention, ImageIO.cpp:60-64). JPEGs can be
decoded on the GPU (nvJPEG through torchvision) straight into device memory, which the executor
consumes with ``gt_on_device`` — the image never exists as floats on the host. A factor > 1 uses
``images_<factor>`` when present and otherwise downsamples on load by box-averaging factor x factor
blocks (dimensions floor(W / factor) x floor(H / factor)).
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import os

import numpy as np

from . import _native as _nat
from ._native import check
from .scene import Camera


@dataclasses.dataclass
class TrainingInput:
    cameras: list          # Camera per registered image, in file order
    image_paths: list      # str per camera
    seed_points: np.ndarray  # [M, 3] float32
    seed_rgb: np.ndarray     # [M, 3] uint8


def _lib():
    return _nat.lib()


def resolve_images_dir(data_dir: str, factor: int) -> tuple[str, bool]:
    """(images folder, downscale on load) for a factor (TrainingInput.h:29-41)."""
    originals = os.path.join(data_dir, "images")
    if factor <= 1:
        return originals, False
    scaled = os.path.join(data_dir, f"images_{factor}")
    if os.path.isdir(scaled):
        return scaled, False
    if os.path.isdir(originals):
        return originals, True
    raise FileNotFoundError(f"resolve_images_dir: neither {scaled} nor {originals} exists")


def load_colmap(sparse_dir: str, images_dir: str = "") -> TrainingInput:
    L = _lib()
    h = C.c_void_p()
    check(L.sxcuda_colmap_open(str(sparse_dir).encode(), str(images_dir).encode(), C.byref(h)))
    try:
        ni, npnt = C.c_int64(), C.c_int64()
        check(L.sxcuda_colmap_counts(h, C.byref(ni), C.byref(npnt)))
        n = ni.value
        vm = np.zeros((n, 16), np.float32)
        K = np.zeros((n, 9), np.float32)
        w = np.zeros(n, np.int32)
        hh = np.zeros(n, np.int32)
        if n:
            check(L.sxcuda_colmap_cameras(h, vm.ctypes.data, K.ctypes.data, w.ctypes.data,
                                          hh.ctypes.data))
        paths = []
        for i in range(n):
            ln = C.c_int64()
            check(L.sxcuda_colmap_image_path(h, i, None, 0, C.byref(ln)))
            buf = C.create_string_buffer(ln.value + 1)
            check(L.sxcuda_colmap_image_path(h, i, buf, ln.value + 1, C.byref(ln)))
            paths.append(buf.raw[:ln.value].decode())
        pts = np.zeros((npnt.value, 3), np.float32)
        rgb = np.zeros((npnt.value, 3), np.uint8)
        check(L.sxcuda_colmap_seed(h, pts.ctypes.data, rgb.ctypes.data))
    finally:
        L.sxcuda_colmap_close(h)
    cams = [Camera(vm[i].copy(), K[i].copy(), int(w[i]), int(hh[i])) for i in range(n)]
    return TrainingInput(cams, paths, pts, rgb)


def scale_camera(cam: Camera, factor: int) -> Camera:
    """The camera of an image downsampled by ``factor`` (intrinsics / factor, floor dims)."""
    if factor <= 1:
        return cam
    K = cam.K.astype(np.float32).copy()
    K[[0, 1, 2, 3, 4, 5]] /= np.float32(factor)
    return Camera(cam.viewmat, K, cam.width // factor, cam.height // factor)


def _box(img: np.ndarray, factor: int) -> np.ndarray:
    h, w = img.shape[0] // factor, img.shape[1] // factor
    v = img[:h * factor, :w * factor].reshape(h, factor, w, factor, 3)
    return v.mean(axis=(1, 3), dtype=np.float64).astype(np.float32)


def load_image(path: str, factor: int = 1) -> np.ndarray:
    """float32 [H, W, 3] in [0, 1] on the host (PIL decode)."""
    from PIL import Image
    with Image.open(path) as im:
        a = np.asarray(im.convert("RGB"), np.uint8)
    img = a.astype(np.float32) * np.float32(1.0 / 255.0)
    return _box(img, factor) if factor > 1 else img


def load_image_device(path: str, factor: int = 1, device: int = 0):
    """float32 [H, W, 3] in [0, 1] as a CUDA tensor: JPEGs decode on the GPU (nvJPEG), other
    formats on the host; the downsampling runs on the device."""
    import torch
    dev = torch.device("cuda", device)
    t = None
    if str(path).lower().endswith((".jpg", ".jpeg")):
        try:
            from torchvision.io import decode_jpeg, read_file
            t = decode_jpeg(read_file(str(path)), device=dev)  # [3, H, W] u8
        except Exception:
            t = None
    if t is None:
        from PIL import Image
        with Image.open(path) as im:
            t = torch.from_numpy(np.asarray(im.convert("RGB"), np.uint8).copy()).permute(2, 0, 1).to(dev)
    img = t.permute(1, 2, 0).float().mul_(float(np.float32(1.0 / 255.0)))
    if factor > 1:
        h, w = img.shape[0] // factor, img.shape[1] // factor
        img = img[:h * factor, :w * factor].reshape(h, factor, w, factor, 3).mean(dim=(1, 3))
    return img.contiguous()
