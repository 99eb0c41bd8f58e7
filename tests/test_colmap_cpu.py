"""COLMAP models on the CPU (ColmapLoader.cpp, TrainingInput.cpp): binary and text models written
here load to the reference's cameras (viewmat and K bit for bit, sizes, image paths) and seed
points; the loader's rejections (distortion models, unknown cameras, truncation, bad tokens)
match the reference's; images decode to float RGB and downsample by box averaging."""
from __future__ import annotations

import struct

import numpy as np
import pytest

import oracle
from splatx_cuda.dataset import load_colmap, load_image, resolve_images_dir, scale_camera


def _model(rng, n_img=5, n_pts=40, model="PINHOLE"):
    cams = [(1, model, 640, 480, [500.0, 510.0, 320.5, 239.25] if model == "PINHOLE" else
             [500.0, 320.5, 239.25] if model == "SIMPLE_PINHOLE" else [500.0, 510.0, 320.0, 240.0, 0.01, 0.0, 0.0, 0.0]),
            (7, "SIMPLE_PINHOLE", 320, 200, [250.25, 160.0, 100.0])]
    imgs = []
    for i in range(n_img):
        q = rng.normal(size=4)
        imgs.append((i + 1, q, rng.normal(size=3) * 3, 1 if i % 2 == 0 else 7, f"img_{i:03d}.jpg"))
    pts = [(i, rng.normal(size=3) * 2, rng.integers(0, 256, 3)) for i in range(n_pts)]
    return cams, imgs, pts


MODEL_ID = {"SIMPLE_PINHOLE": 0, "PINHOLE": 1, "OPENCV": 4}


def _write_bin(d, cams, imgs, pts):
    with open(d / "cameras.bin", "wb") as f:
        f.write(struct.pack("<Q", len(cams)))
        for cid, m, w, h, p in cams:
            f.write(struct.pack("<iiQQ", cid, MODEL_ID[m], w, h) + struct.pack(f"<{len(p)}d", *p))
    with open(d / "images.bin", "wb") as f:
        f.write(struct.pack("<Q", len(imgs)))
        for iid, q, t, cid, name in imgs:
            f.write(struct.pack("<i4d3di", iid, *q, *t, cid) + name.encode() + b"\0")
            f.write(struct.pack("<Q", 2) + struct.pack("<ddq", 1.0, 2.0, -1) * 2)
    with open(d / "points3D.bin", "wb") as f:
        f.write(struct.pack("<Q", len(pts)))
        for pid, xyz, rgb in pts:
            f.write(struct.pack("<Q3d3Bd", pid, *xyz, *[int(c) for c in rgb], 0.5))
            f.write(struct.pack("<Q", 1) + struct.pack("<ii", 1, 0))


def _write_txt(d, cams, imgs, pts):
    with open(d / "cameras.txt", "w") as f:
        f.write("# Camera list\n\n")
        for cid, m, w, h, p in cams:
            f.write(f"{cid} {m} {w} {h} " + " ".join(repr(x) for x in p) + "\r\n")
    with open(d / "images.txt", "w") as f:
        f.write("# Image list with two lines of data per image:\n")
        for iid, q, t, cid, name in imgs:
            f.write(f"{iid} " + " ".join(repr(float(x)) for x in (*q, *t)) + f" {cid} {name}\n")
            f.write("\n" if iid % 2 else "1.0 2.0 -1 3.0 4.0 5\n")
    with open(d / "points3D.txt", "w") as f:
        for pid, xyz, rgb in pts:
            f.write(f"{pid} " + " ".join(repr(float(x)) for x in xyz) + " " +
                    " ".join(str(int(c)) for c in rgb) + " 0.5 1 0 2 3\n")


@pytest.mark.parametrize("fmt", ["bin", "txt"])
def test_colmap_matches_reference(tmp_path, fmt):
    cams, imgs, pts = _model(np.random.default_rng(1))
    (_write_bin if fmt == "bin" else _write_txt)(tmp_path, cams, imgs, pts)
    ti = load_colmap(tmp_path, "/data/images")
    assert len(ti.cameras) == 5 and ti.seed_points.shape == (40, 3)
    assert ti.image_paths[2] == "/data/images/img_002.jpg"
    assert (ti.cameras[1].width, ti.cameras[1].height) == (320, 200)
    assert np.array_equal(ti.seed_rgb, np.array([p[2] for p in pts], np.uint8))
    if not oracle.ref_available():
        return
    L = oracle.ref_lib()
    ni, np_ = oracle.C.c_int64(), oracle.C.c_int64()
    args = [str(tmp_path).encode(), b"/data/images", oracle.C.byref(ni), oracle.C.byref(np_)]
    assert L.sxr_colmap_load(*args, None, None, None, None, None, None, None, oracle.I64(0)) == 0
    vm = np.zeros((5, 16), np.float32)
    K = np.zeros((5, 9), np.float32)
    w, h = np.zeros(5, np.int32), np.zeros(5, np.int32)
    P, rgb = np.zeros((40, 3), np.float32), np.zeros((40, 3), np.uint8)
    names = oracle.C.create_string_buffer(4096)
    assert L.sxr_colmap_load(*args, *[oracle._p(x) for x in (vm, K, w, h, P, rgb)], names,
                             oracle.I64(4096)) == 0
    for i, c in enumerate(ti.cameras):
        assert np.array_equal(c.viewmat.view(np.uint32), vm[i].view(np.uint32)), i
        assert np.array_equal(c.K.view(np.uint32), K[i].view(np.uint32)), i
        assert (c.width, c.height) == (w[i], h[i])
    assert names.raw.split(b"\0")[:5] == [p.encode() for p in ti.image_paths]
    assert np.array_equal(ti.seed_points.view(np.uint32), P.view(np.uint32))
    assert np.array_equal(ti.seed_rgb, rgb)


def test_colmap_rejections(tmp_path):
    rng = np.random.default_rng(2)
    cams, imgs, pts = _model(rng, model="OPENCV")
    _write_bin(tmp_path, cams, imgs, pts)
    with pytest.raises(RuntimeError, match="OPENCV"):
        load_colmap(tmp_path)
    cams, imgs, pts = _model(rng)
    imgs[0] = (1, imgs[0][1], imgs[0][2], 99, "x.jpg")
    _write_bin(tmp_path, cams, imgs, pts)
    with pytest.raises(RuntimeError, match="unknown camera 99"):
        load_colmap(tmp_path)
    d = tmp_path / "t"
    d.mkdir()
    cams, imgs, pts = _model(rng)
    _write_txt(d, cams, imgs, pts)
    (d / "cameras.txt").write_text("1 PINHOLE 640 480 500 510 320\n")
    with pytest.raises(RuntimeError, match="expects 4 params"):
        load_colmap(d)
    _write_bin(tmp_path, cams, imgs, pts)
    data = (tmp_path / "points3D.bin").read_bytes()
    (tmp_path / "points3D.bin").write_bytes(data[:-20])
    with pytest.raises(RuntimeError, match="truncated"):
        load_colmap(tmp_path)
    with pytest.raises(RuntimeError, match="cannot open"):
        load_colmap(tmp_path / "missing")


def test_images_decode_and_downsample(tmp_path):
    from PIL import Image
    rng = np.random.default_rng(3)
    a = rng.integers(0, 256, (37, 50, 3), dtype=np.uint8)
    Image.fromarray(a).save(tmp_path / "a.png")
    img = load_image(tmp_path / "a.png")
    assert np.array_equal(img, a.astype(np.float32) * np.float32(1.0 / 255.0))
    half = load_image(tmp_path / "a.png", factor=2)
    assert half.shape == (18, 25, 3)
    ref = a[:36, :50].astype(np.float64).reshape(18, 2, 25, 2, 3).mean(axis=(1, 3)) / 255.0
    assert np.abs(half - ref).max() < 1e-6
    (tmp_path / "images").mkdir()
    assert resolve_images_dir(str(tmp_path), 2) == (str(tmp_path / "images"), True)
    (tmp_path / "images_2").mkdir()
    assert resolve_images_dir(str(tmp_path), 2) == (str(tmp_path / "images_2"), False)
    from splatx_cuda.scene import Camera
    c = scale_camera(Camera(np.eye(4, dtype=np.float32).ravel(),
                            np.array([500, 0, 320, 0, 500, 240, 0, 0, 1], np.float32), 641, 481), 2)
    assert (c.width, c.height) == (320, 240) and c.K[0] == 250 and c.K[2] == 160
