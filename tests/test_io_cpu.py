"""PLY files, the export filter and the eval metrics on the CPU (PlyIO.cpp, Trainer.cpp:349-418).

Our writer produces the reference writer's bytes; each side reads the other's files back exactly;
the export filter keeps the reference's rows and counts; the numpy restatement of the eval
metrics (used by the GPU eval tests) reproduces the reference's psnr and colour correction. The
reader's rejections (encoding, property types, SH counts) follow the reference's."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from splatx_cuda import io as sio

pytestmark = []


def _needs_ref():
    if not oracle.ref_available():
        pytest.skip("oracle/_ref (the reference's own CPU code) not built here")


def _cloud(n, deg, seed=0):
    rng = np.random.default_rng(seed)
    c = sio.empty_cloud(n, deg)
    for f in sio.FIELDS:
        c[f][...] = rng.normal(0, 1, c[f].shape).astype(np.float32)
    return c


@pytest.mark.parametrize("deg", [0, 1, 2, 3])
@pytest.mark.parametrize("pad", [True, False])
def test_ply_bytes_match_reference_writer(tmp_path, deg, pad):
    _needs_ref()
    c = _cloud(257, deg, seed=deg)
    sio.write_ply(c, tmp_path / "ours.ply", pad)
    oracle.ref_ply_write(c, tmp_path / "ref.ply", pad)
    assert (tmp_path / "ours.ply").read_bytes() == (tmp_path / "ref.ply").read_bytes()


@pytest.mark.parametrize("deg", [0, 1, 3])
def test_ply_round_trips_both_ways(tmp_path, deg):
    c = _cloud(100, deg, seed=10 + deg)
    sio.write_ply(c, tmp_path / "a.ply", pad_sh_full=False)
    back = sio.read_ply(tmp_path / "a.ply")
    assert back["count"] == 100 and back["sh_degree"] == deg
    for f in sio.FIELDS:
        assert np.array_equal(back[f], c[f]), f
    if oracle.ref_available():
        ref = oracle.ref_ply_read(tmp_path / "a.ply")
        for f in sio.FIELDS:
            assert np.array_equal(ref[f], c[f]), f
        oracle.ref_ply_write(c, tmp_path / "b.ply", True)
        back = sio.read_ply(tmp_path / "b.ply")  # padded degree-1 and -2 files read as degree 3
        assert back["sh_degree"] == (3 if deg else 0)
        K = (deg + 1) ** 2 - 1
        assert np.array_equal(back["shN"][:, :K], c["shN"])
        assert not back["shN"][:, K:].any()


def test_ply_reader_rejections(tmp_path):
    p = tmp_path / "bad.ply"
    p.write_bytes(b"ply\nformat ascii 1.0\nelement vertex 0\nend_header\n")
    with pytest.raises(Exception, match="binary_little_endian"):
        sio.read_ply(p)
    p.write_bytes(b"ply\nformat binary_little_endian 1.0\nelement vertex 1\nproperty uchar red\nend_header\n")
    with pytest.raises(Exception, match="only float"):
        sio.read_ply(p)
    hdr = "ply\nformat binary_little_endian 1.0\nelement vertex 1\n" + "".join(
        f"property float {n}\n" for n in ["x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2", "f_rest_0",
                                          "f_rest_1", "opacity"]) + "end_header\n"
    p.write_bytes(hdr.encode() + np.zeros(9, np.float32).tobytes())
    with pytest.raises(Exception, match="f_rest"):
        sio.read_ply(p)
    hdr = "ply\nformat binary_little_endian 1.0\nelement vertex 2\n" + "".join(
        f"property float {n}\n" for n in ["x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2", "opacity",
                                          "scale_0", "scale_1", "scale_2", "rot_0", "rot_1",
                                          "rot_2", "rot_3"]) + "end_header\n"
    p.write_bytes(hdr.encode() + np.zeros(14, np.float32).tobytes())  # one row of two
    with pytest.raises(Exception, match="truncated"):
        sio.read_ply(p)


def test_export_filter_matches_reference():
    c = _cloud(500, 1, seed=3)
    c["opacities"][::7] = -6.0   # sigmoid < 0.005
    c["opacities"][1::11] = -5.2933  # near the threshold
    c["means"][5, 1] = np.nan
    c["shN"][9, 2, 0] = np.inf
    c["opacities"][14] = np.nan
    out, st = sio.filter_for_export(c)
    assert st["input"] == 500 and st["kept"] == out["count"]
    assert st["removed_nonfinite"] == 3
    if oracle.ref_available():
        ref, rst = oracle.ref_filter_for_export(c)
        assert st == rst
        for f in sio.FIELDS:
            assert np.array_equal(out[f], ref[f]), f


def test_eval_metric_restatement_matches_reference():
    _needs_ref()
    rng = np.random.default_rng(4)
    H, W = 40, 52
    gt = rng.uniform(0, 1, H * W * 3).astype(np.float32)
    render = np.clip(gt * 0.8 + 0.1 + rng.normal(0, 0.05, gt.size), -0.2, 1.2).astype(np.float32)
    ps, cc_ps, _, _ = oracle.eval_metrics(render, gt, H, W)
    r = np.clip(render, 0, 1)
    assert ps == oracle.ref_psnr(r, gt)
    cc = oracle.ref_color_correct(r, gt)
    assert cc_ps == oracle.ref_psnr(cc, gt)


def _spz_cloud(n, deg, seed):
    rng = np.random.default_rng(seed)
    c = sio.empty_cloud(n, deg)
    c["means"][...] = rng.normal(0, 3, c["means"].shape)
    c["scales"][...] = rng.normal(-3, 1, c["scales"].shape)
    c["quats"][...] = rng.normal(0, 1, c["quats"].shape)
    c["opacities"][...] = rng.normal(0, 3, c["opacities"].shape)
    c["sh0"][...] = rng.normal(0, 1, c["sh0"].shape)
    c["shN"][...] = rng.normal(0, 0.4, c["shN"].shape)
    c["opacities"][::13] = -8.0          # filtered
    c["means"][7, 0] = np.nan            # filtered
    c["quats"][11] = [0.5, -0.5, 0.5, -0.5]  # ties for the largest component
    c["sh0"][3] = [50.0, -50.0, 0.0]     # clamped colours
    c["opacities"][5] = 20.0              # saturated alpha byte
    return c


@pytest.mark.parametrize("deg", [0, 1, 2, 3])
@pytest.mark.parametrize("aa", [False, True])
def test_spz_bytes_match_reference(tmp_path, deg, aa):
    _needs_ref()
    c = _spz_cloud(400, deg, 20 + deg)
    st = sio.write_spz(c, tmp_path / "ours.spz", antialiased=aa)
    rst = oracle.ref_spz_write(c, tmp_path / "ref.spz", antialiased=aa)
    assert st == rst
    assert (tmp_path / "ours.spz").read_bytes() == (tmp_path / "ref.spz").read_bytes()


@pytest.mark.parametrize("deg", [0, 2, 3])
def test_spz_reads_match_reference(tmp_path, deg):
    c = _spz_cloud(300, deg, 30 + deg)
    sio.write_spz(c, tmp_path / "a.spz", antialiased=True)
    ours = sio.read_spz(tmp_path / "a.spz")
    assert ours["antialiased"] and ours["sh_degree"] == deg
    # the round trip is within the quantisation steps
    keep, _ = sio.filter_for_export(c)
    assert ours["count"] == keep["count"]
    assert np.abs(ours["means"] - keep["means"]).max() <= 0.5 / 4096 + 1e-6
    assert np.abs(ours["scales"] - keep["scales"]).max() <= 0.5 / 16 + 1e-6
    if oracle.ref_available():
        ref = oracle.ref_spz_read(tmp_path / "a.spz")
        for f in sio.FIELDS:
            assert np.array_equal(ours[f].view(np.uint32), ref[f].view(np.uint32)), f
        assert ours["opacities"].max() <= 6.2324481


def test_spz_rejections(tmp_path):
    p = tmp_path / "x.spz"
    p.write_bytes(b"not gzip at all")
    with pytest.raises(Exception):
        sio.read_spz(p)
    import gzip
    p.write_bytes(gzip.compress(b"XGSP" + bytes(12)))
    with pytest.raises(Exception, match="header"):
        sio.read_spz(p)
    hdr = np.array([0x5053474e, 9, 1], np.uint32).tobytes() + bytes([0, 12, 0, 0])
    p.write_bytes(gzip.compress(hdr))
    with pytest.raises(Exception, match="version"):
        sio.read_spz(p)
    hdr = np.array([0x5053474e, 3, 5], np.uint32).tobytes() + bytes([0, 12, 0, 0])
    p.write_bytes(gzip.compress(hdr + bytes(20)))
    with pytest.raises(Exception, match="truncated"):
        sio.read_spz(p)
    with pytest.raises(Exception):
        sio.write_spz({**sio.empty_cloud(3, 3), "sh_degree": 4}, tmp_path / "y.spz")
