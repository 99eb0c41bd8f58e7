"""Clouds in the reference's host layout, INRIA PLY files and the export filter
(Sources/SplatXCore/PlyIO.h:1-60, PlyIO.cpp), over libsplatx_cuda's host IO.

A cloud is a dict with ``count``, ``sh_degree`` and float32 arrays ``means`` [N,3], ``scales``
[N,3] (log), ``quats`` [N,4] (w first), ``opacities`` [N] (logit), ``sh0`` [N,3] and ``shN``
[N,K,3] (coefficient-major, K = (degree+1)^2 - 1) — SplatCloud's fields.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as _nat
from ._native import check

FIELDS = ("means", "scales", "quats", "opacities", "sh0", "shN")


def _k(degree: int) -> int:
    return (degree + 1) ** 2 - 1


def empty_cloud(count: int, sh_degree: int) -> dict:
    n, K = int(count), _k(sh_degree)
    return {"count": n, "sh_degree": int(sh_degree), "means": np.zeros((n, 3), np.float32),
            "scales": np.zeros((n, 3), np.float32), "quats": np.zeros((n, 4), np.float32),
            "opacities": np.zeros(n, np.float32), "sh0": np.zeros((n, 3), np.float32),
            "shN": np.zeros((n, K, 3), np.float32)}


def from_groups(groups, sh_degree: int) -> dict:
    """A cloud from the executor's six groups (D3 order: means, quats, scales, opacities, sh0,
    shN [N, 3K])."""
    n = int(np.asarray(groups[0]).reshape(-1, 3).shape[0])
    c = {"count": n, "sh_degree": int(sh_degree)}
    c["means"] = np.ascontiguousarray(np.asarray(groups[0], np.float32).reshape(n, 3))
    c["quats"] = np.ascontiguousarray(np.asarray(groups[1], np.float32).reshape(n, 4))
    c["scales"] = np.ascontiguousarray(np.asarray(groups[2], np.float32).reshape(n, 3))
    c["opacities"] = np.ascontiguousarray(np.asarray(groups[3], np.float32).reshape(n))
    c["sh0"] = np.ascontiguousarray(np.asarray(groups[4], np.float32).reshape(n, 3))
    c["shN"] = np.ascontiguousarray(np.asarray(groups[5], np.float32).reshape(n, _k(sh_degree), 3))
    return c


def to_groups(c: dict) -> list:
    n = c["count"]
    return [c["means"].reshape(n, 3), c["quats"].reshape(n, 4), c["scales"].reshape(n, 3),
            c["opacities"].reshape(n, 1), c["sh0"].reshape(n, 3), c["shN"].reshape(n, -1)]


def _struct(c: dict) -> _nat.SxCloud:
    for f in FIELDS:
        a = c[f]
        if a.dtype != np.float32 or not a.flags.c_contiguous:
            raise ValueError(f"cloud field {f} must be C-contiguous float32")
    return _nat.SxCloud(int(c["count"]), int(c["sh_degree"]), *[c[f].ctypes.data for f in FIELDS])


def write_ply(c: dict, path: str, pad_sh_full: bool = True):
    """write_inria_ply (PlyIO.h:20)."""
    s = _struct(c)
    check(_nat.lib().sxcuda_ply_write(C.byref(s), str(path).encode(), int(bool(pad_sh_full))))


def ply_info(path: str) -> tuple[int, int]:
    n, d = C.c_int64(), C.c_int32()
    check(_nat.lib().sxcuda_ply_info(str(path).encode(), C.byref(n), C.byref(d)))
    return int(n.value), int(d.value)


def read_ply(path: str) -> dict:
    """read_inria_ply (PlyIO.h:21) for SH degrees 0..3."""
    n, d = ply_info(path)
    c = empty_cloud(n, d)
    s = _struct(c)
    check(_nat.lib().sxcuda_ply_read(str(path).encode(), C.byref(s)))
    return c


def filter_for_export(c: dict, min_opacity: float = 0.005):
    """filter_cloud_for_export (PlyIO.h:48): (the kept cloud, stats dict)."""
    s = _struct(c)
    keep = np.zeros(max(int(c["count"]), 1), np.uint8)
    st = _nat.SxExportFilterStats()
    check(_nat.lib().sxcuda_filter_for_export(C.byref(s), float(min_opacity), keep.ctypes.data,
                                              C.byref(st)))
    k = keep[:c["count"]].astype(bool)
    out = {"count": int(k.sum()), "sh_degree": c["sh_degree"]}
    for f in FIELDS:
        out[f] = np.ascontiguousarray(c[f][k])
    stats = {"input": st.input, "removed_nonfinite": st.removed_nonfinite,
             "removed_low_opacity": st.removed_low_opacity, "kept": st.kept}
    return out, stats


def write_spz(c: dict, path: str, min_opacity: float = 0.005, antialiased: bool = False) -> dict:
    """save_spz (SpzIO.h): the export filter, then an SPZ v3 file; returns the filter stats."""
    s = _struct(c)
    st = _nat.SxExportFilterStats()
    check(_nat.lib().sxcuda_spz_write(C.byref(s), str(path).encode(), float(min_opacity),
                                      int(bool(antialiased)), C.byref(st)))
    return {"input": st.input, "removed_nonfinite": st.removed_nonfinite,
            "removed_low_opacity": st.removed_low_opacity, "kept": st.kept}


def spz_info(path: str) -> tuple[int, int, bool]:
    n, d, aa = C.c_int64(), C.c_int32(), C.c_int32()
    check(_nat.lib().sxcuda_spz_info(str(path).encode(), C.byref(n), C.byref(d), C.byref(aa)))
    return int(n.value), int(d.value), bool(aa.value)


def read_spz(path: str) -> dict:
    """load_spz (SpzIO.h): the cloud in the training frame (and ``antialiased`` from the flags)."""
    n, d, aa = spz_info(path)
    c = empty_cloud(n, d)
    s = _struct(c)
    check(_nat.lib().sxcuda_spz_read(str(path).encode(), C.byref(s)))
    c["antialiased"] = aa
    return c
