"""Import splatx-metal's golden fixtures into tests/golden/ (run once where the reference exists).

The reference commits its gsplat-generated goldens as SXT tensors plus a meta.json of tolerances
under ``fixtures/`` (format: "SXT1" | u32 dtype | u32 ndim | u64 shape[ndim] | LE payload, dtype
0=f32 1=i32 3=u8; Sources/SplatXCore/include/splatx/SXTensor.h:8-26). This script repacks every
hot-path fixture into one ``<name>.npz`` (same tensor names) and copies its ``meta.json`` to
``<name>.json`` so the tests run on machines without the reference tree.

    python tests/golden/import_fixtures.py [/path/to/splatx-metal]
"""
from __future__ import annotations

import json
import os
import pathlib
import struct
import sys

import numpy as np

HOT_PATH = ["adam_basic", "isect_accutile", "isect_std", "isect_ties", "math_quat_scale_to_covar",
            "perturb_basic", "proj_fully_fused", "proj_fused_qs/c1", "proj_fused_qs/c2",
            "raster_dense", "raster_small/nobg", "raster_small/bg", "raster_std",
            "relocation_basic", "sh_k16", "sh_k25", "ssim_basic"]
_CODES = {0: np.float32, 1: np.int32, 3: np.uint8}


def read_sxt(path: pathlib.Path) -> np.ndarray:
    raw = path.read_bytes()
    if raw[:4] != b"SXT1":
        raise ValueError(f"{path}: not an SXT1 tensor")
    code, ndim = struct.unpack_from("<II", raw, 4)
    shape = struct.unpack_from(f"<{ndim}Q", raw, 12)
    arr = np.frombuffer(raw, dtype=_CODES[code], offset=12 + 8 * ndim)
    if arr.size != int(np.prod(shape, dtype=np.int64)):
        raise ValueError(f"{path}: payload does not match shape {shape}")
    return arr.reshape(shape).copy()


def main(ref_root: pathlib.Path) -> None:
    out = pathlib.Path(__file__).resolve().parent
    for name in HOT_PATH:
        src = ref_root / "fixtures" / name
        tensors = {p.stem: read_sxt(p) for p in sorted(src.glob("*.sxt"))}
        tag = name.replace("/", "__")
        np.savez_compressed(out / f"{tag}.npz", **tensors)
        meta_path = src / "meta.json"
        meta = json.loads(meta_path.read_text()) if meta_path.exists() else {}
        (out / f"{tag}.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
        print(f"{tag}: {len(tensors)} tensors")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPLATX_REFERENCE")
    if not root:
        sys.exit("usage: import_fixtures.py <reference checkout>  (or set SPLATX_REFERENCE)")
    main(pathlib.Path(root))
