"""Write the committed golden fixtures back out in the reference's own fixture layout.

The reference's test sources read ``<fixture_dir>/<name>/<tensor>.sxt`` plus ``meta.json``
(SXTensor.h:8-26: "SXT1" | u32 dtype | u32 ndim | u64 shape[ndim] | little-endian payload, dtype
0=f32 1=i32 3=u8). ``import_fixtures.py`` repacked those files into ``<name>.npz`` / ``<name>.json``
here; this script inverts that, so the reference's test runner (oracle/ref_tests_main.cpp) can
run where only this repository exists.

    python tests/golden/export_sxt.py <out_dir>
"""
from __future__ import annotations

import json
import pathlib
import struct
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
_CODES = {np.dtype(np.float32): 0, np.dtype(np.int32): 1, np.dtype(np.uint8): 3}


def write_sxt(path: pathlib.Path, a: np.ndarray) -> None:
    a = np.ascontiguousarray(a)
    code = _CODES[a.dtype]
    head = b"SXT1" + struct.pack("<II", code, a.ndim) + struct.pack(f"<{a.ndim}Q", *a.shape)
    path.write_bytes(head + a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes())


def export(out: pathlib.Path) -> list:
    """Every fixture import_fixtures.py took from the reference (its HOT_PATH list)."""
    sys.path.insert(0, str(HERE))
    from import_fixtures import HOT_PATH
    names = []
    for name in HOT_PATH:
        tag = name.replace("/", "__")
        npz, meta = HERE / f"{tag}.npz", HERE / f"{tag}.json"
        d = out / name
        d.mkdir(parents=True, exist_ok=True)
        for k, v in np.load(npz).items():
            write_sxt(d / f"{k}.sxt", v)
        m = json.loads(meta.read_text())
        if m:  # import_fixtures.py wrote {} where the reference has no meta.json
            (d / "meta.json").write_text(json.dumps(m, indent=1) + "\n")
        names.append(name)
    return names


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: export_sxt.py <out_dir>")
    for n in export(pathlib.Path(sys.argv[1])):
        print(n)
