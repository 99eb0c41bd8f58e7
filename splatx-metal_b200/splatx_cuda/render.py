"""RenderSession — the session-style render API (sx_render_session_open / _frame / _close,
Sources/SplatXTrainC/include/splatx_train_c.h:578-682) over libsplatx_cuda: open loads a PLY
once and keeps it resident on a GPU, frame renders any pinhole camera to RGBA8, close releases.
Error behaviour follows the reference: open raises (the C call returns NULL with a message), frame
raises ValueError for an argument violation (-1) and RuntimeError for a render failure (-2)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as _nat


class RenderSession:
    def __init__(self, ply_path: str, antialiased: bool = False, sh_degree: int = 0,
                 device: int = 0):
        args = _nat.SxRenderSessionArgs(str(ply_path).encode(), int(bool(antialiased)),
                                        int(sh_degree), int(device))
        err = C.create_string_buffer(512)
        h = _nat.lib().sxcuda_render_session_open(C.byref(args), err, len(err))
        if not h:
            raise RuntimeError(err.value.decode())
        self._h = C.c_void_p(h)

    def frame(self, viewmat, fx, fy, cx, cy, width, height) -> np.ndarray:
        vm = np.ascontiguousarray(np.asarray(viewmat, np.float32).ravel())
        if vm.size != 16:
            raise ValueError("viewmat must have 16 floats")
        out = np.empty((max(int(height), 1), max(int(width), 1), 4), np.uint8)
        err = C.create_string_buffer(512)
        rc = _nat.lib().sxcuda_render_session_frame(self._h, vm.ctypes.data, float(fx), float(fy),
                                                    float(cx), float(cy), int(width), int(height),
                                                    out.ctypes.data, err, len(err))
        if rc == -1:
            raise ValueError(err.value.decode())
        if rc != 0:
            raise RuntimeError(err.value.decode())
        return out

    def close(self):
        if getattr(self, "_h", None) and self._h.value:
            _nat.lib().sxcuda_render_session_close(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
