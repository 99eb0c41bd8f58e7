"""splatx_cuda — host mirror of splatx-metal's kernel contract on the B200 library.

``CudaBackend`` mirrors ``KernelBackend`` (per-kernel verification surface), ``TrainStepExecutor``
mirrors the resident step executor; both call libsplatx_cuda.so through include/splatx_cuda.h.
"""
from .build import build, lib_path  # noqa: F401


def __getattr__(name):
    if name == "CudaBackend":
        from .backend import CudaBackend
        return CudaBackend
    if name == "TrainStepExecutor":
        from .executor import TrainStepExecutor
        return TrainStepExecutor
    if name == "make_binoms_lut":
        from .backend import make_binoms_lut
        return make_binoms_lut
    raise AttributeError(name)
