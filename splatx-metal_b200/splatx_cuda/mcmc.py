"""MCMC options and schedule of the reference trainer (Trainer.h:188-200, Trainer.cpp:496-500 and
:1262-1270), for driving ``TrainStepExecutor.mcmc_refine`` / ``inject_noise`` from a training loop.

The reference's order per iteration (Trainer.cpp:943-967): a step with the MCMC noise fused in on
non-refine iterations; on refine iterations the step runs without noise, then the refine, then the
noise on the grown count.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np


@dataclasses.dataclass
class McmcOptions:
    """McmcOptions (Trainer.h:188-196)."""
    enabled: bool = False
    cap_max: int = 1_000_000
    min_opacity: float = 0.005
    refine_start_ratio: float = 500.0 / 30000.0
    refine_stop_ratio: float = 25000.0 / 30000.0
    refine_every_ratio: float = 100.0 / 30000.0
    noise_lr: float = 5e5
    seed: int = 42


def _lround(x: float) -> int:
    """std::lround: halves away from zero."""
    return int(math.floor(x + 0.5)) if x >= 0 else -int(math.floor(-x + 0.5))


def refine_due(m: McmcOptions, it: int, total_iters: int) -> bool:
    """mcmc_refine_due (Trainer.cpp:1262-1270): start < iter < stop and iter % every == 0, the
    bounds rounded from the float ratios times the double total."""
    if not m.enabled:
        return False
    total = float(total_iters)
    start = _lround(total * float(np.float32(m.refine_start_ratio)))
    stop = _lround(total * float(np.float32(m.refine_stop_ratio)))
    every = max(1, _lround(total * float(np.float32(m.refine_every_ratio))))
    return start < it < stop and it % every == 0


def means_lr_at(lr_means: float, scene_scale: float, it: int, total_iters: int) -> float:
    """means_lr_at (Trainer.cpp:496-500): lr_means * scene_scale * 0.01^(iter / total), float."""
    from ._libm import powf
    p = np.float32(it) / np.float32(total_iters) if total_iters > 0 else np.float32(0)
    return float(np.float32(np.float32(lr_means) * np.float32(scene_scale)) * np.float32(powf(0.01, p)))


def noise_scale_at(m: McmcOptions, lr_means: float, scene_scale: float, it: int,
                   total_iters: int) -> float:
    """The MCMC noise scale of iteration ``it`` (Trainer.cpp:949): means lr times noise_lr."""
    return float(np.float32(means_lr_at(lr_means, scene_scale, it, total_iters)) * np.float32(m.noise_lr))
