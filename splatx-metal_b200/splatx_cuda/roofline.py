"""Algorithmic (compulsory) bytes of each segment of the resident step.

Each tensor is counted once per read and once per write at its element size; re-reads are not
counted, so achieved = bytes / time is a lower bound of the DRAM traffic a kernel must move.
Per-unit figures (fp32, SH degree 3 => 48 SH floats, 59 parameters per Gaussian):
  fwd_gauss   per Gaussian: params 236 B read (means 12, quats 16, log-scales 12, opacity 4,
              SH 192) + outputs 50 B written (valid 1, means2d 8, conic 12, opacity 4, colour 12,
              relu mask 1, tile count 4, depth key 4, id 4)                          = 286 B
  depth_sort  per Gaussian per 8-bit pass: key+value read twice (upsweep, downsweep) and written
              once = 4+4+4 + 8 = 20 B, 4 passes                                        = 80 B
  scan        per Gaussian: tile count gather 4 + order 4 + offset write 4              = 12 B
  emit        per intersection: tile key 4 + id 4 written; per Gaussian 24 B read
  tile_sort   per intersection per pass 20 B, ceil(tile_bits/8) passes
  raster_fwd  per intersection: id 4 + xy/opacity 12 + conic 12 + colour 12 = 40 B;
              per pixel: colour 12 + alpha 4 + last id 4 written                         = 20 B
  loss        per pixel-channel: render+gt read by SSIM fwd and bwd (16 B), three coefficient maps
              written and read (24 B), v_render written (4 B)                          = 44 B
  raster_bwd  per intersection: 40 B gather; per pixel: alpha 4 + last id 4 + v_render 12 read;
              per visible Gaussian: 9 gradient floats written (36 B)
  bwd_gauss   per visible Gaussian: params + both moments read and written (59 x 4 x 6 = 1416 B),
              9 gradient floats read and re-zeroed (72 B), conic 12 + valid 1 + mask 1 (14 B)
"""
from __future__ import annotations

import math


def segment_bytes(n_gauss: int, n_visible: int, n_isects: int, width: int, height: int,
                  tile_bits: int, sh_degree: int = 3) -> dict:
    K = (sh_degree + 1) ** 2
    params_per_g = (3 + 4 + 3 + 1 + 3 * K) * 4
    hw = width * height
    tile_passes = max(1, math.ceil(tile_bits / 8))
    return {
        "fwd_gauss": n_gauss * (params_per_g + 50),
        "depth_sort": n_gauss * 80,
        "scan": n_gauss * 12,
        "emit": n_isects * 8 + n_visible * 24,
        "tile_sort": n_isects * 20 * tile_passes,
        "tile_offsets": n_isects * 4,
        "raster_fwd": n_isects * 40 + hw * 20,
        "loss": hw * 3 * 44,
        "raster_bwd": n_isects * 40 + hw * 20 + n_visible * 36,
        "bwd_gauss": n_visible * (params_per_g * 6 + 72 + 14),
    }


def step_bytes(**kw) -> int:
    return int(sum(segment_bytes(**kw).values()))
