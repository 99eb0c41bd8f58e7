"""Algorithmic (compulsory) bytes of each segment of the resident step.

Each tensor is counted once per read and once per write at its element size; re-reads (the raster
gathers hitting L2, SSIM aprons) are not counted, so achieved = bytes / time is what the segment
must move at minimum. Per-unit figures (fp32, SH degree 3 => 48 SH floats, 59 parameters per
Gaussian):

  fwd_gauss   per Gaussian: parameters read 236 B (means 12, quats 16, log-scales 12, opacity 4,
              SH 192) + outputs written 66 B (valid 1, means2d 8, conic 12, raster opacity 4,
              colour 12, relu mask 1, tile count 4, depth key 4, id 4, activations 16)  = 302 B
  depth_sort  per Gaussian: histogram read 4 B, then 4 passes of key+value read (8 B) and
              written (8 B; the last pass writes values only, 4 B)                      = 64 B
  Tile lists by supertile binning (the executor's default; E = (Gaussian, supertile) entries):
  scan        per Gaussian: order 4 + gathered entry count 4 + tile count 4 read, offset 4
              written                                                                   = 16 B
  emit        per entry: supertile key 4 + entry id 4 + (mask, Gaussian id) record 16 written
              (24 B); per visible Gaussian: order 4, offset 4, entry count 4, means2d 8,
              conic 12, opacity 4 read (36 B)
  tile_sort   per entry: key histogram read 4, one pass of key + id read (8) and sorted id
              written (4), the count kernel's sorted id + mask read (12), the write kernel's
              sorted id + record read (20) = 48 B; per intersection: flatten id written 4 B
  Tile lists by the pair sort (tile_bits-bit tile keys in ceil(tile_bits / 8) passes):
  scan        per Gaussian: order 4 + gathered tile count 4 read, offset 4 written      = 12 B
  emit        per intersection: tile key 4 + id 4 written (8 B); per visible Gaussian: order 4,
              offset 4, tile count 4, means2d 8, conic 12, opacity 4 read (36 B)
  tile_sort   per intersection: histogram read 4 B, 2 passes of key+value read and written
              (16 B; the last pass writes ids only, 12 B)                               = 32 B
  raster_fwd  per intersection: id 4 + xy 8 + opacity 4 + conic 12 + colour 12 = 40 B;
              per pixel: colour 12 + alpha 4 + last id 4 written                        = 20 B
  loss        per pixel-channel: SSIM forward reads render+target (8 B) and writes the map and
              three coefficient maps (16 B); the backward reads the three maps (12 B) and
              render+target (8 B) and writes v_render (4 B)                             = 48 B
  raster_bwd  per intersection: the 40 B gather + id 4 = 44 B; per pixel: alpha 4 + last id 4
              + v_render 12 + v_alpha 4 read = 24 B; per visible Gaussian: 9 gradient floats
              accumulated (36 B)
  bwd_gauss   per visible Gaussian (bwd_sh + bwd_geom): parameters and both Adam moments read
              and written (59 x 4 x 6 = 1416 B), 9 gradient floats read and re-zeroed (72 B),
              conic 12, valid 1, relu mask 1, activations 16, v_dir written+read 24, means
              re-read 12                                                                = 1554 B
"""
from __future__ import annotations


def segment_bytes(n_gauss: int, n_visible: int, n_isects: int, width: int, height: int,
                  tile_bits: int, sh_degree: int = 3, n_entries: int = 0) -> dict:
    """n_entries > 0: the step binned its intersections by supertile (that many entries);
    0: it sorted (tile, Gaussian) pairs."""
    K = (sh_degree + 1) ** 2
    params_per_g = (3 + 4 + 3 + 1 + 3 * K) * 4
    hw = width * height
    tile_passes = max(1, -(-tile_bits // 8))
    if n_entries > 0:
        lists = {"scan": n_gauss * 16, "emit": n_entries * 24 + n_visible * 36,
                 "tile_sort": n_entries * 48 + n_isects * 4}
    else:
        lists = {"scan": n_gauss * 12, "emit": n_isects * 8 + n_visible * 36,
                 "tile_sort": n_isects * (4 + 16 * (tile_passes - 1) + 12)}
    return {
        "fwd_gauss": n_gauss * (params_per_g + 66),
        "depth_sort": n_gauss * (4 + 16 * 3 + 12),
        **lists,
        "raster_fwd": n_isects * 40 + hw * 20,
        "loss": hw * 3 * 48,
        "raster_bwd": n_isects * 44 + hw * 24 + n_visible * 36,
        "bwd_gauss": n_visible * (params_per_g * 6 + 72 + 12 + 2 + 16 + 24 + 12),
    }


def step_bytes(**kw) -> int:
    return int(sum(segment_bytes(**kw).values()))


# The fixed per-unit table the measurement plan set before any kernel existed (fp32, SH degree 3,
# the reference's kernel sequence: a 45-bit key sort in 6 passes of 8 bits, a separate
# offset-encode pass): per Gaussian 2,596 B, per intersection 252 B, per pixel 84 B. It does not
# follow the implementation (its sort, fused kernels and binned tile lists move fewer bytes), so
# both step fractions are reported.
FIXED_B_G = 2596
FIXED_B_I = 252
FIXED_B_P = 84


def fixed_table_bytes(n_gauss: int, n_isects: int, width: int, height: int) -> int:
    return n_gauss * FIXED_B_G + n_isects * FIXED_B_I + width * height * FIXED_B_P
