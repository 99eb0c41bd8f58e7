"""The byte model bench.py divides by: roofline.segment_bytes (the implementation's compulsory
bytes per segment, for either way of building the tile lists) and the fixed per-unit table the
step's second fraction uses. Host arithmetic only."""
from splatx_cuda.roofline import FIXED_B_G, FIXED_B_I, FIXED_B_P, fixed_table_bytes, segment_bytes

CFG2 = dict(n_gauss=1_000_000, n_visible=828_644, n_isects=13_506_012, width=1297, height=840,
            tile_bits=13)


def test_binned_tile_lists_count_entries():
    e = 1_597_179
    b = segment_bytes(**CFG2, n_entries=e)
    assert "scan" in b and b["scan"] == CFG2["n_gauss"] * 16
    assert b["emit"] == e * 24 + CFG2["n_visible"] * 36
    assert b["tile_sort"] == e * 48 + CFG2["n_isects"] * 4


def test_pair_sort_counts_every_intersection():
    b = segment_bytes(**CFG2)  # n_entries = 0: the pair sort
    assert b["scan"] == CFG2["n_gauss"] * 12
    assert b["emit"] == CFG2["n_isects"] * 8 + CFG2["n_visible"] * 36
    # histogram 4 B, one full pass of key + value in and out (16 B), the last pass ids only (12 B)
    assert b["tile_sort"] == CFG2["n_isects"] * (4 + 16 + 12)


def test_segments_shared_by_both_methods():
    a = segment_bytes(**CFG2, n_entries=1_597_179)
    b = segment_bytes(**CFG2)
    for k in ("fwd_gauss", "depth_sort", "raster_fwd", "loss", "raster_bwd", "bwd_gauss"):
        assert a[k] == b[k], k
    assert a["fwd_gauss"] == CFG2["n_gauss"] * (236 + 66)         # SH degree 3
    assert a["bwd_gauss"] == CFG2["n_visible"] * 1554


def test_fixed_table():
    assert (FIXED_B_G, FIXED_B_I, FIXED_B_P) == (2596, 252, 84)
    assert fixed_table_bytes(1_000_000, 13_506_012, 1297, 840) == (
        1_000_000 * 2596 + 13_506_012 * 252 + 1297 * 840 * 84)
