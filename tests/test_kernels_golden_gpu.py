"""Golden-fixture parity of every per-kernel entry point on the GPU, through the C-ABI.

Mirrors splatx-metal's own golden suite (Sources/SplatXTests/{Adam,ProjectionMetal,Sh,Isect,Sort,
Scan,Raster,Ssim,Mcmc}Tests.cpp): the same fixtures, the same comparison rules (tolerances only
from meta.json, integers exact, projection outputs compared under the radii>0 mask, backward
kernels fed the golden forward outputs) and the same determinism gates. Projection, SH and raster
forward outputs are in addition held to the north star's 1e-5 relative bar where it is stricter
than the fixture's rtol (conics, compensations and the raster render are 1e-4 in meta.json).
"""
import numpy as np
import pytest

from helpers import NORTH_STAR_FWD_RTOL, Fixture, assert_all_close, join_u64, rel_l2, valid_mask

pytestmark = pytest.mark.gpu


# ------------------------------------------------------------------ Adam (AdamTests.cpp:60-189)
@pytest.mark.parametrize("masked", [False, True])
def test_fused_adam_matches_golden(backend, masked):
    f = Fixture("adam_basic")
    p, m, v = f["param"].copy(), f["exp_avg"].copy(), f["exp_avg_sq"].copy()
    n_gauss = int(f.m("N"))
    backend.fused_adam(p, f["grad"], m, v, valid=f["valid"] if masked else None, n_gauss=n_gauss,
                       lr=f.m("lr"), b1=f.m("b1"), b2=f.m("b2"), eps=f.m("eps"))
    sfx = "_masked" if masked else ""
    assert_all_close(p, f["param_out" + sfx], f.meta, "param_out" + sfx)
    assert_all_close(m, f["exp_avg_out" + sfx], f.meta, "exp_avg_out" + sfx)
    assert_all_close(v, f["exp_avg_sq_out" + sfx], f.meta, "exp_avg_sq_out" + sfx)
    if masked:  # rows with valid==0 keep their inputs bit for bit
        keep = np.repeat(f["valid"].ravel() == 0, p.size // n_gauss)
        assert np.array_equal(p.ravel()[keep], f["param"].ravel()[keep])
        assert np.array_equal(v.ravel()[keep], f["exp_avg_sq"].ravel()[keep])


def test_fused_adam_invalid_arguments(backend):
    p = np.zeros(6, np.float32)
    with pytest.raises(ValueError):
        backend.fused_adam(p, p, p.copy(), p.copy(), n_gauss=4)  # 6 % 4 != 0


# ------------------------------------------------------------------ projection
def _proj_common(f):
    return dict(width=int(f.m("width")), height=int(f.m("height")), eps2d=f.m("eps2d"),
                near_plane=f.m("near_plane"), far_plane=f.m("far_plane"),
                radius_clip=f.m("radius_clip"), camera_model=int(f.m("camera_model")),
                calc_compensations=bool(f.m("calc_compensations")))


def _compare_proj_fwd(out, f):
    assert np.array_equal(out.radii.ravel(), f["radii"].ravel()), "radii must match exactly"
    valid = valid_mask(f["radii"])
    assert 0 < valid.sum() < valid.size
    cap = dict(rtol_cap=NORTH_STAR_FWD_RTOL)
    assert_all_close(out.means2d, f["means2d"], f.meta, "means2d", valid, 2, **cap)
    assert_all_close(out.depths, f["depths"], f.meta, "depths", valid, 1, **cap)
    assert_all_close(out.conics, f["conics"], f.meta, "conics", valid, 3, **cap)
    if f.m("calc_compensations"):
        assert_all_close(out.compensations, f["compensations"], f.meta, "compensations", valid, 1,
                         **cap)


@pytest.mark.parametrize("variant", ["proj_fused_qs/c1", "proj_fused_qs/c2"])
def test_projection_fwd_qs_matches_golden(backend, variant):
    f = Fixture(variant)
    out = backend.projection_fused_fwd(f["means"], f["viewmats"], f["Ks"], quats=f["quats"],
                                       scales=f["scales"], **_proj_common(f))
    _compare_proj_fwd(out, f)
    again = backend.projection_fused_fwd(f["means"], f["viewmats"], f["Ks"], quats=f["quats"],
                                         scales=f["scales"], **_proj_common(f))
    assert np.array_equal(out.means2d, again.means2d) and np.array_equal(out.conics, again.conics)


def test_projection_fwd_covars_matches_golden(backend):
    f = Fixture("proj_fully_fused")
    out = backend.projection_fused_fwd(f["means"], f["viewmats"], f["Ks"], covars=f["covars_triu"],
                                       **_proj_common(f))
    _compare_proj_fwd(out, f)


@pytest.mark.parametrize("variant", ["proj_fused_qs/c1", "proj_fused_qs/c2"])
def test_projection_bwd_matches_golden(backend, variant):
    f = Fixture(variant)
    inject = bool(f.m("bwd_inject_v_compensations"))
    g = backend.projection_fused_bwd(
        f["means"], f["viewmats"], f["Ks"], radii=f["radii"], conics=f["conics"],
        v_means2d=f["v_means2d"], v_depths=f["v_depths"], v_conics=f["v_conics"],
        quats=f["quats"], scales=f["scales"],
        compensations=f["compensations"] if inject else None,
        v_compensations=f["v_compensations"] if inject else None, viewmats_grad=True,
        **_proj_common(f))
    assert_all_close(g.v_means, f["v_means"], f.meta, "v_means")
    assert_all_close(g.v_quats, f["v_quats"], f.meta, "v_quats")
    assert_all_close(g.v_scales, f["v_scales"], f.meta, "v_scales")
    assert_all_close(g.v_viewmats, f["v_viewmats"], f.meta, "v_viewmats")


# ------------------------------------------------------------------ SH (ShTests.cpp:78-224)
def _sh_dims(f):
    B, N = f["dirs"].shape[0], f["dirs"].shape[1]
    K, D = f["coeffs"].shape[1], f["coeffs"].shape[2]
    return B, N, K, D


@pytest.mark.parametrize("deg", [0, 1, 2, 3])
def test_sh_fwd_k16_matches_golden(backend, deg):
    f = Fixture("sh_k16")
    B, N, K, D = _sh_dims(f)
    out = backend.sh_fwd(f["dirs"], f["coeffs"], deg, B, N, K, D, masks=f["masks"])
    assert_all_close(out.colors, f[f"colors_deg{deg}"], f.meta, f"colors_deg{deg}", f["masks"], D,
                     rtol_cap=NORTH_STAR_FWD_RTOL)


def test_sh_fwd_k25_deg4_matches_golden(backend):
    f = Fixture("sh_k25")
    B, N, K, D = _sh_dims(f)
    out = backend.sh_fwd(f["dirs"], f["coeffs"], 4, B, N, K, D)
    assert_all_close(out.colors, f["colors_deg4"], f.meta, "colors_deg4", rtol_cap=NORTH_STAR_FWD_RTOL)


def test_sh_bwd_matches_golden(backend):
    f = Fixture("sh_k16")
    B, N, K, D = _sh_dims(f)
    deg = int(f.m("degrees_to_use_bwd"))
    r1 = backend.sh_bwd(f["dirs"], f["coeffs"], f["v_colors"], deg, B, N, K, D, masks=f["masks"],
                        compute_v_dirs=True)
    assert_all_close(r1.v_coeffs, f["v_coeffs"], f.meta, "v_coeffs")
    assert_all_close(r1.v_dirs, f["v_dirs"], f.meta, "v_dirs")
    masked = f["masks"].ravel() == 0
    assert masked.any() and not np.any(r1.v_dirs.reshape(-1, 3)[masked])
    v_means = r1.v_dirs.reshape(B, N * 3).sum(axis=0)
    assert_all_close(v_means, f["v_means"], f.meta, "v_means")
    r2 = backend.sh_bwd(f["dirs"], f["coeffs"], f["v_colors"], deg, B, N, K, D, masks=f["masks"],
                        compute_v_dirs=True)
    assert rel_l2(r1.v_coeffs, r2.v_coeffs, f["v_coeffs"]) <= 0.1 * f.meta["tolerances"]["v_coeffs"]["rel_l2"]
    r3 = backend.sh_bwd(f["dirs"], f["coeffs"], f["v_colors"], deg, B, N, K, D, masks=f["masks"])
    assert_all_close(r3.v_coeffs, f["v_coeffs"], f.meta, "v_coeffs")
    assert r3.v_dirs.size == 0


def test_sh_bwd_b1_bit_deterministic(backend):
    f = Fixture("sh_k16")
    _, N, K, D = _sh_dims(f)
    dirs = f["dirs"][:1]
    vcol = f["v_colors"].reshape(2, -1)[:1]
    a = backend.sh_bwd(dirs, f["coeffs"], vcol, 3, 1, N, K, D, masks=f["masks"][:1], compute_v_dirs=True)
    b = backend.sh_bwd(dirs, f["coeffs"], vcol, 3, 1, N, K, D, masks=f["masks"][:1], compute_v_dirs=True)
    assert np.array_equal(a.v_coeffs, b.v_coeffs) and np.array_equal(a.v_dirs, b.v_dirs)


# ------------------------------------------------------------------ intersection (IsectTests.cpp)
def _isect(backend, f, accutile):
    kw = dict(conics=f["conics"], opacities=f["opacities"]) if accutile else {}
    return backend.isect_tiles(f["means2d"], f["radii"], f["depths"], int(f.m("I")), int(f.m("N")),
                               int(f.m("tile_size")), int(f.m("tile_width")),
                               int(f.m("tile_height")), **kw)


def _compare_isect(out, f):
    assert out.n_isects == int(f.m("n_isects"))
    assert out.tile_n_bits == int(f.m("tile_n_bits"))
    assert out.image_n_bits == int(f.m("image_n_bits"))
    assert np.array_equal(out.tiles_per_gauss.ravel(), f["tiles_per_gauss"].ravel())
    assert np.array_equal(out.isect_ids, join_u64(f["isect_ids_lo"], f["isect_ids_hi"]).ravel())
    assert np.array_equal(out.flatten_ids.ravel(), f["flatten_ids"].ravel())


@pytest.mark.parametrize("name,accutile", [("isect_std", False), ("isect_ties", False),
                                           ("isect_accutile", True)])
def test_isect_tiles_matches_golden(backend, name, accutile):
    f = Fixture(name)
    out = _isect(backend, f, accutile)
    _compare_isect(out, f)
    again = _isect(backend, f, accutile)
    assert np.array_equal(out.isect_ids, again.isect_ids)
    assert np.array_equal(out.flatten_ids, again.flatten_ids)


@pytest.mark.parametrize("name", ["isect_std", "isect_ties"])
def test_sort_and_offsets_match_golden(backend, name):
    f = Fixture(name)
    keys = join_u64(f["isect_ids_lo"], f["isect_ids_hi"]).ravel()
    bits = 32 + int(f.m("tile_n_bits")) + int(f.m("image_n_bits"))
    s = backend.sort_isect(keys, f["flatten_ids"].ravel(), bits)
    assert np.array_equal(s.keys_sorted, join_u64(f["isect_ids_sorted_lo"], f["isect_ids_sorted_hi"]).ravel())
    assert np.array_equal(s.values_sorted, f["flatten_ids_sorted"].ravel())
    off = backend.isect_offset_encode(s.keys_sorted, len(keys), int(f.m("I")),
                                      int(f.m("tile_width")), int(f.m("tile_height")))
    assert np.array_equal(off, f["offsets"].ravel())


def test_isect_chain_matches_golden(backend):
    f = Fixture("isect_std")
    out = _isect(backend, f, False)
    s = backend.sort_isect(out.isect_ids, out.flatten_ids, 32 + out.tile_n_bits + out.image_n_bits)
    assert np.array_equal(s.values_sorted, f["flatten_ids_sorted"].ravel())
    off = backend.isect_offset_encode(s.keys_sorted, out.n_isects, int(f.m("I")),
                                      int(f.m("tile_width")), int(f.m("tile_height")))
    assert np.array_equal(off, f["offsets"].ravel())


@pytest.mark.parametrize("n,bits", [(1, 40), (1023, 45), (1025, 64), (4097, 33), (300_001, 45),
                                    (3_000_000, 45)])
def test_sort_isect_stable_matches_numpy(backend, n, bits):
    rng = np.random.default_rng(n)
    keys = rng.integers(0, 1 << min(bits, 63), size=n, dtype=np.uint64)
    if bits == 64:
        keys |= (rng.integers(0, 2, size=n, dtype=np.uint64) << np.uint64(63))
    keys[rng.integers(0, n, size=n // 3)] = keys[0]  # plenty of ties
    vals = np.arange(n, dtype=np.int32)
    s = backend.sort_isect(keys, vals, bits)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(s.keys_sorted, keys[order])
    assert np.array_equal(s.values_sorted, vals[order])


@pytest.mark.parametrize("n", [1, 4095, 4096, 4097, 1_000_003, 5_000_011])
def test_prefix_scan_matches_cumsum(backend, n):
    rng = np.random.default_rng(n)
    v = rng.integers(0, 1 << 20, size=n, dtype=np.int32)
    assert np.array_equal(backend.prefix_scan_i64(v), np.cumsum(v, dtype=np.int64))


def test_prefix_scan_int32max_elements_promote(backend):
    v = np.full(4, np.iinfo(np.int32).max, np.int32)
    assert np.array_equal(backend.prefix_scan_i64(v), np.cumsum(v, dtype=np.int64))


def test_offset_encode_empty_is_zero(backend):
    off = backend.isect_offset_encode(np.zeros(0, np.uint64), 0, 2, 4, 3)
    assert off.shape == (24,) and not off.any()


# ------------------------------------------------------------------ raster (RasterTests.cpp)
RASTER = ["raster_small/nobg", "raster_small/bg", "raster_std", "raster_dense"]


def _raster_args(f):
    return dict(means2d=f["means2d"], conics=f["conics"], colors=f["colors"],
                opacities=f["opacities"], isect_offsets=f["isect_offsets"],
                flatten_ids=f["flatten_ids"], I=int(f.m("I")), N=int(f.m("N")),
                n_isects=int(f.m("n_isects")), image_width=int(f.m("width")),
                image_height=int(f.m("height")), tile_size=int(f.m("tile_size")),
                tile_width=int(f.m("tile_width")), tile_height=int(f.m("tile_height")),
                backgrounds=f["backgrounds"] if f.m("has_background") else None)


@pytest.mark.parametrize("name", RASTER)
def test_raster_fwd_matches_golden(backend, name):
    f = Fixture(name)
    out = backend.rasterize_fwd(**_raster_args(f))
    assert_all_close(out.render_colors, f["render_colors"], f.meta, "render_colors",
                     rtol_cap=NORTH_STAR_FWD_RTOL)
    assert_all_close(out.render_alphas, f["render_alphas"], f.meta, "render_alphas",
                     rtol_cap=NORTH_STAR_FWD_RTOL)
    assert np.array_equal(out.last_ids.ravel(), f["last_ids"].ravel())
    again = backend.rasterize_fwd(**_raster_args(f))
    assert np.array_equal(out.render_colors, again.render_colors)


@pytest.mark.parametrize("name", RASTER)
def test_raster_bwd_matches_golden(backend, name):
    f = Fixture(name)
    kw = dict(render_alphas=f["render_alphas"], last_ids=f["last_ids"],
              v_render_colors=f["v_render_colors"], v_render_alphas=f["v_render_alphas"])
    r1 = backend.rasterize_bwd(**_raster_args(f), **kw)
    for t in ("v_means2d", "v_conics", "v_colors", "v_opacities"):
        assert_all_close(getattr(r1, t), f[t], f.meta, t)
    r2 = backend.rasterize_bwd(**_raster_args(f), **kw)
    for t in ("v_means2d", "v_conics", "v_colors", "v_opacities"):
        assert rel_l2(getattr(r1, t), getattr(r2, t), f[t]) <= 0.1 * f.meta["tolerances"][t]["rel_l2"]
    r3 = backend.rasterize_bwd(**_raster_args(f), **kw, absgrad=True)
    assert np.all(r3.v_means2d_abs >= np.abs(r3.v_means2d) - 1e-6)


def test_raster_bwd_empty_is_zero(backend):
    f = Fixture("raster_small/nobg")
    a = _raster_args(f)
    a["n_isects"] = 0
    a["isect_offsets"] = np.zeros_like(f["isect_offsets"])
    r = backend.rasterize_bwd(**a, render_alphas=f["render_alphas"], last_ids=f["last_ids"],
                              v_render_colors=f["v_render_colors"], v_render_alphas=f["v_render_alphas"])
    assert not (r.v_means2d.any() or r.v_conics.any() or r.v_colors.any() or r.v_opacities.any())


def test_raster_rejects_tile_size(backend):
    f = Fixture("raster_small/nobg")
    a = _raster_args(f)
    a["tile_size"] = 8
    with pytest.raises(ValueError):
        backend.rasterize_fwd(**a)


# ------------------------------------------------------------------ SSIM (SsimTests.cpp)
def test_ssim_fwd_bwd_matches_golden(backend):
    f = Fixture("ssim_basic")
    I, H, W, C = 1, int(f.m("height")), int(f.m("width")), int(f.m("C"))
    o = backend.ssim_fwd(f["img1"], f["img2"], I, H, W, C, need_coeffs=True)
    assert_all_close(o.ssim_map, f["ssim_map"], f.meta, "ssim_map")
    assert_all_close([o.ssim], f["ssim"].ravel(), f.meta, "ssim")
    v = backend.ssim_bwd(f["img1"], f["img2"], I, H, W, C, o.coeff_mu, o.coeff_sigma,
                         o.coeff_cross, v_loss=1.0)
    assert_all_close(v, f["v_img1"], f.meta, "v_img1")
    o2 = backend.ssim_fwd(f["img1"], f["img2"], I, H, W, C, need_coeffs=True)
    assert np.array_equal(o.ssim_map, o2.ssim_map) and o.ssim == o2.ssim


def test_ssim_rejects_small_images(backend):
    img = np.zeros((1, 10, 12, 3), np.float32)
    with pytest.raises(ValueError):
        backend.ssim_fwd(img, img, 1, 10, 12, 3)


# ------------------------------------------------------------------ MCMC (McmcTests.cpp)
def test_rng_philox_kat_zero_counter(backend):
    # Random123 philox4x32-10 known answer for counter 0, key 0 (stream thread 0, offset 0, seed 0)
    u = backend.rng_philox_u32(0, 0, 4)
    assert [int(x) for x in u] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]


def test_rng_normal_finite_and_deterministic(backend):
    z = backend.rng_normal_f32(0xDEADBEEFCAFEF00D, 7, 1021)
    assert z.shape == (1021,) and np.isfinite(z).all()
    assert np.array_equal(z, backend.rng_normal_f32(0xDEADBEEFCAFEF00D, 7, 1021))
    assert not np.array_equal(z, backend.rng_normal_f32(0xDEADBEEFCAFEF00D, 8, 1021))
    big = backend.rng_normal_f32(42, 3, 1 << 20)
    assert abs(big.mean()) < 5e-3 and abs(big.std() - 1.0) < 5e-3


def test_mcmc_relocation_matches_golden(backend):
    f = Fixture("relocation_basic")
    o = backend.mcmc_relocation(f["opacities"], f["scales"], f["ratios"], f["binoms"],
                                n_max=int(f.m("n_max")), min_opacity=f.m("min_opacity"))
    assert_all_close(o.new_opacities, f["new_opacities"], f.meta, "new_opacities")
    assert_all_close(o.new_scales, f["new_scales"], f.meta, "new_scales")


def test_binoms_lut_matches_golden():
    from splatx_cuda.backend import make_binoms_lut
    f = Fixture("relocation_basic")
    assert np.array_equal(make_binoms_lut(51), f["binoms"].ravel())


def test_mcmc_perturb_matches_golden(backend):
    f = Fixture("perturb_basic")
    pos = f["positions"].copy()
    backend.mcmc_perturb_positions(pos, f["quats"], f["scales_log"], f["opacities_logit"],
                                   f["noise"], f.m("noise_scale"), f.m("t"), f.m("k"))
    assert_all_close(pos, f["positions_out"], f.meta, "positions_out")
