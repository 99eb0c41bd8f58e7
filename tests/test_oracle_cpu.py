"""CPU tests: the oracle against the reference's goldens and known answers, and against the
reference's own CPU kernels; the C-ABI boundary without a GPU.

The oracle (oracle/sx_oracle.c) is pinned here before any GPU test trusts it:
  * every golden fixture of the reference, with the reference's comparison rules (the same checks
    the GPU suite runs, re-used from test_kernels_golden_gpu with the oracle as backend);
  * the Random123 philox4x32-10 known-answer vectors and the uniform/Box-Muller boundaries the
    reference's McmcTests.cpp:44-106 checks;
  * bit-exact agreement with the reference's CPU kernels (oracle/_ref, compiled from the reference
    tree) on seeded scenes of config-0 shape — skipped where the reference tree was not present to
    build them; tests/golden/ref_cfg0.npz carries the same pin to machines without it.
"""
import ctypes as C
import pathlib

import numpy as np
import pytest

import test_kernels_golden_gpu as G
from helpers import Fixture, assert_all_close

oracle = pytest.importorskip("oracle")


@pytest.fixture(scope="module")
def ob():
    if not oracle.available():
        oracle.build()
    return oracle.OracleBackend()


# ------------------------------------------------------------------ goldens (same checks as GPU)
@pytest.mark.parametrize("masked", [False, True])
def test_oracle_adam_golden(ob, masked):
    G.test_fused_adam_matches_golden(ob, masked)


@pytest.mark.parametrize("variant", ["proj_fused_qs/c1", "proj_fused_qs/c2"])
def test_oracle_projection_fwd_golden(ob, variant):
    G.test_projection_fwd_qs_matches_golden(ob, variant)


def test_oracle_projection_fwd_covars_golden(ob):
    G.test_projection_fwd_covars_matches_golden(ob)


@pytest.mark.parametrize("variant", ["proj_fused_qs/c1", "proj_fused_qs/c2"])
def test_oracle_projection_bwd_golden(ob, variant):
    G.test_projection_bwd_matches_golden(ob, variant)


@pytest.mark.parametrize("deg", [0, 1, 2, 3])
def test_oracle_sh_fwd_golden(ob, deg):
    G.test_sh_fwd_k16_matches_golden(ob, deg)


def test_oracle_sh_fwd_deg4_golden(ob):
    G.test_sh_fwd_k25_deg4_matches_golden(ob)


def test_oracle_sh_bwd_golden(ob):
    G.test_sh_bwd_matches_golden(ob)


@pytest.mark.parametrize("name,accutile", [("isect_std", False), ("isect_ties", False),
                                           ("isect_accutile", True)])
def test_oracle_isect_golden(ob, name, accutile):
    G.test_isect_tiles_matches_golden(ob, name, accutile)


@pytest.mark.parametrize("name", ["isect_std", "isect_ties"])
def test_oracle_sort_offsets_golden(ob, name):
    G.test_sort_and_offsets_match_golden(ob, name)


def test_oracle_isect_chain_golden(ob):
    G.test_isect_chain_matches_golden(ob)


@pytest.mark.parametrize("n,bits", [(1, 40), (1023, 45), (1025, 64), (300_001, 45)])
def test_oracle_sort_stable(ob, n, bits):
    G.test_sort_isect_stable_matches_numpy(ob, n, bits)


@pytest.mark.parametrize("name", G.RASTER)
def test_oracle_raster_fwd_golden(ob, name):
    G.test_raster_fwd_matches_golden(ob, name)


@pytest.mark.parametrize("name", G.RASTER)
def test_oracle_raster_bwd_golden(ob, name):
    G.test_raster_bwd_matches_golden(ob, name)


def test_oracle_ssim_golden(ob):
    G.test_ssim_fwd_bwd_matches_golden(ob)


def test_oracle_relocation_golden(ob):
    G.test_mcmc_relocation_matches_golden(ob)


def test_oracle_perturb_golden(ob):
    G.test_mcmc_perturb_matches_golden(ob)


def test_oracle_binoms_golden():
    assert np.array_equal(oracle.make_binoms_lut(51), Fixture("relocation_basic")["binoms"].ravel())


# ------------------------------------------------------------------ known answers
KATS = [  # Random123 kat_vectors, philox4x32 10 rounds (counter, key, expected)
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,expected", KATS)
def test_oracle_philox_kat(ob, ctr, key, expected):
    assert [int(x) for x in ob.philox4x32_10(ctr, key)] == list(expected)


def test_oracle_rng_normal_finite_tail(ob):
    z = ob.rng_normal_f32(0xDEADBEEFCAFEF00D, 7, 1021)
    assert z.shape == (1021,) and np.isfinite(z).all()
    u = ob.rng_philox_u32(0, 0, 4)
    assert [int(x) for x in u] == list(KATS[0][2])


# ------------------------------------------------------------------ oracle == reference CPU code
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (no reference tree)")


def _scene(seed, n=2048, sh=3):
    import sys
    sys.path.insert(0, str(__import__("pathlib").Path(__file__).resolve().parents[1] / "splatx-metal_b200"))
    from splatx_cuda.scene import small_scene
    return small_scene(seed=seed, n=n, sh_degree=sh)


def _act(scene):
    s = np.exp(scene.scales).astype(np.float32)
    o = (np.float32(1) / (np.float32(1) + np.exp(-scene.opacities).astype(np.float32))).astype(np.float32)
    return s, o


@needs_ref
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_oracle_matches_reference_cpu_forward(ob, seed):
    """Projection, AccuTile/AABB intersection, stable sort, offsets, raster: bit for bit."""
    rb = oracle.RefBackend()
    scene, cam = _scene(seed)
    s, o = _act(scene)
    kw = dict(quats=scene.quats, scales=s, opacities=o, calc_compensations=True)
    pa = ob.projection_fused_fwd(scene.means, cam.viewmat, cam.K, cam.width, cam.height, **kw)
    pb = rb.projection_fused_fwd(scene.means, cam.viewmat, cam.K, cam.width, cam.height, **kw)
    for k in ("radii", "means2d", "depths", "conics", "compensations"):
        assert np.array_equal(getattr(pa, k), getattr(pb, k)), k
    for accu in (False, True):
        extra = dict(conics=pa.conics, opacities=o) if accu else {}
        ia = ob.isect_tiles(pa.means2d, pa.radii, pa.depths, 1, scene.count, 16, 16, 16, **extra)
        ib = rb.isect_tiles(pa.means2d, pa.radii, pa.depths, 1, scene.count, 16, 16, 16, **extra)
        assert ia.n_isects == ib.n_isects > 0
        assert np.array_equal(ia.tiles_per_gauss, ib.tiles_per_gauss)
        assert np.array_equal(ia.isect_ids, ib.isect_ids) and np.array_equal(ia.flatten_ids, ib.flatten_ids)
        sa = ob.sort_isect(ia.isect_ids, ia.flatten_ids, 32 + ia.tile_n_bits)
        sb = rb.sort_isect(ib.isect_ids, ib.flatten_ids, 32 + ib.tile_n_bits)
        assert np.array_equal(sa.keys_sorted, sb.keys_sorted) and np.array_equal(sa.values_sorted, sb.values_sorted)
        oa = ob.isect_offset_encode(sa.keys_sorted, ia.n_isects, 1, 16, 16)
        assert np.array_equal(oa, rb.isect_offset_encode(sb.keys_sorted, ib.n_isects, 1, 16, 16))
    colors = np.random.default_rng(seed).uniform(0, 1, scene.count * 3).astype(np.float32)
    ra = ob.rasterize_fwd(pa.means2d, pa.conics, colors, o, oa, sa.values_sorted, 1, scene.count,
                          ia.n_isects, 256, 256, 16, 16, 16)
    rbb = rb.rasterize_fwd(pa.means2d, pa.conics, colors, o, oa, sa.values_sorted, 1, scene.count,
                           ia.n_isects, 256, 256, 16, 16, 16)
    for k in ("render_colors", "render_alphas", "last_ids"):
        assert np.array_equal(getattr(ra, k), getattr(rbb, k)), k


@needs_ref
def test_oracle_matches_reference_cpu_misc(ob):
    rb = oracle.RefBackend()
    rng = np.random.default_rng(3)
    a = rng.uniform(0, 1, (1, 40, 52, 3)).astype(np.float32)
    b = rng.uniform(0, 1, (1, 40, 52, 3)).astype(np.float32)
    sa, sb = ob.ssim_fwd(a, b, 1, 40, 52, 3, True), rb.ssim_fwd(a, b, 1, 40, 52, 3, True)
    assert sa.ssim == sb.ssim
    for k in ("ssim_map", "coeff_mu", "coeff_sigma", "coeff_cross"):
        assert np.array_equal(getattr(sa, k), getattr(sb, k)), k
    assert np.array_equal(ob.rng_philox_u32(7, 99, 4099), rb.rng_philox_u32(7, 99, 4099))
    assert np.array_equal(ob.rng_normal_f32(7, 99, 4099), rb.rng_normal_f32(7, 99, 4099))
    f = Fixture("relocation_basic")
    x, y = ob.mcmc_relocation(f["opacities"], f["scales"], f["ratios"], f["binoms"]), \
        rb.mcmc_relocation(f["opacities"], f["scales"], f["ratios"], f["binoms"])
    assert np.array_equal(x.new_opacities, y.new_opacities) and np.array_equal(x.new_scales, y.new_scales)
    f = Fixture("perturb_basic")
    pa, pb = f["positions"].copy(), f["positions"].copy()
    args = (f["quats"], f["scales_log"], f["opacities_logit"], f["noise"], f.m("noise_scale"))
    ob.mcmc_perturb_positions(pa, *args)
    rb.mcmc_perturb_positions(pb, *args)
    assert np.array_equal(pa, pb)
    g = Fixture("adam_basic")
    for valid in (None, g["valid"]):
        p1, m1, v1 = g["param"].copy(), g["exp_avg"].copy(), g["exp_avg_sq"].copy()
        p2, m2, v2 = g["param"].copy(), g["exp_avg"].copy(), g["exp_avg_sq"].copy()
        kw = dict(valid=valid, n_gauss=1000, lr=0.01, b1=0.9, b2=0.999, eps=1e-8)
        ob.fused_adam(p1, g["grad"], m1, v1, **kw)
        rb.fused_adam(p2, g["grad"], m2, v2, **kw)
        assert np.array_equal(p1, p2) and np.array_equal(m1, m2) and np.array_equal(v1, v2)


def test_oracle_matches_committed_reference_vectors(ob):
    """tests/golden/ref_cfg0.npz: reference CPU outputs on a config-0 scene (make_ref_vectors.py)."""
    import json
    import pathlib
    d = pathlib.Path(__file__).resolve().parent / "golden"
    if not (d / "ref_cfg0.npz").exists():
        pytest.skip("ref_cfg0.npz not generated")
    r = dict(np.load(d / "ref_cfg0.npz"))
    meta = json.loads((d / "ref_cfg0.json").read_text())
    W, H = meta["width"], meta["height"]
    pa = ob.projection_fused_fwd(r["means"], r["viewmat"], r["K"], W, H, quats=r["quats"],
                                 scales=r["scales"], opacities=r["opacities"])
    for k in ("radii", "means2d", "depths", "conics"):
        assert np.array_equal(getattr(pa, k), r[k]), k
    ia = ob.isect_tiles(pa.means2d, pa.radii, pa.depths, 1, meta["N"], 16, meta["tile_width"],
                        meta["tile_height"], conics=pa.conics, opacities=r["opacities"])
    assert np.array_equal(ia.isect_ids, r["isect_ids"]) and np.array_equal(ia.flatten_ids, r["flatten_ids"])
    sa = ob.sort_isect(ia.isect_ids, ia.flatten_ids, 32 + ia.tile_n_bits)
    assert np.array_equal(sa.values_sorted, r["flatten_ids_sorted"])
    off = ob.isect_offset_encode(sa.keys_sorted, ia.n_isects, 1, meta["tile_width"], meta["tile_height"])
    assert np.array_equal(off, r["offsets"])
    ras = ob.rasterize_fwd(pa.means2d, pa.conics, r["colors"], r["opacities"], off, sa.values_sorted,
                           1, meta["N"], ia.n_isects, W, H, 16, meta["tile_width"], meta["tile_height"])
    assert np.array_equal(ras.render_colors, r["render_colors"])
    assert np.array_equal(ras.last_ids, r["last_ids"])


# ------------------------------------------------------------------ C-ABI boundary (no GPU)
def test_library_exports_every_declared_symbol():
    from splatx_cuda import _native
    L = _native.lib()
    declared = _native.declared_symbols()
    assert len(declared) >= 35
    for name in declared:
        assert hasattr(L, name), name
    assert set(declared) == set(_native._SIGNATURES)


def test_library_host_helpers():
    from splatx_cuda import _native
    from splatx_cuda.backend import make_binoms_lut
    L = _native.lib()
    assert L.sxcuda_abi_version() >= 1
    assert [L.sxcuda_bits_for_count(c) for c in (0, 1, 2, 8, 9, 8160, 4346)] == [0, 0, 1, 3, 4, 13, 13]
    assert np.array_equal(make_binoms_lut(51), oracle.make_binoms_lut(51))


def test_c_abi_rejects_contract_violations_without_touching_the_gpu():
    from splatx_cuda import _native as N
    L = N.lib()
    a = N.SxAdamInputs(None, None, None, None, None, 6, 4, 0.1, 0.9, 0.999, 1e-8)
    assert L.sxcuda_fused_adam(C.byref(a), None) == N.SXCUDA_EINVAL
    assert b"null tensor" in L.sxcuda_last_error()
    p = N.SxProjectionFusedInputs()
    p.camera_model = 1
    p.means = p.viewmats = p.Ks = C.c_void_p(16)
    assert L.sxcuda_projection_fused_fwd(C.byref(p), C.byref(N.SxProjectionFusedOutputs()), None) == N.SXCUDA_ERUNTIME
    sh = N.SxShInputs(C.c_void_p(16), C.c_void_p(16), None, 3, 1, 4, 9, 3, 0)
    assert L.sxcuda_sh_fwd(C.byref(sh), C.c_void_p(16), None) == N.SXCUDA_EINVAL  # (3+1)^2 > 9
    nbytes = C.c_size_t(0)
    assert L.sxcuda_sort_isect(None, None, None, None, 10, 65, None, C.byref(nbytes), None) == N.SXCUDA_EINVAL
    it = N.SxIsectTilesInputs(C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), None,
                              1, 4, 16, 4, 4)
    n = C.c_int64()
    assert L.sxcuda_isect_tile_count(C.byref(it), None, None, C.byref(n), None, C.byref(nbytes), None) == N.SXCUDA_EINVAL
    r = N.SxRasterizeFwdInputs(*([C.c_void_p(16)] * 8), 1, 4, 3, 32, 32, 8, 2, 2)
    assert L.sxcuda_rasterize_fwd(C.byref(r), C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), None) == N.SXCUDA_EINVAL
    s = N.SxSsimInputs(C.c_void_p(16), C.c_void_p(16), 1, 10, 20, 3, 0)
    assert L.sxcuda_ssim_fwd(C.byref(s), None, None, None, None, None, None, C.byref(nbytes), None) == N.SXCUDA_EINVAL
    d = N.SxTrainStepExecutorDesc(0, 3, 0.3, 0.01, 1e10, 0, 0.9, 0.999, 1e-15, 0.2, 0)
    h = C.c_void_p()
    assert L.sxcuda_executor_create(C.byref(d), 0, C.byref(h)) == N.SXCUDA_EINVAL
    assert L.sxcuda_rng_normal_f32(0, 0, -1, None, None) == N.SXCUDA_EINVAL
    assert L.sxcuda_prefix_scan_i64_noalloc(None, None, -5, None) == N.SXCUDA_EINVAL


def test_reference_runner_is_built_and_lists_its_tests():
    """The reference's test runner over the CUDA adapter links and lists its tests without a GPU
    (running them needs one: tests/test_reference_runner_gpu.py)."""
    import subprocess
    runner = pathlib.Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "splatx_ref_tests"
    if not runner.exists():
        pytest.skip("oracle/_ref/splatx_ref_tests not built (needs the reference checkout)")
    names = subprocess.run([str(runner), "--list"], capture_output=True, text=True, check=True).stdout.split()
    assert len(names) >= 99 and "trainer_resident_vs_host_step_contrast" in names
