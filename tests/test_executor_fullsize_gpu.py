"""The benchmarked resident step against the CPU oracle at the benchmarked size.

bench.py times the executor's own kernels (fwd_gauss, the single-sweep depth sort, the supertile
emit, sort and binning that build the tile lists, the fused L1+SSIM loss, bwd_sh/bwd_geom). These
tests read the executor's
intermediate tensors after a step (sxcuda_executor_read_gaussians / _read_isects / _read_images)
and compare each stage with the oracle run on the same inputs — the reference's host-vs-resident
contrast (Sources/SplatXTests/TrainerTests.cpp:1720-1750) taken apart stage by stage:

  * per-Gaussian forward outputs: bit-identical to the API projection kernel on the same
    activations (which is itself pinned to the oracle), AccuTile tile counts bit-identical to the
    oracle's count, colours within 1e-5 of the oracle's SH;
  * the depth order: the stable ascending sort of the depth keys, ties by Gaussian id;
  * the tile-sorted flatten_ids and the tile offsets: bit-identical to the oracle's
    isect_tiles -> sort_isect -> isect_offset_encode on the same projection outputs (the
    reference's 45-bit key sort, IsectTests.cpp:161 / SortTests.cpp:139);
  * render / alpha / last_ids: within 1e-5 of the oracle's rasterize_fwd on the executor's lists,
    with the documented flip budget for alpha-threshold and early-stop decisions;
  * v_render and the loss: the oracle's host loss (L1 + SSIM) on the executor's render;
  * one whole step: both Adam moments against the oracle's Trainer::step host path (rel-L2 1e-4,
    max-abs 1e-3), parameters at the reference's rel-L2 1e-4 gate with max-abs 1e-3 wherever the
    reference's exp_avg_sq is above the eps scale (helpers.assert_adam_params_close), loss within
    1e-6 + 1e-4 |L|,
    n_isects equal up to the radius flips of the float expf activation, counted and bounded;
  * v_render (a gradient) at rel-L2 1e-4, max-abs 1e-4 of its largest value.

The other way to the tile lists (set_tile_lists(1): every (tile, Gaussian) pair emitted in depth
order and sorted stably by tile, the path for grids beyond 16,384 supertiles) must give the same
lists bit for bit.

Scenes: config 2 (1M Gaussians, SH 3, 1297x840: 77 supertiles, a 13-bit tile key in two passes on
the pair-sort path, 245 depth-sort tiles, an image width that is no multiple of the loss tiles),
a tied-depth scene modelled on
fixtures/isect_ties (groups of Gaussians at exactly the same depth over shared tiles) on an odd
257x131 image, and the same at SH degree 0.
A scene of large footprints (1,500 Gaussians tens of tiles across on the config-2 camera) drives
the supertile binning into its fallbacks: blocks of strips over more than four supertiles and
write rounds holding more intersections than the per-warp slot list.
"""
import numpy as np
import pytest

from helpers import assert_adam_params_close, assert_step_close, rel_l2

pytestmark = pytest.mark.gpu
oracle = pytest.importorskip("oracle")

LR = [1.6e-4, 1e-3, 5e-3, 5e-2, 2.5e-3, 2.5e-3 / 20]


@pytest.fixture(scope="module")
def ob():
    if not oracle.available():
        oracle.build()
    return oracle.OracleBackend()


def _act_cr(log_scales, logits):
    """The executor's activations: exp evaluated in double and rounded once to float."""
    s = np.exp(np.asarray(log_scales, np.float64).ravel()).astype(np.float32)
    e = np.exp(-np.asarray(logits, np.float64).ravel()).astype(np.float32)
    o = (np.float32(1) / (np.float32(1) + e)).astype(np.float32)
    return s, o


def _fwd_close(a, b, what, rtol=1e-5, atol=1e-6, flip_budget=1e-5, flip_abs=5e-3):
    """Images within rtol/atol, except a budget of pixels where the alpha >= 1/255 gate or the
    exclusive early stop flips on a last-ulp difference of exp (a discontinuity of the contract)."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    d = np.abs(a - b)
    bad = d > atol + rtol * np.abs(b)
    assert bad.mean() <= flip_budget, f"{what}: {int(bad.sum())} of {a.size} beyond tolerance"
    assert d.max() <= flip_abs, f"{what}: max abs diff {d.max():.3g}"


class Run:
    """One resident step of a scene, its intermediate tensors, and the oracle's host step."""

    def __init__(self, scene, cam, gt, sh, ssim_weight=0.2):
        from splatx_cuda.executor import TrainStepExecutor
        n = scene.count
        self.scene, self.cam, self.gt, self.sh, self.n = scene, cam, gt, sh, n
        self.tw, self.th = (cam.width + 15) // 16, (cam.height + 15) // 16
        P = [np.ascontiguousarray(g.reshape(n, -1)).copy() for g in scene.groups()]
        self.P0 = [x.copy() for x in P]
        Z = [np.zeros_like(x) for x in P]
        ex = TrainStepExecutor(n, sh, ssim_weight=ssim_weight)
        try:
            ex.upload_params(P, Z, Z, n)
            self.loss, self.n_isects, _ = ex.step(cam.viewmat, cam.K, cam.width, cam.height, gt, n,
                                                  degrees_to_use=sh, lr=LR)
            self.g = ex.read_gaussians()
            self.isects = ex.read_isects()
            self.img = ex.read_images(cam.width, cam.height)
            self.bin_stats = ex.bin_stats()
            self.G = [np.zeros_like(x) for x in P]
            self.M1 = [np.zeros_like(x) for x in P]
            self.M2 = [np.zeros_like(x) for x in P]
            ex.download_params(self.G, self.M1, self.M2, n)
        finally:
            ex.close()
        # the oracle's Trainer::step host path from the same parameters
        self.R = [x.copy() for x in self.P0]
        self.RM1 = [np.zeros_like(x) for x in P]
        self.RM2 = [np.zeros_like(x) for x in P]
        self.ref = oracle.host_step(self.R, cam, gt, sh, sh, LR, self.RM1, self.RM2,
                                    ssim_weight=ssim_weight)
        self.memo = {}

    def api_projection(self, backend):
        s, o = _act_cr(self.P0[2], self.P0[3])
        p = backend.projection_fused_fwd(self.P0[0], self.cam.viewmat, self.cam.K, self.cam.width,
                                         self.cam.height, quats=self.P0[1], scales=s, opacities=o)
        return p, s, o


def _target(scene_hidden, cam):
    """The render of a hidden scene (the bench's kind of target), by the executor's forward."""
    from splatx_cuda.executor import TrainStepExecutor
    n = scene_hidden.count
    ex = TrainStepExecutor(n, scene_hidden.sh_degree)
    z = [np.zeros((n, d), np.float32) for d in ex.dims]
    ex.upload_params([np.ascontiguousarray(g.reshape(n, -1)) for g in scene_hidden.groups()], z, z, n)
    _, _, gt = ex.step(cam.viewmat, cam.K, cam.width, cam.height, None, n,
                       degrees_to_use=scene_hidden.sh_degree, forward_only=True, want_render=True)
    ex.close()
    return gt


@pytest.fixture(scope="module")
def cfg2():
    from splatx_cuda.scene import large_scene
    scene, cam = large_scene(seed=0, n=1_000_000, sh_degree=3)
    hidden, _ = large_scene(seed=1, n=200_000, sh_degree=3)
    return Run(scene, cam, _target(hidden, cam), 3)


def tie_scene(n, sh_degree, width=257, height=131, seed=31):
    """Groups of Gaussians at exactly the same camera depth over shared tiles (the tie structure
    of fixtures/isect_ties: equal (tile, depth) keys that only the Gaussian id orders), plus a
    spread of distinct depths, before an identity camera on an odd-sized image."""
    from splatx_cuda.scene import Camera, Scene
    rng = np.random.default_rng(seed)
    fx = 180.0
    depth_set = np.array([2.0, 2.0, 2.0, 3.0, 1.5, 7.25], np.float32)  # exact in float
    z = depth_set[rng.integers(0, depth_set.size, n)]
    spread = rng.random(n) < 0.25
    z[spread] = rng.uniform(1.5, 8.0, int(spread.sum())).astype(np.float32)
    # image-plane positions on a coarse lattice so tied Gaussians share tiles
    u = rng.integers(0, 12, n) * (width / 12.0) + rng.uniform(-6, 6, n)
    v = rng.integers(0, 6, n) * (height / 6.0) + rng.uniform(-6, 6, n)
    means = np.stack([(u - width / 2) / fx * z, (v - height / 2) / fx * z, z], 1).astype(np.float32)
    means[:, 2] = z  # keep the depth bits exact
    q = rng.normal(0, 1, (n, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    s = rng.normal(-3.2, 0.4, (n, 3)).astype(np.float32) + np.log(z)[:, None].astype(np.float32)
    o = rng.normal(0.5, 1.0, n).astype(np.float32)
    sh0 = rng.normal(0, 0.5, (n, 3)).astype(np.float32)
    K = (sh_degree + 1) ** 2
    shN = rng.normal(0, 0.1, (n, K - 1, 3)).astype(np.float32)
    cam = Camera(np.eye(4, dtype=np.float32).ravel(),
                 np.array([fx, 0, width / 2, 0, fx, height / 2, 0, 0, 1], np.float32), width, height)
    return Scene(means, q, s.astype(np.float32), o, sh0, shN, sh_degree), cam


@pytest.fixture(scope="module", params=[3, 0], ids=["sh3", "sh0"])
def ties(request):
    scene, cam = tie_scene(6000, request.param)
    gt = np.random.default_rng(32).uniform(0, 1, cam.width * cam.height * 3).astype(np.float32)
    return Run(scene, cam, gt, request.param)


def big_scene(n=1500, sh_degree=1, seed=41):
    """Large footprints on the config-2 camera: Gaussians of 0.5-2 world units near the origin
    (tens of tiles across each), so the supertile emit meets blocks of strips over more than four
    supertiles and the binning's write kernel meets rounds of 32 entries holding more than 512
    intersections."""
    from splatx_cuda.scene import Scene, large_camera
    rng = np.random.default_rng(seed)
    means = np.stack([rng.normal(0, 1.2, n), rng.normal(0, 0.8, n), rng.normal(0, 1.0, n)],
                     1).astype(np.float32)
    q = rng.normal(0, 1, (n, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    s = rng.normal(np.log(0.8), 0.35, (n, 3)).astype(np.float32)
    o = rng.normal(-1.0, 1.0, n).astype(np.float32)
    sh0 = rng.normal(0, 0.5, (n, 3)).astype(np.float32)
    K = (sh_degree + 1) ** 2
    shN = rng.normal(0, 0.1, (n, K - 1, 3)).astype(np.float32)
    return Scene(means, q, s, o, sh0, shN, sh_degree), large_camera()


@pytest.fixture(scope="module")
def big():
    scene, cam = big_scene()
    gt = np.random.default_rng(42).uniform(0, 1, cam.width * cam.height * 3).astype(np.float32)
    return Run(scene, cam, gt, scene.sh_degree)


def _runs(request, names):
    return [request.getfixturevalue(n) for n in names]


# ------------------------------------------------------------------ per-Gaussian forward outputs
def _check_forward_gaussians(run, backend, ob):
    if "fwd" in run.memo:
        return run.memo["fwd"]
    p, s, o = run.api_projection(backend)
    g = run.g
    valid = (p.radii.reshape(-1, 2) > 0).all(1)
    assert np.array_equal(g["valid"].astype(bool), valid)
    assert valid.sum() > 0
    assert np.array_equal(g["means2d"][valid], p.means2d.reshape(-1, 2)[valid])
    assert np.array_equal(g["conics"][valid], p.conics.reshape(-1, 3)[valid])
    assert np.array_equal(g["opacities"], o)
    # AccuTile tile counts: the oracle's count on the same projection
    it = ob.isect_tiles(p.means2d, p.radii, p.depths, 1, run.n, 16, run.tw, run.th,
                        conics=p.conics, opacities=o)
    assert np.array_equal(g["tiles_per_gauss"], it.tiles_per_gauss)
    has = it.tiles_per_gauss > 0
    dk = np.full(run.n, 0xFFFFFFFF, np.uint32)
    dk[has] = p.depths.reshape(-1)[has].view(np.uint32)
    assert np.array_equal(g["depth_keys"], dk)
    # colours: SH + 0.5, clamped at 0, on the valid rows
    n = run.n
    vm = run.cam.viewmat.reshape(4, 4)
    campos = np.array([-(vm[0, i] * vm[0, 3] + vm[1, i] * vm[1, 3] + vm[2, i] * vm[2, 3])
                       for i in range(3)], np.float32)
    dirs = (run.P0[0] - campos).astype(np.float32)
    K = (run.sh + 1) ** 2
    coeffs = np.concatenate([run.P0[4].reshape(n, 1, 3), run.P0[5].reshape(n, K - 1, 3)], axis=1)
    col = ob.sh_fwd(dirs, coeffs, run.sh, 1, n, K, 3, masks=valid.astype(np.uint8)).colors
    col = np.maximum(col.reshape(n, 3) + np.float32(0.5), np.float32(0))
    np.testing.assert_allclose(g["colors"][valid], col[valid], rtol=1e-5, atol=1e-6)
    run.memo["fwd"] = (p, o, it)
    return p, o, it


def _check_depth_order(run):
    keys = run.g["depth_keys"]
    ref = np.lexsort((np.arange(run.n), keys)).astype(np.int32)  # stable: ties by id
    assert np.array_equal(run.g["depth_order"], ref)


def _check_isects(run, ob, p, o, it):
    if "isects" in run.memo:
        return run.memo["isects"]
    tw, th = run.tw, run.th
    assert run.isects["n_isects"] == it.n_isects == run.n_isects
    bits = 32 + it.tile_n_bits + it.image_n_bits
    st = ob.sort_isect(it.isect_ids, it.flatten_ids, bits)
    off = ob.isect_offset_encode(st.keys_sorted, it.n_isects, 1, tw, th)
    ids = run.isects["flatten_ids"]
    assert np.array_equal(ids, st.values_sorted)
    assert np.array_equal(run.isects["offsets"], off)
    # the executor never materialises the 45-bit keys; rebuild them from its list and compare
    n_tiles = tw * th
    ends = np.append(off[1:], it.n_isects).astype(np.int64)
    tile_of = np.repeat(np.arange(n_tiles, dtype=np.uint64), ends - off.astype(np.int64))
    keys = (tile_of << np.uint64(32)) | p.depths.reshape(-1)[ids].view(np.uint32).astype(np.uint64)
    assert np.array_equal(keys, st.keys_sorted)
    run.memo["isects"] = (st, off)
    return st, off


def _check_entries(run, it):
    """The emit writes exactly one entry per (Gaussian, supertile) that holds some of the
    Gaussian's tiles — none empty, so entries never outnumber intersections."""
    tile = (it.isect_ids >> np.uint64(32)).astype(np.int64) & ((1 << it.tile_n_bits) - 1)
    g = it.flatten_ids.astype(np.int64)
    stw = (run.tw + 7) // 8
    st = (tile // run.tw // 8) * stw + (tile % run.tw) // 8
    distinct = np.unique(g * (stw * ((run.th + 7) // 8)) + st).size
    assert run.bin_stats[0] == distinct, (run.bin_stats, distinct)


def _check_raster(run, ob, o, st, off):
    cam = run.cam
    c = ob.rasterize_fwd(run.g["means2d"], run.g["conics"], run.g["colors"], o, off,
                         st.values_sorted, 1, run.n, run.n_isects, cam.width, cam.height, 16,
                         run.tw, run.th)
    _fwd_close(run.img["render"], c.render_colors, "render_colors")
    _fwd_close(run.img["alpha"], c.render_alphas, "render_alphas")
    flips = float(np.mean(run.img["last_ids"] != c.last_ids))
    print(f"last_ids differing: {flips:.2e} of pixels")
    assert flips <= 1e-4


def _check_loss(run, ssim_weight=0.2):
    cam = run.cam
    loss, v = oracle.train_loss(run.img["render"], run.gt, cam.width, cam.height, ssim_weight)
    assert abs(run.loss - loss) <= 1e-6 + 1e-4 * abs(loss), (run.loss, loss)
    got = run.img["v_render"]
    # v = 0.8 sign(r - gt) / n + SSIM term: the same render, so the signs agree exactly; the SSIM
    # term differs by float summation order only
    r = rel_l2(got, v, v)
    m = float(np.abs(got.astype(np.float64) - v).max())
    print(f"v_render rel-L2 {r:.3g}, max-abs {m:.3g} (max |v| {np.abs(v).max():.3g})")
    assert r <= 1e-4 and m <= 1e-4 * float(np.abs(v).max())


def _radius_flips(run, ob):
    """Gaussians whose tile count differs between the oracle's float-expf activations and the
    executor's correctly rounded ones (the only source of n_isects differences)."""
    s, o = oracle.train_activations(run.P0[2], run.P0[3])
    cam = run.cam
    p = ob.projection_fused_fwd(run.P0[0], cam.viewmat, cam.K, cam.width, cam.height,
                                quats=run.P0[1], scales=s, opacities=o)
    it = ob.isect_tiles(p.means2d, p.radii, p.depths, 1, run.n, 16, run.tw, run.th,
                        conics=p.conics, opacities=o)
    return int(np.sum(it.tiles_per_gauss != run.g["tiles_per_gauss"])), it.n_isects


def _check_step(run, ob):
    flips, n_oracle = _radius_flips(run, ob)
    print(f"radius/tile-count flips vs the oracle's expf activations: {flips}; "
          f"n_isects {run.n_isects} vs {run.ref['n_isects']}")
    assert n_oracle == run.ref["n_isects"]
    assert flips <= 5
    if flips == 0:
        assert run.n_isects == run.ref["n_isects"]
    L = run.ref["loss"]
    assert abs(run.loss - L) <= 1e-6 + 1e-4 * abs(L), (run.loss, L)
    for gi in range(6):
        if run.P0[gi].size == 0:
            continue
        d = np.abs(run.G[gi].astype(np.float64) - run.R[gi]).ravel()
        g_ref = np.abs(run.RM1[gi].astype(np.float64).ravel()) * 10.0  # |grad| = |m1| / (1 - b1)
        g_got = np.abs(run.M1[gi].astype(np.float64).ravel()) * 10.0
        big = d > 1e-3
        print(f"group {gi}: params rel-L2 {rel_l2(run.G[gi], run.R[gi], run.R[gi]):.3g} max-abs "
              f"{d.max():.3g}; {int(big.sum())} entries > 1e-3; grad rms {np.sqrt(np.mean(g_ref**2)):.3g}"
              f" max {g_ref.max():.3g}")
        if big.any():
            idx = np.flatnonzero(big)[:8]
            for i in idx:
                print(f"   [{i}] p {run.G[gi].ravel()[i]:.6g} vs {run.R[gi].ravel()[i]:.6g}; grad "
                      f"{run.M1[gi].ravel()[i] * 10:.4g} vs {run.RM1[gi].ravel()[i] * 10:.4g}; "
                      f"p0 {run.P0[gi].ravel()[i]:.6g}")
        assert_step_close(run.M1[gi], run.RM1[gi], ("exp_avg", gi))
        assert_step_close(run.M2[gi], run.RM2[gi], ("exp_avg_sq", gi))
    for gi in range(6):
        if run.P0[gi].size:
            assert_adam_params_close(run.G[gi], run.R[gi], run.RM2[gi], LR[gi], ("params", gi))


# ------------------------------------------------------------------ config 2, full size
def test_cfg2_forward_gaussians_match_api_projection_and_oracle(backend, ob, cfg2):
    _check_forward_gaussians(cfg2, backend, ob)


def test_cfg2_depth_order_is_the_stable_depth_sort(cfg2):
    assert cfg2.n == 1_000_000
    _check_depth_order(cfg2)


def test_cfg2_sorted_isects_and_offsets_bit_exact(backend, ob, cfg2):
    p, o, it = _check_forward_gaussians(cfg2, backend, ob)
    assert it.n_isects > 5_000_000 and it.tile_n_bits == 13
    _check_isects(cfg2, ob, p, o, it)
    _check_entries(cfg2, it)


def test_cfg2_raster_forward_matches_oracle(backend, ob, cfg2):
    p, o, it = _check_forward_gaussians(cfg2, backend, ob)
    st, off = _check_isects(cfg2, ob, p, o, it)
    _check_raster(cfg2, ob, o, st, off)


def test_cfg2_loss_and_v_render_match_oracle(cfg2):
    _check_loss(cfg2)


def test_cfg2_whole_step_matches_oracle_host_step(ob, cfg2):
    _check_step(cfg2, ob)


# ------------------------------------------------------------------ tied depths, odd image
def test_ties_forward_chain_bit_exact(backend, ob, ties):
    p, o, it = _check_forward_gaussians(ties, backend, ob)
    _check_depth_order(ties)
    keys = ties.g["depth_keys"][ties.g["tiles_per_gauss"] > 0]
    _, counts = np.unique(keys, return_counts=True)
    assert counts.max() >= 500  # large tie groups reach the sorts
    st, off = _check_isects(ties, ob, p, o, it)
    _check_entries(ties, it)
    _check_raster(ties, ob, o, st, off)


def test_ties_loss_and_step_match_oracle(ob, ties):
    _check_loss(ties)
    _check_step(ties, ob)


# ------------------------------------------------------------------ the two ways to the tile lists
def _executor_lists(run, mode):
    """One executor step of `run`'s scene with tile-list mode `mode`: its lists and images."""
    from splatx_cuda.executor import TrainStepExecutor
    n = run.n
    Z = [np.zeros_like(x) for x in run.P0]
    ex = TrainStepExecutor(n, run.sh)
    try:
        ex.set_tile_lists(mode)
        ex.upload_params([x.copy() for x in run.P0], Z, Z, n)
        loss, n_isects, _ = ex.step(run.cam.viewmat, run.cam.K, run.cam.width, run.cam.height,
                                    run.gt, n, degrees_to_use=run.sh, lr=LR)
        return loss, n_isects, ex.read_isects(), ex.read_images(run.cam.width, run.cam.height)
    finally:
        ex.close()


def _check_pair_sort_equals_binning(run):
    """Mode 1 (emit every (tile, Gaussian) pair, sort stably by tile) and the default supertile
    binning give bit-identical flatten_ids and tile offsets, hence identical forward images."""
    loss, n_isects, isects, img = _executor_lists(run, 1)
    assert n_isects == run.n_isects
    for k in isects:
        assert np.array_equal(isects[k], run.isects[k]), k
    for k in ("render", "alpha", "last_ids"):
        assert np.array_equal(img[k], run.img[k]), k
    assert abs(loss - run.loss) <= 1e-6 * abs(run.loss)  # the loss reduction sums in any order


def test_cfg2_pair_sort_and_binning_build_the_same_lists(cfg2):
    _check_pair_sort_equals_binning(cfg2)


def test_ties_pair_sort_and_binning_build_the_same_lists(ties):
    _check_pair_sort_equals_binning(ties)


def test_tile_list_mode_is_checked():
    from splatx_cuda.executor import TrainStepExecutor
    ex = TrainStepExecutor(64, 0)
    try:
        with pytest.raises(Exception, match="mode must be 0 or 1"):
            ex.set_tile_lists(2)
    finally:
        ex.close()


# ------------------------------------------------------------------ large footprints
def _binning_extremes(run, it):
    """From the oracle's lists: the widest block of 8 sweep strips in supertiles (the sweep runs
    along a footprint's shorter axis, so a footprint 33+ tiles across in both directions has
    one over five supertiles), and the most intersections any round of 32 consecutive entries of
    one supertile holds."""
    tw = run.tw
    tile = (it.isect_ids >> np.uint64(32)).astype(np.int64) & ((1 << it.tile_n_bits) - 1)
    g = it.flatten_ids.astype(np.int64)
    tx, ty = tile % tw, tile // tw
    span = np.zeros(run.n, np.int64)
    for a, b in ((tx, ty), (ty, tx)):  # per Gaussian: extent along each axis, take the smaller
        lo = np.full(run.n, 1 << 30); hi = np.full(run.n, -1)
        np.minimum.at(lo, g, a); np.maximum.at(hi, g, a)
        ext = hi - lo + 1
        span = ext if span.sum() == 0 else np.minimum(span, ext)
    stw = (tw + 7) // 8
    st = (ty // 8) * stw + tx // 8
    entry = np.unique(g * 100000 + st)
    pairs = np.bincount(np.searchsorted(entry, g * 100000 + st), minlength=entry.size)
    est = entry % 100000
    depth = np.zeros(run.n, np.uint64)
    depth[g] = it.isect_ids[np.arange(g.size)] & np.uint64(0xffffffff)
    order = np.lexsort((entry // 100000, depth[entry // 100000], est))
    p_sorted, st_sorted = pairs[order], est[order]
    worst = 0
    for s_ in np.unique(st_sorted):
        run_p = p_sorted[st_sorted == s_]
        for r0 in range(0, run_p.size, 64):  # the write kernel's chunks of 64, rounds of 32
            for k in (r0, r0 + 32):
                worst = max(worst, int(run_p[k:min(k + 32, r0 + 64)].sum()))
    return int(span.max()), worst


def test_big_footprints_isects_bit_exact_and_binning_fallbacks_reached(backend, ob, big):
    p, o, it = _check_forward_gaussians(big, backend, ob)
    widest, worst_round = _binning_extremes(big, it)
    assert widest >= 40, widest            # some block of strips spans more than 4 supertiles
    assert worst_round > 512, worst_round  # some round overflows the write kernel's slot list
    st, off = _check_isects(big, ob, p, o, it)
    _check_entries(big, it)
    _check_raster(big, ob, o, st, off)


def test_big_footprints_pair_sort_and_binning_build_the_same_lists(big):
    _check_pair_sort_equals_binning(big)

