"""Shared test helpers: golden fixture loading and the reference's comparison rules.

``assert_all_close`` restates the reference harness (Sources/SplatXTests/TestHarness.h:77-149):
tolerances come only from the fixture's meta (missing key = failure), NaN is a violation, an empty
comparison fails, and ``rel_l2`` (when present) is checked as ||a-e||/||e||.
"""
from __future__ import annotations

import json
import pathlib

import numpy as np

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


class Fixture:
    def __init__(self, name: str):
        tag = name.replace("/", "__")
        self.name = name
        self.t = dict(np.load(GOLDEN / f"{tag}.npz"))
        self.meta = json.loads((GOLDEN / f"{tag}.json").read_text())

    def __getitem__(self, k):
        return self.t[k]

    def __contains__(self, k):
        return k in self.t

    def m(self, k):
        return self.meta[k]


def tol(meta: dict, tensor: str) -> dict:
    t = meta.get("tolerances", {}).get(tensor)
    if t is None or "rtol" not in t or "atol" not in t:
        raise AssertionError(f"meta.json missing tolerances for '{tensor}'")
    return t


# The north star's forward bar (projection, SH and raster forward within 1e-5 relative of the
# goldens). Forward comparisons pass it as rtol_cap, so each is gated on the stricter of it and
# the fixture's own rtol; the fixture's atol still applies.
NORTH_STAR_FWD_RTOL = 1e-5


def assert_all_close(actual, expected, meta: dict, tensor: str, mask=None, mask_period: int = 1,
                     rtol_cap=None):
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    assert a.size == e.size, f"{tensor}: size {a.size} != {e.size}"
    t = dict(tol(meta, tensor))
    if rtol_cap is not None:
        t["rtol"] = min(t["rtol"], rtol_cap)
    if mask is not None:
        keep = np.repeat(np.asarray(mask).ravel() != 0, mask_period)
        a, e = a[keep], e[keep]
    assert a.size > 0, f"{tensor}: compared 0 elements (all masked or empty)"
    d = np.abs(a - e)
    bound = t["atol"] + t["rtol"] * np.abs(e)
    bad = ~(d <= bound)
    if bad.any():
        i = int(np.argmax(np.where(bad, d - bound, -np.inf)))
        raise AssertionError(f"{tensor}: allclose violated {int(bad.sum())}/{a.size} "
                             f"(rtol={t['rtol']} atol={t['atol']}), worst [{i}]: {a[i]!r} vs {e[i]!r}")
    if "rel_l2" in t:
        ref = float(np.sqrt(np.sum(e * e)))
        rel = float(np.sqrt(np.sum(d * d))) / ref if ref > 0 else float(np.sqrt(np.sum(d * d)))
        assert rel <= t["rel_l2"], f"{tensor}: rel_l2 {rel:.3g} > {t['rel_l2']}"


def rel_l2(a, b, ref) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    r = float(np.linalg.norm(np.asarray(ref, np.float64).ravel()))
    return float(np.linalg.norm(a - b)) / (r if r > 0 else 1.0)


def join_u64(lo, hi) -> np.ndarray:
    return (np.asarray(hi).astype(np.uint32).astype(np.uint64) << np.uint64(32)) | \
        np.asarray(lo).astype(np.uint32).astype(np.uint64)


def valid_mask(radii) -> np.ndarray:
    r = np.asarray(radii).reshape(-1, 2)
    return ((r[:, 0] > 0) & (r[:, 1] > 0)).astype(np.uint8)


def assert_step_close(got, ref, what, rel_l2_tol=1e-4, max_abs=1e-3):
    """One training step of two implementations: per-tensor relative L2 and max-abs bounds."""
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    r = rel_l2(got, ref, ref)
    assert r <= rel_l2_tol, (what, "rel_l2", r)
    m = float(np.abs(got - ref).max()) if got.size else 0.0
    assert m <= max_abs, (what, "max_abs", m)


# An entry whose reference exp_avg_sq is below this square has had only eps-sized gradients: with
# eps = 1e-15 its Adam step m / (sqrt(v) + eps) depends on the gradient's last bits (on the first
# step m / sqrt(v) = (1 - b1) / sqrt(1 - b2) sign(g) whatever |g| is), so two implementations whose
# float atomics sum a 1e-14 gradient to values 1e-15 apart move that parameter by visibly different
# amounts. Above it the step is insensitive to such differences.
ADAM_FIRM_SQRT_V = 1e-12


def adam_step_bound(lr, b1=0.9, b2=0.999):
    """The largest |change| of a parameter in one Adam step without bias correction: by
    Cauchy-Schwarz over the moment sums, |m| / sqrt(v) <= (1 - b1) / sqrt((1 - b2)(1 - b1^2 / b2))."""
    return lr * (1.0 - b1) / np.sqrt((1.0 - b2) * (1.0 - b1 * b1 / b2))


def assert_adam_params_close(got, ref, v_ref, lr, what, steps=1, rel_l2_tol=1e-4, max_abs=1e-3,
                             b1=0.9, b2=0.999):
    """Parameters after `steps` Adam steps of two implementations whose gradients agree up to the
    order of float atomics. rel-L2 over the whole tensor is the reference's host-vs-resident gate
    (TrainerTests.cpp:1712-1750). max-abs holds on every entry whose reference exp_avg_sq
    (v_ref) shows gradients above the eps scale (ADAM_FIRM_SQRT_V); the remaining entries, whose
    gradients were eps-sized throughout, are bounded by the largest change `steps` Adam steps can
    make. The split follows the reference's moments, so a wrong gradient (which is not eps-sized
    on the reference side) is held to max-abs."""
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    v = np.asarray(v_ref, np.float64).ravel()
    r = rel_l2(got, ref, ref)
    assert r <= rel_l2_tol, (what, "rel_l2", r)
    d = np.abs(got - ref)
    firm = np.sqrt(np.maximum(v, 0.0)) >= ADAM_FIRM_SQRT_V
    m = float(d[firm].max()) if firm.any() else 0.0
    assert m <= max_abs, (what, "max_abs", m)
    bound = 2.0 * steps * adam_step_bound(lr, b1, b2)
    assert float(d.max(initial=0.0)) <= bound * (1 + 1e-6), (what, "beyond the Adam step bound",
                                                            float(d.max()), bound)


def assert_trajectory_close(got, ref, what, rel_l2_tol=1e-3, max_abs=1e-2, v_ref=None, lr=None,
                            steps=None):
    """Parameters after several training steps of two implementations.

    Inputs that differ in the last bit (a float32 exp against a correctly rounded one, the order
    of the raster backward's float atomics) flip the occasional alpha-threshold or early-stop
    decision, and those small, deterministic changes compound over steps. The bounds are ten times
    the single-step ones; a wrong gradient or update is off by orders of magnitude more. With the
    reference's exp_avg_sq, learning rate and step count, the max-abs bound spares the entries
    whose gradients stayed eps-sized (assert_adam_params_close).
    """
    if v_ref is None:
        assert_step_close(got, ref, what, rel_l2_tol, max_abs)
    else:
        assert_adam_params_close(got, ref, v_ref, lr, what, steps, rel_l2_tol, max_abs)


def mcmc_cloud(op_act, cap, dims=(3, 4, 3, 1, 3, 9)):
    """McmcStrategyTests.cpp make_cloud: every component differs from row to row."""
    n = len(op_act)
    P = [np.zeros((cap, d), np.float32) for d in dims]
    i = np.arange(n, dtype=np.float32)[:, None]
    k3 = np.arange(3, dtype=np.float32)[None, :]
    P[0][:n] = i + np.float32(0.1) * k3
    P[2][:n] = np.log(np.float32(0.1) + np.float32(0.01) * i + np.float32(0.005) * k3)
    P[4][:n] = np.float32(0.05) * i + np.float32(0.01) * k3
    P[1][:n, 0] = 1.0
    P[1][:n, 1] = np.float32(0.01) * i[:, 0]
    p = np.asarray(op_act, np.float32)
    P[3][:n, 0] = np.log(p / (np.float32(1) - p))
    if dims[5]:
        P[5][:n] = -np.float32(0.02) * i - np.float32(0.001) * np.arange(dims[5], dtype=np.float32)[None, :]
    return P


def mcmc_random_cloud(rng, n, cap, sh_degree=3, dead_frac=0.1):
    """A random arena of cap rows, n alive, about dead_frac of them dead (sigmoid <= 0.005),
    with non-zero moments."""
    K3 = ((sh_degree + 1) ** 2 - 1) * 3
    dims = [3, 4, 3, 1, 3, K3]
    P = [np.zeros((cap, d), np.float32) for d in dims]
    M = [np.zeros((cap, d), np.float32) for d in dims]
    V = [np.zeros((cap, d), np.float32) for d in dims]
    P[0][:n] = rng.normal(0, 1, (n, 3))
    P[1][:n] = rng.normal(0, 1, (n, 4))
    P[2][:n] = rng.normal(-3, 0.5, (n, 3))
    logit = rng.normal(0, 1.5, n).astype(np.float32)
    dead = rng.random(n) < dead_frac
    logit[dead] = rng.uniform(-9, -5.3, int(dead.sum()))  # sigmoid <= 0.005
    P[3][:n, 0] = logit
    P[4][:n] = rng.normal(0, 0.5, (n, 3))
    if K3:
        P[5][:n] = rng.normal(0, 0.1, (n, K3))
    for g in range(6):
        M[g][:n] = rng.normal(0, 1e-3, (n, dims[g]))
        V[g][:n] = rng.uniform(0, 1e-6, (n, dims[g]))
    return P, M, V
