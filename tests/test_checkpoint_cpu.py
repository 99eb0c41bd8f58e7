"""SXCK checkpoint headers and the resume fingerprint on the CPU (Checkpoint.cpp): our header
reader reads the reference's files, and the fingerprint check rejects the reference's mismatches
(every field) naming the field, and accepts equal configs."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from splatx_cuda.executor import checkpoint_info, verify_checkpoint_config

CFG = {"sh_degree": 1, "factor": 4, "test_split": 8, "total_iters": 7000, "mcmc_enabled": 1,
       "antialiased": 0, "cap_max": 2000, "mcmc_seed": 42, "scene_scale": 11.25, "ssim_weight": 0.2}


def _arrays(n, deg, seed=0):
    rng = np.random.default_rng(seed)
    dims = [3, 4, 3, 1, 3, ((deg + 1) ** 2 - 1) * 3]
    P = [rng.normal(0, 1, (n, d)).astype(np.float32) for d in dims]
    M = [rng.normal(0, 1e-3, (n, d)).astype(np.float32) for d in dims]
    V = [rng.uniform(0, 1e-6, (n, d)).astype(np.float32) for d in dims]
    return P, M, V


@pytest.mark.parametrize("fp16", [False, True])
def test_header_of_reference_file(tmp_path, fp16):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built here")
    P, M, V = _arrays(37, 1)
    oracle.ref_checkpoint_save(CFG, 123, P, M, V, tmp_path / "ck.sxck", fp16=fp16, rng="1 2 3")
    h = checkpoint_info(tmp_path / "ck.sxck")
    assert h["iter"] == 123 and h["alive_count"] == 37 and h["fp16"] == fp16 and h["version"] == 1
    for k, v in CFG.items():
        assert h["config"][k] == pytest.approx(v), k


def test_fingerprint_mismatches_name_the_field():
    verify_checkpoint_config(CFG, dict(CFG))
    for k, other in (("sh_degree", 3), ("factor", 2), ("test_split", 0), ("total_iters", 30000),
                     ("mcmc_enabled", 0), ("antialiased", 1), ("cap_max", 5), ("mcmc_seed", 7),
                     ("scene_scale", 1.0), ("ssim_weight", 0.0)):
        cur = dict(CFG, **{k: other})
        with pytest.raises(RuntimeError) as e:
            verify_checkpoint_config(CFG, cur)
        name = {"mcmc_enabled": "mcmc", "mcmc_seed": "mcmc seed"}.get(k, k)
        assert name in str(e.value), (k, str(e.value))
        if oracle.ref_available():
            with pytest.raises(ValueError) as r:
                oracle.ref_checkpoint_verify(CFG, cur)
            # the same field, the same saved/current values in the message
            assert str(e.value).split(" — ")[0] == str(r.value).split(" — ")[0]


def test_bad_files_are_rejected(tmp_path):
    p = tmp_path / "x.sxck"
    p.write_bytes(b"NOPE" + bytes(60))
    with pytest.raises(RuntimeError, match="bad magic"):
        checkpoint_info(p)
    p.write_bytes(b"SXCK" + np.uint32(2).tobytes() + bytes(60))
    with pytest.raises(RuntimeError, match="unsupported version"):
        checkpoint_info(p)
    p.write_bytes(b"SXCK" + np.uint32(1).tobytes())
    with pytest.raises(RuntimeError, match="truncated"):
        checkpoint_info(p)
