"""View-parallel training host logic on CPU: gloo ranks drive ViewParallelTrainer over a host
stand-in executor (numpy buffers, deterministic per-view gradients). Two ranks that split a step's
views must end where one rank that renders all of them ends — the shard plan, the reduce-scatter
into owner shards, the owner-shard Adam and the all-gather together are exact up to the order of
the gradient sums."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

from conftest import ROOT

PKG = ROOT / "splatx-metal_b200"

DIMS = [3, 4, 3, 1, 3, 9]  # SH degree 1
ROWS = 100


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class HostExecutor:
    """Stand-in with the executor's view-parallel methods; row-major buffers, so rows [r0, r1)
    of a group are the contiguous floats [r0*d, r1*d) exactly as in the CUDA executor's tiles."""

    def __init__(self, padded, count, seed=0):
        rng = np.random.default_rng(seed)
        self.padded, self.count = padded, count
        self.p = [rng.normal(size=padded * d).astype(np.float32) for d in DIMS]
        self.m = [np.zeros(padded * d, np.float32) for d in DIMS]
        self.v = [np.zeros(padded * d, np.float32) for d in DIMS]
        self.g = [np.zeros(padded * d, np.float32) for d in DIMS]
        self.vis = np.zeros(padded, np.float32)

    def step_accumulate(self, view):
        rows = np.arange(self.padded)
        seen = ((rows + view) % 3 != 0) & (rows < self.count)
        for gi, d in enumerate(DIMS):
            grad = np.sin(self.p[gi] * 0.5 + view).astype(np.float32)
            self.g[gi] += grad * np.repeat(seen, d).astype(np.float32)
        self.vis += seen

    def apply_grads(self, r0, r1, count, n_views, lr, opacity_reg_w=0.0, scale_reg_w=0.0,
                    inject_noise=False, noise_seed=0, noise_offset=0, noise_scale=0.0):
        for gi, d in enumerate(DIMS):
            for i in range(r0, r1):
                sl = slice(i * d, (i + 1) * d)
                if i < count and self.vis[i] > 0:
                    g = self.g[gi][sl] * np.float32(1.0 / n_views)
                    self.m[gi][sl] = np.float32(0.1) * g + np.float32(0.9) * self.m[gi][sl]
                    self.v[gi][sl] = np.float32(0.001) * g * g + np.float32(0.999) * self.v[gi][sl]
                    self.p[gi][sl] += -np.float32(lr[gi]) * self.m[gi][sl] / (np.sqrt(self.v[gi][sl]) + np.float32(1e-15))
                self.g[gi][sl] = 0
        self.vis[r0:r1] = 0

    def clear_grads(self):
        for g in self.g:
            g[:] = 0
        self.vis[:] = 0

    def resident_buffers(self):
        return {"params": self.p, "grads": self.g, "visibility": self.vis, "dims": DIMS,
                "padded_rows": self.padded}


def _worker(rank, world, port, views, steps, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, str(PKG))
    import torch
    import torch.distributed as dist
    from splatx_cuda.parallel import Collectives, ViewParallelTrainer, padded_rows
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ex = HostExecutor(padded_rows(ROWS, 2), ROWS)  # same padding for both runs
        tr = ViewParallelTrainer(ex, ROWS, Collectives(), tensor_of=lambda a, n: torch.from_numpy(a))
        lr = [1e-2, 1e-2, 5e-3, 5e-2, 2.5e-3, 1e-4]
        for _ in range(steps):
            for v in views[rank::world]:
                ex.step_accumulate(v)
            tr.exchange_and_apply(len(views), lr)
        if rank == 0:
            np.savez(out_path, *ex.p)
    finally:
        dist.destroy_process_group()


def _run(world, tmp_path, tag):
    import torch.multiprocessing as mp
    out = str(tmp_path / f"{tag}.npz")
    mp.start_processes(_worker, args=(world, _free_port(), [0, 1, 2, 3], 3, out), nprocs=world,
                       join=True, start_method="spawn")
    z = np.load(out)
    return [z[f"arr_{i}"] for i in range(len(DIMS))]


def test_shard_plan():
    from splatx_cuda.parallel import ShardPlan, padded_rows
    assert padded_rows(100, 2) == 128 and padded_rows(64, 2) == 64 and padded_rows(1, 8) == 256
    plan = ShardPlan(padded_rows(1000, 4), 4)
    spans = [plan.rows(r) for r in range(4)]
    assert spans[0][0] == 0 and spans[-1][1] == plan.padded
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert all((e - s) % 32 == 0 for s, e in spans)
    with pytest.raises(ValueError):
        ShardPlan(100, 2)


@pytest.mark.timeout(300)
def test_two_ranks_match_one_rank(tmp_path):
    one = _run(1, tmp_path, "w1")
    two = _run(2, tmp_path, "w2")
    for g in range(len(DIMS)):
        np.testing.assert_allclose(two[g], one[g], rtol=1e-5, atol=1e-6)
        assert not np.array_equal(one[g], HostExecutor(128, ROWS).p[g])  # training moved them
