"""View-parallel training on two GPUs: the fused peer-memory exchange (stream-ordered NCCL
barriers, or overlapped with the last backward behind device barriers) against the NCCL exchange.

Both ranks render their own views; after several steps the parameters of the two exchanges agree
within the step tolerance (the gradient sums run in different orders), and with the peer exchange
every rank's replica is bit-identical (each row is written by its one owner). Skipped with fewer
than two GPUs; the ranks are child processes on 127.0.0.1 with NVLS off.
"""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

PKG = ROOT / "splatx-metal_b200"
LR = [1.6e-4, 1e-3, 5e-3, 5e-2, 2.5e-3, 2.5e-3 / 20]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, exchange, steps, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, str(PKG))
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from splatx_cuda.executor import TrainStepExecutor
    from splatx_cuda.parallel import (Collectives, PeerExchangeTrainer, ViewParallelTrainer,
                                      padded_rows)
    from splatx_cuda.scene import small_scene
    n, sh = 6000, 1
    scene, cam = small_scene(seed=41, n=n, sh_degree=sh)
    P = [np.ascontiguousarray(g.reshape(n, -1)).copy() for g in scene.groups()]
    Z = [np.zeros_like(x) for x in P]
    ex = TrainStepExecutor(padded_rows(n, world), sh, device=rank)
    ex.upload_params(P, Z, Z, n)
    stream = torch.cuda.ExternalStream(ex.stream_handle())
    tr = (PeerExchangeTrainer(ex, n, stream=stream) if exchange in ("peer", "overlap")
          else ViewParallelTrainer(ex, n, Collectives(), stream=stream))
    rng = np.random.default_rng(100 + rank)
    gts = [torch.from_numpy(rng.uniform(0, 1, cam.width * cam.height * 3).astype(np.float32)).cuda()
           for _ in range(2)]
    for s in range(steps):
        vm = cam.viewmat.copy()
        vm[3] += 0.05 * (rank - 0.5) + 0.01 * s  # each rank its own view
        kw = dict(opacity_reg_w=0.01 / n, scale_reg_w=0.01 / (3 * n), inject_noise=True,
                  noise_seed=7, noise_offset=s, noise_scale=0.01)
        if exchange == "overlap":  # the last view's backward overlapped with the exchange
            from splatx_cuda.scene import Camera
            tr.step_overlapped(Camera(vm, cam.K, cam.width, cam.height), gts[s % 2].data_ptr(),
                               sh, world, LR, chunks=3, **kw)
            continue
        ex.step_accumulate(vm, cam.K, cam.width, cam.height, gts[s % 2].data_ptr(), n, sh)
        tr.exchange_and_apply(world, LR, **kw)
    ex.last_result()
    torch.cuda.synchronize()
    out = [np.zeros_like(x) for x in P]
    ex.download_params(out, [np.zeros_like(x) for x in P], [np.zeros_like(x) for x in P], n)
    np.savez(os.path.join(out_dir, f"{exchange}_{rank}.npz"), *out)
    del tr
    ex.close()
    dist.destroy_process_group()


def _run(exchange, tmp_path, steps=4):
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(2, _free_port(), exchange, steps, str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    return [np.load(tmp_path / f"{exchange}_{r}.npz") for r in range(2)]


@pytest.mark.parametrize("mode", ["peer", "overlap"])
def test_peer_exchange_matches_nccl_exchange(tmp_path, mode):
    """mode "overlap": the last view's backward in row chunks, each chunk's exchange behind a
    device barrier over peer memory (no collective per step)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from helpers import assert_trajectory_close
    peer = _run(mode, tmp_path)
    nccl = _run("nccl", tmp_path)
    for g in range(6):
        a0, a1 = peer[0][f"arr_{g}"], peer[1][f"arr_{g}"]
        assert np.array_equal(a0.view(np.uint32), a1.view(np.uint32)), ("replicas differ", g)
        assert_trajectory_close(a0, nccl[0][f"arr_{g}"], (mode + " vs nccl", g))
