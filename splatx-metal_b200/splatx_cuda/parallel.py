"""View-parallel (data-parallel) training of the resident step across the GPUs of one node.

The reference trains on one GPU; this is the multi-GPU plan of the port. Every rank holds a
replica of the parameters in its executor and renders its own views:

  1. ``step_accumulate`` per local view: forward + backward, the six groups' data-term gradients
     and a visibility count ADDED into the executor's gradient buffers (no Adam);
  2. one in-place sum reduce-scatter per buffer (NCCL over NVLink): rank r's owner shard — rows
     [r*S, (r+1)*S), S = padded_rows / world — receives the sum over all ranks' views;
  3. ``apply_grads`` on the owner shard: gradient = sum / n_views (+ regularisers), Adam on rows
     visible in at least one view, MCMC noise (Philox counter = global row index, so results do
     not depend on the GPU count), accumulators re-zeroed; ``clear_grads`` zeroes the rest;
  4. one in-place all-gather per parameter group returns the updated shards to every replica.

The executor keeps Gaussians in tiles of 32 (a group's d components as d runs of 32 floats), so
rows [r0, r1) with r0, r1 multiples of 32 are the contiguous floats [r0*d, r1*d) of a group's
buffer; ``padded_rows`` makes every shard a whole number of tiles. Any object with the
executor's ``step_accumulate / apply_grads / clear_grads / resident_buffers`` methods and a
``tensor(ptr_or_array, n)`` view works (the CPU tests drive a host stand-in over gloo).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def peer_barrier_selftest(device: int, world: int) -> int:
    """Run the device barrier as rank 0 of `world` ranks that never signal (flag arrays on
    `device` that nothing writes): the bounded wait runs out after about a second for world > 1.
    Returns the status bits the kernel set (2 = peer barrier timeout)."""
    import ctypes as C
    from . import _native as _nat
    st = C.c_uint32(0)
    _nat.check(_nat.lib().sxcuda_peer_barrier_selftest(int(device), int(world), C.byref(st)))
    return int(st.value)


def peer_exchange_selftest(device: int, world: int) -> tuple:
    """The device barrier as in peer_barrier_selftest, then the exchange that follows it in an
    overlapped step, on a small arena of `device`. Returns (status bits, parameters changed):
    after a timed-out barrier the exchange must change nothing."""
    import ctypes as C
    from . import _native as _nat
    st, ap = C.c_uint32(0), C.c_int32(0)
    _nat.check(_nat.lib().sxcuda_peer_exchange_selftest(int(device), int(world), C.byref(st),
                                                        C.byref(ap)))
    return int(st.value), bool(ap.value)


def padded_rows(rows: int, world: int) -> int:
    """Rows rounded up so every rank's shard is a whole number of 32-Gaussian tiles."""
    q = 32 * world
    return -(-int(rows) // q) * q


class ShardPlan:
    def __init__(self, padded: int, world: int):
        if padded % (32 * world):
            raise ValueError("padded rows must be a multiple of 32 * world")
        self.padded, self.world = padded, world
        self.rows_per_rank = padded // world

    def rows(self, rank: int):
        return rank * self.rows_per_rank, (rank + 1) * self.rows_per_rank


class Collectives:
    """In-place sum reduce-scatter and all-gather over 1-D float tensors of `world` equal chunks.

    NCCL runs the real collectives (reduce_scatter_tensor / all_gather_into_tensor with the
    output aliasing the rank's chunk). gloo has no reduce-scatter: an all-reduce leaves the same
    sum in the rank's chunk (the other chunks are cleared by the caller afterwards)."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nccl = dist.get_backend(group) == "nccl"

    def _chunk(self, t):
        n = t.numel() // self.world
        return t.narrow(0, self.rank * n, n)

    def reduce_scatter_(self, t: torch.Tensor):
        if self.world == 1:
            return
        if self.nccl:
            dist.reduce_scatter_tensor(self._chunk(t), t, op=dist.ReduceOp.SUM, group=self.group)
        else:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def all_gather_(self, t: torch.Tensor):
        if self.world == 1:
            return
        if self.nccl:
            dist.all_gather_into_tensor(t, self._chunk(t), group=self.group)
        else:
            own = self._chunk(t).clone()
            dist.all_gather(list(t.chunk(self.world)), own, group=self.group)


class _DeviceFloats:
    """A CUDA float32 array at a raw device pointer, importable by torch without a copy."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (int(n),), "typestr": "<f4",
                                         "data": (int(ptr), False), "version": 3}


def device_tensor(ptr: int, n: int, device: int) -> torch.Tensor:
    with torch.cuda.device(device):
        return torch.as_tensor(_DeviceFloats(ptr, n), device=f"cuda:{device}")


class ViewParallelTrainer:
    """One view-parallel step per call over an executor (see the module docstring)."""

    def __init__(self, ex, count: int, coll: Collectives, tensor_of=None, stream=None):
        self.ex, self.count, self.coll = ex, int(count), coll
        bufs = ex.resident_buffers()
        self.dims = bufs["dims"]
        self.plan = ShardPlan(bufs["padded_rows"], coll.world)
        view = tensor_of or (lambda ptr, n: device_tensor(ptr, n, torch.cuda.current_device()))
        P = self.plan.padded
        self.grads = [view(bufs["grads"][g], P * d) for g, d in enumerate(self.dims) if d]
        self.vis = view(bufs["visibility"], P)
        self.params = [view(bufs["params"][g], P * d) for g, d in enumerate(self.dims) if d]
        self.stream = stream  # torch stream the collectives are ordered on (executor's stream)

    def exchange_and_apply(self, n_views: int, lr, opacity_reg_w=0.0, scale_reg_w=0.0,
                           inject_noise=False, noise_seed=0, noise_offset=0, noise_scale=0.0):
        """Reduce-scatter the accumulated gradients, Adam on this rank's shard, all-gather."""
        ctx = torch.cuda.stream(self.stream) if self.stream is not None else _null()
        with ctx:
            for t in self.grads:
                self.coll.reduce_scatter_(t)
            self.coll.reduce_scatter_(self.vis)
        r0, r1 = self.plan.rows(self.coll.rank)
        self.ex.apply_grads(r0, r1, self.count, n_views, lr, opacity_reg_w, scale_reg_w,
                            inject_noise, noise_seed, noise_offset, noise_scale)
        self.ex.clear_grads()
        with ctx:
            for t in self.params:
                self.coll.all_gather_(t)


class PeerExchangeTrainer:
    """The same step as ViewParallelTrainer with the exchange fused into one kernel per rank
    over peer memory: every rank maps the others' gradient, visibility and parameter buffers
    (CUDA IPC over NVLink); after a barrier each rank reduces its owner rows from all ranks,
    applies Adam and stores the changed rows into every replica; after a second barrier it zeroes
    its accumulators. The barriers are one-element all-reduces ordered on the executor's stream.
    Rows no view saw cross no link, and reduce-scatter, Adam and all-gather overlap inside the
    one pass instead of running back to back."""

    def __init__(self, ex, count: int, group=None, stream=None):
        self.ex, self.count, self.group, self.stream = ex, int(count), group, stream
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        bufs = ex.resident_buffers()
        self.plan = ShardPlan(bufs["padded_rows"], self.world)
        # Device barriers spin on flags other ranks set: each rank needs a GPU of its own, or
        # two spinning kernels could wait on each other on one device.
        dev = torch.cuda.current_device()
        mine = (ex.peer_handles(), str(torch.cuda.get_device_properties(dev).uuid))
        gathered = [None] * self.world
        dist.all_gather_object(gathered, mine, group=group)
        if len({u for _, u in gathered}) != self.world:
            raise RuntimeError("PeerExchangeTrainer: every rank needs its own GPU")
        ex.open_peers(self.rank, self.world, [h for h, _ in gathered])
        self._flag = torch.zeros(1, dtype=torch.int32, device=dev)

    def barrier(self):
        ctx = torch.cuda.stream(self.stream) if self.stream is not None else _null()
        with ctx:
            dist.all_reduce(self._flag, group=self.group)

    def exchange_and_apply(self, n_views: int, lr, opacity_reg_w=0.0, scale_reg_w=0.0,
                           inject_noise=False, noise_seed=0, noise_offset=0, noise_scale=0.0):
        self.barrier()
        r0, r1 = self.plan.rows(self.rank)
        self.ex.exchange_apply(r0, r1, self.count, n_views, lr, opacity_reg_w, scale_reg_w,
                               inject_noise, noise_seed, noise_offset, noise_scale)
        self.barrier()
        self.ex.clear_grads()

    def step_overlapped(self, cam, gt, degrees_to_use: int, n_views: int, lr,
                        chunks: int = 4, opacity_reg_w=0.0, scale_reg_w=0.0, inject_noise=False,
                        noise_seed=0, noise_offset=0, noise_scale=0.0):
        """The last local view of a step together with the exchange (``step_exchange``): the
        view's per-Gaussian backward runs in row chunks and each chunk's exchange overlaps the
        next chunk's backward; the barriers are device-side over the mapped flag arrays, so no
        collective is launched. Replaces ``step_accumulate(last view)`` + ``exchange_and_apply``.
        ``gt``: the view's target as a device pointer or a host array."""
        r0, r1 = self.plan.rows(self.rank)
        self.ex.step_exchange(cam.viewmat, cam.K, cam.width, cam.height, gt,
                              self.count, degrees_to_use, r0, r1, n_views, lr, chunks,
                              opacity_reg_w, scale_reg_w, inject_noise, noise_seed, noise_offset,
                              noise_scale)


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False
