"""The allocation-free prefix scan (sxcuda_prefix_scan_i64_noalloc) through the C-ABI.

It exists for callers that cannot allocate device memory when they call the library — for example
a host that hands out its whole device budget at start-up, or a latency-critical loop that must
not hit cudaMalloc's device-wide synchronisation — so they cannot pass the workspace that
sxcuda_prefix_scan_i64 needs. Its scratch is a fixed array inside the library; this file checks
that two calls in a row (the second on different, shorter data, so stale scratch contents from the
first would show) give exactly what the workspace-taking entry point gives, and that inputs beyond
the fixed capacity are refused. Named so pytest collects it last; it also passes on its own.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _regular_scan(L, tin, n, stream):
    import torch
    out = torch.empty(max(n, 1), dtype=torch.int64, device="cuda")
    nbytes = C.c_size_t(0)
    rc = L.sxcuda_prefix_scan_i64(C.c_void_p(tin.data_ptr()), C.c_void_p(out.data_ptr()), n, None,
                                  C.byref(nbytes), stream)
    assert rc == 0
    ws = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device="cuda")
    rc = L.sxcuda_prefix_scan_i64(C.c_void_p(tin.data_ptr()), C.c_void_p(out.data_ptr()), n,
                                  C.c_void_p(ws.data_ptr()), C.byref(nbytes), stream)
    assert rc == 0
    return out[:n]


def test_noalloc_scan_matches_workspace_scan_on_two_calls():
    import torch
    from splatx_cuda import _native
    L = _native.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for n, seed in ((3_000_017, 1), (123_457, 2)):
        v = np.random.default_rng(seed).integers(0, 1 << 16, size=n, dtype=np.int32)
        tin = torch.from_numpy(v).cuda()
        out = torch.full((n,), -1, dtype=torch.int64, device="cuda")
        rc = L.sxcuda_prefix_scan_i64_noalloc(C.c_void_p(tin.data_ptr()),
                                              C.c_void_p(out.data_ptr()), n, stream)
        assert rc == 0, L.sxcuda_last_error()
        expected = _regular_scan(L, tin, n, stream)
        assert torch.equal(out, expected)
        assert np.array_equal(out.cpu().numpy(), np.cumsum(v, dtype=np.int64))


def _noalloc(L, tin, out, n, stream):
    rc = L.sxcuda_prefix_scan_i64_noalloc(C.c_void_p(tin.data_ptr()), C.c_void_p(out.data_ptr()), n,
                                          stream)
    assert rc == 0, L.sxcuda_last_error()


def test_noalloc_scan_sizes_across_the_block_total_chunks():
    """Sizes that are no multiple of the 4096-element tile, more than 1024 block totals (the
    block-sum pass then walks them in chunks), n == 0 (nothing is written), and the largest n the
    fixed scratch holds; each against the workspace-taking entry point."""
    import torch
    from splatx_cuda import _native
    L = _native.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for n in (1, 4095, 4097, 12_345, 5_000_011):
        tin = torch.randint(0, 1 << 16, (n,), dtype=torch.int32, device="cuda")
        out = torch.full((n,), -1, dtype=torch.int64, device="cuda")
        _noalloc(L, tin, out, n, stream)
        assert torch.equal(out, _regular_scan(L, tin, n, stream)), n
        assert torch.equal(out, torch.cumsum(tin.to(torch.int64), 0)), n
    sentinel = torch.full((4,), -7, dtype=torch.int64, device="cuda")
    tin = torch.ones(4, dtype=torch.int32, device="cuda")
    _noalloc(L, tin, sentinel, 0, stream)
    torch.cuda.synchronize()
    assert bool((sentinel == -7).all())
    n = 65536 * 4096  # the capacity itself
    tin = torch.randint(0, 8, (n,), dtype=torch.int32, device="cuda")
    out = torch.empty(n, dtype=torch.int64, device="cuda")
    _noalloc(L, tin, out, n, stream)
    ref = _regular_scan(L, tin, n, stream)
    assert torch.equal(out, ref)
    assert int(out[-1]) == int(tin.to(torch.int64).sum())
    del tin, out, ref
    torch.cuda.empty_cache()


def test_noalloc_scan_takes_no_device_memory():
    """After a first call (which, under lazy module loading, may load the library's device code),
    further calls leave the device's free memory exactly as it was: no allocation, by the library
    or any routine it calls."""
    import torch
    from splatx_cuda import _native
    L = _native.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    n = 3_000_017
    tin = torch.randint(0, 1 << 16, (n,), dtype=torch.int32, device="cuda")
    out = torch.empty(n, dtype=torch.int64, device="cuda")
    _noalloc(L, tin, out, n, stream)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _noalloc(L, tin, out, n, stream)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert torch.equal(out, torch.cumsum(tin.to(torch.int64), 0))


def test_noalloc_scan_refuses_inputs_beyond_its_fixed_scratch():
    from splatx_cuda import _native
    L = _native.lib()
    too_big = 65536 * 4096 + 1
    rc = L.sxcuda_prefix_scan_i64_noalloc(C.c_void_p(16), C.c_void_p(16), too_big, None)
    assert rc == _native.SXCUDA_EINVAL
    assert b"capacity" in L.sxcuda_last_error()
