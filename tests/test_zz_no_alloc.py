"""The allocation-free FIR backward (pnft_fir_bwd_noalloc) against the
workspace entry point (pnft_fir_bwd), both called through the C ABI.

pnft_fir_bwd_noalloc exists for callers that cannot allocate device memory for
the library: code running inside CUDA stream capture, serving loops that must
not touch an allocator after start-up, and foreign-language bindings that only
hold the buffers their host runtime gave them. It keeps the tap-gradient
partial sums in a static device array instead of a caller workspace. Two calls
in a row (the second smaller, so the first call's leftovers stay in the shared
array) must both reproduce the workspace entry point's results.

This file is named to be collected last; it must pass alone in a fresh process
and after the rest of the suite.
"""
import pytest
import torch

from paper_01_anti_decoy_pnfirtau_b200 import _lib

pytestmark = pytest.mark.gpu

DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def _case(B, N, C, dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    gy = torch.randn(B, N, C, generator=g).to(device, dtype)
    x = torch.randn(B, N, C, generator=g).to(device, dtype)
    taps = torch.rand(7, generator=g).to(device)
    return gy, x, taps / taps.sum()


def _with_workspace(gy, x, taps):
    L = _lib.lib()
    B, N, C = gy.shape
    gx = torch.empty_like(gy)
    dtaps = torch.empty(taps.numel(), device=gy.device)
    ws = torch.empty(max(L.pnft_fir_bwd_workspace_size(B, N, C, taps.numel()), 1), device=gy.device,
                     dtype=torch.uint8)
    rc = L.pnft_fir_bwd(gy.data_ptr(), *gy.stride(), taps.data_ptr(), taps.numel(), gx.data_ptr(), *gx.stride(),
                        x.data_ptr(), *x.stride(), dtaps.data_ptr(), ws.data_ptr(), ws.numel(), B, N, C,
                        DTYPES[gy.dtype], torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "pnft_fir_bwd")
    return gx, dtaps


def _without_workspace(gy, x, taps):
    L = _lib.lib()
    B, N, C = gy.shape
    gx = torch.empty_like(gy)
    dtaps = torch.empty(taps.numel(), device=gy.device)
    rc = L.pnft_fir_bwd_noalloc(gy.data_ptr(), *gy.stride(), taps.data_ptr(), taps.numel(), gx.data_ptr(),
                                *gx.stride(), x.data_ptr(), *x.stride(), dtaps.data_ptr(), B, N, C,
                                DTYPES[gy.dtype], torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "pnft_fir_bwd_noalloc")
    return gx, dtaps


def _rel(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max().clamp_min(1e-30))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_workspace_entry_point_twice(cuda, dtype):
    # first call: large enough to use all 512 partial-sum blocks; second: fewer blocks
    for B, N, C, seed in ((32, 512, 256, 1), (2, 37, 24, 2)):
        gy, x, taps = _case(B, N, C, dtype, seed, cuda)
        gx_ref, dt_ref = _with_workspace(gy, x, taps)
        gx, dt = _without_workspace(gy, x, taps)
        torch.cuda.synchronize()
        assert _rel(gx, gx_ref) <= 1e-6
        assert _rel(dt, dt_ref) <= 1e-6


@pytest.mark.parametrize("ntaps", [7, 5])
def test_noalloc_tap_gradient_only(cuda, ntaps):
    """gx = NULL: the tap gradient alone, with the 7-tap one-pass kernel and with
    the per-lag kernel that other tap counts use; two calls in a row."""
    L = _lib.lib()
    for B, N, C, seed in ((4, 300, 64, 4), (1, 19, 16, 5)):
        gy, x, taps = _case(B, N, C, torch.bfloat16, seed, cuda)
        taps = taps[:ntaps] / taps[:ntaps].sum()
        dt_ref = torch.empty(ntaps, device=cuda)
        ws = torch.empty(max(L.pnft_fir_bwd_workspace_size(B, N, C, ntaps), 1), device=cuda, dtype=torch.uint8)
        _lib.check(L.pnft_fir_bwd(gy.data_ptr(), *gy.stride(), taps.data_ptr(), ntaps, None, 0, 0, 0, x.data_ptr(),
                                  *x.stride(), dt_ref.data_ptr(), ws.data_ptr(), ws.numel(), B, N, C, _lib.DTYPE_BF16,
                                  torch.cuda.current_stream().cuda_stream), "pnft_fir_bwd")
        dt = torch.empty(ntaps, device=cuda)
        _lib.check(L.pnft_fir_bwd_noalloc(gy.data_ptr(), *gy.stride(), taps.data_ptr(), ntaps, None, 0, 0, 0,
                                          x.data_ptr(), *x.stride(), dt.data_ptr(), B, N, C, _lib.DTYPE_BF16,
                                          torch.cuda.current_stream().cuda_stream), "pnft_fir_bwd_noalloc")
        torch.cuda.synchronize()
        assert _rel(dt, dt_ref) <= 1e-6


def test_noalloc_rejects_too_many_taps(cuda):
    L = _lib.lib()
    gy, x, _ = _case(1, 8, 8, torch.float32, 3, cuda)
    taps = torch.ones(65, device=cuda)
    dtaps = torch.empty(65, device=cuda)
    rc = L.pnft_fir_bwd_noalloc(gy.data_ptr(), *gy.stride(), taps.data_ptr(), 65, None, 0, 0, 0, x.data_ptr(),
                                *x.stride(), dtaps.data_ptr(), 1, 8, 8, _lib.DTYPE_F32,
                                torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.EINVAL and "65" in _lib.last_error()


def test_noalloc_captured_in_cuda_graph(cuda):
    """The use case the entry point exists for: captured into a CUDA graph after
    one warm-up call (which resolves the scratch array's address), then replayed
    on new inputs copied into the captured buffers; every replay equals the
    workspace entry point on the same inputs."""
    L = _lib.lib()
    B, N, C = 8, 256, 128
    gy, x, taps = _case(B, N, C, torch.bfloat16, 21, cuda)
    gx = torch.empty_like(gy)
    dtaps = torch.empty(taps.numel(), device=cuda)

    def call(stream):
        return L.pnft_fir_bwd_noalloc(gy.data_ptr(), *gy.stride(), taps.data_ptr(), taps.numel(), gx.data_ptr(),
                                      *gx.stride(), x.data_ptr(), *x.stride(), dtaps.data_ptr(), B, N, C,
                                      _lib.DTYPE_BF16, stream)

    _lib.check(call(torch.cuda.current_stream().cuda_stream), "warm-up")
    torch.cuda.synchronize()
    side = torch.cuda.Stream(cuda)
    side.wait_stream(torch.cuda.current_stream(cuda))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        _lib.check(call(side.cuda_stream), "captured call")
    torch.cuda.current_stream(cuda).wait_stream(side)
    for seed in (22, 23):
        gy1, x1, _ = _case(B, N, C, torch.bfloat16, seed, cuda)
        gy.copy_(gy1)
        x.copy_(x1)
        graph.replay()
        torch.cuda.synchronize()
        gx_ref, dt_ref = _with_workspace(gy1, x1, taps)
        torch.cuda.synchronize()
        assert _rel(gx, gx_ref) <= 1e-6 and _rel(dtaps, dt_ref) <= 1e-6
    del graph
