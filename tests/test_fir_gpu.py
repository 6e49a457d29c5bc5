"""Causal FIR kernel parity (fp32 within 1e-6 relative, as the north star
asks; bf16/fp16 within 1e-2 relative L2 of the fp32 oracle)."""
import pytest
import torch

import paper_01_anti_decoy_pnfirtau_b200 as P
from conftest import rel_l2, rel_max
from oracle import pnfirtau_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["b2n20c12k7", "b1n5c3k7", "b3n33c40k5", "b2n17c8k9"])
def test_fir_golden(cuda, golden, case):
    c = golden("fir")[case]
    x = c["x"].to(cuda).requires_grad_(True)
    taps = c["taps"].to(cuda).requires_grad_(True)
    y = P.triton_causal_fir(x, taps)
    y.backward(c["gy"].to(cuda))
    assert rel_max(y, c["y"]) < 1e-6
    assert rel_max(x.grad, c["gx"]) < 1e-6
    assert rel_max(taps.grad, c["dtaps"]) < 1e-5


def _lm_k(cuda, dtype, B=32, N=512, D=256, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    qkv = torch.randn(B, N, 3 * D, generator=g).to(device=cuda, dtype=dtype)
    return qkv.chunk(3, dim=-1)[1]  # strided [B,N,D] view, as in PnFirTauFlashMHA


def test_fir_lm_shape_fp32(cuda):
    x = _lm_k(cuda, torch.float32)
    assert not x.is_contiguous()
    taps = P.causal_gaussian_taps(7, cuda)
    y = P.triton_causal_fir(x, taps)
    ref = O.causal_fir(x.double(), taps.double())
    assert rel_max(y, ref) < 1e-6
    gy = torch.randn_like(y)
    xr = x.detach().clone().requires_grad_(True)
    tr = taps.clone().requires_grad_(True)
    P.triton_causal_fir(xr, tr).backward(gy)
    assert rel_max(xr.grad, O.causal_fir_transpose(gy.double(), taps.double())) < 1e-6
    assert rel_max(tr.grad, O.causal_fir_dtaps(gy.double(), x.double(), 7)) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fir_lm_shape_low_precision(cuda, dtype):
    x = _lm_k(cuda, dtype)
    taps = P.causal_gaussian_taps(7, cuda)
    y = P.triton_causal_fir(x, taps)
    assert y.dtype == dtype
    ref = O.causal_fir(x.float(), taps)
    assert rel_l2(y, ref) < 1e-2
    assert rel_max(y, ref) < 1e-2
    gy = torch.randn_like(y)
    xr = x.detach().clone().requires_grad_(True)
    P.triton_causal_fir(xr, taps).backward(gy)
    assert rel_l2(xr.grad, O.causal_fir_transpose(gy.float(), taps)) < 1e-2


@pytest.mark.parametrize("B,N,C", [(2, 3, 8), (1, 1, 16), (3, 70, 13), (2, 65, 24)])
def test_fir_edge_shapes(cuda, B, N, C):
    x = torch.randn(B, N, C, device=cuda)
    taps = P.causal_gaussian_taps(7, cuda)
    assert rel_max(P.triton_causal_fir(x, taps), O.causal_fir(x.double(), taps.double())) < 1e-6


def test_fir_non_unit_channel_stride(cuda):
    base = torch.randn(2, 16, 40, device=cuda)
    x = base.transpose(1, 2)  # [2, 40, 16] with stride(-1) == 40
    taps = P.causal_gaussian_taps(7, cuda)
    assert rel_max(P.triton_causal_fir(x, taps), O.causal_fir(x.double(), taps.double())) < 1e-6


@pytest.mark.parametrize("k", [3, 5, 9, 11])
def test_fir_other_tap_counts(cuda, k):
    x = torch.randn(2, 37, 24, device=cuda, requires_grad=True)
    taps = P.causal_gaussian_taps(k, cuda)
    y = P.triton_causal_fir(x, taps)
    assert rel_max(y, O.causal_fir(x.detach().double(), taps.double())) < 1e-6
    gy = torch.randn_like(y)
    y.backward(gy)
    assert rel_max(x.grad, O.causal_fir_transpose(gy.double(), taps.double())) < 1e-6


def test_fir_single_tap_is_identity(cuda):
    x = torch.randn(2, 9, 8, device=cuda)
    assert P.triton_causal_fir(x, torch.ones(1, device=cuda)) is x


def test_fir_empty(cuda):
    x = torch.randn(0, 9, 8, device=cuda)
    assert P.triton_causal_fir(x, P.causal_gaussian_taps(7, cuda)).shape == (0, 9, 8)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fir_long_runs(cuda, dtype):
    """Shapes large enough for the 32-row runs per thread (at least two blocks per
    SM of a B200), with N not a multiple of 32: the last run of every sequence
    takes the per-row bounded path, the others the eight-rows-in-flight path;
    forward, transpose (dx) and tap gradient."""
    B, N, C = 4, 4100, 2048
    g = torch.Generator(device="cpu").manual_seed(7)
    x = torch.randn(B, N, C, generator=g).to(device=cuda, dtype=dtype)
    taps = P.causal_gaussian_taps(7, cuda)
    gy = torch.randn(B, N, C, generator=g).to(device=cuda, dtype=dtype)
    xr = x.detach().clone().requires_grad_(True)
    tr = taps.clone().requires_grad_(True)
    y = P.triton_causal_fir(xr, tr)
    y.backward(gy)
    ref_y = O.causal_fir(x.double(), taps.double())
    ref_gx = O.causal_fir_transpose(gy.double(), taps.double())
    ref_dt = O.causal_fir_dtaps(gy.double(), x.double(), 7)
    if dtype == torch.float32:
        assert rel_max(y, ref_y) < 1e-6
        assert rel_max(xr.grad, ref_gx) < 1e-6
        assert rel_max(tr.grad, ref_dt) < 1e-5
    else:
        assert rel_l2(y, ref_y) < 1e-2 and rel_max(y, ref_y) < 1e-2
        assert rel_l2(xr.grad, ref_gx) < 1e-2
        assert rel_l2(tr.grad, ref_dt) < 1e-2
