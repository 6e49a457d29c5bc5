"""The bounded pipeline waits of the tcgen05 kernels, run out on purpose.

With the test-only flag PNFT_FLASH_TEST_STALL the elementwise warps make their
first pipeline wait on an mbarrier that nothing arrives on, so it runs out after
the kernels' 1 s limit. That is the failure path of every pipeline wait: the warp sets the CTA's abort word and the status
word, the producer and MMA roles stop at their next wait, the producer lets its
own TMA copies land, the MMA issuer waits for its MMAs, TMEM is freed and the
kernel returns. Nothing faults, traps or spins without a limit; the test checks
that the call returns, that the failure reaches the host (through
check_device_status, and through the next call of the operator, which reads the
mapped status word without synchronising), and that the next normal call on
the same device matches the oracle.
"""
import pytest
import torch

import paper_01_anti_decoy_pnfirtau_b200 as P
from conftest import rel_l2
from oracle import pnfirtau_oracle as O
from paper_01_anti_decoy_pnfirtau_b200 import _lib, pnfirtau_ops
from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import check_device_status, flash_pn_fir_tau_forward_stats

pytestmark = pytest.mark.gpu


def _small(cuda, D=64, N=256, seed=31):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(1, 2, N, D, generator=g).to(cuda, torch.bfloat16) for _ in range(4))


def _fwd_bwd(q, k, v, do, tau, fused_fir=False, fused_forward=False):
    qq, kk, vv = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    tt = torch.tensor(tau, device=q.device, requires_grad=True)
    if fused_fir:
        taps = O.gaussian_taps(7).to(q.device)
        out = P.flash_pn_fir_tau_attention_fir(qq, kk, vv, tt, taps, fused_forward=fused_forward)
    else:
        out = P.flash_pn_fir_tau_attention(qq, kk, vv, tt)
    out.backward(do)
    return out.detach(), qq.grad, kk.grad, vv.grad, tt.grad


def _oracle(q, k, v, do, tau, fused_fir=False):
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    tr = torch.tensor(tau, device=q.device, requires_grad=True)
    kt = kr
    if fused_fir:
        # filtered in fp32, rounded to bf16 as the fused kernels (and the reference's
        # bf16 path) do; identity gradient through the rounding
        B, H, N, D = kr.shape
        kt = O.causal_fir(kr.transpose(1, 2).reshape(B, N, H * D), O.gaussian_taps(7).to(q.device))
        kt = kt + (kt.to(torch.bfloat16).float() - kt).detach()
        kt = kt.view(B, N, H, D).transpose(1, 2)
    out = O.pn_fir_tau_attention(qr, kt, vr, tr)
    out.backward(do.float())
    return out.detach(), qr.grad, kr.grad, vr.grad, tr.grad


def _assert_parity(ours, ref):
    for name, a, r in zip(("out", "dq", "dk", "dv"), ours[:4], ref[:4]):
        assert rel_l2(a, r) < 1e-2, (name, rel_l2(a, r))
    assert abs(float(ours[4]) - float(ref[4])) <= 1e-2 * abs(float(ref[4])) + 1e-6


def test_status_word_is_mapped_host_memory(cuda):
    """On a B200 the status word is pinned host memory mapped into the device, so
    a failure is visible to the host without a copy."""
    w = pnfirtau_ops._status_entry(cuda)
    assert w.host is not None and w.host.is_pinned()
    check_device_status(cuda)


@pytest.mark.parametrize("D", [64, 128])
def test_forward_wait_timeout(cuda, D):
    q, k, v, do = _small(cuda, D)
    t = torch.tensor(0.1, device=cuda)
    check_device_status(cuda)  # clean start
    flash_pn_fir_tau_forward_stats(q, k, v, t, extra_flags=_lib.FLASH_TEST_STALL)
    torch.cuda.synchronize()  # the kernel returned
    with pytest.raises(RuntimeError, match="timed out"):
        check_device_status(cuda)
    check_device_status(cuda)  # the word was cleared
    out, *_ = flash_pn_fir_tau_forward_stats(q, k, v, t)
    check_device_status(cuda)
    assert rel_l2(out, O.pn_fir_tau_attention(q.float(), k.float(), v.float(), t)) < 1e-2


def test_pending_timeout_raised_by_next_call(cuda):
    """The operator's next call reports an earlier kernel's timeout by itself."""
    q, k, v, do = _small(cuda)
    t = torch.tensor(0.0, device=cuda)
    flash_pn_fir_tau_forward_stats(q, k, v, t, extra_flags=_lib.FLASH_TEST_STALL)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="earlier call"):
        P.flash_pn_fir_tau_attention(q, k, v, t)
    check_device_status(cuda)  # reported once, then cleared
    ours = _fwd_bwd(q, k, v, do, 0.0)
    check_device_status(cuda)
    _assert_parity(ours, _oracle(q, k, v, do, 0.0))


@pytest.mark.parametrize("fused_fir", [False, True], ids=["plain", "fused_fir"])
@pytest.mark.parametrize("D", [64, 128])
def test_backward_wait_timeout(cuda, D, fused_fir):
    q, k, v, do = _small(cuda, D, N=320, seed=32 + D)
    qq, kk, vv = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    tt = torch.tensor(0.2, device=cuda, requires_grad=True)
    if fused_fir:
        out = P.flash_pn_fir_tau_attention_fir(qq, kk, vv, tt, O.gaussian_taps(7).to(cuda))
    else:
        out = P.flash_pn_fir_tau_attention(qq, kk, vv, tt)
    check_device_status(cuda)  # the forward ran normally
    pnfirtau_ops._TEST_FLAGS = _lib.FLASH_TEST_STALL
    try:
        out.backward(do)  # only the backward kernel stalls
    finally:
        pnfirtau_ops._TEST_FLAGS = 0
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="timed out"):
        check_device_status(cuda)
    ours = _fwd_bwd(q, k, v, do, 0.2, fused_fir=fused_fir)
    check_device_status(cuda)
    _assert_parity(ours, _oracle(q, k, v, do, 0.2, fused_fir=fused_fir))


def test_fused_forward_wait_timeout(cuda):
    """The kernel-fused FIR forward (two filter warps beside the elementwise
    group) unwinds the same way."""
    q, k, v, do = _small(cuda, 64, N=384, seed=40)
    tt = torch.tensor(0.0, device=cuda)
    pnfirtau_ops._TEST_FLAGS = _lib.FLASH_TEST_STALL
    try:
        with torch.no_grad():
            P.flash_pn_fir_tau_attention_fir(q, k, v, tt, O.gaussian_taps(7).to(cuda), fused_forward=True)
    finally:
        pnfirtau_ops._TEST_FLAGS = 0
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="timed out"):
        check_device_status(cuda)
    ours = _fwd_bwd(q, k, v, do, 0.0, fused_fir=True, fused_forward=True)
    check_device_status(cuda)
    _assert_parity(ours, _oracle(q, k, v, do, 0.0, fused_fir=True))
