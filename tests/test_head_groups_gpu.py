"""The tcgen05 kernels' head-grouped CTA order (heads taken in groups whose
per-head data fits in L2; automatic on long sequences such as config 5, where
each head re-reads 8-16 MB). PNFT_HEAD_GROUP forces small groups here so that
the grouped order, including its last partial group and the deterministic
backward's ticket order inside groups, is checked at small sizes against the
fp32 oracle and against the plain order."""
import pytest
import torch

import paper_01_anti_decoy_pnfirtau_b200 as P
from conftest import rel_l2
from oracle import pnfirtau_oracle as O
from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import check_device_status

pytestmark = pytest.mark.gpu


def _inputs(B, H, N, D, seed, device):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(B, H, N, D, generator=g).to(device, torch.bfloat16) for _ in range(4))


def _run(q, k, v, do, tau, deterministic=False):
    qq, kk, vv = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    tt = torch.tensor(tau, device=q.device, requires_grad=True)
    out = P.flash_pn_fir_tau_attention(qq, kk, vv, tt, deterministic=deterministic)
    out.backward(do)
    check_device_status(q.device)
    return out.detach(), qq.grad, kk.grad, vv.grad, tt.grad


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("group", [1, 2, 4])
def test_grouped_order_matches_plain_and_oracle(cuda, monkeypatch, D, group):
    q, k, v, do = _inputs(2, 3, 640, D, 70 + D + group, cuda)  # 6 heads: groups of 4 leave a partial group
    monkeypatch.setenv("PNFT_HEAD_GROUP", "6")
    plain = _run(q, k, v, do, 0.1)
    monkeypatch.setenv("PNFT_HEAD_GROUP", str(group))
    grouped = _run(q, k, v, do, 0.1)
    # same work per CTA, only the order differs: the forward and dK/dV/dtau are equal
    # bit for bit, dQ up to the order of its fp32 accumulation across CTAs
    for name, a, b in zip(("out", "dq", "dk", "dv", "dtau"), grouped, plain):
        if name == "dq":
            assert rel_l2(a, b) < 1e-3, name
        else:
            assert torch.equal(a, b), name
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    tr = torch.tensor(0.1, device=cuda, requires_grad=True)
    outr = O.pn_fir_tau_attention(qr, kr, vr, tr)
    outr.backward(do.float())
    for name, a, r in zip(("out", "dq", "dk", "dv"), grouped, (outr, qr.grad, kr.grad, vr.grad)):
        assert rel_l2(a, r) < 1e-2, (name, rel_l2(a, r))
    assert abs(float(grouped[4]) - float(tr.grad)) <= 1e-2 * abs(float(tr.grad)) + 1e-6


@pytest.mark.parametrize("group", [2, 4])
def test_deterministic_backward_in_groups(cuda, monkeypatch, group):
    """Deterministic mode waits only on lower key tiles of the same head, which the
    grouped ticket order still starts earlier: no stall, bitwise-equal reruns."""
    q, k, v, do = _inputs(2, 3, 896, 64, 81 + group, cuda)
    monkeypatch.setenv("PNFT_HEAD_GROUP", str(group))
    a = _run(q, k, v, do, -0.1, deterministic=True)
    b = _run(q, k, v, do, -0.1, deterministic=True)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    monkeypatch.setenv("PNFT_HEAD_GROUP", "6")
    c = _run(q, k, v, do, -0.1, deterministic=True)
    # the same key order per query tile in either CTA order: bitwise equal
    for x, y in zip(a, c):
        assert torch.equal(x, y)
