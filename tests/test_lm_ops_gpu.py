"""The LM-step kernels (csrc/lm_step.cu via lm_ops) against PyTorch fp32:
the head's one-pass cross-entropy (loss and logit gradient, padding columns,
ignore_index, a bad target reported through the status word, the staged and the
two global-memory variants), the fused head + cross-entropy autograd function,
LayerNorm forward/backward (vector and scalar paths, bf16 and fp32, affine or
not, bitwise-reproducible parameter gradients), and the config-4 LM with the
fused step ops against the same LM with nn.LayerNorm and F.cross_entropy.

Reference composition: experiments/exp4_wikitext2_lm.py:183-259 (Pre-LN
blocks, tied head) and :714-719 (F.cross_entropy on the logits)."""
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_l2
from paper_01_anti_decoy_pnfirtau_b200 import _lib
from paper_01_anti_decoy_pnfirtau_b200.lm import LMConfig, PnFirLM, lm_loss, make_optimizer, train_step
from paper_01_anti_decoy_pnfirtau_b200.lm_ops import (LayerNorm, Linear, add_layer_norm, head_cross_entropy, layer_norm,
                                                     mlp_gelu)
from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import _status_ptr, check_device_status

pytestmark = pytest.mark.gpu


def _ptr(t):
    return None if t is None else t.data_ptr()


def _xent_call(logits, V, t, ignore=-100, scale=1.0):
    M, ld = logits.shape
    loss = torch.empty(M, device=logits.device)
    rc = _lib.lib().pnft_lm_xent(logits.data_ptr(), ld, t.data_ptr(), ignore, loss.data_ptr(), M, V, scale, None,
                                 _status_ptr(logits.device), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "pnft_lm_xent")
    return loss


# (M, V, ld): staged rows (ld % 8 == 0; more rows per CTA than ring stages, so
# stages are refilled and their phases wrap), a scalar global row (odd ld), a
# row too long to stage twice in shared memory (vector global path)
XENT_CASES = {"staged_lm_vocab": (1000, 33278, 33280), "staged_small": (2000, 1000, 1024),
              "global_scalar": (19, 517, 519), "global_vec": (5, 70000, 70008)}


@pytest.mark.parametrize("case", sorted(XENT_CASES))
def test_xent_kernel_against_fp32(cuda, case):
    M, V, ld = XENT_CASES[case]
    g = torch.Generator(device=cuda).manual_seed(M + V)
    x = (torch.randn(M, ld, device=cuda, generator=g) * 3).to(torch.bfloat16)
    t = torch.randint(0, V, (M,), device=cuda, generator=g)
    t[::7] = -100  # ignored rows
    t[1] = V - 1   # the last valid column
    ref_x = x[:, :V].float().requires_grad_(True)
    per_row = F.cross_entropy(ref_x, t, reduction="none")
    counted = (t != -100).sum()
    per_row.sum().backward()
    buf = x.clone()
    loss = _xent_call(buf, V, t, scale=1.0)
    torch.cuda.synchronize()
    check_device_status(cuda)
    assert torch.allclose(loss, per_row.detach(), rtol=2e-6, atol=2e-5), (loss - per_row).abs().max()
    assert float((loss.sum() / counted - per_row.detach().sum() / counted).abs()) < 1e-5
    grad = buf.float()
    assert torch.all(grad[:, V:] == 0)
    assert torch.all(grad[t == -100] == 0)
    # one bf16 rounding (up to 2^-8 relative) of a value within 2^-11 of the exact
    # (softmax - onehot): the kernel keeps exp(x - max) as fp16 between its passes
    assert rel_l2(grad[:, :V], ref_x.grad) < 4e-3
    err = (grad[:, :V] - ref_x.grad).abs()
    bound = ref_x.grad.abs() * (2 ** -8 + 2 ** -10) + 1e-7
    assert torch.all(err <= bound), float((err / bound).max())


def test_xent_bad_target_sets_status(cuda):
    x = torch.randn(4, 64, device=cuda).to(torch.bfloat16)
    t = torch.tensor([1, 64, 3, -5], device=cuda)  # 64 and -5 are outside [0, 64) and not ignore_index
    loss = _xent_call(x.clone(), 64, t)
    with pytest.raises(RuntimeError, match="outside"):
        check_device_status(cuda)
    assert torch.isnan(loss[1]) and torch.isnan(loss[3]) and torch.isfinite(loss[0]) and torch.isfinite(loss[2])
    check_device_status(cuda)  # the word was cleared


@pytest.mark.parametrize("V", [33278, 1000])
def test_head_cross_entropy_matches_autocast_composition(cuda, V):
    g = torch.Generator(device=cuda).manual_seed(V)
    h = torch.randn(4, 63, 256, device=cuda, generator=g).requires_grad_(True)
    w = (torch.randn(V, 256, device=cuda, generator=g) * 0.05).requires_grad_(True)
    t = torch.randint(0, V, (4, 63), device=cuda, generator=g)
    t[0, :5] = -100
    loss = head_cross_entropy(h, w, t)
    loss.backward()
    check_device_status(cuda)
    # reference: the autocast head GEMM (bf16 operands, fp32 accumulation) and an fp32 cross-entropy
    hr = h.detach().clone().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    logits = hr.to(torch.bfloat16).float() @ wr.to(torch.bfloat16).float().t()
    ref = F.cross_entropy(logits.reshape(-1, V), t.reshape(-1))
    ref.backward()
    assert abs(float(loss) - float(ref)) < 2e-3 * abs(float(ref)), (float(loss), float(ref))
    assert rel_l2(h.grad, hr.grad) < 1e-2, rel_l2(h.grad, hr.grad)
    assert rel_l2(w.grad, wr.grad) < 1e-2, rel_l2(w.grad, wr.grad)


LN_CASES = {
    # name: (M, C, x dtype, y dtype, affine)
    "lm_c256_bf16_out": (16384, 256, torch.float32, torch.bfloat16, True),
    "c256_f32": (1000, 256, torch.float32, torch.float32, True),
    "c96_partial_vector": (333, 96, torch.float32, torch.float32, True),
    "c384": (100, 384, torch.bfloat16, torch.float32, True),
    "c512_no_affine": (64, 512, torch.float32, torch.float32, False),
    "c1000_scalar": (77, 1000, torch.float32, torch.bfloat16, True),
    "c6_scalar": (50, 6, torch.float32, torch.float32, True),
}


@pytest.mark.parametrize("case", sorted(LN_CASES))
def test_layer_norm_against_fp32(cuda, case):
    M, C, xdt, ydt, affine = LN_CASES[case]
    g = torch.Generator(device=cuda).manual_seed(M * 7 + C)
    x = (torch.randn(M, C, device=cuda, generator=g) * 2 + 0.5).to(xdt).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(C, device=cuda, generator=g)).requires_grad_(affine) if affine else None
    b = (0.1 * torch.randn(C, device=cuda, generator=g)).requires_grad_(affine) if affine else None
    gy = torch.randn(M, C, device=cuda, generator=g).to(ydt)
    y = layer_norm(x, (C,), w, b, 1e-5, out_dtype=ydt)
    assert y.dtype == ydt
    y.backward(gy)
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True) if affine else None
    br = b.detach().clone().requires_grad_(True) if affine else None
    yr = F.layer_norm(xr, (C,), wr, br, 1e-5)
    yr.backward(gy.float())
    # fp32: rounding of the statistics; bf16: at most one bf16 ulp (2^-7 relative) from the rounded reference
    rtol, atol = (1e-6, 1e-5) if ydt == torch.float32 else (2 ** -7, 1e-4)
    assert torch.allclose(y.float(), yr.detach().to(ydt).float(), rtol=rtol, atol=atol), (
        (y.float() - yr).abs().max())
    tol = 1e-5 if xdt == torch.float32 else 8e-3
    assert rel_l2(x.grad, xr.grad) < tol, rel_l2(x.grad, xr.grad)
    if affine:
        assert rel_l2(w.grad, wr.grad) < 1e-5, rel_l2(w.grad, wr.grad)
        assert rel_l2(b.grad, br.grad) < 1e-5, rel_l2(b.grad, br.grad)
        # the parameter gradients are reduced in a fixed order: bitwise equal on a rerun
        dw1, db1 = w.grad.clone(), b.grad.clone()
        w.grad = b.grad = None
        x.grad = None
        layer_norm(x, (C,), w, b, 1e-5, out_dtype=ydt).backward(gy)
        assert torch.equal(dw1, w.grad) and torch.equal(db1, b.grad)


def test_layernorm_module_is_nn_layernorm(cuda):
    ln = LayerNorm(256).to(cuda)
    ref = torch.nn.LayerNorm(256).to(cuda)
    ref.load_state_dict(ln.state_dict())
    x = torch.randn(2, 8, 256, device=cuda)
    assert torch.allclose(ln(x), ref(x), rtol=1e-6, atol=1e-6)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = ln(x)
        yr = ref(x)
    assert y.dtype == torch.bfloat16 and yr.dtype == torch.float32
    assert torch.equal(y, yr.to(torch.bfloat16)) or rel_l2(y, yr) < 2 ** -8


@pytest.mark.parametrize("C", [256, 100])
def test_add_layer_norm_against_fp32(cuda, C):
    """s = x + r (fp32 + bf16 branch, as in the LM's residual stream) and LN(s) in
    one kernel; gradients of x (with the residual path's own gradient of s
    added), r (bf16), weight, bias. C = 100 takes the scalar path."""
    g = torch.Generator(device=cuda).manual_seed(C)
    M = 3000
    x = torch.randn(M, C, device=cuda, generator=g).requires_grad_(True)
    r = torch.randn(M, C, device=cuda, generator=g).to(torch.bfloat16).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(C, device=cuda, generator=g)).requires_grad_(True)
    b = (0.1 * torch.randn(C, device=cuda, generator=g)).requires_grad_(True)
    gs = torch.randn(M, C, device=cuda, generator=g)
    gy = torch.randn(M, C, device=cuda, generator=g).to(torch.bfloat16)
    s, y = add_layer_norm(x, r, (C,), w, b, 1e-5, out_dtype=torch.bfloat16)
    assert s.dtype == torch.float32 and y.dtype == torch.bfloat16
    torch.autograd.backward((s, y), (gs, gy))
    xr, rr, wr, br = (t.detach().float().clone().requires_grad_(True) for t in (x, r, w, b))
    sr = xr + rr
    yr = F.layer_norm(sr, (C,), wr, br, 1e-5)
    torch.autograd.backward((sr, yr), (gs, gy.float()))
    assert torch.equal(s, sr.detach())
    assert torch.allclose(y.float(), yr.detach().to(torch.bfloat16).float(), rtol=2 ** -7, atol=1e-4)
    assert rel_l2(x.grad, xr.grad) < 1e-5
    assert r.grad.dtype == torch.bfloat16 and rel_l2(r.grad, rr.grad) < 4e-3
    assert rel_l2(w.grad, wr.grad) < 1e-5 and rel_l2(b.grad, br.grad) < 1e-5


@pytest.mark.parametrize("shape", [(16384, 256, 1024), (300, 64, 200)], ids=["lm_mlp", "ragged_scalar"])
def test_mlp_gelu_against_pytorch(cuda, shape):
    """fc2(GELU(fc1(x))) under bf16 autocast: output and every gradient against
    the fp32 composition (bias gradients and the GELU backward on this library's
    column-sum kernels; 200 hidden columns take the scalar path)."""
    M, D, H = shape
    torch.manual_seed(M)
    fc1, fc2 = torch.nn.Linear(D, H).to(cuda), torch.nn.Linear(H, D).to(cuda)
    x = torch.randn(M, D, device=cuda).requires_grad_(True)
    gy = torch.randn(M, D, device=cuda)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = mlp_gelu(x, fc1, fc2)
    assert y.dtype == torch.bfloat16
    y.backward(gy.to(torch.bfloat16))
    grads = [x.grad, fc1.weight.grad, fc1.bias.grad, fc2.weight.grad, fc2.bias.grad]
    ref1, ref2 = torch.nn.Linear(D, H).to(cuda), torch.nn.Linear(H, D).to(cuda)
    ref1.load_state_dict(fc1.state_dict()), ref2.load_state_dict(fc2.state_dict())
    xr = x.detach().clone().requires_grad_(True)
    yr = ref2(F.gelu(ref1(xr)))
    yr.backward(gy.to(torch.bfloat16).float())
    assert rel_l2(y, yr) < 1e-2
    for name, a, b in zip(("x", "w1", "b1", "w2", "b2"), grads,
                          [xr.grad, ref1.weight.grad, ref1.bias.grad, ref2.weight.grad, ref2.bias.grad]):
        assert a.dtype == b.dtype and rel_l2(a, b) < 1.5e-2, (name, rel_l2(a, b))
    # bias gradients are reduced in a fixed order: a rerun is bitwise equal
    b1, b2 = fc1.bias.grad.clone(), fc2.bias.grad.clone()
    for prm in (x, *fc1.parameters(), *fc2.parameters()):
        prm.grad = None
    with torch.autocast("cuda", dtype=torch.bfloat16):
        mlp_gelu(x, fc1, fc2).backward(gy.to(torch.bfloat16))
    assert torch.equal(b1, fc1.bias.grad) and torch.equal(b2, fc2.bias.grad)


def test_colsum_and_gelu_bwd_kernels_exact_sums(cuda):
    """The column sums equal an fp64 sum of the same stored values within fp32
    rounding; the GELU derivative matches PyTorch's GELU backward on bf16."""
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=cuda).manual_seed(9)
    for M, C, dt in ((5000, 1024, torch.bfloat16), (777, 24, torch.float32), (3, 8, torch.bfloat16)):
        dh = torch.randn(M, C, device=cuda, generator=g).to(dt)
        a = torch.randn(M, C, device=cuda, generator=g).to(dt) * 2
        nb = L.pnft_colsum_workspace_size(M, C)
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=cuda)
        out = torch.empty(C, device=cuda)
        _lib.check(L.pnft_colsum(dh.data_ptr(), C, out.data_ptr(), ws.data_ptr(), nb, M, C,
                                 _lib.DTYPE_BF16 if dt == torch.bfloat16 else _lib.DTYPE_F32, st), "colsum")
        ref = dh.double().sum(0)
        assert torch.allclose(out.double(), ref, rtol=1e-5, atol=1e-4 * M ** 0.5)
        da = torch.empty_like(dh)
        tab = torch.empty(_lib.GELU_TABLE_FLOATS, device=cuda)
        _lib.check(L.pnft_gelu_table(tab.data_ptr(), st), "gelu table")
        runs = []
        for table in (None, tab):  # per-CTA tables and the device table give the same values
            _lib.check(L.pnft_gelu_bwd_colsum(dh.data_ptr(), C, a.data_ptr(), C, da.data_ptr(), C, out.data_ptr(),
                                              ws.data_ptr(), nb, M, C,
                                              _lib.DTYPE_BF16 if dt == torch.bfloat16 else _lib.DTYPE_F32,
                                              _ptr(table), st), "gelu")
            runs.append((da.clone(), out.clone()))
        assert torch.equal(runs[0][0], runs[1][0]) and torch.equal(runs[0][1], runs[1][1])
        ar = a.detach().float().requires_grad_(True)
        F.gelu(ar).backward(dh.float())
        tol = 2 ** -7 if dt == torch.bfloat16 else 1e-6
        assert torch.allclose(da.float(), ar.grad.to(dt).float(), rtol=tol, atol=1e-6)
        assert torch.allclose(out.double(), da.double().sum(0), rtol=1e-5, atol=1e-4 * M ** 0.5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gelu_fwd_against_pytorch(cuda, dtype):
    """pnft_gelu_fwd against F.gelu (exact erf form): bf16 through the
    per-CTA table (every binade it covers, and values outside it: tiny, zero,
    |a| >= 16), fp32 and a ragged width through the formula."""
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=cuda).manual_seed(4)
    code = _lib.DTYPE_BF16 if dtype == torch.bfloat16 else _lib.DTYPE_F32
    tab = torch.empty(_lib.GELU_TABLE_FLOATS, device=cuda)
    _lib.check(L.pnft_gelu_table(tab.data_ptr(), st), "gelu table")
    ys = []
    for M, C in ((4096, 1024), (37, 20)):
        a = torch.randn(M, C, device=cuda, generator=g) * torch.exp2(torch.randint(-20, 6, (M, C), device=cuda,
                                                                                    generator=g).float())
        a[0, :8] = torch.tensor([0.0, -0.0, 1e-30, -3e-7, 16.0, -16.0, 40.0, -40.0])
        a = a.to(dtype)
        y = torch.empty_like(a)
        for table in (None, tab):  # per-CTA tables and the device table give the same values
            _lib.check(L.pnft_gelu_fwd(a.data_ptr(), C, y.data_ptr(), C, M, C, code, _ptr(table), st), "gelu")
            ys.append(y.clone())
        assert torch.equal(ys[0], ys[1])
        ys.clear()
        ref = F.gelu(a.float())
        if dtype == torch.bfloat16:
            # the fp32 result rounded to bf16: equal, or one ulp off where the fp32 values round apart
            assert torch.allclose(y.float(), ref.to(dtype).float(), rtol=2 ** -7, atol=1e-30)
            assert (y.float() == ref.to(dtype).float()).float().mean() > 0.995
        else:
            assert torch.allclose(y, ref, rtol=2e-6, atol=1e-30)


GEMM_CASES = {
    # name: (K, M, N, lda pad, ldb pad)
    "lm_fc2": (16384, 256, 1024, 0, 0),
    "lm_qkv": (16384, 768, 256, 0, 0),
    "lm_out": (16384, 256, 256, 0, 0),
    "ragged": (5000, 136, 72, 0, 0),
    "one_split": (300, 128, 128, 0, 0),
    "strided": (4096, 64, 192, 16, 8),
}


@pytest.mark.parametrize("case", sorted(GEMM_CASES))
def test_gemm_at_b_against_fp32(cuda, case):
    """pnft_gemm_at_b (split-K tcgen05, weight gradients) against an fp32
    product of the same bf16 operands; a rerun is bitwise equal."""
    K, M, N, pa, pb = GEMM_CASES[case]
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=cuda).manual_seed(K + M + N)
    a = torch.randn(K, M + pa, device=cuda, generator=g).to(torch.bfloat16)[:, :M]
    b = torch.randn(K, N + pb, device=cuda, generator=g).to(torch.bfloat16)[:, :N]
    nbytes = L.pnft_gemm_at_b_workspace_size(K, M, N)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=cuda)
    outs = []
    for _ in range(2):
        c = torch.full((M, N), float("nan"), device=cuda)
        _lib.check(L.pnft_gemm_at_b(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), c.data_ptr(), N,
                                    ws.data_ptr(), nbytes, K, M, N, _lib.DTYPE_BF16, _status_ptr(cuda), st),
                   "pnft_gemm_at_b")
        outs.append(c)
    check_device_status(cuda)
    ref = a.float().t() @ b.float()
    assert torch.isfinite(outs[0]).all()
    assert (outs[0] - ref).abs().max() <= 1e-5 * ref.abs().max() + 1e-6 * K ** 0.5, float((outs[0] - ref).abs().max())
    assert torch.equal(outs[0], outs[1])


def test_linear_module_matches_nn_linear(cuda):
    """lm_ops.Linear (weight gradient from pnft_gemm_at_b, bias gradient from the
    column sum) against nn.Linear under bf16 autocast on the same parameters."""
    torch.manual_seed(2)
    ref = torch.nn.Linear(256, 768).to(cuda)
    lin = Linear.sharing(torch.nn.Linear(256, 768).to(cuda))
    lin.load_state_dict(ref.state_dict())
    x = torch.randn(32, 512, 256, device=cuda)
    xa, xb = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
    gy = torch.randn(32, 512, 768, device=cuda).to(torch.bfloat16)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ya, yb = lin(xa), ref(xb)
    assert ya.dtype == yb.dtype == torch.bfloat16 and torch.equal(ya, yb)
    ya.backward(gy)
    yb.backward(gy)
    assert rel_l2(xa.grad, xb.grad) < 1e-2
    # the library's gradients are fp32 sums of the bf16 products; autocast's are rounded to bf16
    assert rel_l2(lin.weight.grad, ref.weight.grad) < 5e-3 and rel_l2(lin.bias.grad, ref.bias.grad) < 5e-3


def test_bf16_casts_match_per_tensor_casts(cuda):
    """pnft_cast_bf16 through Bf16Casts: every copy bitwise equal to .to(bf16)
    (16-byte aligned tensors, unaligned views, lengths that are not multiples of
    8, one element), the padded copy's extra rows zero, copies withheld once a
    parameter changes in place and handed out again after the next refresh."""
    from paper_01_anti_decoy_pnfirtau_b200.lm_ops import Bf16Casts

    g = torch.Generator(device=cuda).manual_seed(11)
    flat = torch.randn(50000, device=cuda, generator=g) * 100
    ts = [torch.randn(1000, 256, device=cuda, generator=g), flat[1:1 + 1001], flat[2000:2000 + 8 * 37],
          flat[3003:3004], torch.randn(33278, 16, device=cuda, generator=g)]
    casts = Bf16Casts(ts, padded={id(ts[4]): 33280})
    casts.refresh()
    got = casts.lookup(*ts)
    assert got is not None
    for t, c in zip(ts, got):
        assert c.dtype == torch.bfloat16 and torch.equal(c, t.to(torch.bfloat16))
    pad = casts.padded(ts[4])
    assert pad.shape == (33280, 16) and torch.all(pad[33278:] == 0) and torch.equal(pad[:33278], got[4])
    assert casts.padded(ts[0]) is None  # no padded rows for it: lookup() only
    ts[0].add_(1.0)  # in place: a new version
    assert casts.lookup(ts[0]) is None and casts.lookup(ts[1]) is not None
    casts.refresh()
    assert torch.equal(casts.lookup(ts[0])[0], ts[0].to(torch.bfloat16))
    assert casts.lookup(torch.zeros(3, device=cuda)) is None  # not one of its parameters


def test_lm_step_casts_change_nothing(cuda):
    """The LM's one-launch bf16 copies of its GEMM parameters give the same loss,
    bit for bit, as casting every weight per GEMM, and the same gradients up to
    the attention's dQ accumulation order (atomic adds across key tiles)."""
    cfg = LMConfig(max_seq=128)
    torch.manual_seed(3)
    a = PnFirLM(cfg).to(cuda)
    b = PnFirLM(cfg).to(cuda)
    b.load_state_dict(a.state_dict())
    b._step_casts = lambda dev: None  # per-GEMM casts
    idx = torch.randint(0, cfg.vocab, (2, 128), device=cuda, generator=torch.Generator(device=cuda).manual_seed(4))
    out = []
    for m in (a, b):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = lm_loss(m, idx)
        loss.backward()
        out.append((loss.detach(), {n: p.grad for n, p in m.named_parameters()}))
    check_device_status(cuda)
    assert a._casts is not None and b._casts is None
    assert torch.equal(out[0][0], out[1][0])
    for n in out[0][1]:
        assert rel_l2(out[0][1][n], out[1][1][n]) < 1e-4, (n, rel_l2(out[0][1][n], out[1][1][n]))


def _lm_pair(cuda, N=128, B=4):
    cfg = LMConfig(max_seq=N)
    torch.manual_seed(3)
    fused = PnFirLM(cfg, fused_step_ops=True).to(cuda)
    plain = PnFirLM(cfg, fused_step_ops=False).to(cuda)
    plain.load_state_dict(fused.state_dict())
    g = torch.Generator(device=cuda).manual_seed(5)
    idx = torch.randint(0, cfg.vocab, (B, N), device=cuda, generator=g)
    return cfg, fused, plain, idx


def test_lm_fused_step_ops_match_pytorch_composition(cuda):
    """Config-4 model (D256 H4 L6 V33278) at a shorter sequence: loss and every
    parameter gradient of one bf16-autocast step, fused ops vs nn.LayerNorm +
    F.cross_entropy on the same weights."""
    cfg, fused, plain, idx = _lm_pair(cuda)
    assert list(fused.state_dict()) == list(plain.state_dict())
    losses = []
    for m in (fused, plain):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = lm_loss(m, idx)
        loss.backward()
        losses.append(float(loss))
    check_device_status(cuda)
    assert abs(losses[0] - losses[1]) < 2e-3 * abs(losses[1]), losses
    pf, pp = dict(fused.named_parameters()), dict(plain.named_parameters())
    for name in pf:
        assert rel_l2(pf[name].grad, pp[name].grad) < 2e-2, (name, rel_l2(pf[name].grad, pp[name].grad))


def test_lm_training_steps_track_pytorch_composition(cuda):
    """Three AdamW steps (fused AdamW for the fused model, the default foreach
    AdamW for the other): the loss trajectories stay together."""
    cfg, fused, plain, idx = _lm_pair(cuda)
    opt_f = make_optimizer(fused)
    opt_p = torch.optim.AdamW(plain.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    assert opt_f.defaults.get("fused")
    lf = [float(train_step(fused, opt_f, idx)) for _ in range(3)]
    lp = [float(train_step(plain, opt_p, idx)) for _ in range(3)]
    check_device_status(cuda)
    assert lf[-1] < lf[0] and lp[-1] < lp[0]
    for a, b in zip(lf, lp):
        assert abs(a - b) < 5e-3 * abs(b), (lf, lp)
