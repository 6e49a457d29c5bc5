"""Operators of the LM training step around the attention, on this library's
kernels (csrc/lm_step.cu): LayerNorm (alone or fused with the residual add
before it), the MLP's bias gradients and GELU backward, and the LM head's
next-token cross-entropy. They serve the Pre-LN decoder of the reference's
language-model experiments (experiments/exp4_wikitext2_lm.py:183-259, loss at
:714-719).

- ``LayerNorm``: ``nn.LayerNorm`` with the same parameters, ``eps`` and
  ``state_dict`` keys. Under CUDA autocast the normalised output is written
  directly in the autocast dtype: every consumer in the block is an autocast
  Linear that would round the fp32 output to that dtype anyway, so the values
  the GEMMs see are the same as ``nn.LayerNorm``'s, without the fp32 write and
  the cast copy. The parameter gradients are reduced in a fixed order.
- ``add_layer_norm(x, r, ...)``: ``s = x + r`` and ``LayerNorm(s)`` in one
  pass; its backward adds the residual path's gradient of ``s`` and writes the
  branch's gradient directly in the branch's dtype.
- ``mlp_gelu(x, fc1, fc2)``: ``fc2(GELU(fc1(x)))`` with the autocast GEMMs
  and this library's GELU (bf16: a per-CTA shared-memory table of the exact
  GELU over the bf16 bit patterns); the backward fuses the GELU derivative
  (tabulated the same way) with ``fc1``'s bias gradient, sums
  ``fc2``'s bias gradient with the same column-sum kernel (both fp32, fixed
  order) and produces the weight gradients from fp32-output GEMMs.
- ``Linear``: ``nn.Linear`` whose weight gradient comes from a split-K
  tcgen05 GEMM (the few, long reductions of dW = dY^T X over 16K tokens leave a
  library GEMM with too few CTAs); ``mlp_gelu`` uses the same kernel.
- ``head_cross_entropy``: ``F.cross_entropy(h @ W.T, targets)`` (mean over
  the rows whose target is not ``ignore_index``) with the bf16 head GEMM of
  autocast, and the loss and the logit gradient produced by one kernel pass over
  the logits, in place. The backward is two GEMMs on that gradient; the
  gradients of ``h`` and ``W`` are accumulated in fp32.
- ``Bf16Casts``: bf16 copies of a model's fp32 GEMM parameters made by one
  kernel launch per step (instead of one cast per GEMM), which ``Linear``,
  ``mlp_gelu`` and ``head_cross_entropy`` use while they are current.

CUDA only, like the attention operators; a CPU tensor raises.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .pnfirtau_ops import _check_pending, _require_cuda, _status_ptr, _stream

_LN_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def _ln_code(dtype: torch.dtype, what: str) -> int:
    try:
        return _LN_DTYPES[dtype]
    except KeyError:
        raise RuntimeError(f"{what}: float32 or bfloat16 expected, got {dtype}") from None


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, C: int, eps: float, out_dtype: torch.dtype):
        dev = _require_cuda("layer_norm", x, *(t for t in (weight, bias) if t is not None))
        x2 = x.reshape(-1, C)
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        M = x2.shape[0]
        y = torch.empty((M, C), dtype=out_dtype, device=dev)
        mean = torch.empty(M, dtype=torch.float32, device=dev)
        rstd = torch.empty(M, dtype=torch.float32, device=dev)
        w = None if weight is None else weight.detach().float().contiguous()
        b = None if bias is None else bias.detach().float().contiguous()
        rc = _lib.lib().pnft_layernorm_fwd(x2.data_ptr(), x2.stride(0), _ptr(w), _ptr(b), float(eps), y.data_ptr(),
                                           C, mean.data_ptr(), rstd.data_ptr(), M, C,
                                           _ln_code(x2.dtype, "layer_norm input"), _ln_code(out_dtype, "layer_norm output"),
                                           _stream(dev))
        _lib.check(rc, "pnft_layernorm_fwd")
        ctx.save_for_backward(x2, w, mean, rstd)
        ctx.shape, ctx.C = x.shape, C
        ctx.param_dtypes = (None if weight is None else weight.dtype, None if bias is None else bias.dtype)
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, gy):
        x2, w, mean, rstd = ctx.saved_tensors
        C, M, dev = ctx.C, x2.shape[0], x2.device
        gy2 = gy.reshape(-1, C)
        if gy2.dtype not in _LN_DTYPES:
            gy2 = gy2.float()
        if gy2.stride(-1) != 1:
            gy2 = gy2.contiguous()
        need_w = ctx.needs_input_grad[1] and w is not None
        need_b = ctx.needs_input_grad[2] and ctx.param_dtypes[1] is not None
        dx = torch.empty((M, C), dtype=x2.dtype, device=dev)
        dw = torch.empty(C, dtype=torch.float32, device=dev) if need_w else None
        db = torch.empty(C, dtype=torch.float32, device=dev) if need_b else None
        ws = None
        nbytes = 0
        if need_w or need_b:
            nbytes = _lib.lib().pnft_layernorm_bwd_workspace_size(M, C)
            ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        rc = _lib.lib().pnft_layernorm_bwd(gy2.data_ptr(), gy2.stride(0), x2.data_ptr(), x2.stride(0), _ptr(w),
                                           mean.data_ptr(), rstd.data_ptr(), dx.data_ptr(), C, _ptr(dw), _ptr(db),
                                           _ptr(ws), nbytes, M, C, _ln_code(gy2.dtype, "layer_norm grad"),
                                           _ln_code(x2.dtype, "layer_norm input"), _stream(dev))
        _lib.check(rc, "pnft_layernorm_bwd")
        wdt, bdt = ctx.param_dtypes
        return (dx.view(ctx.shape), None if dw is None else dw.to(wdt), None if db is None else db.to(bdt), None,
                None, None)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _autocast_dtype(x: torch.Tensor) -> torch.dtype:
    if x.is_cuda and torch.is_autocast_enabled("cuda"):
        dt = torch.get_autocast_dtype("cuda")
        if dt in _LN_DTYPES:
            return dt
    return x.dtype


def layer_norm(x: torch.Tensor, normalized_shape, weight: torch.Tensor | None = None,
               bias: torch.Tensor | None = None, eps: float = 1e-5, out_dtype: torch.dtype | None = None):
    """``F.layer_norm`` over the trailing ``normalized_shape`` dims on this
    library's kernels; ``out_dtype`` defaults to the autocast dtype under CUDA
    autocast, else to ``x.dtype``."""
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    C = math.prod(normalized_shape)
    if tuple(x.shape[x.dim() - len(normalized_shape):]) != tuple(normalized_shape):
        raise RuntimeError(f"layer_norm: input {tuple(x.shape)} does not end in {tuple(normalized_shape)}")
    xd = x if x.dtype in _LN_DTYPES else x.float()
    return _LayerNormFn.apply(xd, weight, bias, C, eps, out_dtype or _autocast_dtype(x))


class LayerNorm(nn.LayerNorm):
    """``nn.LayerNorm`` (same constructor, parameters and state_dict keys) on
    this library's LayerNorm kernels; see the module docstring for the output
    dtype under autocast."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return layer_norm(x, self.normalized_shape, self.weight, self.bias, self.eps)


class _AddLayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, r, weight, bias, C: int, eps: float, out_dtype: torch.dtype):
        dev = _require_cuda("add_layer_norm", x, r, *(t for t in (weight, bias) if t is not None))
        x2, r2 = x.reshape(-1, C), r.reshape(-1, C)
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        if r2.stride(-1) != 1:
            r2 = r2.contiguous()
        M = x2.shape[0]
        s = torch.empty((M, C), dtype=x2.dtype, device=dev)
        y = torch.empty((M, C), dtype=out_dtype, device=dev)
        mean = torch.empty(M, dtype=torch.float32, device=dev)
        rstd = torch.empty(M, dtype=torch.float32, device=dev)
        w = None if weight is None else weight.detach().float().contiguous()
        b = None if bias is None else bias.detach().float().contiguous()
        rc = _lib.lib().pnft_add_layernorm_fwd(
            x2.data_ptr(), x2.stride(0), r2.data_ptr(), r2.stride(0), _ln_code(r2.dtype, "add_layer_norm branch"),
            s.data_ptr(), C, _ptr(w), _ptr(b), float(eps), y.data_ptr(), C, mean.data_ptr(), rstd.data_ptr(), M, C,
            _ln_code(x2.dtype, "add_layer_norm input"), _ln_code(out_dtype, "add_layer_norm output"), _stream(dev))
        _lib.check(rc, "pnft_add_layernorm_fwd")
        ctx.save_for_backward(s, w, mean, rstd)
        ctx.shape, ctx.C, ctx.r_dtype = x.shape, C, r.dtype
        ctx.param_dtypes = (None if weight is None else weight.dtype, None if bias is None else bias.dtype)
        return s.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, gs, gy):
        s, w, mean, rstd = ctx.saved_tensors
        C, M, dev = ctx.C, s.shape[0], s.device
        gy2 = _rows(gy, C, s.dtype)
        gs2 = None if gs is None else _rows(gs, C, s.dtype, like=s.dtype)
        need_w = ctx.needs_input_grad[2] and w is not None
        need_b = ctx.needs_input_grad[3] and ctx.param_dtypes[1] is not None
        dx = torch.empty((M, C), dtype=s.dtype, device=dev) if ctx.needs_input_grad[0] else None
        dr = torch.empty((M, C), dtype=ctx.r_dtype, device=dev) if ctx.needs_input_grad[1] else None
        dw = torch.empty(C, dtype=torch.float32, device=dev) if need_w else None
        db = torch.empty(C, dtype=torch.float32, device=dev) if need_b else None
        if dx is None and dr is None:
            dx = torch.empty((M, C), dtype=s.dtype, device=dev)
        ws, nbytes = _ln_workspace(M, C, dev) if (need_w or need_b) else (None, 0)
        rc = _lib.lib().pnft_add_layernorm_bwd(
            gy2.data_ptr(), gy2.stride(0), _ptr(gs2), 0 if gs2 is None else gs2.stride(0), s.data_ptr(), C, _ptr(w),
            mean.data_ptr(), rstd.data_ptr(), _ptr(dx), C, _ptr(dr), C,
            _ln_code(ctx.r_dtype, "add_layer_norm branch"), _ptr(dw), _ptr(db), _ptr(ws), nbytes, M, C,
            _ln_code(gy2.dtype, "add_layer_norm grad"), _ln_code(s.dtype, "add_layer_norm input"), _stream(dev))
        _lib.check(rc, "pnft_add_layernorm_bwd")
        wdt, bdt = ctx.param_dtypes
        return (None if not ctx.needs_input_grad[0] else dx.view(ctx.shape),
                None if dr is None else dr.view(ctx.shape), None if dw is None else dw.to(wdt),
                None if db is None else db.to(bdt), None, None, None)


def _rows(t: torch.Tensor, C: int, fallback: torch.dtype, like: torch.dtype | None = None) -> torch.Tensor:
    """``t`` as contiguous-row ``[M, C]`` in a kernel dtype (``like`` forces one)."""
    t2 = t.reshape(-1, C)
    if like is not None and t2.dtype != like:
        t2 = t2.to(like)
    elif t2.dtype not in _LN_DTYPES:
        t2 = t2.to(fallback)
    return t2 if t2.stride(-1) == 1 else t2.contiguous()


def _ln_workspace(M: int, C: int, dev: torch.device):
    nbytes = _lib.lib().pnft_layernorm_bwd_workspace_size(M, C)
    return torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev), nbytes


def add_layer_norm(x: torch.Tensor, r: torch.Tensor, normalized_shape, weight: torch.Tensor | None = None,
                   bias: torch.Tensor | None = None, eps: float = 1e-5, out_dtype: torch.dtype | None = None):
    """``(s, LayerNorm(s))`` with ``s = x + r`` (PyTorch's type promotion:
    ``s`` takes the wider of the two dtypes), the LayerNorm as ``layer_norm``."""
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    C = math.prod(normalized_shape)
    if x.shape != r.shape:
        raise RuntimeError(f"add_layer_norm: x {tuple(x.shape)} and r {tuple(r.shape)} differ")
    sdt = torch.result_type(x, r)
    xd = x if x.dtype == sdt else x.to(sdt)
    if sdt not in _LN_DTYPES:
        xd = xd.float()
    rd = r if r.dtype in _LN_DTYPES else r.float()
    return _AddLayerNormFn.apply(xd, rd, weight, bias, C, eps, out_dtype or _autocast_dtype(x))


_GELU_TABLES: dict[int, torch.Tensor] = {}


def _gelu_table(dev: torch.device) -> torch.Tensor | None:
    """The device's GELU lookup table (pnft_gelu_table), built at the first call
    made outside CUDA-graph capture; during a capture that comes first the
    kernels build their own per-CTA copies (None)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _GELU_TABLES.get(idx)
    if t is None and not torch.cuda.is_current_stream_capturing():
        t = torch.empty(_lib.GELU_TABLE_FLOATS, dtype=torch.float32, device=dev)
        _lib.check(_lib.lib().pnft_gelu_table(t.data_ptr(), _stream(dev)), "pnft_gelu_table")
        _GELU_TABLES[idx] = t
    return t


def _colsum_ws(M: int, C: int, dev: torch.device):
    nbytes = _lib.lib().pnft_colsum_workspace_size(M, C)
    return torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev), nbytes


def _mm_f32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return torch.mm(a, b) if a.dtype == torch.float32 else torch.mm(a, b, out_dtype=torch.float32)


_SM100: dict[int, bool] = {}


def _is_sm100(dev: torch.device) -> bool:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _SM100:
        _SM100[idx] = torch.cuda.get_device_capability(idx) == (10, 0)
    return _SM100[idx]


def _weight_grad(dy: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """dW = dy^T x in fp32 (dy [K, M], x [K, N]: a Linear layer's weight gradient
    over K tokens): the split-K tcgen05 kernel (pnft_gemm_at_b) for bf16 rows it
    serves, else a library GEMM with fp32 output."""
    K, M = dy.shape
    N = x.shape[1]
    dev = dy.device
    if (dy.dtype == x.dtype == torch.bfloat16 and _is_sm100(dev) and M % 8 == 0 and N % 8 == 0
            and dy.stride(1) == 1 and x.stride(1) == 1 and dy.stride(0) % 8 == 0 and x.stride(0) % 8 == 0
            and dy.data_ptr() % 16 == 0 and x.data_ptr() % 16 == 0):
        out = torch.empty((M, N), dtype=torch.float32, device=dev)
        nbytes = _lib.lib().pnft_gemm_at_b_workspace_size(K, M, N)
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
        _lib.check(_lib.lib().pnft_gemm_at_b(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), out.data_ptr(), N,
                                             ws.data_ptr(), nbytes, K, M, N, _lib.DTYPE_BF16, _status_ptr(dev),
                                             _stream(dev)), "pnft_gemm_at_b")
        return out
    return _mm_f32(dy.t(), x)


def _cast(t: torch.Tensor | None, dt: torch.dtype) -> torch.Tensor | None:
    return None if t is None else t.to(dt)


class Bf16Casts:
    """bfloat16 copies of fp32 CUDA parameters, all refreshed by one kernel
    launch (``pnft_cast_bf16``), for the bf16 GEMMs of a training step: the LM
    refreshes them once at the start of each forward instead of casting every
    weight and bias per GEMM (the values are the same: round to nearest even).

    A copy is handed out only while its parameter still has the storage and the
    version counter seen at the last ``refresh()`` (an in-place update such as
    an optimizer step makes it stale until the next refresh). ``padded``: rows
    to pad a 2-D parameter to (its copy's extra rows stay zero), as the LM head's
    GEMM wants. The device table of addresses is written outside CUDA graph
    capture (the first refresh); a refresh inside a capture records only the
    kernel launch."""

    def __init__(self, params, padded: dict | None = None):
        self.params = [p for p in params if p is not None]
        if not self.params:
            raise ValueError("Bf16Casts: no parameters")
        dev = self.params[0].device
        for t in self.params:
            if t.device != dev or t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError("Bf16Casts: contiguous fp32 parameters on one CUDA device expected")
        self.device = dev
        self.index = {id(t): i for i, t in enumerate(self.params)}
        self.copies, self.full = [], {}
        for t in self.params:
            rows = (padded or {}).get(id(t))
            if rows:
                full = torch.zeros((rows, t.shape[1]), dtype=torch.bfloat16, device=dev)
                self.full[id(t)] = full
                self.copies.append(full[: t.shape[0]])
            else:
                self.copies.append(torch.empty(t.shape, dtype=torch.bfloat16, device=dev))
        self._ptrs: list[int] | None = None
        self._table: torch.Tensor | None = None
        self._seen: list[tuple[int, int]] = []

    def refresh(self) -> None:
        ptrs = [t.data_ptr() for t in self.params]
        if ptrs != self._ptrs:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("Bf16Casts: parameters moved during CUDA graph capture")
            rows = [[t.data_ptr(), c.data_ptr(), t.numel()] for t, c in zip(self.params, self.copies)]
            self._table = torch.tensor(rows, dtype=torch.int64).to(self.device)
            self._ptrs = ptrs
        n = max(t.numel() for t in self.params)
        _lib.check(_lib.lib().pnft_cast_bf16(self._table.data_ptr(), len(self.params), n, _stream(self.device)),
                   "pnft_cast_bf16")
        self._seen = [(t.data_ptr(), t._version) for t in self.params]

    def _current(self, t: torch.Tensor) -> int:
        i = self.index.get(id(t), -1)
        if i < 0 or not self._seen or self._seen[i] != (t.data_ptr(), t._version):
            return -1
        return i

    def lookup(self, *params):
        """The current copies of ``params`` (None entries stay None), or None if
        any of them has no current copy."""
        out = []
        for t in params:
            if t is None:
                out.append(None)
                continue
            i = self._current(t)
            if i < 0:
                return None
            out.append(self.copies[i])
        return tuple(out)

    def padded(self, t: torch.Tensor) -> torch.Tensor | None:
        """The zero-padded current copy of ``t`` (a parameter given ``padded``
        rows), or None."""
        return self.full.get(id(t)) if self._current(t) >= 0 else None


class _MlpGeluFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, dt: torch.dtype, pre=None):
        dev = _require_cuda("mlp_gelu", x, w1, w2)
        D = x.shape[-1]
        x2 = x.reshape(-1, D).to(dt)
        x2 = x2 if x2.stride(-1) == 1 else x2.contiguous()
        # pre: the parameters already cast to dt (Bf16Casts), else cast here
        w1c, b1c, w2c, b2c = pre if pre is not None else (_cast(w1, dt), _cast(b1, dt), _cast(w2, dt), _cast(b2, dt))
        a0 = torch.addmm(b1c, x2, w1c.t()) if b1 is not None else torch.mm(x2, w1c.t())
        a1 = torch.empty_like(a0)
        _lib.check(_lib.lib().pnft_gelu_fwd(a0.data_ptr(), a0.stride(0), a1.data_ptr(), a1.stride(0), a0.shape[0],
                                            a0.shape[1], _ln_code(dt, "mlp_gelu"), _ptr(_gelu_table(dev)),
                                            _stream(dev)), "pnft_gelu_fwd")
        out = torch.addmm(b2c, a1, w2c.t()) if b2 is not None else torch.mm(a1, w2c.t())
        ctx.save_for_backward(x2, w1c, w2c, a0, a1)
        ctx.x_shape, ctx.x_dtype, ctx.dev = x.shape, x.dtype, dev
        ctx.p_dtypes = tuple(None if t is None else t.dtype for t in (w1, b1, w2, b2))
        return out.view(*x.shape[:-1], out.shape[-1])

    @staticmethod
    def backward(ctx, g):
        x2, w1c, w2c, a0, a1 = ctx.saved_tensors
        dev, dt = ctx.dev, a0.dtype
        M, H, Dout = a0.shape[0], a0.shape[1], w2c.shape[0]
        g2 = _rows(g, Dout, dt, like=dt)
        L = _lib.lib()
        st = _stream(dev)
        dw1 = db1 = dw2 = db2 = dx = None
        if ctx.needs_input_grad[3]:
            dw2 = _weight_grad(g2, a1)
        if ctx.needs_input_grad[4]:
            db2 = torch.empty(Dout, dtype=torch.float32, device=dev)
            ws, nb = _colsum_ws(M, Dout, dev)
            _lib.check(L.pnft_colsum(g2.data_ptr(), g2.stride(0), db2.data_ptr(), ws.data_ptr(), nb, M, Dout,
                                     _ln_code(dt, "mlp_gelu"), st), "pnft_colsum")
        da1 = torch.mm(g2, w2c)
        da0 = torch.empty_like(a0)
        db1 = torch.empty(H, dtype=torch.float32, device=dev)
        ws, nb = _colsum_ws(M, H, dev)
        _lib.check(L.pnft_gelu_bwd_colsum(da1.data_ptr(), da1.stride(0), a0.data_ptr(), a0.stride(0), da0.data_ptr(),
                                          da0.stride(0), db1.data_ptr(), ws.data_ptr(), nb, M, H,
                                          _ln_code(dt, "mlp_gelu"), _ptr(_gelu_table(dev)), st),
                   "pnft_gelu_bwd_colsum")
        if ctx.needs_input_grad[1]:
            dw1 = _weight_grad(da0, x2)
        if ctx.needs_input_grad[0]:
            dx = torch.mm(da0, w1c).to(ctx.x_dtype).view(ctx.x_shape)
        pw1, pb1, pw2, pb2 = ctx.p_dtypes
        cast = lambda t, d: None if t is None else t.to(d)  # noqa: E731
        return (dx, cast(dw1, pw1), cast(db1, pb1) if ctx.needs_input_grad[2] else None, cast(dw2, pw2),
                cast(db2, pb2), None, None)


def mlp_gelu(x: torch.Tensor, fc1: nn.Linear, fc2: nn.Linear, casts: "Bf16Casts | None" = None) -> torch.Tensor:
    """``fc2(GELU(fc1(x)))`` (exact GELU) computed in the CUDA autocast dtype when
    autocast is on (else in ``x.dtype``); see the module docstring. ``casts``: a
    ``Bf16Casts`` holding current bf16 copies of the layers' parameters (used
    when the dtype is bf16 and every copy is current)."""
    dt = _autocast_dtype(x)
    if dt not in _LN_DTYPES:
        dt = torch.float32
    pre = casts.lookup(fc1.weight, fc1.bias, fc2.weight, fc2.bias) if casts is not None and dt == torch.bfloat16 else None
    return _MlpGeluFn.apply(x, fc1.weight, fc1.bias, fc2.weight, fc2.bias, dt, pre)


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, dt: torch.dtype, pre=None):
        _require_cuda("Linear", x, weight)
        D = x.shape[-1]
        x2 = x.reshape(-1, D).to(dt)
        x2 = x2 if x2.stride(-1) == 1 else x2.contiguous()
        w, b = pre if pre is not None else (weight.to(dt), _cast(bias, dt))  # pre: cast by Bf16Casts
        y = torch.addmm(b, x2, w.t()) if bias is not None else torch.mm(x2, w.t())
        ctx.save_for_backward(x2, w)
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        ctx.p_dtypes = (weight.dtype, None if bias is None else bias.dtype)
        return y.view(*x.shape[:-1], y.shape[-1])

    @staticmethod
    def backward(ctx, g):
        x2, w = ctx.saved_tensors
        dt, dev = x2.dtype, x2.device
        Dout = w.shape[0]
        g2 = _rows(g, Dout, dt, like=dt)
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = torch.mm(g2, w).to(ctx.x_dtype).view(ctx.x_shape)
        if ctx.needs_input_grad[1]:
            dw = _weight_grad(g2, x2).to(ctx.p_dtypes[0])
        if ctx.needs_input_grad[2]:
            db = torch.empty(Dout, dtype=torch.float32, device=dev)
            ws, nb = _colsum_ws(g2.shape[0], Dout, dev)
            _lib.check(_lib.lib().pnft_colsum(g2.data_ptr(), g2.stride(0), db.data_ptr(), ws.data_ptr(), nb,
                                              g2.shape[0], Dout, _ln_code(dt, "Linear"), _stream(dev)), "pnft_colsum")
            db = db.to(ctx.p_dtypes[1])
        return dx, dw, db, None, None


class Linear(nn.Linear):
    """``nn.Linear`` (same parameters and state_dict keys) whose forward is the
    autocast GEMM and whose backward computes the weight gradient with the
    split-K tcgen05 kernel (``pnft_gemm_at_b``, fp32) and the bias gradient
    with the fixed-order column sum. ``Linear.sharing(lin)`` wraps an existing
    layer's parameters without re-initialising anything. ``casts`` (plain
    attribute, default None): a ``Bf16Casts`` whose current bf16 copies of the
    parameters the bf16 GEMM uses instead of casting them per call."""

    casts: "Bf16Casts | None" = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = _autocast_dtype(x)
        if dt not in _LN_DTYPES:
            dt = torch.float32
        c = self.casts
        pre = c.lookup(self.weight, self.bias) if c is not None and dt == torch.bfloat16 else None
        return _LinearFn.apply(x, self.weight, self.bias, dt, pre)

    @classmethod
    def sharing(cls, lin: nn.Linear) -> "Linear":
        new = torch.nn.utils.skip_init(cls, lin.in_features, lin.out_features, bias=lin.bias is not None,
                                       device=lin.weight.device, dtype=lin.weight.dtype)
        new.weight = lin.weight
        if lin.bias is not None:
            new.bias = lin.bias
        return new


class _HeadXentFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, weight, targets, ignore_index: int, wpad=None):
        dev = _require_cuda("head_cross_entropy", h, weight, targets)
        _check_pending(dev)
        D = h.shape[-1]
        V = weight.shape[0]
        Vp = (V + 63) // 64 * 64  # 16-byte rows for the GEMMs and the staged kernel
        hb = h.reshape(-1, D).to(torch.bfloat16).contiguous()
        t = targets.reshape(-1).to(torch.int64).contiguous()
        M = hb.shape[0]
        if t.numel() != M:
            raise RuntimeError(f"head_cross_entropy: {M} rows but {t.numel()} targets")
        if wpad is not None:  # [Vp, D] bf16: the weight's current copy, zero rows past V
            wp = wpad
        else:
            wp = torch.empty((Vp, D), dtype=torch.bfloat16, device=dev)
            wp[:V].copy_(weight.detach())
            wp[V:].zero_()
        logits = torch.mm(hb, wp.t())  # [M, Vp] bf16, fp32 accumulation (the autocast head GEMM)
        counted = (t != ignore_index).sum(dtype=torch.float32)
        inv = torch.reciprocal(counted)
        row_loss = torch.empty(M, dtype=torch.float32, device=dev)
        rc = _lib.lib().pnft_lm_xent(logits.data_ptr(), Vp, t.data_ptr(), int(ignore_index), row_loss.data_ptr(), M,
                                     V, 1.0, inv.data_ptr(), _status_ptr(dev), _stream(dev))
        _lib.check(rc, "pnft_lm_xent")
        ctx.save_for_backward(logits, hb, wp)  # logits now hold d(loss)/d(logits)
        ctx.V, ctx.h_shape, ctx.h_dtype, ctx.w_dtype = V, h.shape, h.dtype, weight.dtype
        return row_loss.sum() * inv

    @staticmethod
    def backward(ctx, go):
        g, hb, wp = ctx.saved_tensors
        dh = dw = None
        if ctx.needs_input_grad[0]:
            dh = (torch.mm(g, wp, out_dtype=torch.float32) * go).to(ctx.h_dtype).view(ctx.h_shape)
        if ctx.needs_input_grad[1]:
            dw = (torch.mm(g.t(), hb, out_dtype=torch.float32)[: ctx.V] * go).to(ctx.w_dtype)
        return dh, dw, None, None, None


def head_cross_entropy(h: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
                       ignore_index: int = -100, *, casts: "Bf16Casts | None" = None) -> torch.Tensor:
    """Mean next-token cross-entropy of ``h @ weight.T`` against ``targets``
    (``F.cross_entropy`` semantics: rows whose target is ``ignore_index`` are
    left out of the mean). ``h``: ``[..., D]``; ``weight``: ``[V, D]`` (the LM
    head, tied to the embedding in the reference's model); ``targets``: the
    matching ``[...]`` int64 ids. The head GEMM runs in bf16 with fp32
    accumulation (as under bf16 autocast) and the loss is fp32. ``casts``
    (keyword only): a ``Bf16Casts`` holding a current bf16 copy of ``weight``
    padded to a multiple of 64 rows, used instead of casting it here."""
    wpad = casts.padded(weight) if casts is not None else None
    return _HeadXentFn.apply(h, weight, targets, ignore_index, wpad)
