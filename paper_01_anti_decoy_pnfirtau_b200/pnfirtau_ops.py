"""CUDA operators of pn_fir_tau with PyTorch autograd (counterpart of the
reference's ``src/triton_pnfirtau.py``).

Public functions keep the reference's names, signatures, defaults and return
types:

* ``triton_causal_fir(x, taps)``                      (src/triton_pnfirtau.py:685)
* ``triton_pn_fir_tau_scores(raw_scores, score_tau, scale=1.0, p=10.0,
  gamma=0.5, causal_mask=True)``                      (src/triton_pnfirtau.py:788)
* ``flash_pn_fir_tau_attention(q, k_tilde, v, score_tau, scale=None,
  gamma=0.5, causal_mask=True)``                      (src/triton_pnfirtau.py:971)

Every call runs hand-written sm_100a CUDA from libpnfirtau_b200.so through its
C ABI, on the caller's current CUDA stream. There is no Triton, no CPU path and
no silent fallback: CPU tensors raise ``RuntimeError``. Where the reference fell
back to eager PyTorch (more than 7 taps, C > 1024, N > 4096) these kernels
simply serve the shape.
"""
from __future__ import annotations

import math

import torch

from . import _lib

__all__ = [
    "triton_causal_fir",
    "triton_pn_fir_tau_scores",
    "flash_pn_fir_tau_attention",
    "pn_rows",
    "check_device_status",
    "flash_kernel_path",
]

_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}
_SILENCE = {"peak": _lib.SILENCE_PEAK, "mass_relu": _lib.SILENCE_MASS_RELU, "mass_pow": _lib.SILENCE_MASS_POW}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise RuntimeError(f"pn_fir_tau CUDA kernels support float32/bfloat16/float16, got {t.dtype}") from None


def _require_cuda(what: str, *tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(
                f"{what}: tensors must be on a CUDA device (this library has no CPU path); got {t.device}"
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{what}: all tensors must be on the same device ({dev} vs {t.device})")
    return dev


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class _StatusWord:
    """Per-device int32 word the tcgen05 kernels set to a PNFT_DEV_* code when a
    pipeline wait times out (their outputs are then invalid). It lives in pinned
    host memory mapped into the device, so the host sees a code as soon as the
    kernel writes it, with no copy and no synchronisation: every flash call
    first checks the word and raises if an earlier kernel on the device reported
    a failure. Where the mapping is unavailable the word is device memory, read
    only by check_device_status()."""

    def __init__(self, idx: int):
        import ctypes

        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        out = ctypes.c_void_p()
        with torch.cuda.device(idx):
            rc = _lib.lib().pnft_mapped_status_ptr(self.host.data_ptr(), ctypes.byref(out))
        if rc == _lib.OK and out.value:
            self.dev = None
            self.ptr = int(out.value)
        else:
            self.host = None
            self.dev = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            self.ptr = self.dev.data_ptr()

    def peek(self) -> int:
        """The code seen so far without synchronising (0 when only device memory holds it)."""
        return int(self.host[0]) if self.host is not None else _lib.DEV_OK

    def read(self) -> int:
        return int(self.host[0]) if self.host is not None else int(self.dev.item())

    def reset(self) -> None:
        (self.host if self.host is not None else self.dev).zero_()


_status: dict[int, _StatusWord] = {}


def _status_entry(dev: torch.device) -> _StatusWord:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _status.get(idx)
    if w is None:
        w = _status[idx] = _StatusWord(idx)
    return w


def _status_ptr(dev: torch.device) -> int:
    """Device address of `dev`'s status word, for the kernels' `status` argument."""
    return _status_entry(dev).ptr


_DEV_MEANING = {
    _lib.DEV_WAIT_TIMEOUT: "pipeline wait timed out; the outputs of that call are invalid",
    _lib.DEV_BAD_INDEX: "a cross-entropy target outside [0, vocab) that is not ignore_index; that row's loss is NaN",
}


def _raise(v: int, dev, when: str) -> None:
    what = _DEV_MEANING.get(v, "unknown device status")
    raise RuntimeError(f"pn_fir_tau kernel on {dev} reported device status {v} {when} ({what})")


def _check_pending(dev: torch.device) -> None:
    """Raises (and clears the word) if a kernel launched earlier on `dev` has
    reported a failure; costs one host read, no synchronisation."""
    w = _status_entry(dev)
    v = w.peek()
    if v != _lib.DEV_OK:
        w.reset()
        _raise(v, dev, "in an earlier call")


def check_device_status(device: torch.device | int | None = None, reset: bool = True) -> None:
    """Synchronise ``device`` and raise if a kernel on it reported a device-side error."""
    if device is None:
        device = torch.cuda.current_device()
    dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    torch.cuda.synchronize(dev)
    w = _status_entry(dev)
    v = w.read()
    if v != _lib.DEV_OK:
        if reset:
            w.reset()
        _raise(v, dev, "")


def _taps_f32(taps: torch.Tensor, dev: torch.device) -> torch.Tensor:
    if taps.dtype == torch.float32 and taps.is_contiguous() and taps.device == dev:
        return taps.detach()
    return taps.detach().contiguous().to(device=dev, dtype=torch.float32)


# ---------------------------------------------------------------------------
# 1. causal FIR
# ---------------------------------------------------------------------------


class _CausalFirFn(torch.autograd.Function):
    """Depthwise causal FIR along N of x[B,N,C] (src/triton_pnfirtau.py:629-682).

    The backward applies the transpose filter and, when ``taps`` requires grad,
    also returns the tap gradient (the reference returns None, :682).
    """

    @staticmethod
    def forward(ctx, x: torch.Tensor, taps: torch.Tensor) -> torch.Tensor:
        dev = _require_cuda("triton_causal_fir", x)
        B, N, C = x.shape
        taps_f32 = _taps_f32(taps, dev)
        y = torch.empty((B, N, C), device=dev, dtype=x.dtype)
        L = _lib.lib()
        _lib.check(
            L.pnft_fir_fwd(_ptr(x), *x.stride(), _ptr(taps_f32), taps_f32.numel(), _ptr(y), *y.stride(), B, N, C,
                           _dtype_code(x), _stream(dev)),
            "pnft_fir_fwd",
        )
        ctx.save_for_backward(taps_f32, x if ctx.needs_input_grad[1] else None)
        ctx.taps_dtype = taps.dtype
        return y

    @staticmethod
    def backward(ctx, grad_y: torch.Tensor):
        taps_f32, x = ctx.saved_tensors
        dev = grad_y.device
        B, N, C = grad_y.shape
        L = _lib.lib()
        gx = torch.empty((B, N, C), device=dev, dtype=grad_y.dtype) if ctx.needs_input_grad[0] else None
        dtaps = ws = None
        if x is not None:
            if grad_y.dtype != x.dtype:
                grad_y = grad_y.to(x.dtype)
            dtaps = torch.empty(taps_f32.numel(), device=dev, dtype=torch.float32)
            nbytes = L.pnft_fir_bwd_workspace_size(B, N, C, taps_f32.numel())
            ws = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
        if gx is None and x is None:
            return None, None
        _lib.check(
            L.pnft_fir_bwd(
                _ptr(grad_y), *grad_y.stride(), _ptr(taps_f32), taps_f32.numel(),
                _ptr(gx), *(gx.stride() if gx is not None else (0, 0, 0)),
                _ptr(x), *(x.stride() if x is not None else (0, 0, 0)),
                _ptr(dtaps), _ptr(ws), ws.numel() if ws is not None else 0,
                B, N, C, _dtype_code(grad_y), _stream(dev),
            ),
            "pnft_fir_bwd",
        )
        return gx, (dtaps.to(ctx.taps_dtype) if dtaps is not None else None)


def triton_causal_fir(x: torch.Tensor, taps: torch.Tensor) -> torch.Tensor:
    """Fused zero-copy depthwise 1D causal FIR along axis N for x: [B, N, C].

    Reference: src/triton_pnfirtau.py:685-691. Any tap count (1 tap or fewer is
    the identity, as the eager causal_fir, src/pnfirtau_attention.py:69-70)
    and any C run on the CUDA kernel.
    """
    if taps.numel() <= 1:
        _require_cuda("triton_causal_fir", x)
        return x
    return _CausalFirFn.apply(x, taps)


# ---------------------------------------------------------------------------
# 2. row-fused score -> weight op
# ---------------------------------------------------------------------------


def _gamma_args(gamma: float | None) -> tuple[int, float]:
    has_gamma = gamma is not None and gamma > 0.0
    return int(has_gamma), float(gamma) if has_gamma else 0.0


class _PnRowsFn(torch.autograd.Function):
    """Row-fused scale, -tau, causal mask, ReLU, u^p, peak/mass stats and gate.

    Forward/backward follow src/triton_pnfirtau.py:694-785, with the
    ``mass_relu`` / ``mass_pow`` silence modes and general p of the eager
    power_norm_peak_gate (src/pnfirtau_attention.py:87-119).
    """

    @staticmethod
    def forward(ctx, raw_scores, score_tau, scale, p, gamma, causal_mask, silence_mode):
        dev = _require_cuda("pn_fir_tau rows", raw_scores, score_tau)
        orig_shape = raw_scores.shape
        N = orig_shape[-1]
        s_2d = raw_scores.contiguous().view(-1, N)
        R = s_2d.shape[0]
        w_2d = torch.empty_like(s_2d)
        stats = torch.empty((4, R), device=dev, dtype=torch.float32)
        nmax = torch.empty(R, device=dev, dtype=torch.int32)
        tau_f32 = score_tau.detach().to(torch.float32).contiguous()
        has_gamma, gamma_val = _gamma_args(gamma)
        mode = _SILENCE[silence_mode]
        L = _lib.lib()
        _lib.check(
            L.pnft_rows_fwd(_ptr(s_2d), s_2d.stride(0), _ptr(tau_f32), _ptr(w_2d), w_2d.stride(0),
                            _ptr(stats[0]), _ptr(stats[1]), _ptr(nmax), _ptr(stats[2]), R, N, float(scale),
                            float(p), gamma_val, has_gamma, mode, int(bool(causal_mask)), _dtype_code(s_2d),
                            _stream(dev)),
            "pnft_rows_fwd",
        )
        ctx.save_for_backward(s_2d, tau_f32, stats, nmax)
        ctx.orig_shape = orig_shape
        ctx.args = (float(scale), float(p), gamma_val, has_gamma, mode, int(bool(causal_mask)))
        ctx.tau_dtype = score_tau.dtype
        ctx.tau_shape = score_tau.shape
        return w_2d.view(orig_shape)

    @staticmethod
    def backward(ctx, grad_w):
        s_2d, tau_f32, stats, nmax = ctx.saved_tensors
        scale, p, gamma_val, has_gamma, mode, causal = ctx.args
        R, N = s_2d.shape
        dev = s_2d.device
        gw_2d = grad_w.to(s_2d.dtype).contiguous().view(R, N)
        grad_s = torch.empty_like(s_2d)
        dtau_rows = torch.empty(R, device=dev, dtype=torch.float32)
        dtau = torch.empty((), device=dev, dtype=torch.float32)
        L = _lib.lib()
        _lib.check(
            L.pnft_rows_bwd(_ptr(gw_2d), gw_2d.stride(0), _ptr(s_2d), s_2d.stride(0), _ptr(tau_f32),
                            _ptr(stats[0]), _ptr(stats[1]), _ptr(nmax), _ptr(stats[2]), _ptr(grad_s),
                            grad_s.stride(0), _ptr(dtau_rows), _ptr(dtau), R, N, scale, p, gamma_val, has_gamma,
                            mode, causal, _dtype_code(s_2d), _stream(dev)),
            "pnft_rows_bwd",
        )
        grad_tau = dtau.to(ctx.tau_dtype).reshape(ctx.tau_shape)
        return grad_s.view(ctx.orig_shape), grad_tau, None, None, None, None, None


def pn_rows(raw_scores, score_tau, scale=1.0, p=10.0, gamma=0.5, causal_mask=True, silence_mode="peak"):
    """Row op with every silence mode of power_norm_peak_gate (peak, mass_relu, mass_pow)."""
    if silence_mode not in _SILENCE:
        if gamma is not None and gamma > 0:
            raise ValueError(f"unknown silence_mode={silence_mode}")
        silence_mode = "peak"  # the eager primitive only inspects the mode when a gate is applied
    N = raw_scores.shape[-1]
    assert raw_scores.shape[-2] == N or not causal_mask, "Expected [..., N, N] scores tensor"
    return _PnRowsFn.apply(raw_scores, score_tau, scale, p, gamma, causal_mask, silence_mode)


def triton_pn_fir_tau_scores(
    raw_scores: torch.Tensor,
    score_tau: torch.Tensor,
    scale: float = 1.0,
    p: float = 10.0,
    gamma: float | None = 0.5,
    causal_mask: bool = True,
) -> torch.Tensor:
    """Fused row-wise score-to-weight kernel for ``pn_fir_tau`` (src/triton_pnfirtau.py:788-811).

    Same contract as the reference: ``raw_scores`` is ``[..., N, N]``; the
    result has its shape and dtype; the silence test is the row peak.
    """
    N = raw_scores.shape[-1]
    assert raw_scores.shape[-2] == N, "Expected [..., N, N] scores tensor"
    return _PnRowsFn.apply(raw_scores, score_tau, scale, p, gamma, causal_mask, "peak")


# ---------------------------------------------------------------------------
# 3. flash pn_fir_tau attention
# ---------------------------------------------------------------------------


def _flash_flags(deterministic: bool | None = None) -> int:
    """PNFT_FLASH_* bits of a flash call. deterministic=None follows
    torch.are_deterministic_algorithms_enabled()."""
    if deterministic is None:
        deterministic = torch.are_deterministic_algorithms_enabled()
    return ((_lib.FLASH_FORCE_GENERIC if _FORCE_GENERIC else 0) | (_lib.FLASH_DETERMINISTIC if deterministic else 0)
            | _TEST_FLAGS)


_FORCE_GENERIC = False
# Test-only PNFT_FLASH_* bits OR-ed into every flash call (forward and backward),
# e.g. FLASH_TEST_STALL to exercise the kernels' timeout path.
_TEST_FLAGS = 0


def flash_kernel_path(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> str:
    """'sm100' if the tcgen05/TMA kernels serve these tensors, else 'generic'."""
    L = _lib.lib()
    r = L.pnft_flash_path(_ptr(q), _lib.i64x4(q.stride()), _ptr(k), _lib.i64x4(k.stride()), _ptr(v),
                          _lib.i64x4(v.stride()), q.shape[-1], _dtype_code(q), _flash_flags())
    return "sm100" if r == 1 else "generic"


class _FlashPnFirTauFn(torch.autograd.Function):
    """O(N)-memory tiled pn_fir_tau attention, p = 10 (src/triton_pnfirtau.py:814-968).

    q, k, v are read through their strides (no .contiguous() copies). The
    output is allocated ``[B,H,N,D]`` contiguous, or, with ``out_layout ==
    'bnhd'``, as a ``[B,N,H,D]`` buffer returned through a transposed view so
    the module's ``transpose(1,2).reshape`` is free.
    """

    @staticmethod
    def forward(ctx, q, k, v, score_tau, scale, gamma, causal_mask, out_layout, deterministic=None):
        dev = _require_cuda("flash_pn_fir_tau_attention", q, k, v, score_tau)
        _check_pending(dev)
        if not (q.dtype == k.dtype == v.dtype):
            raise RuntimeError(f"flash_pn_fir_tau_attention: q/k/v dtypes differ ({q.dtype}, {k.dtype}, {v.dtype})")
        B, H, N, D = q.shape
        if k.shape != q.shape or v.shape != q.shape:
            raise RuntimeError(f"flash_pn_fir_tau_attention: q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)} must match")
        if out_layout == "bnhd":
            out = torch.empty((B, N, H, D), device=dev, dtype=q.dtype).transpose(1, 2)
        else:
            out = torch.empty((B, H, N, D), device=dev, dtype=q.dtype)
        stats = torch.empty((2, B, H, N), device=dev, dtype=torch.float32)  # peak, mass + 1e-12
        nmax = torch.empty((2, B, H, N), device=dev, dtype=torch.int32)    # tie count, argmax key
        tau_f32 = score_tau.detach().to(torch.float32).contiguous()
        has_gamma, gamma_val = _gamma_args(gamma)
        flags = _flash_flags(deterministic)
        # fp32 copy of O for the backward's per-row <dO,O>/gate (see pnft_flash_fwd)
        needs_grad = any(ctx.needs_input_grad[:4])
        out32 = None
        if needs_grad and q.dtype != torch.float32:
            out32 = torch.empty((B, H, N, D), device=dev, dtype=torch.float32)
        L = _lib.lib()
        # the backward must recompute S with the forward's arithmetic (its tie test
        # is u == peak), so it is pinned to the kernel family the forward used
        if L.pnft_flash_path(_ptr(q), _lib.i64x4(q.stride()), _ptr(k), _lib.i64x4(k.stride()), _ptr(v),
                             _lib.i64x4(v.stride()), D, _dtype_code(q), flags) == 0:
            flags |= _lib.FLASH_FORCE_GENERIC
        _lib.check(
            L.pnft_flash_fwd(_ptr(q), _lib.i64x4(q.stride()), _ptr(k), _lib.i64x4(k.stride()), _ptr(v),
                             _lib.i64x4(v.stride()), _ptr(tau_f32), _ptr(out), _lib.i64x4(out.stride()),
                             _ptr(out32), _ptr(stats[0]), _ptr(stats[1]), _ptr(nmax[0]), _ptr(nmax[1]), B, H, N,
                             D, float(scale), gamma_val, has_gamma, int(bool(causal_mask)), _dtype_code(q), flags,
                             None,
                             _status_ptr(dev), _stream(dev)),
            "pnft_flash_fwd",
        )
        ctx.save_for_backward(q, k, v, tau_f32, out, out32, stats, nmax)
        ctx.args = (float(scale), gamma_val, has_gamma, int(bool(causal_mask)), flags)
        ctx.tau_dtype = score_tau.dtype
        ctx.tau_shape = score_tau.shape
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, tau_f32, out, out32, stats, nmax = ctx.saved_tensors
        scale, gamma_val, has_gamma, causal, flags = ctx.args
        flags |= _TEST_FLAGS
        B, H, N, D = q.shape
        dev = q.device
        _check_pending(dev)
        if grad_out.dtype != q.dtype:
            grad_out = grad_out.to(q.dtype)
        if grad_out.stride(-1) != 1 or any(s % 8 for s in grad_out.stride()[:3]):
            grad_out = grad_out.contiguous()  # TMA-loadable, so the backward keeps the forward's path
        dq = torch.empty((B, H, N, D), device=dev, dtype=q.dtype)
        dk = torch.empty((B, H, N, D), device=dev, dtype=k.dtype)
        dv = torch.empty((B, H, N, D), device=dev, dtype=v.dtype)
        dtau = torch.empty((), device=dev, dtype=torch.float32)
        L = _lib.lib()
        nbytes = L.pnft_flash_bwd_workspace_size(B, H, N, D, flags)
        ws = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
        _lib.check(
            L.pnft_flash_bwd(_ptr(q), _lib.i64x4(q.stride()), _ptr(k), _lib.i64x4(k.stride()), _ptr(v),
                             _lib.i64x4(v.stride()), _ptr(tau_f32), _ptr(out), _lib.i64x4(out.stride()),
                             _ptr(out32), _ptr(grad_out), _lib.i64x4(grad_out.stride()), _ptr(stats[0]),
                             _ptr(stats[1]), _ptr(nmax[0]), _ptr(nmax[1]), _ptr(dq), _lib.i64x4(dq.stride()),
                             _ptr(dk), _lib.i64x4(dk.stride()),
                             _ptr(dv), _lib.i64x4(dv.stride()), _ptr(dtau), _ptr(ws), ws.numel(), B, H, N, D,
                             scale, gamma_val, has_gamma, causal, _dtype_code(q), flags,
                             _status_ptr(dev), _stream(dev)),
            "pnft_flash_bwd",
        )
        grad_tau = dtau.to(ctx.tau_dtype).reshape(ctx.tau_shape)
        return dq, dk, dv, grad_tau, None, None, None, None, None


def flash_pn_fir_tau_attention(
    q: torch.Tensor,
    k_tilde: torch.Tensor,
    v: torch.Tensor,
    score_tau: torch.Tensor,
    scale: float | None = None,
    gamma: float | None = 0.5,
    causal_mask: bool = True,
    *,
    deterministic: bool | None = None,
) -> torch.Tensor:
    """FlashAttention-style O(N)-memory tiled attention for ``pn_fir_tau`` (p = 10).

    Reference: src/triton_pnfirtau.py:971-983. ``scale`` defaults to
    1/sqrt(head_dim). Returns ``[B, H, N, D]`` in q's dtype.

    ``deterministic`` (keyword only, an addition to the reference's signature):
    the backward adds the dQ contributions of the key tiles in a fixed order,
    so every gradient is bitwise reproducible run to run (dK, dV and dtau always
    are); None follows ``torch.use_deterministic_algorithms``. The reference's
    backward accumulates dQ with atomics (src/triton_pnfirtau.py:596-602).
    """
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    return _FlashPnFirTauFn.apply(q, k_tilde, v, score_tau, scale, gamma, causal_mask, "bhnd", deterministic)


def _fir_view(t: torch.Tensor):
    """[B,H,N,D] key tensor as the FIR's [Bf, N, C] (strides, Bf, C): head dims
    adjacent -> [B, N, H*D]; else b and h adjacent -> [B*H, N, D]."""
    B, H, N, D = t.shape
    st = t.stride()
    if st[3] == 1 and (H == 1 or st[1] == D):
        return (st[0], st[2], 1), B, H * D
    if st[3] == 1 and st[0] == H * st[1]:
        return (st[1], st[2], 1), B * H, D
    raise RuntimeError(f"flash_pn_fir_tau_attention_fir: key strides {tuple(st)} have neither (h, d) nor (b, h) "
                       "adjacent")


def _fir_forward(q, k, v, score_tau, taps, scale, gamma, causal_mask, out_layout, fused_forward, deterministic,
                 needs_grad: bool):
    """Forward of flash attention on k~ = causal_fir(k, taps) (see _FlashFirFn).
    Returns (out, saved tensors, saved arguments) for _fir_backward."""
    dev = _require_cuda("flash_pn_fir_tau_attention_fir", q, k, v, score_tau, taps)
    _check_pending(dev)
    if not (q.dtype == k.dtype == v.dtype):
        raise RuntimeError(f"flash_pn_fir_tau_attention_fir: q/k/v dtypes differ ({q.dtype}, {k.dtype}, {v.dtype})")
    B, H, N, D = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise RuntimeError(f"flash_pn_fir_tau_attention_fir: q {tuple(q.shape)}, k {tuple(k.shape)}, "
                           f"v {tuple(v.shape)} must match")
    if taps.numel() != _lib.FIR_FUSED_TAPS:
        raise RuntimeError(f"flash_pn_fir_tau_attention_fir: {taps.numel()} taps; the fused filter has "
                           f"{_lib.FIR_FUSED_TAPS}")
    if out_layout == "bnhd":
        out = torch.empty((B, N, H, D), device=dev, dtype=q.dtype).transpose(1, 2)
    else:
        out = torch.empty((B, H, N, D), device=dev, dtype=q.dtype)
    stats = torch.empty((2, B, H, N), device=dev, dtype=torch.float32)
    nmax = torch.empty((2, B, H, N), device=dev, dtype=torch.int32)
    tau_f32 = score_tau.detach().to(torch.float32).contiguous()
    taps_f32 = taps.detach().to(torch.float32).contiguous()
    has_gamma, gamma_val = _gamma_args(gamma)
    flags = _flash_flags(deterministic)
    out32 = torch.empty((B, H, N, D), device=dev, dtype=torch.float32) if needs_grad else None
    L = _lib.lib()
    if fused_forward:
        _lib.check(
            L.pnft_flash_fwd_fir(_ptr(q), _lib.i64x4(q.stride()), _ptr(k), _lib.i64x4(k.stride()),
                                 _ptr(taps_f32), taps_f32.numel(), _ptr(v), _lib.i64x4(v.stride()),
                                 _ptr(tau_f32), _ptr(out), _lib.i64x4(out.stride()), _ptr(out32),
                                 _ptr(stats[0]), _ptr(stats[1]), _ptr(nmax[0]), _ptr(nmax[1]), B, H, N, D,
                                 float(scale), gamma_val, has_gamma, int(bool(causal_mask)), _dtype_code(q),
                                 flags, None, _status_ptr(dev), _stream(dev)),
            "pnft_flash_fwd_fir",
        )
    else:
        (sxb, sxn, sxc), Bf, C = _fir_view(k)
        # k~ in the layout of k's FIR view, contiguous
        if C == H * D and (H == 1 or k.stride(1) == D):
            kt = torch.empty((B, N, H, D), device=dev, dtype=k.dtype).transpose(1, 2)
            syb, syn = N * H * D, H * D
        else:
            kt = torch.empty((B, H, N, D), device=dev, dtype=k.dtype)
            syb, syn = N * D, D
        _lib.check(L.pnft_fir_fwd(_ptr(k), sxb, sxn, sxc, _ptr(taps_f32), taps_f32.numel(), _ptr(kt), syb, syn,
                                  1, Bf, N, C, _dtype_code(k), _stream(dev)), "pnft_fir_fwd")
        if L.pnft_flash_path(_ptr(q), _lib.i64x4(q.stride()), _ptr(kt), _lib.i64x4(kt.stride()), _ptr(v),
                             _lib.i64x4(v.stride()), D, _dtype_code(q), flags) != 1:
            raise RuntimeError("flash_pn_fir_tau_attention_fir: the sm_100a kernels do not serve these inputs")
        _lib.check(
            L.pnft_flash_fwd(_ptr(q), _lib.i64x4(q.stride()), _ptr(kt), _lib.i64x4(kt.stride()), _ptr(v),
                             _lib.i64x4(v.stride()), _ptr(tau_f32), _ptr(out), _lib.i64x4(out.stride()),
                             _ptr(out32), _ptr(stats[0]), _ptr(stats[1]), _ptr(nmax[0]), _ptr(nmax[1]), B, H, N,
                             D, float(scale), gamma_val, has_gamma, int(bool(causal_mask)), _dtype_code(q),
                             flags, None, _status_ptr(dev), _stream(dev)),
            "pnft_flash_fwd",
        )
    saved = (tau_f32, taps_f32, out, out32, stats, nmax)
    args = (float(scale), gamma_val, has_gamma, int(bool(causal_mask)), flags)
    return out, saved, args


def _fir_backward(q, k, v, saved, args, grad_out, dq, dk, dv, want_dtaps: bool):
    """Backward of _fir_forward into the caller's dq / dk / dv (any strides the
    kernels accept: dk with k's adjacent axes). Returns (dtau fp32 scalar,
    dtaps fp32 or None)."""
    tau_f32, taps_f32, out, out32, stats, nmax = saved
    scale, gamma_val, has_gamma, causal, flags = args
    flags |= _TEST_FLAGS
    B, H, N, D = q.shape
    dev = q.device
    _check_pending(dev)
    if grad_out.dtype != q.dtype:
        grad_out = grad_out.to(q.dtype)
    if grad_out.stride(-1) != 1 or any(s % 8 for s in grad_out.stride()[:3]):
        grad_out = grad_out.contiguous()
    dtau = torch.empty((), device=dev, dtype=torch.float32)
    dtaps = torch.empty(taps_f32.numel(), device=dev, dtype=torch.float32) if want_dtaps else None
    L = _lib.lib()
    nbytes = L.pnft_flash_bwd_fir_workspace_size(B, H, N, D, flags)
    ws = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
    _lib.check(
        L.pnft_flash_bwd_fir(_ptr(q), _lib.i64x4(q.stride()), _ptr(k), _lib.i64x4(k.stride()), _ptr(taps_f32),
                             taps_f32.numel(), _ptr(v), _lib.i64x4(v.stride()), _ptr(tau_f32), _ptr(out),
                             _lib.i64x4(out.stride()), _ptr(out32), _ptr(grad_out),
                             _lib.i64x4(grad_out.stride()), _ptr(stats[0]), _ptr(stats[1]), _ptr(nmax[0]),
                             _ptr(nmax[1]), _ptr(dq), _lib.i64x4(dq.stride()), _ptr(dk),
                             _lib.i64x4(dk.stride()), _ptr(dv), _lib.i64x4(dv.stride()), _ptr(dtau),
                             _ptr(dtaps), _ptr(ws), ws.numel(), B, H, N, D, scale, gamma_val, has_gamma, causal,
                             _dtype_code(q), flags, _status_ptr(dev), _stream(dev)),
        "pnft_flash_bwd_fir",
    )
    return dtau, dtaps


class _FlashFirFn(torch.autograd.Function):
    """Flash attention on the causally filtered keys k~ = causal_fir(k, taps), k
    the raw key projection. Backward: pnft_flash_bwd_fir, which filters its K
    tile in shared memory from k (nothing of k~ is kept) and returns the raw
    key's gradient and the tap gradient. Forward: by default one standalone
    filter pass (pnft_fir_fwd) and pnft_flash_fwd on k~; with fused_forward the
    filter runs in the forward kernel's K-tile load instead (pnft_flash_fwd_fir),
    which repeats it for every query tile that reads a key tile and is slower.
    Both forwards give the same k~ bit for bit."""

    @staticmethod
    def forward(ctx, q, k, v, score_tau, taps, scale, gamma, causal_mask, out_layout, fused_forward=False,
                deterministic=None):
        out, saved, args = _fir_forward(q, k, v, score_tau, taps, scale, gamma, causal_mask, out_layout,
                                        fused_forward, deterministic, any(ctx.needs_input_grad[:5]))
        ctx.save_for_backward(q, k, v, *saved)
        ctx.args = args
        ctx.tau_dtype, ctx.tau_shape = score_tau.dtype, score_tau.shape
        ctx.taps_dtype, ctx.taps_shape = taps.dtype, taps.shape
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, *saved = ctx.saved_tensors
        B, H, N, D = q.shape
        dev = q.device
        dq = torch.empty((B, H, N, D), device=dev, dtype=q.dtype)
        # dk with k's adjacent axes: (h, d) for the module's [B,N,H*D] view, else (b, h)
        if H == 1 or k.stride(1) == D:
            dk = torch.empty((B, N, H, D), device=dev, dtype=k.dtype).transpose(1, 2)
        else:
            dk = torch.empty((B, H, N, D), device=dev, dtype=k.dtype)
        dv = torch.empty((B, H, N, D), device=dev, dtype=v.dtype)
        dtau, dtaps = _fir_backward(q, k, v, saved, ctx.args, grad_out, dq, dk, dv, ctx.needs_input_grad[4])
        grad_tau = dtau.to(ctx.tau_dtype).reshape(ctx.tau_shape)
        grad_taps = dtaps.to(ctx.taps_dtype).reshape(ctx.taps_shape) if dtaps is not None else None
        return dq, dk, dv, grad_tau, grad_taps, None, None, None, None, None, None


def _qkv_views(qkv: torch.Tensor, H: int):
    """q, k, v as [B,H,N,D] views of the three column blocks of qkv [B,N,3*H*D]."""
    B, N, C3 = qkv.shape
    D = C3 // (3 * H)
    return tuple(t.view(B, N, H, D).transpose(1, 2) for t in qkv.split(H * D, dim=-1))


class _FlashFirQkvFn(torch.autograd.Function):
    """_FlashFirFn on the module's fused projection qkv [B,N,3*H*D] (q, k, v its
    column blocks). The backward writes dq, dk and dv straight into the column
    blocks of one d(qkv) tensor, so no gradient concatenation follows it (the
    backward of ``qkv.chunk(3)``); the result is stored as [B,N,H,D]."""

    @staticmethod
    def forward(ctx, qkv, H: int, score_tau, taps, scale, gamma, causal_mask, deterministic=None):
        q, k, v = _qkv_views(qkv, H)
        out, saved, args = _fir_forward(q, k, v, score_tau, taps, scale, gamma, causal_mask, "bnhd", False,
                                        deterministic, any(ctx.needs_input_grad[:4]))
        ctx.save_for_backward(qkv, *saved)
        ctx.H, ctx.args = H, args
        ctx.tau_dtype, ctx.tau_shape = score_tau.dtype, score_tau.shape
        ctx.taps_dtype, ctx.taps_shape = taps.dtype, taps.shape
        return out

    @staticmethod
    def backward(ctx, grad_out):
        qkv, *saved = ctx.saved_tensors
        q, k, v = _qkv_views(qkv, ctx.H)
        dqkv = torch.empty_like(qkv, memory_format=torch.contiguous_format)
        dq, dk, dv = _qkv_views(dqkv, ctx.H)
        dtau, dtaps = _fir_backward(q, k, v, saved, ctx.args, grad_out, dq, dk, dv, ctx.needs_input_grad[3])
        grad_tau = dtau.to(ctx.tau_dtype).reshape(ctx.tau_shape)
        grad_taps = dtaps.to(ctx.taps_dtype).reshape(ctx.taps_shape) if dtaps is not None else None
        return dqkv, None, grad_tau, grad_taps, None, None, None, None


def flash_pn_fir_tau_attention_fir(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    score_tau: torch.Tensor,
    taps: torch.Tensor,
    scale: float | None = None,
    gamma: float | None = 0.5,
    causal_mask: bool = True,
    fused_forward: bool = False,
    *,
    deterministic: bool | None = None,
) -> torch.Tensor:
    """``flash_pn_fir_tau_attention(q, triton_causal_fir(k, taps), v, ...)`` with
    the 7-tap causal FIR in the attention kernels' K-tile load: each K tile is
    staged with its 8 preceding rows and filtered in shared memory, bit-identical
    to ``triton_causal_fir``. The backward always filters in its kernel (one key
    tile per CTA); the forward does with ``fused_forward=True``, and otherwise
    runs one standalone filter pass, which is faster there because every query
    tile re-reads the key tiles. ``k`` is the raw key projection ``[B, H, N, D]``
    (bf16, head dims that are multiples of 16 up to 128; sm_100a kernels only). Gradients reach ``k`` and, when
    it requires grad, ``taps``. ``deterministic`` as in flash_pn_fir_tau_attention.
    Composition replaced: src/pnfirtau_attention.py:285-316."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    return _FlashFirFn.apply(q, k, v, score_tau, taps, scale, gamma, causal_mask, "bhnd", fused_forward, deterministic)


@torch.no_grad()
def flash_pn_fir_tau_forward_stats(q, k_tilde, v, score_tau, scale=None, gamma=0.5, causal_mask=True,
                                   extra_flags: int = 0):
    """Forward only, also returning the per-row statistics and the kernel's
    silent-tile decisions: ``(out, M, Z, Nmax, tile_live)`` with M/Z/Nmax
    ``[B,H,N]`` (peak, mass + 1e-12, tie count, src/triton_pnfirtau.py:440-443)
    and ``tile_live`` bool ``[B,H,nT,nT]`` (nT = ceil(N/64)) true for every
    64x64 tile the kernel processed as live. ``extra_flags`` are PNFT_FLASH_*
    bits (e.g. to select a kernel family for a comparison)."""
    dev = _require_cuda("flash_pn_fir_tau_forward_stats", q, k_tilde, v, score_tau)
    _check_pending(dev)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    B, H, N, D = q.shape
    out = torch.empty((B, H, N, D), device=dev, dtype=q.dtype)
    stats = torch.empty((2, B, H, N), device=dev, dtype=torch.float32)
    nmax = torch.empty((2, B, H, N), device=dev, dtype=torch.int32)
    nT = (N + 63) // 64
    tiles = torch.zeros((B, H, nT, nT), device=dev, dtype=torch.uint8)
    tau_f32 = score_tau.detach().to(torch.float32).contiguous()
    has_gamma, gamma_val = _gamma_args(gamma)
    L = _lib.lib()
    _lib.check(
        L.pnft_flash_fwd(_ptr(q), _lib.i64x4(q.stride()), _ptr(k_tilde), _lib.i64x4(k_tilde.stride()), _ptr(v),
                         _lib.i64x4(v.stride()), _ptr(tau_f32), _ptr(out), _lib.i64x4(out.stride()), None,
                         _ptr(stats[0]), _ptr(stats[1]), _ptr(nmax[0]), _ptr(nmax[1]), B, H, N, D, float(scale),
                         gamma_val, has_gamma, int(bool(causal_mask)), _dtype_code(q), _flash_flags() | extra_flags,
                         _ptr(tiles), _status_ptr(dev), _stream(dev)),
        "pnft_flash_fwd",
    )
    return out, stats[0], stats[1], nmax[0], tiles.bool()


def _flash_bnhd(q, k_tilde, v, score_tau, scale, gamma, causal_mask):
    """Same op; the result's storage is [B,N,H,D] (free transpose back to tokens)."""
    return _FlashPnFirTauFn.apply(q, k_tilde, v, score_tau, scale, gamma, causal_mask, "bnhd")


def _flash_fir_qkv(qkv, H, score_tau, taps, scale, gamma, causal_mask):
    """flash_pn_fir_tau_attention_fir on the column blocks of qkv [B,N,3*H*D];
    the result's storage is [B,N,H,D]; one gradient tensor for qkv."""
    return _FlashFirQkvFn.apply(qkv, H, score_tau, taps, scale, gamma, causal_mask)


def fused_fir_applies(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, fir_k: int) -> bool:
    """Whether flash_pn_fir_tau_attention_fir serves these inputs (7 taps, bf16,
    head dims that are multiples of 16 up to 128, the sm_100a kernels)."""
    return (fir_k == _lib.FIR_FUSED_TAPS and q.is_cuda and q.dtype == torch.bfloat16
            and q.shape[-1] % 16 == 0 and 16 <= q.shape[-1] <= 128 and flash_kernel_path(q, k, v) == "sm100")
