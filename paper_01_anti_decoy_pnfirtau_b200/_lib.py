"""ctypes binding of libpnfirtau_b200.so (the C ABI in include/pnfirtau_b200.h).

The library is built in-tree by ``_build.build()``. Loading never falls back to
anything else: a missing library, or a CUDA call made with CPU tensors, raises.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpnfirtau_b200.so"

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
OK, EINVAL, EUNSUPPORTED, ECUDA = 0, -1, -2, -3
DEV_OK, DEV_WAIT_TIMEOUT, DEV_BAD_INDEX = 0, 1, 2
SILENCE_PEAK, SILENCE_MASS_RELU, SILENCE_MASS_POW = 0, 1, 2
FLASH_FORCE_GENERIC, FLASH_DETERMINISTIC, FLASH_PREFER_SM100 = 0x1, 0x2, 0x4
FLASH_TEST_STALL = 0x100  # test-only: the tcgen05 kernels take their timeout path
FIR_FUSED_TAPS = 7  # PNFT_FIR_FUSED_TAPS
GELU_TABLE_FLOATS = 10240  # PNFT_GELU_TABLE_FLOATS

_I64x4 = c_int64 * 4
_P = c_void_p

# name -> (restype, argtypes); must mirror include/pnfirtau_b200.h exactly
SIGNATURES: dict[str, tuple] = {
    "pnft_version": (c_int, []),
    "pnft_launch_count": (ctypes.c_uint64, []),
    "pnft_last_error": (ctypes.c_char_p, []),
    "pnft_query_caps": (c_int, [c_int, POINTER(c_int), POINTER(c_int), POINTER(c_int), POINTER(c_int), POINTER(c_int)]),
    "pnft_mapped_status_ptr": (c_int, [_P, POINTER(c_void_p)]),
    "pnft_fir_fwd": (
        c_int,
        [_P, c_int64, c_int64, c_int64, _P, c_int, _P, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, _P],
    ),
    "pnft_fir_bwd": (
        c_int,
        [_P, c_int64, c_int64, c_int64, _P, c_int, _P, c_int64, c_int64, c_int64, _P, c_int64, c_int64, c_int64,
         _P, _P, c_size_t, c_int64, c_int64, c_int64, c_int, _P],
    ),
    "pnft_fir_bwd_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int]),
    "pnft_fir_bwd_noalloc": (
        c_int,
        [_P, c_int64, c_int64, c_int64, _P, c_int, _P, c_int64, c_int64, c_int64, _P, c_int64, c_int64, c_int64,
         _P, c_int64, c_int64, c_int64, c_int, _P],
    ),
    "pnft_rows_fwd": (
        c_int,
        [_P, c_int64, _P, _P, c_int64, _P, _P, _P, _P, c_int64, c_int64, c_float, c_float, c_float, c_int, c_int,
         c_int, c_int, _P],
    ),
    "pnft_rows_bwd": (
        c_int,
        [_P, c_int64, _P, c_int64, _P, _P, _P, _P, _P, _P, c_int64, _P, _P, c_int64, c_int64, c_float, c_float,
         c_float, c_int, c_int, c_int, c_int, _P],
    ),
    "pnft_sum_f32": (c_int, [_P, c_int64, _P, _P]),
    "pnft_flash_fwd": (
        c_int,
        [_P, _I64x4, _P, _I64x4, _P, _I64x4, _P, _P, _I64x4, _P, _P, _P, _P, _P, c_int64, c_int64, c_int64,
         c_int64, c_float, c_float, c_int, c_int, c_int, c_int, _P, _P, _P],
    ),
    "pnft_flash_bwd": (
        c_int,
        [_P, _I64x4, _P, _I64x4, _P, _I64x4, _P, _P, _I64x4, _P, _P, _I64x4, _P, _P, _P, _P, _P, _I64x4, _P, _I64x4, _P,
         _I64x4, _P, _P, c_size_t, c_int64, c_int64, c_int64, c_int64, c_float, c_float, c_int, c_int, c_int,
         c_int, _P, _P],
    ),
    "pnft_flash_bwd_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int]),
    "pnft_flash_fwd_fir": (
        c_int,
        [_P, _I64x4, _P, _I64x4, _P, c_int, _P, _I64x4, _P, _P, _I64x4, _P, _P, _P, _P, _P, c_int64, c_int64,
         c_int64, c_int64, c_float, c_float, c_int, c_int, c_int, c_int, _P, _P, _P],
    ),
    "pnft_flash_bwd_fir": (
        c_int,
        [_P, _I64x4, _P, _I64x4, _P, c_int, _P, _I64x4, _P, _P, _I64x4, _P, _P, _I64x4, _P, _P, _P, _P, _P, _I64x4,
         _P, _I64x4, _P, _I64x4, _P, _P, _P, c_size_t, c_int64, c_int64, c_int64, c_int64, c_float, c_float, c_int,
         c_int, c_int, c_int, _P, _P],
    ),
    "pnft_flash_bwd_fir_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int]),
    "pnft_flash_path": (c_int, [_P, _I64x4, _P, _I64x4, _P, _I64x4, c_int64, c_int, c_int]),
    "pnft_lm_xent": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, c_int64, c_float, _P, _P, _P]),
    "pnft_layernorm_fwd": (
        c_int, [_P, c_int64, _P, _P, c_float, _P, c_int64, _P, _P, c_int64, c_int64, c_int, c_int, _P]),
    "pnft_layernorm_bwd": (
        c_int,
        [_P, c_int64, _P, c_int64, _P, _P, _P, _P, c_int64, _P, _P, _P, c_size_t, c_int64, c_int64, c_int, c_int, _P],
    ),
    "pnft_layernorm_bwd_workspace_size": (c_size_t, [c_int64, c_int64]),
    "pnft_add_layernorm_fwd": (
        c_int,
        [_P, c_int64, _P, c_int64, c_int, _P, c_int64, _P, _P, c_float, _P, c_int64, _P, _P, c_int64, c_int64, c_int,
         c_int, _P],
    ),
    "pnft_add_layernorm_bwd": (
        c_int,
        [_P, c_int64, _P, c_int64, _P, c_int64, _P, _P, _P, _P, c_int64, _P, c_int64, c_int, _P, _P, _P, c_size_t,
         c_int64, c_int64, c_int, c_int, _P],
    ),
    "pnft_colsum": (c_int, [_P, c_int64, _P, _P, c_size_t, c_int64, c_int64, c_int, _P]),
    "pnft_colsum_workspace_size": (c_size_t, [c_int64, c_int64]),
    "pnft_gelu_table": (c_int, [_P, _P]),
    "pnft_gemm_at_b": (
        c_int, [_P, c_int64, _P, c_int64, _P, c_int64, _P, c_size_t, c_int64, c_int64, c_int64, c_int, _P, _P]),
    "pnft_gemm_at_b_workspace_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "pnft_gelu_fwd": (c_int, [_P, c_int64, _P, c_int64, c_int64, c_int64, c_int, _P, _P]),
    "pnft_cast_bf16": (c_int, [_P, c_int, c_int64, _P]),
    "pnft_gelu_bwd_colsum": (
        c_int, [_P, c_int64, _P, c_int64, _P, c_int64, _P, _P, c_size_t, c_int64, c_int64, c_int, _P, _P]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once per process)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH.name} is not built; run `python -m paper_01_anti_decoy_pnfirtau_b200._build` "
                        "(nvcc for sm_100a) before using the CUDA operators"
                    )
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().pnft_last_error()
    return msg.decode() if msg else ""


def launch_count() -> int:
    """Kernels launched by the library so far in this process."""
    return int(lib().pnft_launch_count())


def check(rc: int, what: str) -> None:
    if rc != OK:
        kind = {EINVAL: "invalid argument", EUNSUPPORTED: "unsupported", ECUDA: "CUDA error"}.get(rc, f"status {rc}")
        raise RuntimeError(f"{what} failed ({kind}): {last_error()}")


def i64x4(seq) -> "ctypes.Array":
    return _I64x4(*[int(s) for s in seq])
