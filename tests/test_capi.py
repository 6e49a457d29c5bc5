"""The C-ABI library loads and exports exactly what include/pnfirtau_b200.h
declares; host-side argument checking and workspace sizing work without a
GPU (no kernel is launched here)."""
import ctypes
import re
from pathlib import Path

import pytest

from paper_01_anti_decoy_pnfirtau_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "pnfirtau_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"PNFT_API\s+[\w\s\*]+?\b(pnft_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "pnft_flash_fwd" in syms and "pnft_flash_bwd" in syms and "pnft_fir_fwd" in syms
    assert len(syms) >= 13


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
        assert ctypes.cast(getattr(L, name), ctypes.c_void_p).value


def test_binding_table_covers_header():
    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_only_api_symbols_are_exported():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == set(declared_symbols())


def test_version_and_last_error():
    L = _lib.lib()
    assert L.pnft_version() >= 100
    assert isinstance(_lib.last_error(), str)


def test_header_constants_match_binding():
    text = HEADER.read_text()
    consts = dict(re.findall(r"#define (PNFT_\w+) \(?(-?\w+)\)?", text))
    assert int(consts["PNFT_DTYPE_F32"]) == _lib.DTYPE_F32
    assert int(consts["PNFT_DTYPE_BF16"]) == _lib.DTYPE_BF16
    assert int(consts["PNFT_DTYPE_F16"]) == _lib.DTYPE_F16
    assert int(consts["PNFT_EINVAL"]) == _lib.EINVAL
    assert int(consts["PNFT_EUNSUPPORTED"]) == _lib.EUNSUPPORTED
    assert int(consts["PNFT_SILENCE_MASS_POW"]) == _lib.SILENCE_MASS_POW
    assert int(consts["PNFT_FLASH_FORCE_GENERIC"], 16) == _lib.FLASH_FORCE_GENERIC


def test_workspace_sizes():
    L = _lib.lib()
    assert L.pnft_flash_bwd_workspace_size(0, 4, 512, 64, 0) == 0
    ws = L.pnft_flash_bwd_workspace_size(16, 4, 512, 64, 0)
    # fp32 dQ accumulator + 16-byte row coefficients + per-tile tau partials
    assert ws >= 16 * 4 * 512 * 64 * 4 + 16 * 4 * 512 * 16 + 16 * 4 * 8 * 4
    assert ws % 256 == 0
    assert L.pnft_fir_bwd_workspace_size(32, 512, 256, 7) > 0
    assert L.pnft_fir_bwd_workspace_size(0, 512, 256, 7) == 0


@pytest.mark.parametrize("ntaps", [0, 65])
def test_fir_rejects_bad_tap_count(ntaps):
    L = _lib.lib()
    rc = L.pnft_fir_fwd(1, 0, 0, 1, 1, ntaps, 1, 0, 0, 1, 1, 8, 8, _lib.DTYPE_F32, None)
    assert rc == _lib.EINVAL
    assert "ntaps" in _lib.last_error()


def test_fir_empty_is_noop():
    L = _lib.lib()
    assert L.pnft_fir_fwd(None, 0, 0, 1, None, 7, None, 0, 0, 1, 0, 8, 8, _lib.DTYPE_F32, None) == _lib.OK


def test_flash_rejects_large_head_dim_and_bad_dtype():
    L = _lib.lib()
    s = _lib.i64x4([1, 1, 1, 1])
    rc = L.pnft_flash_fwd(1, s, 1, s, 1, s, 1, 1, s, None, 1, 1, 1, 1, 1, 1, 8, 256, 1.0, 0.5, 1, 1, _lib.DTYPE_BF16, 0, None, None, None)
    assert rc == _lib.EUNSUPPORTED and "head dim" in _lib.last_error()
    rc = L.pnft_flash_fwd(1, s, 1, s, 1, s, 1, 1, s, None, 1, 1, 1, 1, 1, 1, 8, 64, 1.0, 0.5, 1, 1, 7, 0, None, None, None)
    assert rc == _lib.EINVAL
    rc = L.pnft_flash_fwd(1, s, 1, s, 1, s, 1, 1, s, None, 1, 1, 1, 1, 1, 1, 8, 64, 1.0, -1.0, 1, 1, 1, 0, None, None, None)
    assert rc == _lib.EINVAL and "gamma" in _lib.last_error()


def test_flash_bwd_checks_workspace():
    L = _lib.lib()
    s = _lib.i64x4([1, 1, 1, 1])
    rc = L.pnft_flash_bwd(1, s, 1, s, 1, s, 1, 1, s, None, 1, s, 1, 1, 1, 1, 1, s, 1, s, 1, s, 1, 1, 16, 2, 2, 64, 64, 0.125,
                          0.5, 1, 1, _lib.DTYPE_BF16, 0, None, None)
    assert rc == _lib.EINVAL and "workspace" in _lib.last_error()


def test_rows_rejects_unknown_mode():
    L = _lib.lib()
    rc = L.pnft_rows_fwd(1, 8, 1, 1, 8, 1, 1, 1, 1, 4, 8, 1.0, 10.0, 0.5, 1, 7, 1, _lib.DTYPE_F32, None)
    assert rc == _lib.EINVAL and "silence mode" in _lib.last_error()


def test_fused_fir_entry_points_check_arguments():
    """The fused-FIR entries reject a tap count other than the fused filter's and
    a null tap pointer on the host, before any device work."""
    L = _lib.lib()
    consts = dict(re.findall(r"#define (PNFT_\w+) \(?(-?\w+)\)?", HEADER.read_text()))
    assert int(consts["PNFT_FIR_FUSED_TAPS"]) == _lib.FIR_FUSED_TAPS == 7
    s = _lib.i64x4((1, 1, 1, 1))
    rc = L.pnft_flash_fwd_fir(1, s, 1, s, None, 7, 1, s, 1, 1, s, None, 1, 1, 1, 1, 1, 1, 64, 64, 0.125, 0.5, 1, 1,
                              _lib.DTYPE_BF16, 0, None, None, None)
    assert rc == _lib.EINVAL and "taps" in _lib.last_error()
    rc = L.pnft_flash_bwd_fir(1, s, 1, s, 1, 5, 1, s, 1, 1, s, None, 1, s, 1, 1, 1, 1, 1, s, 1, s, 1, s, 1, None, 1,
                              1 << 30, 1, 1, 64, 64, 0.125, 0.5, 1, 1, _lib.DTYPE_BF16, 0, None, None)
    assert rc == _lib.EUNSUPPORTED and "taps" in _lib.last_error()
    base = L.pnft_flash_bwd_workspace_size(8, 8, 4096, 64, 0)
    fused = L.pnft_flash_bwd_fir_workspace_size(8, 8, 4096, 64, 0)
    assert fused >= base + 8 * 8 * 4096 * 64 * 2 and fused % 256 == 0
    assert L.pnft_flash_bwd_fir_workspace_size(0, 8, 4096, 64, 0) == 0
