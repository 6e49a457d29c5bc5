"""TEST INFRASTRUCTURE ONLY - stages the reference's own Python package for the
reference arm of bench.py.

The reference (mcfax-arch/paper_01_anti_decoy_pnfirtau) is a Python package with
no build step and no packaging metadata (no setup.py / pyproject.toml), so
`pip install --target` cannot install it. This recipe copies its three package
files, src/__init__.py, src/pnfirtau_attention.py and src/triton_pnfirtau.py,
byte for byte into oracle/_ref/src/ (git-ignored: never committed, but carried
to the GPU box with the working tree like the built library). Only the reference
arm of bench.py imports them from there:

* its CPU baseline runs the reference's stock CPU path of the operator
  (triton_pn_fir_tau_scores falls back to the eager power_norm_peak_gate on CPU
  tensors, src/triton_pnfirtau.py:797-811);
* on a GPU it times the reference's own Triton Flash kernels
  (flash_pn_fir_tau_attention, src/triton_pnfirtau.py:971-983) on one B200.

Run with the reference checkout's root as the argument (or in PNFT_REFERENCE_ROOT);
the copy is skipped when that checkout is absent (the GPU box has none).
"""
from __future__ import annotations

import hashlib
import os
import shutil
import sys
from pathlib import Path

FILES = ("__init__.py", "pnfirtau_attention.py", "triton_pnfirtau.py")
DEST = Path(__file__).resolve().parent / "_ref" / "src"
DEFAULT_ROOT = "/root/reference"


def stage(root: str | os.PathLike | None = None) -> Path | None:
    """Copies the reference package into oracle/_ref/src; returns the directory,
    or None when no reference checkout is present."""
    root = Path(root or os.environ.get("PNFT_REFERENCE_ROOT", DEFAULT_ROOT))
    src = root / "src"
    if not all((src / f).is_file() for f in FILES):
        return None
    DEST.mkdir(parents=True, exist_ok=True)
    for f in FILES:
        shutil.copyfile(src / f, DEST / f)
    manifest = "".join(f"{hashlib.sha256((DEST / f).read_bytes()).hexdigest()}  src/{f}\n" for f in FILES)
    (DEST.parent / "MANIFEST.sha256").write_text(manifest)
    return DEST


def staged() -> Path | None:
    """oracle/_ref (the directory to put on sys.path for `import src...`) if staged."""
    return DEST.parent if all((DEST / f).is_file() for f in FILES) else None


if __name__ == "__main__":
    out = stage(sys.argv[1] if len(sys.argv) > 1 else None)
    print(out if out else "reference checkout not found: nothing staged")
