"""B200-native pn_fir_tau attention: hand-written sm_100a CUDA behind the
reference's Python API (mcfax-arch/paper_01_anti_decoy_pnfirtau, ``src/``).

Exports the reference's eager names (src/__init__.py) plus the fused-op
entry points of src/triton_pnfirtau.py.
"""
from .lm_ops import LayerNorm, head_cross_entropy, layer_norm
from .pnfirtau_attention import (
    PnFirConfig,
    PnFirTauFlashMHA,
    PnFirTauMHA,
    PnFirTauTritonMHA,
    SmFirMHA,
    causal_fir,
    causal_gaussian_taps,
    power_norm_peak_gate,
)
from .pnfirtau_ops import (
    check_device_status,
    flash_kernel_path,
    flash_pn_fir_tau_attention,
    flash_pn_fir_tau_attention_fir,
    pn_rows,
    triton_causal_fir,
    triton_pn_fir_tau_scores,
)
from .sharding import (
    TauGradReducer,
    bh_range,
    shard_bh,
    share_tau,
    sharded_flash_pn_fir_tau_attention,
    unshard_bh,
)

__all__ = [
    "PnFirConfig",
    "PnFirTauMHA",
    "PnFirTauTritonMHA",
    "PnFirTauFlashMHA",
    "SmFirMHA",
    "causal_fir",
    "causal_gaussian_taps",
    "power_norm_peak_gate",
    "triton_causal_fir",
    "triton_pn_fir_tau_scores",
    "flash_pn_fir_tau_attention",
    "flash_pn_fir_tau_attention_fir",
    "pn_rows",
    "check_device_status",
    "flash_kernel_path",
    "bh_range",
    "shard_bh",
    "unshard_bh",
    "share_tau",
    "sharded_flash_pn_fir_tau_attention",
    "TauGradReducer",
    "LayerNorm",
    "layer_norm",
    "head_cross_entropy",
]
