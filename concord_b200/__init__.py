"""concord_b200 — B200-native Concord packed-word hot path.

Public API mirrors the reference's `concord` package (concord/__init__.py:7-31).
"""
from .gated import GatedRebalance  # noqa: F401
from .packed_b import (  # noqa: F401
    ConcordLinearPackedB,
    ConcordConv2dPackedB,
    FusedConcordLinearPackedB,
    FusedConcordConv2dPackedB,
    compute_drift_cancel_C,
    set_fixed_coh,
    set_gate_gain,
    set_coh_weighted_v,
    set_ratio_coh,
    set_ratio_coh_floors,
    set_ratio_floor_tensors,
    set_consolidate,
    set_sigmag_noise,
    set_sigmag_sigma,
    set_conv_backend,
    reset_reb_stats,
    get_reb_stats,
    set_arithmetic,
    get_arithmetic,
    gate_coherence_from_fields,
    measure_coherence,
    DissipationAutoTuner,
    apply_packed_adamw,
    apply_packed_sgd,
    materialize_packed_bf16,
    rebalance_packed,
    vhat_update,
    S_SLOW_FACTOR,
    V_SLOW_FACTOR,
    MANTISSA_BIAS,
)

__all__ = [
    "GatedRebalance",
    "ConcordLinearPackedB",
    "ConcordConv2dPackedB",
    "compute_drift_cancel_C",
    "set_fixed_coh",
    "set_gate_gain",
    "reset_reb_stats",
    "get_reb_stats",
    "set_arithmetic",
    "get_arithmetic",
    "set_conv_backend",
    "S_SLOW_FACTOR",
    "V_SLOW_FACTOR",
    "MANTISSA_BIAS",
]
