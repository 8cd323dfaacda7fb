"""ctypes view of the C ABI declared in include/concord_b200.h.

The CUDA library `concord_b200/_lib/libconcord_b200.so` is built in-tree by
`concord_b200/build.py`.  Loading fails loudly when it is missing: there is
no CPU fallback for any operation of this package.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
ABI_VERSION = 4   # CONCORD_ABI_VERSION of include/concord_b200.h
LIB_PATH = os.path.join(_HERE, "_lib", "libconcord_b200.so")

# flag bits (packed_b.py:451-458 constexprs)
F_MASS_PRESERVE = 1 << 0
F_APPLY_CHASE = 1 << 1
F_TRACK_REBALANCE = 1 << 2
F_GF_TRUST = 1 << 3
F_GF_CONSOL = 1 << 4
F_COHPRE = 1 << 5
F_FIXED_COH = 1 << 6
F_RATIO_COH = 1 << 7

KIND_ADAMW = 0
KIND_SGD = 1

# fp32 arithmetic of the step (CONCORD_ARITH_*)
ARITH_GPU = 0
ARITH_CR = 1

# kernels behind concord_gemm_fwd/dx/dw (CONCORD_GEMM_*)
GEMM_2SM = 0
GEMM_CUTLASS = 1
# implicit-GEMM convolution operators (CONCORD_CONV_*)
CONV_FPROP = 0
CONV_DGRAD = 1
CONV_WGRAD = 2
PEER_SUM_F32 = 0
PEER_MAX_I32 = 1

ERRORS = {
    -1: "invalid argument",
    -2: "unsupported shape/stride",
    -3: "unsupported alignment",
    -4: "workspace missing or too small",
    -5: "CUDA launch/runtime error",
    -6: "no usable CUDA device",
    -7: "size above the fixed maximum",
    -8: "a cross-GPU wait ran out",
}


class StepParams(ctypes.Structure):
    """Mirror of `concord_step_params` (include/concord_b200.h)."""
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("mantissa_bias", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("alpha", ctypes.c_float),
        ("beta1", ctypes.c_float),
        ("weight_decay", ctypes.c_float),
        ("step_cap", ctypes.c_float),
        ("v_scale", ctypes.c_float),
        ("precond_p", ctypes.c_float),
        ("gf_consol", ctypes.c_float),
        ("drift_cancel_C", ctypes.c_float),
        ("alpha_v_fast", ctypes.c_float),
        ("one_minus_alpha_v_fast", ctypes.c_float),
        ("wd_sv", ctypes.c_float),
        ("wd_sf", ctypes.c_float),
        ("gf_trust_delta_sq", ctypes.c_float),
        ("gate_gain", ctypes.c_float),
        ("chase_floor", ctypes.c_float),
        ("one_minus_chase_floor", ctypes.c_float),
        ("leak_floor", ctypes.c_float),
        ("one_minus_leak_floor", ctypes.c_float),
        ("alpha_gate_gain", ctypes.c_float),
        ("consolidate", ctypes.c_void_p),
        ("ratio_floors", ctypes.c_void_p),
        ("arith", ctypes.c_int32),
    ]


def make_step_params(kind="adamw", mantissa_bias=15, alpha=0.1, beta1=0.0,
                     weight_decay=0.0, step_cap=10.0, v_scale=1.0, precond_p=0.5,
                     gf_consol=0.0, drift_cancel_C=0.0, alpha_v_fast=0.001,
                     wd_sv=0.0, wd_sf=0.0, gf_trust_delta_sq=0.0, gate_gain=1.0,
                     chase_floor=0.9, leak_floor=0.999, mass_preserve=False,
                     apply_chase=True, track_rebalance=True, use_cohpre=False,
                     fixed_coh=True, ratio_coh=False, arith=ARITH_GPU):
    """Build the launch scalars the way the reference's launch computes them.

    Flags follow apply_packed_adamw (packed_b.py:897-899, 943-950): the trust
    region is on iff gf_trust_delta_sq > 0, evaporation iff gf_consol > 0.
    Scalars that the reference combines on the host before they meet a tensor
    (`1.0 - alpha_v_fast`, `1.0 - chase_floor`, `alpha * 1.0 * gate_gain`) are
    combined here in double and rounded once to fp32 by ctypes (used by the
    ARITH_CR model; ARITH_GPU recombines them in fp32 as the compiled
    reference does).
    """
    flags = 0
    if mass_preserve:
        flags |= F_MASS_PRESERVE
    if apply_chase:
        flags |= F_APPLY_CHASE
    if track_rebalance:
        flags |= F_TRACK_REBALANCE
    if gf_trust_delta_sq > 0:
        flags |= F_GF_TRUST
    if gf_consol > 0:
        flags |= F_GF_CONSOL
    if use_cohpre:
        flags |= F_COHPRE
    if fixed_coh:
        flags |= F_FIXED_COH
    if ratio_coh:
        flags |= F_RATIO_COH
    alpha = float(alpha)
    return StepParams(
        kind=KIND_ADAMW if kind == "adamw" else KIND_SGD,
        mantissa_bias=int(mantissa_bias), flags=flags,
        alpha=alpha, beta1=float(beta1), weight_decay=float(weight_decay),
        step_cap=float(step_cap), v_scale=float(v_scale),
        precond_p=float(precond_p), gf_consol=float(gf_consol),
        drift_cancel_C=float(drift_cancel_C), alpha_v_fast=float(alpha_v_fast),
        one_minus_alpha_v_fast=1.0 - float(alpha_v_fast),
        wd_sv=float(wd_sv), wd_sf=float(wd_sf),
        gf_trust_delta_sq=float(gf_trust_delta_sq), gate_gain=float(gate_gain),
        chase_floor=float(chase_floor), one_minus_chase_floor=1.0 - float(chase_floor),
        leak_floor=float(leak_floor), one_minus_leak_floor=1.0 - float(leak_floor),
        alpha_gate_gain=alpha * 1.0 * float(gate_gain),
        arith=int(arith),
    )


class PeerSync(ctypes.Structure):
    """Mirror of `concord_peer_sync` (include/concord_b200.h)."""
    _fields_ = [
        ("flags", ctypes.c_void_p),
        ("peer_flags", ctypes.c_void_p),
        ("state", ctypes.c_void_p),
        ("rank", ctypes.c_int32),
        ("n_ranks", ctypes.c_int32),
        ("timeout_ns", ctypes.c_int64),
    ]


_LIB = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F = ctypes.c_float
# (name, restype, argtypes); device addresses are passed as c_void_p
_SIGS = [
    ("concord_abi_version", ctypes.c_int, []),
    ("concord_last_error", ctypes.c_char_p, []),
    ("concord_salt_bump", ctypes.c_int, [_P, _P]),
    ("concord_vhat_workspace_bytes", ctypes.c_size_t, [_I64, _I64]),
    ("concord_vhat_update", ctypes.c_int,
     [_P, _I64, _I64, _I64, _P, _P, _P, _F, _F, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    ("concord_vhat_noalloc_max_scratch_bytes", ctypes.c_size_t, []),
    ("concord_vhat_update_noalloc", ctypes.c_int,
     [_P, _I64, _I64, _I64, _P, _P, _P, _F, _F, _P, _P, _P, _P]),
    ("concord_vhat_partial", ctypes.c_int,
     [_P, _I64, _I64, _I64, _P, _F, _F, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    ("concord_vhat_finish", ctypes.c_int, [_P, _P, _P, _P, _I64, _F, _F, _P]),
    ("concord_step", ctypes.c_int,
     [ctypes.POINTER(StepParams), _P, _I64, _P, _I64, _P, _I64, _P, _P, _P, _P,
      _P, _P, _P, _P, _I64, _P, _P, _P, _I64, _I64, _I64, _P, _P]),
    ("concord_step_sharded", ctypes.c_int,
     [ctypes.POINTER(StepParams), _P, _I64, _P, _I64, _P, _I64, _P, _P, _P, _P,
      _P, _P, _P, _P, _I64, _P, _P, _P, _I64, _I64, _I64, _P, _P, _I32, _P]),
    ("concord_ipc_handle_bytes", ctypes.c_size_t, []),
    ("concord_peer_alloc", ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    ("concord_peer_free", ctypes.c_int, [_P]),
    ("concord_ipc_export", ctypes.c_int, [_P, _P]),
    ("concord_ipc_open", ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    ("concord_ipc_close", ctypes.c_int, [_P]),
    ("concord_peer_push_rows", ctypes.c_int,
     [_P, _I64, _I64, _I64, _P, ctypes.POINTER(PeerSync), _P]),
    ("concord_peer_reduce_vhat", ctypes.c_int,
     [_P, _P, _I64, _I64, _I64, _P, _P, _F, _F, _P, _P, _P, _P, _P, _P, ctypes.c_size_t,
      ctypes.POINTER(PeerSync), _P]),
    ("concord_peer_allreduce", ctypes.c_int,
     [_P, _P, _I64, _I32, _P, _I64, ctypes.POINTER(PeerSync), _P]),
    ("concord_rebalance_gated_layer_workspace_bytes", ctypes.c_size_t, [_I64, _I64]),
    ("concord_rebalance_gated_layer_layout", ctypes.c_int, [_I64, _I64, _P, _P]),
    ("concord_rebalance_gated", ctypes.c_int,
     [_P, _I32, _I64, _P, _I64, _P, _I64, _I32, _P, _P, _P]),
    ("concord_rebalance_workspace_bytes", ctypes.c_size_t, [_I64, _I64]),
    ("concord_rebalance", ctypes.c_int,
     [_P, _I64, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32,
      _I64, _I64, _I64, _I64, _P, _P, _P, ctypes.c_size_t, _P]),
    ("concord_materialize", ctypes.c_int,
     [_P, _I64, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _P]),
    ("concord_quantize", ctypes.c_int,
     [_P, _I64, _P, _I64, _P, _P, _I64, _I64, _I32, _I32, _I32, _I32, _P]),
    ("concord_coherence", ctypes.c_int, [_P, _I64, _I64, _I64, _F, _P, _P]),
    ("concord_garbage_fraction", ctypes.c_int,
     [_P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I32, _F, _P, _P, _P]),
    ("concord_gemm_workspace_bytes", ctypes.c_size_t, [_I64, _I64, _I64]),
    ("concord_gemm_fwd", ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _P, ctypes.c_size_t, _P]),
    ("concord_gemm_dx", ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _P, ctypes.c_size_t, _P]),
    ("concord_gemm_dw", ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _P, ctypes.c_size_t, _P]),
    ("concord_gemm_dw_vhat_workspace_bytes", ctypes.c_size_t, [_I64, _I64, _I64]),
    ("concord_gemm_dw_vhat", ctypes.c_int,
     [_P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _F, _F, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    ("concord_im2col", ctypes.c_int,
     [_P, _I64, _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I32, _I32, _P, _P]),
    ("concord_col2im", ctypes.c_int,
     [_P, _I64, _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I32, _I32, _P, _P]),
    ("concord_transpose_bf16", ctypes.c_int, [_P, _I64, _I64, _I64, _P, _P]),
    ("concord_gemm2sm", ctypes.c_int, [_P, _I32, _I64, _P, _I32, _I64, _P, _I64, _I64, _I64, _I64, _P]),
    ("concord_gemm2sm_error", ctypes.c_int, [_I32]),
    ("concord_gemm2sm_pairs", ctypes.c_int, []),
    ("concord_gemm_set_impl", ctypes.c_int, [_I32]),
    ("concord_gemm_get_impl", ctypes.c_int, []),
    ("concord_conv_nhwc_workspace_bytes", ctypes.c_size_t, [ctypes.c_int] + [_I64] * 11),
    ("concord_conv_fprop_nhwc", ctypes.c_int, [_P, _P, _P] + [_I64] * 11 + [_P, ctypes.c_size_t, _P]),
    ("concord_conv_dgrad_nhwc", ctypes.c_int, [_P, _P, _P] + [_I64] * 11 + [_P, ctypes.c_size_t, _P]),
    ("concord_conv_wgrad_nhwc", ctypes.c_int, [_P, _P, _P] + [_I64] * 11 + [_P, ctypes.c_size_t, _P]),
]

EXPORTED = [s[0] for s in _SIGS]


def load():
    """Load the CUDA library (raises if it was not built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"concord_b200 CUDA library not built: {LIB_PATH} is missing "
            "(run `python -m concord_b200.build`); there is no CPU fallback")
    lib = ctypes.CDLL(LIB_PATH)
    for name, res, args in _SIGS:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.concord_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{LIB_PATH} has ABI version {lib.concord_abi_version()}, this package "
                           f"needs {ABI_VERSION}: rebuild with `python -m concord_b200.build`")
    _LIB = lib
    return lib


def check(status, what):
    """Map a C status code to RuntimeError (the reference raises on bad input)."""
    if status != 0:
        msg = _LIB.concord_last_error().decode() if _LIB is not None else ""
        raise RuntimeError(f"{what} failed: {ERRORS.get(status, status)}: {msg}")
