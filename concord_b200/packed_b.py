"""ConcordLinearPackedB on B200: the reference's layer API over hand-written CUDA.

Drop-in for `concord.packed_b` (Theophite/Concord concord/packed_b.py): same
constants, module-level flags and setters, functional launchers
(`apply_packed_adamw`, `apply_packed_sgd`, `materialize_packed_bf16`,
`rebalance_packed`), autograd Functions and `nn.Module`s with the same
attribute and buffer names (so `state_dict()` keys match).  Every tensor
operation on the packed state runs in `concord_b200/_lib/libconcord_b200.so`
through its C ABI (include/concord_b200.h); the module raises if that
library is missing or a tensor is not on a CUDA device.  The dense GEMMs of
forward / dX / dW run through `concord_b200.gemm`.
"""
import ctypes
from types import SimpleNamespace

import numpy as np
import torch
import torch.nn as nn

from . import _abi
from . import gemm as _gemm

MANTISSA_BIAS = 15
INT8_MIN, INT8_MAX = -128, 127
INT16_MIN, INT16_MAX = -32768, 32767
S_SLOW_FACTOR = 128
V_SLOW_FACTOR = 128


def compute_drift_cancel_C(alpha, alpha_v_fast, alpha_v_slow=0.0, refit_period=1,
                           mass_preserve=True):
    """Drift-cancellation coefficient C* (packed_b.py:52-102).

    L = (1-alpha)/alpha, rho = alpha_v_fast + alpha_v_slow/T_r.  With the
    mass-preserving leak the telescope relaxes at 2*rho per step, giving
    C* = L*2rho/(1-2rho); otherwise the legacy C* = L*rho/(1-L*alpha_v_fast).
    """
    L = (1.0 - alpha) / max(alpha, 1e-12)
    rho = alpha_v_fast + alpha_v_slow / max(refit_period, 1)
    if mass_preserve:
        rho2 = 2.0 * rho
        return L * rho2 / (1.0 - rho2)
    return L * rho / (1.0 - L * alpha_v_fast)


# ---- module-level switches (packed_b.py:797-860), read at launch time ----
_USE_FIXED_COH = True
_GATE_GAIN = 1.0
_COH_WEIGHTED_V = False
_RATIO_COH = False
_RATIO_CHASE_FLOOR = 0.9
_RATIO_LEAK_FLOOR = 0.999


def set_fixed_coh(enabled):
    global _USE_FIXED_COH
    _USE_FIXED_COH = bool(enabled)


def set_gate_gain(g):
    global _GATE_GAIN
    _GATE_GAIN = float(g)


def set_coh_weighted_v(enabled):
    """Experimental coh_pre-weighted v-hat accumulation (packed_b.py:815-833)."""
    global _COH_WEIGHTED_V
    _COH_WEIGHTED_V = bool(enabled)


def set_ratio_coh(enabled):
    global _RATIO_COH
    _RATIO_COH = bool(enabled)


def set_ratio_coh_floors(chase, leak):
    global _RATIO_CHASE_FLOOR, _RATIO_LEAK_FLOOR
    _RATIO_CHASE_FLOOR = float(chase)
    _RATIO_LEAK_FLOOR = float(leak)
    for t in _FLOOR_TENSORS.values():   # device copies, read by captured graphs
        t[0] = _RATIO_CHASE_FLOOR
        t[1] = _RATIO_LEAK_FLOOR


# fp32 arithmetic of the packed step: "gpu" reproduces the reference as it
# runs compiled on NVIDIA GPUs (ex2.approx, CUDA log2f, div.full, its fma
# contractions), "cr" the correctly rounded model that the CPU oracle restates.
_ARITH = _abi.ARITH_GPU


def set_arithmetic(mode):
    """Select the step's fp32 arithmetic: "gpu" (default) or "cr".  Read at
    every launch; a captured CUDA graph keeps the mode it was captured with."""
    global _ARITH
    modes = {"gpu": _abi.ARITH_GPU, "cr": _abi.ARITH_CR}
    if mode not in modes:
        raise ValueError(f"arithmetic must be one of {sorted(modes)}, got {mode!r}")
    _ARITH = modes[mode]


def get_arithmetic():
    return "gpu" if _ARITH == _abi.ARITH_GPU else "cr"


_REB_STATS = None      # host-side counts while instrumentation is on
_REB_COUNTERS = {}     # device -> int64[3] counters the rebalance kernels add to


def reset_reb_stats():
    """Start (or restart) the rebalance instrumentation (packed_b.py:1100-1106).

    Tick counts and clipped words are counted on the GPU by the rebalance
    launch itself; nothing synchronises until get_reb_stats() reads them."""
    global _REB_STATS
    _REB_STATS = dict(calls=0, dim_total=0, elem_total=0)
    for t in _REB_COUNTERS.values():
        t.zero_()


def _reb_counters(device):
    key = str(device)
    if key not in _REB_COUNTERS:
        _REB_COUNTERS[key] = torch.zeros(3, dtype=torch.int64, device=device)
    return _REB_COUNTERS[key]


def get_reb_stats():
    """The reference's rebalance statistics: calls, rows+columns ticked up and
    down, their total, words clipped by a tick-down shift and the words seen
    (None until reset_reb_stats())."""
    if _REB_STATS is None:
        return None
    dev = [0, 0, 0]
    for t in _REB_COUNTERS.values():
        dev = [a + int(b) for a, b in zip(dev, t.tolist())]
    return dict(calls=_REB_STATS["calls"], tickup_dim=dev[0], tickdown_dim=dev[1],
                dim_total=_REB_STATS["dim_total"], clip_elems=dev[2],
                elem_total=_REB_STATS["elem_total"])


# ---- device scalars (packed_b.py:315-359) ----
_STEP_COUNTERS = {}
_LR_SCALAR_CACHE = {}
_EPS_SCALAR_CACHE = {}
_REB_SEED_CACHE = {}


def _dev_key(device):
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return str(device)


def _get_step_counter(device):
    """Per-device int32 step salt, bumped before every step launch (all layers share it)."""
    key = _dev_key(device)
    if key not in _STEP_COUNTERS:
        _STEP_COUNTERS[key] = torch.zeros(1, dtype=torch.int32, device=device)
    return _STEP_COUNTERS[key]


def _scalar_buf(cache, value, device):
    if isinstance(value, torch.Tensor):
        return value
    key = _dev_key(device)
    buf = cache.get(key)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.float32, device=device)
        cache[key] = buf
    buf.fill_(float(value))
    return buf


def _ensure_lr_tensor(lr, device):
    return _scalar_buf(_LR_SCALAR_CACHE, lr, device)


def _ensure_eps_tensor(eps, device):
    return _scalar_buf(_EPS_SCALAR_CACHE, eps, device)


def _ensure_reb_seed_tensor(device):
    key = _dev_key(device)
    buf = _REB_SEED_CACHE.get(key)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=device)
        _REB_SEED_CACHE[key] = buf
    return buf


# ---- C-ABI plumbing ----
def _lib():
    return _abi.load()


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("concord_b200 runs on CUDA tensors only (no CPU fallback); "
                               f"got a tensor on {t.device}")


_WORKSPACES = {}


def _workspace(kind, nbytes, device):
    """Zero-initialised scratch shared per (kind, device, current stream);
    grown on demand.

    The kernels leave their counters at zero after every launch, so one
    buffer serves every layer launched on a stream (launches on one stream are
    ordered).  Layers stepped on different streams get different buffers, so
    they neither race on the counters nor free a buffer another stream still
    reads (a replaced buffer was only ever used on this stream, and the
    caching allocator reuses its memory in that stream's order).
    """
    key = (kind, _dev_key(device), torch.cuda.current_stream(device).cuda_stream)
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = buf
    return buf


def materialize_packed_bf16(packed_w, row_exp, col_exp, out, mantissa_bias=15,
                            consolidated=False):
    """bf16 weight from the packed words (packed_b.py:158-170); `consolidated`
    drops s_fast as consolidated_weight() does (1632-1649)."""
    N, K = packed_w.shape
    assert packed_w.dtype == torch.int32
    assert out.dtype == torch.bfloat16 and out.shape == packed_w.shape
    _need_cuda(packed_w, row_exp, col_exp, out)
    lib = _lib()
    _abi.check(lib.concord_materialize(
        _ptr(packed_w), packed_w.stride(0), _ptr(row_exp), _ptr(col_exp), _ptr(out), out.stride(0),
        N, K, int(mantissa_bias), int(bool(consolidated)), _stream(packed_w.device)),
        "concord_materialize")
    return out


def _step_launch(params, packed_w, grad_W, weight_buf, row_exp, col_exp, row_max, col_max,
                 v_row, v_col, sum_v_inv, coh_pre, lr_t, eps_t, salt, row0=0, coh_stats=None,
                 wbuf_peers=None):
    """One concord_step launch; with `wbuf_peers` (int64 device tensor of other
    ranks' forward-weight base addresses) the step also stores every bf16
    weight it writes into those buffers (concord_step_sharded)."""
    N, K = packed_w.shape
    assert packed_w.stride(1) == 1 and grad_W.stride(1) == 1 and weight_buf.stride(1) == 1
    _need_cuda(packed_w, grad_W, weight_buf, row_exp, col_exp, row_max, col_max, v_row, v_col,
               sum_v_inv, coh_pre, lr_t, eps_t, salt)
    lib = _lib()
    args = (ctypes.byref(params), _ptr(packed_w), packed_w.stride(0), _ptr(grad_W), grad_W.stride(0),
            _ptr(weight_buf), weight_buf.stride(0), _ptr(row_exp), _ptr(col_exp), _ptr(row_max),
            _ptr(col_max), _ptr(v_row), _ptr(v_col), _ptr(sum_v_inv), _ptr(coh_pre),
            coh_pre.stride(0) if coh_pre is not None else K, _ptr(lr_t), _ptr(eps_t), _ptr(salt),
            N, K, int(row0), _ptr(coh_stats))
    if wbuf_peers is not None and wbuf_peers.numel() > 0:
        _abi.check(lib.concord_step_sharded(*args, _ptr(wbuf_peers), int(wbuf_peers.numel()),
                                            _stream(packed_w.device)), "concord_step_sharded")
    else:
        _abi.check(lib.concord_step(*args, _stream(packed_w.device)), "concord_step")


def _salt_bump(salt):
    _abi.check(_lib().concord_salt_bump(_ptr(salt), _stream(salt.device)), "concord_salt_bump")


def adamw_params(alpha=0.1, beta1=0.0, weight_decay=0.0, step_cap=10.0, v_scale=1.0,
                 precond_p=0.5, gf_consol=0.0, drift_cancel_C=None, alpha_v_fast=0.001,
                 wd_sv=0.0, wd_sf=0.0, mass_preserve=False, apply_chase=True,
                 track_rebalance=True, gf_trust_delta_sq=0.0, use_cohpre=False,
                 mantissa_bias=15, device=None):
    """Launch scalars of the AdamW path with the module switches read now.
    With `device`, the device scalars in use on it are attached: the
    gradient-accumulation flag once set_consolidate() has been called there,
    the ratio-floor tensors once set_ratio_floor_tensors(True)."""
    if drift_cancel_C is None:
        drift_cancel_C = compute_drift_cancel_C(alpha, alpha_v_fast, mass_preserve=mass_preserve)
    p = _abi.make_step_params(
        kind="adamw", mantissa_bias=mantissa_bias, alpha=alpha, beta1=beta1,
        weight_decay=weight_decay, step_cap=step_cap, v_scale=v_scale, precond_p=precond_p,
        gf_consol=gf_consol, drift_cancel_C=drift_cancel_C, alpha_v_fast=alpha_v_fast,
        wd_sv=wd_sv, wd_sf=wd_sf, gf_trust_delta_sq=gf_trust_delta_sq, gate_gain=_GATE_GAIN,
        chase_floor=_RATIO_CHASE_FLOOR, leak_floor=_RATIO_LEAK_FLOOR,
        mass_preserve=mass_preserve, apply_chase=apply_chase, track_rebalance=track_rebalance,
        use_cohpre=use_cohpre, fixed_coh=_USE_FIXED_COH, ratio_coh=_RATIO_COH, arith=_ARITH)
    if device is not None:
        key = _dev_key(device)
        if key in _CONSOLIDATE_FLAGS:
            p.consolidate = _CONSOLIDATE_FLAGS[key].data_ptr()
        if _FLOOR_TENSORS_ON:
            p.ratio_floors = _ensure_floor_tensors(device).data_ptr()
    return p


# ---- centered Sigma_g-shaped gradient noise (prototype_packed_b.py:881-915, 1477-1501) ----
# EXPERIMENTAL in the reference and off by default: adds a draw shaped like the
# per-token gradient covariance, mean-subtracted,
#   noise = sum_i eps_i (g_i - gbar) = (eps * grad_y)^T x - (sum eps) gbar,  eps ~ N(0, 1),
# scaled to sigma * ||grad_W|| (isotropic white noise of the same norm as an
# ablation).  sigma is a device scalar, so a captured graph follows its schedule.
_SIGMAG_NOISE = False
_SIGMAG_ISO = False
_SIGMAG_SIGMA = 0.0
_SIGMAG_TENSORS = {}


def set_sigmag_noise(enabled, isotropic=False):
    global _SIGMAG_NOISE, _SIGMAG_ISO
    _SIGMAG_NOISE = bool(enabled)
    _SIGMAG_ISO = bool(isotropic)


def set_sigmag_sigma(sigma):
    global _SIGMAG_SIGMA
    _SIGMAG_SIGMA = float(sigma)
    for t in _SIGMAG_TENSORS.values():
        t.fill_(_SIGMAG_SIGMA)


# ConcordConv2dPackedB convolution backend:
#   "implicit": implicit-GEMM convolutions on channels-last tensors (no column
#               matrix; channel counts multiples of 8, stride 1), else "gemm"
#   "gemm":     this package's im2col / col2im + tcgen05 GEMMs (GEMM extents
#               multiples of 8), else cuDNN
#   "cudnn":    torch's conv2d and its grad functions (the reference's route)
_CONV_BACKEND = "implicit"


def set_conv_backend(name):
    """Choose how ConcordConv2dPackedB runs its convolutions ("implicit",
    "gemm" or "cudnn").  The packed step is this package's kernels either way."""
    global _CONV_BACKEND
    if name not in ("implicit", "gemm", "cudnn"):
        raise ValueError(f"conv backend must be 'implicit', 'gemm' or 'cudnn', not {name!r}")
    _CONV_BACKEND = name


def get_conv_backend():
    return _CONV_BACKEND


def _get_sigmag_sigma(device):
    key = _dev_key(device)
    if key not in _SIGMAG_TENSORS:
        _SIGMAG_TENSORS[key] = torch.full((1,), _SIGMAG_SIGMA, dtype=torch.float32, device=device)
    return _SIGMAG_TENSORS[key]


@torch.no_grad()
def sigmag_noise(grad_W, grad_y_flat, x_flat):
    """grad_W plus the centered Sigma_g-shaped noise (torch ops, in the
    reference's order); returns bf16."""
    gwf = grad_W.float()
    if _SIGMAG_ISO:
        noise = torch.randn_like(gwf)
    else:
        gyf = grad_y_flat.float()
        M = gyf.shape[0]
        e = torch.randn(M, device=gyf.device, dtype=torch.float32)
        gbar = gwf / max(M, 1)
        noise = (e[:, None] * gyf).transpose(0, 1) @ x_flat.float() - e.sum() * gbar
    sig_t = _get_sigmag_sigma(gwf.device)
    nrm = noise.norm().clamp_min(1e-12)
    return (gwf + noise * (sig_t * gwf.norm() / nrm)).to(torch.bfloat16).contiguous()


# ---- gradient accumulation and device-tensor schedules (prototype_packed_b.py:325-353, 1000-1010) ----
_CONSOLIDATE_FLAGS = {}
_FLOOR_TENSORS = {}
_FLOOR_TENSORS_ON = False


def _get_consolidate_flag(device):
    key = _dev_key(device)
    if key not in _CONSOLIDATE_FLAGS:
        _CONSOLIDATE_FLAGS[key] = torch.ones(1, dtype=torch.int32, device=device)
    return _CONSOLIDATE_FLAGS[key]


def set_consolidate(device, consolidate: bool):
    """Trainer hook for gradient accumulation: with False the next backward(s)
    only SR-tick this micro-batch's gradient into s_fast (weight, slow
    accumulators and rebalance maxima stay frozen); with True the step
    consolidates as usual.  In a cycle of N micro-steps call False for the
    first N-1 and True for the last.  An in-place fill of a device flag, so a
    captured CUDA graph follows it.  The first call routes this device's AdamW
    steps through the kernel variant that reads the flag."""
    _get_consolidate_flag(device).fill_(1 if consolidate else 0)


def _ensure_floor_tensors(device):
    key = _dev_key(device)
    if key not in _FLOOR_TENSORS:
        _FLOOR_TENSORS[key] = torch.tensor([_RATIO_CHASE_FLOOR, _RATIO_LEAK_FLOOR], dtype=torch.float32,
                                           device=device)
    return _FLOOR_TENSORS[key]


def set_ratio_floor_tensors(enabled):
    """Read the ratio-coherence floors from device tensors (so a per-step
    schedule set with set_ratio_coh_floors reaches a captured CUDA graph), as
    the reference's prototype kernel does; 1 - floor is then computed in fp32
    in the kernel, not in double on the host."""
    global _FLOOR_TENSORS_ON
    _FLOOR_TENSORS_ON = bool(enabled)


def apply_packed_adamw(packed_w, grad_W, weight_buf, row_exp, col_exp, row_max, col_max,
                       lr, mantissa_bias=15, alpha=0.1, beta1=0.0, weight_decay=0.0, eps=1.0,
                       step_cap=10.0, v_scale=1.0, precond_p=0.5, gf_consol=0.0,
                       drift_cancel_C=None, alpha_v_fast=0.001, wd_sv=0.0, wd_sf=0.0,
                       mass_preserve=False, apply_chase=True, track_rebalance=True,
                       v_row=None, v_col=None, sum_v_inv=None, gf_trust_delta_sq=0.0,
                       coh_pre=None, bump_salt=True, row0=0, coh_stats=None):
    """The AdamW three-accumulator packed step (packed_b.py:863-951).

    Same arguments and defaults as the reference.  Bumps the per-device step
    salt first (unless `bump_salt=False`, used when a preceding v-hat launch
    already bumped it), then runs the fused CUDA step in place.
    """
    N, K = packed_w.shape
    assert packed_w.dtype == torch.int32
    assert grad_W.dtype == torch.bfloat16
    assert weight_buf.dtype == torch.bfloat16
    assert weight_buf.shape == packed_w.shape
    use_cohpre = coh_pre is not None
    if gf_trust_delta_sq > 0 or gf_consol > 0 or use_cohpre or _RATIO_COH:
        assert v_row is not None and v_col is not None and sum_v_inv is not None, \
            "gf_trust/gf_consol/coh_pre require v_row, v_col, sum_v_inv"
    params = adamw_params(alpha=alpha, beta1=beta1, weight_decay=weight_decay, step_cap=step_cap,
                          v_scale=v_scale, precond_p=precond_p, gf_consol=gf_consol,
                          drift_cancel_C=drift_cancel_C, alpha_v_fast=alpha_v_fast, wd_sv=wd_sv,
                          wd_sf=wd_sf, mass_preserve=mass_preserve, apply_chase=apply_chase,
                          track_rebalance=track_rebalance, gf_trust_delta_sq=gf_trust_delta_sq,
                          use_cohpre=use_cohpre, mantissa_bias=mantissa_bias, device=packed_w.device)
    salt = _get_step_counter(packed_w.device)
    if bump_salt:
        _salt_bump(salt)
    lr_t = _ensure_lr_tensor(lr, packed_w.device)
    eps_t = _ensure_eps_tensor(eps, packed_w.device)
    _step_launch(params, packed_w, grad_W, weight_buf, row_exp, col_exp, row_max, col_max,
                 v_row, v_col, sum_v_inv, coh_pre, lr_t, eps_t, salt, row0=row0,
                 coh_stats=coh_stats)


def apply_packed_sgd(packed_w, grad_W, weight_buf, row_exp, col_exp, row_max, col_max, lr,
                     mantissa_bias=15, alpha=0.1, beta1=0.0, alpha_v_fast=0.001,
                     mass_preserve=False, track_rebalance=True, bump_salt=True, row0=0):
    """The legacy SGD chase step (packed_b.py:362-394)."""
    assert packed_w.dtype == torch.int32
    assert grad_W.dtype == torch.bfloat16
    assert weight_buf.dtype == torch.bfloat16
    assert weight_buf.shape == packed_w.shape
    params = _abi.make_step_params(kind="sgd", mantissa_bias=mantissa_bias, alpha=alpha,
                                   beta1=beta1, alpha_v_fast=alpha_v_fast,
                                   mass_preserve=mass_preserve, track_rebalance=track_rebalance,
                                   arith=_ARITH)
    salt = _get_step_counter(packed_w.device)
    if bump_salt:
        _salt_bump(salt)
    lr_t = _ensure_lr_tensor(lr, packed_w.device)
    _step_launch(params, packed_w, grad_W, weight_buf, row_exp, col_exp, row_max, col_max,
                 None, None, None, None, lr_t, None, salt, row0=row0)


def vhat_update(grad_W, v_row, v_col, sum_v_inv, beta2=0.999, row_max=None, col_max=None,
                bump_salt=False):
    """Adafactor EMA of the row/col sums of g^2 and 1/sum(v_row) (packed_b.py:1288-1303),
    in one deterministic launch; optionally zeroes row_max/col_max and bumps the salt."""
    N, K = grad_W.shape
    assert grad_W.dtype == torch.bfloat16 and grad_W.stride(1) == 1
    _need_cuda(grad_W, v_row, v_col, sum_v_inv)
    lib = _lib()
    nbytes = lib.concord_vhat_workspace_bytes(N, K)
    ws = _workspace("vhat", nbytes, grad_W.device)
    salt = _get_step_counter(grad_W.device) if bump_salt else None
    _abi.check(lib.concord_vhat_update(
        _ptr(grad_W), grad_W.stride(0), N, K, _ptr(v_row), _ptr(v_col), _ptr(sum_v_inv),
        float(beta2), 1.0 - float(beta2), _ptr(row_max), _ptr(col_max), _ptr(salt), _ptr(ws),
        ws.numel(), _stream(grad_W.device)), "concord_vhat_update")


# The layer backward's dW GEMM computes the v-hat partials in its epilogue
# (concord_gemm_dw_vhat) instead of re-reading dW in a separate v-hat launch.
_FUSED_DW_VHAT = True


def set_fused_dw_vhat(enabled):
    """Whether the layer backward uses concord_gemm_dw_vhat (dW GEMM with the
    v-hat partials in its epilogue; default) or the dW GEMM followed by the
    standalone v-hat launch.  The stored dW is identical either way; v-hat
    agrees to fp32 rounding (the in-tile summation order differs)."""
    global _FUSED_DW_VHAT
    _FUSED_DW_VHAT = bool(enabled)


def dw_vhat_update(grad_y_flat, x_flat, v_row, v_col, sum_v_inv, beta2=0.999, row_max=None,
                   col_max=None, bump_salt=False):
    """dW = dY^T X (bf16, [N, K]) and the v-hat update of vhat_update on it,
    through concord_gemm_dw_vhat; returns dW."""
    M, N = grad_y_flat.shape
    K = x_flat.shape[1]
    _need_cuda(grad_y_flat, x_flat, v_row, v_col, sum_v_inv)
    lib = _lib()
    dy = grad_y_flat.contiguous()
    x = x_flat.contiguous()
    dw = torch.empty(N, K, dtype=torch.bfloat16, device=x.device)
    ws = _workspace("dw_vhat", lib.concord_gemm_dw_vhat_workspace_bytes(M, N, K), x.device)
    salt = _get_step_counter(x.device) if bump_salt else None
    _abi.check(lib.concord_gemm_dw_vhat(
        _ptr(dy), _ptr(x), _ptr(dw), M, N, K, _ptr(v_row), _ptr(v_col), _ptr(sum_v_inv),
        float(beta2), 1.0 - float(beta2), _ptr(row_max), _ptr(col_max), _ptr(salt), _ptr(ws),
        ws.numel(), _stream(x.device)), "concord_gemm_dw_vhat")
    return dw


def _fused_dw_vhat_ok(ctx, grad_y_flat, x_flat):
    """The backward may take the dW-with-v-hat path: the plain single-GPU
    AdamW-family step with v-hat tracking, on bf16 CUDA operands whose
    extents the GEMMs take (multiples of 8), on a layer large enough for the
    epilogue form."""
    if not _FUSED_DW_VHAT or _SIGMAG_NOISE or _sharded_of(ctx.packed_w) is not None:
        return False
    if not (ctx.track_adafactor_v and ctx.v_row is not None):
        return False
    if _COH_WEIGHTED_V and ctx.coh_pre is not None:
        return False
    M, N = grad_y_flat.shape
    K = x_flat.shape[1]
    # the epilogue form needs >= 148 output tiles of 128 x 256 (smaller layers
    # keep the two-launch path here, as concord_gemm_dw_vhat itself would)
    tiles = ((N + 127) // 128) * ((K + 255) // 256)
    return (grad_y_flat.is_cuda and grad_y_flat.dtype == torch.bfloat16 and x_flat.dtype == torch.bfloat16
            and M > 0 and M % 8 == 0 and N % 8 == 0 and K % 8 == 0 and tiles >= 148)


def rebalance_packed(packed_w, row_exp, col_exp, row_max, col_max, MAX_M=24000, EXP_MAX=7,
                     EXP_MIN=-8, seed_buf=None, allow_tickdown=False, row_hwm=None, col_hwm=None,
                     fired_out=None, bump_seed=False, row0=0, n_total=None):
    """Rebalance ratchet (packed_b.py:1129-1190).

    As in the reference, the caller bumps `seed_buf` before the call unless
    `bump_seed=True` asks the kernel to do it (what ConcordLinearPackedB.rebalance
    uses, together with the high-watermark fold).
    """
    if seed_buf is None:
        seed_buf = _ensure_reb_seed_tensor(packed_w.device)
    N, K = packed_w.shape
    _need_cuda(packed_w, row_exp, col_exp, row_max, col_max, seed_buf)
    if not bump_seed:
        seed_buf.sub_(1)   # the kernel adds it back: the launch sees the caller's value
    stats = None
    if _REB_STATS is not None:
        stats = _reb_counters(packed_w.device)
        _REB_STATS["calls"] += 1
        _REB_STATS["dim_total"] += N + K
        _REB_STATS["elem_total"] += N * K
    lib = _lib()
    nbytes = lib.concord_rebalance_workspace_bytes(N, K)
    ws = _workspace("rebalance", nbytes, packed_w.device)
    _abi.check(lib.concord_rebalance(
        _ptr(packed_w), packed_w.stride(0), _ptr(row_exp), _ptr(col_exp), _ptr(row_max),
        _ptr(col_max), _ptr(row_hwm), _ptr(col_hwm), _ptr(seed_buf), int(MAX_M), int(EXP_MAX),
        int(EXP_MIN), int(bool(allow_tickdown)), N, K, int(row0),
        int(N if n_total is None else n_total), _ptr(fired_out), _ptr(stats), _ptr(ws), ws.numel(),
        _stream(packed_w.device)), "concord_rebalance")


# ============================================================
# Autograd Function + nn.Module (packed_b.py:1197-1856)
# ============================================================

# Data-parallel layers: packed_w.data_ptr() -> the RowShardedStep that owns the
# layer's optimizer half (concord_b200.distributed registers it).  The
# autograd backward and rebalance() of a registered layer go through it, so
# `loss.backward()` trains data-parallel with no extra calls and a layer is
# never stepped twice (once on its local dW and once sharded).
_SHARDED = {}


def _sharded_of(packed_w):
    return _SHARDED.get(packed_w.data_ptr()) if _SHARDED else None


def _optimizer_half(ctx, grad_W, step_events=None, vhat_done=False):
    """The backward's optimizer half: this rank's row shard of the sharded
    step when the layer is data-parallel, else the single-GPU step."""
    dp = _sharded_of(ctx.packed_w)
    if dp is not None:
        dp.step(grad_W)
    else:
        _packed_backward_step(ctx, grad_W, step_events, vhat_done)


def _packed_backward_step(ctx, grad_W, step_events=None, vhat_done=False):
    """The optimizer half of the backward (packed_b.py:1278-1337).

    One launch updates v_row/v_col/sum_v_inv (and zeroes the row/col max
    buffers, bumps the salt) unless `vhat_done` (the dW GEMM did it); one
    launch runs the fused packed step.
    `step_events` (optional [_, start, end] CUDA events) bracket the step launch.
    """
    track = bool(ctx.track_rebalance)
    rmax = ctx.row_max_buf if track else None
    cmax = ctx.col_max_buf if track else None
    salt = _get_step_counter(grad_W.device)
    if vhat_done:
        pass
    elif ctx.track_adafactor_v and ctx.v_row is not None:
        if _COH_WEIGHTED_V and ctx.coh_pre is not None:
            raise NotImplementedError("set_coh_weighted_v(True) is not supported by concord_b200")
        vhat_update(grad_W, ctx.v_row, ctx.v_col, ctx.sum_v_inv, ctx.adafactor_beta2,
                    row_max=rmax, col_max=cmax, bump_salt=True)
    else:
        if track:
            rmax.zero_()
            cmax.zero_()
        _salt_bump(salt)
    if step_events is not None:
        step_events[1].record()
    if ctx.optimizer_kind == 'adamw':
        apply_packed_adamw(
            ctx.packed_w, grad_W, ctx.weight_buf, ctx.row_exp, ctx.col_exp,
            ctx.row_max_buf, ctx.col_max_buf, lr=ctx.lr, mantissa_bias=ctx.mantissa_bias,
            alpha=ctx.alpha, beta1=ctx.beta1, weight_decay=ctx.weight_decay, eps=ctx.eps,
            step_cap=ctx.step_cap, v_scale=ctx.v_scale, precond_p=ctx.precond_p,
            gf_consol=ctx.gf_consol, drift_cancel_C=ctx.drift_cancel_C,
            alpha_v_fast=ctx.alpha_v_fast, wd_sv=ctx.wd_sv, wd_sf=ctx.wd_sf,
            mass_preserve=ctx.mass_preserve, apply_chase=ctx.apply_chase,
            track_rebalance=ctx.track_rebalance, v_row=ctx.v_row, v_col=ctx.v_col,
            sum_v_inv=ctx.sum_v_inv, gf_trust_delta_sq=ctx.gf_trust_delta_sq,
            coh_pre=ctx.coh_pre, bump_salt=False, coh_stats=ctx.coh_stats)
    else:
        apply_packed_sgd(
            ctx.packed_w, grad_W, ctx.weight_buf, ctx.row_exp, ctx.col_exp,
            ctx.row_max_buf, ctx.col_max_buf, lr=ctx.lr, mantissa_bias=ctx.mantissa_bias,
            alpha=ctx.alpha, beta1=ctx.beta1, alpha_v_fast=ctx.alpha_v_fast,
            mass_preserve=ctx.mass_preserve, track_rebalance=ctx.track_rebalance,
            bump_salt=False)
    if step_events is not None:
        step_events[2].record()


_CTX_FIELDS = ("packed_w", "row_exp", "col_exp", "lr", "alpha", "beta1", "mantissa_bias",
               "optimizer_kind", "weight_decay", "eps", "step_cap", "v_scale", "precond_p",
               "gf_consol", "drift_cancel_C", "alpha_v_fast", "wd_sv", "wd_sf", "mass_preserve",
               "apply_chase", "track_rebalance", "weight_buf", "row_max_buf", "col_max_buf",
               "v_row", "v_col", "sum_v_inv", "adafactor_beta2", "track_adafactor_v",
               "gf_trust_delta_sq", "coh_pre")


class FusedConcordLinearPackedB(torch.autograd.Function):
    """Linear layer whose backward is the optimizer step (packed_b.py:1197-1353).

    Same positional arguments as the reference's Function.  The forward reads
    the bf16 weight emitted by the previous step (materialize-merge).
    """

    @staticmethod
    def forward(ctx, x, packed_w, row_exp, col_exp, bias, lr, alpha, beta1, mantissa_bias,
                optimizer_kind, weight_decay, eps, step_cap, v_scale, precond_p, gf_consol,
                drift_cancel_C, alpha_v_fast, wd_sv, wd_sf, mass_preserve, apply_chase,
                track_rebalance, weight_buf, row_max_buf, col_max_buf, v_row, v_col, sum_v_inv,
                adafactor_beta2, track_adafactor_v, gf_trust_delta_sq, coh_pre, coh_stats=None):
        bias_bf16 = (bias.to(torch.bfloat16)
                     if bias is not None and bias.dtype != torch.bfloat16 else bias)
        y = _gemm.forward(x, weight_buf, bias_bf16)
        ctx.save_for_backward(x, weight_buf)
        vals = (packed_w, row_exp, col_exp, lr, alpha, beta1, mantissa_bias, optimizer_kind,
                weight_decay, eps, step_cap, v_scale, precond_p, gf_consol, drift_cancel_C,
                alpha_v_fast, wd_sv, wd_sf, mass_preserve, apply_chase, track_rebalance,
                weight_buf, row_max_buf, col_max_buf, v_row, v_col, sum_v_inv, adafactor_beta2,
                track_adafactor_v, gf_trust_delta_sq, coh_pre)
        for k, v in zip(_CTX_FIELDS, vals):
            setattr(ctx, k, v)
        ctx.coh_stats = coh_stats
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx, grad_y):
        x, weight = ctx.saved_tensors
        if grad_y.dtype != torch.bfloat16:
            grad_y = grad_y.to(torch.bfloat16)
        if not grad_y.is_contiguous():
            grad_y = grad_y.contiguous()
        grad_x = _gemm.grad_input(grad_y, weight)
        out_features, in_features = weight.shape
        x_flat = x.reshape(-1, in_features)
        grad_y_flat = grad_y.reshape(-1, out_features)
        if _fused_dw_vhat_ok(ctx, grad_y_flat, x_flat):
            track = bool(ctx.track_rebalance)
            grad_W = dw_vhat_update(grad_y_flat, x_flat, ctx.v_row, ctx.v_col, ctx.sum_v_inv,
                                    ctx.adafactor_beta2, ctx.row_max_buf if track else None,
                                    ctx.col_max_buf if track else None, bump_salt=True)
            _packed_backward_step(ctx, grad_W, vhat_done=True)
        else:
            grad_W = _gemm.grad_weight(grad_y_flat, x_flat)
            if _SIGMAG_NOISE:
                grad_W = sigmag_noise(grad_W, grad_y_flat, x_flat)
            _optimizer_half(ctx, grad_W)
        grad_bias = grad_y_flat.sum(0) if ctx.has_bias else None
        return (grad_x, None, None, None, grad_bias) + (None,) * 29


class ConcordLinearPackedB(nn.Module):
    """One int32 word per parameter (int16 s_fast | int8 s_slow | int8 v_slow) on
    shared row/col exponents; the backward is the optimizer step.

    Same constructor, attributes, buffers and methods as the reference
    (packed_b.py:1356-1856).  A bare layer is the validated optimizer:
    rank-1 v-hat AdamW (v_scale=0, gf_trust_delta_sq=1, eps=1e-10,
    precond_p=0.5) with the fixed coherence gate (coh_pre) on.
    """

    MANTISSA_BIAS = 15
    EXP_MIN = -8
    EXP_MAX = 7
    MAX_M = 24000

    def __init__(self, in_features, out_features, bias=True, device='cuda', alpha=0.1,
                 beta1=0.0, lr=0.01):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.alpha = alpha
        self.beta1 = beta1
        self._lr_value = float(lr)
        self.optimizer_kind = 'adamw'
        self.weight_decay = 0.0
        self._eps_value = 1e-10
        self.step_cap = 10.0
        self.v_scale = 0.0
        self.precond_p = 0.5
        self.gf_consol = 0.0
        self._coh_pre = None
        self.fast_gain = 1.0
        self.alpha_v_fast = 0.001
        self.drift_cancel_C = compute_drift_cancel_C(alpha, self.alpha_v_fast, mass_preserve=True)
        self.track_adafactor_v = True
        self.adafactor_beta2 = 0.999
        self.gf_trust_delta_sq = 1.0
        self.allow_tickdown = False
        self.wd_sv = 0.0
        self.wd_sf = 0.0
        self.mass_preserve_v = True
        self.apply_chase = True
        self.track_rebalance = True
        # fused coherence meter: (sum of coh, count) accumulated by the step kernel
        self.coh_stats = None
        self.register_buffer('_reb_seed', torch.zeros(1, dtype=torch.int32, device=device))
        self.register_buffer('packed_w', torch.zeros(out_features, in_features,
                                                     dtype=torch.int32, device=device))
        self.register_buffer('row_exp', torch.zeros(out_features, dtype=torch.int8, device=device))
        self.register_buffer('col_exp', torch.zeros(in_features, dtype=torch.int8, device=device))
        self.register_buffer('v_row', torch.zeros(out_features, dtype=torch.float32, device=device))
        self.register_buffer('v_col', torch.zeros(in_features, dtype=torch.float32, device=device))
        self.register_buffer('_sum_v_inv', torch.ones(1, dtype=torch.float32, device=device))
        self._coh_pre = torch.ones_like(self.packed_w, dtype=torch.float32)
        self.register_buffer('_row_max_hwm', torch.zeros(out_features, dtype=torch.int32,
                                                         device=device))
        self.register_buffer('_col_max_hwm', torch.zeros(in_features, dtype=torch.int32,
                                                         device=device))
        self.register_buffer('_lr_buf', torch.full((1,), self._lr_value, dtype=torch.float32,
                                                   device=device))
        self.register_buffer('_eps_buf', torch.full((1,), self._eps_value, dtype=torch.float32,
                                                    device=device))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16, device=device))
        else:
            self.register_parameter('bias', None)
        self._init_weight()
        self._ensure_buffers()

    @property
    def weight(self):
        """Read-only bf16 view of the live weight (kept fresh by the step)."""
        return getattr(self, '_bf16_weight_buf', None)

    @property
    def lr(self):
        return self._lr_value

    @lr.setter
    def lr(self, value):
        v = float(value)
        self._lr_value = v
        buf = getattr(self, '_lr_buf', None)
        if buf is not None:
            buf.fill_(v)

    @property
    def eps(self):
        return self._eps_value

    @eps.setter
    def eps(self, value):
        v = float(value)
        self._eps_value = v
        buf = getattr(self, '_eps_buf', None)
        if buf is not None:
            buf.fill_(v)

    @torch.no_grad()
    def enable_cohpre(self):
        self._coh_pre = torch.ones_like(self.packed_w, dtype=torch.float32)
        return self._coh_pre

    @torch.no_grad()
    def disable_cohpre(self):
        self._coh_pre = None

    def set_optimizer_kind(self, kind, weight_decay=0.0, eps=1.0, step_cap=10.0):
        if kind not in ('sgd', 'adamw'):
            raise ValueError("optimizer kind must be 'sgd' or 'adamw'")
        self.optimizer_kind = kind
        self.weight_decay = float(weight_decay)
        self.eps = float(eps)
        self.step_cap = float(step_cap)

    def _init_weight(self):
        std = (2.0 / (self.in_features + self.out_features)) ** 0.5
        w = torch.randn(self.out_features, self.in_features, device=self.packed_w.device) * std
        self.load_weights(w)

    def _quantize(self, W, finetune):
        W = W.to(device=self.packed_w.device, dtype=torch.float32).contiguous()
        _need_cuda(W, self.packed_w)
        N, K = self.packed_w.shape
        assert W.shape == (N, K)
        _abi.check(_lib().concord_quantize(
            _ptr(W), W.stride(0), _ptr(self.packed_w), self.packed_w.stride(0), _ptr(self.row_exp),
            _ptr(self.col_exp), N, K, self.MANTISSA_BIAS, self.EXP_MIN, self.EXP_MAX,
            int(finetune), _stream(W.device)), "concord_quantize")
        self._resync_weight_buf()

    @torch.no_grad()
    def load_weights(self, W):
        """Whole mantissa into s_fast; row_exp from the row max, col_exp = 0
        (packed_b.py:1570-1603)."""
        self._quantize(W, finetune=False)

    @torch.no_grad()
    def load_weights_finetune(self, W):
        """Pretrained init at the zero-gradient steady state: half the mantissa
        in v_slow, the rest in s_slow, the residual in s_fast (packed_b.py:1816-1856)."""
        self._quantize(W, finetune=True)

    @torch.no_grad()
    def _resync_weight_buf(self):
        wbuf = getattr(self, '_bf16_weight_buf', None)
        if wbuf is not None:
            materialize_packed_bf16(self.packed_w, self.row_exp, self.col_exp, out=wbuf,
                                    mantissa_bias=self.MANTISSA_BIAS)

    @torch.no_grad()
    def get_weight(self):
        """Live bf16 weight (s_slow*128 + s_fast + v_slow*128) * 2^exp."""
        out = torch.empty(self.packed_w.shape, dtype=torch.bfloat16, device=self.packed_w.device)
        return materialize_packed_bf16(self.packed_w, self.row_exp, self.col_exp, out,
                                       self.MANTISSA_BIAS)

    @torch.no_grad()
    def consolidated_weight(self):
        """Deployable weight: the slow accumulators only, s_fast dropped."""
        out = torch.empty(self.packed_w.shape, dtype=torch.bfloat16, device=self.packed_w.device)
        return materialize_packed_bf16(self.packed_w, self.row_exp, self.col_exp, out,
                                       self.MANTISSA_BIAS, consolidated=True)

    @torch.no_grad()
    def get_state(self):
        s_fast = self.packed_w >> 16
        s_slow_i8 = (self.packed_w << 16) >> 24
        v_slow_i8 = (self.packed_w << 24) >> 24
        return s_fast, s_slow_i8, v_slow_i8

    @torch.no_grad()
    def get_rebalance_watermark_stats(self):
        if getattr(self, '_row_max_buf', None) is None or not self.track_rebalance:
            return None, None
        return self._row_max_hwm.clone(), self._col_max_hwm.clone()

    @torch.no_grad()
    def get_garbage_fraction_stats(self):
        """Summary of the per-weight garbage fraction noise^2 / v-hat in [0, 1]
        (packed_b.py:1676-1730): mean, quartiles and the fractions below 0.1
        and above 0.9; None before the first v-hat update.  One pass of the
        garbage-fraction kernel; the quartiles sort its output on the GPU."""
        if self.v_row is None:
            return None
        sum_v = self.v_row.float().sum().reshape(1)
        if float(sum_v.item()) <= 0.0:
            return None
        sum_v.clamp_(min=1e-30)
        N, K = self.packed_w.shape
        gf = torch.empty(N * K, dtype=torch.float32, device=self.packed_w.device)
        acc = torch.zeros(3, dtype=torch.float64, device=self.packed_w.device)
        _abi.check(_lib().concord_garbage_fraction(
            _ptr(self.packed_w), self.packed_w.stride(0), _ptr(self.row_exp), _ptr(self.col_exp),
            _ptr(self.v_row), _ptr(self.v_col), _ptr(sum_v), N, K, int(self.MANTISSA_BIAS),
            float(self.drift_cancel_C), _ptr(gf), _ptr(acc), _stream(self.packed_w.device)),
            "concord_garbage_fraction")
        srt = torch.sort(gf).values
        qs = []
        for q in (0.25, 0.5, 0.75):   # linear interpolation between order statistics
            pos = q * (N * K - 1)
            lo = int(pos)
            hi = min(lo + 1, N * K - 1)
            qs.append((srt[lo], srt[hi], pos - lo))
        qv = torch.stack([a + (b - a) * f for a, b, f in qs]).tolist()
        tot, lo_n, hi_n = acc.tolist()
        cnt = float(N * K)
        return {'mean': tot / cnt, 'p25': qv[0], 'median': qv[1], 'p75': qv[2],
                'frac_signal_dominated': lo_n / cnt, 'frac_noise_dominated': hi_n / cnt}

    def _ensure_buffers(self):
        N, K = self.packed_w.shape
        wbuf = getattr(self, '_bf16_weight_buf', None)
        if wbuf is None or wbuf.shape != self.packed_w.shape:
            wbuf = torch.empty(self.packed_w.shape, dtype=torch.bfloat16, device=self.packed_w.device)
            self._bf16_weight_buf = wbuf
            materialize_packed_bf16(self.packed_w, self.row_exp, self.col_exp, out=wbuf,
                                    mantissa_bias=self.MANTISSA_BIAS)
        rmbuf = getattr(self, '_row_max_buf', None)
        if rmbuf is None or rmbuf.shape[0] != N:
            self._row_max_buf = torch.zeros(N, dtype=torch.int32, device=self.packed_w.device)
        cmbuf = getattr(self, '_col_max_buf', None)
        if cmbuf is None or cmbuf.shape[0] != K:
            self._col_max_buf = torch.zeros(K, dtype=torch.int32, device=self.packed_w.device)
        return self._bf16_weight_buf, self._row_max_buf, self._col_max_buf

    def _apply_args(self, wbuf, rmbuf, cmbuf):
        return (self._lr_buf, self.alpha, self.beta1, self.MANTISSA_BIAS, self.optimizer_kind,
                self.weight_decay, self._eps_buf, self.step_cap, self.v_scale, self.precond_p,
                self.gf_consol, self.drift_cancel_C, self.alpha_v_fast, self.wd_sv, self.wd_sf,
                self.mass_preserve_v, self.apply_chase, self.track_rebalance, wbuf, rmbuf, cmbuf,
                self.v_row, self.v_col, self._sum_v_inv, float(self.adafactor_beta2),
                bool(self.track_adafactor_v), float(self.gf_trust_delta_sq), self._coh_pre,
                self.coh_stats)

    def _gated_forward_weight(self, wbuf):
        """fast_gain < 1: forward through (s_slow + g*s_fast + v_slow) * 2^exp
        (packed_b.py:1762-1772)."""
        pw = self.packed_w
        sf = (pw >> 16).to(torch.float32)
        ss = ((pw << 16) >> 24).to(torch.float32)
        vs = ((pw << 24) >> 24).to(torch.float32)
        exp = self.row_exp.float()[:, None] + self.col_exp.float()[None, :] - self.MANTISSA_BIAS
        m_gated = (ss * 128.0 + self.fast_gain * sf + vs * 128.0) * torch.exp2(exp)
        wbuf.copy_(m_gated.to(wbuf.dtype))

    def forward(self, x):
        in_dtype = x.dtype
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        wbuf, rmbuf, cmbuf = self._ensure_buffers()
        if self.fast_gain < 1.0:
            with torch.no_grad():
                self._gated_forward_weight(wbuf)
        y = FusedConcordLinearPackedB.apply(x, self.packed_w, self.row_exp, self.col_exp,
                                            self.bias, *self._apply_args(wbuf, rmbuf, cmbuf))
        return y.to(in_dtype)

    @torch.no_grad()
    def optimizer_step(self, grad_W, coh_stats=None, step_events=None):
        """Run the optimizer half of the backward for a given bf16 dW [N, K]
        (what the autograd backward does after its GEMMs)."""
        _optimizer_half(self._step_ctx(coh_stats), grad_W.contiguous(), step_events)

    def _step_ctx(self, coh_stats=None):
        """The fields the backward's optimizer half reads, as the autograd ctx holds them."""
        wbuf, rmbuf, cmbuf = self._ensure_buffers()
        vals = (self.packed_w, self.row_exp, self.col_exp) + self._apply_args(wbuf, rmbuf, cmbuf)[:-1]
        ctx = SimpleNamespace(**dict(zip(_CTX_FIELDS, vals)))
        ctx.coh_stats = coh_stats if coh_stats is not None else self.coh_stats
        return ctx

    @torch.no_grad()
    def rebalance(self, fired_out=None):
        """Tick-up rebalance from the last step's row/col max; folds the
        high-watermarks and bumps the seed on the device (packed_b.py:1792-1814)."""
        dp = _sharded_of(self.packed_w)
        if dp is not None:
            dp.rebalance(fired_out)
            return
        rmbuf = getattr(self, '_row_max_buf', None)
        cmbuf = getattr(self, '_col_max_buf', None)
        if rmbuf is None or cmbuf is None:
            return
        rebalance_packed(self.packed_w, self.row_exp, self.col_exp, rmbuf, cmbuf,
                         MAX_M=self.MAX_M, EXP_MAX=self.EXP_MAX, EXP_MIN=self.EXP_MIN,
                         seed_buf=self._reb_seed, allow_tickdown=self.allow_tickdown,
                         row_hwm=self._row_max_hwm, col_hwm=self._col_max_hwm,
                         fired_out=fired_out, bump_seed=True)


class FusedConcordConv2dPackedB(torch.autograd.Function):
    """Conv2d whose backward is the packed step (packed_b.py:1863-2021).

    The weight is the packed [O, I*kh*kw] matrix.  When the GEMM extents
    (B*Ho*Wo, O, I*kh*kw) are multiples of 8 the convolutions run as this
    package's GEMMs over the unfolded input (gemm.conv2d_forward /
    conv2d_backward); other shapes use cuDNN, as the reference does for every
    shape.  The optimizer half is the same launches as the Linear layer.
    """

    @staticmethod
    def forward(ctx, x, packed_w, row_exp, col_exp, bias, in_channels, out_channels, kh, kw,
                stride, padding, lr, alpha, beta1, mantissa_bias, optimizer_kind, weight_decay,
                eps, step_cap, v_scale, precond_p, gf_consol, drift_cancel_C, alpha_v_fast, wd_sv,
                wd_sf, mass_preserve, apply_chase, track_rebalance, weight_buf, row_max_buf,
                col_max_buf, v_row, v_col, sum_v_inv, adafactor_beta2, track_adafactor_v,
                gf_trust_delta_sq, coh_pre, coh_stats=None):
        weight_4d = weight_buf.view(out_channels, in_channels, kh, kw)
        x_bf16 = x.to(torch.bfloat16) if x.dtype != torch.bfloat16 else x
        bias_bf16 = (bias.to(torch.bfloat16)
                     if bias is not None and bias.dtype != torch.bfloat16 else bias)
        ctx.implicit = _CONV_BACKEND == "implicit" and _gemm.conv_nhwc_usable(x_bf16, weight_buf, kh, kw,
                                                                              stride, padding)
        if ctx.implicit:
            # channels-last activations, the filter permuted once per forward
            x_bf16 = x_bf16.contiguous(memory_format=torch.channels_last)
            w_krsc = _gemm.filter_krsc(weight_buf, in_channels, kh, kw)
            ctx.gemm = False
            y = _gemm.conv2d_forward_nhwc(x_bf16, w_krsc, bias_bf16, kh, kw, stride, padding)
            ctx.save_for_backward(x_bf16, w_krsc)
        else:
            # a channels-last input on the implicit backend whose convolution the
            # implicit GEMM does not run (odd channel counts, strides) goes to cuDNN
            # in channels-last rather than through an NCHW column matrix
            cl = (_CONV_BACKEND == "implicit" and not x_bf16.is_contiguous()
                  and x_bf16.is_contiguous(memory_format=torch.channels_last))
            x_bf16 = x_bf16.contiguous(memory_format=torch.channels_last) if cl else x_bf16.contiguous()
            ctx.gemm = (not cl and _CONV_BACKEND in ("implicit", "gemm")
                        and _gemm.conv_usable(x_bf16, weight_buf, kh, kw, stride, padding))
            if ctx.gemm:
                y = _gemm.conv2d_forward(x_bf16, weight_buf, bias_bf16, kh, kw, stride, padding)
            else:
                y = torch.nn.functional.conv2d(x_bf16, weight_4d, bias=bias_bf16, stride=stride,
                                               padding=padding)
            ctx.save_for_backward(x_bf16, weight_4d)
        vals = (packed_w, row_exp, col_exp, lr, alpha, beta1, mantissa_bias, optimizer_kind,
                weight_decay, eps, step_cap, v_scale, precond_p, gf_consol, drift_cancel_C,
                alpha_v_fast, wd_sv, wd_sf, mass_preserve, apply_chase, track_rebalance,
                weight_buf, row_max_buf, col_max_buf, v_row, v_col, sum_v_inv, adafactor_beta2,
                track_adafactor_v, gf_trust_delta_sq, coh_pre)
        for k, v in zip(_CTX_FIELDS, vals):
            setattr(ctx, k, v)
        ctx.coh_stats = coh_stats
        ctx.conv = (in_channels, out_channels, kh, kw, stride, padding)
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx, grad_y):
        x_bf16, weight_4d = ctx.saved_tensors
        in_c, out_c, kh, kw, stride, padding = ctx.conv
        if grad_y.dtype != torch.bfloat16:
            grad_y = grad_y.to(torch.bfloat16)
        if ctx.implicit:                 # weight_4d holds the [O, kh, kw, C] filter here
            grad_x, grad_W = _gemm.conv2d_backward_nhwc(x_bf16, weight_4d, grad_y, kh, kw, stride, padding)
        elif ctx.gemm:
            grad_y = grad_y.contiguous()
            grad_x, grad_W = _gemm.conv2d_backward(x_bf16, weight_4d.view(out_c, -1), grad_y, kh, kw,
                                                   stride, padding)
        else:
            grad_y = grad_y.contiguous()
            grad_x = torch.nn.grad.conv2d_input(x_bf16.shape, weight_4d, grad_y, stride=stride,
                                                padding=padding)
            grad_W = torch.nn.grad.conv2d_weight(x_bf16, (out_c, in_c, kh, kw), grad_y,
                                                 stride=stride, padding=padding)
            grad_W = grad_W.reshape(out_c, -1).to(torch.bfloat16).contiguous()
        _optimizer_half(ctx, grad_W)
        grad_bias = grad_y.sum(dim=(0, 2, 3)) if ctx.has_bias else None
        return (grad_x, None, None, None, grad_bias) + (None,) * 35


class ConcordConv2dPackedB(ConcordLinearPackedB):
    """Conv2d variant: the same packed state viewed as [O, I*kh*kw] (packed_b.py:2024-2065)."""

    def __init__(self, in_channels, out_channels, kernel_size, stride=1, padding=0, bias=True,
                 device='cuda', alpha=0.1, beta1=0.0, lr=0.01):
        if isinstance(kernel_size, int):
            kh = kw = kernel_size
        else:
            kh, kw = kernel_size
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kh, self.kw = kh, kw
        self.stride = stride
        self.padding = padding
        super().__init__(in_features=in_channels * kh * kw, out_features=out_channels, bias=bias,
                         device=device, alpha=alpha, beta1=beta1, lr=lr)

    def forward(self, x):
        in_dtype = x.dtype
        wbuf, rmbuf, cmbuf = self._ensure_buffers()
        y = FusedConcordConv2dPackedB.apply(
            x, self.packed_w, self.row_exp, self.col_exp, self.bias, self.in_channels,
            self.out_channels, self.kh, self.kw, self.stride, self.padding,
            *self._apply_args(wbuf, rmbuf, cmbuf))
        return y.to(in_dtype)


# ============================================================
# Coherence meter + dissipation autotuner (packed_b.py:2068-2225)
# ============================================================

def gate_coherence_from_fields(s_fast, s_slow_i8, v_slow_i8, drift_cancel_C):
    """The fixed-coh Wiener gain from unpacked fields (float tensors); the row/col
    exponents cancel in the ratio (packed_b.py:2081-2091)."""
    d_fs = s_fast
    d_sv = (s_slow_i8 - v_slow_i8) * 128.0
    sig = drift_cancel_C * d_sv
    noise = d_fs - sig
    sig2 = sig * sig
    return sig2 / (sig2 + noise * noise + 1e-30)


def coherence_sum(packed_w, drift_cancel_C, out=None):
    """Device (sum of coh, count) over a packed tensor, accumulated into `out`
    (float64[2], zeroed here when not given)."""
    _need_cuda(packed_w)
    if out is None:
        out = torch.zeros(2, dtype=torch.float64, device=packed_w.device)
    N, K = packed_w.shape
    _abi.check(_lib().concord_coherence(_ptr(packed_w), packed_w.stride(0), N, K,
                                        float(drift_cancel_C), _ptr(out),
                                        _stream(packed_w.device)), "concord_coherence")
    return out


@torch.no_grad()
def measure_coherence(layer):
    """Mean gate coherence of one layer's packed state (packed_b.py:2094-2106),
    reduced on the GPU by the coherence kernel."""
    s = coherence_sum(layer.packed_w, float(layer.drift_cancel_C))
    s = s.cpu()
    return float(s[0] / s[1])


class DissipationAutoTuner:
    """Probe-then-commit choice of the evaporation rate kappa (`gf_consol`) and
    of beta1 (packed_b.py:2109-2225).

    Schedule: from construction until `probe_end` every layer runs at
    `probe_kappa` with beta1 = 0.  Every `measure_every` steps inside
    [probe_start, probe_end) the mean gate coherence of the layers (`meter`,
    default `measure_coherence`) is recorded.  At `probe_end` the window mean
    picks kappa by piecewise-linear interpolation in `table` (pairs
    (coherence, kappa) with coherence strictly descending; flat beyond either
    end), and beta1 = `beta1_on` when that mean reaches
    `beta1_coh_threshold`.  With `peak_lr`, the table's kappas and
    `probe_kappa` are friction values F = lr * kappa and are divided by it.
    """

    def __init__(self, layers, probe_start, probe_end, table, probe_kappa=50.0,
                 measure_every=10, verbose=True, beta1_on=0.1, beta1_coh_threshold=0.35,
                 peak_lr=None, meter=None):
        coh = np.asarray([float(c) for c, _ in table], dtype=np.float64)
        kap = np.asarray([float(k) for _, k in table], dtype=np.float64)
        if not 0 <= probe_start < probe_end:
            raise AssertionError(f"need 0 <= probe_start < probe_end, got {probe_start}, {probe_end}")
        if coh.size == 0 or np.any(np.diff(coh) >= 0):
            raise AssertionError("the table's coherence column must be strictly descending")
        unit = 1.0 if peak_lr is None else 1.0 / float(peak_lr)
        # np.interp wants ascending abscissae: keep the table reversed
        self._coh_up, self._kappa_up = coh[::-1].copy(), kap[::-1] * unit
        self.table = [(float(c), float(k)) for c, k in zip(coh, kap * unit)]
        self.layers = list(layers)
        self.probe_start, self.probe_end = int(probe_start), int(probe_end)
        self.probe_kappa = float(probe_kappa) * unit
        self.measure_every = max(1, int(measure_every))
        self.verbose = verbose
        self.beta1_on = float(beta1_on)
        self.beta1_coh_threshold = float(beta1_coh_threshold)
        self.meter = measure_coherence if meter is None else meter
        self._samples = []
        self.committed = None
        self.committed_beta1 = None
        self._set_all(self.probe_kappa, 0.0)

    def _set_all(self, kappa, beta1):
        for layer in self.layers:
            layer.gf_consol = kappa
            layer.beta1 = beta1

    def kappa_from_coh(self, c):
        """kappa for a window-mean coherence c (linear between table rows)."""
        return float(np.interp(float(c), self._coh_up, self._kappa_up))

    def _probing(self, t):
        return self.probe_start <= t < self.probe_end and (t - self.probe_start) % self.measure_every == 0

    def step(self, t):
        """Call at every step t before its backward.  Returns the committed kappa
        at the step that commits it (t >= probe_end, once), otherwise None."""
        if self.committed is not None:
            return None
        if self._probing(t) and self.layers:
            self._samples.append(float(np.mean([self.meter(m) for m in self.layers])))
        if t < self.probe_end:
            return None
        window = float(np.mean(self._samples)) if self._samples else self.table[0][0]
        self.committed = self.kappa_from_coh(window)
        use_b1 = self.beta1_on > 0 and window >= self.beta1_coh_threshold
        self.committed_beta1 = self.beta1_on if use_b1 else 0.0
        self._set_all(self.committed, self.committed_beta1)
        if self.verbose:
            print(f"[concord_b200] autotuner committed kappa={self.committed:g}, "
                  f"beta1={self.committed_beta1:g} from mean coherence {window:.4f} "
                  f"over {len(self._samples)} probes in steps [{self.probe_start}, {self.probe_end})")
        return self.committed
