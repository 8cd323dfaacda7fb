"""Fixtures for the gradient-accumulation gate from the REFERENCE's prototype
kernel (notebook/src/prototype_packed_b.py:454-790, the only reference kernel
with the consolidate flag), run under Triton's CPU interpreter:

    TRITON_INTERPRET=1 python tests/golden/make_golden_accum.py /path/to/Concord

The interpreter's two implementation-defined primitives are pinned as in
make_golden.py (correctly rounded exp2/log2, RNE fp32->bf16).  The prototype
differs from the canonical kernel outside the gate (a coherence-gated +beta1
term, gap feedback, a v-hat bias-correction buffer); the fixtures keep those
inert (beta1 = 0, gap feedback off, bias correction 1.0) so that they pin
exactly the gate: micro-steps with consolidate = 0 (tick-only, weight and
maxima frozen) interleaved with consolidating steps.  Ratio floors come from
the prototype's device tensors.  Output: accum_<case>.npz beside this file.
"""
import os
import sys

import numpy as np

assert os.environ.get("TRITON_INTERPRET") == "1", "run with TRITON_INTERPRET=1"
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CONCORD_REF", "")
assert REF and os.path.isdir(os.path.join(REF, "notebook", "src")), "pass the reference checkout"
sys.path.insert(0, os.path.join(REF, "notebook", "src"))

import torch  # noqa: E402
import triton.language as tl  # noqa: E402
from triton.runtime import interpreter as _interp  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def _cr_unary(fn):
    def op(self, arg):
        d = arg.data
        r = fn(d.astype(np.longdouble)).astype(np.float32) if d.dtype == np.float32 else fn(d)
        return _interp.TensorHandle(r, arg.dtype.scalar)
    return op


_interp.InterpreterBuilder.create_exp2 = _cr_unary(np.exp2)
_interp.InterpreterBuilder.create_log2 = _cr_unary(np.log2)
_orig_cast = _interp.InterpreterBuilder.cast_impl


def _cast_rne(self, src, dst_type):
    if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
        u = src.data.view(np.uint32).astype(np.uint64)
        nan = (u & 0x7FFFFFFF) > 0x7F800000
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
        return _interp.TensorHandle(r, dst_type.scalar)
    return _orig_cast(self, src, dst_type)


_interp.InterpreterBuilder.cast_impl = _cast_rne

import prototype_packed_b as pp  # noqa: E402  (the unmodified prototype)

CSTAR = pp.compute_drift_cancel_C(0.1, 0.001, mass_preserve=True)
BASE = dict(alpha=0.1, beta1=0.0, weight_decay=0.0, eps=1e-10, step_cap=10.0, v_scale=0.0, precond_p=0.5,
            gf_consol=0.0, drift_cancel_C=CSTAR, alpha_v_fast=0.001, wd_sv=0.0, wd_sf=0.0,
            mass_preserve=True, apply_chase=True, track_rebalance=True, gf_trust_delta_sq=1.0,
            cohpre=True, lr=5e-3)
CASES = {
    "bare": (dict(BASE), [0, 0, 1, 0, 1]),
    "consol": (dict(BASE, gf_consol=5.0), [0, 1, 0, 1]),
    "ratio": (dict(BASE, cohpre=False, ratio=True, floors=(0.6, 0.95)), [0, 0, 1]),
    "wd": (dict(BASE, weight_decay=0.01, wd_sv=1.0, wd_sf=0.5, gate_gain=0.7, mass_preserve=False,
                v_scale=1.0, eps=1e-8, precond_p=0.4, step_cap=3.0, gf_trust_delta_sq=0.5,
                drift_cancel_C=pp.compute_drift_cancel_C(0.1, 0.001, mass_preserve=False)), [0, 1, 1]),
}


def np_(t):
    return t.detach().clone().contiguous().numpy()


def bf16_bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def run(name, cfg, seq, N=36, K=70, seed=3):
    g = torch.Generator().manual_seed(seed)
    sf = torch.randint(-3000, 3001, (N, K), generator=g, dtype=torch.int32)
    ss = torch.randint(-100, 101, (N, K), generator=g, dtype=torch.int32)
    vs = torch.randint(-100, 101, (N, K), generator=g, dtype=torch.int32)
    packed = ((sf & 0xFFFF) << 16) | ((ss & 0xFF) << 8) | (vs & 0xFF)
    row_exp = torch.randint(-3, 5, (N,), generator=g, dtype=torch.int8)
    col_exp = torch.randint(-2, 3, (K,), generator=g, dtype=torch.int8)
    v_row = torch.rand(N, generator=g) * 1e-4 + 1e-6
    v_col = torch.rand(K, generator=g) * 1e-4 + 1e-6
    sum_v_inv = (1.0 / v_row.sum()).reshape(1).float()
    coh_pre = torch.rand(N, K, generator=g) if cfg.get("cohpre") else None
    wbuf = torch.full((N, K), 7, dtype=torch.int16).view(torch.bfloat16)
    rec = dict(N=N, K=K, init_packed=np_(packed), row_exp=np_(row_exp), col_exp=np_(col_exp),
               v_row=np_(v_row), v_col=np_(v_col), sum_v_inv=np_(sum_v_inv),
               init_coh_pre=np_(coh_pre) if coh_pre is not None else np.zeros(0, np.float32),
               consolidate=np.array(seq, np.int32))
    pp._USE_FIXED_COH, pp._RATIO_COH, pp._GAP_FEEDBACK = True, cfg.get("ratio", False), False
    pp._GATE_GAIN = cfg.get("gate_gain", 1.0)
    fl = cfg.get("floors", (0.9, 0.999))
    pp._RATIO_CHASE_FLOOR, pp._RATIO_LEAK_FLOOR = fl
    pp._RATIO_CHASE_FLOOR_T.clear()
    pp._RATIO_LEAK_FLOOR_T.clear()
    dev = torch.device("cpu")
    ctr = pp._get_step_counter(dev)
    for t, cons in enumerate(seq):
        grad = (torch.randn(N, K, generator=g) * 1e-3 + torch.randn(N, 1, generator=g) * 5e-4).to(torch.bfloat16)
        rmax = torch.zeros(N, dtype=torch.int32)
        cmax = torch.zeros(K, dtype=torch.int32)
        pp.set_consolidate(dev, bool(cons))
        salt = int(ctr.item()) + 1
        pp.apply_packed_adamw(
            packed, grad, wbuf, row_exp, col_exp, rmax, cmax, lr=cfg["lr"], alpha=cfg["alpha"],
            beta1=cfg["beta1"], weight_decay=cfg["weight_decay"], eps=cfg["eps"], step_cap=cfg["step_cap"],
            v_scale=cfg["v_scale"], precond_p=cfg["precond_p"], gf_consol=cfg["gf_consol"],
            drift_cancel_C=cfg["drift_cancel_C"], alpha_v_fast=cfg["alpha_v_fast"], wd_sv=cfg["wd_sv"],
            wd_sf=cfg["wd_sf"], mass_preserve=cfg["mass_preserve"], apply_chase=cfg["apply_chase"],
            track_rebalance=cfg["track_rebalance"], v_row=v_row, v_col=v_col, sum_v_inv=sum_v_inv,
            gf_trust_delta_sq=cfg["gf_trust_delta_sq"], coh_pre=coh_pre)
        assert int(ctr.item()) == salt
        rec[f"grad{t}"] = bf16_bits(grad)
        rec[f"salt{t}"] = np.int32(salt)
        rec[f"packed{t}"] = np_(packed)
        rec[f"wbuf{t}"] = bf16_bits(wbuf)
        rec[f"rmax{t}"] = np_(rmax)
        rec[f"cmax{t}"] = np_(cmax)
        if coh_pre is not None:
            rec[f"coh_pre{t}"] = np_(coh_pre)
    pp.set_consolidate(dev, True)
    for k in ["alpha", "beta1", "weight_decay", "eps", "step_cap", "v_scale", "precond_p", "gf_consol",
              "drift_cancel_C", "alpha_v_fast", "wd_sv", "wd_sf", "gf_trust_delta_sq", "lr"]:
        rec["cfg_" + k] = np.float64(cfg[k])
    rec["cfg_gate_gain"] = np.float64(cfg.get("gate_gain", 1.0))
    rec["cfg_kind"] = np.array("adamw")
    for b in ["mass_preserve", "apply_chase", "track_rebalance", "cohpre", "ratio"]:
        rec["cfg_" + b] = np.bool_(cfg.get(b, False))
    rec["cfg_fixed_coh"] = np.bool_(True)
    rec["cfg_chase_floor"], rec["cfg_leak_floor"] = np.float64(fl[0]), np.float64(fl[1])
    rec["steps"] = np.int32(len(seq))
    np.savez_compressed(os.path.join(OUT, f"accum_{name}.npz"), **rec)
    print("accum", name, "ok", flush=True)


if __name__ == "__main__":
    for name, (cfg, seq) in CASES.items():
        run(name, cfg, seq)
