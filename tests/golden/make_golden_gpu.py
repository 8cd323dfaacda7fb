"""Generate fixtures from the REFERENCE as it runs compiled on a B200.

Run on a GPU box where `baseline/_ref` holds the unmodified reference
(installed by `baseline/install_ref.sh`); the fixtures it writes are small and
committed, so the tests need neither the reference nor its checkout:

    python tests/golden/make_golden_gpu.py [step] [c1] [c2]

* `gpu_step_<case>.npz`: the reference's `apply_packed_adamw` /
  `apply_packed_sgd` (Triton, compiled for the GPU) on the flag sets of
  the interpreter fixtures, three steps each on a ragged 96 x 200 state:
  every word, bf16 weight, coh_pre and row/col maximum.
* `gpu_c1.npz`: BASELINE config 1 through the reference layer's own
  autograd backward (`ConcordLinearPackedB`, 1024 x 1024, 200 steps, lr 5e-4,
  seed 0, bare defaults and `disable_cohpre`), dW made equal to G_t by a
  bf16 identity input (dW = G_t^T-as-grad_y^T @ I is exact).  Per step the
  SHA-256 of the words, exponents, bf16 weight and v-hat buffers; at the end
  the exponents and the consolidated weight's hash.
* `gpu_c2.npz`: ten steps of config 2's largest layer (10240 x 2048) through
  the reference's functional step with a seeded bf16 dW and the reference's
  own torch v-hat expression; per-step hashes as above.
"""
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
sys.path.insert(0, HERE)

import concord.packed_b as pb  # noqa: E402  (the unmodified reference)
from gpu_cases import (BARE, C1_LR, C1_N, C1_STEPS, STEP_CASES, c1_grad, c1_inputs, c2_grad,  # noqa: E402
                       rand_step_inputs)

BARE_C2 = dict(BARE, lr=5e-4)

DEV = torch.device("cuda:0")


def sha(t):
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def bits(t):
    t = t.detach().contiguous().cpu()
    return t.view(torch.int16).numpy().view(np.uint16).copy() if t.dtype == torch.bfloat16 else t.numpy().copy()


def _knobs(cfg):
    pb._USE_FIXED_COH = cfg.get("fixed_coh", True)
    pb._RATIO_COH = cfg.get("ratio", False)
    pb._RATIO_CHASE_FLOOR, pb._RATIO_LEAK_FLOOR = cfg.get("floors", (0.9, 0.999))
    pb._GATE_GAIN = cfg.get("gate_gain", 1.0)


def _reset_knobs():
    pb._USE_FIXED_COH, pb._RATIO_COH, pb._GATE_GAIN = True, False, 1.0
    pb._RATIO_CHASE_FLOOR, pb._RATIO_LEAK_FLOOR = 0.9, 0.999


def ref_apply(cfg, st, grad):
    """One reference launch on the state dict `st` (mutated in place)."""
    _knobs(cfg)
    st["rmax"].zero_()
    st["cmax"].zero_()
    if cfg["kind"] == "sgd":
        pb.apply_packed_sgd(st["packed"], grad, st["wbuf"], st["row_exp"], st["col_exp"], st["rmax"], st["cmax"],
                            lr=cfg["lr"], alpha=cfg["alpha"], beta1=cfg["beta1"],
                            alpha_v_fast=cfg["alpha_v_fast"], mass_preserve=cfg["mass_preserve"],
                            track_rebalance=cfg["track_rebalance"])
    else:
        pb.apply_packed_adamw(
            st["packed"], grad, st["wbuf"], st["row_exp"], st["col_exp"], st["rmax"], st["cmax"], lr=cfg["lr"],
            alpha=cfg["alpha"], beta1=cfg["beta1"], weight_decay=cfg["weight_decay"], eps=cfg["eps"],
            step_cap=cfg["step_cap"], v_scale=cfg["v_scale"], precond_p=cfg["precond_p"],
            gf_consol=cfg["gf_consol"], drift_cancel_C=cfg["drift_cancel_C"], alpha_v_fast=cfg["alpha_v_fast"],
            wd_sv=cfg["wd_sv"], wd_sf=cfg["wd_sf"], mass_preserve=cfg["mass_preserve"],
            apply_chase=cfg["apply_chase"], track_rebalance=cfg["track_rebalance"], v_row=st["v_row"],
            v_col=st["v_col"], sum_v_inv=st["svi"], gf_trust_delta_sq=cfg["gf_trust_delta_sq"],
            coh_pre=st["coh_pre"] if cfg.get("cohpre") else None)
    _reset_knobs()


def gen_steps():
    for ci, (name, cfg) in enumerate(STEP_CASES.items()):
        d = rand_step_inputs(1000 + ci)
        st = {k: v.to(DEV) for k, v in d.items() if k != "grads"}
        N, K = st["packed"].shape
        st["wbuf"] = torch.zeros(N, K, dtype=torch.bfloat16, device=DEV)
        st["rmax"] = torch.zeros(N, dtype=torch.int32, device=DEV)
        st["cmax"] = torch.zeros(K, dtype=torch.int32, device=DEV)
        rec = {}
        ctr = pb._get_step_counter(DEV)
        for t, gr in enumerate(d["grads"]):
            rec[f"salt{t}"] = np.int32(int(ctr.item()) + 1)
            ref_apply(cfg, st, gr.to(DEV))
            for k in ("packed", "wbuf", "rmax", "cmax", "coh_pre"):
                rec[f"{k}{t}"] = bits(st[k])
        np.savez_compressed(os.path.join(HERE, f"gpu_step_{name}.npz"), **rec)
        print("gpu step", name, "ok", flush=True)


def gen_c1():
    rec = {}
    for arm, gate in (("gate", True), ("nogate", False)):
        g, W0, U, V = c1_inputs()
        layer = pb.ConcordLinearPackedB(C1_N, C1_N, bias=False, device=DEV, lr=C1_LR)
        layer.load_weights(W0.to(DEV))
        if not gate:
            layer.disable_cohpre()
        eye = torch.eye(C1_N, dtype=torch.bfloat16, device=DEV)
        rec[f"{arm}_init"] = sha(layer.packed_w)
        rec[f"{arm}_salt0"] = np.int32(int(pb._get_step_counter(DEV).item()))
        h = {k: [] for k in ("packed", "rexp", "cexp", "wbuf", "v_row", "v_col", "svi")}
        for t in range(C1_STEPS):
            G = c1_grad(g, U, V).to(DEV)
            x = eye.clone().requires_grad_(True)
            y = layer(x)
            y.backward(G.t().contiguous())       # dW = G @ I = G exactly
            layer.rebalance()
            torch.cuda.synchronize()
            for k, tt in (("packed", layer.packed_w), ("rexp", layer.row_exp), ("cexp", layer.col_exp),
                          ("wbuf", layer._bf16_weight_buf), ("v_row", layer.v_row), ("v_col", layer.v_col),
                          ("svi", layer._sum_v_inv)):
                h[k].append(sha(tt))
        for k, v in h.items():
            rec[f"{arm}_{k}"] = np.array(v)
        rec[f"{arm}_final_rexp"] = bits(layer.row_exp)
        rec[f"{arm}_final_cexp"] = bits(layer.col_exp)
        rec[f"{arm}_consolidated"] = sha(layer.consolidated_weight())
        print("gpu c1", arm, "ok", flush=True)
    np.savez_compressed(os.path.join(HERE, "gpu_c1.npz"), **rec)


def gen_c2():
    from gpu_cases import C2_N, C2_K, C2_STEPS, c2_state, torch_vhat
    g, W0 = c2_state()
    layer = pb.ConcordLinearPackedB(C2_K, C2_N, bias=False, device=DEV, lr=5e-4)
    layer.load_weights(W0.to(DEV))
    st = dict(packed=layer.packed_w, row_exp=layer.row_exp, col_exp=layer.col_exp, v_row=layer.v_row,
              v_col=layer.v_col, svi=layer._sum_v_inv, coh_pre=layer._coh_pre,
              wbuf=torch.zeros(C2_N, C2_K, dtype=torch.bfloat16, device=DEV),
              rmax=torch.zeros(C2_N, dtype=torch.int32, device=DEV),
              cmax=torch.zeros(C2_K, dtype=torch.int32, device=DEV))
    cfg = dict(BARE_C2)
    rec = {"init": sha(layer.packed_w), "salt0": np.int32(int(pb._get_step_counter(DEV).item()))}
    h = {k: [] for k in ("packed", "wbuf", "coh_pre", "rmax", "cmax")}
    for t in range(C2_STEPS):
        G = c2_grad(g).to(DEV)
        torch_vhat(G, st["v_row"], st["v_col"], st["svi"])
        ref_apply(cfg, st, G)
        torch.cuda.synchronize()
        for k in h:
            h[k].append(sha(st[k]))
    for k, v in h.items():
        rec[k] = np.array(v)
    np.savez_compressed(os.path.join(HERE, "gpu_c2.npz"), **rec)
    print("gpu c2 ok", flush=True)


if __name__ == "__main__":
    groups = sys.argv[1:] or ["step", "c1", "c2"]
    print("reference:", pb.__file__, flush=True)
    if "step" in groups:
        gen_steps()
    if "c1" in groups:
        gen_c1()
    if "c2" in groups:
        gen_c2()
