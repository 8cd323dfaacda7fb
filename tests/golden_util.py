"""Helpers that turn a committed golden fixture into step parameters / inputs."""
import os

import numpy as np

from concord_b200._abi import ARITH_CR, make_step_params

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
STEP_CASES = ["bare", "nocohpre", "consol", "ratio", "legacycoh", "wd_beta1", "nochase",
              "notrust", "sgd_mp", "sgd"]


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def params_of(z):
    """StepParams for a fixture, built by the same host rule the package uses.
    The interpreter fixtures record the correctly rounded model (ARITH_CR)."""
    f = lambda k, d=0.0: float(z["cfg_" + k]) if ("cfg_" + k) in z else d  # noqa: E731
    b = lambda k: bool(z["cfg_" + k])  # noqa: E731
    kind = str(z["cfg_kind"])
    if kind == "sgd":
        return make_step_params(kind="sgd", alpha=f("alpha"), beta1=f("beta1"),
                                alpha_v_fast=f("alpha_v_fast"), mass_preserve=b("mass_preserve"),
                                track_rebalance=b("track_rebalance"), arith=ARITH_CR)
    return make_step_params(
        kind="adamw", alpha=f("alpha"), beta1=f("beta1"), weight_decay=f("weight_decay"),
        step_cap=f("step_cap"), v_scale=f("v_scale"), precond_p=f("precond_p"),
        gf_consol=f("gf_consol"), drift_cancel_C=f("drift_cancel_C"),
        alpha_v_fast=f("alpha_v_fast"), wd_sv=f("wd_sv"), wd_sf=f("wd_sf"),
        gf_trust_delta_sq=f("gf_trust_delta_sq"), gate_gain=f("gate_gain", 1.0),
        chase_floor=f("chase_floor"), leak_floor=f("leak_floor"),
        mass_preserve=b("mass_preserve"), apply_chase=b("apply_chase"),
        track_rebalance=b("track_rebalance"), use_cohpre=b("cohpre"),
        fixed_coh=b("fixed_coh"), ratio_coh=b("ratio"), arith=ARITH_CR)


def lr_eps(z):
    return float(z["cfg_lr"]), float(z.get("cfg_eps", 1.0))
