"""The CPU oracle against the reference's own outputs (committed fixtures).

Fixtures come from tests/golden/make_golden.py, which runs the unmodified
reference kernels (concord/packed_b.py) under Triton's interpreter.
"""
import numpy as np
import pytest

from golden_util import STEP_CASES, load, lr_eps, params_of


@pytest.mark.parametrize("case", STEP_CASES + ["tall"])
def test_step_bit_exact(oracle_mod, case):
    z = load("step_" + case)
    P = params_of(z)
    lr, eps = lr_eps(z)
    packed = z["init_packed"].copy()
    N, K = packed.shape
    coh_pre = z["init_coh_pre"].copy() if z["init_coh_pre"].size else None
    for t in range(int(z["steps"])):
        wbuf = np.zeros((N, K), np.uint16)
        rmax = np.zeros(N, np.int32)
        cmax = np.zeros(K, np.int32)
        oracle_mod.step(P, packed, z[f"grad{t}"], wbuf, z["row_exp"], z["col_exp"], rmax, cmax,
                        z["v_row"], z["v_col"], z["sum_v_inv"], coh_pre, lr, eps,
                        int(z[f"salt{t}"]))
        np.testing.assert_array_equal(packed, z[f"packed{t}"], err_msg=f"words step {t}")
        np.testing.assert_array_equal(wbuf, z[f"wbuf{t}"], err_msg=f"wbuf step {t}")
        np.testing.assert_array_equal(rmax, z[f"rmax{t}"])
        np.testing.assert_array_equal(cmax, z[f"cmax{t}"])
        if coh_pre is not None:
            np.testing.assert_array_equal(coh_pre, z[f"coh_pre{t}"])


@pytest.mark.parametrize("case", ["up", "down"])
def test_rebalance_bit_exact(oracle_mod, case):
    z = load("rebalance_" + case)
    packed = z["init_packed"].copy()
    rexp, cexp = z["init_row_exp"].copy(), z["init_col_exp"].copy()
    seed = np.array([int(z["seed0"]) - 1], np.int32)
    for t in range(2):
        oracle_mod.rebalance(packed, rexp, cexp, z["rmax"], z["cmax"], None, None, seed,
                             allow_tickdown=bool(z["allow_tickdown"]))
        assert int(seed[0]) == int(z[f"seed{t}"])
        np.testing.assert_array_equal(packed, z[f"packed{t}"])
        np.testing.assert_array_equal(rexp, z[f"row_exp{t}"])
        np.testing.assert_array_equal(cexp, z[f"col_exp{t}"])


def test_quantize_and_materialize(oracle_mod):
    z = load("quantize")
    for ft in (False, True):
        tag = "ft" if ft else "base"
        packed, rexp, cexp = oracle_mod.quantize(z["W"], finetune=ft)
        np.testing.assert_array_equal(packed, z["packed_" + tag])
        np.testing.assert_array_equal(rexp, z["row_exp_" + tag])
        np.testing.assert_array_equal(oracle_mod.materialize(packed, rexp, cexp),
                                      z["get_weight_" + tag])
        np.testing.assert_array_equal(
            oracle_mod.materialize(packed, rexp, cexp, consolidated=True), z["consolidated_" + tag])


def test_rng_and_hash(oracle_mod):
    z = load("coherence_rng")
    lib = oracle_mod.lib()
    for i in range(5):
        seed = int(z[f"seed{i}"])
        r = np.array([lib.oracle_tl_rand(seed, int(p)) for p in z[f"pos{i}"]], np.float32)
        np.testing.assert_array_equal(r, z[f"rand{i}"])
        h = np.array([lib.oracle_hash_uniform(int(a), int(b), int(c))
                      for a, b, c in zip(z[f"x{i}"], z[f"pos{i}"], z[f"salt{i}"])], np.float32)
        np.testing.assert_array_equal(h, z[f"hash{i}"])


def test_coherence_mean(oracle_mod):
    z = load("coherence_rng")
    s, n = oracle_mod.coherence(z["coh_packed"], float(z["coh_C"]))
    assert abs(s / n - float(z["coh_mean"])) < 1e-6


def test_layer_trajectory(oracle_mod):
    """Bare layer, 4 steps: words bit-exact given the reference's v-hat, and the
    oracle's fixed-order v-hat within fp32 summation-order tolerance."""
    z = load("layer_bare")
    from concord_b200._abi import ARITH_CR, make_step_params
    from concord_b200.packed_b import compute_drift_cancel_C
    P = make_step_params(kind="adamw", arith=ARITH_CR, alpha=0.1, v_scale=0.0, precond_p=0.5, step_cap=10.0,
                         drift_cancel_C=compute_drift_cancel_C(0.1, 0.001, mass_preserve=True),
                         alpha_v_fast=0.001, gf_trust_delta_sq=1.0, mass_preserve=True,
                         use_cohpre=True)
    packed = z["packed_init"].copy()
    N, K = packed.shape
    rexp, cexp = z["row_exp_init"].copy(), np.zeros(K, np.int8)
    coh_pre = np.ones((N, K), np.float32)
    hwm_r, hwm_c = np.zeros(N, np.int32), np.zeros(K, np.int32)
    seed = np.zeros(1, np.int32)
    for t in range(4):
        np.testing.assert_array_equal(packed, z[f"packed_before{t}"])
        vr, vc, svi = z[f"v_row_prev{t}"].copy(), z[f"v_col_prev{t}"].copy(), np.ones(1, np.float32)
        oracle_mod.vhat(z[f"grad{t}"], vr, vc, svi)
        np.testing.assert_allclose(vr, z[f"v_row{t}"], rtol=2e-6, atol=0)
        np.testing.assert_allclose(vc, z[f"v_col{t}"], rtol=2e-6, atol=0)
        np.testing.assert_allclose(svi, z[f"sum_v_inv{t}"], rtol=2e-6)
        wbuf = np.zeros((N, K), np.uint16)
        rmax, cmax = np.zeros(N, np.int32), np.zeros(K, np.int32)
        oracle_mod.step(P, packed, z[f"grad{t}"], wbuf, rexp, cexp, rmax, cmax,
                        z[f"v_row{t}"], z[f"v_col{t}"], z[f"sum_v_inv{t}"], coh_pre, 5e-3, 1e-10,
                        int(z[f"salt{t}"]))
        np.testing.assert_array_equal(packed, z[f"packed{t}"])
        np.testing.assert_array_equal(wbuf, z[f"wbuf{t}"])
        np.testing.assert_array_equal(coh_pre, z[f"coh_pre{t}"])
        oracle_mod.rebalance(packed, rexp, cexp, rmax, cmax, hwm_r, hwm_c, seed)
        np.testing.assert_array_equal(packed, z[f"packed_reb{t}"])
        np.testing.assert_array_equal(rexp, z[f"row_exp{t}"])
        np.testing.assert_array_equal(hwm_r, z[f"row_hwm{t}"])
        assert int(seed[0]) == int(z[f"reb_seed{t}"])
    np.testing.assert_array_equal(oracle_mod.materialize(packed, rexp, cexp), z["get_weight"])
    np.testing.assert_array_equal(oracle_mod.materialize(packed, rexp, cexp, consolidated=True),
                                  z["consolidated"])
