"""The oracle's gradient-accumulation gate, on the CPU (the CUDA kernel is
compared with it in tests/test_gpu_accum.py).  Rule restated from the
reference's prototype kernel (notebook/src/prototype_packed_b.py:661-782)."""
import numpy as np


def _case(oracle_mod, cons):
    from concord_b200._abi import ARITH_CR, make_step_params
    rng = np.random.default_rng(7)
    N, K = 24, 40
    sf = rng.integers(-3000, 3001, (N, K))
    ss = rng.integers(-100, 101, (N, K))
    vs = rng.integers(-100, 101, (N, K))
    packed = (((sf & 0xFFFF) << 16) | ((ss & 0xFF) << 8) | (vs & 0xFF)).astype(np.uint32).view(np.int32)
    grad = oracle_mod.f32_to_bf16(rng.normal(0, 1e-2, (N, K)).astype(np.float32))
    P = make_step_params(kind="adamw", arith=ARITH_CR, v_scale=0.0, precond_p=0.5, drift_cancel_C=0.018,
                         gf_trust_delta_sq=1.0, gf_consol=30.0, beta1=0.3, wd_sv=0.1, wd_sf=0.05,
                         mass_preserve=True, use_cohpre=True)
    flag = np.array([0 if cons is None else cons], np.int32)
    if cons is not None:
        P.consolidate = flag.ctypes.data
    out = packed.copy()
    w = np.full((N, K), 7, np.uint16)
    rm, cm = np.zeros(N, np.int32), np.zeros(K, np.int32)
    coh = np.full((N, K), 0.5, np.float32)
    oracle_mod.step(P, out, grad, w, np.zeros(N, np.int8), np.zeros(K, np.int8), rm, cm,
                    np.full(N, 1e-4, np.float32), np.full(K, 1e-4, np.float32),
                    np.array([1.0 / (N * 1e-4)], np.float32), coh, 0.05, 1e-10, 12345)
    return packed, out, w, rm, cm, coh


def test_tick_only_micro_step(oracle_mod):
    packed, out, w, rm, cm, coh = _case(oracle_mod, 0)
    assert np.array_equal(out & 0xFFFF, packed & 0xFFFF)     # s_slow, v_slow untouched
    assert not np.array_equal(out, packed)                    # the gradient ticked s_fast
    assert (w == 7).all() and not rm.any() and not cm.any()   # weight and maxima frozen
    assert not (coh == 0.5).all()                             # coh_pre still updated


def test_consolidate_one_is_the_plain_step(oracle_mod):
    a = _case(oracle_mod, 1)
    b = _case(oracle_mod, None)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


ACCUM_CASES = ["bare", "consol", "ratio", "wd"]


def replay_accum_fixture(z, step_fn):
    """Drive `step_fn(P, packed, grad, wbuf, rmax, cmax, coh, lr, eps, salt)` through
    a prototype fixture's micro-step sequence; returns the per-step mismatches."""
    from golden_util import lr_eps, params_of
    P = params_of(z)
    lr, eps = lr_eps(z)
    N, K = int(z["N"]), int(z["K"])
    flag = np.zeros(1, np.int32)
    floors = np.array([z["cfg_chase_floor"], z["cfg_leak_floor"]], np.float32)
    packed = z["init_packed"].copy()
    coh = z["init_coh_pre"].copy() if z["init_coh_pre"].size else None
    wbuf = np.full((N, K), 7, np.uint16)
    bad = []
    for t, cons in enumerate(z["consolidate"]):
        flag[0] = cons
        rm, cm = np.zeros(N, np.int32), np.zeros(K, np.int32)
        step_fn(P, flag, floors if bool(z["cfg_ratio"]) else None, packed, z[f"grad{t}"], wbuf, rm, cm, coh,
                lr, eps, int(z[f"salt{t}"]))
        for name, got in (("packed", packed), ("wbuf", wbuf), ("rmax", rm), ("cmax", cm)) + \
                (((("coh_pre", coh),)) if coh is not None else ()):
            if not np.array_equal(got, z[f"{name}{t}"]):
                bad.append((t, name, int((got != z[f"{name}{t}"]).sum())))
    return bad


def test_oracle_matches_prototype_accumulation_fixtures(oracle_mod):
    """The gate pinned to the reference's prototype kernel itself
    (tests/golden/make_golden_accum.py): tick-only micro-steps and
    consolidating steps, bit for bit."""
    from golden_util import load

    for case in ACCUM_CASES:
        z = load("accum_" + case)

        def step(P, flag, floors, packed, grad, wbuf, rm, cm, coh, lr, eps, salt):
            P.consolidate = flag.ctypes.data
            P.ratio_floors = floors.ctypes.data if floors is not None else None
            oracle_mod.step(P, packed, grad, wbuf, z["row_exp"], z["col_exp"], rm, cm, z["v_row"].copy(),
                            z["v_col"].copy(), z["sum_v_inv"].copy(), coh, lr, eps, salt)
        assert replay_accum_fixture(z, step) == [], case
