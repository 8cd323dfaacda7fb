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
