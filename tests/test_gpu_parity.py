"""CUDA path vs the reference's outputs and the CPU oracle (needs a B200).

Everything here goes through the C ABI of concord_b200/_lib/libconcord_b200.so.
Integer state (packed words, exponents, maxima, salts) and every value the
reference computes in a fixed order must match bit for bit.
"""
import zlib

import numpy as np
import pytest
import torch

from golden_util import STEP_CASES, load, lr_eps, params_of

pytestmark = pytest.mark.gpu

DEV = "cuda"


def T(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.to(DEV)


def bf16(a):
    return T(a.view(np.int16), None).view(torch.bfloat16)


def N_(t):
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


@pytest.fixture(scope="module")
def pb():
    from concord_b200 import packed_b
    packed_b._lib()
    return packed_b


def run_cuda_step(pb, P, packed, grad_bits, row_exp, col_exp, v_row, v_col, svi, coh_pre, lr, eps,
                  salt, row0=0, coh_stats=None):
    """One concord_step launch on device copies; returns numpy results."""
    N, K = packed.shape
    p = T(packed)
    w = torch.zeros(N, K, dtype=torch.bfloat16, device=DEV)
    rm = torch.zeros(N, dtype=torch.int32, device=DEV)
    cm = torch.zeros(K, dtype=torch.int32, device=DEV)
    cp = T(coh_pre) if coh_pre is not None else None
    lr_t = torch.tensor([lr], dtype=torch.float32, device=DEV)
    eps_t = torch.tensor([eps], dtype=torch.float32, device=DEV)
    s_t = torch.tensor([salt], dtype=torch.int32, device=DEV)
    pb._step_launch(P, p, bf16(grad_bits), w, T(row_exp), T(col_exp), rm, cm,
                    T(v_row) if v_row is not None else None, T(v_col) if v_col is not None else None,
                    T(svi) if svi is not None else None, cp, lr_t, eps_t, s_t, row0=row0,
                    coh_stats=coh_stats)
    torch.cuda.synchronize()
    return N_(p), N_(w), N_(rm), N_(cm), (N_(cp) if cp is not None else None)


@pytest.mark.parametrize("case", STEP_CASES + ["tall"])
def test_step_matches_reference_golden(pb, case):
    z = load("step_" + case)
    P = params_of(z)
    lr, eps = lr_eps(z)
    packed = z["init_packed"]
    coh_pre = z["init_coh_pre"] if z["init_coh_pre"].size else None
    for t in range(int(z["steps"])):
        packed, w, rm, cm, cp = run_cuda_step(pb, P, packed, z[f"grad{t}"], z["row_exp"], z["col_exp"],
                                              z["v_row"], z["v_col"], z["sum_v_inv"], coh_pre, lr, eps,
                                              int(z[f"salt{t}"]))
        np.testing.assert_array_equal(packed, z[f"packed{t}"])
        np.testing.assert_array_equal(w, z[f"wbuf{t}"])
        np.testing.assert_array_equal(rm, z[f"rmax{t}"])
        np.testing.assert_array_equal(cm, z[f"cmax{t}"])
        if coh_pre is not None:
            np.testing.assert_array_equal(cp, z[f"coh_pre{t}"])
            coh_pre = cp


def random_state(rng, N, K, sf=4000, i8=120):
    sfv = rng.integers(-sf, sf + 1, (N, K), dtype=np.int64)
    ss = rng.integers(-i8, i8 + 1, (N, K), dtype=np.int64)
    vs = rng.integers(-i8, i8 + 1, (N, K), dtype=np.int64)
    return (((sfv & 0xFFFF) << 16) | ((ss & 0xFF) << 8) | (vs & 0xFF)).astype(np.uint32).view(np.int32)


@pytest.mark.parametrize("case", ["bare", "consol", "ratio", "wd_beta1", "sgd_mp", "notrust"])
@pytest.mark.parametrize("shape", [(256, 1024), (131, 520), (64, 72), (33, 65)])
def test_step_matches_oracle_random(pb, oracle_mod, case, shape):
    """Vector path (K % 8 == 0) and generic path (odd K), ragged row counts."""
    rng = np.random.default_rng(zlib.crc32(repr((case, shape)).encode()))
    N, K = shape
    z = load("step_" + case)
    P = params_of(z)
    lr, eps = lr_eps(z)
    packed = random_state(rng, N, K)
    grad = oracle_mod.f32_to_bf16(rng.normal(0, 1e-3, (N, K)).astype(np.float32))
    rexp = rng.integers(-5, 6, N).astype(np.int8)
    cexp = rng.integers(-3, 4, K).astype(np.int8)
    v_row = (rng.random(N) * 1e-4 + 1e-7).astype(np.float32)
    v_col = (rng.random(K) * 1e-4 + 1e-7).astype(np.float32)
    svi = np.array([1.0 / v_row.sum()], np.float32)
    coh_pre = rng.random((N, K)).astype(np.float32) if bool(z["cfg_cohpre"]) else None
    salt = int(rng.integers(-2**31, 2**31 - 1))
    row0 = 40000 if N == 131 else 0
    stats = torch.zeros(2, dtype=torch.float64, device=DEV)
    got = run_cuda_step(pb, P, packed, grad, rexp, cexp, v_row, v_col, svi, coh_pre, lr, eps, salt,
                        row0=row0, coh_stats=stats)
    ref_p = packed.copy()
    ref_w = np.zeros((N, K), np.uint16)
    ref_rm, ref_cm = np.zeros(N, np.int32), np.zeros(K, np.int32)
    ref_cp = coh_pre.copy() if coh_pre is not None else None
    ref_stats = np.zeros(2)
    oracle_mod.step(P, ref_p, grad, ref_w, rexp, cexp, ref_rm, ref_cm, v_row, v_col, svi, ref_cp,
                    lr, eps, salt, row0=row0, coh_stats=ref_stats)
    np.testing.assert_array_equal(got[0], ref_p)
    np.testing.assert_array_equal(got[1], ref_w)
    np.testing.assert_array_equal(got[2], ref_rm)
    np.testing.assert_array_equal(got[3], ref_cm)
    if ref_cp is not None:
        np.testing.assert_array_equal(got[4], ref_cp)
    s = stats.cpu().numpy()
    assert s[1] == ref_stats[1]
    if ref_stats[1] > 0:
        assert abs(s[0] - ref_stats[0]) <= 1e-5 * max(1.0, abs(ref_stats[0]))


@pytest.mark.parametrize("shape", [(1, 1), (37, 70), (128, 256), (300, 1000), (1024, 1024),
                                   (129, 4104), (2000, 24)])
def test_vhat_bit_exact(pb, oracle_mod, shape):
    rng = np.random.default_rng(shape[0] * 7 + shape[1])
    N, K = shape
    grad = oracle_mod.f32_to_bf16(rng.normal(0, 1e-2, (N, K)).astype(np.float32))
    v_row = (rng.random(N) * 1e-4).astype(np.float32)
    v_col = (rng.random(K) * 1e-4).astype(np.float32)
    vr_d, vc_d, svi_d = T(v_row), T(v_col), torch.ones(1, device=DEV)
    rm = torch.full((N,), 7, dtype=torch.int32, device=DEV)
    cm = torch.full((K,), 7, dtype=torch.int32, device=DEV)
    salt = pb._get_step_counter(DEV)
    s0 = int(salt.item())
    for _ in range(2):   # twice: the workspace counters must come back to zero
        pb.vhat_update(bf16(grad), vr_d, vc_d, svi_d, 0.999, row_max=rm, col_max=cm, bump_salt=True)
    torch.cuda.synchronize()
    vr, vc, svi = v_row.copy(), v_col.copy(), np.ones(1, np.float32)
    for _ in range(2):
        oracle_mod.vhat(grad, vr, vc, svi)
    np.testing.assert_array_equal(N_(vr_d), vr)
    np.testing.assert_array_equal(N_(vc_d), vc)
    np.testing.assert_array_equal(N_(svi_d), svi)
    assert int(rm.abs().sum()) == 0 and int(cm.abs().sum()) == 0
    assert int(salt.item()) == s0 + 2


@pytest.mark.parametrize("case", ["up", "down"])
def test_rebalance_matches_reference_golden(pb, case):
    z = load("rebalance_" + case)
    p, re, ce = T(z["init_packed"]), T(z["init_row_exp"]), T(z["init_col_exp"])
    seed = torch.tensor([int(z["seed0"]) - 1], dtype=torch.int32, device=DEV)
    for t in range(2):
        pb.rebalance_packed(p, re, ce, T(z["rmax"]), T(z["cmax"]), seed_buf=seed,
                            allow_tickdown=bool(z["allow_tickdown"]), bump_seed=True)
        torch.cuda.synchronize()
        assert int(seed.item()) == int(z[f"seed{t}"])
        np.testing.assert_array_equal(N_(p), z[f"packed{t}"])
        np.testing.assert_array_equal(N_(re), z[f"row_exp{t}"])
        np.testing.assert_array_equal(N_(ce), z[f"col_exp{t}"])


@pytest.mark.parametrize("shape,td", [((512, 768), False), ((97, 130), True), ((300, 256), True)])
def test_rebalance_matches_oracle_random(pb, oracle_mod, shape, td):
    rng = np.random.default_rng(shape[0])
    N, K = shape
    packed = random_state(rng, N, K, sf=30000, i8=127 if not td else 20)
    rexp = rng.integers(-7, 6, N).astype(np.int8)
    cexp = rng.integers(-7, 6, K).astype(np.int8)
    rmax = np.where(rng.random(N) < 0.2, rng.integers(24001, 40000, N), rng.integers(0, 24001, N)).astype(np.int32)
    cmax = np.where(rng.random(K) < 0.2, rng.integers(24001, 40000, K), rng.integers(0, 24001, K)).astype(np.int32)
    hr, hc = rng.integers(0, 30000, N).astype(np.int32), rng.integers(0, 30000, K).astype(np.int32)
    p, re, ce, hr_d, hc_d = T(packed), T(rexp), T(cexp), T(hr), T(hc)
    seed = torch.tensor([123], dtype=torch.int32, device=DEV)
    fired = torch.zeros(1, dtype=torch.int32, device=DEV)
    pb.rebalance_packed(p, re, ce, T(rmax), T(cmax), seed_buf=seed, allow_tickdown=td,
                        row_hwm=hr_d, col_hwm=hc_d, fired_out=fired, bump_seed=True)
    torch.cuda.synchronize()
    sd = np.array([123], np.int32)
    f = oracle_mod.rebalance(packed, rexp, cexp, rmax, cmax, hr, hc, sd, allow_tickdown=td)
    np.testing.assert_array_equal(N_(p), packed)
    np.testing.assert_array_equal(N_(re), rexp)
    np.testing.assert_array_equal(N_(ce), cexp)
    np.testing.assert_array_equal(N_(hr_d), hr)
    np.testing.assert_array_equal(N_(hc_d), hc)
    assert int(seed.item()) == int(sd[0]) and int(fired.item()) == f


def test_rebalance_no_fire_is_noop(pb):
    rng = np.random.default_rng(5)
    packed = random_state(rng, 64, 128)
    p = T(packed)
    z = torch.zeros(64, dtype=torch.int32, device=DEV)
    zc = torch.zeros(128, dtype=torch.int32, device=DEV)
    re, ce = torch.zeros(64, dtype=torch.int8, device=DEV), torch.zeros(128, dtype=torch.int8, device=DEV)
    fired = torch.ones(1, dtype=torch.int32, device=DEV)
    seed = torch.zeros(1, dtype=torch.int32, device=DEV)
    pb.rebalance_packed(p, re, ce, z, zc, seed_buf=seed, fired_out=fired, bump_seed=True)
    torch.cuda.synchronize()
    assert int(fired.item()) == 0 and int(seed.item()) == 1
    np.testing.assert_array_equal(N_(p), packed)


def test_quantize_materialize_match_reference(pb, oracle_mod):
    z = load("quantize")
    from concord_b200 import ConcordLinearPackedB
    N, K = z["W"].shape
    for ft in (False, True):
        tag = "ft" if ft else "base"
        layer = ConcordLinearPackedB(K, N, bias=False, device=DEV)
        (layer.load_weights_finetune if ft else layer.load_weights)(torch.from_numpy(z["W"]))
        np.testing.assert_array_equal(N_(layer.packed_w), z["packed_" + tag])
        np.testing.assert_array_equal(N_(layer.row_exp), z["row_exp_" + tag])
        np.testing.assert_array_equal(N_(layer.get_weight()), z["get_weight_" + tag])
        np.testing.assert_array_equal(N_(layer.consolidated_weight()), z["consolidated_" + tag])
        np.testing.assert_array_equal(N_(layer.weight), z["get_weight_" + tag])


def test_coherence_meter(pb, oracle_mod):
    z = load("coherence_rng")
    from concord_b200.packed_b import coherence_sum

    class L:
        pass
    lay = L()
    lay.packed_w = T(z["coh_packed"])
    lay.drift_cancel_C = float(z["coh_C"])
    assert abs(pb.measure_coherence(lay) - float(z["coh_mean"])) < 1e-6
    s = coherence_sum(lay.packed_w, float(z["coh_C"])).cpu().numpy()
    ref = oracle_mod.coherence(z["coh_packed"], float(z["coh_C"]))
    assert s[1] == ref[1] and abs(s[0] - ref[0]) < 1e-9 * ref[1]


@pytest.mark.parametrize("lr", [5e-5, 0.05, 2.0])
def test_step_across_lr_scales(pb, oracle_mod, lr):
    """From tiny to huge |delta_t| (lr 5e-5 .. 2): SR ticks of every size and
    the step clamp must stay bit-exact."""
    rng = np.random.default_rng(int(lr * 1e5) + 7)
    N, K = 300, 512
    z = load("step_bare")
    P = params_of(z)
    packed = random_state(rng, N, K)
    grad = oracle_mod.f32_to_bf16(rng.normal(0, 1e-2, (N, K)).astype(np.float32))
    rexp = rng.integers(-6, 3, N).astype(np.int8)
    cexp = rng.integers(-2, 3, K).astype(np.int8)
    v_row = (rng.random(N) * 1e-4 + 1e-7).astype(np.float32)
    v_col = (rng.random(K) * 1e-4 + 1e-7).astype(np.float32)
    svi = np.array([1.0 / v_row.sum()], np.float32)
    coh_pre = rng.random((N, K)).astype(np.float32)
    got = run_cuda_step(pb, P, packed, grad, rexp, cexp, v_row, v_col, svi, coh_pre, lr, 1e-10, 99)
    ref_p, ref_w = packed.copy(), np.zeros((N, K), np.uint16)
    ref_rm, ref_cm, ref_cp = np.zeros(N, np.int32), np.zeros(K, np.int32), coh_pre.copy()
    oracle_mod.step(P, ref_p, grad, ref_w, rexp, cexp, ref_rm, ref_cm, v_row, v_col, svi, ref_cp,
                    lr, 1e-10, 99)
    np.testing.assert_array_equal(got[0], ref_p)
    np.testing.assert_array_equal(got[1], ref_w)
    np.testing.assert_array_equal(got[2], ref_rm)
    np.testing.assert_array_equal(got[3], ref_cm)
    np.testing.assert_array_equal(got[4], ref_cp)
