"""CPU-only checks: the C-ABI library loads and exports what the header
declares, the host-side math and launch-scalar rules, and the ports of the
reference's CPU tests (experiments/cpu_dynamics/test_autotuner_parity.py)."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def built():
    from concord_b200 import build
    build.build()
    return build


def test_library_exports_header_symbols(built):
    from concord_b200 import _abi
    hdr = open(os.path.join(ROOT, "include", "concord_b200.h")).read()
    declared = set(re.findall(r"\b(concord_[a-z0-9_]+)\s*\(", hdr))
    lib = ctypes.CDLL(_abi.LIB_PATH)
    for name in sorted(declared):
        assert hasattr(lib, name), name
    out = subprocess.check_output(["nm", "-D", "--defined-only", _abi.LIB_PATH]).decode()
    exported = set(re.findall(r" T (concord_[a-z0-9_]+)", out))
    assert declared == exported
    assert declared == set(_abi.EXPORTED)
    _abi.load()
    assert _abi.load().concord_abi_version() == _abi.ABI_VERSION == 4


def test_gemm_dw_split_decision(built):
    """A dW with fewer output tiles than SMs and a long reduction reserves
    fp32 partials for its split (S * N * K * 4 bytes of workspace); the C2
    Linear shapes do not split."""
    from concord_b200 import _abi
    ws = _abi.load().concord_gemm_workspace_bytes
    assert ws(8192, 320, 2880) >= 8 * 320 * 2880 * 4       # 36 tiles: 8 slices
    assert ws(4096, 64, 1024) >= 4 * 64 * 1024 * 4         # 4 tiles, 1024-row slices
    assert ws(16384, 1280, 1280) >= 2 * 1280 * 1280 * 4    # 50 tiles: 2 slices
    assert ws(512, 1280, 1280) < 1280 * 1280 * 4           # reduction too short
    assert ws(8192, 10240, 2048) < 10240 * 2048 * 4        # 640 tiles


def test_crmath_host_matches_extended_precision(built):
    lib = ctypes.CDLL(os.path.join(ROOT, "concord_b200", "_lib", "libcrmath_check.so"))
    rng = np.random.default_rng(1)

    def run(fn, x, slow):
        y = np.empty_like(x)
        getattr(lib, fn)(x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p),
                         ctypes.c_long(x.size), ctypes.c_int(slow))
        return y
    x = rng.integers(1, 0x7f800000, size=300_000, dtype=np.uint32).view(np.float32)
    x = np.concatenate([x, np.array([1.0, 2.0, 0.5, 1e-10, 1.0000001, 0.99999994], np.float32)])
    ref = np.log2(x.astype(np.longdouble)).astype(np.float32)
    for slow in (0, 1):
        np.testing.assert_array_equal(run("crm_log2f_v", x, slow), ref)
    y = np.concatenate([(rng.random(300_000) * 300 - 160).astype(np.float32),
                        np.arange(-160, 130, dtype=np.float32),
                        (rng.random(20000) * 2 - 151).astype(np.float32)])
    with np.errstate(over="ignore"):
        ref = np.exp2(y.astype(np.longdouble)).astype(np.float32)
    for slow in (0, 1):
        np.testing.assert_array_equal(run("crm_exp2f_v", y, slow), ref)


def test_crmath_agrees_with_oracle(built, oracle_mod):
    lib = ctypes.CDLL(os.path.join(ROOT, "concord_b200", "_lib", "libcrmath_check.so"))
    lib.crm_log2f.restype = ctypes.c_float
    lib.crm_log2f.argtypes = [ctypes.c_float]
    lib.crm_exp2f.restype = ctypes.c_float
    lib.crm_exp2f.argtypes = [ctypes.c_float]
    o = oracle_mod.lib()
    rng = np.random.default_rng(2)
    for v in rng.random(2000) * 1e-3:
        assert lib.crm_log2f(float(v)) == o.oracle_log2f(float(v))
        assert lib.crm_exp2f(float(v * -3e4)) == o.oracle_exp2f(float(v * -3e4))


def test_drift_cancel_C():
    from concord_b200 import compute_drift_cancel_C
    assert abs(compute_drift_cancel_C(0.1, 0.001) - 0.018036) < 1e-6
    assert abs(compute_drift_cancel_C(0.1, 0.001, mass_preserve=False) - 9 * 0.001 / (1 - 0.009)) < 1e-12


def test_step_params_fold_host_scalars_in_double():
    from concord_b200._abi import F_COHPRE, F_GF_CONSOL, F_GF_TRUST, make_step_params
    p = make_step_params(alpha=0.1, gate_gain=0.7, chase_floor=0.9, alpha_v_fast=0.001,
                         gf_trust_delta_sq=1.0, use_cohpre=True)
    f32 = lambda v: float(np.float32(v))  # noqa: E731
    assert p.one_minus_chase_floor == f32(1.0 - 0.9)           # not 1 - fp32(0.9)
    assert p.one_minus_chase_floor != f32(1.0 - f32(0.9))
    assert p.alpha_gate_gain == f32(0.1 * 0.7)
    assert p.one_minus_alpha_v_fast == f32(1.0 - 0.001)
    assert p.flags & F_GF_TRUST and p.flags & F_COHPRE and not p.flags & F_GF_CONSOL


def test_cpu_tensors_rejected():
    from concord_b200 import ConcordLinearPackedB
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ConcordLinearPackedB(8, 4, device="cpu")


# ---- port of experiments/cpu_dynamics/test_autotuner_parity.py ----
def _torch_meter(layer):
    from concord_b200 import gate_coherence_from_fields
    p = layer.packed_w
    return float(gate_coherence_from_fields((p >> 16).float(), ((p << 16) >> 24).float(),
                                            ((p << 24) >> 24).float(), float(layer.drift_cancel_C)).mean())


def test_autotuner_parity():
    from concord_b200 import DissipationAutoTuner, gate_coherence_from_fields
    torch.manual_seed(0)
    N, K, C = 64, 96, 0.018036
    s_fast = torch.randint(-2000, 2000, (N, K)).float()
    s_slow = torch.randint(-128, 128, (N, K)).float()
    v_slow = torch.randint(-128, 128, (N, K)).float()
    coh_pkg = gate_coherence_from_fields(s_fast, s_slow, v_slow, C)
    for _ in range(3):
        re_ = torch.randint(-8, 8, (N, 1)).float()
        ce_ = torch.randint(-8, 8, (1, K)).float()
        scale = torch.exp2(re_ + ce_ - 15)
        u, S, A = s_fast * scale, 128.0 * s_slow * scale, 128.0 * v_slow * scale
        mu = C * (S - A)
        nse = u - mu
        coh_ref = (mu * mu) / (mu * mu + nse * nse + 1e-30)
        assert torch.allclose(coh_pkg, coh_ref, atol=1e-5)
    packed = (((s_fast.int() & 0xFFFF) << 16) | ((s_slow.int() & 0xFF) << 8) | (v_slow.int() & 0xFF))

    class FakeLayer:
        def __init__(self):
            self.packed_w = packed
            self.drift_cancel_C = C
            self.gf_consol = 0.0
    assert abs(_torch_meter(FakeLayer()) - float(coh_pkg.mean())) < 1e-6
    TABLE = [(0.387, 0.0), (0.314, 100.0), (0.288, 200.0), (0.274, 400.0), (0.256, 400.0)]
    layers = [FakeLayer(), FakeLayer()]
    tuner = DissipationAutoTuner(layers, 10, 50, TABLE, probe_kappa=50.0, measure_every=10,
                                 verbose=False, meter=_torch_meter)
    assert all(m.gf_consol == 50.0 for m in layers)
    committed = None
    for t in range(60):
        r = tuner.step(t)
        if r is not None:
            committed = (t, r)
    assert committed is not None and committed[0] == 50
    assert all(m.gf_consol == committed[1] for m in layers)
    assert abs(committed[1] - tuner.kappa_from_coh(float(coh_pkg.mean()))) < 1e-9
    probe_coh = float(coh_pkg.mean())
    assert tuner.committed_beta1 == (0.1 if probe_coh >= 0.35 else 0.0)
    lo = DissipationAutoTuner([FakeLayer()], 0, 5, TABLE, verbose=False, beta1_coh_threshold=0.0,
                              meter=_torch_meter)
    assert all(m.beta1 == 0.0 for m in lo.layers)
    for t in range(6):
        lo.step(t)
    assert lo.committed_beta1 == 0.1 and lo.layers[0].beta1 == 0.1
    off = DissipationAutoTuner([FakeLayer()], 0, 5, TABLE, verbose=False, beta1_on=0.0,
                               meter=_torch_meter)
    for t in range(6):
        off.step(t)
    assert off.committed_beta1 == 0.0
    F_TABLE = [(0.387, 0.0), (0.314, 0.1), (0.288, 0.2), (0.274, 0.4), (0.256, 0.4)]
    fu = DissipationAutoTuner([FakeLayer()], 0, 5, F_TABLE, verbose=False, probe_kappa=0.05,
                              peak_lr=1e-3, beta1_on=0.0, meter=_torch_meter)
    assert abs(fu.probe_kappa - 50.0) < 1e-9 and abs(fu.table[3][1] - 400.0) < 1e-9
    assert tuner.kappa_from_coh(0.50) == 0.0 and tuner.kappa_from_coh(0.20) == 400.0
    assert 100.0 < tuner.kappa_from_coh(0.301) < 200.0


def test_autotuner_table_interpolation():
    """kappa_from_coh is the table's piecewise-linear interpolant, flat beyond
    its ends; peak_lr turns F = lr * kappa units into kappa."""
    from concord_b200 import DissipationAutoTuner
    TABLE = [(0.387, 0.0), (0.314, 100.0), (0.288, 200.0), (0.274, 400.0), (0.256, 400.0)]
    tu = DissipationAutoTuner([], 0, 1, TABLE, verbose=False)
    assert tu.kappa_from_coh(0.5) == 0.0 and tu.kappa_from_coh(0.1) == 400.0
    for (c1, k1), (c2, k2) in zip(TABLE, TABLE[1:]):
        for f in (0.0, 0.25, 0.5, 1.0):
            c = c1 + f * (c2 - c1)
            assert abs(tu.kappa_from_coh(c) - (k1 + f * (k2 - k1))) < 1e-9
    tu = DissipationAutoTuner([], 0, 1, TABLE, probe_kappa=0.5, verbose=False, peak_lr=1e-3)
    assert abs(tu.probe_kappa - 500.0) < 1e-9
    assert abs(tu.kappa_from_coh(0.301) - 150.0 * 1e3) < 1e-6
    with pytest.raises(AssertionError):
        DissipationAutoTuner([], 0, 1, TABLE[::-1], verbose=False)
    with pytest.raises(AssertionError):
        DissipationAutoTuner([], 5, 5, TABLE, verbose=False)
