"""Gradient accumulation gate, device-tensor ratio floors and Sigma_g noise.

The gate follows the reference's prototype kernel
(notebook/src/prototype_packed_b.py:481-515, 661-782): with
*consolidate == 0 the SR tick of this micro-batch's gradient still lands in
s_fast, while the beta1/evaporation terms, the chase, the leak and the weight
decays are multiplied by 0 and the bf16 weight and the rebalance maxima are
not written; with 1 the step is the ordinary one, bit for bit.  The CUDA
kernel (which reads the flag and the floors from device memory) is compared
with the CPU oracle given the same values.
"""
import zlib

import numpy as np
import pytest
import torch

from golden_util import load, lr_eps, params_of
from test_gpu_parity import N_, T, bf16, random_state

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def pb():
    from concord_b200 import packed_b
    packed_b._lib()
    return packed_b


def _copy(P):
    from concord_b200._abi import StepParams
    Q = StepParams()
    ctypes_fields = [f for f, _ in StepParams._fields_]
    for f in ctypes_fields:
        setattr(Q, f, getattr(P, f))
    return Q


@pytest.mark.parametrize("case", ["bare", "consol", "ratio", "wd_beta1"])
@pytest.mark.parametrize("cons", [0, 1])
@pytest.mark.parametrize("shape", [(131, 520), (33, 65)])
def test_consolidate_gate_matches_oracle(pb, oracle_mod, case, cons, shape):
    rng = np.random.default_rng(zlib.crc32(repr((case, cons, shape)).encode()))
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
    floors_h = np.array([0.8, 0.95], np.float32)
    cons_h = np.array([cons], np.int32)
    cons_d = torch.tensor([cons], dtype=torch.int32, device=DEV)
    floors_d = T(floors_h)
    Pd, Ph = _copy(P), _copy(P)
    Pd.consolidate, Ph.consolidate = cons_d.data_ptr(), cons_h.ctypes.data
    if case == "ratio":
        Pd.ratio_floors, Ph.ratio_floors = floors_d.data_ptr(), floors_h.ctypes.data

    p, w = T(packed), torch.zeros(N, K, dtype=torch.bfloat16, device=DEV)
    rm, cm = torch.zeros(N, dtype=torch.int32, device=DEV), torch.zeros(K, dtype=torch.int32, device=DEV)
    cp = T(coh_pre) if coh_pre is not None else None
    pb._step_launch(Pd, p, bf16(grad), w, T(rexp), T(cexp), rm, cm, T(v_row), T(v_col), T(svi), cp,
                    torch.tensor([lr], device=DEV), torch.tensor([eps], device=DEV),
                    torch.tensor([salt], dtype=torch.int32, device=DEV))
    torch.cuda.synchronize()
    ref_p, ref_w = packed.copy(), np.zeros((N, K), np.uint16)
    ref_rm, ref_cm = np.zeros(N, np.int32), np.zeros(K, np.int32)
    ref_cp = coh_pre.copy() if coh_pre is not None else None
    oracle_mod.step(Ph, ref_p, grad, ref_w, rexp, cexp, ref_rm, ref_cm, v_row, v_col, svi, ref_cp,
                    lr, eps, salt)
    np.testing.assert_array_equal(N_(p), ref_p)
    np.testing.assert_array_equal(N_(w), ref_w)
    np.testing.assert_array_equal(N_(rm), ref_rm)
    np.testing.assert_array_equal(N_(cm), ref_cm)
    if ref_cp is not None:
        np.testing.assert_array_equal(N_(cp), ref_cp)
    if cons == 0:
        # tick-only: slow accumulators untouched, weight and maxima not written
        assert np.array_equal(ref_p & 0xFFFF, packed & 0xFFFF)
        assert not ref_w.any() and not ref_rm.any() and not ref_cm.any()
    else:
        # consolidate == 1 through the flag == the step without it
        q, w2 = T(packed), torch.zeros(N, K, dtype=torch.bfloat16, device=DEV)
        rm2, cm2 = torch.zeros_like(rm), torch.zeros_like(cm)
        cp2 = T(coh_pre) if coh_pre is not None else None
        P0 = _copy(P)
        if case != "ratio":   # (with device floors the host-floor step differs by design)
            pb._step_launch(P0, q, bf16(grad), w2, T(rexp), T(cexp), rm2, cm2, T(v_row), T(v_col), T(svi),
                            cp2, torch.tensor([lr], device=DEV), torch.tensor([eps], device=DEV),
                            torch.tensor([salt], dtype=torch.int32, device=DEV))
            torch.cuda.synchronize()
            np.testing.assert_array_equal(N_(q), ref_p)
            np.testing.assert_array_equal(N_(w2), ref_w)


def test_accumulation_cycle_on_a_layer(pb):
    """Three tick-only micro-steps and one consolidate step through the layer
    API: the forward weight stays frozen until the consolidate step."""
    from concord_b200 import ConcordLinearPackedB, set_consolidate
    dev = torch.device(DEV)
    key = pb._dev_key(dev)
    torch.manual_seed(0)
    layer = ConcordLinearPackedB(256, 128, bias=False, device=DEV, lr=0.05)
    layer.load_weights(torch.randn(128, 256) * 0.05)
    try:
        w0 = layer._bf16_weight_buf.clone()
        p0 = layer.packed_w.clone()
        set_consolidate(dev, False)
        for t in range(3):
            g = (torch.randn(128, 256, generator=torch.Generator().manual_seed(t)) * 1e-2)
            layer.optimizer_step(g.to(torch.bfloat16).to(DEV))
        assert torch.equal(layer._bf16_weight_buf, w0)
        assert torch.equal(layer.packed_w & 0xFFFF, p0 & 0xFFFF)      # s_slow, v_slow frozen
        assert not torch.equal(layer.packed_w, p0)                      # s_fast accumulated
        assert int(layer._row_max_buf.abs().sum()) == 0
        set_consolidate(dev, True)
        layer.optimizer_step((torch.randn(128, 256) * 1e-2).to(torch.bfloat16).to(DEV))
        assert not torch.equal(layer._bf16_weight_buf, w0)
        assert int(layer._row_max_buf.max()) > 0
    finally:
        pb._CONSOLIDATE_FLAGS.pop(key, None)   # back to the kernel without the flag


@pytest.mark.parametrize("iso", [False, True])
def test_sigmag_noise(pb, iso):
    from concord_b200.packed_b import set_sigmag_noise, set_sigmag_sigma, sigmag_noise
    g = torch.Generator(device="cpu").manual_seed(3)
    gy = torch.randn(512, 96, generator=g).to(torch.bfloat16).to(DEV)
    x = torch.randn(512, 64, generator=g).to(torch.bfloat16).to(DEV)
    gw = (gy.float().t() @ x.float()).to(torch.bfloat16)
    try:
        set_sigmag_noise(True, isotropic=iso)
        set_sigmag_sigma(0.0)
        assert torch.equal(sigmag_noise(gw, gy, x), gw)
        set_sigmag_sigma(0.25)
        out = sigmag_noise(gw, gy, x).float()
        rel = float((out - gw.float()).norm() / gw.float().norm())
        assert abs(rel - 0.25) < 0.01, rel
    finally:
        set_sigmag_noise(False)
        set_sigmag_sigma(0.0)


@pytest.mark.parametrize("case", ["bare", "consol", "ratio", "wd"])
def test_gate_matches_prototype_fixtures(pb, case):
    """The CUDA gate against the reference's prototype kernel itself
    (tests/golden/make_golden_accum.py), micro-step by micro-step."""
    import ctypes
    from concord_b200 import _abi
    from test_oracle_accum import replay_accum_fixture
    z = load("accum_" + case)
    lib = _abi.load()
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    rexp, cexp = dev(z["row_exp"]), dev(z["col_exp"])
    vr, vc, svi = dev(z["v_row"]), dev(z["v_col"]), dev(z["sum_v_inv"])
    flag_d = torch.zeros(1, dtype=torch.int32, device=DEV)
    floors_d = torch.zeros(2, dtype=torch.float32, device=DEV)
    lr_d, eps_d, salt_d = (torch.zeros(1, device=DEV), torch.zeros(1, device=DEV),
                           torch.zeros(1, dtype=torch.int32, device=DEV))
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def step(P, flag, floors, packed, grad, wbuf, rm, cm, coh, lr, eps, salt):
        flag_d.fill_(int(flag[0]))
        P.consolidate = flag_d.data_ptr()
        if floors is not None:
            floors_d.copy_(torch.from_numpy(floors))
            P.ratio_floors = floors_d.data_ptr()
        lr_d.fill_(lr)
        eps_d.fill_(eps)
        salt_d.fill_(salt)
        pk, w = dev(packed), dev(wbuf.view(np.int16))
        g = dev(grad.view(np.int16))
        rmd, cmd = dev(rm), dev(cm)
        cd = dev(coh) if coh is not None else None
        N, K = packed.shape
        rc = lib.concord_step(ctypes.byref(P), p(pk), K, p(g), K, p(w), K, p(rexp), p(cexp), p(rmd), p(cmd),
                              p(vr), p(vc), p(svi), p(cd), K, p(lr_d), p(eps_d), p(salt_d), N, K, 0, None,
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, lib.concord_last_error()
        torch.cuda.synchronize()
        packed[...] = pk.cpu().numpy()
        wbuf[...] = w.cpu().numpy().view(np.uint16)
        rm[...] = rmd.cpu().numpy()
        cm[...] = cmd.cpu().numpy()
        if coh is not None:
            coh[...] = cd.cpu().numpy()
    assert replay_accum_fixture(z, step) == []
