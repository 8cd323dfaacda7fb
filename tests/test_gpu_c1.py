"""BASELINE config 1 on the GPU: one 1024x1024 layer, 200 steps.

W0 ~ N(0, 0.02); per step G_t = N(0, 1e-3) noise + a fixed rank-4 drift
(U, V ~ N(0, 1e-4)), rounded to bf16; lr = 5e-4; seed 0.  A step is the
optimizer half of the backward (v-hat + packed step) followed by rebalance().

Arm (i), bare defaults (coherence gate on): the CUDA words, exponents and
consolidated weight equal the CPU oracle's bit for bit after every step.
Arm (ii), gate off (disable_cohpre): bit-exact against the oracle as well, and
the consolidated (deploy) weight tracks the real-valued update rule of the
reference's CPU experiments (experiments/cpu_dynamics/concord_ref.py) within
the statistical tolerance of stochastic rounding: correlation >= 0.995 and
relative Frobenius error <= 8 % (measured: 0.9988 and 5.0 %).
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
N = K = 1024
STEPS = 200


def _inputs():
    g = torch.Generator().manual_seed(0)
    W0 = torch.randn(N, K, generator=g) * 0.02
    U = torch.randn(N, 4, generator=g) * 1e-4
    V = torch.randn(K, 4, generator=g) * 1e-4
    return g, W0, U, V


@pytest.mark.parametrize("gate", [True, False])
def test_config1_trajectory(oracle_mod, gate):
    from concord_b200 import ConcordLinearPackedB, packed_b
    from oracle.realvalued import RealValuedRule
    O = oracle_mod
    g, W0, U, V = _inputs()
    layer = ConcordLinearPackedB(K, N, bias=False, device="cuda", lr=5e-4)
    layer.load_weights(W0)
    if not gate:
        layer.disable_cohpre()
    packed, rexp, cexp = O.quantize(W0.numpy())
    np.testing.assert_array_equal(layer.packed_w.cpu().numpy(), packed)
    vr, vc, svi = np.zeros(N, np.float32), np.zeros(K, np.float32), np.ones(1, np.float32)
    coh = np.ones((N, K), np.float32) if gate else None
    hr, hc, seed = np.zeros(N, np.int32), np.zeros(K, np.int32), np.zeros(1, np.int32)
    P = packed_b.adamw_params(v_scale=0.0, precond_p=0.5, drift_cancel_C=layer.drift_cancel_C,
                              mass_preserve=True, gf_trust_delta_sq=1.0, use_cohpre=gate)
    ref = RealValuedRule(W0, lr=5e-4)
    salt = packed_b._get_step_counter(layer.packed_w.device)
    threads = max(1, min(32, len(os.sched_getaffinity(0))))
    for t in range(STEPS):
        G = torch.randn(N, K, generator=g) * 1e-3 + U @ V.T
        gb = O.f32_to_bf16(G.numpy())
        s0 = int(salt.item())
        layer.optimizer_step(torch.from_numpy(gb.view(np.int16)).view(torch.bfloat16).cuda())
        layer.rebalance()
        O.vhat(gb, vr, vc, svi)
        w = np.zeros((N, K), np.uint16)
        rm, cm = np.zeros(N, np.int32), np.zeros(K, np.int32)
        O.step_threaded(P, packed, gb, w, rexp, cexp, rm, cm, vr, vc, svi, coh, 5e-4, 1e-10,
                        s0 + 1, threads=threads)
        O.rebalance(packed, rexp, cexp, rm, cm, hr, hc, seed)
        if not gate:
            ref.step(torch.from_numpy(O.bf16_to_f32(gb).copy()))
        if t in (0, 1, 9, 49, 99, STEPS - 1):
            np.testing.assert_array_equal(layer.packed_w.cpu().numpy(), packed, err_msg=f"step {t}")
            np.testing.assert_array_equal(layer.row_exp.cpu().numpy(), rexp, err_msg=f"step {t}")
            np.testing.assert_array_equal(layer.v_row.cpu().numpy(), vr)
    dep = layer.consolidated_weight().view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(dep, O.materialize(packed, rexp, cexp, consolidated=True))
    assert int(np.abs(rexp.astype(int) - O.quantize(W0.numpy())[1]).sum()) > 0, "rebalance never fired"
    if not gate:
        a = O.bf16_to_f32(dep).reshape(N, K)
        b = ref.deploy().numpy()
        corr = np.corrcoef(a.ravel(), b.ravel())[0, 1]
        rel = np.linalg.norm(a - b) / np.linalg.norm(b)
        assert corr >= 0.995 and rel <= 0.08, (corr, rel)
