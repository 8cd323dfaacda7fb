"""End-to-end layer tests on the GPU: the module's self-stepping backward,
rebalance and salts against the CPU oracle, and the reference's own
regression checks (concord/test_baked_defaults.py)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"


def N_(t):
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def test_mlp_backward_matches_oracle(oracle_mod):
    """Two stacked layers, 6 steps with a large lr so rebalance fires: every
    step's words, exponents, weights, coh_pre and v-hat equal the oracle's fed
    the same bf16 dW (captured from the GEMM), in reverse layer order."""
    from concord_b200 import ConcordLinearPackedB, packed_b
    torch.manual_seed(0)
    l1 = ConcordLinearPackedB(96, 64, bias=True, device=DEV, lr=0.05)
    l2 = ConcordLinearPackedB(64, 40, bias=False, device=DEV, lr=0.05)
    layers = [l1, l2]
    orc = []
    for l in layers:
        orc.append(dict(packed=N_(l.packed_w).copy(), rexp=N_(l.row_exp).copy(),
                        cexp=N_(l.col_exp).copy(), v_row=np.zeros(l.out_features, np.float32),
                        v_col=np.zeros(l.in_features, np.float32), svi=np.ones(1, np.float32),
                        coh=np.ones((l.out_features, l.in_features), np.float32),
                        hr=np.zeros(l.out_features, np.int32), hc=np.zeros(l.in_features, np.int32),
                        seed=np.zeros(1, np.int32)))
    captured = []
    orig = packed_b._gemm.grad_weight

    def spy(gy, x):
        g = orig(gy, x)
        captured.append(N_(g).copy())
        return g
    packed_b._gemm.grad_weight = spy
    salt = packed_b._get_step_counter(DEV)
    fired_any = 0
    try:
        for step in range(6):
            captured.clear()
            s0 = int(salt.item())
            x = torch.randn(32, 96, device=DEV)
            y = l2(torch.relu(l1(x)))
            loss = (y.float() ** 2).mean()
            loss.backward()
            fired = torch.zeros(2, dtype=torch.int32, device=DEV)
            for i, l in enumerate(layers):
                l.rebalance(fired_out=fired[i:i + 1])
            torch.cuda.synchronize()
            fired_any += int(fired.sum())
            # backward runs l2 then l1: salts s0+1, s0+2
            for li, g, sl in ((1, captured[0], s0 + 1), (0, captured[1], s0 + 2)):
                o, l = orc[li], layers[li]
                oracle_mod.vhat(g, o["v_row"], o["v_col"], o["svi"])
                w = np.zeros_like(g)
                rm = np.zeros(l.out_features, np.int32)
                cm = np.zeros(l.in_features, np.int32)
                P = packed_b.adamw_params(alpha=0.1, v_scale=0.0, precond_p=0.5,
                                          drift_cancel_C=l.drift_cancel_C, mass_preserve=True,
                                          gf_trust_delta_sq=1.0, use_cohpre=True)
                oracle_mod.step(P, o["packed"], g, w, o["rexp"], o["cexp"], rm, cm, o["v_row"],
                                o["v_col"], o["svi"], o["coh"], 0.05, 1e-10, sl)
                np.testing.assert_array_equal(N_(l.v_row), o["v_row"])
                np.testing.assert_array_equal(N_(l._sum_v_inv), o["svi"])
                np.testing.assert_array_equal(N_(l._coh_pre), o["coh"])
                np.testing.assert_array_equal(N_(l.weight), w)
                oracle_mod.rebalance(o["packed"], o["rexp"], o["cexp"], rm, cm, o["hr"], o["hc"],
                                     o["seed"])
                np.testing.assert_array_equal(N_(l.packed_w), o["packed"], err_msg=f"step {step} layer {li}")
                np.testing.assert_array_equal(N_(l.row_exp), o["rexp"])
                np.testing.assert_array_equal(N_(l.col_exp), o["cexp"])
                np.testing.assert_array_equal(N_(l._row_max_hwm), o["hr"])
            assert int(salt.item()) == s0 + 2
    finally:
        packed_b._gemm.grad_weight = orig
    assert fired_any > 0, "the test is meant to exercise rebalance"


def test_baked_defaults_and_trains():
    """Port of concord/test_baked_defaults.py (reference regression)."""
    import concord_b200.packed_b as ppb
    from concord_b200 import ConcordConv2dPackedB, ConcordLinearPackedB
    assert ppb._USE_FIXED_COH is True
    for m in (ConcordLinearPackedB(64, 128, bias=False, device=DEV),
              ConcordConv2dPackedB(3, 16, 3, padding=1, bias=False, device=DEV)):
        assert m.optimizer_kind == 'adamw'
        assert abs(m._eps_value - 1e-10) < 1e-20
        assert m.v_scale == 0.0 and m.gf_trust_delta_sq == 1.0 and m.precond_p == 0.5
        assert m._coh_pre is not None and m._coh_pre.shape == m.packed_w.shape
    torch.manual_seed(1)
    W = ConcordLinearPackedB(32, 32, bias=False, device=DEV)
    W.lr = 0.02
    tgt = torch.randn(32, 32, device=DEV) * 0.3
    x = torch.randn(256, 32, device=DEV)
    y = x @ tgt.T
    losses = []
    for _ in range(80):
        loss = F.mse_loss(W(x.detach().requires_grad_(True)), y)
        loss.backward()
        W.rebalance()
        losses.append(loss.item())
    assert losses[-1] < 0.9 * losses[0], losses[::10]
    W.disable_cohpre()
    assert W._coh_pre is None
    loss = F.mse_loss(W(x.detach().requires_grad_(True)), y)
    loss.backward()
    W.rebalance()
    torch.cuda.synchronize()


def test_conv2d_layer_steps():
    from concord_b200 import ConcordConv2dPackedB
    torch.manual_seed(2)
    c = ConcordConv2dPackedB(4, 8, 3, padding=1, device=DEV, lr=0.01)
    before = c.packed_w.clone()
    x = torch.randn(2, 4, 10, 10, device=DEV, requires_grad=True)
    y = c(x)
    assert y.shape == (2, 8, 10, 10)
    y.float().pow(2).mean().backward()
    assert x.grad is not None and c.bias.grad is not None
    assert not torch.equal(before, c.packed_w)


def test_state_dict_keys_match_reference():
    from concord_b200 import ConcordLinearPackedB
    keys = set(ConcordLinearPackedB(8, 4, device=DEV).state_dict().keys())
    assert keys == {"_reb_seed", "packed_w", "row_exp", "col_exp", "v_row", "v_col", "_sum_v_inv",
                    "_row_max_hwm", "_col_max_hwm", "_lr_buf", "_eps_buf", "bias"}

