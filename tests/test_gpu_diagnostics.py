"""The reference's two optional diagnostics, computed on the GPU: the
rebalance statistics (counted by the rebalance launch) and the garbage
fraction summary (one kernel pass), each against a torch restatement of its
definition (concord/packed_b.py:1161-1179 and 1676-1730)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _state(g, N, K):
    sf = torch.randint(-3000, 3001, (N, K), generator=g, dtype=torch.int32)
    ss = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int32)
    vs = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int32)
    # small int8 fields in the first rows/columns so the lower medians allow tick-downs
    ss[:8] //= 8
    vs[:8] //= 8
    ss[:, :6] //= 8
    vs[:, :6] //= 8
    return ((sf & 0xFFFF) << 16) | ((ss & 0xFF) << 8) | (vs & 0xFF)


def _expected_reb_stats(packed, rexp, cexp, rmax, cmax, MAX_M, EXP_MAX, EXP_MIN):
    """The statistics' definition, evaluated on the pre-rebalance state."""
    ss = (packed << 16) >> 24
    vs = (packed << 24) >> 24
    mag = torch.maximum(ss.abs(), vs.abs())
    re, ce = rexp.int(), cexp.int()
    up_r, up_c = (rmax > MAX_M) & (re < EXP_MAX), (cmax > MAX_M) & (ce < EXP_MAX)
    med_r = mag.median(dim=1).values
    med_c = mag.median(dim=0).values
    dn_r = (rmax <= MAX_M) & (med_r <= 31) & (re > EXP_MIN)
    dn_c = (cmax <= MAX_M) & (med_c <= 31) & (ce > EXP_MIN)
    net = (up_r.int() - dn_r.int())[:, None] + (up_c.int() - dn_c.int())[None, :]
    lsh = (-net).clamp(min=0)
    clip = int(((mag << lsh) > 127).sum())
    return dict(tickup_dim=int(up_r.sum() + up_c.sum()), tickdown_dim=int(dn_r.sum() + dn_c.sum()),
                clip_elems=clip)


def test_rebalance_stats_counted_on_gpu():
    from concord_b200 import ConcordLinearPackedB, get_reb_stats, reset_reb_stats
    g = torch.Generator().manual_seed(3)
    N, K = 96, 160
    layer = ConcordLinearPackedB(K, N, bias=False, device=DEV)
    layer.allow_tickdown = True
    assert get_reb_stats() is None or isinstance(get_reb_stats(), dict)
    reset_reb_stats()
    want = dict(tickup_dim=0, tickdown_dim=0, clip_elems=0)
    for call in range(3):
        packed = _state(g, N, K)
        rexp = torch.randint(-3, 5, (N,), generator=g, dtype=torch.int8)
        cexp = torch.randint(-2, 3, (K,), generator=g, dtype=torch.int8)
        rmax = torch.randint(0, 30000, (N,), generator=g, dtype=torch.int32)
        cmax = torch.randint(0, 30000, (K,), generator=g, dtype=torch.int32)
        e = _expected_reb_stats(packed, rexp, cexp, rmax, cmax, layer.MAX_M, layer.EXP_MAX, layer.EXP_MIN)
        assert e["tickdown_dim"] > 0 and e["tickup_dim"] > 0 and e["clip_elems"] > 0
        for k in want:
            want[k] += e[k]
        layer.packed_w.copy_(packed.to(DEV))
        layer.row_exp.copy_(rexp.to(DEV))
        layer.col_exp.copy_(cexp.to(DEV))
        layer._ensure_buffers()
        layer._row_max_buf.copy_(rmax.to(DEV))
        layer._col_max_buf.copy_(cmax.to(DEV))
        layer.rebalance()
    st = get_reb_stats()
    assert st["calls"] == 3 and st["dim_total"] == 3 * (N + K) and st["elem_total"] == 3 * N * K
    for k, v in want.items():
        assert st[k] == v, (k, st[k], v)
    reset_reb_stats()
    assert get_reb_stats()["tickup_dim"] == 0


def test_garbage_fraction_stats():
    from concord_b200 import ConcordLinearPackedB
    g = torch.Generator().manual_seed(5)
    N, K = 200, 328
    layer = ConcordLinearPackedB(K, N, bias=False, device=DEV)
    assert layer.get_garbage_fraction_stats() is None    # v-hat not populated yet
    layer.packed_w.copy_(_state(g, N, K).to(DEV))
    layer.row_exp.copy_(torch.randint(-3, 5, (N,), generator=g, dtype=torch.int8).to(DEV))
    layer.col_exp.copy_(torch.randint(-2, 3, (K,), generator=g, dtype=torch.int8).to(DEV))
    # v-hat spread over six decades so both tails of the garbage fraction fill
    layer.v_row.copy_((torch.rand(N, generator=g) + 0.5).to(DEV))
    layer.v_col.copy_(torch.pow(10.0, torch.rand(K, generator=g) * 6 - 3).to(DEV))
    st = layer.get_garbage_fraction_stats()
    # the definition in torch (fp32, the same operation order)
    p = layer.packed_w
    s_fast = (p >> 16).float()
    d_sv = ((p << 16) >> 24).float() * 128.0 - ((p << 24) >> 24).float() * 128.0
    noise = s_fast - float(layer.drift_cancel_C) * d_sv
    scale = torch.pow(2.0, layer.row_exp[:, None].float() + layer.col_exp[None, :].float() - 15)
    var_w = (noise * scale) ** 2
    sv = layer.v_row.float().sum().clamp(min=1e-30)
    v_hat = layer.v_row[:, None] * layer.v_col[None, :] / sv
    gf = (var_w / (v_hat + 1e-30)).clamp(0.0, 1.0).flatten()
    q = torch.quantile(gf, torch.tensor([0.25, 0.5, 0.75], device=DEV))
    assert 0.05 < st["frac_signal_dominated"] and 0.05 < st["frac_noise_dominated"]
    assert abs(st["mean"] - gf.mean().item()) < 1e-6
    for name, v in zip(("p25", "median", "p75"), q.tolist()):
        assert abs(st[name] - v) <= 1e-6 * max(1.0, abs(v)), name
    assert st["frac_signal_dominated"] == pytest.approx(int((gf < 0.1).sum()) / gf.numel(), abs=1e-12)
    assert st["frac_noise_dominated"] == pytest.approx(int((gf > 0.9).sum()) / gf.numel(), abs=1e-12)
