"""Checkpoint / resume and dense export (concord_b200.checkpoint).

A two-layer MLP of packed layers trains 3 steps (autograd backward = the
packed step, then rebalance), is checkpointed through torch.save, and trains
3 more.  A second model of the same architecture but another init, other
knobs, another step salt and other module-wide gate settings restores the
checkpoint and trains the same 3 steps: every buffer, coh_pre, the forward
weight and the salt must equal the uninterrupted run's bit for bit.
"""
import io

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


class MLP(torch.nn.Module):
    def __init__(self, seed):
        super().__init__()
        from concord_b200 import ConcordLinearPackedB
        torch.manual_seed(seed)
        self.l1 = ConcordLinearPackedB(64, 128, bias=True, device=DEV, lr=0.05)
        self.l2 = ConcordLinearPackedB(128, 32, bias=False, device=DEV, lr=0.05)

    def forward(self, x):
        return self.l2(torch.relu(self.l1(x)))


def _batch(t):
    g = torch.Generator(device="cpu").manual_seed(100 + t)
    x = torch.randn(256, 64, generator=g).to(torch.bfloat16).to(DEV)
    y = torch.randn(256, 32, generator=g).to(DEV)
    return x, y


def _train(model, steps):
    for t in steps:
        x, y = _batch(t)
        loss = ((model(x).float() - y) ** 2).mean()
        loss.backward()
        for m in (model.l1, model.l2):
            m.rebalance()


def _snapshot(model):
    from concord_b200.checkpoint import get_step_salt
    out = {k: v.detach().clone() for k, v in model.state_dict().items()}
    for name in ("l1", "l2"):
        m = getattr(model, name)
        out[name + ".coh_pre"] = m._coh_pre.clone()
        out[name + ".wbuf"] = m._bf16_weight_buf.view(torch.int16).clone()
    out["salt"] = torch.tensor(get_step_salt(DEV))
    return out


def test_resume_is_bit_exact():
    from concord_b200 import packed_b as pb
    from concord_b200.checkpoint import load_state, save_state, set_step_salt
    set_step_salt(DEV, 0)
    a = MLP(seed=0)
    a.l1.gf_consol = 40.0          # a knob changed mid-run (as the autotuner does)
    _train(a, range(3))
    buf = io.BytesIO()
    torch.save(save_state(a), buf)
    _train(a, range(3, 6))
    ref = _snapshot(a)

    b = MLP(seed=1)
    b.l1.gf_consol = 0.0
    b.l2.beta1 = 0.5
    set_step_salt(DEV, 12345)
    gate_gain = pb._GATE_GAIN
    pb.set_gate_gain(0.7)
    try:
        buf.seek(0)
        load_state(b, torch.load(buf, weights_only=False))
        assert pb._GATE_GAIN == gate_gain
        _train(b, range(3, 6))
    finally:
        pb.set_gate_gain(gate_gain)
    got = _snapshot(b)
    assert ref.keys() == got.keys()
    for k in ref:
        assert torch.equal(ref[k], got[k]), k


def test_export_dense_matches_the_consolidated_weight():
    from concord_b200 import ConcordConv2dPackedB
    from concord_b200.checkpoint import export_dense
    a = MLP(seed=3)
    _train(a, range(2))
    d = export_dense(a)
    assert isinstance(d.l1, torch.nn.Linear) and isinstance(d.l2, torch.nn.Linear)
    assert torch.equal(d.l1.weight.view(torch.int16), a.l1.consolidated_weight().view(torch.int16))
    assert torch.equal(d.l1.bias, a.l1.bias.detach())
    assert d.l2.bias is None
    x, _ = _batch(0)
    ref = torch.nn.functional.linear(torch.relu(torch.nn.functional.linear(
        x, a.l1.consolidated_weight(), a.l1.bias.detach())), a.l2.consolidated_weight())
    assert torch.equal(d(x), ref)
    assert a.l1.packed_w.dtype == torch.int32          # the original is untouched

    conv = ConcordConv2dPackedB(4, 8, 3, padding=1, bias=True, device=DEV)
    dc = export_dense(conv)
    assert isinstance(dc, torch.nn.Conv2d) and dc.padding == (1, 1)
    assert torch.equal(dc.weight.view(torch.int16),
                       conv.consolidated_weight().view(8, 4, 3, 3).view(torch.int16))


def test_consolidated_safetensors_export(tmp_path):
    """The final save: a safetensors file of plain Linear / Conv2d weights equal to
    export_dense(model)'s state_dict, loadable into the dense model."""
    import torch.nn as nn
    from safetensors.torch import load_file
    from concord_b200 import ConcordConv2dPackedB, ConcordLinearPackedB
    from concord_b200.checkpoint import export_dense, save_consolidated
    torch.manual_seed(0)
    model = nn.Sequential(ConcordLinearPackedB(64, 48, bias=True, device="cuda"), nn.LayerNorm(48),
                          ConcordLinearPackedB(48, 32, bias=False, device="cuda")).cuda()
    conv = ConcordConv2dPackedB(8, 16, 3, padding=1, device="cuda")
    model.add_module("conv", conv)
    x = torch.randn(16, 64, device="cuda", requires_grad=True)
    model[2](model[1](model[0](x))).float().pow(2).mean().backward()
    path = str(tmp_path / "dense.safetensors")
    keys = save_consolidated(model, path)
    got = load_file(path)
    want = export_dense(model).state_dict()
    assert sorted(want) == keys
    for k, v in want.items():
        assert torch.equal(got[k], v.detach().cpu().to(got[k].dtype)), k
