"""GatedRebalance (device gate, batched launches) against the reference's
host-gated semantics (notebook/src/concord_winner.py:206-262).

Two identical sets of three layers take the same gradients.  Set A follows
the reference: the layers' max buffers are slices of two shared tensors,
the host reads their maximum and, when it exceeds MAX_M, calls every
layer's rebalance().  Set B calls concord_b200.gated.GatedRebalance.  After
every step the words, exponents, seeds and high-watermarks must agree bit
for bit, and the run must contain steps that fire and steps that do not.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
SHAPES = [(96, 64), (128, 200), (64, 48)]   # (out, in)


def _layers(seed):
    from concord_b200 import ConcordLinearPackedB
    out = []
    for i, (n, k) in enumerate(SHAPES):
        torch.manual_seed(seed + i)
        m = ConcordLinearPackedB(k, n, bias=False, device=DEV, lr=0.3)
        m.load_weights(torch.randn(n, k, generator=torch.Generator().manual_seed(50 + i)) * 0.05)
        out.append(m)
    return out


class HostGated:
    """The reference's GatedRebalance, restated."""

    def __init__(self, layers):
        self.layers, self.MAX_M, self.row_all = layers, max(m.MAX_M for m in layers), None

    def __call__(self):
        if self.row_all is None:
            rs = [m._row_max_buf.shape[0] for m in self.layers]
            cs = [m._col_max_buf.shape[0] for m in self.layers]
            self.row_all = torch.zeros(sum(rs), dtype=torch.int32, device=DEV)
            self.col_all = torch.zeros(sum(cs), dtype=torch.int32, device=DEV)
            ro = co = 0
            for m, n, k in zip(self.layers, rs, cs):
                m._row_max_buf = self.row_all[ro:ro + n]; ro += n
                m._col_max_buf = self.col_all[co:co + k]; co += k
            return False
        if bool((torch.maximum(self.row_all.max(), self.col_all.max()) > self.MAX_M).item()):
            for m in self.layers:
                m.rebalance()
            return True
        return False


def _state(layers):
    keys = ("packed_w", "row_exp", "col_exp", "_reb_seed", "_row_max_hwm", "_col_max_hwm")
    return [{k: getattr(m, k).clone() for k in keys} for m in layers]


def test_gated_rebalance_matches_host_gating():
    from concord_b200 import packed_b as pb
    from concord_b200.gated import GatedRebalance
    a, b = _layers(0), _layers(0)
    ga, gb = HostGated(a), GatedRebalance(b)
    salt = pb._get_step_counter(torch.device(DEV))
    fired = []
    for t in range(12):
        gens = [torch.Generator(device="cpu").manual_seed(1000 * t + i) for i in range(len(SHAPES))]
        grads = [(torch.randn(n, k, generator=g) * (0.5 if t % 4 == 3 else 0.02)).to(torch.bfloat16).to(DEV)
                 for (n, k), g in zip(SHAPES, gens)]
        s0 = int(salt.item())
        for m, g in zip(a, grads):
            m.optimizer_step(g)
        fa = ga()
        salt.fill_(s0)                         # set B sees the same step salts
        for m, g in zip(b, grads):
            m.optimizer_step(g)
        fb = gb()
        fired.append(fa)
        if t > 0:
            assert int(fb.item()) == int(fa), t
        for sa, sb in zip(_state(a), _state(b)):
            for k in sa:
                assert torch.equal(sa[k], sb[k]), (t, k)
    assert any(fired) and not all(fired[1:]), fired
    assert gb.calls == 12 and gb.fires == sum(fired)
