"""The dW GEMM with the v-hat partials in its epilogue (concord_gemm_dw_vhat).

Against the two-launch path it replaces (concord_gemm_dw, then
concord_vhat_update on the stored dW): the stored dW bit for bit; v_row,
v_col and sum_v_inv to fp32 summation rounding (the tiles and the fold order
are the same, the in-tile order is the epilogue's), and both checked against
float64 sums of the squared bf16 dW; row/col maxima zeroed and the salt
bumped as the standalone update does.  A layer of fewer output tiles than
SMs runs the two-launch path inside the call: identical bits.  Through a
layer's loss.backward(): the step that follows is the ordinary step on the
fused v-hat, bit for bit.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    dy = (torch.randn(M, N, generator=g) * 0.1).to(torch.bfloat16).cuda()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    v_row = (torch.rand(N, generator=g) * 1e-4 + 1e-6).cuda()
    v_col = (torch.rand(K, generator=g) * 1e-4 + 1e-6).cuda()
    return dy, x, v_row, v_col


def _run_both(M, N, K, seed=0):
    from concord_b200 import gemm, packed_b as pb
    dy, x, v_row, v_col = _inputs(M, N, K, seed)
    vr_a, vc_a, sv_a = v_row.clone(), v_col.clone(), torch.zeros(1, device="cuda")
    rmax_a = torch.full((N,), 77, dtype=torch.int32, device="cuda")
    cmax_a = torch.full((K,), 77, dtype=torch.int32, device="cuda")
    salt = pb._get_step_counter(torch.device("cuda"))
    s0 = int(salt.item())
    dw_a = pb.dw_vhat_update(dy, x, vr_a, vc_a, sv_a, 0.999, rmax_a, cmax_a, bump_salt=True)
    torch.cuda.synchronize()
    s1 = int(salt.item())
    dw_b = gemm.grad_weight(dy, x)
    vr_b, vc_b, sv_b = v_row.clone(), v_col.clone(), torch.zeros(1, device="cuda")
    pb.vhat_update(dw_b, vr_b, vc_b, sv_b, 0.999)
    torch.cuda.synchronize()
    return dict(dy=dy, x=x, v_row=v_row, v_col=v_col, dw_a=dw_a, dw_b=dw_b, vr_a=vr_a, vc_a=vc_a, sv_a=sv_a,
                vr_b=vr_b, vc_b=vc_b, sv_b=sv_b, rmax=rmax_a, cmax=cmax_a, bump=s1 - s0)


def _exact(dw, v_row, v_col, b2=0.999):
    g = dw.float().double().cpu().numpy()
    g2 = g * g
    vr = b2 * v_row.double().cpu().numpy() + (1 - b2) * g2.sum(axis=1)
    vc = b2 * v_col.double().cpu().numpy() + (1 - b2) * g2.sum(axis=0)
    return vr, vc, 1.0 / vr.sum()


# (M, N, K): >= 148 output tiles of 128 x 256 (the epilogue form), ragged
# edges, and a small layer (4 tiles) that takes the two-launch path inside the call
@pytest.mark.parametrize("M,N,K", [(512, 2048, 2560), (264, 2056, 2568), (2048, 256, 512)])
def test_dw_vhat_matches_two_launch_path(M, N, K):
    r = _run_both(M, N, K)
    assert torch.equal(r["dw_a"].view(torch.int16), r["dw_b"].view(torch.int16))
    assert int(r["rmax"].abs().sum()) == 0 and int(r["cmax"].abs().sum()) == 0
    assert r["bump"] == 1
    split = ((N + 127) // 128) * ((K + 255) // 256) < 148   # the two-launch path inside the call
    vr, vc, sv = _exact(r["dw_b"], r["v_row"], r["v_col"])
    for got, ref in ((r["vr_a"], vr), (r["vc_a"], vc), (r["sv_a"], [sv])):
        np.testing.assert_allclose(got.double().cpu().numpy(), ref, rtol=2e-6, atol=0)
    if split:
        for a, b in (("vr_a", "vr_b"), ("vc_a", "vc_b"), ("sv_a", "sv_b")):
            assert torch.equal(r[a], r[b]), a
    else:
        for a, b in (("vr_a", "vr_b"), ("vc_a", "vc_b"), ("sv_a", "sv_b")):
            np.testing.assert_allclose(r[a].double().cpu().numpy(), r[b].double().cpu().numpy(), rtol=2e-6)


def test_dw_vhat_deterministic():
    a = _run_both(512, 2048, 2560, seed=3)
    b = _run_both(512, 2048, 2560, seed=3)
    for k in ("vr_a", "vc_a", "sv_a"):
        assert torch.equal(a[k], b[k]), k


def test_layer_backward_uses_fused_vhat_then_the_ordinary_step():
    """loss.backward() through a layer takes the fused path; the words equal
    the ordinary step (vhat_done) run on the same dW and the fused v-hat."""
    from concord_b200 import ConcordLinearPackedB, packed_b as pb
    torch.manual_seed(0)
    M, N, K = 512, 2048, 2560
    layer = ConcordLinearPackedB(K, N, bias=False, device="cuda", lr=1e-2)
    layer.load_weights(torch.randn(N, K) * 0.02)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    gy = (torch.randn(M, N, generator=g) * 0.1).to(torch.bfloat16).cuda()
    layer(x)  # buffers
    keys = ("packed_w", "v_row", "v_col", "_sum_v_inv", "_coh_pre")
    before = {k: getattr(layer, k).detach().clone() for k in keys}
    salt = pb._get_step_counter(torch.device("cuda"))
    s_before = salt.clone()
    layer(x.requires_grad_(True)).backward(gy)
    torch.cuda.synchronize()
    after = {k: getattr(layer, k).detach().clone() for k in keys}
    # replay: the fused v-hat as the step's input, the standalone dW GEMM
    with torch.no_grad():
        for k in keys:
            if k not in ("v_row", "v_col", "_sum_v_inv"):
                getattr(layer, k).copy_(before[k])
        salt.copy_(s_before + 1)
    from concord_b200 import gemm
    dw = gemm.grad_weight(gy, x.detach())
    pb._packed_backward_step(layer._step_ctx(), dw, vhat_done=True)
    torch.cuda.synchronize()
    assert torch.equal(layer.packed_w, after["packed_w"])
    assert torch.equal(layer._coh_pre, after["_coh_pre"])
