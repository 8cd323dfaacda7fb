"""Conv2d through this package's GEMMs over the unfolded input.

ConcordConv2dPackedB runs its three convolutions as the Linear layer's GEMMs
on unfold(x) when the GEMM extents are multiples of 8.  Checked: the
forward, dX and dW against fp32 convolutions of the same bf16 values (bf16
output tolerance written per check), and the whole layer step against a
Linear layer with the same packed state fed the unfolded input, which must
give the same words bit for bit (the same dW reaches the same step).
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"

CASES = [  # B, C, H, W, O, k, stride, padding
    (2, 16, 16, 16, 32, 3, 1, 1),
    (2, 16, 16, 16, 32, 3, 2, 1),
    (4, 32, 8, 8, 64, 1, 1, 0),
    (1, 8, 12, 22, 16, 3, 1, 0),
]


def _bf(t):
    return t.to(torch.bfloat16)


@pytest.mark.parametrize("case", CASES)
def test_conv_gemm_matches_fp32_conv(case):
    from concord_b200 import gemm
    B, C, H, W, O, k, st, pd = case
    g = torch.Generator(device="cpu").manual_seed(sum(case))
    x = _bf(torch.randn(B, C, H, W, generator=g)).to(DEV)
    w = _bf(torch.randn(O, C * k * k, generator=g) * 0.1).to(DEV)
    bias = _bf(torch.randn(O, generator=g)).to(DEV)
    assert gemm.conv_usable(x, w, k, k, st, pd)
    w4 = w.float().view(O, C, k, k)
    y_ref = F.conv2d(x.float(), w4, bias.float(), stride=st, padding=pd)
    y = gemm.conv2d_forward(x, w, bias, k, k, st, pd)
    assert y.dtype == torch.bfloat16 and y.shape == y_ref.shape
    # one bf16 rounding of the product, one of the bias add
    tol = 2.0 ** -7 * y_ref.abs().max().item()
    assert (y.float() - y_ref).abs().max().item() <= tol

    gy = _bf(torch.randn(*y_ref.shape, generator=g)).to(DEV)
    dx, dW = gemm.conv2d_backward(x, w, gy, k, k, st, pd)
    dx_ref = torch.nn.grad.conv2d_input(x.shape, w4, gy.float(), stride=st, padding=pd)
    dW_ref = torch.nn.grad.conv2d_weight(x.float(), w4.shape, gy.float(), stride=st, padding=pd)
    assert dW.shape == (O, C * k * k) and dW.dtype == torch.bfloat16
    # dW: fp32 accumulation rounded once to bf16
    assert (dW.float() - dW_ref.view(O, -1)).abs().max().item() <= 2.0 ** -8 * dW_ref.abs().max().item()
    # dX: up to k*k bf16-rounded partials summed per pixel, rounded again
    assert (dx.float() - dx_ref).abs().max().item() <= 2.0 ** -6 * dx_ref.abs().max().item()


def test_conv_layer_step_equals_linear_on_unfolded_input():
    from concord_b200 import ConcordConv2dPackedB, ConcordLinearPackedB, gemm
    from concord_b200.checkpoint import set_step_salt
    B, C, H, W, O, k = 2, 16, 12, 12, 32, 3
    torch.manual_seed(5)
    conv = ConcordConv2dPackedB(C, O, k, padding=1, bias=False, device=DEV, lr=0.02)
    lin = ConcordLinearPackedB(C * k * k, O, bias=False, device=DEV, lr=0.02)
    lin.load_state_dict(conv.state_dict())
    for m in (conv, lin):          # the forward weight from the (now equal) words, as on resume
        m._ensure_buffers()
        m._resync_weight_buf()
    g = torch.Generator(device="cpu").manual_seed(9)
    for t in range(3):
        x = _bf(torch.randn(B, C, H, W, generator=g)).to(DEV).requires_grad_(True)
        gy = _bf(torch.randn(B, O, H, W, generator=g)).to(DEV)
        set_step_salt(DEV, 100 + t)
        y = conv(x)
        y.backward(gy)
        cols, Ho, Wo = gemm._conv_cols(x.detach(), k, k, 1, 1)
        cols.requires_grad_(True)
        set_step_salt(DEV, 100 + t)
        yl = lin(cols)
        yl.backward(gy.permute(0, 2, 3, 1).reshape(B * Ho * Wo, O))
        assert torch.equal(y.permute(0, 2, 3, 1).reshape(-1, O), yl)
        assert torch.equal(conv.packed_w, lin.packed_w), t
        conv.rebalance()
        lin.rebalance()
        assert torch.equal(conv.packed_w, lin.packed_w), t
