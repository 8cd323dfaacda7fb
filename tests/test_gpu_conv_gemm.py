"""Conv2d through this package's GEMMs over a column matrix (im2col).

ConcordConv2dPackedB runs its three convolutions as the Linear layer's GEMMs
on the column matrix when the GEMM extents are multiples of 8.  Checked:
concord_im2col against torch's unfold (bit for bit: a copy),
concord_col2im against a float64 fold of the same bf16 column gradient,
the forward, dX and dW against fp32 convolutions of the same bf16 values
(bf16 output tolerance written per check), and the whole layer step against
a Linear layer with the same packed state fed the column matrix, which must
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
def test_im2col_col2im_match_unfold_fold(case):
    from concord_b200 import gemm
    B, C, H, W, O, k, st, pd = case
    g = torch.Generator(device="cpu").manual_seed(7 + sum(case))
    x = _bf(torch.randn(B, C, H, W, generator=g)).to(DEV)
    cols, Ho, Wo = gemm._conv_cols(x, k, k, st, pd)
    ref = F.unfold(x, (k, k), padding=pd, stride=st).transpose(1, 2).reshape(B * Ho * Wo, -1)
    assert torch.equal(cols, ref)
    dct = _bf(torch.randn(C * k * k, B * Ho * Wo, generator=g)).to(DEV)
    dx = torch.empty_like(x)
    import ctypes
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    from concord_b200 import _abi
    _abi.check(_abi.load().concord_col2im(ctypes.c_void_p(dct.data_ptr()), *gemm._geom(x, k, k, st, pd),
                                          ctypes.c_void_p(dx.data_ptr()), s), "col2im")
    cols64 = dct.double().view(C * k * k, B, Ho * Wo).transpose(0, 1)
    dx64 = F.fold(cols64, (H, W), (k, k), padding=pd, stride=st)
    # fp32 sum of at most k*k terms, then one bf16 rounding
    err = (dx.double() - dx64).abs()
    assert (err <= 2.0 ** -8 * dx64.abs() + 1e-5 * dx64.abs().max()).all()


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


@pytest.fixture
def im2col_backend():
    import concord_b200
    old = concord_b200.get_conv_backend()
    concord_b200.set_conv_backend("gemm")
    yield
    concord_b200.set_conv_backend(old)


def test_conv_layer_step_equals_linear_on_unfolded_input(im2col_backend):
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
        # same products, GEMMs in the other orientation: within bf16 rounding
        yc = y.permute(0, 2, 3, 1).reshape(-1, O).float()
        assert (yc - yl.float()).abs().max().item() <= 2.0 ** -7 * yl.float().abs().max().item()
        assert torch.equal(conv.packed_w, lin.packed_w), t
        conv.rebalance()
        lin.rebalance()
        assert torch.equal(conv.packed_w, lin.packed_w), t


def test_cudnn_backend_switch():
    """set_conv_backend("cudnn") routes a GEMM-able shape through torch's
    convolutions; the dW each backend hands to the packed step agrees to bf16
    rounding (2^-7 of its largest entry), and the layer steps either way."""
    import concord_b200
    from concord_b200 import ConcordConv2dPackedB, gemm
    from concord_b200 import packed_b as pb
    calls, dws = [], []
    orig_bwd, orig_step = gemm.conv2d_backward, pb._packed_backward_step

    def spy_bwd(*a):
        calls.append(1)
        return orig_bwd(*a)

    def spy_step(ctx, grad_W, *rest):
        dws.append(grad_W.float().clone())
        return orig_step(ctx, grad_W, *rest)
    gemm.conv2d_backward, pb._packed_backward_step = spy_bwd, spy_step
    default = concord_b200.get_conv_backend()
    try:
        for backend in ("cudnn", "gemm"):
            concord_b200.set_conv_backend(backend)
            torch.manual_seed(4)
            c = ConcordConv2dPackedB(16, 32, 3, padding=1, device=DEV, lr=0.01)
            before = c.packed_w.clone()
            x = torch.randn(2, 16, 8, 8, device=DEV, requires_grad=True)
            c(x).float().pow(2).mean().backward()
            assert not torch.equal(before, c.packed_w)
        assert len(calls) == 1          # only the "gemm" run used the GEMM path
        assert (dws[0] - dws[1]).abs().max().item() <= 2.0 ** -7 * dws[1].abs().max().item()
    finally:
        gemm.conv2d_backward, pb._packed_backward_step = orig_bwd, orig_step
        concord_b200.set_conv_backend(default)
    with pytest.raises(ValueError):
        concord_b200.set_conv_backend("winograd")


@pytest.mark.parametrize("shape", [(2, 32, 100), (3, 7, 45), (1, 640, 4096)])
def test_transpose_bf16(shape):
    import ctypes
    from concord_b200 import _abi
    b, r, c = shape
    x = torch.randn(b, r, c, device=DEV).to(torch.bfloat16)
    out = torch.empty(b, c, r, device=DEV, dtype=torch.bfloat16)
    _abi.check(_abi.load().concord_transpose_bf16(ctypes.c_void_p(x.data_ptr()), b, r, c,
                                                  ctypes.c_void_p(out.data_ptr()),
                                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
               "transpose")
    assert torch.equal(out, x.transpose(1, 2))
