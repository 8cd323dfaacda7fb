"""Implicit-GEMM convolutions on channels-last tensors (concord_conv_*_nhwc).

No column matrix: the activation is read by TMA in im2col mode.  Checked
against fp32 convolutions of the same bf16 values (fp32 accumulation, one
bf16 rounding per output: tolerance 2^-7 of the largest reference entry for
y and dX, 2^-8 for dW, as the column-matrix path's tests), the data-gradient
split of the filter gradient (wgrad splits its reduction over the SMs when
the output has few tiles) for run-to-run determinism, and the conv layer on
the "implicit" backend against the "gemm" backend: the same packed step on a
dW that agrees to bf16 rounding.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"

CASES = [  # B, C, H, W, O, k, padding
    (2, 16, 16, 16, 32, 3, 1),
    (1, 8, 12, 22, 16, 3, 0),
    (4, 32, 8, 8, 64, 1, 0),
    (2, 64, 64, 64, 64, 3, 1),      # wgrad splits its 8192-row reduction
    (1, 320, 32, 32, 320, 3, 1),    # an SDXL level-1 shape
    (3, 24, 9, 7, 40, 3, 1),        # ragged tiles everywhere
]


def _bf(t):
    return t.to(torch.bfloat16)


def _inputs(case, seed):
    B, C, H, W, O, k, pd = case
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = _bf(torch.randn(B, C, H, W, generator=g)).to(DEV)
    w = _bf(torch.randn(O, C * k * k, generator=g) * 0.1).to(DEV)
    return g, x, w


@pytest.mark.parametrize("case", CASES)
def test_implicit_conv_matches_fp32_conv(case):
    from concord_b200 import gemm
    B, C, H, W, O, k, pd = case
    g, x, w = _inputs(case, sum(case))
    bias = _bf(torch.randn(O, generator=g)).to(DEV)
    assert gemm.conv_nhwc_usable(x, w, k, k, 1, pd)
    w4 = w.float().view(O, C, k, k)
    wk = gemm.filter_krsc(w, C, k, k)
    assert torch.equal(wk, w.view(O, C, k, k).permute(0, 2, 3, 1).contiguous())
    y_ref = F.conv2d(x.float(), w4, bias.float(), padding=pd)
    y = gemm.conv2d_forward_nhwc(x, wk, bias, k, k, 1, pd)
    assert y.dtype == torch.bfloat16 and y.shape == y_ref.shape
    assert y.is_contiguous(memory_format=torch.channels_last)
    # one bf16 rounding of the product, one of the bias add
    assert (y.float() - y_ref).abs().max().item() <= 2.0 ** -7 * y_ref.abs().max().item()

    gy = _bf(torch.randn(*y_ref.shape, generator=g)).to(DEV)
    dx, dW = gemm.conv2d_backward_nhwc(x, wk, gy, k, k, 1, pd)
    dx_ref = torch.nn.grad.conv2d_input(x.shape, w4, gy.float(), padding=pd)
    dW_ref = torch.nn.grad.conv2d_weight(x.float(), w4.shape, gy.float(), padding=pd).view(O, -1)
    assert dx.shape == x.shape and dx.dtype == torch.bfloat16
    assert dW.shape == (O, C * k * k) and dW.is_contiguous()
    assert (dx.float() - dx_ref).abs().max().item() <= 2.0 ** -7 * dx_ref.abs().max().item()
    assert (dW.float() - dW_ref).abs().max().item() <= 2.0 ** -8 * dW_ref.abs().max().item()


def test_implicit_conv_is_deterministic():
    from concord_b200 import gemm
    case = (2, 64, 64, 64, 64, 3, 1)
    B, C, H, W, O, k, pd = case
    g, x, w = _inputs(case, 3)
    wk = gemm.filter_krsc(w, C, k, k)
    gy = _bf(torch.randn(B, O, H, W, generator=g)).to(DEV)
    a = gemm.conv2d_backward_nhwc(x, wk, gy, k, k, 1, pd)
    b = gemm.conv2d_backward_nhwc(x, wk, gy, k, k, 1, pd)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_implicit_conv_rejects_what_it_does_not_run():
    import ctypes
    from concord_b200 import _abi, gemm
    x = torch.zeros(1, 12, 8, 8, dtype=torch.bfloat16, device=DEV)        # C not a multiple of 8
    w = torch.zeros(16, 12 * 9, dtype=torch.bfloat16, device=DEV)
    assert not gemm.conv_nhwc_usable(x, w, 3, 3, 1, 1)
    x = torch.zeros(1, 16, 8, 8, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(16, 16 * 9, dtype=torch.bfloat16, device=DEV)
    assert not gemm.conv_nhwc_usable(x, w, 3, 3, 2, 1)                     # stride 2: column path
    lib = _abi.load()
    p = ctypes.c_void_p(x.data_ptr())
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.concord_conv_dgrad_nhwc(p, p, p, 1, 8, 8, 16, 16, 3, 3, 2, 2, 1, 1, p, 1 << 20, s)
    assert rc == -2                                                         # CONCORD_ESHAPE
    rc = lib.concord_conv_fprop_nhwc(p, p, p, 1, 8, 8, 12, 16, 3, 3, 1, 1, 1, 1, p, 1 << 20, s)
    assert rc == -2


def test_conv_layer_implicit_backend_against_column_backend():
    """The layer on the implicit backend: output channels-last, a dW that
    agrees with the column-matrix backend's to bf16 rounding, and a step; a
    stride-2 layer on the implicit backend takes the column path."""
    import concord_b200
    from concord_b200 import ConcordConv2dPackedB, gemm
    from concord_b200 import packed_b as pb
    dws, calls = {}, []
    orig_step, orig_nhwc = pb._packed_backward_step, gemm.conv2d_backward_nhwc

    def spy_step(ctx, grad_W, *rest, **kw):
        dws.setdefault(concord_b200.get_conv_backend(), []).append(grad_W.float().clone())
        return orig_step(ctx, grad_W, *rest, **kw)

    def spy_nhwc(*a):
        calls.append(1)
        return orig_nhwc(*a)
    default = concord_b200.get_conv_backend()
    pb._packed_backward_step, gemm.conv2d_backward_nhwc = spy_step, spy_nhwc
    try:
        for backend in ("gemm", "implicit"):
            concord_b200.set_conv_backend(backend)
            torch.manual_seed(4)
            c = ConcordConv2dPackedB(32, 64, 3, padding=1, device=DEV, lr=0.01)
            before = c.packed_w.clone()
            x = torch.randn(2, 32, 16, 16, device=DEV).to(torch.bfloat16).requires_grad_(True)
            y = c(x)
            if backend == "implicit":
                assert y.is_contiguous(memory_format=torch.channels_last)
            y.float().pow(2).mean().backward()
            assert x.grad is not None and x.grad.shape == x.shape
            assert not torch.equal(before, c.packed_w)
        assert len(calls) == 1
        a, b = dws["gemm"][0], dws["implicit"][0]
        assert (a - b).abs().max().item() <= 2.0 ** -7 * a.abs().max().item()
        concord_b200.set_conv_backend("implicit")
        c2 = ConcordConv2dPackedB(16, 32, 3, stride=2, padding=1, device=DEV, lr=0.01)
        c2(torch.randn(1, 16, 8, 8, device=DEV)).float().sum().backward()
        assert len(calls) == 1
    finally:
        pb._packed_backward_step, gemm.conv2d_backward_nhwc = orig_step, orig_nhwc
        concord_b200.set_conv_backend(default)
