"""Dense GEMMs around the packed step: forward Y = X W^T, dX = dY W, dW = dY^T X.

bf16 operands, fp32 accumulation, bf16 results (the reference's numerics,
packed_b.py:1219, 1263, 1271-1277).  Shapes whose extents are multiples of 8
run this package's tcgen05/TMEM kernels (`concord_gemm_*` in the C ABI);
other shapes (tiny or odd layers) use torch's cuBLAS matmul, as the
reference does for every shape.
"""
import ctypes

import torch
import torch.nn.functional as F

from . import _abi

_WS = {}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _ok(*dims):
    return all(int(d) % 8 == 0 for d in dims)


def _workspace(M, N, K, device):
    """GEMM scratch (CUTLASS workspace, split-K partials) per (device, current
    stream), grown on demand: launches on one stream are ordered, and a buffer
    replaced on one stream was never used by another."""
    lib = _abi.load()
    need = lib.concord_gemm_workspace_bytes(M, N, K)
    key = (str(device), torch.cuda.current_stream(device).cuda_stream)
    buf = _WS.get(key)
    if buf is None or buf.numel() < max(need, 1):
        buf = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def _run(fn, a, b, out, M, N, K):
    lib = _abi.load()
    ws = _workspace(M, N, K, out.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(out.device).cuda_stream)
    _abi.check(getattr(lib, fn)(_ptr(a), _ptr(b), _ptr(out), M, N, K, _ptr(ws), ws.numel(), stream), fn)
    return out


def _usable(*ts):
    return all(t.is_cuda and t.dtype == torch.bfloat16 for t in ts)


def forward(x, weight_bf16, bias=None):
    """y = x W^T (+ bias) over the last dim of x."""
    N, K = weight_bf16.shape
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    if _usable(x2, weight_bf16) and _ok(M, N, K) and M > 0:
        x2 = x2.contiguous()
        y = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
        _run("concord_gemm_fwd", x2, weight_bf16.contiguous(), y, M, N, K)
        if bias is not None:
            y.add_(bias)
        return y.reshape(*x.shape[:-1], N)
    return F.linear(x, weight_bf16, bias)


def grad_input(grad_y, weight_bf16):
    """dX = dY W over the last dim of dY."""
    N, K = weight_bf16.shape
    g2 = grad_y.reshape(-1, N)
    M = g2.shape[0]
    if _usable(g2, weight_bf16) and _ok(M, N, K) and M > 0:
        dx = torch.empty(M, K, dtype=torch.bfloat16, device=grad_y.device)
        _run("concord_gemm_dx", g2.contiguous(), weight_bf16.contiguous(), dx, M, N, K)
        return dx.reshape(*grad_y.shape[:-1], K)
    return grad_y @ weight_bf16


def grad_weight(grad_y_flat, x_flat):
    """dW = dY^T X rounded to bf16, contiguous [N, K]."""
    M, N = grad_y_flat.shape
    K = x_flat.shape[1]
    if _usable(grad_y_flat, x_flat) and _ok(M, N, K) and M > 0:
        dw = torch.empty(N, K, dtype=torch.bfloat16, device=x_flat.device)
        return _run("concord_gemm_dw", grad_y_flat.contiguous(), x_flat.contiguous(), dw, M, N, K)
    g = grad_y_flat.transpose(0, 1) @ x_flat
    if g.dtype != torch.bfloat16:
        g = g.to(torch.bfloat16)
    return g.contiguous()


# ---- convolutions as GEMMs over a column matrix (im2col) ----
#
# The packed conv weight is the [O, I*kh*kw] matrix (the reference views its
# Conv2d state that way, packed_b.py:2024-2065).  concord_im2col writes
# cols [B*Ho*Wo, I*kh*kw] with columns in (channel, kernel row, kernel
# column) order, the order of that matrix's columns, so
#   y^T [O, B*Ho*Wo]      = forward GEMM of (W, cols)      (NCHW at B == 1)
#   dW  [O, I*kh*kw]      = dW GEMM of (dY as [B*Ho*Wo, O], cols)
#   dcols^T [I*kh*kw, M]  = forward GEMM of (W^T, dY as [M, O]), then
#                           concord_col2im sums each pixel's kh*kw entries.

def _pair(v):
    return (int(v), int(v)) if isinstance(v, int) else tuple(int(a) for a in v)


def _conv_out(H, W, kh, kw, stride, padding):
    st, pd = _pair(stride), _pair(padding)
    if H + 2 * pd[0] < kh or W + 2 * pd[1] < kw:
        return 0, 0
    return (H + 2 * pd[0] - kh) // st[0] + 1, (W + 2 * pd[1] - kw) // st[1] + 1


def _geom(x, kh, kw, stride, padding):
    B, C, H, W = x.shape
    st, pd = _pair(stride), _pair(padding)
    return (B, C, H, W, kh, kw, st[0], st[1], pd[0], pd[1])


def _conv_cols(x, kh, kw, stride, padding):
    """The column matrix [B*Ho*Wo, C*kh*kw] of the bf16 NCHW input, plus (Ho, Wo)."""
    B, C, H, W = x.shape
    Ho, Wo = _conv_out(H, W, kh, kw, stride, padding)
    x = x.contiguous()
    cols = torch.empty(B * Ho * Wo, C * kh * kw, dtype=torch.bfloat16, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    _abi.check(_abi.load().concord_im2col(_ptr(x), *_geom(x, kh, kw, stride, padding), _ptr(cols), stream),
               "concord_im2col")
    return cols, Ho, Wo


def conv_usable(x, weight_2d, kh, kw, stride, padding):
    """True when the GEMM form of this convolution runs this package's kernels."""
    if x.dim() != 4 or not _usable(x, weight_2d):
        return False
    B, C, H, W = x.shape
    Ho, Wo = _conv_out(H, W, kh, kw, stride, padding)
    O, IK = weight_2d.shape
    return Ho > 0 and Wo > 0 and IK == C * kh * kw and _ok(B * Ho * Wo, O, IK)


def _pointwise(x, kh, kw, stride, padding):
    """A 1x1, stride-1, unpadded convolution whose per-image GEMMs fit the
    kernels: each image's NCHW plane [C, H*W] is already a GEMM operand."""
    return (kh == 1 and kw == 1 and _pair(stride) == (1, 1) and _pair(padding) == (0, 0)
            and _ok(x.shape[2] * x.shape[3]))


def _transpose(t, batches, R, C):
    out = torch.empty(batches * C, R, dtype=torch.bfloat16, device=t.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)
    _abi.check(_abi.load().concord_transpose_bf16(_ptr(t), batches, R, C, _ptr(out), stream),
               "concord_transpose_bf16")
    return out


def conv2d_forward(x, weight_2d, bias, kh, kw, stride, padding):
    """y = conv2d(x, W) (NCHW, bf16): the forward GEMM of (W, cols); for a
    pointwise convolution y_b = W x_b per image (the dX-layout GEMM), with
    no column matrix."""
    B = x.shape[0]
    O = weight_2d.shape[0]
    if _pointwise(x, kh, kw, stride, padding):
        C, L = x.shape[1], x.shape[2] * x.shape[3]
        x = x.contiguous()
        y = torch.empty(B, O, x.shape[2], x.shape[3], dtype=torch.bfloat16, device=x.device)
        for b in range(B):
            _run("concord_gemm_dx", weight_2d, x[b], y[b], O, C, L)
        if bias is not None:
            y.add_(bias.view(1, O, 1, 1))
        return y
    cols, Ho, Wo = _conv_cols(x, kh, kw, stride, padding)
    yt = forward(weight_2d, cols)                                  # [O, B*Ho*Wo]
    if B == 1:
        y = yt.view(1, O, Ho, Wo)
    else:
        y = yt.view(O, B, Ho, Wo).transpose(0, 1).contiguous()
    if bias is not None:
        y.add_(bias.view(1, O, 1, 1))
    return y


def conv2d_backward(x, weight_2d, grad_y, kh, kw, stride, padding):
    """(dX, dW) of conv2d(x, W) for the NCHW gradient grad_y.  dW is the bf16
    [O, I*kh*kw] matrix the packed step consumes (fp32 accumulation, one
    rounding); dX sums each pixel's kh*kw bf16 column gradients in fp32
    (concord_col2im) and rounds again."""
    B, C, H, W = x.shape
    O = weight_2d.shape[0]
    grad_y = grad_y.contiguous()
    if _pointwise(x, kh, kw, stride, padding):
        L = H * W
        x = x.contiguous()
        dW = grad_weight(_transpose(grad_y, B, O, L), _transpose(x, B, C, L))
        wt = weight_2d.t().contiguous()
        dx = torch.empty(B, C, H, W, dtype=torch.bfloat16, device=x.device)
        for b in range(B):                     # dx_b = W^T dy_b: one rounding per pixel
            _run("concord_gemm_dx", wt, grad_y[b], dx[b], C, O, L)
        return dx, dW
    cols, Ho, Wo = _conv_cols(x, kh, kw, stride, padding)
    gy = _transpose(grad_y, B, O, Ho * Wo)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    dW = grad_weight(gy, cols)
    del cols
    dcols_t = forward(weight_2d.t().contiguous(), gy)               # [C*kh*kw, B*Ho*Wo]
    dx = torch.empty(B, C, H, W, dtype=torch.bfloat16, device=x.device)
    _abi.check(_abi.load().concord_col2im(_ptr(dcols_t), *_geom(x, kh, kw, stride, padding), _ptr(dx),
                                          stream), "concord_col2im")
    return dx, dW


# ---- implicit-GEMM convolutions on channels-last tensors (concord_conv_*_nhwc) ----

def conv_nhwc_usable(x, weight_2d, kh, kw, stride, padding):
    """True when the implicit-GEMM convolutions (no column matrix) can run all
    three of this convolution's passes: channel counts multiples of 8 and
    stride 1 (the data-gradient kernel is the stride-1 one)."""
    if x.dim() != 4 or not _usable(x, weight_2d):
        return False
    B, C, H, W = x.shape
    O, IK = weight_2d.shape
    Ho, Wo = _conv_out(H, W, kh, kw, stride, padding)
    return (Ho > 0 and Wo > 0 and IK == C * kh * kw and C % 8 == 0 and O % 8 == 0
            and _pair(stride) == (1, 1))


def _nhwc(t):
    """[B, C, H, W] tensor as its channels-last storage viewed [B, H, W, C]
    (a copy only when t is not already channels-last contiguous)."""
    return t.contiguous(memory_format=torch.channels_last).permute(0, 2, 3, 1)


def _conv_call(name, op, a, b, out, B, H, W, C, O, kh, kw, stride, padding):
    lib = _abi.load()
    st, pd = _pair(stride), _pair(padding)
    dims = (B, H, W, C, O, kh, kw, st[0], st[1], pd[0], pd[1])
    need = lib.concord_conv_nhwc_workspace_bytes(op, *dims)
    ws = torch.empty(max(int(need), 256), dtype=torch.uint8, device=out.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(out.device).cuda_stream)
    _abi.check(getattr(lib, name)(_ptr(a), _ptr(b), _ptr(out), *dims, _ptr(ws), ws.numel(), stream), name)


def filter_krsc(weight_2d, C, kh, kw):
    """The packed layer's [O, C*kh*kw] bf16 weight (channel, kernel row,
    kernel column order) as the [O, kh, kw, C] filter the kernels read."""
    O = weight_2d.shape[0]
    return weight_2d.view(O, C, kh, kw).permute(0, 2, 3, 1).contiguous()


def conv2d_forward_nhwc(x, w_krsc, bias, kh, kw, stride, padding):
    """y = conv2d(x, W) without a column matrix: x read channels-last, y
    returned as a channels-last [B, O, Ho, Wo] tensor (one bf16 rounding,
    then the bias add)."""
    B, C, H, W = x.shape
    O = w_krsc.shape[0]
    Ho, Wo = _conv_out(H, W, kh, kw, stride, padding)
    xh = _nhwc(x)
    y = torch.empty(B, Ho, Wo, O, dtype=torch.bfloat16, device=x.device)
    _conv_call("concord_conv_fprop_nhwc", _abi.CONV_FPROP, xh, w_krsc, y, B, H, W, C, O, kh, kw, stride, padding)
    y = y.permute(0, 3, 1, 2)
    if bias is not None:
        y.add_(bias.view(1, O, 1, 1))
    return y


def conv2d_backward_nhwc(x, w_krsc, grad_y, kh, kw, stride, padding):
    """(dX, dW) without column matrices: dX channels-last [B, C, H, W] (one
    bf16 rounding per pixel), dW the [O, C*kh*kw] bf16 matrix the packed step
    consumes (fp32 accumulation, one rounding, permuted from the kernel's
    [O, kh, kw, C])."""
    B, C, H, W = x.shape
    O = w_krsc.shape[0]
    xh, gyh = _nhwc(x), _nhwc(grad_y)
    dx = torch.empty(B, H, W, C, dtype=torch.bfloat16, device=x.device)
    _conv_call("concord_conv_dgrad_nhwc", _abi.CONV_DGRAD, gyh, w_krsc, dx, B, H, W, C, O, kh, kw, stride, padding)
    dwk = torch.empty(O, kh, kw, C, dtype=torch.bfloat16, device=x.device)
    _conv_call("concord_conv_wgrad_nhwc", _abi.CONV_WGRAD, gyh, xh, dwk, B, H, W, C, O, kh, kw, stride, padding)
    dW = dwk.permute(0, 3, 1, 2).reshape(O, C * kh * kw)
    return dx.permute(0, 3, 1, 2), dW
