"""Dense GEMMs around the packed step: forward Y = X W^T, dX = dY W, dW = dY^T X.

These are plain bf16 library GEMMs (cuBLAS via torch) with fp32
accumulation, as in the reference (packed_b.py:1219, 1263, 1273).
"""
import torch
import torch.nn.functional as F


def forward(x, weight_bf16, bias=None):
    return F.linear(x, weight_bf16, bias)


def grad_input(grad_y, weight_bf16):
    return grad_y @ weight_bf16


def grad_weight(grad_y_flat, x_flat):
    """dW = dY^T X rounded to bf16, contiguous [N, K]."""
    g = grad_y_flat.transpose(0, 1) @ x_flat
    if g.dtype != torch.bfloat16:
        g = g.to(torch.bfloat16)
    return g.contiguous()
