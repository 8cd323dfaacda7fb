"""The 2-SM tcgen05 GEMM written in this package (concord_gemm2sm) in the
three operand layouts of the layer's GEMMs, against a torch fp32 reference.

bf16 inputs, fp32 accumulation, bf16 output: the result equals the fp32
product up to the bf16 rounding of the output (2^-8 of the value) plus an fp32
accumulation term bounded by K * 2^-23 * (|A| |B|).  Shapes cover one tile,
ragged edges in every dimension (zero-filled TMA boxes, masked stores), more
tiles than CTA pairs, and reductions longer than the shared-memory ring.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
SHAPES = [(256, 256, 64), (512, 768, 512), (264, 520, 136), (2048, 2560, 1024), (8, 16, 24), (4096, 1280, 5120)]


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _close(got, ref, absprod, K):
    ref = ref.float()
    err = (got.float() - ref).abs()
    tol = ref.abs() * 2.0 ** -8 + absprod * (K * 2.0 ** -23) + 1e-30
    assert bool((err <= tol).all()), float((err / tol).max())


def _gemm(a, a_mn, b, b_mn, M, N, K):
    from concord_b200 import _abi
    lib = _abi.load()
    d = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _abi.check(lib.concord_gemm2sm(_p(a), a_mn, a.stride(0), _p(b), b_mn, b.stride(0), _p(d), N, M, N, K, s),
               "concord_gemm2sm")
    torch.cuda.synchronize()
    assert lib.concord_gemm2sm_error(1) == 0
    return d


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm2sm_layouts(M, N, K):
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N * 3 + K)
    a = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)       # K-major A
    b = (torch.randn(N, K, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    ref = a.float() @ b.float().T
    absprod = a.float().abs() @ b.float().abs().T
    _close(_gemm(a, 0, b, 0, M, N, K), ref, absprod, K)                      # forward layout
    bt = b.T.contiguous()                                                    # [K, N]: MN-major B
    _close(_gemm(a, 0, bt, 1, M, N, K), ref, absprod, K)                     # dX layout
    at = a.T.contiguous()                                                    # [K, M]: MN-major A
    _close(_gemm(at, 1, bt, 1, M, N, K), ref, absprod, K)                    # dW layout
    _close(_gemm(at, 1, b, 0, M, N, K), ref, absprod, K)


def test_gemm2sm_deterministic():
    g = torch.Generator(device=DEV).manual_seed(1)
    a = torch.randn(1024, 4096, generator=g, device=DEV).to(torch.bfloat16)
    b = torch.randn(2048, 4096, generator=g, device=DEV).to(torch.bfloat16)
    assert torch.equal(_gemm(a, 0, b, 0, 1024, 2048, 4096), _gemm(a, 0, b, 0, 1024, 2048, 4096))
