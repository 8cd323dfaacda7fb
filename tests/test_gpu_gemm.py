"""tcgen05 GEMMs (concord_gemm_fwd/dx/dw) against a torch fp32 reference.

bf16 inputs, fp32 accumulation, bf16 output: the result must equal the fp32
product up to the bf16 rounding of the output (at most half a bf16 ulp,
2^-8 of the value) plus an fp32 accumulation term bounded by
K * 2^-23 * (|A| |B|) (any summation order of K fp32 products).  A dW with fewer output tiles than SMs and a long
reduction runs split over the reduction (fp32 partials summed in order): same
bound.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
SHAPES = [(512, 1280, 1280), (256, 5120, 1280), (384, 1280, 5120), (1024, 10240, 2048), (8, 16, 24),
          # long reductions onto small dW outputs: the split-K dW (8, 4 and 2 slices)
          (8192, 320, 2880), (4096, 64, 1024), (16384, 1280, 1280)]


def _close(got, ref, absprod, K):
    ref = ref.float()
    err = (got.float() - ref).abs()
    tol = ref.abs() * 2.0 ** -8 + absprod * (K * 2.0 ** -23) + 1e-30
    assert bool((err <= tol).all()), float((err / tol).max())


@pytest.fixture(params=["2sm", "cutlass"])
def impl(request):
    """Both kernel families behind concord_gemm_fwd/dx/dw: the package's own
    2-SM kernel (default) and the CUTLASS 1-SM kernels."""
    from concord_b200 import _abi
    lib = _abi.load()
    old = lib.concord_gemm_get_impl()
    _abi.check(lib.concord_gemm_set_impl(_abi.GEMM_2SM if request.param == "2sm" else _abi.GEMM_CUTLASS),
               "concord_gemm_set_impl")
    yield request.param
    lib.concord_gemm_set_impl(old)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_fwd_dx_dw(M, N, K, impl):
    from concord_b200 import gemm
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    dy = torch.randn(M, N, generator=g, device=DEV).to(torch.bfloat16)
    xa, wa, da = x.float().abs(), w.float().abs(), dy.float().abs()
    _close(gemm.forward(x, w), x.float() @ w.float().T, xa @ wa.T, K)
    _close(gemm.grad_input(dy, w), dy.float() @ w.float(), da @ wa, N)
    _close(gemm.grad_weight(dy, x), dy.float().T @ x.float(), da.T @ xa, M)


def test_gemm_batched_input_and_bias():
    from concord_b200 import gemm
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(4, 64, 256, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(512, 256, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    b = torch.randn(512, generator=g, device=DEV).to(torch.bfloat16)
    y = gemm.forward(x, w, b)
    assert y.shape == (4, 64, 512)
    xw = x.float() @ w.float().T
    # two bf16 roundings (product, then + bias): bound by the operands' size
    err = (y.float() - (xw + b.float())).abs()
    assert bool((err <= (xw.abs() + b.float().abs()) * 2.0 ** -7 + 1e-6).all())


def test_gemm_native_kernel_is_used():
    """Aligned shapes must run the library's kernels, not torch's matmul."""
    from concord_b200 import gemm
    calls = []
    orig = gemm._run

    def spy(fn, *a):
        calls.append(fn)
        return orig(fn, *a)
    gemm._run = spy
    try:
        x = torch.randn(128, 256, device=DEV).to(torch.bfloat16)
        w = torch.randn(64, 256, device=DEV).to(torch.bfloat16)
        gemm.forward(x, w)
        gemm.grad_input(torch.randn(128, 64, device=DEV).to(torch.bfloat16), w)
        gemm.grad_weight(torch.randn(128, 64, device=DEV).to(torch.bfloat16), x)
    finally:
        gemm._run = orig
    assert calls == ["concord_gemm_fwd", "concord_gemm_dx", "concord_gemm_dw"]
