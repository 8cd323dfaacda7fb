"""The allocation-free v-hat entry point, through the C ABI.

`concord_vhat_update_noalloc` exists for callers that may not allocate device
memory themselves (a host framework that owns all device memory behind a fixed
budget, or a caller that cannot afford cudaMalloc's implicit synchronisation).
It keeps its scratch in a fixed array inside the library.  Two calls in a row
must give the same v_row / v_col / sum_v_inv bits as the workspace-taking
`concord_vhat_update` (exact equality: both run the same fixed-order sums), and
a size beyond the fixed scratch must be refused.  This file is collected last
so that a failure here leaves every other test already run.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def lib():
    from concord_b200 import _abi
    return _abi.load()


def _inputs(N, K, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    grad = (torch.randn(N, K, generator=g) * 1e-2).to(torch.bfloat16).to(DEV)
    v_row = (torch.rand(N, generator=g) * 1e-4).to(DEV)
    v_col = (torch.rand(K, generator=g) * 1e-4).to(DEV)
    return grad, v_row, v_col


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("shape", [(300, 1000), (1024, 1024), (37, 70)])
def test_noalloc_matches_workspace_entry_point_twice(lib, shape):
    N, K = shape
    grad, v_row0, v_col0 = _inputs(N, K, seed=N + K)
    ref = [v_row0.clone(), v_col0.clone(), torch.ones(1, device=DEV)]
    got = [v_row0.clone(), v_col0.clone(), torch.ones(1, device=DEV)]
    rmax_ref = torch.full((N,), 5, dtype=torch.int32, device=DEV)
    cmax_ref = torch.full((K,), 5, dtype=torch.int32, device=DEV)
    rmax_got, cmax_got = rmax_ref.clone(), cmax_ref.clone()
    salt_ref = torch.zeros(1, dtype=torch.int32, device=DEV)
    salt_got = torch.zeros(1, dtype=torch.int32, device=DEV)
    ws = torch.zeros(lib.concord_vhat_workspace_bytes(N, K), dtype=torch.uint8, device=DEV)
    for _ in range(2):   # two calls in a row: the shared scratch must come back clean
        assert lib.concord_vhat_update(
            _ptr(grad), K, N, K, _ptr(ref[0]), _ptr(ref[1]), _ptr(ref[2]), 0.999, 1.0 - 0.999,
            _ptr(rmax_ref), _ptr(cmax_ref), _ptr(salt_ref), _ptr(ws), ws.numel(), _stream()) == 0
        rc = lib.concord_vhat_update_noalloc(
            _ptr(grad), K, N, K, _ptr(got[0]), _ptr(got[1]), _ptr(got[2]), 0.999, 1.0 - 0.999,
            _ptr(rmax_got), _ptr(cmax_got), _ptr(salt_got), _stream())
        assert rc == 0, lib.concord_last_error().decode()
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
    assert int(rmax_got.abs().sum()) == 0 and int(cmax_got.abs().sum()) == 0
    assert int(salt_got.item()) == 2 == int(salt_ref.item())


def _largest_rows_within_scratch(lib, K):
    cap = lib.concord_vhat_noalloc_max_scratch_bytes()
    lo, hi = 1, 1 << 20
    while lo < hi:   # largest N whose workspace still fits the fixed array
        mid = (lo + hi + 1) // 2
        if lib.concord_vhat_workspace_bytes(mid, K) <= cap:
            lo = mid
        else:
            hi = mid - 1
    return lo


def test_noalloc_at_the_scratch_limit(lib):
    """The largest N for K = 4096 that fits: the partial regions and counters
    then reach the end of the fixed array; still bit-identical, twice."""
    K = 4096
    N = _largest_rows_within_scratch(lib, K)
    cap = lib.concord_vhat_noalloc_max_scratch_bytes()
    assert lib.concord_vhat_workspace_bytes(N, K) <= cap < lib.concord_vhat_workspace_bytes(N + 1, K)
    grad, v_row0, v_col0 = _inputs(N, K, seed=11)
    ref = [v_row0.clone(), v_col0.clone(), torch.ones(1, device=DEV)]
    got = [v_row0.clone(), v_col0.clone(), torch.ones(1, device=DEV)]
    ws = torch.zeros(lib.concord_vhat_workspace_bytes(N, K), dtype=torch.uint8, device=DEV)
    for _ in range(2):
        assert lib.concord_vhat_update(_ptr(grad), K, N, K, _ptr(ref[0]), _ptr(ref[1]), _ptr(ref[2]), 0.999,
                                       1.0 - 0.999, None, None, None, _ptr(ws), ws.numel(), _stream()) == 0
        assert lib.concord_vhat_update_noalloc(_ptr(grad), K, N, K, _ptr(got[0]), _ptr(got[1]), _ptr(got[2]),
                                               0.999, 1.0 - 0.999, None, None, None, _stream()) == 0
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_noalloc_on_a_second_device(lib):
    """The array's address is looked up for whichever device is current."""
    N, K = 300, 1000
    with torch.cuda.device(1):
        dev = "cuda:1"
        g = torch.Generator().manual_seed(5)
        grad = (torch.randn(N, K, generator=g) * 1e-2).to(torch.bfloat16).to(dev)
        ref = [torch.zeros(N, device=dev), torch.zeros(K, device=dev), torch.ones(1, device=dev)]
        got = [t.clone() for t in ref]
        ws = torch.zeros(lib.concord_vhat_workspace_bytes(N, K), dtype=torch.uint8, device=dev)
        s = ctypes.c_void_p(torch.cuda.current_stream(1).cuda_stream)
        for _ in range(2):
            assert lib.concord_vhat_update(_ptr(grad), K, N, K, _ptr(ref[0]), _ptr(ref[1]), _ptr(ref[2]), 0.999,
                                           1.0 - 0.999, None, None, None, _ptr(ws), ws.numel(), s) == 0
            assert lib.concord_vhat_update_noalloc(_ptr(grad), K, N, K, _ptr(got[0]), _ptr(got[1]),
                                                   _ptr(got[2]), 0.999, 1.0 - 0.999, None, None, None, s) == 0
            torch.cuda.synchronize(1)
            for a, b in zip(got, ref):
                np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())


def test_noalloc_rejects_sizes_beyond_its_scratch(lib):
    cap = lib.concord_vhat_noalloc_max_scratch_bytes()
    N, K = 20000, 20000
    assert lib.concord_vhat_workspace_bytes(N, K) > cap
    dummy = torch.zeros(1, dtype=torch.float32, device=DEV)
    rc = lib.concord_vhat_update_noalloc(_ptr(dummy), K, N, K, _ptr(dummy), _ptr(dummy), _ptr(dummy),
                                         0.999, 0.001, None, None, None, _stream())
    assert rc == -7
    assert "4 MiB" in lib.concord_last_error().decode()
