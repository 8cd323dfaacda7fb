"""Row-sharded data-parallel step on 2, 4 and 8 GPUs (skipped with fewer GPUs).

Every rank must end with identical packed words, exponents, v-hat state and
forward weight, equal bit for bit to a one-GPU emulation of the same sharded
arithmetic through the same CUDA kernels (the reduced gradient of the
emulation is the fp32 sum of the ranks' partials in rank order, rounded once
to bf16).  Both transports: "collective" (NCCL reduce-scatter / all-gather;
at 2 ranks NCCL's bf16 sum rounds once, like the emulation) and "peer"
(NVLink loads and stores through CUDA IPC mappings).  NVLS is switched off
(NCCL_NVLS_ENABLE=0) in every multi-rank test.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
K, STEPS = 512, 4


def _grad(N, step, rank, dev):
    g = torch.Generator(device="cpu").manual_seed(1000 * step + rank)
    return (torch.randn(N, K, generator=g) * 3e-2).to(torch.bfloat16).to(dev)


def _xy(N, step, rank, dev, M=64):
    """This rank's input and upstream gradient for one step (the DP-backward tests)."""
    g = torch.Generator(device="cpu").manual_seed(7000 + 1000 * step + rank)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
    gy = (torch.randn(M, N, generator=g) * 0.1).to(torch.bfloat16).to(dev)
    return x, gy


def _grad_bwd(N, step, rank, dev):
    """The dW the layer's backward computes from _xy (the same GEMM)."""
    from concord_b200 import gemm
    x, gy = _xy(N, step, rank, dev)
    return gemm.grad_weight(gy, x)


def _layer(N, dev):
    from concord_b200 import ConcordLinearPackedB
    torch.manual_seed(5)
    layer = ConcordLinearPackedB(K, N, bias=False, device=dev, lr=0.05)
    W = torch.randn(N, K, generator=torch.Generator().manual_seed(6)) * 0.05
    layer.load_weights(W)
    return layer


def _state(layer):
    w, rm, cm = layer._ensure_buffers()
    out = {k: getattr(layer, k).detach().cpu().numpy().copy()
           for k in ("packed_w", "row_exp", "col_exp", "v_row", "v_col", "_sum_v_inv", "_reb_seed")}
    out["wbuf"] = w.view(torch.int16).cpu().numpy().copy()
    return out


def _worker(rank, world, port, out_dir, N, transport, via_backward=False):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    from concord_b200 import packed_b
    from concord_b200.distributed import RowShardedStep
    packed_b.set_arithmetic("cr")        # the same arithmetic as the emulation in the test process
    dev = torch.device("cuda", rank)
    layer = _layer(N, dev)
    st = RowShardedStep(layer, transport=transport)
    assert st.transport == transport
    for s in range(STEPS):
        if via_backward:
            # the drop-in path: the registered layer's backward steps its shard
            x, gy = _xy(N, s, rank, dev)
            layer(x.requires_grad_(True)).backward(gy)
            layer.rebalance()
        else:
            st.step(_grad(N, s, rank, dev))
            st.rebalance()
    st.check()
    st.gather_state()
    torch.cuda.synchronize()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **_state(layer))
    st.close()
    dist.barrier()
    dist.destroy_process_group()


def _emulate(world, N, grad_fn=_grad):
    """The same sharded arithmetic on one GPU, shard by shard."""
    from concord_b200 import packed_b as pb
    from concord_b200.distributed import CudaKernels as KK
    dev = torch.device("cuda", 0)
    L = _layer(N, dev)
    S = (N + world - 1) // world
    wbuf, rmax, cmax = L._ensure_buffers()
    red = torch.zeros(K + 1, dtype=torch.float32, device=dev)
    salt = pb._get_step_counter(dev)
    salt.zero_()          # the workers' counters start at 0 in fresh processes
    for s in range(STEPS):
        tot = grad_fn(N, s, 0, dev).float()
        for r in range(1, world):
            tot = tot + grad_fn(N, s, r, dev).float()
        g = tot.to(torch.bfloat16)
        acc = torch.zeros(K + 1, dtype=torch.float32, device=dev)
        for r in range(world):
            r0, r1 = min(N, r * S), min(N, r * S + S)
            if r1 <= r0:
                continue          # a rank without rows adds zero partials
            KK.vhat_partial(g[r0:r1].contiguous(), L.v_row[r0:r1], L.adafactor_beta2, rmax[r0:r1],
                            cmax if r == 0 else torch.empty_like(cmax), r == 0, red[:K], red[K:])
            acc = acc + red
        KK.vhat_finish(acc[:K], acc[K:], L.v_col, L._sum_v_inv, L.adafactor_beta2)
        P = pb.adamw_params(v_scale=0.0, precond_p=0.5, drift_cancel_C=L.drift_cancel_C,
                            mass_preserve=True, gf_trust_delta_sq=1.0, use_cohpre=True)
        cm_all = torch.zeros_like(cmax)
        for r in range(world):
            r0, r1 = min(N, r * S), min(N, r * S + S)
            if r1 <= r0:
                continue
            cm = torch.zeros_like(cmax)
            w = torch.empty(r1 - r0, K, dtype=torch.bfloat16, device=dev)
            KK.step(P, L.packed_w[r0:r1], g[r0:r1].contiguous(), w, L.row_exp[r0:r1], L.col_exp,
                    rmax[r0:r1], cm, L.v_row[r0:r1], L.v_col, L._sum_v_inv, L._coh_pre[r0:r1],
                    L._lr_buf, L._eps_buf, salt, r0)
            cm_all = torch.maximum(cm_all, cm)
        cmax.copy_(cm_all)
        KK.materialize(L.packed_w, L.row_exp, L.col_exp, wbuf, L.MANTISSA_BIAS)
        L.rebalance()
    torch.cuda.synchronize()
    return _state(L)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,transport", [(2, "collective"), (2, "peer"), (4, "peer"), (8, "peer")])
# even split (in-place collectives), padded, and fewer rows than ranks (rank 1+ owns none)
@pytest.mark.parametrize("N", [300, 301, 1])
def test_row_sharded_step(tmp_path, N, world, transport):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), N, transport),
                       nprocs=world, join=True, start_method="spawn")
    r = [dict(np.load(tmp_path / f"rank{i}.npz")) for i in range(world)]
    ref = _emulate(world, N)
    for key in ref:
        for i in range(1, world):
            np.testing.assert_array_equal(r[0][key], r[i][key], err_msg=key)
        np.testing.assert_array_equal(r[0][key], ref[key], err_msg=key)


@pytest.mark.parametrize("world,transport", [(2, "collective"), (2, "peer")])
def test_data_parallel_through_loss_backward(tmp_path, world, transport):
    """Data-parallel training through the drop-in API: each rank calls
    layer(x).backward(dY) and layer.rebalance() on its own batch; the layer,
    registered with a RowShardedStep, steps only its row shard of the reduced
    gradient.  Every rank ends identical and equal to the one-GPU emulation
    fed the ranks' dW (no local step happened on the way)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    N = 304
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), N, transport, True),
                       nprocs=world, join=True, start_method="spawn")
    r = [dict(np.load(tmp_path / f"rank{i}.npz")) for i in range(world)]
    ref = _emulate(world, N, grad_fn=_grad_bwd)
    for key in ref:
        for i in range(1, world):
            np.testing.assert_array_equal(r[0][key], r[i][key], err_msg=key)
        np.testing.assert_array_equal(r[0][key], ref[key], err_msg=key)
