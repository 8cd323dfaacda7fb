"""The row-sharded data-parallel step's host orchestration on 2 CPU ranks (gloo).

The CUDA kernels are replaced by the CPU oracle (test infrastructure) behind
the same kernel interface, so this checks the sharding, the collectives and
the bookkeeping around them: both ranks must end with identical state, equal
bit for bit to a single-process emulation of the same sharded arithmetic.  A
second test makes one rank fail on the host before its first collective and
checks that the other rank gets an error from a short process-group timeout
instead of hanging.
"""
import os
import socket
from types import SimpleNamespace

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
N, K = 37, 24


def _np_bf16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


class OracleKernels:
    """CPU stand-ins for CudaKernels (numpy views share the torch storage)."""

    def __init__(self):
        from oracle import oracle
        self.o = oracle
        self._salt = torch.zeros(1, dtype=torch.int32)

    def vhat_partial(self, grad, v_row, beta2, row_max, col_max, bump_salt, col_sum, vsum):
        cs, vs = self.o.vhat_partial(_np_bf16(grad), v_row.numpy(), beta2)
        col_sum.copy_(torch.from_numpy(cs))
        vsum.copy_(torch.from_numpy(vs))
        if row_max is not None:
            row_max.zero_()
            col_max.zero_()
        if bump_salt:
            self._salt += 1

    def vhat_finish(self, col_sum, vsum, v_col, sum_v_inv, beta2):
        b2, omb2 = np.float32(beta2), np.float32(1.0 - beta2)
        vc = v_col.numpy()
        vc[:] = b2 * vc + omb2 * col_sum.numpy()
        sum_v_inv.numpy()[0] = np.float32(1.0) / np.maximum(vsum.numpy()[0], np.float32(1e-30))

    def step(self, params, packed, grad, wbuf, row_exp, col_exp, row_max, col_max, v_row, v_col,
             sum_v_inv, coh_pre, lr_t, eps_t, salt, row0):
        w = np.zeros(tuple(wbuf.shape), np.uint16)
        self.o.step(params, packed.numpy(), _np_bf16(grad), w, row_exp.numpy(), col_exp.numpy(),
                    row_max.numpy(), col_max.numpy(), v_row.numpy(), v_col.numpy(),
                    sum_v_inv.numpy(), None if coh_pre is None else coh_pre.numpy(),
                    float(lr_t[0]), float(eps_t[0]), int(salt[0]), row0=row0)
        wbuf.copy_(torch.from_numpy(w.view(np.int16)).view(torch.bfloat16))

    def rebalance(self, packed, row_exp, col_exp, row_max, col_max, row_hwm, col_hwm, seed, max_m,
                  exp_max, exp_min, row0, n_total, fired_out=None):
        self.o.rebalance(packed.numpy(), row_exp.numpy(), col_exp.numpy(), row_max.numpy(),
                         col_max.numpy(), row_hwm.numpy(), col_hwm.numpy(), seed.numpy(), max_m,
                         exp_max, exp_min, row0=row0, n_total=n_total)

    def materialize(self, packed, row_exp, col_exp, out, mantissa_bias):
        w = self.o.materialize(packed.numpy(), row_exp.numpy(), col_exp.numpy(), mantissa_bias)
        out.copy_(torch.from_numpy(w.view(np.int16)).view(torch.bfloat16))

    def salt(self, device):
        return self._salt


def make_layer_W(seed=0, n=N):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, K)) * 0.05).astype(np.float32)


def make_layer(seed=0, n=N):
    from oracle import oracle
    from concord_b200.packed_b import compute_drift_cancel_C
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((n, K)) * 0.05).astype(np.float32)
    packed, rexp, cexp = oracle.quantize(W)
    L = SimpleNamespace(
        packed_w=torch.from_numpy(packed), row_exp=torch.from_numpy(rexp),
        col_exp=torch.from_numpy(cexp), v_row=torch.zeros(n), v_col=torch.zeros(K),
        _sum_v_inv=torch.ones(1), _coh_pre=torch.ones(n, K), _lr_buf=torch.tensor([0.5]),
        _eps_buf=torch.tensor([1e-10]), track_rebalance=True, adafactor_beta2=0.999,
        optimizer_kind='adamw', alpha=0.1, beta1=0.0, weight_decay=0.0, step_cap=10.0,
        v_scale=0.0, precond_p=0.5, gf_consol=0.0,
        drift_cancel_C=compute_drift_cancel_C(0.1, 0.001), alpha_v_fast=0.001, wd_sv=0.0,
        wd_sf=0.0, mass_preserve_v=True, apply_chase=True, gf_trust_delta_sq=1.0,
        MANTISSA_BIAS=15, MAX_M=24000, EXP_MAX=7, EXP_MIN=-8, allow_tickdown=False,
        _reb_seed=torch.zeros(1, dtype=torch.int32), _row_max_hwm=torch.zeros(n, dtype=torch.int32),
        _col_max_hwm=torch.zeros(K, dtype=torch.int32))
    bufs = (torch.zeros(n, K, dtype=torch.bfloat16), torch.zeros(n, dtype=torch.int32),
            torch.zeros(K, dtype=torch.int32))
    L._bf16_weight_buf, L._row_max_buf, L._col_max_buf = bufs
    L._ensure_buffers = lambda: (L._bf16_weight_buf, L._row_max_buf, L._col_max_buf)
    return L


def grads(step, rank, n=N):
    g = torch.Generator().manual_seed(100 * step + rank)
    return (torch.randn(n, K, generator=g) * 1e-3).to(torch.bfloat16)


def _worker(rank, world, port, out_dir, mode="manual"):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from concord_b200.distributed import DeferredColumnMaxima, RowShardedStep
    n = 1 if mode == "empty_rank" else N     # rank 1 of 2 owns no row of a 1-row layer
    L = make_layer(n=n)
    st = RowShardedStep(L, kernels=OracleKernels())
    from concord_b200 import packed_b as pb
    dm = other = None
    if mode == "deferred":
        # a second layer first in the flat buffer, so this layer's maxima sit at an offset
        other = RowShardedStep(make_layer(seed=1), kernels=OracleKernels())
        dm = DeferredColumnMaxima([other, st])
    for s in range(3):
        if mode == "deferred":
            other.step(grads(s + 10, rank))
            st.step(grads(s, rank))
            assert dm.pending
            st.rebalance()              # all-reduces both layers' maxima once
            assert not dm.pending
            other.rebalance()
        elif mode in ("manual", "empty_rank"):
            st.step(grads(s, rank, n))
            st.rebalance()
        else:
            # what the layer's autograd backward and rebalance() do once the
            # layer is registered as data-parallel
            pb._optimizer_half(SimpleNamespace(packed_w=L.packed_w), grads(s, rank))
            pb.ConcordLinearPackedB.rebalance(L)
    st.gather_state()
    if dm is not None:
        dm.close()
        other.close()
    if mode == "backward":
        assert pb._sharded_of(L.packed_w) is st
        st.close()
        assert pb._sharded_of(L.packed_w) is None
    wbuf, rmax, cmax = L._ensure_buffers()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), packed=L.packed_w.numpy(),
             v_row=L.v_row.numpy(), v_col=L.v_col.numpy(), svi=L._sum_v_inv.numpy(),
             wbuf=_np_bf16(wbuf), cmax=cmax.numpy(), coh=L._coh_pre.numpy(),
             row_exp=L.row_exp.numpy(), col_exp=L.col_exp.numpy(), seed=L._reb_seed.numpy(),
             hwm=L._row_max_hwm.numpy())
    dist.destroy_process_group()


def emulate(world, n=N):
    """Single-process emulation of the sharded arithmetic (same order as 2 ranks)."""
    from oracle import oracle
    from concord_b200.packed_b import adamw_params
    L = make_layer(n=n)
    S = (n + world - 1) // world
    coh = L._coh_pre.numpy()
    packed, v_row, v_col = L.packed_w.numpy(), L.v_row.numpy(), L.v_col.numpy()
    svi = np.ones(1, np.float32)
    P = adamw_params(v_scale=0.0, precond_p=0.5, drift_cancel_C=L.drift_cancel_C,
                     mass_preserve=True, gf_trust_delta_sq=1.0, use_cohpre=True)
    rexp, cexp = L.row_exp.numpy(), L.col_exp.numpy()
    seed = np.zeros(1, np.int32)
    hr, hc = np.zeros(n, np.int32), np.zeros(K, np.int32)
    wbuf = np.zeros((n, K), np.uint16)
    for s in range(3):
        tot = grads(s, 0, n).float()
        for r in range(1, world):
            tot = tot + grads(s, r, n).float()
        g = _np_bf16(tot.to(torch.bfloat16))
        cs_sum, vs_sum = np.zeros(K, np.float32), np.zeros(1, np.float32)
        for r in range(world):
            r0, r1 = r * S, min(n, r * S + S)
            cs, vs = oracle.vhat_partial(np.ascontiguousarray(g[r0:r1]), v_row[r0:r1])
            cs_sum = cs_sum + cs
            vs_sum = vs_sum + vs
        v_col[:] = np.float32(0.999) * v_col + np.float32(1.0 - 0.999) * cs_sum
        svi[0] = np.float32(1.0) / np.maximum(vs_sum[0], np.float32(1e-30))
        rmax, cmax = np.zeros(n, np.int32), np.zeros(K, np.int32)
        for r in range(world):
            r0, r1 = r * S, min(n, r * S + S)
            w = np.zeros((r1 - r0, K), np.uint16)
            oracle.step(P, packed[r0:r1], np.ascontiguousarray(g[r0:r1]), w, rexp[r0:r1], cexp,
                        rmax[r0:r1], cmax, v_row[r0:r1], v_col, svi, coh[r0:r1],
                        0.5, 1e-10, s + 1, row0=r0)
            wbuf[r0:r1] = w
        oracle.rebalance(packed, rexp, cexp, rmax, cmax, hr, hc, seed)
    return dict(packed=packed, v_row=v_row, v_col=v_col, svi=svi, wbuf=wbuf, cmax=cmax, coh=coh,
                row_exp=rexp, col_exp=cexp, seed=seed, hwm=hr)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


import pytest  # noqa: E402


@pytest.mark.parametrize("mode", ["manual", "backward", "deferred", "empty_rank"])
def test_row_sharded_step_two_ranks(tmp_path, oracle_mod, mode):
    """`manual`: the caller hands each rank's dW to RowShardedStep.step.
    `backward`: the layer's own backward path (registered as data-parallel)
    hands it over.  `deferred`: the column maxima of two layers are
    all-reduced once per step (DeferredColumnMaxima) instead of per layer.
    `empty_rank`: a 1-row layer, so rank 1 owns no row; it must still apply
    the shared column decisions of the rebalance.  All must give the same
    sharded state."""
    world = 2
    n = 1 if mode == "empty_rank" else N
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), mode), nprocs=world,
                       join=True, start_method="spawn")
    r = [dict(np.load(tmp_path / f"rank{i}.npz")) for i in range(world)]
    ref = emulate(world, n)
    for key in ("packed", "v_row", "v_col", "svi", "wbuf", "cmax", "coh", "row_exp", "col_exp",
                "seed", "hwm"):
        np.testing.assert_array_equal(r[0][key], r[1][key], err_msg=key)
        np.testing.assert_array_equal(r[0][key], ref[key], err_msg=key)
    from oracle import oracle
    q = oracle.quantize(make_layer_W(n=n))
    assert (r[0]["row_exp"] != q[1]).any() and (r[0]["col_exp"] != q[2]).any(), "rebalance never fired"


def _failing_worker(rank, world, port, out_dir):
    import datetime
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=4))
    from concord_b200.distributed import RowShardedStep
    L = make_layer()
    st = RowShardedStep(L, kernels=OracleKernels())
    if rank == 1:
        open(os.path.join(out_dir, "rank1_left"), "w").close()
        os._exit(0)          # leaves between steps, before any collective
    try:
        st.step(grads(0, rank))
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 - any collective error is the detection
        outcome = "error: " + type(e).__name__
    open(os.path.join(out_dir, "rank0_outcome"), "w").write(outcome)
    os._exit(0)


def test_rank_failure_is_detected(tmp_path, oracle_mod):
    world = 2
    ctx = mp.start_processes(_failing_worker, args=(world, _free_port(), str(tmp_path)),
                             nprocs=world, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(60)
    assert (tmp_path / "rank1_left").exists()
    outcome = (tmp_path / "rank0_outcome").read_text()
    assert outcome.startswith("error"), outcome
