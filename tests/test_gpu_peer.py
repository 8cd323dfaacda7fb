"""The peer-memory kernels of the data-parallel step, on one GPU.

Every launch here is a single kernel that waits on nothing but flags that are
already set (or, in the timeout test, on a flag that nothing sets, with a
0.2 s limit): no test makes two launches wait on one another.  The "peers"
are ordinary allocations of this GPU, which the kernels cannot tell from
CUDA IPC mappings of other GPUs; the other ranks' pushes are stood in for by
filling this rank's receive buffer.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def lib():
    from concord_b200 import _abi
    return _abi.load()


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _sync(lib, n_ranks, rank=0, preset=None, timeout_s=5.0):
    """Flag arrays for n_ranks (all local), own flags optionally preset."""
    from concord_b200 import _abi
    flags = [torch.zeros(64, dtype=torch.int32, device=DEV) for _ in range(n_ranks)]
    if preset is not None:
        flags[rank][:n_ranks] = preset
    table = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=DEV)
    state = torch.zeros(4, dtype=torch.int32, device=DEV)
    s = _abi.PeerSync(flags=flags[rank].data_ptr(), peer_flags=table.data_ptr(),
                      state=state.data_ptr(), rank=rank, n_ranks=n_ranks,
                      timeout_ns=int(timeout_s * 1e9))
    return s, (flags, table, state)


def _grads(P, N, K, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return [(torch.randn(N, K, generator=g) * 10.0 ** float(q - 2)).to(torch.bfloat16).to(DEV)
            for q in range(P)]


def _push(lib, grad, S, recvs, sync):
    N, K = grad.shape
    table = torch.tensor([r.data_ptr() for r in recvs], dtype=torch.int64, device=DEV)
    rc = lib.concord_peer_push_rows(ctypes.c_void_p(grad.data_ptr()), N, K, S, ctypes.c_void_p(table.data_ptr()),
                                    ctypes.byref(sync), _stream())
    assert rc == 0, lib.concord_last_error().decode()
    torch.cuda.synchronize()


@pytest.mark.parametrize("P,N,rank", [(1, 37, 0), (2, 64, 1), (3, 100, 0), (3, 100, 2), (4, 9, 3), (8, 1000, 5)])
def test_push_rows_delivers_each_shard_to_its_owner(lib, P, N, rank):
    K = 264
    S = (N + P - 1) // P
    grad = _grads(1, N, K, seed=N + rank)[0]
    recvs = [torch.full((P * S, K), -7.0, dtype=torch.bfloat16, device=DEV) for _ in range(P)]
    sync, (flags, _, state) = _sync(lib, P, rank=rank)
    _push(lib, grad, S, recvs, sync)
    for q in range(P):
        lo, hi = min(N, q * S), min(N, (q + 1) * S)
        if q == rank:
            assert bool((recvs[q].float() == -7.0).all())        # nothing sent to itself
        else:
            blk = recvs[q][rank * S: rank * S + (hi - lo)]
            assert torch.equal(blk.view(torch.int16), grad[lo:hi].view(torch.int16)), q
            rest = torch.cat([recvs[q][:rank * S], recvs[q][rank * S + (hi - lo):]])
            assert bool((rest.float() == -7.0).all())
        assert int(flags[q][rank]) == 1                           # announced to every rank
    assert state.tolist()[:3] == [1, 0, 0]


def _reduce_vhat(lib, own, recv, S, n, sync, outs):
    K = recv.shape[1]
    out = torch.full((max(n, 1), K), -7.0, dtype=torch.bfloat16, device=DEV)
    ws = torch.zeros(lib.concord_vhat_workspace_bytes(max(n, 1), K), dtype=torch.uint8, device=DEV)
    rc = lib.concord_peer_reduce_vhat(
        ctypes.c_void_p(own.data_ptr()), ctypes.c_void_p(recv.data_ptr()), S, K, n, ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(outs["v_row"].data_ptr()), 0.999, 0.001, ctypes.c_void_p(outs["rmax"].data_ptr()),
        ctypes.c_void_p(outs["cmax"].data_ptr()), ctypes.c_void_p(outs["salt"].data_ptr()),
        ctypes.c_void_p(outs["red"].data_ptr()), ctypes.c_void_p(outs["red"].data_ptr() + 4 * K),
        ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.byref(sync), _stream())
    assert rc == 0, lib.concord_last_error().decode()
    torch.cuda.synchronize()
    return out


def _outs(n, K, seed=9):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return dict(v_row=(torch.rand(max(n, 1), generator=g) * 1e-4).to(DEV),
                rmax=torch.full((max(n, 1),), 9, dtype=torch.int32, device=DEV),
                cmax=torch.full((K,), 9, dtype=torch.int32, device=DEV),
                salt=torch.zeros(1, dtype=torch.int32, device=DEV),
                red=torch.full((K + 1,), -1.0, device=DEV))


def _recv_and_own(P, rank, S, K, seed):
    """This rank's receive buffer (blocks of the other ranks filled) and own rows."""
    parts = _grads(P, S, K, seed)
    recv = torch.full((P * S, K), -7.0, dtype=torch.bfloat16, device=DEV)
    for q in range(P):
        if q != rank:
            recv[q * S:(q + 1) * S] = parts[q]
    return recv, parts[rank].contiguous(), parts


@pytest.mark.parametrize("P,rank", [(1, 0), (3, 1), (8, 7)])
@pytest.mark.parametrize("S,n", [(300, 300), (130, 129), (130, 0)])
def test_reduce_vhat_equals_sum_then_vhat_partial(lib, P, rank, S, n):
    """The fused rank-order sum + v-hat partials == the fp32 rank-order sum
    rounded to bf16, then concord_vhat_partial on it, bit for bit."""
    K = 264
    recv, own, parts = _recv_and_own(P, rank, S, K, seed=P * 10 + S)
    sync, (flags, _, state) = _sync(lib, P, rank=rank, preset=3)
    state[0] = 3                     # the epoch the pushes announced
    got = _outs(n, K)
    out = _reduce_vhat(lib, own, recv, S, n, sync, got)
    ref = _outs(n, K)
    if n:
        acc = parts[0][:n].float()
        for q in range(1, P):
            acc = acc + parts[q][:n].float()
        ref_g = acc.to(torch.bfloat16)
        assert torch.equal(out[:n].view(torch.int16), ref_g.view(torch.int16))
        ws = torch.zeros(lib.concord_vhat_workspace_bytes(n, K), dtype=torch.uint8, device=DEV)
        assert lib.concord_vhat_partial(
            ctypes.c_void_p(ref_g.data_ptr()), K, n, K, ctypes.c_void_p(ref["v_row"].data_ptr()), 0.999, 0.001,
            ctypes.c_void_p(ref["rmax"].data_ptr()), ctypes.c_void_p(ref["cmax"].data_ptr()),
            ctypes.c_void_p(ref["salt"].data_ptr()), ctypes.c_void_p(ref["red"].data_ptr()),
            ctypes.c_void_p(ref["red"].data_ptr() + 4 * K), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
            _stream()) == 0
        torch.cuda.synchronize()
    else:   # no rows: zero partials, column maxima zeroed, salt bumped
        ref["red"].zero_()
        ref["cmax"].zero_()
        ref["salt"] += 1
    for k in ref:
        assert torch.equal(ref[k], got[k]), k
    assert state.tolist()[:3] == [3, 0, 0]            # waiting does not advance the epoch


def test_reduce_vhat_wait_runs_out_and_reports(lib):
    """A rank whose push never arrives: the wait gives up after 0.2 s, the
    error word is set, nothing is written, and the context stays usable."""
    P, S, K = 2, 64, 64
    recv, own, parts = _recv_and_own(P, 0, S, K, seed=5)
    sync, (flags, _, state) = _sync(lib, P, rank=0, timeout_s=0.2)
    state[0] = 1
    flags[0][0] = 1                   # this rank announced; rank 1 never does
    got = _outs(S, K)
    before = {k: v.clone() for k, v in got.items()}
    out = _reduce_vhat(lib, own, recv, S, S, sync, got)
    assert int(state[2]) == 1
    assert bool((out.float() == -7.0).all())
    for k in got:
        assert torch.equal(got[k], before[k]), k
    out = _reduce_vhat(lib, own, recv, S, S, sync, got)      # sticky: skips at once
    assert bool((out.float() == -7.0).all())
    state[2] = 0                                               # cleared, rank 1 arrived: works
    flags[0][1] = 1
    out = _reduce_vhat(lib, own, recv, S, S, sync, got)
    acc = (parts[0].float() + parts[1].float()).to(torch.bfloat16)
    assert torch.equal(out.view(torch.int16), acc.view(torch.int16))


def test_epochs_are_exact_on_grids_larger_than_one_wave(lib):
    """Many more blocks than fit on the GPU at once (and a 2-D grid): the push
    advances the epoch by exactly one, and the fused kernel waits for exactly
    the current epoch (the other rank's flag says 1, not more), so a block
    that computed another epoch would run out of time and set the error word."""
    P, K, S = 2, 512, 128 * 300
    N = P * S
    grad = _grads(1, N, K, seed=11)[0]
    recvs = [torch.zeros(P * S, K, dtype=torch.bfloat16, device=DEV) for _ in range(P)]
    sync, (flags, _, state) = _sync(lib, P, rank=0, timeout_s=1.0)
    _push(lib, grad, S, recvs, sync)                           # 1184 blocks
    assert state.tolist()[:3] == [1, 0, 0] and int(flags[1][0]) == 1
    flags[0][1] = 1                                            # rank 1's push of epoch 1
    recv, own, parts = _recv_and_own(P, 0, S, K, seed=12)
    got = _outs(S, K)
    out = _reduce_vhat(lib, own, recv, S, S, sync, got)       # 2 x 300 blocks
    assert state.tolist()[:3] == [1, 0, 0]
    acc = (parts[0].float() + parts[1].float()).to(torch.bfloat16)
    assert torch.equal(out.view(torch.int16), acc.view(torch.int16))


def test_peer_calls_reject_bad_arguments(lib):
    grad = _grads(1, 8, 64, seed=3)[0]
    sync, keep = _sync(lib, 2)
    table = torch.tensor([grad.data_ptr()] * 2, dtype=torch.int64, device=DEV)
    args = lambda N, K, S: (ctypes.c_void_p(grad.data_ptr()), N, K, S, ctypes.c_void_p(table.data_ptr()),
                            ctypes.byref(sync), _stream())
    assert lib.concord_peer_push_rows(*args(8, 60, 4)) == -2      # K not a multiple of 8
    assert lib.concord_peer_push_rows(*args(8, 64, 3)) == -2      # S * n_ranks < N
    sync.n_ranks = 9
    assert lib.concord_peer_push_rows(*args(8, 64, 4)) == -1


@pytest.mark.parametrize("shape,row0", [((64, 256), 0), ((37, 260), 50), ((13, 70), 3)])
def test_step_sharded_stores_the_weight_into_every_peer(shape, row0):
    """concord_step_sharded == concord_step on the words, and each peer buffer
    receives exactly rows row0..row0+N of the weight (vector and generic paths)."""
    from concord_b200 import ConcordLinearPackedB, packed_b as pb
    n, K = shape
    NT = row0 + n + 5
    torch.manual_seed(0)
    layer = ConcordLinearPackedB(K, NT, bias=False, device=DEV, lr=0.05)
    layer.load_weights(torch.randn(NT, K) * 0.05)
    g = (torch.randn(NT, K) * 3e-2).to(torch.bfloat16).to(DEV)
    layer.optimizer_step(g)     # v-hat state and coh_pre away from their initial values
    P = pb.adamw_params(v_scale=0.0, precond_p=0.5, drift_cancel_C=layer.drift_cancel_C,
                        mass_preserve=True, gf_trust_delta_sq=1.0, use_cohpre=True)
    r = slice(row0, row0 + n)

    def run(peers):
        st = {k: getattr(layer, k)[r].clone() for k in ("packed_w", "row_exp", "_coh_pre")}
        w = torch.zeros(n, K, dtype=torch.bfloat16, device=DEV)
        rm = torch.zeros(n, dtype=torch.int32, device=DEV)
        cm = torch.zeros(K, dtype=torch.int32, device=DEV)
        salt = torch.full((1,), 7, dtype=torch.int32, device=DEV)
        pb._step_launch(P, st["packed_w"], g[r].contiguous(), w, st["row_exp"], layer.col_exp, rm, cm,
                        layer.v_row[r], layer.v_col, layer._sum_v_inv, st["_coh_pre"], layer._lr_buf,
                        layer._eps_buf, salt, row0=row0, wbuf_peers=peers)
        torch.cuda.synchronize()
        return st, w, rm, cm

    ref = run(None)
    bufs = [torch.full((NT, K), 3.0, dtype=torch.bfloat16, device=DEV) for _ in range(2)]
    peers = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=DEV)
    got = run(peers)
    for a, b in zip(ref[0].values(), got[0].values()):
        assert torch.equal(a, b)
    for a, b in zip(ref[1:], got[1:]):
        assert torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                           b.view(torch.int16) if b.dtype == torch.bfloat16 else b)
    for b in bufs:
        assert torch.equal(b[r].view(torch.int16), ref[1].view(torch.int16))
        assert bool((b[:row0].float() == 3.0).all()) and bool((b[row0 + n:].float() == 3.0).all())



def _slots(P, count):
    bufs = [torch.zeros(2 * P * count, dtype=torch.int32, device=DEV) for _ in range(P)]
    table = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=DEV)
    return bufs, table


@pytest.mark.parametrize("P", [1, 3, 8])
def test_peer_allreduce_sum_and_max(lib, P):
    """Rank 0 of P: the other ranks' contributions are pre-placed in its slots
    (what their pushes would have written); the result is the rank-order fp32
    sum / int32 max, and rank 0's own input lands in every rank's slots."""
    count, cap = 1000, 1003
    g = torch.Generator(device="cpu").manual_seed(P)
    vals = [(torch.randn(count, generator=g) * 10.0 ** (q % 4)).to(DEV) for q in range(P)]
    ivals = [torch.randint(-1000, 1000, (count,), generator=g, dtype=torch.int32).to(DEV) for q in range(P)]
    for op, data in ((0, vals), (1, ivals)):
        sync, (flags, _, state) = _sync(lib, P, rank=0, preset=1 << 20)
        bufs, table = _slots(P, cap)
        e = int(state[0]) + 1
        half = (e & 1) * P * cap
        for q in range(1, P):
            bufs[0][half + q * cap: half + q * cap + count] = data[q].view(torch.int32)
        x = data[0].clone()
        rc = lib.concord_peer_allreduce(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()), count, op,
                                        ctypes.c_void_p(table.data_ptr()), cap, ctypes.byref(sync), _stream())
        assert rc == 0, lib.concord_last_error().decode()
        torch.cuda.synchronize()
        if op == 0:
            acc = data[0].clone()
            for q in range(1, P):
                acc = acc + data[q]
        else:
            acc = torch.stack(data).max(0).values
        assert torch.equal(x, acc)
        for b in bufs:   # the push of rank 0 into every rank's row 0
            assert torch.equal(b[half: half + count], data[0].view(torch.int32))
        assert int(state[0]) == 1 and int(state[2]) == 0


def test_peer_allreduce_barrier_and_errors(lib):
    sync, (flags, _, state) = _sync(lib, 2, rank=1, preset=1 << 20)
    bufs, table = _slots(2, 4)
    assert lib.concord_peer_allreduce(None, None, 0, 0, ctypes.c_void_p(table.data_ptr()), 4,
                                      ctypes.byref(sync), _stream()) == 0
    torch.cuda.synchronize()
    assert int(state[0]) == 1 and int(flags[0][1]) == 1
    x = torch.zeros(8, device=DEV)
    assert lib.concord_peer_allreduce(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()), 8, 0,
                                      ctypes.c_void_p(table.data_ptr()), 4, ctypes.byref(sync), _stream()) == -2
    assert lib.concord_peer_allreduce(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()), 4, 5,
                                      ctypes.c_void_p(table.data_ptr()), 4, ctypes.byref(sync), _stream()) == -1
