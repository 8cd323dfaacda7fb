"""Row-sharded data-parallel packed step (one process per GPU).

The reference has no multi-GPU code.  Its update needs, for word (n, k),
only row n's data (v_row[n], row_exp[n], the row max), column k's data
(v_col[k], col_exp[k], the column max) and three global scalars (sum_v_inv,
the step salt, lr) -- so the optimizer half of the backward shards by rows,
and so does the optimizer state (ZeRO-style: rank r owns rows
[r*S, (r+1)*S), S = ceil(N / P), of the packed words, coh_pre, v_row and the
row exponents):

  1. reduce-scatter (sum) of the bf16 dW partials over rows;
  2. v-hat on the shard: v_row of its rows, the shard's column sums of g^2 and
     the sum of its v_row; one all-reduce of those K+1 floats; v_col and
     sum_v_inv finished identically on every rank;
  3. the fused packed step on the shard, with global row offsets (the SR
     hash position uses the global row) and the same salt on every rank; it
     writes the shard's rows of the bf16 forward weight;
  4. all-reduce(max) of the column maxima; all-gather of the bf16 forward
     weight.

Two transports carry steps 1 and 4:
  * "peer" (NCCL process group, all ranks on one node): CUDA IPC mappings of
    every rank's receive buffer, forward-weight buffer, all-reduce slots and
    rendezvous flags; NCCL carries nothing per step.  Step 1 is a push kernel
    (each rank stores the other shards' rows of its dW into their owners'
    receive buffers over NVLink, then announces it) and a local kernel that
    waits (bounded) for every rank's announcement and sums the rows in fp32
    in rank order (rounded once to bf16: the same bits for any rank count),
    fused with the shard's v-hat partials.  The K+1-float and the K-int
    all-reduces go through peer slots (rank-order sums); step 4's all-gather
    is fused into the step kernel, which stores each bf16 weight into every
    rank's buffer as it computes it.
  * "collective": NCCL (or gloo) reduce-scatter and all-gather.  The bf16
    ring sum of NCCL rounds after every addition, so for P > 2 its gradient
    differs from the fp32 sum.
`rebalance()` then runs on each shard with the shared column decisions (the
Philox offsets use global rows), so column exponents stay identical across
ranks.  Per step the wire carries 2 B/param each way; `gather_state()`
assembles the full packed state on every rank when it is needed
(checkpoints, consolidated_weight()).

The compute goes through a kernel backend: `CudaKernels` (this package's
CUDA library) in production; tests may pass another object with the same
methods to check the orchestration on CPU ranks (gloo).
"""
import ctypes
import os

import torch
import torch.distributed as dist

from . import _abi
from . import packed_b as _pb


class CudaKernels:
    """The CUDA library calls the sharded step needs."""

    @staticmethod
    def vhat_partial(grad, v_row, beta2, row_max, col_max, bump_salt, col_sum, vsum):
        N, K = grad.shape
        lib = _pb._lib()
        ws = _pb._workspace("vhat", lib.concord_vhat_workspace_bytes(N, K), grad.device)
        salt = _pb._get_step_counter(grad.device) if bump_salt else None
        _pb._abi.check(lib.concord_vhat_partial(
            _pb._ptr(grad), grad.stride(0), N, K, _pb._ptr(v_row), float(beta2), 1.0 - float(beta2),
            _pb._ptr(row_max), _pb._ptr(col_max), _pb._ptr(salt), _pb._ptr(col_sum), _pb._ptr(vsum),
            _pb._ptr(ws), ws.numel(), _pb._stream(grad.device)), "concord_vhat_partial")

    @staticmethod
    def vhat_finish(col_sum, vsum, v_col, sum_v_inv, beta2):
        _pb._abi.check(_pb._lib().concord_vhat_finish(
            _pb._ptr(col_sum), _pb._ptr(vsum), _pb._ptr(v_col), _pb._ptr(sum_v_inv), v_col.numel(),
            float(beta2), 1.0 - float(beta2), _pb._stream(v_col.device)), "concord_vhat_finish")

    @staticmethod
    def step(params, packed, grad, wbuf, row_exp, col_exp, row_max, col_max, v_row, v_col,
             sum_v_inv, coh_pre, lr_t, eps_t, salt, row0, wbuf_peers=None):
        _pb._step_launch(params, packed, grad, wbuf, row_exp, col_exp, row_max, col_max, v_row,
                         v_col, sum_v_inv, coh_pre, lr_t, eps_t, salt, row0=row0,
                         wbuf_peers=wbuf_peers)

    @staticmethod
    def materialize(packed, row_exp, col_exp, out, mantissa_bias):
        _pb.materialize_packed_bf16(packed, row_exp, col_exp, out, mantissa_bias)

    @staticmethod
    def salt(device):
        return _pb._get_step_counter(device)

    @staticmethod
    def rebalance(packed, row_exp, col_exp, row_max, col_max, row_hwm, col_hwm, seed, max_m,
                  exp_max, exp_min, row0, n_total, fired_out=None):
        _pb.rebalance_packed(packed, row_exp, col_exp, row_max, col_max, MAX_M=max_m,
                             EXP_MAX=exp_max, EXP_MIN=exp_min, seed_buf=seed, allow_tickdown=False,
                             row_hwm=row_hwm, col_hwm=col_hwm, fired_out=fired_out,
                             bump_seed=True, row0=row0, n_total=n_total)


class _DeviceArray:
    """A device allocation seen through __cuda_array_interface__ (zero-copy)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


def _wrap_bf16(ptr, shape, device):
    t = torch.as_tensor(_DeviceArray(ptr, shape, "<i2"), device=device)
    assert t.data_ptr() == int(ptr), "zero-copy wrap of a peer buffer failed"
    return t.view(torch.bfloat16)


class PeerTransport:
    """CUDA IPC buffers of one row-sharded layer: every rank's receive buffer
    for the reduce-scatter (P blocks of S rows), its forward-weight buffer,
    the all-reduce slots and the rendezvous flags.

    Allocated with the library's own cudaMalloc (an IPC handle covers a whole
    allocation), exported as IPC handles, exchanged over the process group
    and opened on every other rank.  `close()` unmaps and frees them
    collectively.
    """

    def __init__(self, N, K, S, group, device, timeout_s=10.0, slot_count=None):
        lib = _pb._lib()
        self.lib, self.group, self.device = lib, group, device
        self.P, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.P > 8:
            raise ValueError("the peer transport handles at most 8 ranks")
        self.N, self.K, self.S = N, K, S
        self._own, self._opened = [], []
        self.slot_count = int(slot_count if slot_count is not None else K + 1)
        with torch.cuda.device(device):
            mine = [self._alloc(self.P * S * K * 2),              # receive buffer
                    self._alloc(N * K * 2),                       # forward weight
                    self._alloc(256),                             # flags (one int32 per rank)
                    self._alloc(2 * self.P * self.slot_count * 4)]  # all-reduce slots
            hb = lib.concord_ipc_handle_bytes()
            handles = []
            for p in mine:
                buf = ctypes.create_string_buffer(hb)
                _abi.check(lib.concord_ipc_export(ctypes.c_void_p(p), buf), "concord_ipc_export")
                handles.append(buf.raw)
            every = [None] * self.P
            dist.all_gather_object(every, handles, group=group)
            table = []
            for q in range(self.P):
                if q == self.rank:
                    table.append(mine)
                    continue
                row = []
                for h in every[q]:
                    p = ctypes.c_void_p()
                    _abi.check(lib.concord_ipc_open(h, ctypes.byref(p)), "concord_ipc_open")
                    self._opened.append(p.value)
                    row.append(p.value)
                table.append(row)
        i64 = dict(dtype=torch.int64, device=device)
        self.recv_table = torch.tensor([table[q][0] for q in range(self.P)], **i64)
        self.wbuf_peers = torch.tensor([table[q][1] for q in range(self.P) if q != self.rank], **i64)
        self.flag_table = torch.tensor([table[q][2] for q in range(self.P)], **i64)
        self.slot_table = torch.tensor([table[q][3] for q in range(self.P)], **i64)
        self.recv = mine[0]
        self.wbuf = _wrap_bf16(mine[1], (N, K), device)
        self.state = torch.zeros(4, dtype=torch.int32, device=device)
        self.sync = _abi.PeerSync(flags=mine[2], peer_flags=self.flag_table.data_ptr(),
                                  state=self.state.data_ptr(), rank=self.rank, n_ranks=self.P,
                                  timeout_ns=int(timeout_s * 1e9))

    def _alloc(self, nbytes):
        p = ctypes.c_void_p()
        _abi.check(self.lib.concord_peer_alloc(nbytes, ctypes.byref(p)), "concord_peer_alloc")
        self._own.append(p.value)
        return p.value

    def push(self, grad):
        """Send every other rank its shard's rows of this rank's dW."""
        _abi.check(self.lib.concord_peer_push_rows(
            _pb._ptr(grad), self.N, self.K, self.S, ctypes.c_void_p(self.recv_table.data_ptr()),
            ctypes.byref(self.sync), _pb._stream(self.device)), "concord_peer_push_rows")

    def reduce_vhat(self, own_rows, n_rows, out, v_row, beta2, row_max, col_max, salt, col_sum, vsum):
        """Wait for every rank's push, then the rank-order sum of the shard's dW
        rows fused with the shard's v-hat partials."""
        lib, K = self.lib, self.K
        ws = _pb._workspace("vhat", lib.concord_vhat_workspace_bytes(max(n_rows, 1), K), self.device)
        _abi.check(lib.concord_peer_reduce_vhat(
            _pb._ptr(own_rows), ctypes.c_void_p(self.recv), self.S, K, n_rows, _pb._ptr(out),
            _pb._ptr(v_row), float(beta2), 1.0 - float(beta2), _pb._ptr(row_max), _pb._ptr(col_max),
            _pb._ptr(salt), _pb._ptr(col_sum), _pb._ptr(vsum), _pb._ptr(ws), ws.numel(),
            ctypes.byref(self.sync), _pb._stream(self.device)), "concord_peer_reduce_vhat")

    def allreduce(self, t, op):
        """In-place all-reduce of a small fp32 (sum, rank order) or int32 (max) tensor."""
        n = 0 if t is None else t.numel()
        _abi.check(self.lib.concord_peer_allreduce(
            _pb._ptr(t), _pb._ptr(t), n, op, ctypes.c_void_p(self.slot_table.data_ptr()),
            self.slot_count, ctypes.byref(self.sync), _pb._stream(self.device)),
            "concord_peer_allreduce")

    def error(self):
        """Non-zero when a cross-GPU wait ran out (reads the device; synchronises)."""
        return int(self.state[2].item())

    def close(self):
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)          # no rank still reads or writes a peer buffer
        for p in self._opened:
            self.lib.concord_ipc_close(ctypes.c_void_p(p))
        dist.barrier(group=self.group)          # every mapping of our buffers is gone
        for p in self._own:
            self.lib.concord_peer_free(ctypes.c_void_p(p))
        self._own, self._opened = None, []


def params_of(L):
    """The layer's launch scalars for the adamw packed step."""
    if L.optimizer_kind != 'adamw':
        raise NotImplementedError("the row-sharded step implements the adamw path")
    return _pb.adamw_params(
        alpha=L.alpha, beta1=L.beta1, weight_decay=L.weight_decay, step_cap=L.step_cap,
        v_scale=L.v_scale, precond_p=L.precond_p, gf_consol=L.gf_consol,
        drift_cancel_C=L.drift_cancel_C, alpha_v_fast=L.alpha_v_fast, wd_sv=L.wd_sv,
        wd_sf=L.wd_sf, mass_preserve=L.mass_preserve_v, apply_chase=L.apply_chase,
        track_rebalance=L.track_rebalance, gf_trust_delta_sq=L.gf_trust_delta_sq,
        use_cohpre=L._coh_pre is not None, mantissa_bias=L.MANTISSA_BIAS, device=L.packed_w.device)


def _reduce_scatter(out, inp, group):
    if dist.get_backend(group) == "nccl":
        dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.SUM, group=group)
    else:  # gloo has no reduce-scatter: all-reduce then keep this rank's rows
        buf = inp.clone()
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
        r = dist.get_rank(group)
        out.copy_(buf.view(dist.get_world_size(group), *out.shape)[r])


def _all_gather(out, inp, group):
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, inp, group=group)
    else:
        parts = list(out.view(dist.get_world_size(group), *inp.shape).unbind(0))
        dist.all_gather(parts, inp.contiguous(), group=group)


class RowShardedStep:
    """Data-parallel optimizer half of one ConcordLinearPackedB's backward.

    Every rank holds a full-size layer; rank r keeps rows [r0, r1) of its packed
    state current.  `step(grad_local)` takes this rank's bf16 dW partial [N, K];
    afterwards every rank holds the same bf16 forward weight, v_col and
    sum_v_inv.  Call `gather_state()` before reading the full packed state.

    Constructing it registers the layer as data-parallel: from then on the
    layer's own autograd backward hands its local dW to `step()` (instead of
    stepping on it), and `layer.rebalance()` runs `rebalance()` here, so a
    model trains data-parallel through `loss.backward()` with no extra calls.
    Calling `step()` by hand as well would step the layer a second time.
    `close()` unregisters the layer.
    """

    def __init__(self, layer, group=None, kernels=None, transport=None, timeout_s=10.0):
        self.layer = layer
        self.group = group
        self.kernels = kernels if kernels is not None else CudaKernels()
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        N, K = layer.packed_w.shape
        self.N, self.K = N, K
        self.S = (N + self.P - 1) // self.P
        self.r0 = min(N, self.rank * self.S)
        self.r1 = min(N, self.r0 + self.S)
        dev = layer.packed_w.device
        if transport is None:
            transport = os.environ.get("CONCORD_DP_TRANSPORT") or (
                "peer" if (dist.get_backend(group) == "nccl" and isinstance(self.kernels, CudaKernels)
                           and self.P <= 8 and K % 8 == 0) else "collective")
        if transport not in ("peer", "collective"):
            raise ValueError(f"transport must be 'peer' or 'collective', not {transport!r}")
        self.transport = transport
        pad = self.P * self.S
        self.even = (N == pad)   # no padding: collectives work in place on the layer's tensors
        self.grad_shard = torch.empty(self.S, K, dtype=torch.bfloat16, device=dev)
        self.red = torch.zeros(K + 1, dtype=torch.float32, device=dev)
        self.step_events = None   # optional [_, start, end] CUDA events around the shard's step
        # optional dict name -> CUDA event, recorded after each phase of the peer
        # transport's step (instrumentation for the bench's phase breakdown)
        self.phase_events = None
        # column maxima all-reduced once per step for many layers
        # (DeferredColumnMaxima) instead of after this layer's step
        self.deferred = None
        self.peer = None
        if transport == "peer":
            wbuf, _, _ = layer._ensure_buffers()
            self.peer = PeerTransport(N, K, self.S, group, dev, timeout_s=timeout_s)
            self.peer.wbuf.copy_(wbuf)
            layer._bf16_weight_buf = self.peer.wbuf      # peers store their rows into it
            self.grad_pad = self.wpad = self.wshard = None
        else:
            self.grad_pad = None if self.even else torch.zeros(pad, K, dtype=torch.bfloat16, device=dev)
            self.wpad = None if self.even else torch.zeros(pad, K, dtype=torch.bfloat16, device=dev)
            self.wshard = torch.zeros(self.S, K, dtype=torch.bfloat16, device=dev)
        key = layer.packed_w.data_ptr()
        if key in _pb._SHARDED:
            raise RuntimeError("this layer already has a RowShardedStep; close() it first")
        _pb._SHARDED[key] = self

    def check(self):
        """Raise if a cross-GPU wait of the peer transport ran out (synchronises)."""
        if self.peer is not None and self.peer.error():
            raise RuntimeError("concord: a cross-GPU wait ran out in the peer reduce-scatter "
                               "(a rank did not reach the step within the timeout)")

    def close(self):
        """Collective: give the layer an ordinary forward-weight buffer back and
        release the peer mappings.  The layer steps on its own again afterwards."""
        if _pb._SHARDED.get(self.layer.packed_w.data_ptr()) is self:
            del _pb._SHARDED[self.layer.packed_w.data_ptr()]
        if self.peer is not None:
            L = self.layer
            L._bf16_weight_buf = self.peer.wbuf.clone()
            self.peer.close()
            self.peer = None

    @torch.no_grad()
    def step(self, grad_local):
        if self.deferred is not None:
            self.deferred.pending = True
        L, kern, g = self.layer, self.kernels, self.group
        N, K, S, r0, r1 = self.N, self.K, self.S, self.r0, self.r1
        n_loc = r1 - r0
        wbuf, rmax, cmax = L._ensure_buffers()
        track = bool(L.track_rebalance)
        if self.peer is not None:
            # 1+2. the shard's dW rows of every other rank pushed over NVLink;
            # one kernel waits for them and sums them in rank order together
            # with the shard's v-hat partials; the K+1 partials all-reduced
            # through the peer slots; v_col / sum_v_inv finished locally
            ph = self.phase_events or {}
            grad_local = grad_local.contiguous()
            self.peer.push(grad_local)
            if "push" in ph:
                ph["push"].record()
            self.peer.reduce_vhat(grad_local[r0:r1], n_loc, self.grad_shard, L.v_row[r0:r1],
                                  L.adafactor_beta2, rmax[r0:r1] if track else None,
                                  cmax if track else None, kern.salt(L.packed_w.device),
                                  self.red[:K], self.red[K:])
            if "reduce_vhat" in ph:
                ph["reduce_vhat"].record()
            self.peer.allreduce(self.red, _abi.PEER_SUM_F32)
            if "allreduce_vhat" in ph:
                ph["allreduce_vhat"].record()
            kern.vhat_finish(self.red[:K], self.red[K:], L.v_col, L._sum_v_inv, L.adafactor_beta2)
            self._step_shard(params_of(L), n_loc, wbuf[r0:r1], rmax, cmax)
            # 4. column maxima through the peer slots.  The rendezvous inside
            # completes on a rank only after every rank's step kernel has
            # finished (its weight rows stored into every buffer), so no rank
            # reads its forward weight before all rows have landed; a rank
            # without column tracking still meets the others (count 0).  The
            # same ordering protects the receive buffers: a rank pushes its next
            # dW only after the v-hat all-reduce, i.e. after every rank finished
            # reading this one.
            if self.deferred is None:
                self.peer.allreduce(cmax if track else None, _abi.PEER_MAX_I32)
                if "allreduce_cmax" in ph:
                    ph["allreduce_cmax"].record()
            return
        # 1. reduce-scatter of the bf16 gradient over rows
        if self.even and grad_local.is_contiguous():
            _reduce_scatter(self.grad_shard, grad_local, g)
        else:
            self.grad_pad[:N].copy_(grad_local)
            _reduce_scatter(self.grad_shard, self.grad_pad, g)
        gs = self.grad_shard[:n_loc]
        # 2. v-hat: shard partials, one all-reduce, replicated finish
        if n_loc > 0:
            kern.vhat_partial(gs, L.v_row[r0:r1], L.adafactor_beta2,
                              rmax[r0:r1] if track else None, cmax if track else None, True,
                              self.red[:K], self.red[K:])
        else:
            self.red.zero_()
            cmax.zero_()
            kern.salt(L.packed_w.device).add_(1)
        dist.all_reduce(self.red, op=dist.ReduceOp.SUM, group=g)
        kern.vhat_finish(self.red[:K], self.red[K:], L.v_col, L._sum_v_inv, L.adafactor_beta2)
        # 3. the packed step on this rank's rows (writes its rows of the forward weight)
        wdst = wbuf[r0:r1] if self.even else self.wshard[:n_loc]
        self._step_shard(params_of(L), n_loc, wdst, rmax, cmax)
        # 4. column maxima and the forward weight to every rank
        if track and self.deferred is None:
            dist.all_reduce(cmax, op=dist.ReduceOp.MAX, group=g)
        if self.even:
            _all_gather(wbuf, wbuf[r0:r1], g)                 # in place
        else:
            _all_gather(self.wpad, self.wshard, g)
            wbuf.copy_(self.wpad[:N])

    def _step_shard(self, params, n_loc, wdst, rmax, cmax):
        L, kern, r0, r1 = self.layer, self.kernels, self.r0, self.r1
        ev = self.step_events
        if ev is not None:
            ev[1].record()
        if n_loc > 0:
            kern.step(params, L.packed_w[r0:r1], self.grad_shard[:n_loc], wdst, L.row_exp[r0:r1],
                      L.col_exp, rmax[r0:r1], cmax, L.v_row[r0:r1], L.v_col, L._sum_v_inv,
                      None if L._coh_pre is None else L._coh_pre[r0:r1], L._lr_buf, L._eps_buf,
                      kern.salt(L.packed_w.device), r0,
                      **({} if self.peer is None else {"wbuf_peers": self.peer.wbuf_peers}))
        if ev is not None:
            ev[2].record()

    @torch.no_grad()
    def rebalance(self, fired_out=None):
        """The layer's rebalance() on this rank's rows, with the shared column maxima."""
        if self.deferred is not None:
            self.deferred.sync()      # a no-op unless a step ran since the last sync
        L = self.layer
        if L.allow_tickdown:
            raise NotImplementedError("tick-down needs whole-matrix column medians; "
                                      "not supported on a row-sharded layer")
        rmax, cmax = L._row_max_buf, L._col_max_buf
        r0, r1 = self.r0, self.r1
        # a rank that owns no rows still applies the shared column decisions
        # (column exponents, column high-watermarks, the seed): zero rows
        self.kernels.rebalance(L.packed_w[r0:r1], L.row_exp[r0:r1], L.col_exp, rmax[r0:r1], cmax,
                               L._row_max_hwm[r0:r1], L._col_max_hwm, L._reb_seed, L.MAX_M,
                               L.EXP_MAX, L.EXP_MIN, r0, self.N, fired_out)

    @torch.no_grad()
    def gather_state(self):
        """Make the packed words, row exponents, v_row, row high-watermarks and
        coh_pre identical on every rank (each rank contributes its rows)."""
        L, g, S, N = self.layer, self.group, self.S, self.N
        r0, r1 = self.r0, self.r1
        n_loc = r1 - r0
        tensors = [L.packed_w, L.row_exp, L.v_row, L._row_max_hwm]
        if L._coh_pre is not None:
            tensors.append(L._coh_pre)
        for t in tensors:
            if self.even:
                _all_gather(t, t[r0:r1], g)
            else:
                loc = torch.zeros((S,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
                loc[:n_loc] = t[r0:r1]
                full = torch.zeros((self.P * S,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
                _all_gather(full, loc, g)
                t.copy_(full[:N])


class DeferredColumnMaxima:
    """One all-reduce of the column maxima of many row-sharded layers per step.

    Each RowShardedStep ends its step with a cross-rank rendezvous: the
    all-reduce (max) of the layer's column maxima, which rebalance() needs,
    and which, on the peer transport, is also what guarantees that every
    rank's forward-weight rows have landed before the next forward reads them.
    A model of hundreds of layers pays that rendezvous (tens of microseconds
    of waiting for the slowest rank at 8 GPUs) once per layer.  This object
    takes the steppers of one model: their layers' column-maxima buffers
    become views of one flat int32 buffer, their steps skip the per-layer
    all-reduce, and `sync()` all-reduces the flat buffer once (NCCL, max).

    `sync()` must run after the backward and before the next forward: the
    first `rebalance()` of any of these layers calls it, so a training loop
    that rebalances (or calls `sync()`) after every backward needs no other
    change.  Every rank must call it equally often (it is a collective).
    Results are identical to the per-layer all-reduce.
    """

    def __init__(self, steppers, group=None):
        steppers = list(steppers)
        if not steppers:
            raise ValueError("no steppers")
        dev = steppers[0].layer.packed_w.device
        self.group = group
        self.steppers = steppers
        self.flat = torch.zeros(sum(st.K for st in steppers), dtype=torch.int32, device=dev)
        off = 0
        for st in steppers:
            if st.deferred is not None:
                raise RuntimeError("a stepper can belong to one DeferredColumnMaxima only")
            L = st.layer
            L._ensure_buffers()
            view = self.flat[off:off + st.K]
            view.copy_(L._col_max_buf)
            L._col_max_buf = view
            st.deferred = self
            off += st.K
        self.pending = False

    @torch.no_grad()
    def sync(self):
        """All-reduce (max) every layer's column maxima; a no-op when no step ran
        since the last call."""
        if not self.pending:
            return
        dist.all_reduce(self.flat, op=dist.ReduceOp.MAX, group=self.group)
        self.pending = False

    def close(self):
        """Back to per-layer all-reduces (the layers keep their current maxima)."""
        for st in self.steppers:
            st.layer._col_max_buf = st.layer._col_max_buf.clone()
            st.deferred = None

