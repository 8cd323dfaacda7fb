"""Row-sharded data-parallel packed step over NCCL (one process per GPU).

The reference has no multi-GPU code.  Its update needs, for word (n, k),
only row n's data (v_row[n], row_exp[n], the row max), column k's data
(v_col[k], col_exp[k], the column max) and three global scalars (sum_v_inv,
the step salt, lr) -- so the optimizer half of the backward shards by rows:

  1. reduce-scatter (sum) of the bf16 dW partials: rank r receives rows
     [r*S, (r+1)*S) of the summed gradient (S = ceil(N / P); N padded to P*S);
  2. v-hat on the shard: v_row of its rows, the shard's column sums of g^2 and
     the sum of its v_row; one all-reduce of those K+1 floats; v_col and
     sum_v_inv finished identically on every rank;
  3. the fused packed step on the shard, with global row offsets (the SR
     hash position uses the global row) and the same salt on every rank;
  4. all-reduce(max) of the column maxima, one all-gather of (row maxima,
     v_row), one all-gather of the packed words (4 B/param, in place when N
     divides evenly); every rank re-derives the bf16 forward weight from the
     gathered words (what the step emitted).
rebalance() then runs replicated on identical inputs, so exponents, seeds and
words stay identical on every rank with no further traffic.

The compute goes through a kernel backend: `CudaKernels` (this package's
CUDA library) in production; tests may pass another object with the same
methods to check the orchestration on CPU ranks (gloo).
"""
import torch
import torch.distributed as dist

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
             sum_v_inv, coh_pre, lr_t, eps_t, salt, row0):
        _pb._step_launch(params, packed, grad, wbuf, row_exp, col_exp, row_max, col_max, v_row,
                         v_col, sum_v_inv, coh_pre, lr_t, eps_t, salt, row0=row0)

    @staticmethod
    def materialize(packed, row_exp, col_exp, out, mantissa_bias):
        _pb.materialize_packed_bf16(packed, row_exp, col_exp, out, mantissa_bias)

    @staticmethod
    def salt(device):
        return _pb._get_step_counter(device)


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

    Every rank holds the full (replicated) layer.  `step(grad_local)` takes this
    rank's bf16 dW partial [N, K] and leaves every rank with identical packed
    words, exponents, v_row/v_col/sum_v_inv and bf16 forward weight; coh_pre is
    kept up to date only on each rank's own rows (it is per-word state that no
    other rank reads).
    """

    def __init__(self, layer, group=None, kernels=None):
        self.layer = layer
        self.group = group
        self.kernels = kernels if kernels is not None else CudaKernels()
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        N, K = layer.packed_w.shape
        self.N, self.K = N, K
        self.S = (N + self.P - 1) // self.P
        self.r0 = self.rank * self.S
        self.r1 = min(N, self.r0 + self.S)
        dev = layer.packed_w.device
        pad = self.P * self.S
        self.grad_pad = torch.zeros(pad, K, dtype=torch.bfloat16, device=dev)
        self.grad_shard = torch.empty(self.S, K, dtype=torch.bfloat16, device=dev)
        self.words_pad = torch.zeros(pad, K, dtype=torch.int32, device=dev)
        self.red = torch.zeros(K + 1, dtype=torch.float32, device=dev)
        self.wshard = torch.empty(self.S, K, dtype=torch.bfloat16, device=dev)
        self.loc_w = torch.zeros(self.S, K, dtype=torch.int32, device=dev)
        # row maxima and v_row of the shard travel together in one all-gather
        self.loc_rv = torch.zeros(2, self.S, dtype=torch.int32, device=dev)
        self.all_rv = torch.zeros(self.P, 2, self.S, dtype=torch.int32, device=dev)
        self.even = (N == pad)   # no padding: collectives work in place on the layer's tensors
        self.step_events = None   # optional [_, start, end] CUDA events around the shard's step

    @torch.no_grad()
    def step(self, grad_local):
        L, kern, g = self.layer, self.kernels, self.group
        N, K, S, r0, r1 = self.N, self.K, self.S, self.r0, self.r1
        n_loc = r1 - r0
        wbuf, rmax, cmax = L._ensure_buffers()
        # 1. reduce-scatter of the bf16 gradient over rows
        if self.even and grad_local.is_contiguous():
            _reduce_scatter(self.grad_shard, grad_local, g)
        else:
            self.grad_pad[:N].copy_(grad_local)
            _reduce_scatter(self.grad_shard, self.grad_pad, g)
        gs = self.grad_shard[:n_loc]
        # 2. v-hat: shard partials, one all-reduce, replicated finish
        track = bool(L.track_rebalance)
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
        # 3. the packed step on this rank's rows
        if L.optimizer_kind != 'adamw':
            raise NotImplementedError("the row-sharded step implements the adamw path")
        params = _pb.adamw_params(
            alpha=L.alpha, beta1=L.beta1, weight_decay=L.weight_decay, step_cap=L.step_cap,
            v_scale=L.v_scale, precond_p=L.precond_p, gf_consol=L.gf_consol,
            drift_cancel_C=L.drift_cancel_C, alpha_v_fast=L.alpha_v_fast, wd_sv=L.wd_sv,
            wd_sf=L.wd_sf, mass_preserve=L.mass_preserve_v, apply_chase=L.apply_chase,
            track_rebalance=L.track_rebalance, gf_trust_delta_sq=L.gf_trust_delta_sq,
            use_cohpre=L._coh_pre is not None, mantissa_bias=L.MANTISSA_BIAS)
        ev = self.step_events
        if ev is not None:
            ev[1].record()
        if n_loc > 0:
            kern.step(params, L.packed_w[r0:r1], gs, self.wshard[:n_loc], L.row_exp[r0:r1], L.col_exp,
                      rmax[r0:r1], cmax, L.v_row[r0:r1], L.v_col, L._sum_v_inv,
                      None if L._coh_pre is None else L._coh_pre[r0:r1], L._lr_buf, L._eps_buf,
                      kern.salt(L.packed_w.device), r0)
        if ev is not None:
            ev[2].record()
        # 4. maxima, words and v_row back to every rank; forward weight re-derived
        if track:
            dist.all_reduce(cmax, op=dist.ReduceOp.MAX, group=g)
        self.loc_rv[0, :n_loc].copy_(rmax[r0:r1])
        self.loc_rv[1, :n_loc].copy_(L.v_row[r0:r1].view(torch.int32))
        _all_gather(self.all_rv, self.loc_rv, g)
        if track:
            rmax.copy_(self.all_rv[:, 0].reshape(-1)[:N])
        L.v_row.copy_(self.all_rv[:, 1].reshape(-1)[:N].view(torch.float32))
        if self.even:
            _all_gather(L.packed_w, L.packed_w[r0:r1], g)     # in place
        else:
            self.loc_w[:n_loc].copy_(L.packed_w[r0:r1])
            _all_gather(self.words_pad, self.loc_w, g)
            L.packed_w.copy_(self.words_pad[:N])
        kern.materialize(L.packed_w, L.row_exp, L.col_exp, wbuf, L.MANTISSA_BIAS)
