"""Row-sharded data-parallel packed step over NCCL (one process per GPU).

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
     weight (2 B/param, in place when N divides evenly).
`rebalance()` then runs on each shard with the shared column decisions (the
Philox offsets use global rows), so column exponents stay identical across
ranks.  Per step the wire carries 2 B/param each way; `gather_state()`
assembles the full packed state on every rank when it is needed
(checkpoints, consolidated_weight()).

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

    @staticmethod
    def rebalance(packed, row_exp, col_exp, row_max, col_max, row_hwm, col_hwm, seed, max_m,
                  exp_max, exp_min, row0, n_total, fired_out=None):
        _pb.rebalance_packed(packed, row_exp, col_exp, row_max, col_max, MAX_M=max_m,
                             EXP_MAX=exp_max, EXP_MIN=exp_min, seed_buf=seed, allow_tickdown=False,
                             row_hwm=row_hwm, col_hwm=col_hwm, fired_out=fired_out,
                             bump_seed=True, row0=row0, n_total=n_total)


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
    sum_v_inv.  Call `rebalance()` (not the layer's) after each step, and
    `gather_state()` before reading the full packed state.
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
        self.even = (N == pad)   # no padding: collectives work in place on the layer's tensors
        self.grad_pad = None if self.even else torch.zeros(pad, K, dtype=torch.bfloat16, device=dev)
        self.grad_shard = torch.empty(self.S, K, dtype=torch.bfloat16, device=dev)
        self.wpad = None if self.even else torch.zeros(pad, K, dtype=torch.bfloat16, device=dev)
        self.red = torch.zeros(K + 1, dtype=torch.float32, device=dev)
        self.wshard = torch.zeros(self.S, K, dtype=torch.bfloat16, device=dev)
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
        # 3. the packed step on this rank's rows (writes its rows of the forward weight)
        if L.optimizer_kind != 'adamw':
            raise NotImplementedError("the row-sharded step implements the adamw path")
        params = _pb.adamw_params(
            alpha=L.alpha, beta1=L.beta1, weight_decay=L.weight_decay, step_cap=L.step_cap,
            v_scale=L.v_scale, precond_p=L.precond_p, gf_consol=L.gf_consol,
            drift_cancel_C=L.drift_cancel_C, alpha_v_fast=L.alpha_v_fast, wd_sv=L.wd_sv,
            wd_sf=L.wd_sf, mass_preserve=L.mass_preserve_v, apply_chase=L.apply_chase,
            track_rebalance=L.track_rebalance, gf_trust_delta_sq=L.gf_trust_delta_sq,
            use_cohpre=L._coh_pre is not None, mantissa_bias=L.MANTISSA_BIAS)
        wdst = wbuf[r0:r1] if self.even else self.wshard[:n_loc]
        ev = self.step_events
        if ev is not None:
            ev[1].record()
        if n_loc > 0:
            kern.step(params, L.packed_w[r0:r1], gs, wdst, L.row_exp[r0:r1], L.col_exp,
                      rmax[r0:r1], cmax, L.v_row[r0:r1], L.v_col, L._sum_v_inv,
                      None if L._coh_pre is None else L._coh_pre[r0:r1], L._lr_buf, L._eps_buf,
                      kern.salt(L.packed_w.device), r0)
        if ev is not None:
            ev[2].record()
        # 4. column maxima and the forward weight to every rank
        if track:
            dist.all_reduce(cmax, op=dist.ReduceOp.MAX, group=g)
        if self.even:
            _all_gather(wbuf, wbuf[r0:r1], g)                 # in place
        else:
            _all_gather(self.wpad, self.wshard, g)
            wbuf.copy_(self.wpad[:N])

    @torch.no_grad()
    def rebalance(self, fired_out=None):
        """The layer's rebalance() on this rank's rows, with the shared column maxima."""
        L = self.layer
        if L.allow_tickdown:
            raise NotImplementedError("tick-down needs whole-matrix column medians; "
                                      "not supported on a row-sharded layer")
        rmax, cmax = L._row_max_buf, L._col_max_buf
        r0, r1 = self.r0, self.r1
        if r1 <= r0:
            L._reb_seed.add_(1)
            return
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
