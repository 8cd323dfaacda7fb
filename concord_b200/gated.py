"""GatedRebalance: one device-side gate and two batched launches for every layer.

Mirrors the trainer utility of the reference (notebook/src/concord_winner.py:
206-262): every layer's per-row / per-column maxima live in slices of two
shared tensors; when any of them exceeds MAX_M, every layer runs its
rebalance, otherwise none does.  The reference decides on the host (a
reduction and a device->host read each step) and then launches each layer's
rebalance; here `concord_rebalance_gated` keeps the decision on the device
(three launches whatever the number of layers, no host synchronisation, so
the whole optimizer step can be captured in one CUDA graph).  As in the
reference, the first call only wires the shared buffers.
"""
import ctypes

import torch

from . import _abi
from . import packed_b as _pb


class RebLayer(ctypes.Structure):
    """Mirror of `concord_reb_layer` (include/concord_b200.h)."""
    _fields_ = [
        ("packed", ctypes.c_void_p), ("ldp", ctypes.c_int64),
        ("row_exp", ctypes.c_void_p), ("col_exp", ctypes.c_void_p),
        ("row_max", ctypes.c_void_p), ("col_max", ctypes.c_void_p),
        ("row_hwm", ctypes.c_void_p), ("col_hwm", ctypes.c_void_p),
        ("seed", ctypes.c_void_p),
        ("max_m", ctypes.c_int32), ("exp_max", ctypes.c_int32), ("exp_min", ctypes.c_int32),
        ("pad0", ctypes.c_int32),
        ("N", ctypes.c_int64), ("K", ctypes.c_int64), ("row0", ctypes.c_int64),
        ("N_total", ctypes.c_int64), ("decide_off", ctypes.c_int64),
        ("rt", ctypes.c_void_p), ("ct", ctypes.c_void_p), ("fired", ctypes.c_void_p),
        ("rowlist", ctypes.c_void_p), ("collist", ctypes.c_void_p),
    ]


class GatedRebalance:
    """Drop-in for `for m in layers: m.rebalance()`: call the instance after
    the backward.  Returns a device int32[1] flag (1 when the layers ran; the
    reference returns a host bool, which would need a synchronisation).
    `fires` / `calls` count as in the reference (`fires` reads the device)."""

    def __init__(self, layers):
        self.layers = [m for m in (layers or []) if hasattr(m, "rebalance")]
        self.MAX_M = max((getattr(m, "MAX_M", 24000) for m in self.layers), default=24000)
        self.row_all = None
        self.col_all = None
        self.calls = 0
        self._fire_count = None

    @property
    def fires(self):
        return 0 if self._fire_count is None else int(self._fire_count.item())

    def _wire(self):
        """Back every layer's max buffers with slices of two shared tensors and
        build the device descriptors.  Call again after a layer's buffers are
        replaced (e.g. a new packed_w tensor)."""
        for m in self.layers:
            if getattr(m, "allow_tickdown", False):
                raise NotImplementedError("GatedRebalance: tick-down layers are not supported")
        dev = self.layers[0].packed_w.device
        rs = [m._row_max_buf.shape[0] for m in self.layers]
        cs = [m._col_max_buf.shape[0] for m in self.layers]
        self.row_all = torch.zeros(sum(rs), dtype=torch.int32, device=dev)
        self.col_all = torch.zeros(sum(cs), dtype=torch.int32, device=dev)
        ro = co = 0
        for m, n, k in zip(self.layers, rs, cs):
            m._row_max_buf = self.row_all[ro:ro + n]; ro += n
            m._col_max_buf = self.col_all[co:co + k]; co += k
        lib = _pb._lib()
        descs = (RebLayer * len(self.layers))()
        self._ws = []
        off = 0
        for d, m in zip(descs, self.layers):
            N, K = m.packed_w.shape
            ws = torch.zeros(lib.concord_rebalance_gated_layer_workspace_bytes(N, K), dtype=torch.uint8,
                             device=dev)
            self._ws.append(ws)
            _abi.check(lib.concord_rebalance_gated_layer_layout(N, K, ctypes.c_void_p(ws.data_ptr()),
                                                                 ctypes.byref(d)),
                       "concord_rebalance_gated_layer_layout")
            d.packed, d.ldp = m.packed_w.data_ptr(), m.packed_w.stride(0)
            d.row_exp, d.col_exp = m.row_exp.data_ptr(), m.col_exp.data_ptr()
            d.row_max, d.col_max = m._row_max_buf.data_ptr(), m._col_max_buf.data_ptr()
            d.row_hwm, d.col_hwm = m._row_max_hwm.data_ptr(), m._col_max_hwm.data_ptr()
            d.seed = m._reb_seed.data_ptr()
            d.max_m, d.exp_max, d.exp_min = int(m.MAX_M), int(m.EXP_MAX), int(m.EXP_MIN)
            d.N, d.K, d.row0, d.N_total, d.decide_off = N, K, 0, N, off
            off += N + K
        self._total = off
        raw = bytes(descs)
        self._descs = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(dev)
        self._gate = torch.zeros(2, dtype=torch.int32, device=dev)
        self._fired = torch.zeros(1, dtype=torch.int32, device=dev)
        self._fire_count = torch.zeros(1, dtype=torch.int64, device=dev)

    @torch.no_grad()
    def __call__(self):
        if not self.layers:
            return None
        self.calls += 1
        if self.row_all is None:
            if getattr(self.layers[0], "_row_max_buf", None) is None:
                return None                   # no step has run yet
            self._wire()                      # first wired call: nothing is rebalanced
            return self._fired
        _abi.check(_pb._lib().concord_rebalance_gated(
            ctypes.c_void_p(self._descs.data_ptr()), len(self.layers), self._total,
            _pb._ptr(self.row_all), self.row_all.numel(), _pb._ptr(self.col_all), self.col_all.numel(),
            int(self.MAX_M), _pb._ptr(self._gate), _pb._ptr(self._fired),
            _pb._stream(self.row_all.device)), "concord_rebalance_gated")
        self._fire_count += self._fired
        return self._fired
