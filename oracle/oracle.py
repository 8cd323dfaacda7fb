"""Python (numpy + ctypes) front end of the CPU parity oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference legs, never by the concord_b200 package.
The arithmetic lives in concord_oracle.c (a restatement of the reference's
Triton kernels in concord/packed_b.py, cited per function there).  Arrays are
numpy; bf16 tensors are uint16 bit patterns.
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32


def build():
    subprocess.check_call(["make", "-s", "-C", _HERE])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        for name, res, args in [
            ("oracle_hash_uniform", ctypes.c_float, [_I32] * 3),
            ("oracle_tl_rand", ctypes.c_float, [_I32, _I32]),
            ("oracle_log2f", ctypes.c_float, [ctypes.c_float]),
            ("oracle_exp2f", ctypes.c_float, [ctypes.c_float]),
            ("oracle_f32_to_bf16", ctypes.c_uint16, [ctypes.c_float]),
        ]:
            getattr(_lib, name).restype = res
            getattr(_lib, name).argtypes = args
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dt):
    assert a.dtype == dt and a.flags["C_CONTIGUOUS"], (a.dtype, dt)
    return a


def step(params, packed, grad_bf16, wbuf, row_exp, col_exp, row_max, col_max,
         v_row, v_col, sum_v_inv, coh_pre, lr, eps, salt, row0=0, coh_stats=None):
    """In-place packed step over numpy arrays (oracle_step)."""
    N, K = packed.shape
    _c(packed, np.int32); _c(grad_bf16, np.uint16); _c(wbuf, np.uint16)
    lib().oracle_step(
        ctypes.byref(params), _p(packed), _I64(K), _p(grad_bf16), _I64(K),
        _p(wbuf), _I64(K), _p(_c(row_exp, np.int8)), _p(_c(col_exp, np.int8)),
        _p(row_max), _p(col_max), _p(v_row), _p(v_col), _p(sum_v_inv),
        _p(coh_pre), _I64(K), ctypes.c_float(lr), ctypes.c_float(eps),
        _I32(salt), _I64(N), _I64(K), _I64(row0), _p(coh_stats))


def vhat(grad_bf16, v_row, v_col, sum_v_inv, beta2=0.999):
    N, K = grad_bf16.shape
    lib().oracle_vhat(_p(_c(grad_bf16, np.uint16)), _I64(K), _I64(N), _I64(K),
                      _p(_c(v_row, np.float32)), _p(_c(v_col, np.float32)),
                      _p(_c(sum_v_inv, np.float32)), ctypes.c_float(beta2),
                      ctypes.c_float(1.0 - beta2))


def vhat_partial(grad_bf16, v_row, beta2=0.999):
    """Shard form: updates v_row; returns (column sums of g^2, sum of v_row)."""
    N, K = grad_bf16.shape
    col_sum = np.zeros(K, np.float32)
    vsum = np.zeros(1, np.float32)
    lib().oracle_vhat_ex(_p(_c(grad_bf16, np.uint16)), _I64(K), _I64(N), _I64(K),
                         _p(_c(v_row, np.float32)), None, None, ctypes.c_float(beta2),
                         ctypes.c_float(1.0 - beta2), _p(col_sum), _p(vsum))
    return col_sum, vsum


def rebalance(packed, row_exp, col_exp, row_max, col_max, row_hwm, col_hwm, seed,
              max_m=24000, exp_max=7, exp_min=-8, allow_tickdown=False, row0=0,
              n_total=None):
    N, K = packed.shape
    fired = np.zeros(1, np.int32)
    lib().oracle_rebalance(
        _p(packed), _I64(K), _p(row_exp), _p(col_exp), _p(row_max), _p(col_max),
        _p(row_hwm), _p(col_hwm), _p(_c(seed, np.int32)), _I32(max_m),
        _I32(exp_max), _I32(exp_min), _I32(int(allow_tickdown)),
        _I64(N), _I64(K), _I64(row0), _I64(N if n_total is None else n_total), _p(fired))
    return int(fired[0])


def materialize(packed, row_exp, col_exp, mantissa_bias=15, consolidated=False):
    N, K = packed.shape
    out = np.empty((N, K), np.uint16)
    lib().oracle_materialize(_p(_c(packed, np.int32)), _I64(K), _p(row_exp), _p(col_exp),
                             _p(out), _I64(K), _I64(N), _I64(K), _I32(mantissa_bias),
                             _I32(int(consolidated)))
    return out


def quantize(W, mantissa_bias=15, exp_min=-8, exp_max=7, finetune=False):
    W = np.ascontiguousarray(W, dtype=np.float32)
    N, K = W.shape
    packed = np.empty((N, K), np.int32)
    row_exp = np.empty(N, np.int8)
    col_exp = np.empty(K, np.int8)
    lib().oracle_quantize(_p(W), _I64(K), _p(packed), _I64(K), _p(row_exp), _p(col_exp),
                          _I64(N), _I64(K), _I32(mantissa_bias), _I32(exp_min),
                          _I32(exp_max), _I32(int(finetune)))
    return packed, row_exp, col_exp


def coherence(packed, C):
    N, K = packed.shape
    out = np.zeros(2, np.float64)
    lib().oracle_coherence(_p(_c(packed, np.int32)), _I64(K), _I64(N), _I64(K),
                           ctypes.c_float(C), _p(out))
    return out


def f32_to_bf16(x):
    """RNE fp32 -> bf16 bit patterns (vectorised numpy, same rule as the C side)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h):
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def step_threaded(params, packed, grad_bf16, wbuf, row_exp, col_exp, row_max, col_max,
                  v_row, v_col, sum_v_inv, coh_pre, lr, eps, salt, threads=8, row0=0):
    """oracle_step split over row blocks on host threads (ctypes drops the GIL).

    Row/col maxima are merged after the threads finish, so the result equals
    the single-threaded call."""
    import threading
    N, K = packed.shape
    bounds = np.linspace(0, N, threads + 1).astype(int)
    cms = []
    ths = []
    for a, b in zip(bounds[:-1], bounds[1:]):
        if b <= a:
            continue
        cm = np.zeros(K, np.int32)
        cms.append(cm)
        p, g, w = packed[a:b], grad_bf16[a:b], wbuf[a:b]
        cp = coh_pre[a:b] if coh_pre is not None else None

        def work(p=p, g=g, w=w, cp=cp, a=a, b=b, cm=cm):
            rm = row_max[a:b] if row_max is not None else None
            lib().oracle_step(
                ctypes.byref(params), _p(p), _I64(K), _p(g), _I64(K), _p(w), _I64(K),
                _p(row_exp[a:b]), _p(col_exp), _p(rm), _p(cm), _p(None if v_row is None else v_row[a:b]),
                _p(v_col), _p(sum_v_inv), _p(cp), _I64(K), ctypes.c_float(lr), ctypes.c_float(eps),
                _I32(salt), _I64(b - a), _I64(K), _I64(row0 + a), None)
        ths.append(threading.Thread(target=work))
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    if col_max is not None:
        np.maximum.reduce([col_max] + cms, out=col_max)
