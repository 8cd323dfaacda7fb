"""Generate the committed golden fixtures from the REFERENCE implementation.

Run in a container where the reference checkout is readable (it is not on
the GPU box; the fixtures it writes travel instead):

    TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/Concord [groups...]

It imports the unmodified reference package (`concord/packed_b.py`) and runs
its Triton kernels under Triton's CPU interpreter.  Two interpreter
primitives are pinned to a machine-independent meaning before any kernel
runs (the reference's source is not touched):

* `tl.exp2` / `tl.log2` on fp32: the interpreter calls numpy's float32
  ufuncs, whose SIMD implementations are not correctly rounded and differ
  between CPUs; here they are evaluated in extended precision and rounded
  once to fp32 (correct rounding).
* fp32 -> bf16 casts: the interpreter truncates; compiled Triton rounds to
  nearest even, which is what is recorded here.

Everything else (integer hashing, Philox, SR decisions, clamps, exponent
bookkeeping, torch host code) is the reference's own code.  Output: one
compressed .npz per fixture group in this directory.
"""
import os
import sys

import numpy as np

assert os.environ.get("TRITON_INTERPRET") == "1", "run with TRITON_INTERPRET=1"
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CONCORD_REF", "")
assert REF and os.path.isdir(os.path.join(REF, "concord")), "pass the reference checkout"
sys.path.insert(0, REF)

import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402
from triton.runtime import interpreter as _interp  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


# ---- pin the two implementation-defined interpreter primitives ----------
def _cr_unary(fn):
    def op(self, arg):
        d = arg.data
        if d.dtype == np.float32:
            r = fn(d.astype(np.longdouble)).astype(np.float32)
        else:
            r = fn(d)
        return _interp.TensorHandle(r, arg.dtype.scalar)
    return op


_interp.InterpreterBuilder.create_exp2 = _cr_unary(np.exp2)
_interp.InterpreterBuilder.create_log2 = _cr_unary(np.log2)
_orig_cast = _interp.InterpreterBuilder.cast_impl


def _cast_rne(self, src, dst_type):
    if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
        u = src.data.view(np.uint32).astype(np.uint64)
        nan = (u & 0x7FFFFFFF) > 0x7F800000
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
        return _interp.TensorHandle(r, dst_type.scalar)
    return _orig_cast(self, src, dst_type)


_interp.InterpreterBuilder.cast_impl = _cast_rne

import concord.packed_b as pb  # noqa: E402


def bf16_bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def np_(t):
    return t.detach().clone().contiguous().numpy()


def rand_state(g, N, K, sf_lim=3000, i8_lim=100):
    sf = torch.randint(-sf_lim, sf_lim + 1, (N, K), generator=g, dtype=torch.int32)
    ss = torch.randint(-i8_lim, i8_lim + 1, (N, K), generator=g, dtype=torch.int32)
    vs = torch.randint(-i8_lim, i8_lim + 1, (N, K), generator=g, dtype=torch.int32)
    return ((sf & 0xFFFF) << 16) | ((ss & 0xFF) << 8) | (vs & 0xFF)


C_STAR = pb.compute_drift_cancel_C(0.1, 0.001, mass_preserve=True)
BARE = dict(kind="adamw", alpha=0.1, beta1=0.0, weight_decay=0.0, eps=1e-10, step_cap=10.0,
            v_scale=0.0, precond_p=0.5, gf_consol=0.0, drift_cancel_C=C_STAR,
            alpha_v_fast=0.001, wd_sv=0.0, wd_sf=0.0, mass_preserve=True, apply_chase=True,
            track_rebalance=True, gf_trust_delta_sq=1.0, cohpre=True, lr=5e-3)
STEP_CASES = {
    "bare": dict(BARE),
    "nocohpre": dict(BARE, cohpre=False),
    "consol": dict(BARE, gf_consol=5.0),
    "ratio": dict(BARE, cohpre=False, ratio=True, floors=(0.6, 0.95)),
    "legacycoh": dict(BARE, fixed_coh=False),
    "wd_beta1": dict(BARE, weight_decay=0.01, wd_sv=1.0, wd_sf=0.5, beta1=0.1, gate_gain=0.7,
                     mass_preserve=False, v_scale=1.0, eps=1e-8, precond_p=0.4, step_cap=3.0,
                     gf_trust_delta_sq=0.5),
    "nochase": dict(BARE, apply_chase=False, track_rebalance=False),
    "notrust": dict(BARE, gf_trust_delta_sq=0.0, cohpre=False, v_scale=1.0, eps=1e-6),
    "sgd_mp": dict(kind="sgd", alpha=0.1, beta1=0.05, alpha_v_fast=0.001, mass_preserve=True,
                   track_rebalance=True, lr=0.02),
    "sgd": dict(kind="sgd", alpha=0.2, beta1=0.0, alpha_v_fast=0.01, mass_preserve=False,
                track_rebalance=True, lr=0.05),
}


def run_step_case(name, cfg, N=36, K=70, steps=3, seed=0):
    g = torch.Generator().manual_seed(seed)
    packed = rand_state(g, N, K)
    row_exp = torch.randint(-3, 5, (N,), generator=g, dtype=torch.int8)
    col_exp = torch.randint(-2, 3, (K,), generator=g, dtype=torch.int8)
    v_row = torch.rand(N, generator=g) * 1e-4 + 1e-6
    v_col = torch.rand(K, generator=g) * 1e-4 + 1e-6
    sum_v_inv = (1.0 / v_row.sum()).reshape(1).float()
    coh_pre = torch.rand(N, K, generator=g) if cfg.get("cohpre") else None
    wbuf = torch.zeros(N, K, dtype=torch.bfloat16)
    rec = dict(N=N, K=K, init_packed=np_(packed), row_exp=np_(row_exp), col_exp=np_(col_exp),
               v_row=np_(v_row), v_col=np_(v_col), sum_v_inv=np_(sum_v_inv),
               init_coh_pre=np_(coh_pre) if coh_pre is not None else np.zeros(0, np.float32))
    pb._USE_FIXED_COH = cfg.get("fixed_coh", True)
    pb._RATIO_COH = cfg.get("ratio", False)
    fl = cfg.get("floors", (0.9, 0.999))
    pb._RATIO_CHASE_FLOOR, pb._RATIO_LEAK_FLOOR = fl
    pb._GATE_GAIN = cfg.get("gate_gain", 1.0)
    ctr = pb._get_step_counter(torch.device("cpu"))
    for t in range(steps):
        grad = (torch.randn(N, K, generator=g) * 1e-3
                + torch.randn(N, 1, generator=g) * 5e-4).to(torch.bfloat16)
        rmax = torch.zeros(N, dtype=torch.int32)
        cmax = torch.zeros(K, dtype=torch.int32)
        salt = int(ctr.item()) + 1
        if cfg["kind"] == "sgd":
            pb.apply_packed_sgd(packed, grad, wbuf, row_exp, col_exp, rmax, cmax,
                                lr=cfg["lr"], alpha=cfg["alpha"], beta1=cfg["beta1"],
                                alpha_v_fast=cfg["alpha_v_fast"],
                                mass_preserve=cfg["mass_preserve"],
                                track_rebalance=cfg["track_rebalance"])
        else:
            pb.apply_packed_adamw(
                packed, grad, wbuf, row_exp, col_exp, rmax, cmax, lr=cfg["lr"],
                alpha=cfg["alpha"], beta1=cfg["beta1"], weight_decay=cfg["weight_decay"],
                eps=cfg["eps"], step_cap=cfg["step_cap"], v_scale=cfg["v_scale"],
                precond_p=cfg["precond_p"], gf_consol=cfg["gf_consol"],
                drift_cancel_C=cfg["drift_cancel_C"], alpha_v_fast=cfg["alpha_v_fast"],
                wd_sv=cfg["wd_sv"], wd_sf=cfg["wd_sf"], mass_preserve=cfg["mass_preserve"],
                apply_chase=cfg["apply_chase"], track_rebalance=cfg["track_rebalance"],
                v_row=v_row, v_col=v_col, sum_v_inv=sum_v_inv,
                gf_trust_delta_sq=cfg["gf_trust_delta_sq"], coh_pre=coh_pre)
        assert int(ctr.item()) == salt
        rec[f"grad{t}"] = bf16_bits(grad)
        rec[f"salt{t}"] = np.int32(salt)
        rec[f"packed{t}"] = np_(packed)
        rec[f"wbuf{t}"] = bf16_bits(wbuf)
        rec[f"rmax{t}"] = np_(rmax)
        rec[f"cmax{t}"] = np_(cmax)
        if coh_pre is not None:
            rec[f"coh_pre{t}"] = np_(coh_pre)
    pb._USE_FIXED_COH, pb._RATIO_COH, pb._GATE_GAIN = True, False, 1.0
    pb._RATIO_CHASE_FLOOR, pb._RATIO_LEAK_FLOOR = 0.9, 0.999
    rec["steps"] = np.int32(steps)
    return rec


def cfg_arrays(cfg):
    """Launch scalars of a case, stored beside its tensors."""
    keys = ["alpha", "beta1", "weight_decay", "eps", "step_cap", "v_scale", "precond_p",
            "gf_consol", "drift_cancel_C", "alpha_v_fast", "wd_sv", "wd_sf",
            "gf_trust_delta_sq", "lr", "gate_gain"]
    out = {}
    for k in keys:
        if k in cfg:
            out["cfg_" + k] = np.float64(cfg[k])
    out["cfg_kind"] = np.array(cfg["kind"])
    for b in ["mass_preserve", "apply_chase", "track_rebalance", "cohpre", "ratio"]:
        out["cfg_" + b] = np.bool_(cfg.get(b, False))
    out["cfg_fixed_coh"] = np.bool_(cfg.get("fixed_coh", True))
    fl = cfg.get("floors", (0.9, 0.999))
    out["cfg_chase_floor"], out["cfg_leak_floor"] = np.float64(fl[0]), np.float64(fl[1])
    return out


def gen_steps():
    for name, cfg in STEP_CASES.items():
        rec = run_step_case(name, cfg)
        rec.update(cfg_arrays(cfg))
        np.savez_compressed(os.path.join(OUT, f"step_{name}.npz"), **rec)
        print("step", name, "ok", flush=True)
    # tall shard: global rows >= 32768 make (n << 16) wrap into the sign bit
    rec = run_step_case("tall", BARE, N=32800, K=3, steps=1, seed=7)
    rec.update(cfg_arrays(BARE))
    np.savez_compressed(os.path.join(OUT, "step_tall.npz"), **rec)
    print("step tall ok", flush=True)


def gen_rebalance():
    """rebalance_packed (packed_b.py:1129-1190) on states with forced ticks."""
    cases = {}
    g = torch.Generator().manual_seed(11)
    N, K = 40, 70
    # tick-up: big fields, some rows/cols over MAX_M, one row pinned at EXP_MAX
    packed = rand_state(g, N, K, sf_lim=30000, i8_lim=127)
    row_exp = torch.randint(-6, 5, (N,), generator=g, dtype=torch.int8)
    row_exp[3] = 7
    col_exp = torch.randint(-4, 4, (K,), generator=g, dtype=torch.int8)
    rmax = torch.where(torch.rand(N, generator=g) < 0.3,
                       torch.randint(24001, 40000, (N,), generator=g, dtype=torch.int32),
                       torch.randint(0, 24001, (N,), generator=g, dtype=torch.int32))
    rmax[3] = 30000
    cmax = torch.where(torch.rand(K, generator=g) < 0.3,
                       torch.randint(24001, 40000, (K,), generator=g, dtype=torch.int32),
                       torch.randint(0, 24001, (K,), generator=g, dtype=torch.int32))
    cmax[5] = 24000
    cases["up"] = (packed, row_exp, col_exp, rmax, cmax, False, 41)
    # tick-down allowed: small int8 fields on most rows, maxima mostly under MAX_M
    packed = rand_state(g, N, K, sf_lim=2000, i8_lim=20)
    big = torch.rand(N, generator=g) < 0.4
    packed = torch.where(big[:, None], rand_state(g, N, K, sf_lim=2000, i8_lim=120), packed)
    row_exp = torch.randint(-6, 5, (N,), generator=g, dtype=torch.int8)
    col_exp = torch.randint(-5, 4, (K,), generator=g, dtype=torch.int8)
    rmax = torch.randint(0, 30000, (N,), generator=g, dtype=torch.int32)
    cmax = torch.randint(0, 24001, (K,), generator=g, dtype=torch.int32)
    cases["down"] = (packed, row_exp, col_exp, rmax, cmax, True, -5)
    for name, (packed, row_exp, col_exp, rmax, cmax, td, seed) in cases.items():
        rec = dict(init_packed=np_(packed), init_row_exp=np_(row_exp), init_col_exp=np_(col_exp),
                   rmax=np_(rmax), cmax=np_(cmax), allow_tickdown=np.bool_(td))
        seed_buf = torch.tensor([seed], dtype=torch.int32)
        for t in range(2):
            seed_buf.add_(1)                 # ConcordLinearPackedB.rebalance bumps first
            rec[f"seed{t}"] = np.int32(seed_buf.item())
            pb.rebalance_packed(packed, row_exp, col_exp, rmax, cmax, seed_buf=seed_buf,
                                allow_tickdown=td)
            rec[f"packed{t}"] = np_(packed)
            rec[f"row_exp{t}"] = np_(row_exp)
            rec[f"col_exp{t}"] = np_(col_exp)
        np.savez_compressed(os.path.join(OUT, f"rebalance_{name}.npz"), **rec)
        print("rebalance", name, "ok", flush=True)


def gen_layer():
    """Bare ConcordLinearPackedB on CPU: forward, self-stepping backward, rebalance."""
    torch.manual_seed(3)
    N, K = 36, 70
    layer = pb.ConcordLinearPackedB(K, N, bias=True, device="cpu", lr=5e-3)
    W0 = torch.randn(N, K) * 0.05
    layer.load_weights(W0)
    rec = dict(W0=np_(W0), packed_init=np_(layer.packed_w), row_exp_init=np_(layer.row_exp),
               wbuf_init=bf16_bits(layer._bf16_weight_buf))
    captured = {}
    orig = pb.apply_packed_adamw

    def spy(packed_w, grad_W, *a, **kw):
        captured.update(packed_before=np_(packed_w), grad=bf16_bits(grad_W),
                        v_row=np_(kw["v_row"]), v_col=np_(kw["v_col"]),
                        sum_v_inv=np_(kw["sum_v_inv"]),
                        salt=int(pb._get_step_counter(packed_w.device).item()) + 1)
        return orig(packed_w, grad_W, *a, **kw)

    pb.apply_packed_adamw = spy
    try:
        for t in range(4):
            x = torch.randn(4, 6, K)
            rec[f"x{t}"] = np_(x)
            rec[f"v_row_prev{t}"] = np_(layer.v_row)
            rec[f"v_col_prev{t}"] = np_(layer.v_col)
            y = layer(x)
            loss = (y.float() ** 2).mean()
            loss.backward()
            for k, v in captured.items():
                rec[f"{k}{t}"] = np.asarray(v)
            rec[f"loss{t}"] = np.float32(loss.item())
            rec[f"packed{t}"] = np_(layer.packed_w)
            rec[f"wbuf{t}"] = bf16_bits(layer._bf16_weight_buf)
            rec[f"coh_pre{t}"] = np_(layer._coh_pre)
            rec[f"rmax{t}"] = np_(layer._row_max_buf)
            rec[f"cmax{t}"] = np_(layer._col_max_buf)
            rec[f"bias_grad{t}"] = np_(layer.bias.grad.float())
            layer.bias.grad = None
            layer.rebalance()
            rec[f"reb_seed{t}"] = np.int32(layer._reb_seed.item())
            rec[f"packed_reb{t}"] = np_(layer.packed_w)
            rec[f"row_exp{t}"] = np_(layer.row_exp)
            rec[f"col_exp{t}"] = np_(layer.col_exp)
            rec[f"row_hwm{t}"] = np_(layer._row_max_hwm)
    finally:
        pb.apply_packed_adamw = orig
    rec["get_weight"] = bf16_bits(layer.get_weight())
    rec["consolidated"] = bf16_bits(layer.consolidated_weight())
    np.savez_compressed(os.path.join(OUT, "layer_bare.npz"), **rec)
    print("layer ok", flush=True)


def gen_quantize():
    g = torch.Generator().manual_seed(5)
    N, K = 24, 50
    W = torch.randn(N, K, generator=g) * torch.logspace(-4, 1, N)[:, None]
    W[2] = 0.0
    W[4] = W[4].clamp(-0.2, 0.2)
    W[4, 7] = 0.25                       # exact power-of-two maximum
    W[6] = W[6] * 1e3                    # clamps at EXP_MAX
    W[8, :4] = torch.tensor([0.5, -0.5, 1.5, -2.5]) * 2.0 ** -9   # ties for round-half-even
    rec = dict(W=np_(W))
    for ft in (False, True):
        layer = pb.ConcordLinearPackedB(K, N, bias=False, device="cpu")
        (layer.load_weights_finetune if ft else layer.load_weights)(W)
        tag = "ft" if ft else "base"
        rec[f"packed_{tag}"] = np_(layer.packed_w)
        rec[f"row_exp_{tag}"] = np_(layer.row_exp)
        rec[f"get_weight_{tag}"] = bf16_bits(layer.get_weight())
        rec[f"consolidated_{tag}"] = bf16_bits(layer.consolidated_weight())
    np.savez_compressed(os.path.join(OUT, "quantize.npz"), **rec)
    print("quantize ok", flush=True)


def gen_coherence_and_rng():
    g = torch.Generator().manual_seed(9)
    packed = rand_state(g, 64, 96, sf_lim=2000, i8_lim=127)

    class FakeLayer:
        pass
    fl = FakeLayer()
    fl.packed_w = packed
    fl.drift_cancel_C = C_STAR
    coh = pb.measure_coherence(fl)

    @triton.jit
    def _rng_kernel(seed_ptr, x_ptr, pos_ptr, salt_ptr, r_ptr, h_ptr, n):
        offs = tl.arange(0, 1024)
        m = offs < n
        seed = tl.load(seed_ptr)
        x = tl.load(x_ptr + offs, mask=m, other=0)
        pos = tl.load(pos_ptr + offs, mask=m, other=0)
        salt = tl.load(salt_ptr + offs, mask=m, other=0)
        tl.store(r_ptr + offs, tl.rand(seed, pos), mask=m)
        tl.store(h_ptr + offs, pb._hash_uniform(x, pos, salt), mask=m)

    n = 1000
    rec = dict(coh_packed=np_(packed), coh_C=np.float64(C_STAR), coh_mean=np.float64(coh))
    for i, seed in enumerate([0, 1, 12345, -7, 2**31 - 1]):
        x = torch.randint(-2**31, 2**31 - 1, (n,), generator=g, dtype=torch.int32)
        pos = torch.randint(-2**31, 2**31 - 1, (n,), generator=g, dtype=torch.int32)
        salt = torch.randint(-2**31, 2**31 - 1, (n,), generator=g, dtype=torch.int32)
        r = torch.empty(n)
        h = torch.empty(n)
        _rng_kernel[(1,)](torch.tensor([seed], dtype=torch.int32), x, pos, salt, r, h, n)
        rec.update({f"seed{i}": np.int32(seed), f"x{i}": np_(x), f"pos{i}": np_(pos),
                    f"salt{i}": np_(salt), f"rand{i}": np_(r), f"hash{i}": np_(h)})
    np.savez_compressed(os.path.join(OUT, "coherence_rng.npz"), **rec)
    print("coherence/rng ok", flush=True)


if __name__ == "__main__":
    which = sys.argv[2:] or ["rng", "quantize", "rebalance", "layer", "steps"]
    if "rng" in which:
        gen_coherence_and_rng()
    if "quantize" in which:
        gen_quantize()
    if "rebalance" in which:
        gen_rebalance()
    if "layer" in which:
        gen_layer()
    if "steps" in which:
        gen_steps()
