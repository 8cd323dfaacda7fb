"""Benchmark of the Concord packed-step hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (largest shape): one ConcordLinearPackedB
weight W [N=10240, K=2048] (21.0 M packed words) with bare-default flags;
its dW = dY^T X comes from M=8192 bf16 activations.  One timed "step" is the
optimizer half of the layer's backward, the path this repo rebuilds:
  concord_vhat_update (v_row/v_col/sum_v_inv, max-buffer zeroing, salt bump)
  + concord_step (the fused packed-word step)
  + concord_rebalance (decide + gated shift).
`value` = algorithmic HBM bytes of that path per step / device time:
  step 20 B/param (word r+w 8, bf16 grad 2, coh_pre r+w 8, bf16 weight 2)
  + v-hat 2 B/param (one read of the bf16 grad).
The working set (~460 MB) is larger than L2 (126 MB), so no flush is needed.
The dense GEMMs of the same layer (fwd / dX / dW) are timed beside it.
On N > 1 GPUs that layer's update is row-sharded (strong scaling of one
layer).  The same line carries, under `weak_scaling`, the whole-job training
throughput of configs 5 (Llama-style decoder, tokens/s) and 4 (SDXL UNet,
samples/s and steps/s) at this GPU count, so one run at N = 1, 2, 4, 8 gives
their weak-scaling curves (`--no-models` skips them).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M, K, N = 8192, 2048, 10240
STEP_BYTES_PER_PARAM = 20
VHAT_BYTES_PER_PARAM = 2


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                smax.append(float(f[1]))
            except ValueError:
                continue
            for nm, v in zip(names, f[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def setup_layer(n_rows, k_cols, device, seed=0):
    from concord_b200 import ConcordLinearPackedB
    g = torch.Generator(device="cpu").manual_seed(seed)
    layer = ConcordLinearPackedB(k_cols, n_rows, bias=False, device=device, lr=5e-4)
    W0 = torch.randn(n_rows, k_cols, generator=g) * 0.02
    layer.load_weights(W0)
    return layer


def make_grads(n_rows, k_cols, device, count=2, seed=1):
    """dW = dY^T X (bf16) for `count` synthetic batches; also times the layer's
    GEMMs (this package's tcgen05 kernels, and cuBLAS through torch beside them)."""
    from concord_b200 import gemm
    g = torch.Generator(device=device).manual_seed(seed)
    grads, gemm_ms = [], {}
    for i in range(count):
        X = torch.randn(M, k_cols, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
        dY = torch.randn(M, n_rows, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
        grads.append(gemm.grad_weight(dY, X) * (1.0 / M))
        if i == 0:
            W = torch.randn(n_rows, k_cols, device=device, dtype=torch.bfloat16) * 0.02
            for name, fn in (("fwd", lambda: gemm.forward(X, W)), ("dx", lambda: gemm.grad_input(dY, W)),
                             ("dw", lambda: gemm.grad_weight(dY, X)),
                             ("cublas_fwd", lambda: X @ W.T), ("cublas_dx", lambda: dY @ W),
                             ("cublas_dw", lambda: dY.T @ X)):
                for _ in range(3):
                    fn()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                for _ in range(10):
                    fn()
                e.record()
                torch.cuda.synchronize()
                gemm_ms[name] = s.elapsed_time(e) / 10
    return grads, gemm_ms


def backward_time(n_rows, k_cols, device, iters=20):
    """The whole layer backward through the drop-in API: `layer(x)` then
    `y.backward(dY)` (dX and dW GEMMs, v-hat, packed step) and `rebalance()`,
    timed with CUDA events on the stream autograd runs on (the forward is
    outside the timed region).  Host launch gaps inside the backward count."""
    layer = setup_layer(n_rows, k_cols, device, seed=3)
    g = torch.Generator(device=device).manual_seed(7)
    x = torch.randn(M, k_cols, generator=g, device=device).to(torch.bfloat16).requires_grad_(True)
    dY = (torch.randn(M, n_rows, generator=g, device=device) / M).to(torch.bfloat16)
    ts, fs = [], []
    for i in range(iters + 3):
        f0, f1, b1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        f0.record()
        y = layer(x)
        f1.record()
        y.backward(dY)
        layer.rebalance()
        b1.record()
        torch.cuda.synchronize()
        if i >= 3:
            ts.append(f1.elapsed_time(b1))
            fs.append(f0.elapsed_time(f1))
    x.grad = None
    return statistics.mean(ts), statistics.mean(fs)


SHARDED = None
STEP_TRAFFIC_PER_PARAM = (83.988224e6 + 29.4656e6) / (4096 * 2048)


def optimizer_step(layer, grad, coh_stats=None, ev=None):
    """The timed unit: v-hat + fused packed step + rebalance of one layer
    (on N > 1 GPUs: the row-sharded data-parallel step, collectives included)."""
    if ev is not None:
        ev[0].record()
    if SHARDED is not None:
        SHARDED.step_events = ev
        SHARDED.step(grad)
        SHARDED.rebalance()
    else:
        layer.optimizer_step(grad, coh_stats=coh_stats, step_events=ev)
        layer.rebalance()


def kernel_times(layer, grad, reps):
    """Mean duration of the packed-step launch and of the v-hat launches, each
    captured alone in a CUDA graph and replayed `reps` times between events."""
    from concord_b200 import packed_b as pb
    from concord_b200.distributed import params_of
    wbuf, rmax, cmax = layer._ensure_buffers()
    P = params_of(layer)
    salt = pb._get_step_counter(layer.packed_w.device)

    def step_only():
        pb._step_launch(P, layer.packed_w, grad, wbuf, layer.row_exp, layer.col_exp, rmax, cmax,
                        layer.v_row, layer.v_col, layer._sum_v_inv, layer._coh_pre, layer._lr_buf,
                        layer._eps_buf, salt)

    def vhat_only():
        pb.vhat_update(grad, layer.v_row, layer.v_col, layer._sum_v_inv, layer.adafactor_beta2,
                       row_max=rmax, col_max=cmax, bump_salt=True)

    out = []
    for fn in (step_only, vhat_only):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        out.append(a.elapsed_time(b) / reps)
    return tuple(out)


def bench_ours(args, rank, world, device):
    global SHARDED
    n_rows, k_cols = args.rows, args.cols
    layer = setup_layer(n_rows, k_cols, device)
    grads, gemm_ms = make_grads(n_rows, k_cols, device, seed=1 + rank)
    if world > 1:
        from concord_b200.distributed import RowShardedStep
        SHARDED = RowShardedStep(layer)
    params = n_rows * k_cols
    bytes_step = params * (STEP_BYTES_PER_PARAM + VHAT_BYTES_PER_PARAM)
    for i in range(args.warmup):
        optimizer_step(layer, grads[i % 2])
    torch.cuda.synchronize()
    # kernel timing pass (eager, CUDA events around the v-hat and step launches;
    # on N > 1 also after every phase of the peer transport)
    n_ev = min(args.steps, 200)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n_ev)]
    names = ("push", "reduce_vhat", "allreduce_vhat", "allreduce_cmax")
    use_ph = SHARDED is not None and SHARDED.peer is not None
    phs = [{k: torch.cuda.Event(enable_timing=True) for k in names} for _ in range(n_ev)]
    for i in range(n_ev):
        if use_ph:
            SHARDED.phase_events = phs[i]
        optimizer_step(layer, grads[i % 2], ev=evs[i])
    if use_ph:
        SHARDED.phase_events = None
    torch.cuda.synchronize()
    step_kernel_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    vhat_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    if world == 1 and args.graph:
        # the eager events above include host gaps when a launch is shorter than
        # its Python: time the step and v-hat launches as back-to-back replays of
        # one-launch CUDA graphs instead (the roofline's kernel time)
        step_kernel_ms, vhat_ms = kernel_times(layer, grads[0], reps=min(args.steps, 50))
    phases = None
    if use_ph:
        seq = [lambda i: evs[i][0], lambda i: phs[i]["push"], lambda i: phs[i]["reduce_vhat"],
               lambda i: phs[i]["allreduce_vhat"], lambda i: evs[i][1], lambda i: evs[i][2],
               lambda i: phs[i]["allreduce_cmax"]]
        labels = ("push", "reduce_vhat", "allreduce_vhat", "vhat_finish", "step", "allreduce_cmax")
        phases = {lab: statistics.mean(seq[j](i).elapsed_time(seq[j + 1](i)) for i in range(n_ev))
                  for j, lab in enumerate(labels)}
    # the timed pass replays the step as CUDA graphs (one per gradient buffer):
    # the optimizer path has no host synchronisation, so it captures whole
    graphs = None
    if args.graph:
        try:
            graphs = []
            for gbuf in grads:
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr):
                    optimizer_step(layer, gbuf)
                graphs.append(gr)
            for i in range(2):
                graphs[i % 2].replay()
            torch.cuda.synchronize()
        except Exception as ex:  # noqa: BLE001 - report and time eagerly
            print(f"[bench] graph capture unavailable ({type(ex).__name__}: {ex}); timing eagerly",
                  file=sys.stderr)
            graphs = None
            torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    time.sleep(1.5)   # let nvidia-smi start before the timed launches
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        if graphs is not None:
            graphs[i % 2].replay()
        else:
            optimizer_step(layer, grads[i % 2])
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    # end to end through the public API: every step's dW copied from pinned
    # host memory and the coherence meter read back.  The copy of step i+1
    # runs on a copy stream while step i computes (two device buffers; a
    # buffer is refilled only after the step that read it has finished).
    host_grads = [g.cpu().pin_memory() for g in grads]
    dev_grads = [torch.empty_like(grads[0]) for _ in range(2)]
    stats = [torch.zeros(2, dtype=torch.float64, device=device) for _ in range(2)]
    host_stats = [torch.zeros(2, dtype=torch.float64).pin_memory() for _ in range(2)]
    copy_stream = torch.cuda.Stream(device)
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        b = i % 2
        cur = torch.cuda.current_stream()
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(consumed[b])
            dev_grads[b].copy_(host_grads[b], non_blocking=True)
            copied[b].record(copy_stream)
        cur.wait_event(copied[b])
        stats[b].zero_()
        optimizer_step(layer, dev_grads[b], coh_stats=stats[b])
        consumed[b].record(cur)
        host_stats[b].copy_(stats[b], non_blocking=True)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    copy_stream.wait_event(e0)
    for i in range(args.steps):
        e2e_step(i)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if SHARDED is not None:
        SHARDED.check()   # a cross-GPU wait that ran out would have skipped work: no number then
    t = torch.tensor([ms, e2e_ms, step_kernel_ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, step_kernel_ms = t.tolist()
    if phases is not None:   # max over ranks, like every other multi-GPU time
        pt = torch.tensor(list(phases.values()), device=device)
        dist.all_reduce(pt, op=dist.ReduceOp.MAX)
        phases = dict(zip(phases.keys(), pt.tolist()))
    return dict(ms=ms, e2e_ms=e2e_ms, step_kernel_ms=step_kernel_ms, vhat_ms=vhat_ms,
                bytes_step=bytes_step, params=params, gemm_ms=gemm_ms, clocks=clk,
                h2d=grads[0].numel() * 2, d2h=16, graphs=graphs is not None, phases=phases)


def oracle_sample(rows, k_cols, seed=3):
    """A bounded CPU sample of the same workload: `rows` rows of W and dW."""
    from oracle import oracle
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((rows, k_cols)) * 0.02).astype(np.float32)
    packed, rexp, cexp = oracle.quantize(W)
    grad = oracle.f32_to_bf16((rng.standard_normal((rows, k_cols)) * 1e-3).astype(np.float32))
    return oracle, packed, rexp, cexp, grad


def cpu_step_sample(oracle, packed, rexp, cexp, grad, row0, v_row, v_col, svi, coh, wbuf, rm, cm):
    from concord_b200.packed_b import adamw_params, compute_drift_cancel_C
    P = adamw_params(alpha=0.1, v_scale=0.0, precond_p=0.5,
                     drift_cancel_C=compute_drift_cancel_C(0.1, 0.001), mass_preserve=True,
                     gf_trust_delta_sq=1.0, use_cohpre=True)
    oracle.vhat(grad, v_row, v_col, svi)
    oracle.step(P, packed, grad, wbuf, rexp, cexp, rm, cm, v_row, v_col, svi, coh, 5e-4, 1e-10, 7,
                row0=row0)


def cpu_baseline(rows=2048, threads=1, reps=1):
    """Time the CPU restatement (oracle port) on `rows` x K of the workload."""
    oracle, packed, rexp, cexp, grad = oracle_sample(rows, K)
    chunks = np.array_split(np.arange(rows), threads)
    state = []
    for c in chunks:
        sl = slice(int(c[0]), int(c[-1]) + 1)
        n = sl.stop - sl.start
        state.append((np.ascontiguousarray(packed[sl]), rexp[sl].copy(), cexp, np.ascontiguousarray(grad[sl]),
                      sl.start, np.zeros(n, np.float32), np.zeros(K, np.float32), np.ones(1, np.float32),
                      np.ones((n, K), np.float32), np.zeros((n, K), np.uint16), np.zeros(n, np.int32),
                      np.zeros(K, np.int32)))
    t0 = time.perf_counter()
    for _ in range(reps):
        ths = [threading.Thread(target=cpu_step_sample, args=(oracle,) + s) for s in state]
        for t in ths:
            t.start()
        for t in ths:
            t.join()
    dt = (time.perf_counter() - t0) / reps
    bytes_ = rows * K * (STEP_BYTES_PER_PARAM + VHAT_BYTES_PER_PARAM)
    return bytes_ / dt / 1e9, dt


def ref_cpu_rule(rows, threads, steps=2):
    """Time the reference's own CPU update rule, ConcordRef.step
    (experiments/cpu_dynamics/concord_ref.py:107-156, installed unmodified under
    baseline/_ref), on `rows` x K of the workload with `threads` torch threads.
    Bare mapping: gate, noise and evaporation off, lr constant.  Returns
    (GB/s in this bench's algorithmic bytes per parameter, s/step), or None when
    the reference is not installed."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "experiments")):
        return None
    if ref not in sys.path:
        sys.path.append(ref)
    from experiments.cpu_dynamics.concord_ref import ConcordRef
    old = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        g = torch.Generator().manual_seed(0)
        lin = torch.nn.Linear(K, rows, bias=False)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(rows, K, generator=g) * 0.02)
        lin.weight.grad = (torch.randn(rows, K, generator=g) * 1e-3).to(torch.bfloat16).float()
        opt = ConcordRef(lin, lr=5e-4, total_steps=1000, warmup=0, gate=False, noise=False, kappa=0.0,
                         lr_min_frac=1.0)
        opt.step()                                   # warm-up
        t0 = time.perf_counter()
        for _ in range(steps):
            opt.step()
        dt = (time.perf_counter() - t0) / steps
    finally:
        torch.set_num_threads(old)
    return rows * K * (STEP_BYTES_PER_PARAM + VHAT_BYTES_PER_PARAM) / dt / 1e9, dt


def chargpt_cpu_baseline(threads, steps=3, batch=64):
    """BASELINE config 3's model on the host CPU with the reference's CPU
    optimizer (ConcordRef on the Linears, its SGD-momentum on the rest), fp32:
    steps/s on `threads` torch threads, or None without the reference."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "experiments")):
        return None
    if ref not in sys.path:
        sys.path.append(ref)
    from experiments.cpu_dynamics.concord_ref import ConcordRef
    import workloads
    old = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        torch.manual_seed(0)
        data = workloads.MarkovChars(n_chains=256, length=600, device="cpu")
        model = workloads.CharGPT()
        opt = ConcordRef(model, lr=5e-4, total_steps=2000, warmup=100, gate=False, noise=False, kappa=0.0)
        times = []
        for it in range(steps + 1):
            x, y = data.batch(batch, 256)
            t0 = time.perf_counter()
            loss = model(x, y)
            loss.backward()
            opt.step()
            opt.zero_grad()
            if it:
                times.append(time.perf_counter() - t0)
    finally:
        torch.set_num_threads(old)
    return 1.0 / statistics.mean(times)


def bench_chargpt(args, cores):
    """Config 3 end to end on one GPU: steps/s over the run, loss curve."""
    import workloads
    steps = args.steps
    torch.cuda.reset_peak_memory_stats()
    r = workloads.train_chargpt(steps=steps, graph=args.graph)
    d = {"metric": "char-GPT (config 3) train steps/s", "unit": "steps/s", "n_gpus": 1, "steps": steps,
         "warmup": 10, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
         "dtype": "bf16 autocast; packed int32 words", "data": "synthetic: order-2 Markov chain, 65 symbols, "
         "Dirichlet(0.3) rows, seed 0", "config": {"workload": "config 3: 6L/6H/384d char-GPT, ctx 256, batch 64, "
         "Concord on all Linears, SGD(0.9) on embeddings/norms, lr 5e-4", "seq_len": 256, "global_batch": 64},
         "value": r["steps_per_s"], "ms_per_step": r["ms_per_step"],
         "tokens_per_s": r["steps_per_s"] * r["tokens_per_step"], "losses": r["losses"],
         "entropy_floor_nats": r["entropy_floor"], "concord_params": r["concord_params"],
         "aux_params": r["aux_params"], "peak_mem_gb": torch.cuda.max_memory_allocated() / 1e9,
         "cuda_graph": r["cuda_graph"],
         "timing": "CUDA events around each training step (one CUDA graph replay after 10 eager steps "
                   "unless --no-graph), mean over steps 10.."}
    if not args.no_cpu_baseline:
        v1 = chargpt_cpu_baseline(1, steps=1)
        if v1 is not None:
            d["cpu_baseline"] = {"value": v1, "unit": "steps/s", "cores": 1, "kind": "reference",
                                 "sample": "the same model in fp32 on the host with ConcordRef.step (2-D weights), 1 step"}
            d["cpu_baseline_all_cores"] = {"value": chargpt_cpu_baseline(cores, steps=2), "unit": "steps/s",
                                           "cores": cores, "kind": "reference", "sample": "same, all threads, 2 steps"}
    emit(d)


def bench_llama(args, rank, world, steps=None, warmup=None, ret=False):
    """Config 5: weak-scaling data-parallel training step (whole job tokens/s).
    With `ret` the line is returned (rank 0; None elsewhere) instead of printed."""
    import workloads
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    torch.cuda.reset_peak_memory_stats()
    r = workloads.train_llama_dp(steps=steps, warmup=warmup, batch_per_gpu=args.batch,
                                 n_layer=args.layers, graph=args.graph)
    ms = statistics.mean(r["ms"])
    mem = torch.tensor([torch.cuda.max_memory_allocated() / 1e9], device="cuda")
    if world > 1:
        dist.all_reduce(mem, op=dist.ReduceOp.MAX)
    if rank != 0:
        return None
    d = {"metric": "Llama-style decoder (config 5) data-parallel train tokens/s", "unit": "tokens/s",
          "n_gpus": world, "steps": steps, "warmup": warmup, "higher_is_better": True,
          "scaling": "weak", "vs_baseline": None, "dtype": "bf16 autocast; packed int32 words",
          "data": "synthetic: uniform random token ids, vocab 32000",
          "config": {"workload": f"config 5: {args.layers}-layer d=2048 16-head SwiGLU-5504 decoder, seq 2048, "
                                 f"{args.batch} sequences per GPU (global batch {args.batch * world})",
                     "seq_len": 2048, "global_batch": args.batch * world,
                     "parallelism": f"dp{world}: row-sharded packed step per layer inside loss.backward()"},
          "value": r["tokens_per_step"] / (ms * 1e-3), "ms_per_step": ms,
          "ms_per_step_all": r["ms"], "loss_first_last": [r["losses"][0], r["losses"][-1]],
          "concord_params": r["concord_params"], "peak_mem_gb_max_rank": float(mem.item()),
          "cuda_graph": args.graph,
          "timing": "CUDA events around one training step (forward, backward with the packed steps, aux update, "
                    "rebalance; replayed as one CUDA graph unless --no-graph), barrier before, max over ranks"}
    if ret:
        return d
    emit(d)


def bench_sdxl(args, rank, world, steps=None, warmup=None, ret=False):
    """Config 4: SDXL-architecture UNet training steps, weak scaling.
    With `ret` the line is returned (rank 0; None elsewhere) instead of printed."""
    import workloads
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    batch = args.batch if args.batch != 8 else 4
    r = workloads.train_sdxl_dp(steps=steps, warmup=warmup, batch_per_gpu=batch, gate=not args.nogate,
                                ckpt=args.ckpt, graph=args.graph, channels_last=not args.nchw)
    ms = statistics.mean(r["ms"])
    mem = torch.tensor([r["peak_gb"], r["state_gb"]], device="cuda")
    if world > 1:
        dist.all_reduce(mem, op=dist.ReduceOp.MAX)
    if rank != 0:
        return None
    d = {"metric": "SDXL UNet train steps/s", "unit": "samples/s", "n_gpus": world, "steps": steps,
          "warmup": warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
          "dtype": "bf16 autocast; packed int32 words", "data": "synthetic: latents, text context, pooled ~ N(0,1), "
          "t ~ U{0..999}, epsilon-prediction MSE",
          "config": {"workload": f"config 4: SDXL-architecture UNet ({r['params'] / 1e9:.3f} B params, random init), "
                                 f"latents [{batch},4,128,128] per GPU, Concord on all {r['n_layers']} Linear and conv "
                                 f"layers ({r['concord_params'] / 1e9:.3f} B params), coh_pre gate "
                                 f"{'off' if args.nogate else 'on'}, activation checkpointing "
                                 f"{'on' if args.ckpt else 'off'}, lr 5e-5, "
                                 f"{'NCHW' if args.nchw else 'channels-last'} activations, conv backend "
                                 f"{__import__('concord_b200').get_conv_backend()}",
                     "global_batch": batch * world, "parallelism": f"dp{world}"},
          "value": r["samples_per_step"] / (ms * 1e-3), "steps_per_s": 1e3 / ms, "ms_per_step": ms,
          "ms_per_step_all": r["ms"], "loss_first_last": [r["losses"][0], r["losses"][-1]],
          "peak_mem_gb_max_rank": float(mem[0].item()), "state_mem_gb_max_rank": float(mem[1].item()),
          "cuda_graph": args.graph,
          "timing": "CUDA events around one training step (forward, backward with the packed steps, aux update, "
                    "rebalance; replayed as one CUDA graph unless --no-graph), barrier before, max over ranks"}
    if ret:
        return d
    emit(d)


def model_steps(args, rank, world, out=None):
    """The training steps of configs 5 and 4 on every rank, in the same run as
    the packed-step line: BASELINE's scaling half ("SDXL UNet train steps/s at
    1/2/4/8") and the data-parallel decoder, each a weak-scaling whole-job
    figure at this GPU count.  A few timed CUDA-graph replays each (the timed
    count is min(K, 10), after max(3, min(W, 5)) eager steps); a failure is
    recorded in the line instead of ending the run."""
    import gc
    steps, warmup = max(3, min(args.steps, 10)), max(3, min(args.warmup, 5))
    out = {} if out is None else out
    out["note"] = ("whole-job weak-scaling throughput at this GPU count (fixed per-GPU batch); "
                   "llama: config 5, 8 sequences x 2048 tokens per GPU; sdxl: config 4, 4 latents per GPU, "
                   "coh_pre gate on; each through loss.backward() with the row-sharded packed step "
                   f"on more than one GPU; {steps} timed steps after {warmup} eager ones")
    for name, fn in (("llama", bench_llama), ("sdxl", bench_sdxl)):
        try:
            line = fn(args, rank, world, steps=steps, warmup=warmup, ret=True)
            if line is not None:
                keep = ("value", "unit", "ms_per_step", "ms_per_step_all", "steps_per_s", "loss_first_last",
                        "peak_mem_gb_max_rank", "state_mem_gb_max_rank", "concord_params")
                out[name] = {k: line[k] for k in keep if k in line}
                out[name]["workload"] = line["config"]["workload"]
        except Exception as e:          # noqa: BLE001 - recorded in the line
            out[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
        gc.collect()
        torch.cuda.empty_cache()
    return out


def model_steps_guarded(args, rank, world, line):
    """model_steps under a wall-clock limit (CONCORD_BENCH_MODEL_LIMIT seconds,
    default 540): if the model workloads have not finished by then (a first
    run at a new GPU count that is slow to set up, or a rank stuck in a
    collective), rank 0 prints `line` with the results finished so far and an
    error note, and every rank exits 0, so the packed-step line is never lost."""
    import threading
    limit = float(os.environ.get("CONCORD_BENCH_MODEL_LIMIT", "540"))
    out = {}

    def fire():
        if rank == 0 and line is not None:
            part = dict(out)
            part["error"] = f"model workloads did not finish within {limit:.0f} s; results so far"
            line["weak_scaling"] = part
            emit(line)
        sys.stdout.flush()
        os._exit(0)
    timer = threading.Timer(limit, fire)
    timer.daemon = True
    timer.start()
    try:
        return model_steps(args, rank, world, out)
    finally:
        timer.cancel()


CONV_SHAPES = [  # B, C, O, H=W, k (SDXL UNet channel counts, stride 1)
    (2, 320, 320, 64, 3), (2, 640, 640, 32, 3), (2, 1280, 1280, 16, 3), (2, 320, 640, 64, 1),
    (8, 320, 320, 64, 3), (4, 320, 320, 128, 3)]


def bench_conv(args):
    """The conv layer's three convolutions on one GPU, per backend: implicit
    GEMM (channels-last, no column matrix), im2col + GEMMs, cuDNN.  CUDA
    events, mean of 20 runs after 3 warm-ups, eager."""
    from concord_b200 import gemm

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(20):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 20 * 1e3
    rows = []
    g = torch.Generator(device="cuda").manual_seed(0)
    shapes = CONV_SHAPES if not args.conv_shapes else \
        [tuple(int(v) for v in sh.split(",")) for sh in args.conv_shapes.split(";")]
    for B, C, O, HW, k in shapes:
        pd = k // 2
        x = torch.randn(B, C, HW, HW, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(O, C * k * k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        gy = torch.randn(B, O, HW, HW, device="cuda", generator=g).to(torch.bfloat16)
        xc, gyc = x.contiguous(memory_format=torch.channels_last), gy.contiguous(memory_format=torch.channels_last)
        wk = gemm.filter_krsc(w, C, k, k)
        w4 = w.view(O, C, k, k)
        flops = 2.0 * B * HW * HW * O * C * k * k
        r = {"shape": f"B={B} {C}->{O} {HW}x{HW} k={k}", "gflop_per_pass": flops / 1e9}
        r["implicit_fwd_us"] = timed(lambda: gemm.conv2d_forward_nhwc(xc, wk, None, k, k, 1, pd))
        r["implicit_bwd_us"] = timed(lambda: gemm.conv2d_backward_nhwc(xc, wk, gyc, k, k, 1, pd))
        r["im2col_fwd_us"] = timed(lambda: gemm.conv2d_forward(x, w, None, k, k, 1, pd))
        r["im2col_bwd_us"] = timed(lambda: gemm.conv2d_backward(x, w, gy, k, k, 1, pd))
        r["cudnn_fwd_us"] = timed(lambda: F_conv(x, w4, pd))
        r["cudnn_bwd_us"] = timed(lambda: (torch.nn.grad.conv2d_input(x.shape, w4, gy, padding=pd),
                                           torch.nn.grad.conv2d_weight(x, w4.shape, gy, padding=pd)))
        r["cudnn_cl_fwd_us"] = timed(lambda: F_conv(xc, w4.contiguous(memory_format=torch.channels_last), pd))
        r["implicit_fwd_tflops"] = flops / (r["implicit_fwd_us"] * 1e-6) / 1e12
        r["implicit_bwd_tflops"] = 2 * flops / (r["implicit_bwd_us"] * 1e-6) / 1e12
        rows.append(r)
    emit({"metric": "conv2d fwd / bwd (dX + dW) microseconds per backend", "unit": "us", "n_gpus": 1,
          "higher_is_better": False, "data": "synthetic N(0,1) bf16", "dtype": "bf16, fp32 accumulation",
          "config": {"workload": "ConcordConv2dPackedB's convolutions at SDXL UNet channel counts"},
          "rows": rows})


def bench_gemm(args):
    """The layer's three GEMMs at config 2's largest shape (M=8192 tokens,
    K=2048, N=10240) per implementation: this package's 2-SM tcgen05 kernel
    (concord_gemm2sm), the CUTLASS 1-SM kernels, cuBLAS (torch).  CUDA events,
    mean of 20 after 3 warm-ups, eager."""
    import ctypes
    from concord_b200 import _abi, gemm
    lib = _abi.load()
    Mt, Kt, Nt = M, args.cols, args.rows
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(Mt, Kt, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(Nt, Kt, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    dy = torch.randn(Mt, Nt, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.empty(Mt, Nt, dtype=torch.bfloat16, device="cuda")
    dx = torch.empty(Mt, Kt, dtype=torch.bfloat16, device="cuda")
    dw = torch.empty(Nt, Kt, dtype=torch.bfloat16, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def p(t):
        return ctypes.c_void_p(t.data_ptr())

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(20):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 20
    runs = {
        "2sm_fwd": lambda: lib.concord_gemm2sm(p(x), 0, Kt, p(w), 0, Kt, p(y), Nt, Mt, Nt, Kt, s),
        "2sm_dx": lambda: lib.concord_gemm2sm(p(dy), 0, Nt, p(w), 1, Kt, p(dx), Kt, Mt, Kt, Nt, s),
        "2sm_dw": lambda: lib.concord_gemm2sm(p(dy), 1, Nt, p(x), 1, Kt, p(dw), Kt, Nt, Kt, Mt, s),
        "cutlass1sm_fwd": lambda: gemm.forward(x, w), "cutlass1sm_dx": lambda: gemm.grad_input(dy, w),
        "cutlass1sm_dw": lambda: gemm.grad_weight(dy, x),
        "cublas_fwd": lambda: x @ w.T, "cublas_dx": lambda: dy @ w, "cublas_dw": lambda: dy.T @ x}
    flops = 2.0 * Mt * Nt * Kt
    out = {}
    old_impl = lib.concord_gemm_get_impl()
    for k, fn in runs.items():
        lib.concord_gemm_set_impl(_abi.GEMM_CUTLASS if k.startswith("cutlass") else _abi.GEMM_2SM)
        ms = timed(fn)
        out[k] = {"us": ms * 1e3, "tflops": flops / (ms * 1e-3) / 1e12}
    lib.concord_gemm_set_impl(old_impl)
    torch.cuda.synchronize()
    emit({"metric": "layer GEMM TFLOP/s per implementation", "unit": "TFLOP/s", "n_gpus": 1,
          "higher_is_better": True, "data": "synthetic N(0,1) bf16", "dtype": "bf16, fp32 accumulation",
          "config": {"workload": f"config 2 largest layer: M={Mt}, K={Kt}, N={Nt}"}, "results": out,
          "gemm2sm_error_word": int(lib.concord_gemm2sm_error(1)), "gemm2sm_pairs": int(lib.concord_gemm2sm_pairs())})


def F_conv(x, w4, pd):
    return torch.nn.functional.conv2d(x, w4, padding=pd)


def ms_share(part, whole):
    return part / whole if whole > 0 else None


def emit(d):
    print(json.dumps(d), flush=True)


def base_line(args, world):
    return {"metric": "fused bwd+packed-step HBM GB/s", "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "int32 words / fp32 math / bf16 grad",
            "data": "synthetic: W0~N(0,0.02) quantized, dW = dY^T X / M with X,dY ~ N(0,1) bf16",
            "config": {"workload": f"C2 dequant-matmul + packed-step sweep, largest shape "
                                   f"(M={M}, K={args.cols}, N={args.rows}); bare-default ConcordLinearPackedB",
                       "M": M, "K": args.cols, "N": args.rows, "params": args.rows * args.cols,
                       "l2_flush": "not needed: working set > 126 MB L2",
                       "parallelism": (f"dp{world}: row-sharded packed step and state; "
                                       + (SHARDED.transport if SHARDED is not None else "?") +
                                       " transport (peer: dW rows pushed over NVLink to their owners, summed with the v-hat pass, "
                                       "bf16 weight pushed to every rank by the step kernel; "
                                       "collective: NCCL reduce-scatter / all-gather)")
                                      if world > 1 else "single"}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--rows", type=int, default=N)
    ap.add_argument("--cols", type=int, default=K)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-models", action="store_true",
                    help="c2: skip the config 4/5 weak-scaling training steps the default line carries")
    ap.add_argument("--batch", type=int, default=8, help="llama: sequences per GPU")
    ap.add_argument("--layers", type=int, default=24, help="llama: decoder layers")
    ap.add_argument("--nogate", action="store_true", help="sdxl: disable_cohpre on every layer")
    ap.add_argument("--ckpt", action="store_true", help="sdxl: activation checkpointing per block")
    ap.add_argument("--workload", default="c2", choices=["c2", "chargpt", "llama", "sdxl", "conv", "gemm"],
                    help="c2: the packed-step path on config 2's largest layer (default); "
                         "chargpt: config 3's char-level GPT trained end to end; "
                         "llama: config 5's data-parallel decoder (weak scaling); "
                         "sdxl: config 4's UNet fine-tune (weak scaling); "
                         "conv: the conv layer's convolutions per backend; "
                         "gemm: the layer's GEMMs per implementation")
    ap.add_argument("--conv-backend", default=None, choices=["implicit", "gemm", "cudnn"],
                    help="sdxl/conv: ConcordConv2dPackedB's convolution backend (default: the package's)")
    ap.add_argument("--nchw", action="store_true", help="sdxl: NCHW activations instead of channels-last")
    ap.add_argument("--conv-shapes", default=None,
                    help="conv: ';'-separated B,C,O,HW,k shapes instead of the default list")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="time eager launches instead of CUDA-graph replays")
    args = ap.parse_args()
    if args.conv_backend:
        import concord_b200
        concord_b200.set_conv_backend(args.conv_backend)
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cores = len(os.sched_getaffinity(0))
    if args.impl == "reference":
        if rank != 0:
            return
        # the reference's CPU implementation of the path: its real-valued update
        # rule ConcordRef (the Triton step has no CPU build), on every host
        # core; the oracle port stands in only when the reference is absent
        probe = ref_cpu_rule(rows=256, threads=cores, steps=1)
        if probe is not None:
            per_row = probe[1] / 256
            rows = int(min(args.rows, max(256, 20.0 / max(1, args.steps + args.warmup) / per_row)))
            ref_cpu_rule(rows=rows, threads=cores, steps=max(1, args.warmup))
            vals = [ref_cpu_rule(rows=rows, threads=cores, steps=1)[0] for _ in range(args.steps)]
            kind, what = "reference", "ConcordRef.step (experiments/cpu_dynamics/concord_ref.py), torch CPU"
        else:
            _, t64 = cpu_baseline(rows=max(64, cores), threads=cores)
            per_row = t64 / max(64, cores)
            rows = int(min(4096, max(cores, 60.0 / max(1, args.steps + args.warmup) / per_row)))
            for _ in range(args.warmup):
                cpu_baseline(rows=rows, threads=cores)
            vals = [cpu_baseline(rows=rows, threads=cores)[0] for _ in range(args.steps)]
            kind, what = "port", "oracle port (C restatement)"
        v = statistics.mean(vals)
        d = base_line(args, 1)
        d.update({"impl": "reference", "value": v, "ms_per_step": rows * K * 22 / v / 1e6,
                  "cpu_baseline": {"value": v, "unit": "GB/s", "cores": cores, "kind": kind,
                                   "sample": f"{rows} rows x {K} cols of the workload per step; {what}"},
                  "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        emit(d)
        return
    if args.workload == "chargpt":
        if rank == 0:
            bench_chargpt(args, cores)
        return
    if args.workload == "conv":
        if rank == 0:
            bench_conv(args)
        return
    if args.workload == "gemm":
        if rank == 0:
            bench_gemm(args)
        return
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl")
    device = torch.device("cuda", torch.cuda.current_device())
    if args.workload in ("llama", "sdxl"):
        (bench_llama if args.workload == "llama" else bench_sdxl)(args, rank, world)
        if world > 1:
            dist.destroy_process_group()
        return
    from concord_b200 import packed_b
    packed_b._lib()
    r = bench_ours(args, rank, world, device)
    hbm, tf, src = peaks()
    # one layer update per step whatever the GPU count (the update is sharded)
    value = r["bytes_step"] / (r["ms"] * 1e-3) / 1e9
    shard_params = r["params"] if world == 1 else SHARDED.S * args.cols
    achieved = shard_params * STEP_BYTES_PER_PARAM / (r["step_kernel_ms"] * 1e-3) / 1e9
    if rank != 0:
        if not args.no_models:
            model_steps_guarded(args, rank, world, None)
        return
    d = base_line(args, world)
    flops = 2.0 * M * args.rows * args.cols
    d.update({
        "value": value, "ms_per_step": r["ms"],
        "e2e": {"value": r["bytes_step"] / (r["e2e_ms"] * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"],
                "note": "dW H2D of step i+1 on a copy stream, overlapped with step i"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm,
                     # DRAM bytes per launch from the ncu capture of this kernel at N=4096
                     # (135.6 MB for 8.39 M params), scaled by the params one launch steps
                     "traffic": STEP_TRAFFIC_PER_PARAM * shard_params,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                                       "step_vec_kernel at N=4096, K=2048, scaled by params",
                     "peak_source": src,
                     "kernel": "concord_step (step_vec_kernel<adamw>)",
                     "algorithmic_bytes_per_launch": shard_params * STEP_BYTES_PER_PARAM,
                     "kernel_ms": r["step_kernel_ms"]},
        "vhat_ms": r["vhat_ms"],
        **({"dp_phases_ms": r["phases"],
            "dp_phases_note": "eager pass, CUDA events between the peer transport's launches, "
                              "mean over steps, max over ranks"} if r.get("phases") else {}),
        "cuda_graph": r["graphs"],
        "gemm": {k: {"ms": v, "tflops": flops / (v * 1e-3) / 1e12} for k, v in r["gemm_ms"].items()},
        "gemm_impl": "fwd/dx/dw: concord tcgen05 kernels (CUTLASS sm100 templates); cublas_*: torch",
        "clocks": r["clocks"],
        "gpu_launches": args.steps * (4 if world == 1 else (6 if SHARDED.peer is not None else 5)),
        "gpu_launches_note": ("per step: vhat 1 + step 1 + rebalance decide 1 + shift 1 (+1 memset node)"
                              if world == 1 else
                              "per step: [peer reduce 1] + vhat partial 1 + finish 1 + step 1 + rebalance 2; "
                              "plus NCCL collectives (not counted)"),
    })
    if world == 1:
        bms, fms = backward_time(args.rows, args.cols, device)
        packed_b.set_fused_dw_vhat(False)
        bms_sep, _ = backward_time(args.rows, args.cols, device)
        packed_b.set_fused_dw_vhat(True)
        d["backward"] = {"ms": bms, "forward_ms": fms, "tokens": M,
                         "gemm_tflops": 2 * 2.0 * M * args.rows * args.cols / (bms * 1e-3) / 1e12,
                         "packed_path_share": ms_share(r["ms"], bms),
                         "ms_vhat_separate": bms_sep,
                         "note": "loss.backward() of one bare layer through the drop-in API: dX GEMM, "
                                 "dW GEMM with the v-hat partials in its epilogue + v-hat fold, packed step, "
                                 "then rebalance(); CUDA events, eager.  ms_vhat_separate: the same with "
                                 "the dW GEMM and a standalone v-hat launch"}
    if not args.no_cpu_baseline and world == 1:     # the CPU baseline is a one-GPU figure
        v1, dt = cpu_baseline(rows=2048, threads=1)
        port = {"value": v1, "unit": "GB/s", "cores": 1, "kind": "port",
                "sample": f"2048 rows x {args.cols} cols (v-hat + step), {dt:.2f} s; oracle port (C restatement)"}
        r1 = ref_cpu_rule(rows=2048, threads=1, steps=3)
        if r1 is not None:
            rall = ref_cpu_rule(rows=2048, threads=cores, steps=5)
            d["cpu_baseline"] = {"value": r1[0], "unit": "GB/s", "cores": 1, "kind": "reference",
                                 "sample": f"2048 rows x {args.cols} cols, ConcordRef.step "
                                           f"(experiments/cpu_dynamics/concord_ref.py), {r1[1]:.3f} s/step"}
            d["cpu_baseline_all_cores"] = {"value": rall[0], "unit": "GB/s", "cores": cores, "kind": "reference",
                                           "sample": f"same, torch CPU on {cores} threads, {rall[1]:.3f} s/step"}
            d["cpu_baseline_port"] = port
        else:
            d["cpu_baseline"] = port
    if not args.no_models:
        d["weak_scaling"] = model_steps_guarded(args, rank, world, d)
    emit(d)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
