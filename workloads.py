"""Synthetic training workloads of the benchmark configurations that run
whole models, built in plain torch with Concord on
their weight matrices.  Random init and seeded synthetic data: no dataset or
checkpoint is read.

* Config 3, char-level GPT: the reference's nanoGPT architecture
  (notebook/src/nanogpt.py:15-101: pre-LN blocks, bias-free Linears, GELU
  MLP, learned positions, causal SDPA), 6 layers, 6 heads, d=384, context
  256, vocab 65, batch 64, on tokens from a seeded order-2 Markov chain over
  65 symbols whose transition rows are Dirichlet(0.3).
* Config 5, Llama-style decoder (24 layers, d=2048, 16 heads, SwiGLU 5504,
  vocab 32000, seq 2048) on uniform random token ids.
"""
import math
import os
import time

import torch
import torch.nn as nn
import torch.nn.functional as F


# ---------------------------------------------------------------- data
class MarkovChars:
    """Order-2 Markov chain over `vocab` symbols, transition rows ~ Dirichlet(alpha).

    Generates `n_chains` independent chains of `length` tokens on the device
    (vectorised over chains) and serves random windows of them."""

    def __init__(self, vocab=65, alpha=0.3, n_chains=4096, length=1024, seed=0, device="cuda"):
        g = torch.Generator().manual_seed(seed)
        conc = torch.full((vocab,), float(alpha))
        self.P = torch.distributions.Dirichlet(conc).sample((vocab * vocab,)).to(device)  # [V*V, V]
        gd = torch.Generator(device=device).manual_seed(seed + 1)
        toks = torch.empty(n_chains, length, dtype=torch.long, device=device)
        toks[:, :2] = torch.randint(0, vocab, (n_chains, 2), generator=gd, device=device)
        cdf = self.P.cumsum(dim=1)
        cdf[:, -1] = 1.0
        for t in range(2, length):
            state = toks[:, t - 2] * vocab + toks[:, t - 1]
            u = torch.rand(n_chains, 1, generator=gd, device=device)
            toks[:, t] = torch.searchsorted(cdf[state], u).squeeze(1).clamp_(max=vocab - 1)
        self.toks, self.vocab, self.gen = toks, vocab, torch.Generator(device=device).manual_seed(seed + 2)

    def entropy_rate(self):
        """Mean next-token entropy (nats) under the chain's empirical pair
        frequencies: the loss floor a perfect model reaches."""
        V = self.vocab
        pair = self.toks[:, :-1] * V + self.toks[:, 1:]
        freq = torch.bincount(pair[:, 1:].reshape(-1), minlength=V * V).float()   # states after burn-in
        freq = freq / freq.sum()
        h = -(self.P.clamp_min(1e-30) * self.P.clamp_min(1e-30).log()).sum(dim=1)
        return float((freq * h).sum())

    def batch(self, B, T):
        n, L = self.toks.shape
        c = torch.randint(0, n, (B,), generator=self.gen, device=self.toks.device)
        o = torch.randint(0, L - T - 1, (B,), generator=self.gen, device=self.toks.device)
        idx = o[:, None] + torch.arange(T + 1, device=self.toks.device)[None, :]
        w = self.toks[c[:, None], idx]
        return w[:, :-1], w[:, 1:]


# ---------------------------------------------------------------- config 3: char GPT
class CausalSelfAttention(nn.Module):
    def __init__(self, d, h):
        super().__init__()
        self.c_attn = nn.Linear(d, 3 * d, bias=False)
        self.c_proj = nn.Linear(d, d, bias=False)
        self.h, self.d = h, d

    def forward(self, x):
        B, T, C = x.shape
        q, k, v = self.c_attn(x).split(self.d, dim=2)
        q, k, v = (t.view(B, T, self.h, C // self.h).transpose(1, 2) for t in (q, k, v))
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.c_proj(y.transpose(1, 2).reshape(B, T, C))


class GPTBlock(nn.Module):
    def __init__(self, d, h):
        super().__init__()
        self.ln_1, self.ln_2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.attn = CausalSelfAttention(d, h)
        self.c_fc = nn.Linear(d, 4 * d, bias=False)
        self.mlp_proj = nn.Linear(4 * d, d, bias=False)

    def forward(self, x):
        x = x + self.attn(self.ln_1(x))
        return x + self.mlp_proj(F.gelu(self.c_fc(self.ln_2(x))))


class CharGPT(nn.Module):
    def __init__(self, vocab=65, block=256, n_layer=6, n_head=6, d=384):
        super().__init__()
        self.wte, self.wpe = nn.Embedding(vocab, d), nn.Embedding(block, d)
        self.blocks = nn.ModuleList([GPTBlock(d, n_head) for _ in range(n_layer)])
        self.ln_f = nn.LayerNorm(d)
        self.lm_head = nn.Linear(d, vocab, bias=False)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, 0.0, 0.02)
        for b in self.blocks:   # nanoGPT's residual-projection scaling
            for lin in (b.attn.c_proj, b.mlp_proj):
                nn.init.normal_(lin.weight, 0.0, 0.02 / math.sqrt(2 * n_layer))

    def forward(self, idx, targets):
        T = idx.shape[1]
        x = self.wte(idx) + self.wpe(torch.arange(T, device=idx.device))[None]
        for b in self.blocks:
            x = b(x)
        logits = self.lm_head(self.ln_f(x)).float()
        return F.cross_entropy(logits.view(-1, logits.shape[-1]), targets.reshape(-1))


def lr_at(it, peak, warmup, total, floor=0.1):
    if it < warmup:
        return peak * (it + 1) / warmup
    p = (it - warmup) / max(1, total - warmup)
    return peak * (floor + (1 - floor) * 0.5 * (1 + math.cos(math.pi * p)))


def train_chargpt(steps=2000, batch=64, block=256, lr=5e-4, aux_lr=0.05, seed=0, device="cuda",
                  log_every=100, warmup=100, graph=True):
    """Config 3 on one GPU.  Concord on every Linear (self-stepping backward,
    rebalance every step), SGD with momentum 0.9 on embeddings and norms,
    bf16 autocast.  The Concord lr follows warm-up + cosine through the
    layers' device lr scalars (so a captured graph follows it); the aux lr is
    constant.  With `graph`, the whole training step is one CUDA graph after
    10 eager steps.  Returns losses, timings and the chain's entropy floor."""
    from concord_b200.convert import aux_parameters, concordify
    torch.manual_seed(seed)
    data = MarkovChars(seed=seed, device=device)
    model = CharGPT(block=block).to(device)
    layers = concordify(model, lr=lr)
    aux = aux_parameters(model)
    opt = torch.optim.SGD(aux, lr=aux_lr, momentum=0.9)
    n_concord = sum(l.packed_w.numel() for l in layers)
    n_aux = sum(p.numel() for p in aux)
    x = torch.zeros(batch, block, dtype=torch.long, device=device)
    y = torch.zeros_like(x)
    for p in aux:
        p.grad = torch.zeros_like(p)

    def step():
        opt.zero_grad(set_to_none=False)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(x, y)
        loss.backward()               # Concord layers step inside the backward
        opt.step()
        for l in layers:
            l.rebalance()
        return loss

    g, static_loss, log, t_dev = None, None, [], []
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        log, t_dev, g = _chargpt_loop(steps, lr, warmup, layers, data, batch, block, x, y, graph, step, log_every)
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in t_dev) / len(t_dev)
    return dict(losses=log, steps_per_s=1e3 / ms, ms_per_step=ms, concord_params=n_concord, aux_params=n_aux,
                entropy_floor=data.entropy_rate(), tokens_per_step=batch * block, cuda_graph=graph)


def _chargpt_loop(steps, lr, warmup, layers, data, batch, block, x, y, graph, step, log_every):
    g, static_loss, log, t_dev = None, None, [], []
    for it in range(steps):
        cur = lr_at(it, lr, warmup, steps)
        for l in layers:
            l.lr = cur
        xb, yb = data.batch(batch, block)
        x.copy_(xb)
        y.copy_(yb)
        if graph and g is None and it == 10:
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                static_loss = step()
            x.copy_(xb)
            y.copy_(yb)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if g is not None:
            g.replay()
            loss = static_loss
        else:
            loss = step()
        e1.record()
        if it >= 10:
            t_dev.append((e0, e1))
        if it % log_every == 0 or it == steps - 1:
            log.append((it, float(loss.item())))
        if g is None:
            del loss
    return log, t_dev, g


def run_steps(step_fn, refill, steps, warmup, layers, lr, graph, world=1, group=None):
    """Run `warmup` eager steps, then `steps` timed ones.  With `graph` the
    whole training step (forward, backward with the packed steps inside, the
    other parameters' update, rebalance) is captured once as a CUDA graph and
    replayed.  `refill(it)` writes the next batch into the step's static
    inputs (outside the timed region).  Returns per-step device times (max over
    ranks) and losses."""
    import torch.distributed as dist
    dev = torch.device("cuda", torch.cuda.current_device())
    times, losses = [], []
    g = None
    static_loss = None
    # every step, eager or captured, runs on one side stream: the parameters'
    # AccumulateGrad nodes are created on the stream of the first backward,
    # and a captured backward must not depend on the legacy default stream
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for it in range(warmup + steps):
            for l in layers:              # linear lr warm-up over 100 steps, as the reference's trainers
                l.lr = lr * min(1.0, (it + 1) / 100)
            refill(it)
            if graph and g is None and it == warmup:   # capture after the eager warm-up
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    static_loss = step_fn()
                refill(it)
            if world > 1:
                dist.barrier(group=group)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            if g is not None:
                g.replay()
                loss = static_loss
            else:
                loss = step_fn()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            if world > 1:
                tt = torch.tensor([ms], device=dev)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX, group=group)
                ms = float(tt.item())
            if it >= warmup:
                times.append(ms)
            losses.append(float(loss.item()))
            if g is None:
                del loss                  # no autograd graph kept alive into the capture
    torch.cuda.current_stream(dev).wait_stream(side)
    return times, losses


def _defer_column_maxima(steppers, group):
    """On more than one rank: every layer's column maxima all-reduced once per
    step (the first rebalance() of the step does it) instead of once per
    layer inside the backward.  CONCORD_DP_DEFER_CMAX=0 keeps the per-layer
    all-reduce."""
    if not steppers or os.environ.get("CONCORD_DP_DEFER_CMAX", "1") == "0":
        return None
    from concord_b200.distributed import DeferredColumnMaxima
    return DeferredColumnMaxima(steppers, group=group)


def allreduce_grads(params, flat, world, group=None):
    """Average the ordinary parameters' gradients over the ranks (one bucket)."""
    import torch.distributed as dist
    off = 0
    for p in params:
        flat[off:off + p.numel()].copy_(p.grad.view(-1))
        off += p.numel()
    dist.all_reduce(flat, group=group)
    flat.div_(world)
    off = 0
    for p in params:
        p.grad.view(-1).copy_(flat[off:off + p.numel()])
        off += p.numel()


# ---------------------------------------------------------------- config 5: Llama-style decoder
class RMSNorm(nn.Module):
    def __init__(self, d, eps=1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight).to(x.dtype)


def rope_tables(T, hd, device, base=10000.0):
    inv = 1.0 / (base ** (torch.arange(0, hd, 2, device=device).float() / hd))
    f = torch.outer(torch.arange(T, device=device).float(), inv)
    return f.cos().to(torch.bfloat16), f.sin().to(torch.bfloat16)


def apply_rope(x, cos, sin):
    x1, x2 = x[..., 0::2], x[..., 1::2]
    return torch.stack((x1 * cos - x2 * sin, x1 * sin + x2 * cos), dim=-1).flatten(-2)


class LlamaBlock(nn.Module):
    def __init__(self, d, h, ffn):
        super().__init__()
        self.h = h
        self.attn_norm, self.ffn_norm = RMSNorm(d), RMSNorm(d)
        self.wq, self.wk, self.wv, self.wo = (nn.Linear(d, d, bias=False) for _ in range(4))
        self.w_gate, self.w_up = nn.Linear(d, ffn, bias=False), nn.Linear(d, ffn, bias=False)
        self.w_down = nn.Linear(ffn, d, bias=False)

    def forward(self, x, cos, sin):
        B, T, D = x.shape
        a = self.attn_norm(x)
        q, k, v = (lin(a).view(B, T, self.h, D // self.h).transpose(1, 2) for lin in (self.wq, self.wk, self.wv))
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.wo(y.transpose(1, 2).reshape(B, T, D))
        f = self.ffn_norm(x)
        return x + self.w_down(F.silu(self.w_gate(f)) * self.w_up(f))


class Llama(nn.Module):
    def __init__(self, vocab=32000, d=2048, n_layer=24, n_head=16, ffn=5504):
        super().__init__()
        self.emb = nn.Embedding(vocab, d)
        self.blocks = nn.ModuleList([LlamaBlock(d, n_head, ffn) for _ in range(n_layer)])
        self.norm = RMSNorm(d)
        self.lm_head = nn.Linear(d, vocab, bias=False)
        self.hd = d // n_head
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, 0.0, 0.02)

    def forward(self, idx, targets):
        T = idx.shape[1]
        cos, sin = rope_tables(T, self.hd, idx.device)
        x = self.emb(idx)
        for b in self.blocks:
            x = b(x, cos, sin)
        logits = self.lm_head(self.norm(x))
        return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), targets.reshape(-1))


def train_llama_dp(steps, warmup, batch_per_gpu=8, seq=2048, lr=5e-4, aux_lr=0.01, seed=0, n_layer=24,
                   group=None, graph=True):
    """Config 5: data-parallel training steps of the Llama-style decoder, one
    process per GPU (torch.distributed already initialised when world > 1).

    Weak scaling: each rank trains on its own `batch_per_gpu` sequences of
    uniform random token ids (global batch = world * batch_per_gpu; 64 at 8
    GPUs).  Concord on the 168 block Linears; on more than one rank each is
    registered with a RowShardedStep, so `loss.backward()` reduce-scatters
    every layer's dW over NVLink, steps the rank's row shard and all-gathers
    the bf16 forward weight.  Embedding, norms and lm_head take SGD (momentum
    0.9) on gradients all-reduced in one bucket.  Returns per-step device
    times (max over ranks) and the loss."""
    import torch.distributed as dist
    from concord_b200.convert import concordify
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(seed)
    model = Llama(n_layer=n_layer).to(dev)
    layers = concordify(model, lr=lr, skip=lambda name, m: name == "lm_head")
    steppers = []
    if world > 1:
        from concord_b200.distributed import RowShardedStep
        steppers = [RowShardedStep(l, group=group) for l in layers]
    deferred = _defer_column_maxima(steppers, group)
    aux = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.SGD(aux, lr=aux_lr, momentum=0.9)
    flat = torch.zeros(sum(p.numel() for p in aux), dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed * 1000 + rank)
    x = torch.zeros(batch_per_gpu, seq + 1, dtype=torch.long, device=dev)

    def refill(it):
        x.copy_(torch.randint(0, 32000, (batch_per_gpu, seq + 1), generator=g, device=dev))

    def step():
        opt.zero_grad(set_to_none=False)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(x[:, :-1], x[:, 1:])
        loss.backward()                       # every Concord layer steps (its shard) here
        if world > 1:                         # the ordinary parameters: one bucketed all-reduce
            allreduce_grads(aux, flat, world, group)
        opt.step()
        for l in layers:
            l.rebalance()
        return loss

    for p in aux:                             # gradients accumulate into fixed buffers (graph replay)
        p.grad = torch.zeros_like(p)
    times, losses = run_steps(step, refill, steps, warmup, layers, lr, graph, world, group)
    for st in steppers:
        st.check()
    params = sum(l.packed_w.numel() for l in layers)
    if deferred is not None:
        deferred.close()
    for st in steppers:
        st.close()
    return dict(ms=times, losses=losses, concord_params=params, world=world,
                tokens_per_step=world * batch_per_gpu * seq)


# ---------------------------------------------------------------- config 4: SDXL-architecture UNet
# The public SDXL UNet layout (diffusers UNet2DConditionModel as configured for
# SDXL base): channels (320, 640, 1280), two ResNet blocks per level, linear
# projections in and out of the transformers, transformer depth (0, 2, 10)
# with 64-dim heads, cross-attention to a 2048-wide text context, and the
# "text_time" additional embedding (pooled text 1280 + six 256-dim Fourier
# time ids).  Written here from that public description; random init.
def timestep_features(t, dim, max_period=10000.0):
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
    a = t.float()[:, None] * freqs[None]
    return torch.cat([torch.cos(a), torch.sin(a)], dim=-1)


class ResBlock(nn.Module):
    def __init__(self, cin, cout, temb=1280):
        super().__init__()
        self.norm1, self.norm2 = nn.GroupNorm(32, cin, eps=1e-5), nn.GroupNorm(32, cout, eps=1e-5)
        self.conv1, self.conv2 = nn.Conv2d(cin, cout, 3, padding=1), nn.Conv2d(cout, cout, 3, padding=1)
        self.time_emb_proj = nn.Linear(temb, cout)
        self.conv_shortcut = nn.Conv2d(cin, cout, 1) if cin != cout else None

    def forward(self, x, emb):
        h = self.conv1(F.silu(self.norm1(x)))
        h = h + self.time_emb_proj(F.silu(emb))[:, :, None, None].to(h.dtype)
        h = self.conv2(F.silu(self.norm2(h)))
        return (x if self.conv_shortcut is None else self.conv_shortcut(x)) + h


class Attention(nn.Module):
    def __init__(self, c, ctx=None, head_dim=64):
        super().__init__()
        kv = ctx or c
        self.heads = c // head_dim
        self.to_q, self.to_k, self.to_v = nn.Linear(c, c, bias=False), nn.Linear(kv, c, bias=False), nn.Linear(kv, c, bias=False)
        self.to_out = nn.Linear(c, c)

    def forward(self, x, ctx=None):
        B, T, C = x.shape
        src = x if ctx is None else ctx
        q = self.to_q(x).view(B, T, self.heads, -1).transpose(1, 2)
        k = self.to_k(src).view(B, src.shape[1], self.heads, -1).transpose(1, 2)
        v = self.to_v(src).view(B, src.shape[1], self.heads, -1).transpose(1, 2)
        y = F.scaled_dot_product_attention(q, k, v)
        return self.to_out(y.transpose(1, 2).reshape(B, T, C))


class TransformerBlock(nn.Module):
    def __init__(self, c, ctx):
        super().__init__()
        self.norm1, self.norm2, self.norm3 = nn.LayerNorm(c), nn.LayerNorm(c), nn.LayerNorm(c)
        self.attn1, self.attn2 = Attention(c), Attention(c, ctx)
        self.ff_proj = nn.Linear(c, 8 * c)          # GEGLU: value and gate halves
        self.ff_out = nn.Linear(4 * c, c)

    def forward(self, x, ctx):
        x = x + self.attn1(self.norm1(x))
        x = x + self.attn2(self.norm2(x), ctx)
        a, gate = self.ff_proj(self.norm3(x)).chunk(2, dim=-1)
        return x + self.ff_out(a * F.gelu(gate))


class Transformer2D(nn.Module):
    def __init__(self, c, depth, ctx=2048):
        super().__init__()
        self.norm = nn.GroupNorm(32, c, eps=1e-6)
        self.proj_in, self.proj_out = nn.Linear(c, c), nn.Linear(c, c)
        self.blocks = nn.ModuleList([TransformerBlock(c, ctx) for _ in range(depth)])

    def forward(self, x, ctx):
        B, C, H, W = x.shape
        h = self.proj_in(self.norm(x).permute(0, 2, 3, 1).reshape(B, H * W, C))
        for b in self.blocks:
            h = b(h, ctx)
        return x + self.proj_out(h).reshape(B, H, W, C).permute(0, 3, 1, 2).to(x.dtype)


class SDXLUNet(nn.Module):
    def __init__(self, ch=(320, 640, 1280), depth=(0, 2, 10), ctx=2048, pooled=1280, in_ch=4):
        super().__init__()
        c0, c1, c2 = ch
        temb = 4 * c0
        self.time_lin1, self.time_lin2 = nn.Linear(c0, temb), nn.Linear(temb, temb)
        self.add_lin1, self.add_lin2 = nn.Linear(pooled + 6 * 256, temb), nn.Linear(temb, temb)
        self.conv_in = nn.Conv2d(in_ch, c0, 3, padding=1)
        self.down = nn.ModuleList()
        skips, prev = [c0], c0
        for lvl, (c, d) in enumerate(zip(ch, depth)):
            blk = nn.Module()
            blk.res = nn.ModuleList([ResBlock(prev if i == 0 else c, c, temb) for i in range(2)])
            blk.attn = nn.ModuleList([Transformer2D(c, d, ctx) for _ in range(2)]) if d else None
            skips += [c, c]
            blk.downsample = nn.Conv2d(c, c, 3, stride=2, padding=1) if lvl < len(ch) - 1 else None
            if blk.downsample is not None:
                skips.append(c)
            self.down.append(blk)
            prev = c
        self.mid_res1, self.mid_attn, self.mid_res2 = (ResBlock(c2, c2, temb), Transformer2D(c2, depth[-1], ctx),
                                                      ResBlock(c2, c2, temb))
        self.up = nn.ModuleList()
        for lvl, (c, d) in enumerate(zip(reversed(ch), reversed(depth))):
            blk = nn.Module()
            res = []
            for i in range(3):
                res.append(ResBlock(prev + skips.pop(), c, temb))
                prev = c
            blk.res = nn.ModuleList(res)
            blk.attn = nn.ModuleList([Transformer2D(c, d, ctx) for _ in range(3)]) if d else None
            blk.upsample = nn.Conv2d(c, c, 3, padding=1) if lvl < len(ch) - 1 else None
            self.up.append(blk)
        self.norm_out = nn.GroupNorm(32, c0, eps=1e-5)
        self.conv_out = nn.Conv2d(c0, in_ch, 3, padding=1)

    ckpt = False   # recompute each ResNet / transformer block in the backward

    def _run(self, mod, *args):
        if self.ckpt and torch.is_grad_enabled():
            from torch.utils.checkpoint import checkpoint
            return checkpoint(mod, *args, use_reentrant=False)
        return mod(*args)

    def forward(self, x, t, ctx, pooled, time_ids):
        emb = self.time_lin2(F.silu(self.time_lin1(timestep_features(t, self.time_lin1.in_features))))
        tid = timestep_features(time_ids.reshape(-1), 256).reshape(x.shape[0], -1)
        add = self.add_lin2(F.silu(self.add_lin1(torch.cat([pooled, tid.to(pooled.dtype)], dim=-1))))
        emb = emb + add
        h = self.conv_in(x)
        skips = [h]
        for blk in self.down:
            for i, r in enumerate(blk.res):
                h = self._run(r, h, emb)
                if blk.attn is not None:
                    h = self._run(blk.attn[i], h, ctx)
                skips.append(h)
            if blk.downsample is not None:
                h = blk.downsample(h)
                skips.append(h)
        h = self._run(self.mid_res2, self._run(self.mid_attn, self._run(self.mid_res1, h, emb), ctx), emb)
        for blk in self.up:
            for i, r in enumerate(blk.res):
                h = self._run(r, torch.cat([h, skips.pop().to(h.dtype)], dim=1), emb)
                if blk.attn is not None:
                    h = self._run(blk.attn[i], h, ctx)
            if blk.upsample is not None:
                h = blk.upsample(F.interpolate(h, scale_factor=2.0, mode="nearest"))
        return self.conv_out(F.silu(self.norm_out(h)))


def sdxl_batch(B, gen, device, res=128):
    """Config 4's synthetic batch: latents [B,4,res,res], context [B,77,2048],
    pooled [B,1280] ~ N(0,1), timesteps U{0..999}, noise target."""
    lat = torch.randn(B, 4, res, res, generator=gen, device=device)
    ctx = torch.randn(B, 77, 2048, generator=gen, device=device)
    pooled = torch.randn(B, 1280, generator=gen, device=device)
    t = torch.randint(0, 1000, (B,), generator=gen, device=device)
    noise = torch.randn(B, 4, res, res, generator=gen, device=device)
    ids = torch.tensor([1024.0, 1024.0, 0.0, 0.0, 1024.0, 1024.0], device=device).repeat(B, 1)
    return lat, ctx, pooled, t, noise, ids


def train_sdxl_dp(steps, warmup, batch_per_gpu=4, res=128, lr=5e-5, aux_lr=1e-4, seed=0, group=None,
                  gate=True, ckpt=False, graph=True, channels_last=True):
    """Config 4: epsilon-prediction MSE fine-tune steps of the SDXL-architecture
    UNet (~2.6 B parameters, random init), bf16 autocast, Concord on every
    Linear and every convolution (3x3 ones as their reshaped [O, I*9] weight),
    SGD (momentum 0.9) on norms and biases.  One process per GPU; with more
    than one rank every packed layer is data-parallel (RowShardedStep inside
    loss.backward()) and the other parameters' gradients are all-reduced.
    Weak scaling: `batch_per_gpu` samples per GPU.  lr 5e-5 is the
    reference's SDXL setting (notebook/src/sdxl_train.py:154); `ckpt` recomputes
    every block in the backward (activation checkpointing).  `channels_last`
    keeps the activations NHWC end to end (the latents and every conv output),
    the layout the implicit-GEMM convolutions read and write without copies."""
    import torch.distributed as dist
    from concord_b200.convert import concordify
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(seed)
    model = SDXLUNet().to(dev)
    if channels_last:
        model = model.to(memory_format=torch.channels_last)
    model.ckpt = ckpt
    n_total = sum(p.numel() for p in model.parameters())
    layers = concordify(model, lr=lr, convs=True)
    if not gate:
        for l in layers:
            l.disable_cohpre()
    steppers = []
    if world > 1:
        from concord_b200.distributed import RowShardedStep
        steppers = [RowShardedStep(l, group=group) for l in layers]
    deferred = _defer_column_maxima(steppers, group)
    aux = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.SGD(aux, lr=aux_lr, momentum=0.9)
    flat = torch.zeros(sum(p.numel() for p in aux), dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed * 1000 + rank)
    torch.cuda.synchronize()
    base_mem = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    static = [t.clone() for t in sdxl_batch(batch_per_gpu, g, dev, res)]
    if channels_last:                         # latents and noise NHWC
        static[0] = static[0].contiguous(memory_format=torch.channels_last)
        static[4] = static[4].contiguous(memory_format=torch.channels_last)

    def refill(it):
        lat, ctx, pooled, t, noise, ids = sdxl_batch(batch_per_gpu, g, dev, res)
        alpha_bar = torch.cos(t.float() / 1000 * math.pi / 2) ** 2
        noisy = alpha_bar.sqrt()[:, None, None, None] * lat + (1 - alpha_bar).sqrt()[:, None, None, None] * noise
        for dst, src in zip(static, (noisy, ctx, pooled, t, noise, ids)):
            dst.copy_(src)

    def step():
        opt.zero_grad(set_to_none=False)
        noisy, ctx, pooled, t, noise, ids = static
        with torch.autocast("cuda", dtype=torch.bfloat16):
            pred = model(noisy, t, ctx, pooled, ids)
        loss = F.mse_loss(pred.float(), noise)
        loss.backward()
        if world > 1:
            allreduce_grads(aux, flat, world, group)
        opt.step()
        for l in layers:
            l.rebalance()
        return loss

    for p in aux:                             # gradients accumulate into fixed buffers (graph replay)
        p.grad = torch.zeros_like(p)
    times, losses = run_steps(step, refill, steps, warmup, layers, lr, graph, world, group)
    for st in steppers:
        st.check()
    out = dict(ms=times, losses=losses, params=n_total, concord_params=sum(l.packed_w.numel() for l in layers),
               n_layers=len(layers), world=world, samples_per_step=world * batch_per_gpu,
               state_gb=base_mem / 1e9, peak_gb=torch.cuda.max_memory_allocated() / 1e9)
    if deferred is not None:
        deferred.close()
    for st in steppers:
        st.close()
    return out
