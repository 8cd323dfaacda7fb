"""Seeded inputs shared by make_golden_gpu.py (which feeds them to the
reference on a B200) and the GPU parity tests (which feed them to this
package), so both sides see the same bits."""
import torch

BARE = dict(kind="adamw", alpha=0.1, beta1=0.0, weight_decay=0.0, eps=1e-10, step_cap=10.0,
            v_scale=0.0, precond_p=0.5, gf_consol=0.0, drift_cancel_C=None,   # None: C* of (alpha, alpha_v_fast)
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
STEP_N, STEP_K, STEP_STEPS = 96, 200, 3

C1_N = 1024
C1_STEPS = 200
C1_LR = 5e-4
C2_N, C2_K, C2_STEPS = 10240, 2048, 10


def rand_step_inputs(seed, N=STEP_N, K=STEP_K, steps=STEP_STEPS):
    """State, v-hat, coh_pre and per-step bf16 gradients of one step case (CPU tensors)."""
    g = torch.Generator().manual_seed(seed)
    sf = torch.randint(-3000, 3001, (N, K), generator=g, dtype=torch.int32)
    ss = torch.randint(-100, 101, (N, K), generator=g, dtype=torch.int32)
    vs = torch.randint(-100, 101, (N, K), generator=g, dtype=torch.int32)
    packed = ((sf & 0xFFFF) << 16) | ((ss & 0xFF) << 8) | (vs & 0xFF)
    d = dict(packed=packed,
             row_exp=torch.randint(-3, 5, (N,), generator=g, dtype=torch.int8),
             col_exp=torch.randint(-2, 3, (K,), generator=g, dtype=torch.int8),
             v_row=torch.rand(N, generator=g) * 1e-4 + 1e-6,
             v_col=torch.rand(K, generator=g) * 1e-4 + 1e-6)
    d["svi"] = (1.0 / d["v_row"].sum()).reshape(1).float()
    d["coh_pre"] = torch.rand(N, K, generator=g)
    d["grads"] = [(torch.randn(N, K, generator=g) * s + torch.randn(N, 1, generator=g) * s / 2).to(torch.bfloat16)
                  for s in (1e-3, 3e-2, 1e-5)[:steps]]
    return d


def c1_inputs():
    """Config 1: W0 ~ N(0, 0.02), rank-4 drift U, V ~ N(0, 1e-4), and the
    generator that then draws G_t = N(0, 1e-3) + U V^T per step."""
    g = torch.Generator().manual_seed(0)
    W0 = torch.randn(C1_N, C1_N, generator=g) * 0.02
    U = torch.randn(C1_N, 4, generator=g) * 1e-4
    V = torch.randn(C1_N, 4, generator=g) * 1e-4
    return g, W0, U, V


def c1_grad(g, U, V):
    return (torch.randn(C1_N, C1_N, generator=g) * 1e-3 + U @ V.T).to(torch.bfloat16)


def c2_state():
    g = torch.Generator().manual_seed(2)
    return g, torch.randn(C2_N, C2_K, generator=g) * 0.02


def c2_grad(g):
    return (torch.randn(C2_N, C2_K, generator=g) * 1e-3).to(torch.bfloat16)


@torch.no_grad()
def torch_vhat(grad_W, v_row, v_col, sum_v_inv, beta2=0.999):
    """The reference backward's v-hat update in its own torch expression
    (concord/packed_b.py:1288-1303); the same torch kernels on the same GPU
    give the reference's bits."""
    g2 = grad_W.float() ** 2
    g2_row = g2.sum(dim=1)
    g2_col = g2.sum(dim=0)
    v_row.mul_(beta2).add_(g2_row, alpha=1.0 - beta2)
    v_col.mul_(beta2).add_(g2_col, alpha=1.0 - beta2)
    sum_v = v_row.sum().clamp(min=1e-30)
    sum_v_inv.fill_(0).add_(1.0 / sum_v)
