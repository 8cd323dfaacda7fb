"""Real-valued Concord update rule on CPU (torch) — the reference's CPU oracle.

TEST INFRASTRUCTURE ONLY (tests/ and bench.py baselines).  Restates
`ConcordRef.step` of the reference (experiments/cpu_dynamics/concord_ref.py:
107-156) for one 2-D weight at the mapping that the packed kernel reaches in
expectation: gate=False, noise=False, kappa=0, constant lr, beta1=0 — i.e.
the package with disable_cohpre(), ratio gate off and gf_consol=0.  The
stochastic-rounding integer kernel equals this rule only in expectation, so
it pins consolidated weights within a statistical tolerance, never words.

State in weight units: u = velocity (s_fast), S = slow half (128 s_slow),
A = anchor half (128 v_slow); deploy weight P = S + A; live weight u + S + A.
"""
import torch


class RealValuedRule:
    def __init__(self, W0, lr, alpha=0.1, alpha_v=0.001, beta2=0.999, eps=1e-10, step_cap=10.0):
        W0 = W0.float()
        self.u = W0.clone()                 # load_weights: all mass in the velocity
        self.S = torch.zeros_like(W0)
        self.A = torch.zeros_like(W0)
        self.v_row = torch.zeros(W0.shape[0])
        self.v_col = torch.zeros(W0.shape[1])
        self.lr, self.alpha, self.alpha_v = lr, alpha, alpha_v
        self.beta2, self.eps, self.cap = beta2, eps, step_cap

    @torch.no_grad()
    def step(self, g):
        g = g.float()
        g2 = g * g
        self.v_row.mul_(self.beta2).add_(g2.sum(1), alpha=1 - self.beta2)
        self.v_col.mul_(self.beta2).add_(g2.sum(0), alpha=1 - self.beta2)
        vhat = self.v_row[:, None] * self.v_col[None, :] / self.v_row.sum().clamp_min(1e-30)
        step_ = (g / (vhat + self.eps).sqrt()).clamp_(-self.cap, self.cap)
        self.u -= self.lr * step_
        tr = self.alpha * self.u            # chase (gate fully open)
        self.S += tr
        self.u -= tr
        lk = self.alpha_v * (self.S - self.A)   # mass-preserving leak
        self.A += lk
        self.S -= lk

    def deploy(self):
        return self.S + self.A

    def live(self):
        return self.u + self.S + self.A
