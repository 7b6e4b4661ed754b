"""Fused AdamW over a flat parameter buffer (one kernel launch per step).

Same hyper-parameters and update as the reference's torch.optim.AdamW (bench_train.py:467-469:
lr 3e-4, betas (0.9, 0.95), weight decay 0.1 on every parameter, eps 1e-8). The kernel
also writes the bf16 shadow weights that the GEMMs read and, unless `zero_grad` is off (the
gradient writers then store on the step's first write), zeroes the gradient buffer for the next
step's accumulation. lr and the step count live on the device, so `step()` can be
captured in a CUDA graph and replayed.

State layout: exp_avg / exp_avg_sq flat fp32 buffers; `state_dict()` returns them per
parameter under torch.optim.AdamW's keys (exp_avg, exp_avg_sq, step) so checkpoints keep the
reference optimizer layout.
"""
from __future__ import annotations

import torch

from llmt.ops import native as N


class FusedAdamW:
    def __init__(self, master, grad, shadow, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                 grad_scale=1.0, zero_grad=True):
        self.master, self.grad, self.shadow = master, grad, shadow
        self.zero_grad = zero_grad
        self.exp_avg = torch.zeros_like(master)
        self.exp_avg_sq = torch.zeros_like(master)
        self.lr_t = torch.full((1,), float(lr), dtype=torch.float32, device=master.device)
        self.step_t = torch.zeros(1, dtype=torch.int32, device=master.device)
        self.betas, self.eps, self.weight_decay, self.grad_scale = betas, eps, weight_decay, grad_scale

    @property
    def lr(self):
        return float(self.lr_t.item())

    def set_lr(self, lr):
        self.lr_t.fill_(float(lr))

    @torch.no_grad()
    def step(self):
        self.step_t.add_(1)
        N.adamw_step(self.master, self.grad, self.exp_avg, self.exp_avg_sq, self.shadow, self.lr_t, self.step_t,
                     self.betas[0], self.betas[1], self.eps, self.weight_decay, self.grad_scale,
                     zero_grad=self.zero_grad)

    def state_dict(self, flat=None):
        """torch.optim.AdamW-style state: {'state': {i: {step, exp_avg, exp_avg_sq}}, 'param_groups': [...]}."""
        st = {}
        if flat is not None:
            step = float(self.step_t.item())
            for i, (p, o) in enumerate(zip(flat.params, flat.offsets)):
                n = p.numel()
                st[i] = {"step": torch.tensor(step),
                         "exp_avg": self.exp_avg[o:o + n].view(p.shape).clone(),
                         "exp_avg_sq": self.exp_avg_sq[o:o + n].view(p.shape).clone()}
        return {"state": st, "param_groups": [{"lr": self.lr, "betas": self.betas, "eps": self.eps,
                                               "weight_decay": self.weight_decay,
                                               "params": list(range(len(st)))}]}

    def load_state_dict(self, sd, flat):
        for i, (p, o) in enumerate(zip(flat.params, flat.offsets)):
            s = sd["state"].get(i)
            if s is None:
                continue
            n = p.numel()
            self.exp_avg[o:o + n].copy_(s["exp_avg"].reshape(-1))
            self.exp_avg_sq[o:o + n].copy_(s["exp_avg_sq"].reshape(-1))
            self.step_t.fill_(int(float(s["step"])))
        g = sd["param_groups"][0]
        self.set_lr(g["lr"])
