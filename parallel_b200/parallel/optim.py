"""AdamW whose CUDA step is one multi-tensor sm_100a kernel.

``FusedAdamW`` is a ``torch.optim.AdamW`` (same hyper-parameters, same
``state_dict`` layout: per-parameter ``step`` / ``exp_avg`` / ``exp_avg_sq``,
DTensor states for DTensor parameters), so optimizer checkpoints interchange
with the reference, which steps ``torch.optim.AdamW`` on its bf16 DTensor
shards (parallel/parallel/engine/engine.py:61-66).

On CUDA bf16 parameters ``step(grad_scale=..., skip=...)`` runs
``csrc/optim.cu``: fp32 math, the clip coefficient applied to the gradient
inside the kernel (a device scalar: no host sync), and a device flag that
turns the update into a no-op when the gradients were non-finite.  Other
parameters take the stock PyTorch path.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch.distributed.tensor import DTensor

from ..ops._ext import ext


def _local(t):
    return t._local_tensor if isinstance(t, DTensor) else t


class FusedAdamW(torch.optim.AdamW):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2,
                 state_dtype: str = "param"):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, foreach=False)
        self.state_dtype = state_dtype

    def _init_state(self, p):
        st = self.state[p]
        if len(st) == 0:
            st["step"] = torch.tensor(0.0, dtype=torch.float32)
            if self.state_dtype == "fp32":
                st["exp_avg"] = torch.zeros_like(p, dtype=torch.float32, memory_format=torch.preserve_format)
                st["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32, memory_format=torch.preserve_format)
            else:
                st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
        return st

    @torch.no_grad()
    def step(self, closure=None, grad_scale: Optional[torch.Tensor] = None, skip: Optional[torch.Tensor] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        fallback = []
        for group in self.param_groups:
            lr, (b1, b2), eps, wd = group["lr"], group["betas"], group["eps"], group["weight_decay"]
            by_step: dict = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                lp = _local(p)
                if not (lp.is_cuda and lp.dtype == torch.bfloat16):
                    fallback.append((group, p))
                    continue
                st = self._init_state(p)
                st["step"] += 1
                key = (int(st["step"].item()), _local(p.grad).dtype, _local(st["exp_avg"]).dtype)
                by_step.setdefault(key, []).append(p)
            for (step, _, _), ps in by_step.items():
                ls = [_local(p) for p in ps]
                gs = [_local(p.grad) for p in ps]
                ms = [_local(self.state[p]["exp_avg"]) for p in ps]
                vs = [_local(self.state[p]["exp_avg_sq"]) for p in ps]
                keep = [i for i, t in enumerate(ls) if t.numel() > 0]
                if keep:
                    ext().adamw([ls[i] for i in keep], [gs[i].contiguous() for i in keep], [ms[i] for i in keep],
                                [vs[i] for i in keep], lr, b1, b2, eps, wd, step, grad_scale, skip)
        if fallback:
            self._fallback_step(fallback, grad_scale, skip)
        return loss

    def _fallback_step(self, items, grad_scale, skip):
        if skip is not None and bool(skip.item()):
            return
        for group, p in items:
            st = self._init_state(p)
            st["step"] += 1
            step = float(st["step"].item())
            lr, (b1, b2), eps, wd = group["lr"], group["betas"], group["eps"], group["weight_decay"]
            lp, g = _local(p), _local(p.grad)
            if grad_scale is not None:
                g = g * grad_scale.to(g.device, g.dtype)
            m, v = _local(st["exp_avg"]), _local(st["exp_avg_sq"])
            lp.mul_(1 - lr * wd)
            m.lerp_(g.to(m.dtype), 1 - b1)
            v.mul_(b2).addcmul_(g.to(v.dtype), g.to(v.dtype), value=1 - b2)
            bc1 = 1 - b1 ** step
            bc2 = 1 - b2 ** step
            denom = (v.sqrt() / (bc2 ** 0.5)).add_(eps)
            lp.addcdiv_(m.to(lp.dtype), denom.to(lp.dtype), value=-lr / bc1)
