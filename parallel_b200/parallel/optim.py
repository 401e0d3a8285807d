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
parameters take the stock PyTorch path.  Inside a CUDA-graph capture the
kernel reads lr and the bias corrections from a device tensor per parameter
group, which ``advance_graph_step`` refreshes before each replay.
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
        # CUDA-graph mode: per param group a device tensor {lr, 1 - b1^t, sqrt(1 - b2^t)}
        # that the kernel reads instead of its scalar arguments, refreshed on the
        # host before every replay (``advance_graph_step``)
        self._graph_hyper: Optional[list[torch.Tensor]] = None
        self._graph_params: list[tuple[int, torch.nn.Parameter]] = []

    # ------------------------------------------------------------ CUDA graphs
    def enable_graph_hyper(self, device) -> None:
        self._graph_hyper = [torch.zeros(3, dtype=torch.float32, device=device) for _ in self.param_groups]
        self._graph_params = []

    def graph_step_counts(self) -> dict:
        return {id(p): st["step"].clone() for p, st in self.state.items() if "step" in st}

    def restore_step_counts(self, counts: dict) -> None:
        """Undo the host-side step increments of a capture (nothing ran)."""
        for p, st in self.state.items():
            if id(p) in counts:
                st["step"].copy_(counts[id(p)])

    def advance_graph_step(self) -> None:
        """Host half of one replayed step: bump the step counters of the
        parameters the captured step updates and upload the group's lr and
        bias corrections (pinned staging, ordered before the replay)."""
        steps: dict[int, float] = {}
        for gi, p in self._graph_params:
            st = self.state[p]
            st["step"] += 1
            t = float(st["step"])
            if steps.setdefault(gi, t) != t:
                raise RuntimeError("CUDA-graph AdamW needs one step count per parameter group")
        for gi, t in steps.items():
            group = self.param_groups[gi]
            b1, b2 = group["betas"]
            vals = torch.tensor([group["lr"], 1.0 - b1 ** t, (1.0 - b2 ** t) ** 0.5], dtype=torch.float32)
            self._graph_hyper[gi].copy_(vals.pin_memory(), non_blocking=True)

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
        capturing = torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()
        if capturing:
            if self._graph_hyper is None:
                raise RuntimeError("FusedAdamW: call enable_graph_hyper() before capturing a step")
            self._graph_params = []
        for gi, group in enumerate(self.param_groups):
            lr, (b1, b2), eps, wd = group["lr"], group["betas"], group["eps"], group["weight_decay"]
            hyper = self._graph_hyper[gi] if capturing else None
            by_step: dict = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                lp = _local(p)
                if not (lp.is_cuda and lp.dtype == torch.bfloat16):
                    fallback.append((group, p))
                    continue
                if capturing and len(self.state[p]) == 0:
                    raise RuntimeError("FusedAdamW: optimizer state must exist before a CUDA-graph capture "
                                       "(run an eager step first)")
                st = self._init_state(p)
                st["step"] += 1
                key = (int(st["step"].item()), _local(p.grad).dtype, _local(st["exp_avg"]).dtype)
                by_step.setdefault(key, []).append(p)
                if capturing:
                    self._graph_params.append((gi, p))
            for (step, _, _), ps in by_step.items():
                ls = [_local(p) for p in ps]
                gs = [_local(p.grad) for p in ps]
                ms = [_local(self.state[p]["exp_avg"]) for p in ps]
                vs = [_local(self.state[p]["exp_avg_sq"]) for p in ps]
                keep = [i for i, t in enumerate(ls) if t.numel() > 0]
                if keep:
                    ext().adamw([ls[i] for i in keep], [gs[i].contiguous() for i in keep], [ms[i] for i in keep],
                                [vs[i] for i in keep], lr, b1, b2, eps, wd, step, grad_scale, skip, hyper)
        if fallback:
            if capturing:
                raise RuntimeError("FusedAdamW: only CUDA bf16 parameters can be stepped inside a CUDA graph")
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
