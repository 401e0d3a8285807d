"""Bits-per-byte evaluation (reference: parallel/parallel/eval.py).

bpb = sum of per-token CE nats over tokens with a non-zero byte length,
divided by ln(2) x total UTF-8 bytes of the target tokens; nats and bytes
are summed over the data-parallel world.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


def get_token_bytes(tokenizer) -> torch.Tensor:
    special = set(tokenizer.all_special_ids)
    out = torch.zeros(tokenizer.vocab_size, dtype=torch.int64)
    for t in range(tokenizer.vocab_size):
        if t in special:
            continue
        out[t] = len(tokenizer.decode([t]).encode("utf-8"))
    return out


@torch.no_grad()
def eval_bpb(model, dataloader, eval_steps, device, pconfig, use_amp, amp_dtype, token_bytes, loss_fn=None):
    model.eval()
    token_bytes = token_bytes.to(device)
    nats = torch.tensor(0.0, dtype=torch.float32, device=device)
    nbytes = torch.tensor(0, dtype=torch.int64, device=device)
    state = None
    for _ in range(eval_steps):
        x, y, state = next(dataloader)
        with torch.autocast(device_type=pconfig.device_type or "cpu", dtype=amp_dtype,
                            enabled=use_amp and torch.device(device).type == "cuda"):
            out = model(input_ids=x, return_logits=True)
        logits = out.logits
        if loss_fn is None:
            per = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)).float(), y.reshape(-1),
                                                    reduction="none")
        else:
            per = loss_fn(logits, y, reduction="none")
        b = token_bytes[y.reshape(-1)]
        nats += (per * (b > 0)).sum()
        nbytes += b.sum()
    if pconfig.is_distributed and pconfig.dp_size > 1:
        dist.all_reduce(nats, op=dist.ReduceOp.SUM)
        dist.all_reduce(nbytes, op=dist.ReduceOp.SUM)
    model.train()
    total = nbytes.item()
    if total == 0:
        return float("inf"), state
    return nats.item() / (math.log(2) * total), state
