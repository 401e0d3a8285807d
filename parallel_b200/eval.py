"""Bits-per-byte evaluation.

bpb = (sum of cross-entropy nats over target tokens that decode to at least
one UTF-8 byte) / (ln 2 x sum of the UTF-8 byte lengths of all target
tokens), with both sums taken over the data-parallel ranks - the metric of
the reference's ``parallel/parallel/eval.py``.  Special tokens count zero
bytes.  Here the two sums travel as one float64 pair on the device (one
all-reduce at the end, one host read), and the per-token losses come from
the engine's fused cross-entropy when a ``loss_fn`` is given.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


def get_token_bytes(tokenizer) -> torch.Tensor:
    """int64 [vocab]: UTF-8 length of each token decoded on its own (0 for
    special tokens)."""
    ids = list(range(tokenizer.vocab_size))
    texts = tokenizer.batch_decode([[i] for i in ids])
    lengths = torch.tensor([len(t.encode("utf-8")) for t in texts], dtype=torch.int64)
    special = [i for i in tokenizer.all_special_ids if 0 <= i < len(ids)]
    if special:
        lengths[torch.tensor(special, dtype=torch.int64)] = 0
    return lengths


class _BpbMeter:
    def __init__(self, token_bytes: torch.Tensor, device):
        self.token_bytes = token_bytes.to(device)
        self.sums = torch.zeros(2, dtype=torch.float64, device=device)  # [nats, bytes]

    def add(self, per_token_nats: torch.Tensor, targets: torch.Tensor) -> None:
        nbytes = self.token_bytes[targets.reshape(-1)]
        counted = per_token_nats.reshape(-1).double() * (nbytes > 0)
        self.sums += torch.stack([counted.sum(), nbytes.sum().double()])

    def result(self, reduce: bool) -> float:
        if reduce:
            dist.all_reduce(self.sums, op=dist.ReduceOp.SUM)
        nats, nbytes = self.sums.tolist()
        return float("inf") if nbytes == 0 else nats / (math.log(2) * nbytes)


@torch.no_grad()
def eval_bpb(model, dataloader, eval_steps, device, pconfig, use_amp, amp_dtype, token_bytes, loss_fn=None):
    """Run ``eval_steps`` batches of ``dataloader`` through ``model`` in eval
    mode; returns (bpb, the loader state after the last batch)."""
    meter = _BpbMeter(token_bytes, device)
    autocast_on = use_amp and torch.device(device).type == "cuda"
    state = None
    model.eval()
    try:
        for _ in range(eval_steps):
            x, y, state = next(dataloader)
            with torch.autocast(device_type=pconfig.device_type or "cpu", dtype=amp_dtype, enabled=autocast_on):
                logits = model(input_ids=x, return_logits=True).logits
            if loss_fn is not None:
                nats = loss_fn(logits, y, reduction="none")
            else:
                nats = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), y.reshape(-1),
                                                         reduction="none")
            meter.add(nats, y)
    finally:
        model.train()
    return meter.result(reduce=pconfig.is_distributed and pconfig.dp_size > 1), state
