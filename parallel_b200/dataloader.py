"""Distributed, exactly-resumable pre-training data loader (+ synthetic loader).

``dist_data_loader(tokenizer, B, T, split, ...)`` yields ``(x, y, state)``:
row groups of the parquet shards are strided over data ranks
(``rg = data_rank + k * data_world_size``), documents are tokenised with BOS
prepended and packed best-fit into rows of T+1 tokens (the longest buffered
document that fits; when none fits, the shortest one is cropped), and the
rows are staged in pinned memory and copied to the device asynchronously.
``state`` (pq_idx, rg_idx, epoch, batch_idx, doc_buffer, dataset identity,
loader config) resumes the stream exactly; resuming rejects changed data
files or loader configuration.  Semantics follow parallel/parallel/
dataloader.py:11-213; the packer keeps its buffer ordered by (length,
arrival) so each pick is O(log n) instead of a scan.

``synthetic_data_loader`` yields uniform random token ids of the same shape
(``data.synthetic=true``).
"""
from __future__ import annotations

import bisect
import copy
import itertools
from pathlib import Path

import torch

from .dataset import list_data_files


def _split_data_files(split: str, data_dir: str | None = None) -> list[str]:
    paths = list_data_files(data_dir)
    if not paths:
        raise RuntimeError("No data found; run dataset.py first")
    if split == "train" and len(paths) < 2:
        raise RuntimeError("Training requires at least two data files because the final file is reserved for "
                           "validation")
    sel = paths[:-1] if split == "train" else paths[-1:]
    return [str(Path(p).resolve()) for p in sel]


def _dataset_identity(paths: list[str]) -> list[dict]:
    out = []
    for p in paths:
        st = Path(p).stat()
        out.append({"path": p, "size": st.st_size, "mtime_ns": st.st_mtime_ns})
    return out


def _create_batches(split, resume, tokenizer_batch_size, data_rank, data_world_size, file_paths):
    import pyarrow.parquet as pq

    r_pq = resume["pq_idx"] if resume is not None else 0
    r_rg = resume["rg_idx"] if resume is not None else None
    r_batch = resume.get("batch_idx") if resume is not None else None
    epoch = resume.get("epoch", 1) if resume is not None else 1
    first = True
    while True:
        pq_idx = r_pq if first else 0
        while pq_idx < len(file_paths):
            pf = pq.ParquetFile(file_paths[pq_idx])
            if first and r_rg is not None and pq_idx == r_pq:
                rg = ((r_rg // data_world_size) + 1) * data_world_size + data_rank if r_batch is None else r_rg
            else:
                rg = data_rank
            while rg < pf.num_row_groups:
                texts = pf.read_row_group(rg).column("text").to_pylist()
                start = 0
                if first and pq_idx == r_pq and rg == r_rg and r_batch is not None:
                    start = r_batch + 1
                for bi, i in enumerate(range(0, len(texts), tokenizer_batch_size)):
                    if bi < start:
                        continue
                    yield texts[i:i + tokenizer_batch_size], (pq_idx, rg, epoch, bi)
                r_rg = None
                r_batch = None
                rg += data_world_size
            pq_idx += 1
        first = False
        epoch += 1


class _BestFitBuffer:
    """Document buffer with the reference's best-fit choices in O(log n).

    ``docs`` is the live list in arrival order (this is what checkpoints
    store); an index sorted by (length, arrival) answers "first-arrived
    longest doc with length <= r" and "first-arrived shortest doc"."""

    def __init__(self, docs: list):
        self.docs = docs
        self._seq = itertools.count()
        self._entries: dict[int, list] = {}
        self._keys: list = []
        for d in docs:
            self._index(d)

    def _index(self, doc):
        s = next(self._seq)
        self._entries[s] = doc
        bisect.insort(self._keys, (len(doc), s))

    def append(self, doc):
        self.docs.append(doc)
        self._index(doc)

    def __len__(self):
        return len(self.docs)

    def _pop_key(self, pos):
        ln, s = self._keys.pop(pos)
        doc = self._entries.pop(s)
        # remove the same object from the ordered live list
        for i, d in enumerate(self.docs):
            if d is doc:
                del self.docs[i]
                break
        return doc

    def pop_best_fit(self, remaining: int):
        """Longest doc with len <= remaining (earliest among equals), else None."""
        pos = bisect.bisect_right(self._keys, (remaining, float("inf"))) - 1
        if pos < 0:
            return None
        ln = self._keys[pos][0]
        first = bisect.bisect_left(self._keys, (ln, -1))
        return self._pop_key(first)

    def pop_shortest(self):
        return self._pop_key(0)


def dist_data_loader(tokenizer, B, T, split, tokenizer_batch_size=128, device="cuda", resume_state_dict=None,
                     buffer_size=1000, pconfig=None, data_dir: str | None = None):
    assert split in ("train", "val"), "split must be train/val"
    cap = T + 1
    data_rank = pconfig.data_rank if pconfig is not None else 0
    data_world = pconfig.data_world_size if pconfig is not None else 1
    paths = _split_data_files(split, data_dir)
    identity = _dataset_identity(paths)
    loader_config = {
        "split": split, "batch_size": B, "sequence_length": T, "tokenizer_batch_size": tokenizer_batch_size,
        "buffer_size": buffer_size, "data_rank": data_rank, "data_world_size": data_world,
        "tokenizer_class": f"{type(tokenizer).__module__}.{type(tokenizer).__qualname__}",
        "tokenizer_name": getattr(tokenizer, "name_or_path", None),
        "tokenizer_vocab_size": getattr(tokenizer, "vocab_size", None),
        "bos_token_id": tokenizer.bos_token_id,
    }
    if resume_state_dict is not None:
        if resume_state_dict.get("dataset") != identity:
            raise RuntimeError("Cannot resume dataloader because the dataset files have changed")
        if resume_state_dict.get("loader_config") != loader_config:
            raise RuntimeError("Cannot resume dataloader because its configuration has changed")
    batches = _create_batches(split, resume_state_dict, tokenizer_batch_size, data_rank, data_world, paths)
    bos = tokenizer.bos_token_id
    docs = copy.deepcopy(resume_state_dict.get("doc_buffer", []) if resume_state_dict is not None else [])
    buf = _BestFitBuffer(docs)
    pos_state = {"pq_idx": 0, "rg_idx": 0, "epoch": 1, "batch_idx": -1}

    def refill():
        texts, (pq_i, rg_i, ep, bi) = next(batches)
        pos_state.update(pq_idx=pq_i, rg_idx=rg_i, epoch=ep, batch_idx=bi)
        for ids in tokenizer(texts, add_special_tokens=False)["input_ids"]:
            buf.append(([bos] + ids) if bos is not None else ids)

    use_cuda = torch.device(device).type == "cuda"
    rows = torch.empty((B, cap), dtype=torch.long)
    dev = torch.empty(2 * B * T, dtype=torch.long, device=device)
    x, y = dev[:B * T].view(B, T), dev[B * T:].view(B, T)
    while True:
        for r in range(B):
            pos = 0
            while pos < cap:
                while len(buf) < buffer_size:
                    refill()
                rem = cap - pos
                doc = buf.pop_best_fit(rem)
                if doc is not None:
                    rows[r, pos:pos + len(doc)] = torch.tensor(doc, dtype=torch.long)
                    pos += len(doc)
                else:
                    doc = buf.pop_shortest()
                    rows[r, pos:pos + rem] = torch.tensor(doc[:rem], dtype=torch.long)
                    pos += rem
        # a fresh pinned staging tensor per batch (from the caching host allocator,
        # which keeps it alive until its asynchronous copy has run): refilling one
        # reused buffer could overwrite a batch whose copy is still queued
        cpu = torch.empty(2 * B * T, dtype=torch.long, pin_memory=use_cuda)
        cpu[:B * T].view(B, T).copy_(rows[:, :-1])
        cpu[B * T:].view(B, T).copy_(rows[:, 1:])
        state = {**pos_state, "doc_buffer": buf.docs, "dataset": identity, "loader_config": loader_config}
        dev.copy_(cpu, non_blocking=use_cuda)
        yield x, y, state


def synthetic_data_loader(B, T, vocab_size, device="cuda", seed: int = 0, pconfig=None, resume_state_dict=None):
    """Uniform random token ids (per-data-rank stream); state = step count."""
    rank = pconfig.data_rank if pconfig is not None else 0
    step = int(resume_state_dict.get("step", 0)) if resume_state_dict else 0
    use_cuda = torch.device(device).type == "cuda"
    while True:
        g = torch.Generator().manual_seed(seed * 1_000_003 + rank * 7919 + step)
        # a fresh host tensor per batch: a reused buffer would alias the previous
        # batch on CPU and could be refilled before its asynchronous copy ran on
        # CUDA (the pinned block is kept alive by the host allocator until then)
        host = torch.randint(0, vocab_size, (B, T + 1), generator=g)
        tok = host.pin_memory().to(device, non_blocking=True) if use_cuda else host
        step += 1
        yield tok[:, :-1], tok[:, 1:], {"step": step, "synthetic": True, "seed": seed, "data_rank": rank}
