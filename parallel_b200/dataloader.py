"""Distributed, exactly-resumable pre-training data loader (+ synthetic loader).

``dist_data_loader(tokenizer, B, T, split, ...)`` yields ``(x, y, state)``:
row groups of the parquet shards are strided over data ranks
(``rg = data_rank + k * data_world_size``), documents are tokenised with BOS
prepended and packed best-fit into rows of T+1 tokens (the longest buffered
document that fits; when none fits, the shortest one is cropped), and the
rows are staged in pinned memory and copied to the device asynchronously.
``state`` (pq_idx, rg_idx, epoch, batch_idx, doc_buffer, dataset identity,
loader config) resumes the stream exactly; resuming rejects changed data
files or loader configuration.  Behaviour (row-group striding, packing
choices, resume position and state keys) is that of the reference's
parallel/parallel/dataloader.py:11-213; the packer keeps its buffer ordered by
(length, arrival) so each pick is O(log n) instead of a scan.

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
    """Resolved shard paths of ``split``: the last shard is validation, the
    rest are training (which therefore needs at least two shards)."""
    shards = [str(Path(p).resolve()) for p in list_data_files(data_dir)]
    if not shards:
        raise RuntimeError("no data shards found; download them with python -m parallel_b200.dataset")
    if split == "train":
        if len(shards) == 1:
            raise RuntimeError("training needs two or more shards: the last shard is the validation split")
        return shards[:-1]
    return shards[-1:]


def _dataset_identity(paths: list[str]) -> list[dict]:
    """(path, size, modification time) of every shard: a resumed loader must
    see the very same files."""
    stats = [(p, Path(p).stat()) for p in paths]
    return [{"path": p, "size": st.st_size, "mtime_ns": st.st_mtime_ns} for p, st in stats]


def _resume_position(resume, data_rank: int, data_world: int):
    """(shard, row group, first text chunk, epoch) to continue from.

    A state records the last chunk handed out (``batch_idx``); the walk goes
    on with the next chunk of that row group.  A state without a chunk index
    continues with this rank's next row group of that shard."""
    if resume is None:
        return 0, data_rank, 0, 1
    shard, group, chunk, epoch = resume["pq_idx"], resume.get("rg_idx"), resume.get("batch_idx"), resume.get("epoch", 1)
    if group is None:
        return shard, data_rank, 0, epoch
    if chunk is None:
        return shard, (group // data_world + 1) * data_world + data_rank, 0, epoch
    return shard, group, chunk + 1, epoch


def _create_batches(split, resume, tokenizer_batch_size, data_rank, data_world_size, file_paths):
    """Endless walk over this data rank's row groups (every ``data_world_size``-th
    group of every shard, starting at ``data_rank``), yielding text chunks of
    ``tokenizer_batch_size`` documents with their position
    (shard, row group, epoch, chunk); the next epoch restarts at shard 0."""
    import pyarrow.parquet as pq

    shard, group0, chunk0, epoch = _resume_position(resume, data_rank, data_world_size)
    while True:
        for s in range(shard, len(file_paths)):
            reader = pq.ParquetFile(file_paths[s])
            first_group = group0 if s == shard else data_rank
            for g in range(first_group, reader.num_row_groups, data_world_size):
                texts = reader.read_row_group(g).column("text").to_pylist()
                starts = range(0, len(texts), tokenizer_batch_size)
                skip = chunk0 if (s == shard and g == first_group) else 0
                for c in range(skip, len(starts)):
                    yield texts[starts[c]:starts[c] + tokenizer_batch_size], (s, g, epoch, c)
        shard, group0, chunk0, epoch = 0, data_rank, 0, epoch + 1


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
            raise RuntimeError("dataloader state was saved for different data files; refusing to resume")
        if resume_state_dict.get("loader_config") != loader_config:
            raise RuntimeError("dataloader state was saved with a different batch / sequence / tokenizer setup; refusing to resume")
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
