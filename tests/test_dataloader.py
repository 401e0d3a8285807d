"""Resumable best-fit packing loader over tiny parquet shards."""
import pyarrow as pa
import pyarrow.parquet as pq
import pytest
import torch

from parallel_b200 import dataloader as DL


class FakeTokenizer:
    bos_token_id = 1
    vocab_size = 100
    name_or_path = "fake"

    def __call__(self, texts, add_special_tokens=False):
        return {"input_ids": [[2 + (ord(c) % 90) for c in t] for t in texts]}


def _write(tmp_path, nfiles=3, groups=4, docs=6):
    for f in range(nfiles):
        tbl = [[f"doc{f}-{g}-{i}" + "x" * ((f * 7 + g * 3 + i * 5) % 13) for i in range(docs)]
               for g in range(groups)]
        with pq.ParquetWriter(tmp_path / f"shard_{f:05d}.parquet", pa.schema([("text", pa.string())])) as w:
            for rows in tbl:
                w.write_table(pa.table({"text": rows}))


def _loader(tmp_path, state=None, **kw):
    return DL.dist_data_loader(FakeTokenizer(), 2, 16, "train", tokenizer_batch_size=2, device="cpu",
                               resume_state_dict=state, buffer_size=5, data_dir=str(tmp_path), **kw)


def test_exact_resume_replays_next_batch(tmp_path):
    import copy

    _write(tmp_path)
    it = _loader(tmp_path)
    for _ in range(3):
        x, y, st = next(it)
    saved = copy.deepcopy(st)
    nxt = [next(it)[0].clone() for _ in range(3)]
    it2 = _loader(tmp_path, state=saved)
    again = [next(it2)[0].clone() for _ in range(3)]
    for a, b in zip(nxt, again):
        assert torch.equal(a, b)


def test_targets_are_shifted_inputs(tmp_path):
    _write(tmp_path)
    x, y, _ = next(_loader(tmp_path))
    assert torch.equal(x[:, 1:], y[:, :-1])


def test_state_buffer_is_live_reference(tmp_path):
    _write(tmp_path)
    it = _loader(tmp_path)
    _, _, s1 = next(it)
    buf = s1["doc_buffer"]
    _, _, s2 = next(it)
    assert s2["doc_buffer"] is buf


def test_resume_rejects_changed_config_or_data(tmp_path):
    import copy
    import os

    _write(tmp_path)
    _, _, st = next(_loader(tmp_path))
    st = copy.deepcopy(st)
    bad = copy.deepcopy(st)
    bad["loader_config"]["batch_size"] = 99
    with pytest.raises(RuntimeError, match="different batch"):
        next(_loader(tmp_path, state=bad))
    p = tmp_path / "shard_00000.parquet"
    os.utime(p, ns=(p.stat().st_atime_ns, p.stat().st_mtime_ns + 10 ** 9))
    with pytest.raises(RuntimeError, match="different data files"):
        next(_loader(tmp_path, state=st))


def test_best_fit_buffer_matches_linear_scan():
    import random

    rng = random.Random(0)
    docs = [[0] * rng.randint(1, 20) for _ in range(40)]
    ref = [list(d) for d in docs]
    buf = DL._BestFitBuffer([list(d) for d in docs])
    for _ in range(30):
        rem = rng.randint(1, 25)
        best, best_len = -1, 0
        for i, d in enumerate(ref):
            if len(d) <= rem and len(d) > best_len:
                best, best_len = i, len(d)
        got = buf.pop_best_fit(rem)
        if best >= 0:
            assert got is not None and len(got) == len(ref.pop(best))
        else:
            assert got is None
            short = min(range(len(ref)), key=lambda i: len(ref[i]))
            assert len(buf.pop_shortest()) == len(ref.pop(short))
        assert [len(d) for d in buf.docs] == [len(d) for d in ref]


def test_synthetic_loader_shapes_and_resume():
    it = DL.synthetic_data_loader(2, 8, 50, device="cpu", seed=3)
    a = [next(it) for _ in range(3)]
    it2 = DL.synthetic_data_loader(2, 8, 50, device="cpu", seed=3, resume_state_dict=a[1][2])
    assert torch.equal(next(it2)[0], a[2][0])
    assert a[0][0].shape == (2, 8) and int(a[0][0].max()) < 50
