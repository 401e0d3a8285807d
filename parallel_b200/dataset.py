"""Pre-training corpus shards: listing, reading and downloading.

The corpus is the climbmix parquet shard set the reference trains on
(``parallel/parallel/dataset.py``): ``shard_00000.parquet`` ...
``shard_06542.parquet`` with the last one pinned as the validation split, each
row holding a ``text`` column.  CLI (same flags as the reference):
``python -m parallel_b200.dataset -n 50 -w 24 [data.dir=...]`` fetches the
first N training shards plus the validation shard into ``data.dir``.

Downloads stream into a hidden temporary file in the target directory and
are renamed into place only when complete, so an interrupted or failed
download never leaves a file that ``list_data_files`` would pick up.  A
failed attempt is retried after 2, 4, 8, ... seconds, a bounded number of
times.  Transfers use the standard library's ``urllib`` and run on a thread
pool (the work is network-bound).
"""
from __future__ import annotations

import argparse
import os
import shutil
import tempfile
import time
import urllib.error
import urllib.request
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

from .config import load_cfg

BASE_URL = "https://huggingface.co/datasets/karpathy/climbmix-400b-shuffle/resolve/main"
MAX_SHARD = 6542  # index of the validation shard (the last one)
_TIMEOUT_S = 30


def index_to_filename(index: int) -> str:
    return f"shard_{index:05d}.parquet"


def list_data_files(data_dir: str | None = None) -> list[str]:
    """Paths of the complete local shards in name order (validation last)."""
    if data_dir is None:
        data_dir = load_cfg(argv=[a for a in os.sys.argv[1:] if "=" in a]).data.dir
    root = Path(data_dir) if data_dir else None
    if root is None or not root.is_dir():
        raise RuntimeError(f"data directory {data_dir!r} does not exist (download shards first)")
    return [str(p) for p in sorted(root.glob("*.parquet"))]


def iter_batched(split: str, start: int = 0, step: int = 1, data_dir: str | None = None):
    """Yield the ``text`` column of row groups start, start+step, ... of every
    shard of ``split`` ("train": all but the last shard, "val": the last)."""
    import pyarrow.parquet as pq

    if split not in ("train", "val"):
        raise ValueError(f"split must be 'train' or 'val', got {split!r}")
    shards = list_data_files(data_dir)
    for path in (shards[:-1] if split == "train" else shards[-1:]):
        reader = pq.ParquetFile(path)
        for group in range(start, reader.num_row_groups, step):
            yield reader.read_row_group(group).column("text").to_pylist()


def _fetch(url: str, target: Path) -> None:
    """One attempt: stream ``url`` into a temporary sibling of ``target``,
    then rename it into place; the temporary file never survives a failure."""
    fd, partial = tempfile.mkstemp(prefix=f".{target.name}.", suffix=".tmp", dir=target.parent)
    try:
        with os.fdopen(fd, "wb") as out, urllib.request.urlopen(url, timeout=_TIMEOUT_S) as response:
            shutil.copyfileobj(response, out, length=1 << 20)
        os.replace(partial, target)
    finally:
        if os.path.exists(partial):
            os.unlink(partial)


def download_single_file(data_dir: str, idx: int, max_attempts: int = 5) -> bool:
    """Fetch shard ``idx`` into ``data_dir`` unless it is already there.
    Returns whether the shard is present afterwards."""
    target = Path(data_dir) / index_to_filename(idx)
    if target.exists():
        print(f"{target.name}: present, not fetched")
        return True
    url = f"{BASE_URL}/{target.name}"
    for attempt in range(1, max_attempts + 1):
        try:
            _fetch(url, target)
            print(f"{target.name}: fetched")
            return True
        except (urllib.error.URLError, OSError) as exc:
            print(f"{target.name}: attempt {attempt} of {max_attempts} failed ({exc})")
            if attempt < max_attempts:
                time.sleep(2 ** attempt)
    print(f"{target.name}: giving up after {max_attempts} attempts")
    return False


def main(argv=None):
    parser = argparse.ArgumentParser(description="Fetch pre-training corpus shards")
    parser.add_argument("-n", "--num-files", type=int, default=-1, help="training shards to fetch (-1: all)")
    parser.add_argument("-w", "--num-workers", type=int, default=24, help="parallel transfers")
    args, overrides = parser.parse_known_args(argv)
    data_dir = load_cfg(argv=overrides).data.dir
    os.makedirs(data_dir, exist_ok=True)
    train = MAX_SHARD if args.num_files < 0 else min(args.num_files, MAX_SHARD)
    wanted = [*range(train), MAX_SHARD]
    print(f"fetching {len(wanted)} shards into {data_dir} with {args.num_workers} workers")
    with ThreadPoolExecutor(max_workers=max(1, args.num_workers)) as pool:
        present = list(pool.map(lambda i: download_single_file(data_dir, i), wanted))
    print(f"{sum(present)} of {len(wanted)} shards present in {data_dir}")
    return 0 if all(present) else 1


if __name__ == "__main__":
    raise SystemExit(main())
