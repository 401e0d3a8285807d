"""Pre-training shard downloader / lister (climbmix parquet shards).

Same CLI and layout as the reference (parallel/parallel/dataset.py):
``python -m parallel_b200.dataset -n 50 -w 24 [data.dir=...]`` downloads the
first N train shards plus the pinned validation shard (the last file) into
``data.dir`` with retries and temp-file renames.  ``list_data_files`` lists
the local shards in order; the final file is the validation split.
"""
from __future__ import annotations

import argparse
import os
import time
from functools import partial
from multiprocessing import Pool

from .config import load_cfg

BASE_URL = "https://huggingface.co/datasets/karpathy/climbmix-400b-shuffle/resolve/main"
MAX_SHARD = 6542  # shard_06542.parquet is the validation shard


def index_to_filename(index: int) -> str:
    return f"shard_{index:05d}.parquet"


def list_data_files(data_dir: str | None = None) -> list[str]:
    if data_dir is None:
        data_dir = load_cfg(argv=[a for a in os.sys.argv[1:] if "=" in a]).data.dir
    if not data_dir or not os.path.isdir(data_dir):
        raise RuntimeError("Data directory does not exist")
    return sorted(os.path.join(data_dir, f) for f in os.listdir(data_dir)
                  if f.endswith(".parquet") and not f.endswith(".tmp"))


def iter_batched(split: str, start: int = 0, step: int = 1, data_dir: str | None = None):
    import pyarrow.parquet as pq

    assert split in ("train", "val"), "split must be train/val"
    paths = list_data_files(data_dir)
    paths = paths[:-1] if split == "train" else paths[-1:]
    for path in paths:
        pf = pq.ParquetFile(path)
        for rg in range(start, pf.num_row_groups, step):
            yield pf.read_row_group(rg).column("text").to_pylist()


def download_single_file(data_dir: str, idx: int, max_attempts: int = 5) -> bool:
    import requests

    name = index_to_filename(idx)
    path = os.path.join(data_dir, name)
    if os.path.exists(path):
        print(f"Skipping {path} -- already exists")
        return True
    url = f"{BASE_URL}/{name}"
    for attempt in range(1, max_attempts + 1):
        tmp = path + ".tmp"
        try:
            with requests.get(url, stream=True, timeout=30) as r:
                r.raise_for_status()
                with open(tmp, "wb") as f:
                    for chunk in r.iter_content(chunk_size=1 << 20):
                        if chunk:
                            f.write(chunk)
            os.rename(tmp, path)
            print(f"Successfully downloaded {name}")
            return True
        except (requests.RequestException, OSError) as e:
            print(f"Attempt {attempt}/{max_attempts} failed for {name}: {e}")
            for p in (tmp, path):
                if os.path.exists(p):
                    try:
                        os.remove(p)
                    except OSError:
                        pass
            if attempt < max_attempts:
                time.sleep(2 ** attempt)
    print(f"Failed to download {name} after {max_attempts} attempts")
    return False


def main(argv=None):
    ap = argparse.ArgumentParser(description="Download pretraining dataset shards")
    ap.add_argument("-n", "--num-files", type=int, default=-1, help="train shards to download (-1 = all)")
    ap.add_argument("-w", "--num-workers", type=int, default=24)
    args, rest = ap.parse_known_args(argv)
    cfg = load_cfg(argv=rest)
    data_dir = cfg.data.dir
    os.makedirs(data_dir, exist_ok=True)
    n = MAX_SHARD if args.num_files == -1 else min(args.num_files, MAX_SHARD)
    ids = list(range(n)) + [MAX_SHARD]
    print(f"Downloading {len(ids)} shards using {args.num_workers} workers into {data_dir}")
    with Pool(processes=args.num_workers) as pool:
        ok = pool.map(partial(download_single_file, data_dir), ids)
    print(f"Done! Downloaded: {sum(ok)}/{len(ids)} shards to {data_dir}")


if __name__ == "__main__":
    main()
