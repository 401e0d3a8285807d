"""Dataset shard downloader against a local HTTP server on 127.0.0.1 (no
external network): download, skip of existing shards, bounded retries that
leave no partial file behind."""
import functools
import http.server
import os
import threading

import pytest

from parallel_b200 import dataset as D


@pytest.fixture()
def server(tmp_path):
    root = tmp_path / "remote"
    root.mkdir()
    handler = functools.partial(http.server.SimpleHTTPRequestHandler, directory=str(root))
    handler.log_message = lambda *a, **k: None
    httpd = http.server.ThreadingHTTPServer(("127.0.0.1", 0), handler)
    t = threading.Thread(target=httpd.serve_forever, daemon=True)
    t.start()
    yield root, f"http://127.0.0.1:{httpd.server_address[1]}"
    httpd.shutdown()
    httpd.server_close()


def test_download_skip_and_bounded_retries(tmp_path, server, monkeypatch):
    root, url = server
    monkeypatch.setattr(D, "BASE_URL", url)
    sleeps = []
    monkeypatch.setattr(D.time, "sleep", sleeps.append)
    local = tmp_path / "data"
    local.mkdir()
    name = D.index_to_filename(3)
    (root / name).write_bytes(b"parquet bytes" * 1000)
    assert D.download_single_file(str(local), 3)
    assert (local / name).read_bytes() == (root / name).read_bytes()
    # an existing shard is not fetched again
    (root / name).write_bytes(b"changed")
    assert D.download_single_file(str(local), 3)
    assert (local / name).read_bytes() != b"changed"
    # a missing shard: bounded retries with backoff, nothing left behind
    assert not D.download_single_file(str(local), 4, max_attempts=3)
    assert sleeps == [2, 4]
    assert sorted(os.listdir(local)) == [name]
