"""The node scripts beside the package (install.sh, sync.sh): they parse, and
sync.sh refuses to run without a host (no ssh attempt is made)."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_scripts_parse():
    for name in ("install.sh", "sync.sh"):
        subprocess.run(["bash", "-n", os.path.join(ROOT, name)], check=True)


def test_sync_requires_a_host():
    r = subprocess.run(["bash", os.path.join(ROOT, "sync.sh")], capture_output=True, text=True)
    assert r.returncode != 0
    assert "usage" in r.stderr
