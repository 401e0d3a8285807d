#!/usr/bin/env bash
# Prepare a B200 node for parallel_b200: check the toolchain, build the sm_100a
# kernels in-tree and point the Hugging Face caches at one shared directory.
#
#   ./install.sh                 # build in-tree (parallel_b200/_C*.so)
#   ./install.sh --editable      # also `pip install -e .` (console script parallel-b200-train)
#   CACHE_ROOT=/data/cache ./install.sh
#
# Nothing is downloaded: PyTorch (with CUDA 12.8+ and NCCL), nvcc 12.8+ and
# ninja must already be present.  The script never changes GPU settings.
set -euo pipefail
cd "$(dirname "$0")"

PY=${PYTHON:-python}
CACHE_ROOT=${CACHE_ROOT:-$HOME/.cache}

need() { command -v "$1" >/dev/null 2>&1 || { echo "install.sh: '$1' not found on PATH" >&2; exit 1; }; }
need "$PY"
need nvcc
need ninja

"$PY" - <<'PYCHECK'
import sys
import torch
v = tuple(int(x) for x in torch.__version__.split("+")[0].split(".")[:2])
if v < (2, 4):
    sys.exit(f"install.sh: PyTorch {torch.__version__} is too old (2.4 or newer)")
if not torch.distributed.is_nccl_available():
    sys.exit("install.sh: this PyTorch build has no NCCL backend")
print(f"torch {torch.__version__}, CUDA {torch.version.cuda}, NCCL {'.'.join(map(str, torch.cuda.nccl.version()))}")
if torch.cuda.is_available():
    caps = {torch.cuda.get_device_capability(i) for i in range(torch.cuda.device_count())}
    if caps != {(10, 0)}:
        print(f"install.sh: warning: the kernels target sm_100a (B200); this node reports {sorted(caps)}")
PYCHECK

nvcc --version | tail -n 2
MAX_JOBS=${MAX_JOBS:-$(nproc)} "$PY" setup.py build_ext --inplace
"$PY" -c "import parallel_b200._C as C; print('built', C.__file__)"

if [[ "${1:-}" == "--editable" ]]; then
    "$PY" -m pip install --no-build-isolation --no-deps -e .
fi

cat <<ENV
# add to the shell profile of the training user:
export HF_HOME=$CACHE_ROOT/huggingface
export HF_HUB_CACHE=$CACHE_ROOT/huggingface/hub
export HF_DATASETS_CACHE=$CACHE_ROOT/huggingface/datasets
ENV
