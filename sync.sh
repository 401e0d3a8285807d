#!/usr/bin/env bash
# Mirror this source tree to a training node over ssh (rsync), leaving out
# build products, caches and run outputs; with --watch, re-sync on every
# change (needs inotifywait or fswatch locally).
#
#   ./sync.sh HOST [PORT] [--watch]
#   REMOTE_USER=ubuntu REMOTE_DIR=work/parallel_b200 SSH_KEY=~/.ssh/id_ed25519 ./sync.sh 10.0.0.5 22
#
# REMOTE_DIR is relative to the remote user's home unless it starts with /.
#
# The compiled extension is not copied: run ./install.sh on the node (the
# kernels are built for the node's own toolchain).
set -euo pipefail
cd "$(dirname "$0")"

HOST=${1:?usage: ./sync.sh HOST [PORT] [--watch]}
PORT=22
WATCH=0
for a in "${@:2}"; do
    case "$a" in
        --watch) WATCH=1 ;;
        *) PORT=$a ;;
    esac
done
REMOTE_USER=${REMOTE_USER:-root}
REMOTE_DIR=${REMOTE_DIR:-parallel_b200}
SSH_KEY=${SSH_KEY:-$HOME/.ssh/id_ed25519}
SSH="ssh -p $PORT -i $SSH_KEY -o StrictHostKeyChecking=accept-new"

sync_once() {
    rsync -az --delete -e "$SSH" \
        --exclude '.git/' --exclude '__pycache__/' --exclude '*.pyc' --exclude '.pytest_cache/' \
        --exclude 'build/' --exclude '*.egg-info/' --exclude '*.so' --exclude '*.o' \
        --exclude '.ninja*' --exclude 'checkpoints/' --exclude 'wandb/' --exclude 'baseline/_ref/' \
        ./ "$REMOTE_USER@$HOST:$REMOTE_DIR/"
    echo "synced to $HOST:$REMOTE_DIR"
}

sync_once
if [[ $WATCH == 1 ]]; then
    if command -v inotifywait >/dev/null 2>&1; then
        while inotifywait -qq -r -e modify,create,delete,move --exclude '(\.git|__pycache__|build)/' .; do
            sync_once
        done
    elif command -v fswatch >/dev/null 2>&1; then
        fswatch -o -r --exclude '\.git/' --exclude '__pycache__' --exclude 'build/' . | while read -r _; do
            sync_once
        done
    else
        echo "sync.sh: --watch needs inotifywait or fswatch" >&2
        exit 1
    fi
fi
