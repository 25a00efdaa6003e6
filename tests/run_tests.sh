#!/usr/bin/env bash
# CPU correctness suite (Gloo) plus a torchrun smoke test of the trainer; on a
# CUDA machine also the GPU tier (`-m gpu`).
set -euo pipefail
cd "$(dirname "$0")/.."
# Syntax / undefined-name check of every Python file (ruff when installed, else byte-compilation).
if command -v ruff >/dev/null 2>&1; then
  ruff check --select E9,F63,F7,F82 minidist tests benchmarks examples bench.py
else
  python -m compileall -q minidist tests benchmarks examples bench.py >/dev/null
fi
python -m pytest tests -q -m "not gpu" "$@"
python -m torch.distributed.run --nnodes=1 --nproc-per-node=4 --master-addr=127.0.0.1 --master-port=29562 \
  examples/train_gpt.py --tp 2 --pp 2 --strategy none --microbatches 4 --layers 4 --embd 128 --heads 4 \
  --vocab 1024 --seq-len 64 --batch-size 8 --steps 4 --backend gloo
if python -c 'import torch, sys; sys.exit(0 if torch.cuda.is_available() else 1)'; then
  python -m pytest tests -q -m gpu
fi
echo "all green"
