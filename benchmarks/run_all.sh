#!/usr/bin/env bash
# Run the benchmark suite and keep every artefact under results/<timestamp>/.
#
#   benchmarks/run_all.sh                        # all visible GPUs
#   NPROC=4 benchmarks/run_all.sh
#   BACKEND=gloo NPROC=4 benchmarks/run_all.sh   # CPU dry run (exercises code, not performance)
set -euo pipefail
cd "$(dirname "$0")/.."
NPROC="${NPROC:-$(python -c 'import torch; print(max(1, torch.cuda.device_count()))')}"
BACKEND_ARG=""
[ -n "${BACKEND:-}" ] && BACKEND_ARG="--backend $BACKEND"
OUT="results/$(date +%Y%m%d_%H%M%S)"
mkdir -p "$OUT/traces"
RUN="python -m torch.distributed.run --nnodes=1 --nproc-per-node=$NPROC --master-addr=127.0.0.1 --master-port=${PORT:-29561}"
{
  echo "host:  $(uname -a)"
  echo "nproc: $NPROC"
  python -c 'import torch; print("torch:", torch.__version__, "cuda:", torch.version.cuda)'
  python -c 'import torch; [print("gpu", i, torch.cuda.get_device_name(i)) for i in range(torch.cuda.device_count())]'
} | tee "$OUT/environment.txt"
PREC=""
[ -z "${BACKEND:-}" ] && python -c 'import torch, sys; sys.exit(0 if torch.cuda.is_available() else 1)' && PREC="--precision bf16"
$RUN benchmarks/bench_collectives.py --max-mb 256 --json "$OUT/collectives.jsonl" $BACKEND_ARG 2>&1 | tee "$OUT/collectives.txt"
$RUN benchmarks/bench_parallelism.py --trace-dir "$OUT/traces" --json "$OUT/parallelism.jsonl" $PREC $BACKEND_ARG 2>&1 | tee "$OUT/parallelism.txt"
if [ "$NPROC" -ge 2 ]; then
  $RUN benchmarks/bench_pipeline.py --microbatches 1,2,4,8,16 --gantt --json "$OUT/pipeline.jsonl" $PREC $BACKEND_ARG 2>&1 | tee "$OUT/pipeline.txt"
fi
python benchmarks/analyze_trace.py "$OUT"/traces/*_rank*.json --kernels 15 --csv "$OUT/overlap.csv" --json "$OUT/overlap.json" 2>&1 | tee "$OUT/overlap.txt" || true
echo "done -> $OUT"
