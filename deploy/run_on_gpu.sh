#!/bin/bash
# Staged, resumable measurement run on a B200 box. Each stage writes a marker
# under $OUT/.stages; a rerun skips finished stages (delete a marker to redo it).
#
#   bash deploy/run_on_gpu.sh [out_dir] [gpus]
set -uo pipefail
OUT=${1:-results}
GPUS=${2:-$(nvidia-smi -L 2>/dev/null | wc -l)}
mkdir -p "$OUT/.stages" "$OUT/logs"

stage() {  # stage <name> <command...>
  local name=$1; shift
  if [ -f "$OUT/.stages/$name" ]; then echo "[skip] $name"; return 0; fi
  echo "[run ] $name"
  if "$@" > "$OUT/logs/$name.log" 2>&1; then touch "$OUT/.stages/$name"; echo "[ok  ] $name";
  else echo "[FAIL] $name (see $OUT/logs/$name.log)"; return 1; fi
}

stage preflight   python -m gpt2_harness_b200.preflight --world-sizes 1 "$GPUS" --out "$OUT/preflight.json" || exit 1
stage build       python -c "import __graft_entry__ as g; g.build(); g.smoke()" || exit 1
stage gpu_tests   python -m pytest tests -m gpu -q
stage bench_1gpu  bash -c "python bench.py --gpus 1 >> '$OUT/scaling.jsonl'"
for n in 2 4 8; do
  if [ "$GPUS" -ge "$n" ]; then
    stage "bench_${n}gpu" bash -c "timeout -k 60 900 python -m torch.distributed.run --nnodes=1 --nproc-per-node=$n \
      --master-addr 127.0.0.1 --master-port $((29520 + n)) bench.py --gpus $n >> '$OUT/scaling.jsonl'"
  fi
done
stage kernels     python -m gpt2_harness_b200.perf.kernel_bench --json "$OUT/kernels.json"
stage roofline    python -m gpt2_harness_b200.perf.roofline --out "$OUT/roofline.json"
stage parallel    python -m gpt2_harness_b200.parallel.run_parallel --world-size 2 --out "$OUT/parallel_comms.json"
stage collectives python -m gpt2_harness_b200.cluster.collbench --world "$((GPUS >= 2 ? GPUS : 2))" \
                    --json "$OUT/collectives.json"
stage cluster     python -m gpt2_harness_b200.cluster.run_cluster --out "$OUT/cluster.json" --skip collectives
stage experiments python -m gpt2_harness_b200.experiments all --out "$OUT" --figures "$OUT/figures"
# a second pass must run nothing (every stage already has its marker)
if [ -z "${G2B_SECOND_PASS:-}" ]; then
  stage idempotent bash -c "G2B_SECOND_PASS=1 bash '$0' '$OUT' '$GPUS' | grep -q '\[run \]' && exit 1 || exit 0"
fi
echo "done: $OUT"
