#!/usr/bin/env bash
# Launch menu for the common jobs (reference: run.sh).  Usage: ./run.sh [command] [args...]
#   data      <input> <out_dir>         curate + tokenise a corpus
#   train     <config> [n_gpus] [...]   pre-train (DP over n GPUs; pass --ep N for expert parallelism)
#   train4d   <config> <n_gpus> [...]   4-D parallel pre-training (--dp/--tp/--pp/--ep)
#   grpo      <config> <ckpt> [...]     GRPO / S-GRPO fine-tuning
#   generate  <config> [ckpt] [...]     interactive generation (add --thinking DeepThink ...)
#   eval      <config> [ckpt] [...]     benchmark evaluation
#   bench     [n_gpus]                  headline throughput benchmark
#   test                                run the test suite
set -euo pipefail
cd "$(dirname "$0")"
PY=${PYTHON:-python}
launch() {  # n_gpus script args...
  local n=$1; shift
  if [ "$n" -gt 1 ]; then
    $PY -m torch.distributed.run --standalone --local-addr 127.0.0.1 --nproc-per-node "$n" "$@"
  else
    $PY "$@"
  fi
}
cmd=${1:-help}; shift || true
case "$cmd" in
  data)     $PY scripts/data_pipeline.py --input "$1" --output "$2/mixed" && \
            $PY scripts/prepare_data.py --input "$2/mixed/mixed.jsonl" --output "$2/bin" "${@:3}" ;;
  train)    cfg=$1; n=${2:-1}; launch "$n" scripts/train.py --config "$cfg" --bf16 "${@:3}" ;;
  train4d)  cfg=$1; n=$2; launch "$n" scripts/train_distributed.py --config "$cfg" --bf16 "${@:3}" ;;
  grpo)     $PY scripts/train_grpo.py --config "$1" --checkpoint "$2" --bf16 "${@:3}" ;;
  generate) cfg=$1; shift; ck=${1:-}; [ -n "$ck" ] && shift; \
            $PY scripts/generate.py --config "$cfg" ${ck:+--checkpoint "$ck"} --device cuda --bf16 "$@" ;;
  eval)     cfg=$1; shift; ck=${1:-}; [ -n "$ck" ] && shift; \
            $PY scripts/evaluate.py --config "$cfg" ${ck:+--checkpoint "$ck"} --device cuda "$@" ;;
  bench)    n=${1:-1}; if [ "$n" -gt 1 ]; then
              $PY -m torch.distributed.run --nnodes=1 --nproc-per-node "$n" --master-addr 127.0.0.1 \
                  --master-port 29500 bench.py --gpus "$n"; else $PY bench.py; fi ;;
  test)     $PY scripts/test_all.py ;;
  *)        sed -n '2,11p' "$0" ;;
esac
