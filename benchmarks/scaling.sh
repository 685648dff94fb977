#!/bin/sh
# Training throughput scaling, two parts.
#
# 1. Host ranks (CPU, fp32 model of the reference's benchmarks/scaling.sh: 8
#    sequences of 64 tokens per rank per step), through the launcher: single,
#    DDP with and without overlap, ZeRO-1, plus the convergence comparison of
#    4-rank DDP against the identical global batch in one process.
# 2. GPUs (when GPUS is set, e.g. GPUS="1 2 4 8"): bench.py at each GPU count, one
#    rank per GPU under torchrun, this framework and then the reference's torch
#    arm, device-timed.  Every run appends one JSON line to $OUT/bench.jsonl.
#
# Writes JSONL logs to $OUT; benchmarks/report.py renders them.
set -e
OUT=${OUT:-benchmarks/results/$(date +%F)}
STEPS=${STEPS:-30}
mkdir -p "$OUT"
export OMP_NUM_THREADS=1 OPENBLAS_NUM_THREADS=1
M="--dim 128 --heads 4 --layers 4 --ctx 64 --batch 8 --lr 1e-3 --warmup 10 --dtype float32 --device cpu"
L() { rm -f "$OUT/$1.jsonl"; echo "$OUT/$1.jsonl"; }
python3 -m dtrain_b200.train --mode single --steps "$STEPS" $M --log "$(L tp_single_w1)"
for W in 2 4; do
  python3 -m dtrain_b200.launch --nproc $W -- python3 -m dtrain_b200.train --mode ddp --steps "$STEPS" $M --log "$(L tp_ddp_w$W)"
  python3 -m dtrain_b200.launch --nproc $W -- python3 -m dtrain_b200.train --mode ddp --no-overlap --steps "$STEPS" $M --log "$(L tp_ddp_nooverlap_w$W)"
  python3 -m dtrain_b200.launch --nproc $W -- python3 -m dtrain_b200.train --mode zero --steps "$STEPS" $M --log "$(L tp_zero_w$W)"
done
CSTEPS=${CSTEPS:-300}
python3 -m dtrain_b200.launch --nproc 4 -- python3 -m dtrain_b200.train --mode ddp --steps "$CSTEPS" $M --log "$(L conv_ddp_w4)"
python3 -m dtrain_b200.train --mode single --emulate-world 4 --steps "$CSTEPS" $M --log "$(L conv_single_emul4)"

if [ -n "${GPUS:-}" ]; then
  CONFIG=${CONFIG:-gpt2-small-ddp}
  for N in $GPUS; do
    for IMPL in reference ours; do
      if [ "$N" = 1 ]; then
        python3 bench.py --gpus 1 --impl $IMPL --config "$CONFIG" >> "$OUT/bench.jsonl"
      else
        timeout -k 60 900 python3 -m torch.distributed.run --nnodes=1 --nproc-per-node "$N" \
          --master-addr 127.0.0.1 --master-port $((29600 + N)) \
          bench.py --gpus "$N" --impl $IMPL --config "$CONFIG" >> "$OUT/bench.jsonl"
      fi
    done
  done
fi
