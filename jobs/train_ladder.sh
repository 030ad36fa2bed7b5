#!/usr/bin/env bash
# jobs/train_ladder.sh SIZE D NB NT STEPS [main.py args...]: one training launch on this node (the reference's
# jobs/train_ladder.sh interface). Records the launch, runs the GPU-health gate in the background (main.py waits for
# its verdict and exits 98 on a failure), resumes from the newest last*.ckpt of the run directory with the same shard
# seed, builds the callback list (ms-step every STEPS/4, last.ckpt every LADDER_LAST_EVERY, warm-up, host tuning,
# shard clock, save-on-term, None refcount, first-step marker), launches one process per GPU with torchrun under the
# launch guard (watchdog, retries, leftover cleanup) and checks that ms-step=<STEPS>.ckpt exists at the end (exit 99
# otherwise).
set -o pipefail
HERE=$(cd "$(dirname "$(readlink -f "$0")")/.." && pwd)
source $HERE/jobs/env.sh
SIZE=$1 D=$2 NB=$3 NT=$4 STEPS=$5; shift 5
ROOT=${LADDER_RUN_ROOT:-$GPIC_WC/runs/gpic-speed}
RUN=$ROOT/exp_ladder_$SIZE
if [ $((STEPS % 32)) -ne 0 ] || [ $((D % 64)) -ne 0 ]; then echo "max_steps must be a multiple of 32 and d of 64"; exit 2; fi
MS=$((STEPS / 4)); LAST=${LADDER_LAST_EVERY:-$((STEPS / 32))}
mkdir -p $RUN
echo "$(date -u +%FT%TZ) $(git -C $HERE rev-parse HEAD 2>/dev/null) size=$SIZE d=$D nb=$NB nt=$NT max_steps=$STEPS ms_every=$MS last_every=$LAST host=$(hostname)" >> $RUN/launches.txt
export GPIC_HEALTH_FILE=$RUN/gpu_health_$(date +%s).verdict
if [ "${GPIC_SKIP_HEALTH:-0}" != 1 ]; then
  ( cd $HERE && python -m nano_gpic_b200.tools.gpu_health --verdict $GPIC_HEALTH_FILE > $RUN/gpu_health.log 2>&1 ) &
else
  echo "OK skipped" > $GPIC_HEALTH_FILE
fi
CKPT_ARGS=()
LASTCK=$(ls -t $RUN/last*.ckpt 2>/dev/null | head -1)
if [ -n "$LASTCK" ]; then CKPT_ARGS=(--ckpt_path "$LASTCK"); echo "resuming from $LASTCK"; fi
SEEDF=$RUN/shard_seed.txt
if [ -n "$LASTCK" ]; then
  read -r KEEP_T CK_SEED CK_STEP < <(cd $HERE && python -m nano_gpic_b200.tools.ckpt_shard_clock "$LASTCK") || { echo "cannot read the shard clock of $LASTCK"; exit 2; }
  if [ "$CK_SEED" != - ]; then
    [ -s $SEEDF ] || echo "$CK_SEED" > $SEEDF
    [ "$(cat $SEEDF)" = "$CK_SEED" ] || { echo "$SEEDF ($(cat $SEEDF)) differs from the seed in $LASTCK ($CK_SEED)"; exit 2; }
  fi
  for f in $RUN/shards_started_rank*.txt; do   # shards started after the checkpoint are read again
    [ -f "$f" ] || continue
    awk -v T=$KEEP_T '$1 <= T' "$f" > "$f.tmp" && mv "$f.tmp" "$f"
  done
fi
[ -s $SEEDF ] || date +%s > $SEEDF
export GPIC_SHARD_SEED=$(cat $SEEDF) GPIC_SHARD_LOG_DIR=$RUN
CB='[{"class_path":"nano_gpic_b200.train.callbacks.CheckpointHook","init_args":{"filename":"ms-{step:06d}","save_last":false,"save_top_k":-1,"every_n_train_steps":'$MS'}},{"class_path":"nano_gpic_b200.train.callbacks.CheckpointHook","init_args":{"filename":"resume-{step:06d}","save_last":true,"save_top_k":0,"every_n_train_steps":'$LAST'}},{"class_path":"nano_gpic_b200.train.callbacks.Warmup"},{"class_path":"nano_gpic_b200.train.callbacks.HostTuning"},{"class_path":"nano_gpic_b200.train.callbacks.ShardClock"},{"class_path":"nano_gpic_b200.train.callbacks.SaveOnTermCallback"},{"class_path":"nano_gpic_b200.train.callbacks.NoneRefcount","init_args":{"every":1000}},{"class_path":"nano_gpic_b200.train.callbacks.FirstStepMarker"}]'
NGPU=${GPUS:-$(nvidia-smi -L 2>/dev/null | wc -l)}; [ "$NGPU" -ge 1 ] || NGPU=1
cd $HERE
# the launch guard (nano_gpic_b200/train/launch_guard.py): first-step watchdog (GPIC_LAUNCH_START_TIMEOUT_S, 1500 s of
# no first step and no warm-up progress -> TERM, KILL, status 125), retries before the first step
# (GPIC_LAUNCH_RETRIES, 2), and no process of the launch left behind (GPIC_LAUNCH_ID)
timeout -k 60 ${GPIC_LAUNCH_TIMEOUT:-1000000} python -m nano_gpic_b200.train.launch_guard --run $RUN -- \
  torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node $NGPU main.py fit \
  --config configs/lite_ladder.yaml \
  --model.denoiser.init_args.hidden_size $D --model.denoiser.init_args.num_groups $((D / 64)) \
  --model.denoiser.init_args.num_blocks $NB --model.denoiser.init_args.num_text_blocks $NT \
  --trainer.max_steps $STEPS --trainer.default_root_dir $ROOT --tags.exp ladder_$SIZE \
  --trainer.callbacks "$CB" \
  "$@" "${CKPT_ARGS[@]}"
RC=$?
[ $RC -eq 0 ] || exit $RC
F=$(printf "%s/ms-step=%06d.ckpt" $RUN $STEPS)
[ -f "$F" ] || { echo "missing $F at the end of the run"; exit 99; }
