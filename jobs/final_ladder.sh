#!/usr/bin/env bash
# One size of the final scaling ladder on one 8-GPU node:  jobs/final_ladder.sh <d10|d11|d12|d13|d14|d16|d18> [main.py args]
# Same interface as the reference's jobs/final_ladder.sh: the size's width/layers/steps/learning rates come from
# nano_gpic_b200/config/ladder.py (one table for the scripts and the library), warmup = S/100,
# cooldown = floor(S/2/32)*32, accumulation = 1024 / GPUS / micro-batch, zero mode (sharded optimizer) from d14.
# GPIC_DATA: the data root (train/, val/, train_emb_qwen3_1.7b/); GPIC_SYNTHETIC=1 trains on synthetic batches.
set -eo pipefail
SIZE=${1:?usage: final_ladder.sh <size> [main.py arguments...]}; shift
HERE=$(cd "$(dirname "$(readlink -f "$0")")/.." && pwd)
source $HERE/jobs/env.sh
GPUS=${GPUS:-8}
eval "$(cd $HERE && python -m nano_gpic_b200.config.ladder --shell $SIZE $GPUS)" || { echo "unknown size $SIZE"; exit 2; }
DATA=${GPIC_DATA:-$GPIC_WC/data/gpic}
if [ "${GPIC_SYNTHETIC:-0}" != 1 ]; then
  for d in train val train_emb_qwen3_1.7b; do [ -d "$DATA/$d" ] || { echo "missing $DATA/$d (or set GPIC_SYNTHETIC=1)"; exit 2; }; done
fi
export GPIC_MFU_NO_EMA=${GPIC_MFU_NO_EMA:-1}   # the ladder keeps no EMA: checkpoints mirror the raw weights
export LADDER_RUN_ROOT=${GPIC_OUT:-$GPIC_WC/runs/final_ladder}/$SIZE LADDER_LAST_EVERY=$((S / 8))
mkdir -p $LADDER_RUN_ROOT/exp_ladder_d$D
[ -s $LADDER_RUN_ROOT/exp_ladder_d$D/shard_seed.txt ] || echo 20261106 > $LADDER_RUN_ROOT/exp_ladder_d$D/shard_seed.txt
STRAT=DDPStrategy; [ "$DP" = zero ] && STRAT=FSDPStrategy
exec bash $HERE/jobs/train_ladder.sh d$D $D $NB $NT $S \
  --config configs/muon_ladder.yaml \
  --trainer.strategy.class_path $STRAT \
  --model.optimizer.init_args.lr $ALR --model.optimizer.init_args.muon_lr $MLR \
  --model.optimizer.init_args.weight_decay 0 --model.optimizer.init_args.muon_weight_decay $WDK \
  --model.lr_scheduler.init_args.num_warmup_steps $WU --model.lr_scheduler.init_args.num_cooldown_steps $CD \
  --model.lr_scheduler.init_args.max_steps $S --model.lr_scheduler.init_args.min_lr 3e-5 \
  --data.train_batch_size $MB --trainer.accumulate_grad_batches $ACC \
  --data.train_dataset.init_args.shared_bucket true --data.train_dataset.init_args.tar_pattern "gpic_train_{00000..07999}.tar" \
  --data.train_dataset.init_args.tar_dir $DATA/train/ --data.train_dataset.init_args.emb_dir $DATA/train_emb_qwen3_1.7b \
  --model.conditioner.init_args.emb_dir $DATA/train_emb_qwen3_1.7b \
  "$@"
