#!/usr/bin/env bash
# jobs/eval_final_ladder.sh <size> [step]: score a ladder checkpoint (the reference's jobs/eval_final_ladder.sh):
# the fixed-noise held-out loss (16 noise levels), Euler-50 samples for the test prompts on every GPU (main.py predict,
# raw weights: the ladder's EMA slot mirrors them), then FD / PRDC / MMD of DINOv2 features against the reference
# statistics. Needs GPIC_DATA with gpic_test_50k.jsonl, reference_stats/test_stats.npz and the held-out cache.
set -eo pipefail
SIZE=${1:?usage: eval_final_ladder.sh <size> [step]}; STEP=${2:-}
HERE=$(cd "$(dirname "$(readlink -f "$0")")/.." && pwd)
source $HERE/jobs/env.sh
eval "$(cd $HERE && python -m nano_gpic_b200.config.ladder --shell $SIZE)"
DATA=${GPIC_DATA:-$GPIC_WC/data/gpic}
STEP=${STEP:-$S}
S6=$(printf %06d $((10#$STEP)))
CKPT=${GPIC_CKPT:-${GPIC_OUT:-$GPIC_WC/runs/final_ladder}/$SIZE/exp_ladder_d$D/ms-step=$S6.ckpt}
[ -f "$CKPT" ] || { echo "no checkpoint $CKPT"; exit 2; }
OUT=${GPIC_EVAL_OUT:-$(dirname $CKPT)/eval_${S6}_euler50}
mkdir -p $OUT
NGPU=${GPUS:-$(nvidia-smi -L 2>/dev/null | wc -l)}; [ "$NGPU" -ge 1 ] || NGPU=1
cd $HERE
python -m nano_gpic_b200.tools.heldout_loss work --ckpt "$CKPT" --data $DATA/heldout --out $OUT/heldout.jsonl \
  > $OUT/heldout.log 2>&1 || { echo "held-out loss failed (see $OUT/heldout.log)"; exit 3; }
torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node $NGPU main.py predict \
  --config configs/lite_ladder.yaml --config configs/lite_ladder_sample.yaml \
  --trainer.default_root_dir $OUT/pred --ckpt_path $CKPT \
  --model.denoiser.init_args.hidden_size $D --model.denoiser.init_args.num_groups $((D / 64)) \
  --model.denoiser.init_args.num_blocks $NB --model.denoiser.init_args.num_text_blocks $NT \
  --data.pred_dataset.init_args.jsonl_path $DATA/gpic_test_50k.jsonl > $OUT/predict.log 2>&1 \
  || { echo "predict failed (see $OUT/predict.log)"; exit 4; }
NPZ=$(find $OUT/pred -name "output.npz" | head -1)
[ -n "$NPZ" ] || { echo "no samples (see $OUT/predict.log)"; exit 4; }
torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node $NGPU -m nano_gpic_b200.tools.fast_eval "$NPZ" \
  $DATA/reference_stats/test_stats.npz $OUT/metrics.json > $OUT/eval.log 2>&1 \
  || { echo "scoring failed (see $OUT/eval.log)"; exit 5; }
cat $OUT/metrics.json
