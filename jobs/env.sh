# Environment shared by the job scripts. Sourced, not run.
export GPIC_WC=${GPIC_WC:-$PWD}
export NCCL_DEBUG=${NCCL_DEBUG:-WARN}
export OMP_NUM_THREADS=${OMP_NUM_THREADS:-8}
export PYTORCH_CUDA_ALLOC_CONF=${PYTORCH_CUDA_ALLOC_CONF:-expandable_segments:True}
export GPIC_PG_TIMEOUT_MIN=${GPIC_PG_TIMEOUT_MIN:-30}
export WANDB_MODE=${WANDB_MODE:-offline}   # W&B runs (when a WandbLogger node is configured) stay on this machine
