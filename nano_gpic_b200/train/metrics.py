"""Training metrics of `main.py fit`: what a log step records and where it goes.

Values (written only on log steps, so the other steps run without host synchronisation; the reference's
lightning_model_gpic.py:315-340 does the same): loss, lr, images/s and the per-caption-type losses
train/loss_{tag,short,medium,long}. A caption type's loss on one rank is the mean of its samples' losses in that
step (0 when the rank saw none), averaged over ranks, as the reference's sync_dist logging gives.

Sinks: rank 0 appends every log step to <run>/metrics.jsonl. When the trainer's logger node names a W&B logger
(class_path ending in WandbLogger, as the reference's configs_h100/lite_ladder.yaml:16-50) or GPIC_WANDB=1, the same
values also go to a W&B run in offline mode by default (WANDB_MODE decides; the reference's jobs/env.sh exports
offline), with the run's project and name from the node. Without the wandb package the JSONL file is the only sink and
a one-line note says so.
"""
import json
import os

import torch
import torch.distributed as dist

CAPTION_TYPES = ("tag", "short", "medium", "long")


def caption_type_losses(per_sample, types, group=None):
    """{"train/loss_<type>": value} from per-sample losses [N] (device) and their caption types (N strings): one
    device reduction per type, one all-reduce over ranks of the four per-rank means, one host read."""
    dev = per_sample.device
    means = []
    for ct in CAPTION_TYPES:
        idx = [i for i, t in enumerate(types) if t == ct]
        if idx:
            means.append(per_sample.float()[torch.tensor(idx, device=dev)].mean())
        else:
            means.append(torch.zeros((), device=dev))
    vals = torch.stack(means)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.SUM, group=group)
        vals = vals / dist.get_world_size(group)
    return {f"train/loss_{ct}": float(v) for ct, v in zip(CAPTION_TYPES, vals.tolist())}


class MetricSinks:
    """Rank 0's sinks for log-step values: metrics.jsonl always, a W&B run when asked for and available."""

    def __init__(self, run_dir, rank, logger_node=None, config=None):
        self.run_dir, self.rank = run_dir, rank
        self.wandb = None
        if rank != 0:
            return
        wanted = os.environ.get("GPIC_WANDB") == "1"
        args = {}
        if isinstance(logger_node, dict) and str(logger_node.get("class_path", "")).endswith("WandbLogger"):
            wanted = os.environ.get("GPIC_WANDB", "1") != "0"
            args = dict(logger_node.get("init_args") or {})
        if not wanted:
            return
        try:
            import wandb
        except ImportError:
            print("[metrics] a W&B logger is configured but the wandb package is not installed: metrics.jsonl only",
                  flush=True)
            return
        mode = os.environ.get("WANDB_MODE") or args.get("mode") or ("offline" if args.get("offline", True) else "online")
        self.wandb = wandb.init(project=args.get("project") or "gpic-speed", name=args.get("name"), dir=run_dir,
                                mode=mode, config=config, resume=args.get("resume"), id=args.get("id"))

    def log(self, values, step):
        if self.rank != 0:
            return
        with open(os.path.join(self.run_dir, "metrics.jsonl"), "a") as f:
            f.write(json.dumps({"step": step, **values}) + "\n")
        if self.wandb is not None:
            self.wandb.log(dict(values), step=step)

    def close(self):
        if self.wandb is not None:
            self.wandb.finish()
            self.wandb = None
