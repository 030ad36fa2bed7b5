"""The command-line surface: LightningCLI-compatible YAML composition and dotted overrides, without Lightning.

    python main.py fit --config configs/lite_ladder.yaml --config configs/muon_ladder.yaml \
        --model.denoiser.init_args.hidden_size 1024 --trainer.max_steps 40192 --ckpt_path last.ckpt

* `--config a.yaml --config b.yaml`: deep-merged left to right (mappings merge, lists and scalars replace), as
  jsonargparse composes them (reference jobs/train_ladder.sh:263-268, baselines/PixelGen/main.py).
* `--a.b.c VALUE` and `--a.b.c=VALUE`: set one key; VALUE is parsed as YAML (numbers, true/false, null, lists).
* `class_path` + `init_args` nodes build objects. The reference's class paths (`src.models...`,
  `lightning.pytorch.strategies.DDPStrategy`, ...) resolve through ALIASES to this package, so the reference's YAML
  files load unchanged; Lightning-only nodes (loggers, plugins, strategies) become plain settings.
* The resolved configuration is written to `<run_dir>/config-<stage>-<stamp>.yaml` (reference main.py:19-25), where
  run_dir = <trainer.default_root_dir>/exp_<tags.exp> (the reference's ReWriteRootDirCli).
"""
import copy
import importlib
import os
import sys
import time

import yaml

# reference class / function path -> this package's
ALIASES = {
    "src.models.transformer.JiT_T2I.JiT_T2I": "nano_gpic_b200.models.jit_t2i.JiT_T2I",
    "src.models.autoencoder.pixel.PixelAE": "nano_gpic_b200.models.autoencoder.PixelAE",
    "src.models.conditioner.cached_text.CachedTextConditioner":
        "nano_gpic_b200.models.conditioner.CachedTextConditioner",
    "src.models.conditioner.qwen3_text_encoder.Qwen3TextEncoder": "nano_gpic_b200.models.conditioner.Qwen3TextEncoder",
    "src.diffusion.flow_matching.training_JiT.JiTTrainer": "nano_gpic_b200.diffusion.flow_matching.JiTTrainer",
    "src.diffusion.flow_matching.training_JiT.constant": "nano_gpic_b200.diffusion.flow_matching.constant",
    "src.diffusion.flow_matching.scheduling.LinearScheduler": "nano_gpic_b200.diffusion.flow_matching.LinearScheduler",
    "src.diffusion.flow_matching.sampling.EulerSamplerJiT": "nano_gpic_b200.diffusion.sampling.EulerSamplerJiT",
    "src.diffusion.flow_matching.sampling.ode_step_fn": "nano_gpic_b200.diffusion.sampling.ode_step_fn",
    "src.diffusion.base.guidance.simple_guidance_fn": "nano_gpic_b200.diffusion.sampling.simple_guidance_fn",
    "src.callbacks.simple_ema.SimpleEMA": "nano_gpic_b200.train.callbacks.EMASpec",
    "src.optim.muon.MuonAdamW": "nano_gpic_b200.optim.muon.MuonAdamW",
    "src.utils.lr_scheduler.WarmupFlatCooldown": "nano_gpic_b200.optim.lr_scheduler.WarmupFlatCooldown",
    "src.utils.lr_scheduler.ConstantWithWarmup": "nano_gpic_b200.optim.lr_scheduler.ConstantWithWarmup",
    "src.data.dataset.gpic_dataset.GPICWebDataset": "nano_gpic_b200.data.gpic.GPICWebDataset",
    "src.data.dataset.gpic_jsonl_dataset.GPICJsonlDataset": "nano_gpic_b200.data.gpic.GPICJsonlDataset",
    "src.callbacks.model_checkpoint.CheckpointHook": "nano_gpic_b200.train.callbacks.CheckpointHook",
    "src.callbacks.compile_warmup.CompileWarmup": "nano_gpic_b200.train.callbacks.Warmup",
    "src.callbacks.save_on_term.SaveOnTerm": "nano_gpic_b200.train.callbacks.SaveOnTermCallback",
    "src.callbacks.shard_clock.ShardClock": "nano_gpic_b200.train.callbacks.ShardClock",
    "src.callbacks.host_tuning.HostTuning": "nano_gpic_b200.train.callbacks.HostTuning",
    "src.callbacks.first_step.FirstStepMarker": "nano_gpic_b200.train.callbacks.FirstStepMarker",
    "src.callbacks.bench.BenchTimer": "nano_gpic_b200.train.callbacks.BenchTimer",
    "src.callbacks.launch_fingerprint.LaunchFingerprint": "nano_gpic_b200.train.callbacks.LaunchFingerprint",
    "src.callbacks.none_refcount.NoneRefcount": "nano_gpic_b200.train.callbacks.NoneRefcount",
    "src.callbacks.grad.GradientMonitor": "nano_gpic_b200.train.callbacks.GradientMonitor",
    "src.callbacks.save_images.SaveImagesHook": "nano_gpic_b200.train.callbacks.SaveImagesHook",
}
# Lightning strategies -> data-parallel mode of this package
STRATEGIES = {"DDPStrategy": "ddp", "ddp": "ddp", "FSDPStrategy": "zero", "ModelParallelStrategy": "zero",
              "fsdp": "zero", "zero": "zero", "auto": "ddp", "SingleDeviceStrategy": "ddp"}


# ------------------------------------------------------------------------------------------------ composition
def deep_merge(a, b):
    """b over a: mappings merge recursively, everything else is replaced. A class_path node whose class changes is
    replaced as a whole (the old class's init_args do not carry over to the new one)."""
    if is_spec(a) and is_spec(b) and a["class_path"] != b["class_path"]:
        return copy.deepcopy(b)
    if isinstance(a, dict) and isinstance(b, dict):
        out = dict(a)
        for k, v in b.items():
            out[k] = deep_merge(a[k], v) if k in a else copy.deepcopy(v)
        return out
    return copy.deepcopy(b)


def set_dotted(cfg, key, value):
    """cfg[a][b][c] = value for key "a.b.c"; intermediate mappings are created. A list index may appear
    ("trainer.callbacks.0.init_args.every_n_train_steps")."""
    parts = key.split(".")
    node = cfg
    for i, p in enumerate(parts[:-1]):
        nxt = parts[i + 1]
        if isinstance(node, list):
            node = node[int(p)]
            continue
        if p not in node or node[p] is None:
            node[p] = [] if nxt.isdigit() else {}
        node = node[p]
    last = parts[-1]
    if isinstance(node, list):
        node[int(last)] = value
    else:
        node[last] = value


def get_dotted(cfg, key, default=None):
    node = cfg
    for p in key.split("."):
        if isinstance(node, list) and p.isdigit() and int(p) < len(node):
            node = node[int(p)]
        elif isinstance(node, dict) and p in node:
            node = node[p]
        else:
            return default
    return node


def parse_value(text):
    try:
        return yaml.safe_load(text)
    except yaml.YAMLError:
        return text


def parse_args(argv):
    """argv (without the program) -> (subcommand, config dict). The first non-option word is the subcommand."""
    argv = list(argv)
    sub = None
    if argv and not argv[0].startswith("-"):
        sub = argv.pop(0)
    cfg, overrides = {}, []
    i = 0
    while i < len(argv):
        a = argv[i]
        if not a.startswith("--"):
            raise SystemExit(f"unexpected argument {a!r}")
        key, eq, val = a[2:].partition("=")
        if not eq:
            if i + 1 >= len(argv) or (argv[i + 1].startswith("--") and not _is_number(argv[i + 1])):
                val = "true"  # a bare flag
            else:
                i += 1
                val = argv[i]
        if key == "config":
            with open(val) as f:
                cfg = deep_merge(cfg, yaml.safe_load(f) or {})
        elif key == "print_config":
            overrides.append(("__print__", True))
        else:
            overrides.append((key, parse_value(val)))
        i += 1
    show = False
    for k, v in overrides:
        if k == "__print__":
            show = True
        else:
            set_dotted(cfg, k, v)
    if show:
        cfg["__print__"] = True
    return sub, cfg


def _is_number(s):
    try:
        float(s)
        return True
    except ValueError:
        return False


# ----------------------------------------------------------------------------------------------- instantiation
def resolve(path):
    """A dotted path to a class or function, through ALIASES."""
    path = ALIASES.get(path, path)
    mod, _, name = path.rpartition(".")
    return getattr(importlib.import_module(mod), name)


def is_spec(node):
    return isinstance(node, dict) and "class_path" in node


def instantiate(node, **extra):
    """Build the object of a class_path/init_args node (init_args instantiated recursively; strings naming an
    aliased callable become the callable). extra keyword arguments are added (e.g. params of an optimizer)."""
    if not is_spec(node):
        return node
    cls = resolve(node["class_path"])
    kwargs = {k: _build(v) for k, v in (node.get("init_args") or {}).items()}
    kwargs.update(extra)
    return cls(**kwargs)


def _build(v):
    if is_spec(v):
        return instantiate(v)
    if isinstance(v, str) and v in ALIASES:
        return resolve(v)
    if isinstance(v, list):
        return [_build(x) for x in v]
    return v


def strategy_mode(trainer_cfg):
    s = (trainer_cfg or {}).get("strategy", "ddp")
    name = s["class_path"].rsplit(".", 1)[-1] if is_spec(s) else str(s)
    return STRATEGIES.get(name, "ddp")


# -------------------------------------------------------------------------------------------------- run dir
def run_dir(cfg):
    root = get_dotted(cfg, "trainer.default_root_dir") or "."
    tag = get_dotted(cfg, "tags.exp")
    return os.path.join(root, f"exp_{tag}") if tag else root


def write_config(cfg, directory, stage="TrainerFn.FITTING"):
    os.makedirs(directory, exist_ok=True)
    stamp = time.strftime("%Y%m%d-%H%M%S")
    path = os.path.join(directory, f"config-{stage}-{stamp}.yaml")
    with open(path, "w") as f:
        yaml.safe_dump({k: v for k, v in cfg.items() if not k.startswith("__")}, f, sort_keys=False)
    return path


def main(argv=None):
    sub, cfg = parse_args(sys.argv[1:] if argv is None else argv)
    if cfg.pop("__print__", False):
        print(yaml.safe_dump(cfg, sort_keys=False))
        return 0
    if sub == "fit":
        from ..train.fit import fit
        return fit(cfg)
    if sub == "predict":
        from ..train.fit import predict
        return predict(cfg)
    raise SystemExit("usage: main.py {fit,predict} --config FILE [--config FILE ...] [--a.b.c VALUE ...]")
