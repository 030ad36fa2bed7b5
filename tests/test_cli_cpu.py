"""The command-line surface on CPU: YAML composition and overrides, the reference's own YAML files resolving to this
package, and BASELINE's CPU plumbing run (gloo, world size 2, tiny JiT-T2I, 64x64 images, 32 x 2048 captions,
global batch 8, Muon + AdamW) with checkpoint save and resume reproducible launch to launch."""
import os
import shutil
import socket

import pytest
import torch
import torch.multiprocessing as mp

from refpath import ref_root

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFGS = [os.path.join(HERE, "configs", f) for f in ("lite_ladder.yaml", "muon_ladder.yaml", "tiny_cpu.yaml")]


def test_compose_and_override():
    from nano_gpic_b200.config.cli import parse_args
    sub, cfg = parse_args(["fit", "--config", CFGS[0], "--config", CFGS[1], "--model.optimizer.init_args.muon_lr",
                           "6.8e-3", "--trainer.callbacks.0.init_args.every_n_train_steps=7", "--tags.exp", "d12"])
    assert sub == "fit"
    o = cfg["model"]["optimizer"]
    assert o["class_path"].endswith("MuonAdamW") and o["init_args"]["muon_lr"] == 6.8e-3
    assert "fused" not in o["init_args"]  # the AdamW node's arguments do not leak into the MuonAdamW node
    assert cfg["trainer"]["accumulate_grad_batches"] == 4
    assert cfg["trainer"]["callbacks"][0]["init_args"]["every_n_train_steps"] == 7
    from nano_gpic_b200.config.cli import run_dir
    assert run_dir(cfg).endswith("exp_d12")


def test_reference_yaml_resolves():
    """The reference's ladder YAML (its class paths) builds this package's objects."""
    root = ref_root()
    base = os.path.join(root, "baselines", "PixelGen", "configs_h100") if root else ""
    if not os.path.isdir(base):
        pytest.skip("reference configs not available")
    from nano_gpic_b200.config.cli import instantiate, parse_args, strategy_mode
    _, cfg = parse_args(["fit", "--config", os.path.join(base, "lite_ladder.yaml"), "--config",
                         os.path.join(base, "muon_ladder.yaml"), "--model.denoiser.init_args.hidden_size", "128",
                         "--model.denoiser.init_args.num_groups", "2", "--model.denoiser.init_args.num_blocks", "1",
                         "--model.denoiser.init_args.num_text_blocks", "1"])
    m = cfg["model"]
    from nano_gpic_b200.diffusion.flow_matching import JiTTrainer
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    from nano_gpic_b200.optim.muon import MuonAdamW
    den = instantiate(m["denoiser"])
    assert isinstance(den, JiT_T2I) and den.hidden_size == 128
    obj = instantiate(m["diffusion_trainer"])
    assert isinstance(obj, JiTTrainer) and obj.loss_weight_fn(1.0, 0.0) == 1.0
    opt = instantiate(m["optimizer"], params=list(den.parameters()))
    assert isinstance(opt, MuonAdamW)
    sched = instantiate(m["lr_scheduler"])(opt)
    assert sched is not None
    assert strategy_mode(cfg["trainer"]) == "ddp"
    cbs = [instantiate(c) for c in cfg["trainer"]["callbacks"]]
    assert [type(c).__name__ for c in cbs] == ["CheckpointHook", "CheckpointHook", "Warmup"]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _fit_worker(rank, world, port, argv):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), GPIC_MFU_ASYNC_CKPT="0")
    torch.set_num_threads(2)
    from nano_gpic_b200.config.cli import main
    assert main(argv) == 0


def _fit(tmp, extra, world=2):
    argv = ["fit"] + sum((["--config", c] for c in CFGS), []) + ["--trainer.default_root_dir", str(tmp)] + extra
    mp.spawn(_fit_worker, args=(world, _port(), argv), nprocs=world, join=True)


def _weights(path):
    sd = torch.load(path, map_location="cpu", weights_only=False)["state_dict"]
    return {k: v for k, v in sd.items() if k.startswith("denoiser.")}


def test_tiny_fit_checkpoint_resume(tmp_path):
    run = tmp_path / "run"
    _fit(run, ["--trainer.max_steps", "10", "--model.lr_scheduler.init_args.max_steps", "20"])
    exp = run / "exp_tiny"
    assert (exp / "ms-step=000010.ckpt").exists() and (exp / "last.ckpt").exists()
    ck = torch.load(exp / "last.ckpt", map_location="cpu", weights_only=False)
    assert ck["global_step"] == 10 and ck["optimizer_states"] and ck["lr_schedulers"]
    outs = []
    for i in range(2):  # two launches resumed from the same checkpoint draw the same numbers
        r = tmp_path / f"resume{i}"
        (r / "exp_tiny").mkdir(parents=True)
        shutil.copy(exp / "last.ckpt", r / "exp_tiny" / "last.ckpt")
        _fit(r, ["--trainer.max_steps", "14", "--model.lr_scheduler.init_args.max_steps", "20", "--ckpt_path", "last"])
        outs.append(_weights(r / "exp_tiny" / "ms-step=000014.ckpt"))
    for k in outs[0]:
        assert torch.equal(outs[0][k], outs[1][k]), k
    w10 = _weights(exp / "ms-step=000010.ckpt")
    assert any(not torch.equal(w10[k], outs[0][k]) for k in w10)  # the resumed launches trained
