"""Checkpoints: the reference's layout (its own loader reads ours strictly), save/resume continuity, the async writer
with EMA twins, the save policy, and SaveOnTerm's cross-rank agreement (gloo, 2 ranks)."""
import importlib.util
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from refpath import ref_root, reference_imports
from test_train_cpu import _batch, _trainer

TINY = dict(input_size=64, in_channels=3, num_groups=2, hidden_size=128, num_blocks=2, num_text_blocks=1,
            patch_size=16, txt_embed_dim=32, txt_max_length=32, bottleneck_dim=16)


def test_reference_loader_reads_our_ms_checkpoint(tmp_path):
    from nano_gpic_b200.train.checkpoint import build_checkpoint, save_sync
    tr = _trainer()
    tr.global_step = 7
    path = tmp_path / "ms-step=000007.ckpt"
    save_sync(build_checkpoint(tr, full=False), str(path))
    ck = torch.load(path, map_location="cpu", weights_only=False)
    assert ck["global_step"] == 7 and "optimizer_states" not in ck
    with reference_imports():
        spec = importlib.util.spec_from_file_location("ref_heldout", os.path.join(ref_root(), "tools", "heldout_loss.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        for prefix in ("denoiser.", "ema_denoiser."):
            net = mod.build_denoiser(TINY, ck["state_dict"], prefix, "cpu")  # strict load on the meta device
            ours = tr.model.state_dict()
            for k, v in net.state_dict().items():
                assert torch.equal(v, ours[k].float()), k
        assert mod.twin_weights(ck["state_dict"])  # no-EMA checkpoint: the EMA slot holds the raw weights


def test_resume_continues_bit_for_bit(tmp_path):
    from nano_gpic_b200.train.checkpoint import build_checkpoint, load_into, save_sync
    img, cap, mask = _batch()
    t = torch.full((4,), 0.3)
    noise = torch.randn(4, 3, 64, 64, generator=torch.Generator().manual_seed(5))
    a = _trainer()
    for _ in range(2):
        a.train_step(img, cap, mask, t=t, noise=noise)
    save_sync(build_checkpoint(a, full=True), str(tmp_path / "last.ckpt"))
    for _ in range(2):
        a.train_step(img, cap, mask, t=t, noise=noise)
    b = _trainer()
    load_into(b, torch.load(tmp_path / "last.ckpt", map_location="cpu", weights_only=False))
    assert b.global_step == 2
    for _ in range(2):
        b.train_step(img, cap, mask, t=t, noise=noise)
    assert torch.equal(a.flat.data, b.flat.data)
    assert a.opt.param_groups[0]["lr"] == b.opt.param_groups[0]["lr"]


def test_async_writer_and_twins(tmp_path):
    from nano_gpic_b200.train.checkpoint import AsyncWriter, build_checkpoint
    tr = _trainer()
    w = AsyncWriter()
    try:
        paths = [str(tmp_path / f"ms-step={i:06d}.ckpt") for i in (1, 2, 3)]
        for p in paths:  # three saves with two buffers: the third waits for a free one
            w.save(build_checkpoint(tr, full=True), p)
        w.wait()
    finally:
        w.close()
    for p in paths:
        ck = torch.load(p, map_location="cpu", weights_only=False)
        sd = ck["state_dict"]
        k = "blocks.0.attn.qkv_x.weight"
        assert torch.equal(sd["denoiser." + k], tr.model.state_dict()[k])
        # twins: one storage in the file
        assert sd["denoiser." + k].untyped_storage().data_ptr() == sd["ema_denoiser." + k].untyped_storage().data_ptr()
    assert not [f for f in os.listdir(tmp_path) if ".part-" in f]


def test_policy_names_and_resume_skip(tmp_path):
    from nano_gpic_b200.train.checkpoint import CheckpointPolicy
    pol = CheckpointPolicy(str(tmp_path), ms_every=4, last_every=2, max_steps=10)
    pol.on_start(4)
    assert pol.due(4) == []            # never at the step a launch resumed from
    assert pol.due(6) == [("last.ckpt", True)]
    assert pol.due(8) == [("ms-step=000008.ckpt", False), ("last.ckpt", True)]
    assert pol.due(10) == [("ms-step=000010.ckpt", False), ("last.ckpt", True)]


def _term_rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from nano_gpic_b200.train.checkpoint import SaveOnTerm
    sot = SaveOnTerm(every=5, install=False)
    stop = None
    for step in range(1, 31):
        if rank == 1 and step == 7:
            sot._handler(15, None)     # the TERM reaches one rank only
        if sot.check(step):
            stop = step
            break
    out[rank] = stop
    dist.destroy_process_group()


def test_save_on_term_agreement():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = mp.Manager().dict()
    mp.start_processes(_term_rank, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    assert out[0] == out[1] == 10


def test_partial_files_of_dead_writers_are_removed(tmp_path):
    """A partial checkpoint whose writer process is gone is removed; one of a live process is kept."""
    from nano_gpic_b200.train.checkpoint import clean_tmp
    import subprocess
    p = subprocess.Popen(["true"])
    p.wait()  # a pid that no longer exists
    dead = tmp_path / f"last.ckpt.part-{p.pid}"
    live = tmp_path / f"ms-step=000004.ckpt.part-{os.getpid()}"
    dead.write_bytes(b"x")
    live.write_bytes(b"y")
    assert clean_tmp(str(tmp_path)) == 1
    assert not dead.exists() and live.exists()
