"""The Euler sampler against the reference's EulerSamplerJiT (baselines/PixelGen/src/diffusion/flow_matching/
sampling.py:114-201) on the same network, noise and conditions (CFG 1, and CFG != 1 with a guidance interval), and a
tiny `main.py predict` on CPU (YAML composition, checkpoint EMA weights, JSONL prompts, images written)."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from refpath import reference_imports

from nano_gpic_b200.diffusion.sampling import EulerSamplerJiT, fp2uint8, simple_guidance_fn
from nano_gpic_b200.models.conditioner import BaseConditioner

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _toy_net():
    """A smooth x-prediction net of (x, t, condition): the samplers only call it."""
    g = torch.Generator().manual_seed(0)
    a = torch.randn(3, 3, generator=g) * 0.3

    def net(x, t, c):
        mix = torch.einsum("ij,bjhw->bihw", a, x)
        return torch.tanh(mix * (1 + t.view(-1, 1, 1, 1)) + c.mean(dim=(1, 2)).view(-1, 1, 1, 1))
    return net


@pytest.mark.parametrize("guidance,interval,shift", [(1.0, (0.0, 1.0), 1.0), (4.0, (0.1, 0.7), 1.0),
                                                     (2.5, (0.0, 1.0), 3.0)])
def test_euler_matches_the_reference(guidance, interval, shift):
    net = _toy_net()
    g = torch.Generator().manual_seed(1)
    noise = torch.randn(3, 3, 8, 8, generator=g)
    cond = torch.randn(3, 5, 16, generator=g)
    uncond = torch.zeros(3, 5, 16)
    ours = EulerSamplerJiT(num_steps=12, guidance=guidance, timeshift=shift, guidance_interval_min=interval[0],
                           guidance_interval_max=interval[1])
    x = ours(net, noise, cond, uncond)
    with reference_imports():
        from src.diffusion.base.guidance import simple_guidance_fn as ref_guidance
        from src.diffusion.flow_matching.sampling import EulerSamplerJiT as RefEuler
        from src.diffusion.flow_matching.scheduling import LinearScheduler
        ref = RefEuler(scheduler=LinearScheduler(), guidance_fn=ref_guidance, num_steps=12, guidance=guidance,
                       timeshift=shift, guidance_interval_min=interval[0], guidance_interval_max=interval[1])
        x_ref = ref(net, noise, cond, uncond)
        assert torch.equal(ours.timesteps, ref.timesteps)
    torch.testing.assert_close(x, x_ref, rtol=1e-6, atol=1e-6)
    # CFG 1 never evaluates the unconditional half; the guided mix is uncond + cfg (cond - uncond)
    a, b = torch.ones(2, 1), torch.full((2, 1), 3.0)
    assert torch.equal(simple_guidance_fn(torch.cat([a, b]), 2.0), a + 2.0 * (b - a))


def test_fp2uint8():
    x = torch.tensor([-1.0, -0.999, 0.0, 0.5, 1.0, 1.5])
    assert fp2uint8(x).tolist() == [0, 0, 128, 191, 255, 255]


class CharConditioner(BaseConditioner):
    """A deterministic stand-in for the text encoder (no model weights offline): caption character codes spread over
    embed_dim features, one token per character, left-aligned mask."""

    def __init__(self, embed_dim=2048, max_length=32, **unused):
        super().__init__()
        self.embed_dim, self.max_length = embed_dim, max_length

    def _impl_condition(self, y, metadata):
        T = min(self.max_length, max(len(c) for c in y))
        out = torch.zeros(len(y), T, self.embed_dim)
        mask = torch.zeros(len(y), T, dtype=torch.bool)
        for i, c in enumerate(y):
            for j, ch in enumerate(c[:T]):
                g = torch.Generator().manual_seed(ord(ch))
                out[i, j] = torch.randn(self.embed_dim, generator=g)
                mask[i, j] = True
        metadata["y_mask"] = mask
        return out.bfloat16()

    def _impl_uncondition(self, y, metadata):
        T = metadata["y_mask"].shape[1]
        return torch.zeros(len(y), T, self.embed_dim).bfloat16()


def test_main_predict_on_cpu(tmp_path):
    """main.py predict: the EMA weights of an ms checkpoint, Euler sampling over JSONL prompts, images in output.npz
    equal to sampling the same network directly."""
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    kw = dict(input_size=64, in_channels=3, num_groups=2, hidden_size=128, num_blocks=2, num_text_blocks=1,
              patch_size=16, txt_embed_dim=2048, txt_max_length=32, bottleneck_dim=16)
    torch.manual_seed(3)
    net = JiT_T2I(**kw).eval()
    with torch.no_grad():
        for p in net.parameters():
            p.add_(0.03 * torch.randn_like(p))
    sd = {"ema_denoiser." + k: v for k, v in net.state_dict().items()}
    sd.update({"denoiser." + k: torch.zeros_like(v) for k, v in net.state_dict().items()})  # must not be used
    ckpt = tmp_path / "ms-step=000010.ckpt"
    torch.save({"state_dict": sd, "global_step": 10}, ckpt)
    prompts = tmp_path / "prompts.jsonl"
    recs = [{"key": "a1", "caption": "a red cube", "caption_type": "short"},
            {"key": "b2", "caption": "two birds on a wire at dusk", "caption_type": "medium"}]
    prompts.write_text("".join(json.dumps(r) + "\n" for r in recs))
    cfg = tmp_path / "predict.yaml"
    cfg.write_text(f"""
model:
  denoiser:
    init_args: {json.dumps(kw)}
  conditioner:
    class_path: test_sampling_cpu.CharConditioner
    init_args: {{embed_dim: 2048, max_length: 32}}
  diffusion_sampler:
    class_path: nano_gpic_b200.diffusion.sampling.EulerSamplerJiT
    init_args: {{num_steps: 4, guidance: 1.0, timeshift: 1.0}}
  eval_original_model: false
data:
  pred_dataset:
    class_path: nano_gpic_b200.data.gpic.GPICJsonlDataset
    init_args: {{jsonl_path: {prompts}, num_samples_per_instance: 1, latent_shape: [3, 64, 64]}}
  pred_batch_size: 2
trainer:
  default_root_dir: {tmp_path / "runs"}
tags:
  exp: pred
""")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONPATH=os.pathsep.join([HERE, os.path.join(HERE, "tests")]),
               GPIC_PRED_DIR="samples")
    r = subprocess.run([sys.executable, os.path.join(HERE, "main.py"), "predict", "--config",
                        os.path.join(HERE, "configs", "lite_ladder.yaml"), "--config", str(cfg), "--ckpt_path",
                        str(ckpt)], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    out = list((tmp_path / "runs").rglob("samples/output.npz"))
    assert len(out) == 1, list((tmp_path / "runs").rglob("*"))
    imgs = np.load(out[0])["arr_0"]
    assert imgs.shape == (2, 64, 64, 3) and imgs.dtype == np.uint8
    # the same samples directly
    cond = CharConditioner()
    meta = {}
    y = cond._impl_condition([r_["caption"] for r_ in recs], meta)
    noise = torch.stack([torch.randn(3, 64, 64, generator=torch.Generator().manual_seed(0)) for _ in recs])
    sampler = EulerSamplerJiT(num_steps=4)
    x = sampler(lambda xx, t, yy: net(xx, t, yy, y_mask=meta["y_mask"]), noise, y)
    want = fp2uint8(x).permute(0, 2, 3, 1).numpy()
    assert np.abs(imgs.astype(int) - want.astype(int)).max() <= 1
