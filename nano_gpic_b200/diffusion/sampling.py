"""Euler ODE sampler for the x-prediction flow model, with classifier-free guidance.

Reference EulerSamplerJiT (baselines/PixelGen/src/diffusion/flow_matching/sampling.py:114-201), guidance
(src/diffusion/base/guidance.py:3-6):
    t_k = time_shift(linspace(0, 1 - last_step, N) ++ [1])        (last_step = 1 / N by default)
    v   = (net(x, t) - x) / max(1 - t, 0.05)                       (x-prediction turned into a velocity)
    x  <- x + v dt
From noise at t = 0 to the image at t = 1. With guidance != 1 the batch is [uncond ; cond] and
v = v_u + cfg (v_c - v_u) inside the guidance interval; guidance == 1 runs the conditional half only.
"""
import torch

from .flow_matching import LinearScheduler


def shift_respace_fn(t, shift=3.0):
    return t / (t + (1 - t) * shift)


def ode_step_fn(x, v, dt, s, w):
    return x + v * dt


def simple_guidance_fn(out, cfg):
    uncond, cond = out.chunk(2, dim=0)
    return uncond + cfg * (cond - uncond)


class EulerSamplerJiT:
    def __init__(self, scheduler=None, w_scheduler=None, num_steps=50, guidance=1.0, guidance_fn=simple_guidance_fn,
                 timeshift=1.0, guidance_interval_min=0.0, guidance_interval_max=1.0, step_fn=ode_step_fn,
                 last_step=None, last_step_fn=ode_step_fn, t_eps=5e-2):
        self.scheduler = scheduler or LinearScheduler()
        self.w_scheduler = w_scheduler
        self.num_steps, self.guidance, self.guidance_fn = num_steps, guidance, guidance_fn
        self.timeshift = timeshift
        self.guidance_interval_min, self.guidance_interval_max = guidance_interval_min, guidance_interval_max
        self.step_fn, self.last_step_fn = step_fn, last_step_fn
        self.last_step = 1.0 / num_steps if (last_step is None or num_steps == 1) else last_step
        ts = torch.linspace(0.0, 1 - self.last_step, num_steps)
        self.timesteps = shift_respace_fn(torch.cat([ts, torch.tensor([1.0])]), timeshift)
        self.t_eps = t_eps

    @torch.no_grad()
    def __call__(self, net, noise, condition, uncondition=None, return_trajectory=False):
        """net(x, t, cond) -> x-prediction. noise [B, C, H, W] at t = 0."""
        B = noise.shape[0]
        steps = self.timesteps.to(noise.device, noise.dtype)
        cfg_on = float(self.guidance) != 1.0
        cond2 = torch.cat([uncondition, condition], dim=0) if cfg_on else None
        x = noise
        traj = [x]
        for i, (t_cur, t_next) in enumerate(zip(steps[:-1], steps[1:])):
            dt = t_next - t_cur
            t = t_cur.repeat(B)
            if cfg_on:
                x2, t2 = torch.cat([x, x], 0), t.repeat(2)
                out = (net(x2, t2, cond2).float() - x2) / (1.0 - t2.view(-1, 1, 1, 1)).clamp_min(self.t_eps)
                g = self.guidance if self.guidance_interval_min < float(t_cur) <= self.guidance_interval_max else 1.0
                v = self.guidance_fn(out, g)
            else:
                v = (net(x, t, condition).float() - x) / (1.0 - t.view(-1, 1, 1, 1)).clamp_min(self.t_eps)
            w = self.w_scheduler.w(t) if self.w_scheduler is not None else 0.0
            step = self.step_fn if i < self.num_steps - 1 else self.last_step_fn
            x = step(x, v, dt, None, w)
            traj.append(x)
        return (x, traj) if return_trajectory else x


def fp2uint8(x):
    """[-1, 1] floats -> uint8 (reference src/models/autoencoder/base.py:5-11)."""
    return torch.clip_((x + 1) * 127.5 + 0.5, 0, 255).to(torch.uint8)
