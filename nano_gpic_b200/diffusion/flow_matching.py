"""Flow-matching objective with x-prediction and the loss in v-space (JiT), and its linear schedule.

Reference: JiTTrainer (baselines/PixelGen/src/diffusion/flow_matching/training_JiT.py:14-64), LinearScheduler
(baselines/PixelGen/src/diffusion/flow_matching/scheduling.py:6-15) and BaseTrainer's caption dropout
(baselines/PixelGen/src/diffusion/base/training.py:8-36):
    t   = time_shift(sigmoid(P_std z + P_mean)), z ~ N(0, 1)   (logit-normal; uniform when lognorm_t is False)
    x_t = t x + (1 - t) eps                                     (alpha = t, sigma = 1 - t; t = 1 is data)
    v   = (x - x_t) / max(1 - t, t_eps),   v_hat = (net(x_t, t, y) - x_t) / max(1 - t, t_eps)
    loss = mean((v_hat - v)^2)                                  (constant weight)
The random draws happen in the reference's order: t first, then the noise.
"""
import torch


def time_shift_fn(t, timeshift=1.0):
    return t / (t + (1 - t) * timeshift)


class LinearScheduler:
    def alpha(self, t):
        return t.view(-1, 1, 1, 1)

    def sigma(self, t):
        return (1 - t).view(-1, 1, 1, 1)

    def dalpha(self, t):
        return torch.full_like(t.view(-1, 1, 1, 1), 1.0)

    def dsigma(self, t):
        return torch.full_like(t.view(-1, 1, 1, 1), -1.0)

    def dalpha_over_alpha(self, t):
        return self.dalpha(t) / self.alpha(t)

    def dsigma_mul_sigma(self, t):
        return self.dsigma(t) * self.sigma(t)


class JiTTrainer:
    """The training objective. `__call__` is the reference's call (any net with net(x_t, t, y, y_mask=...));
    `train_step` is the fused path for nano_gpic_b200's JiT_T2I: x_t is built and patchified by one kernel, the
    network runs on patch tokens, and the loss kernel returns the per-sample losses together with the gradient of the
    (scaled) mean, which is back-propagated at once."""

    def __init__(self, scheduler=None, loss_weight_fn=None, lognorm_t=True, timeshift=1.0, P_mean=-0.8, P_std=0.8,
                 t_eps=0.05, null_condition_p=0.0):
        self.scheduler = scheduler or LinearScheduler()
        self.loss_weight_fn = loss_weight_fn
        self.lognorm_t, self.timeshift = lognorm_t, timeshift
        self.P_mean, self.P_std, self.t_eps = P_mean, P_std, t_eps
        self.null_condition_p = null_condition_p

    def sample_t(self, batch, device, generator=None):
        if self.lognorm_t:
            base = (torch.randn(batch, device=device, dtype=torch.float32, generator=generator) * self.P_std
                    + self.P_mean).sigmoid()
        else:
            base = torch.rand(batch, device=device, dtype=torch.float32, generator=generator)
        return time_shift_fn(base, self.timeshift)

    def caption_dropout(self, y, y_mask, uncond):
        """BaseTrainer.preproprocess: with probability null_condition_p a sample takes the null caption (one token)."""
        if self.null_condition_p <= 0:
            return y, y_mask
        drop = torch.rand(y.shape[0], device=y.device) < self.null_condition_p
        if y_mask is not None:
            null_row = torch.zeros_like(y_mask[:1])
            null_row[:, 0] = True
            y_mask = torch.where(drop[:, None], null_row, y_mask)
        dm = drop.view(-1, *([1] * (y.dim() - 1))).to(y.dtype)
        return y * (1 - dm) + uncond * dm, y_mask

    def __call__(self, net, x, y, y_mask=None, t=None, noise=None):
        B = x.shape[0]
        t = self.sample_t(B, x.device) if t is None else t
        noise = torch.randn_like(x) if noise is None else noise
        alpha, sigma = self.scheduler.alpha(t), self.scheduler.sigma(t)
        x_t = alpha * x + noise * sigma
        den = (1 - t.view(-1, 1, 1, 1)).clamp_min(self.t_eps)
        v_t = (x - x_t) / den
        pred = net(x_t, t, y, y_mask=y_mask)
        out = (pred.float() - x_t) / den
        w = 1.0 if self.loss_weight_fn is None else self.loss_weight_fn(alpha, sigma)
        fm = w * (out - v_t) ** 2
        return dict(fm_loss=fm.mean(), loss=fm.mean(), loss_per_sample=fm.mean(dim=(1, 2, 3)))

    def train_step(self, net, x, y, y_mask=None, t=None, noise=None, grad_scale=None, backward=True, y_pack=None):
        """Forward + backward of the objective through the fused kernels. grad_scale multiplies the gradient of the
        sum of squared errors (default 1 / numel(x): the batch mean); with gradient accumulation over k micro-batches
        pass 1 / (k numel(x)). y_pack: packed captions (y [S, D] then; parallel.rebalance.pack_captions). Returns
        loss_per_sample [B] (fp32, on the device, no host sync)."""
        from ..ops import elementwise as E
        if y_pack is not None and self.null_condition_p > 0:
            raise ValueError("packed captions have no caption dropout (as in the reference: training.py:17-18)")
        B = x.shape[0]
        t = self.sample_t(B, x.device) if t is None else t
        noise = torch.randn_like(x) if noise is None else noise
        p = net.patch_size
        tok = E.fm_prep(x, noise, t, p)
        with torch.set_grad_enabled(backward):
            pred = net.forward_tokens(tok, t, y, y_mask, y_pack) if y_pack is not None else \
                net.forward_tokens(tok, t, y, y_mask)
        per, g = E.fm_loss(pred.detach(), x, noise, t, p, self.t_eps, grad_scale, need_grad=backward)
        if backward:
            pred.backward(g)
        return per


def constant(alpha, sigma):
    """Loss weight 1 at every noise level (reference training_JiT.constant)."""
    return 1.0
