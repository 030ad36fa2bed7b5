"""Learning-rate schedules (reference baselines/PixelGen/src/utils/lr_scheduler.py:27-57).

WarmupFlatCooldown: linear warmup over num_warmup_steps, a flat rate, then a linear cooldown over the last
num_cooldown_steps of max_steps to an absolute min_lr that every param group reaches (each group gets its own floor
min_lr / its initial rate; min_lr = 0 decays to 0 with one shared lambda). A factory: `WarmupFlatCooldown(...)(opt)`
returns the LambdaLR, as the reference's LightningCLI callable does.
"""
from torch.optim.lr_scheduler import LambdaLR


class WarmupFlatCooldown:
    def __init__(self, num_warmup_steps: int, num_cooldown_steps: int, max_steps: int, min_lr: float = 0.0):
        self.num_warmup_steps = num_warmup_steps
        self.num_cooldown_steps = num_cooldown_steps
        self.max_steps = max_steps
        self.min_lr = min_lr

    def lr_lambda(self, floor):
        warmup, cooldown, total = self.num_warmup_steps, self.num_cooldown_steps, self.max_steps

        def f(step):
            if step < warmup:
                return step / max(1, warmup)
            if step < total - cooldown:
                return 1.0
            frac = min(1.0, (step - (total - cooldown)) / max(1, cooldown))
            return 1.0 - (1.0 - floor) * frac
        return f

    def __call__(self, optimizer):
        if not self.min_lr:
            return LambdaLR(optimizer, lr_lambda=self.lr_lambda(0.0))
        floors = [min(1.0, self.min_lr / g.get("initial_lr", g["lr"])) for g in optimizer.param_groups]
        return LambdaLR(optimizer, lr_lambda=[self.lr_lambda(f) for f in floors])


class ConstantWithWarmup:
    """Linear warmup then constant (reference lr_scheduler.py:19-24, transformers' get_constant_schedule_with_warmup)."""

    def __init__(self, num_warmup_steps: int):
        self.num_warmup_steps = num_warmup_steps

    def __call__(self, optimizer):
        w = self.num_warmup_steps
        return LambdaLR(optimizer, lr_lambda=lambda s: min(1.0, s / max(1.0, w)))
