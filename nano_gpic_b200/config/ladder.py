"""The scaling ladder: per-size model shape and recipe, and the FLOP/parameter formulas used for MFU.

Sizes and recipe values are the reference's final ladder (jobs/final_ladder_sizes.sh:6-17, README.md:15-46):
width D = 128 x (image layers - 4), heads = D / 64, Muon lr, AdamW lr, Muon weight decay, steps at batch 1024 and the
per-GPU micro-batch of an 8-GPU node. FLOPs per image follow tools/ladder_flops.py:19-28 (forward; training = 3 x
forward; the frozen text encoder is not counted).
"""
from dataclasses import dataclass

L_TOKENS, PATCH_DIM, BOTTLENECK, TXT_DIM, TXT_MAX = 256, 768, 256, 2048, 320
GLOBAL_BATCH = 1024


@dataclass(frozen=True)
class LadderSize:
    name: str
    width: int
    image_layers: int
    text_layers: int
    steps: int
    muon_lr: float
    adamw_lr: float
    muon_wd: float
    micro_batch: int

    @property
    def heads(self):
        return self.width // 64

    def model_kwargs(self):
        return dict(input_size=256, in_channels=3, num_groups=self.heads, hidden_size=self.width,
                    num_blocks=self.image_layers, num_text_blocks=self.text_layers, patch_size=16,
                    txt_embed_dim=TXT_DIM, txt_max_length=TXT_MAX, bottleneck_dim=BOTTLENECK)

    def schedule(self):
        """(warmup, cooldown) of the final ladder: 1% warmup, linear cooldown over the last half (multiple of 32)."""
        return self.steps // 100, self.steps // 2 // 32 * 32


SIZES = {s.name: s for s in [
    LadderSize("d10", 768, 10, 2, 21248, 1.36e-2, 5.01e-4, 0.0173, 128),
    LadderSize("d11", 896, 11, 2, 28800, 9.617e-3, 4.06e-4, 0.01805, 128),
    LadderSize("d12", 1024, 12, 3, 40192, 6.8e-3, 3.26e-4, 0.01829, 128),
    LadderSize("d13", 1152, 13, 3, 59136, 4.808e-3, 2.77e-4, 0.01758, 128),
    LadderSize("d14", 1280, 14, 3, 89600, 3.4e-3, 2.38e-4, 0.01641, 128),
    LadderSize("d16", 1536, 16, 4, 108800, 2.404e-3, 1.79e-4, 0.01912, 128),
    LadderSize("d18", 1792, 18, 4, 143872, 1.7e-3, 1.44e-4, 0.02044, 64),
]}


def fwd_flops(d, nb, nt, T, T2=None):
    """Forward FLOPs per image at caption length T (E[T]) and E[T^2] (tools/ladder_flops.py:19-24)."""
    T2 = T * T if T2 is None else T2
    L, P, B = L_TOKENS, PATCH_DIM, BOTTLENECK
    main = nb * (32 * L * d * d + 4 * T * d * d + 4 * L * (L + T) * d)
    text = nt * (32 * T * d * d + 4 * T2 * d)
    emb = 2 * L * P * B + 2 * L * B * d + 2 * T * TXT_DIM * d + 2 * L * d * P
    return main + text + emb


def train_flops_per_image(size, T):
    s = SIZES[size] if isinstance(size, str) else size
    return 3 * fwd_flops(s.width, s.image_layers, s.text_layers, T)


def params_formula(d, nb, nt):
    """All parameters (tools/ladder_flops.py:27-28)."""
    L, P, B = L_TOKENS, PATCH_DIM, BOTTLENECK
    return nb * 24 * d * d + nt * 22 * d * d + P * B + B * d + TXT_DIM * d + TXT_MAX * d + 256 * d + d * d + d * P


def muon_lr_rule(flops):
    """Muon lr = 1.36e-2 (C / 3.6e18)^-0.5 (README.md:36-41)."""
    return 1.36e-2 * (flops / 3.6e18) ** -0.5


def adamw_lr_rule(n_params):
    """AdamW lr = 6.4e-4 (N / 109.4M)^-0.547 (README.md:36-41)."""
    return 6.4e-4 * (n_params / 109.4e6) ** -0.547


def muon_wd_rule(muon_lr, steps):
    """Muon weight decay = 5 / (lr x steps) (README.md:36-41)."""
    return 5.0 / (muon_lr * steps)


def dp_mode(size):
    """Data-parallel mode of a ladder size: the reference shards from d14 up (FSDP2, jobs/final_ladder.sh:30); here
    zero mode (reduce-scatter to owners, sharded optimizer state) from d14, ddp below."""
    s = SIZES[size] if isinstance(size, str) else size
    return "zero" if s.width >= 1280 else "ddp"


def shell_vars(size, gpus=8):
    """The launch variables of a size as shell assignments (consumed by jobs/final_ladder.sh): width, layers, steps,
    learning rates, weight decay, micro-batch, warmup/cooldown, accumulation for `gpus` GPUs, data-parallel mode."""
    s = SIZES[size]
    wu, cd = s.schedule()
    acc = GLOBAL_BATCH // gpus // s.micro_batch
    return (f"D={s.width} NB={s.image_layers} NT={s.text_layers} S={s.steps} MLR={s.muon_lr} ALR={s.adamw_lr} "
            f"WDK={s.muon_wd} MB={s.micro_batch} WU={wu} CD={cd} ACC={acc} DP={dp_mode(s)}")


if __name__ == "__main__":
    import sys
    if len(sys.argv) >= 3 and sys.argv[1] == "--shell":
        print(shell_vars(sys.argv[2], int(sys.argv[3]) if len(sys.argv) > 3 else 8))
    else:
        for name, s in SIZES.items():
            print(name, shell_vars(name))
