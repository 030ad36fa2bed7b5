"""Ladder sizes, FLOPs per image, and steps for an iso-FLOP budget (reference tools/ladder_flops.py:19-106).

    python -m nano_gpic_b200.tools.ladder_flops [--budget 1.426e19] [--lengths caption_lengths.txt | --mean-T 51]
    python -m nano_gpic_b200.tools.ladder_flops --check     # formulas vs the real module (params; FLOPs on CPU)

FLOPs are the denoiser's training FLOPs (3 x forward) from its matmuls and attention (config.ladder.fwd_flops); the
frozen text encoder is not counted. With --lengths (one caption token length per line) the padded caption length T is
measured under the loader's length grouping: windows of 1024 sorted by length, cut into batches of --group-batch,
each padded to its longest caption rounded up to --pad-multiple (at most 320); E[T] and E[T^2] feed the formula.
"""
import argparse
import json
import random

from ..config.ladder import BOTTLENECK, L_TOKENS, PATCH_DIM, SIZES, TXT_DIM, TXT_MAX, fwd_flops, params_formula


def padded_lengths(lens, window=1024, batch=32, pad_multiple=8, max_len=TXT_MAX, seed=0):
    lens = list(lens)
    random.Random(seed).shuffle(lens)  # stand-in for the shard + sample shuffles
    Ts = []
    for w in range(0, len(lens) - window + 1, window):
        win = sorted(lens[w:w + window])
        for c in range(0, window, batch):
            Ts.append(min(-(-max(win[c:c + batch]) // pad_multiple) * pad_multiple, max_len))
    return Ts


def iso_flop_table(budget, ET, ET2, batch=1024, round_to=32):
    rows = []
    for name, s in SIZES.items():
        g = 3 * fwd_flops(s.width, s.image_layers, s.text_layers, ET, ET2)
        N = params_formula(s.width, s.image_layers, s.text_layers)
        steps = max(round_to, int(round(budget / (batch * g) / round_to)) * round_to)
        rows.append({"size": name, "d": s.width, "nb": s.image_layers, "nt": s.text_layers, "heads": s.heads,
                     "params_M": round(N / 1e6, 1), "gflop_per_img": round(g / 1e9, 1), "max_steps": steps,
                     "ms_every": steps // 4, "tpp": round(steps * batch * L_TOKENS / N, 1),
                     "budget_flops": steps * batch * g})
    return rows


def check(sizes=("d10",), T=64, batch=1):
    """Parameter count of the real module (meta device) and its forward FLOPs (FlopCounterMode over the CPU paths of
    the ops, which are plain torch matmuls) against the formulas."""
    import torch
    from torch.utils.flop_counter import FlopCounterMode
    from ..models.jit_t2i import JiT_T2I
    out = []
    for name in sizes:
        s = SIZES[name]
        kw = s.model_kwargs()
        with torch.device("meta"):
            n = sum(p.numel() for p in JiT_T2I(**kw).parameters() if p.requires_grad)
        f = params_formula(s.width, s.image_layers, s.text_layers)
        row = {"size": name, "params_real": n, "params_formula": f}
        m = JiT_T2I(**kw)
        x = torch.randn(batch, 3, 256, 256)
        y = torch.randn(batch, T, TXT_DIM)
        mask = torch.ones(batch, T, dtype=torch.bool)
        with torch.no_grad(), FlopCounterMode(display=False) as fc:
            m(x, torch.rand(batch), y, y_mask=mask)
        row.update(fwd_gflop_real=fc.get_total_flops() / batch / 1e9, fwd_gflop_formula=fwd_flops(
            s.width, s.image_layers, s.text_layers, T) / 1e9)
        out.append(row)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--budget", type=float, default=1.426e19)
    ap.add_argument("--batch", type=int, default=1024)
    ap.add_argument("--lengths", default=None)
    ap.add_argument("--mean-T", type=float, default=128.0)
    ap.add_argument("--group-batch", type=int, default=32)
    ap.add_argument("--pad-multiple", type=int, default=8)
    ap.add_argument("--out", default=None)
    ap.add_argument("--check", action="store_true")
    a = ap.parse_args(argv)
    if a.check:
        for r in check():
            print(json.dumps(r))
        return 0
    if a.lengths:
        with open(a.lengths) as f:
            Ts = padded_lengths([min(int(x), TXT_MAX) for x in f if x.strip()], batch=a.group_batch,
                                pad_multiple=a.pad_multiple)
        ET, ET2 = sum(Ts) / len(Ts), sum(t * t for t in Ts) / len(Ts)
    else:
        ET, ET2 = a.mean_T, a.mean_T ** 2
    rows = iso_flop_table(a.budget, ET, ET2, a.batch)
    print(f"budget {a.budget:.4e} FLOPs, E[T] {ET:.1f}, batch {a.batch}  (patch dim {PATCH_DIM}, bottleneck "
          f"{BOTTLENECK})")
    for r in rows:
        print(f"{r['size']:4s} {r['nb']}+{r['nt']} {r['params_M']:7.1f}M {r['gflop_per_img']:7.1f} GFLOP/img "
              f"{r['max_steps']:7d} steps  TPP {r['tpp']:6.1f}")
    if a.out:
        with open(a.out, "w") as f:
            json.dump({"budget": a.budget, "mean_padded_T": ET, "runs": rows}, f, indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
