"""CPU tests of nano_gpic_b200.tools.heldout_loss on a tiny JiT-T2I, modelled on the reference's
tools/test_heldout_loss.py:97-426 (H1 loss, H2 levels and noise, H3 repeatability, H4 inputs, H5 end-to-end work and
task hand-out, H6 one pass). The reference's own tool serves as the oracle where it can run here (its evaluate with
the same nets, data, levels and noise)."""
import importlib.util
import json
import math
import os
import statistics
import sys
import threading

import pytest
import torch
import yaml

from refpath import ref_root, reference_imports

from nano_gpic_b200.diffusion.flow_matching import JiTTrainer
from nano_gpic_b200.models.jit_t2i import JiT_T2I
from nano_gpic_b200.tools import heldout_loss as H

SMALL = dict(input_size=64, in_channels=3, num_groups=2, hidden_size=128, num_blocks=2, num_text_blocks=1, patch_size=16,
             txt_embed_dim=32, txt_max_length=32, bottleneck_dim=16)
LOSS = dict(timeshift=1.0, P_mean=-0.8, P_std=0.8, t_eps=0.05)


def fake_split(n, seed=0, max_len=20):
    g = torch.Generator().manual_seed(seed)
    img = torch.randint(0, 256, (n, 64, 64, 3), generator=g, dtype=torch.uint8)
    lens = torch.randint(1, max_len + 1, (n,), generator=g).tolist()
    emb = torch.randn(sum(lens), 32, generator=g)
    return H.HeldoutSplit(img, emb, lens, text_max_length=SMALL["txt_max_length"])


def tiny_net(seed):
    torch.manual_seed(seed)
    net = JiT_T2I(**SMALL).eval()
    with torch.no_grad():  # the final layer and adaLN start at zero: give every weight a value
        for p in net.parameters():
            p.add_(0.05 * torch.randn_like(p))
    return net


def objective_per_level(net, split, ts, seed, groups):
    """[num_t, N] per-image losses from JiTTrainer's own call with the level and the image's noise given."""
    obj = JiTTrainer(t_eps=LOSS["t_eps"])
    N, num_t = len(split), len(ts)
    per = torch.zeros(num_t, N, dtype=torch.float64)
    for idx in groups:
        x = split.images(idx, "cpu")
        y, mask = split.captions(idx, "cpu")
        for k in range(num_t):
            noise = torch.stack([H.image_noise(seed, j, num_t, split.image_shape)[k] for j in idx])
            with torch.no_grad():
                out = obj(net, x, y, mask, t=ts[k].expand(len(idx)).clone(), noise=noise)
            per[k, torch.as_tensor(idx)] = out["loss_per_sample"].double()
    return per


def test_H1_loss_equals_the_objective():
    """evaluate() equals JiTTrainer's loss per image and level on the same images, captions, t and noise, for any
    grouping of the images into batches."""
    torch.set_num_threads(4)
    split = fake_split(7)
    nets = {"a": tiny_net(1), "b": tiny_net(2)}
    ts = H.levels(**{k: LOSS[k] for k in ("P_mean", "P_std", "timeshift")})
    res = H.evaluate(nets, split, ts, seed=3, batch=3, threads=2)
    res4 = H.evaluate(nets, split, ts, seed=3, batch=4, threads=3)
    for name, net in nets.items():
        per = objective_per_level(net, split, ts, 3, [[0, 1, 2, 3], [4, 5, 6]])
        lm, im = res[name]["level_mean"], res[name]["image_mean"]
        assert lm.dtype == torch.float64 and lm.shape == (16,) and im.shape == (7,)
        torch.testing.assert_close(lm, per.mean(1), rtol=1e-5, atol=0)
        torch.testing.assert_close(im, per.mean(0), rtol=1e-5, atol=0)
        torch.testing.assert_close(res4[name]["level_mean"], lm, rtol=1e-5, atol=0)


def _reference_tool():
    root = ref_root()
    if root is None:
        pytest.skip("reference tree not available")
    spec = importlib.util.spec_from_file_location("ref_heldout_loss", os.path.join(root, "tools", "heldout_loss.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_H1_matches_the_reference_tool():
    """The reference tool's evaluate (its levels, noise feed, batching and loss) gives the same numbers for the same
    nets and data (the oracle)."""
    torch.set_num_threads(4)
    split = fake_split(9, seed=4)
    nets = {"a": tiny_net(5)}
    with reference_imports():
        R = _reference_tool()
        tr = R.make_trainer(dict(LOSS))
        rts = R.levels(LOSS["P_mean"], LOSS["P_std"], LOSS["timeshift"])
        rsplit = dict(img=split.img, emb=split.emb, lens=list(split.lens), offs=list(split.starts),
                      pad_multiple=split.pad_multiple, text_max_length=split.text_max_length,
                      order=sorted(range(len(split)), key=lambda i: (split.lens[i], i)))
        ref = R.evaluate(nets, tr, rsplit, rts, seed=0, batch=4, device="cpu", autocast=False, threads=2)
        ref_noise = R.image_noise(0, 5, 16, (3, 64, 64))
    ts = H.levels()
    assert torch.equal(ts, rts)
    assert torch.equal(H.image_noise(0, 5, 16, (3, 64, 64)), ref_noise)
    got = H.evaluate(nets, split, ts, seed=0, batch=4, threads=3)
    torch.testing.assert_close(got["a"]["level_mean"], ref["a"]["level_mean"], rtol=1e-6, atol=0)
    torch.testing.assert_close(got["a"]["image_mean"], ref["a"]["image_mean"], rtol=1e-6, atol=0)


def test_H2_levels_and_noise():
    """The 16 levels from an independent formula (statistics.NormalDist), for two time shifts; image j's noise is the
    draw of a generator seeded SEED * 1_000_003 + j and does not depend on the other images."""
    nd = statistics.NormalDist()
    for shift in (1.0, 3.0):
        ts = H.levels(-0.8, 0.8, shift)
        for k in range(16):
            base = 1 / (1 + math.exp(-(-0.8 + 0.8 * nd.inv_cdf((k + 0.5) / 16))))
            base = float(torch.tensor(base, dtype=torch.float32))
            want = base / (base + (1 - base) * shift)
            assert abs(float(ts[k]) - want) < 1e-6, (shift, k, float(ts[k]), want)
    g = torch.Generator().manual_seed(0 * 1_000_003 + 11)
    assert torch.equal(H.image_noise(0, 11, 16, (3, 8, 8)), torch.randn((16, 3, 8, 8), generator=g))
    out = torch.empty(16, 3, 8, 8)
    H.image_noise(2, 4, 16, (3, 8, 8), out=out)
    assert torch.equal(out, H.image_noise(2, 4, 16, (3, 8, 8)))


def test_H3_repeatable_bit_for_bit():
    """Two evaluations give identical numbers."""
    split = fake_split(6, seed=2)
    nets = {"a": tiny_net(3)}
    ts = H.levels()
    r1 = H.evaluate(nets, split, ts, seed=0, batch=4, threads=3)
    r2 = H.evaluate(nets, split, ts, seed=0, batch=4, threads=1)
    assert torch.equal(r1["a"]["level_mean"], r2["a"]["level_mean"])
    assert torch.equal(r1["a"]["image_mean"], r2["a"]["image_mean"])


def test_H4_inputs():
    """to_input is ToTensor + Normalize(0.5, 0.5) bit for bit; captions pad to the batch's longest rounded up to 8, at
    most text_max_length, with zeros and False after each caption; batches go in order of caption length."""
    u8 = torch.randint(0, 256, (2, 5, 4, 3), dtype=torch.uint8)
    ref = torch.stack([((im.permute(2, 0, 1).float().div(255)) - 0.5) / 0.5 for im in u8])
    assert torch.equal(H.to_input(u8), ref)
    img, emb, lens = torch.zeros(4, 2, 2, 3, dtype=torch.uint8), torch.arange(60.).view(30, 2), [3, 11, 1, 15]
    split = H.HeldoutSplit(img, emb, lens, text_max_length=20)
    y, m = split.captions([0, 1, 2], "cpu")  # longest 11 -> 16
    assert y.shape == (3, 16, 2) and m.sum(1).tolist() == [3, 11, 1]
    assert torch.equal(y[1, :11], torch.arange(6., 28.).view(11, 2)) and not y[1, 11:].any() and not m[1, 11:].any()
    capped = H.HeldoutSplit(img, emb, lens, text_max_length=12)
    y, m = capped.captions([3], "cpu")  # 15 tokens -> 16, capped at 12
    assert y.shape == (1, 12, 2) and m.all() and torch.equal(y[0], torch.arange(30., 54.).view(12, 2))
    assert split.batches(3) == [[2, 0, 1], [3]]


# ------------------------------------------------------------------------------------------- fake runs (H5, H6)
def _write_run(root, name, steps, twins, seed=0):
    run = os.path.join(root, name)
    os.makedirs(run, exist_ok=True)
    cfg = {"model": {"denoiser": {"class_path": "src.models.transformer.JiT_T2I.JiT_T2I", "init_args": dict(SMALL)},
                     "diffusion_trainer": {"init_args": dict(LOSS)}}}
    with open(os.path.join(run, "config-TrainerFn.FITTING-2026-01-01_00-00-00.yaml"), "w") as f:
        yaml.safe_dump(cfg, f)
    paths = []
    for s in steps:
        raw = tiny_net(seed + s).state_dict()
        ema = {k: v.clone() for k, v in raw.items()} if twins else tiny_net(seed + s + 100).state_dict()
        sd = {**{"denoiser." + k: v for k, v in raw.items()}, **{"ema_denoiser." + k: v for k, v in ema.items()}}
        p = os.path.join(run, f"ms-step={s:06d}.ckpt")
        torch.save({"state_dict": sd, "global_step": s}, p)
        paths.append(p)
    return paths


def _data_file(path):
    val, train = fake_split(5, seed=7), fake_split(4, seed=8)
    torch.save(dict(version=1, n_val=5, n_train=4, val=val.to_saved(), train=train.to_saved()), path)


def _records(path):
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


def test_H5_work_list_and_claims(tmp_path, capsys):
    """work on fake checkpoints writes one record per (checkpoint, weights) with the asked fields; a second run adds
    nothing; list skips what is done and lists a checkpoint with one weights missing; claim files hand out every task
    once among concurrent workers; a checkpoint still being written is left out of the listing."""
    torch.set_num_threads(2)
    root = str(tmp_path)
    ckpts = _write_run(root, "exp_ladder_d128", [10, 20], twins=False)
    data = os.path.join(root, "data_v1.pt")
    _data_file(data)
    out = os.path.join(root, "heldout.jsonl")
    base = ["--n-val", "5", "--n-train", "4", "--data", data, "--out", out]
    assert H.main(["work", *base, "--device", "cpu", "--batch", "3", "--threads", "2", "--ckpt", *ckpts]) == 0
    recs = _records(out)
    assert sorted((r["step"], r["weights"]) for r in recs) == [(10, "ema"), (10, "raw"), (20, "ema"), (20, "raw")]
    r = recs[0]
    for k in ("ckpt", "run_root", "size", "step", "weights", "n_val", "n_train", "num_t", "seed", "data", "t", "d",
              "nb", "nt", "loss_val", "loss_val_t", "loss_val_se", "loss_train", "loss_train_t", "loss_train_se",
              "elapsed_s", "one_pass", "weights_in_task"):
        assert k in r, k
    assert r["size"] == "d128" and r["num_t"] == 16 and len(r["loss_val_t"]) == 16 and r["data"] == "data_v1"
    assert not r["one_pass"] and r["d"] == 128
    assert abs(r["loss_val"] - sum(r["loss_val_t"]) / 16) < 1e-9
    # the record equals a direct evaluation of the same weights
    sd = torch.load(ckpts[0])["state_dict"]
    net = H.build_denoiser(dict(SMALL), sd, "denoiser.", "cpu")
    direct = H.evaluate({"raw": net}, H.load_data(data)["val"], H.levels(), batch=3)["raw"]["level_mean"]
    raw10 = next(x for x in recs if x["step"] == 10 and x["weights"] == "raw")
    assert abs(raw10["loss_val"] - float(direct.mean())) < 1e-6
    # idempotent: a second run adds nothing
    assert H.main(["work", *base, "--device", "cpu", "--ckpt", *ckpts]) == 0
    assert len(_records(out)) == 4
    # list: nothing to do; drop one record and the checkpoint comes back
    capsys.readouterr()
    H.main(["list", *base, "--runs", root, "--min-age", "0"])
    assert capsys.readouterr().out.strip() == ""
    with open(out, "w") as f:
        f.writelines(json.dumps(x) + "\n" for x in recs if not (x["step"] == 20 and x["weights"] == "ema"))
    H.main(["list", *base, "--runs", root, "--min-age", "0"])
    listed = [json.loads(line) for line in capsys.readouterr().out.splitlines() if line.strip()]
    assert [t["step"] for t in listed] == [20]
    # a young file that is not a whole zip yet is left out and named in --skipped
    young = os.path.join(root, "exp_ladder_d128", "ms-step=000030.ckpt")
    with open(young, "wb") as f:
        f.write(b"PK\x03\x04 partial")
    skipped = os.path.join(root, "skipped.txt")
    H.main(["list", *base, "--runs", root, "--min-age", "3600", "--skipped", skipped])
    assert [json.loads(line)["step"] for line in capsys.readouterr().out.splitlines() if line.strip()] == [20]
    assert open(skipped).read().strip() == os.path.abspath(young)
    # claims: 4 workers over 50 tasks, each index handed out once
    counter = os.path.join(root, "counter")
    got, lock = [], threading.Lock()

    def worker():
        c = H.ClaimDir(counter + ".claims")
        while (i := c.next(50)) is not None:
            with lock:
                got.append(i)
    ths = [threading.Thread(target=worker) for _ in range(4)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    assert sorted(got) == list(range(50))


def test_H6_one_pass_for_twin_weights(tmp_path):
    """A checkpoint whose EMA slot holds the raw weights' bytes gives both records from one pass, marked one_pass, with
    the values a separate pass gives; one flipped bit in one EMA tensor gives the two-pass path."""
    torch.set_num_threads(2)
    root = str(tmp_path)
    (twin,) = _write_run(root, "exp_ladder_d128", [5], twins=True)
    data = os.path.join(root, "data_v1.pt")
    _data_file(data)
    out = os.path.join(root, "a.jsonl")
    assert H.main(["work", "--n-val", "5", "--n-train", "4", "--data", data, "--out", out, "--device", "cpu",
                   "--ckpt", twin]) == 0
    recs = {r["weights"]: r for r in _records(out)}
    assert recs["ema"]["one_pass"] and recs["raw"]["one_pass"]
    assert recs["ema"]["loss_val_t"] == recs["raw"]["loss_val_t"]
    ck = torch.load(twin)
    assert H.ema_is_raw(ck["state_dict"])
    key = next(k for k in ck["state_dict"] if k.startswith("ema_denoiser.") and ck["state_dict"][k].numel() > 3)
    t = ck["state_dict"][key].clone()
    t.view(-1).view(torch.int32)[3] ^= 1
    ck["state_dict"][key] = t
    assert not H.ema_is_raw(ck["state_dict"])
    torch.save(ck, twin)
    out2 = os.path.join(root, "b.jsonl")
    assert H.main(["work", "--n-val", "5", "--n-train", "4", "--data", data, "--out", out2, "--device", "cpu",
                   "--ckpt", twin]) == 0
    recs2 = {r["weights"]: r for r in _records(out2)}
    assert not recs2["ema"]["one_pass"] and not recs2["raw"]["one_pass"]
    assert recs2["raw"]["loss_val_t"] == recs["raw"]["loss_val_t"]
    assert abs(recs2["ema"]["loss_val"] - recs["ema"]["loss_val"]) < 1e-6
