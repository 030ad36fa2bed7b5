"""Offline tools on CPU: the GPU-health verdict (fake NVML and fake worker results; nothing touches a GPU), ladder
formulas against the module, the scaling-law fit, the sample-quality metrics against closed forms, and the text-cache
builder/checker with a tiny random Qwen3."""
import io
import json
import os
import tarfile

import numpy as np
import pytest
import torch


# ----------------------------------------------------------------------------------------------- gpu health
class FakeNVML:
    NVML_CLOCK_SM, NVML_TEMPERATURE_GPU = 1, 0

    def __init__(self, clock, temp, reasons):
        self.v = (clock, temp, reasons)

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetClockInfo(self, h, kind):
        return self.v[0]

    def nvmlDeviceGetTemperature(self, h, kind):
        return self.v[1]

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return self.v[2]


def test_gpu_health_verdicts():
    from nano_gpic_b200.tools.gpu_health import judge, sample_nvml
    assert sample_nvml(3, FakeNVML(1860, 61, 0x4)) == (1860, 61, 0x4)
    good = {g: {"tflops": 1400 + g, "clock": 1860, "temp": 60, "reasons": 0x4} for g in range(8)}  # sw_power_cap: ok
    ok, lines, bad = judge(good)
    assert ok and not bad and lines[-1].endswith("healthy")
    slow = dict(good)
    slow[5] = {**good[5], "tflops": 900}
    ok, _, bad = judge(slow)
    assert not ok and bad == [5]
    hot = dict(good)
    hot[2] = {**good[2], "reasons": 0x40}
    ok, lines, bad = judge(hot)
    assert not ok and bad == [2] and "hw_thermal_slowdown" in lines[2]
    err = dict(good)
    err[1] = {"error": "CUDA init failed"}
    ok, lines, bad = judge(err)
    assert not ok and bad == [] and lines[-1] == "check failed, node unknown"


# ---------------------------------------------------------------------------------------------- ladder / fits
def test_ladder_formulas():
    from nano_gpic_b200.config.ladder import SIZES, params_formula, shell_vars
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    from nano_gpic_b200.tools.ladder_flops import iso_flop_table, padded_lengths
    for name in ("d10", "d12"):
        s = SIZES[name]
        with torch.device("meta"):
            n = sum(p.numel() for p in JiT_T2I(**s.model_kwargs()).parameters() if p.requires_grad)
        assert abs(params_formula(s.width, s.image_layers, s.text_layers) / n - 1) < 2e-3
    assert shell_vars("d12").startswith("D=1024 NB=12 NT=3 S=40192") and "ACC=1 DP=ddp" in shell_vars("d12")
    assert "DP=zero" in shell_vars("d18") and "ACC=2" in shell_vars("d18")
    rows = iso_flop_table(1.426e19, 128, 128 ** 2)
    assert [r["max_steps"] % 32 for r in rows] == [0] * len(rows)
    assert all(a["max_steps"] > b["max_steps"] for a, b in zip(rows, rows[1:]))
    Ts = padded_lengths([5] * 2048, window=1024, batch=32)
    assert set(Ts) == {8} and len(Ts) == 64


def test_scaling_law_recovers_a_known_law():
    from nano_gpic_b200.tools.scaling_law import C0, loss_at, optimum, run
    p = {"E": 0.046, "A": 5e-5, "B": 4e-4, "alpha": 0.5, "beta": 0.55, "k": 0.2}
    N, D, C = [], [], []
    for j in range(5):
        Cb = C0 * 2 ** j
        n0, _ = optimum(p, Cb)
        for f in (0.4, 0.6, 1.0, 1.6, 2.5):
            n = n0 * f
            N.append(n)
            D.append(Cb / (6 * n))
            C.append(Cb)
    N, D, C = map(np.array, (N, D, C))
    L = np.array([loss_at(p, n, d) for n, d in zip(N, D)])
    res = run(N, D, L, C)
    assert res["rms_rel_err"] < 1e-4
    assert abs(res["N_exponent"] - p["beta"] / (p["alpha"] + p["beta"])) < 0.02


def test_scaling_law_on_reference_runs():
    from nano_gpic_b200.tools.scaling_law import default_csv, load, run
    if not os.path.exists(default_csv()):
        pytest.skip("reference run table not available")
    _, N, D, L, C = load(default_csv())
    res = run(N, D, L, C)
    # the published law: E 0.0457, N* ~ C^0.50, a 0.057% RMS loss error
    assert abs(res["params"]["E"] - 0.0457) < 1e-3 and abs(res["N_exponent"] - 0.50) < 0.02
    assert res["rms_rel_err"] < 8e-4


# -------------------------------------------------------------------------------------------------- metrics
def test_metrics_closed_forms():
    from nano_gpic_b200.eval.metrics import frechet_distance, mmd2_unbiased, prdc, statistics
    rng = np.random.default_rng(0)
    s1 = np.diag([1.0, 2.0, 3.0])
    s2 = np.diag([2.0, 1.0, 0.5])
    mu1, mu2 = np.zeros(3), np.array([1.0, 0.0, 2.0])
    want = 5.0 + np.sum(np.diag(s1) + np.diag(s2) - 2 * np.sqrt(np.diag(s1) * np.diag(s2)))
    assert abs(frechet_distance(mu1, s1, mu2, s2) - want) < 1e-9
    x = rng.normal(size=(2000, 8))
    y = rng.normal(size=(2000, 8))
    m1, c1 = statistics(x)
    assert abs(frechet_distance(m1, c1, m1, c1)) < 1e-6
    r = prdc(x[:500], y[:500], k=5)
    assert r["precision"] > 0.7 and r["recall"] > 0.7 and r["coverage"] > 0.7
    far = prdc(x[:500], y[:500] + 10, k=5)
    assert far["precision"] == 0 and far["coverage"] == 0
    assert abs(mmd2_unbiased(x[:500], y[:500])) < 0.02 < mmd2_unbiased(x[:500], y[:500] + 1.0)


# --------------------------------------------------------------------------------------------------- text cache
class ByteTokenizer:
    eos_token_id = 1

    def __call__(self, texts, truncation=True, max_length=320, padding="longest", pad_to_multiple_of=8,
                 return_tensors="pt"):
        ids = [[2 + (ord(c) % 200) for c in t][:max_length] for t in texts]
        T = max(len(i) for i in ids)
        T = min(-(-T // pad_to_multiple_of) * pad_to_multiple_of, max_length)
        out = torch.zeros(len(ids), T, dtype=torch.long)
        mask = torch.zeros(len(ids), T, dtype=torch.long)
        for r, i in enumerate(ids):
            out[r, :len(i)] = torch.tensor(i)
            mask[r, :len(i)] = 1
        return {"input_ids": out, "attention_mask": mask}


def _tiny_qwen3():
    from transformers import Qwen3Config, Qwen3Model
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=1,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=32, max_position_embeddings=512)
    return Qwen3Model(cfg)


def _write_tar(path, n):
    from PIL import Image
    with tarfile.open(path, "w") as tar:
        for i in range(n):
            key = f"s{i:04d}"
            buf = io.BytesIO()
            Image.new("RGB", (32, 32), (i, 2 * i, 3)).save(buf, format="JPEG")
            meta = json.dumps({"caption": "a photo " + "x" * (i * 7 % 40), "caption_type": "short"}).encode()
            for suffix, data in (("jpg", buf.getvalue()), ("json", meta)):
                ti = tarfile.TarInfo(f"{key}.{suffix}")
                ti.size = len(data)
                tar.addfile(ti, io.BytesIO(data))


def test_text_cache_build_and_check(tmp_path):
    from nano_gpic_b200.data.text_cache import TextCache
    from nano_gpic_b200.models.conditioner import Qwen3TextEncoder
    from nano_gpic_b200.tools.check_text_cache import check_shard
    from nano_gpic_b200.tools.encode_captions import encode_shard
    tar = tmp_path / "gpic_train_00000.tar"
    _write_tar(str(tar), 6)
    enc = Qwen3TextEncoder(model=_tiny_qwen3(), tokenizer=ByteTokenizer(), embed_dim=2048)
    out = tmp_path / "emb"
    assert encode_shard(enc, str(tar), str(out), batch=4) == 6
    assert check_shard(str(tar), str(out)) == []
    cache = TextCache(str(out))
    e = cache.read("gpic_train_00000", "s0003")
    ids, mask = enc.tokenize(["a photo " + "x" * (3 * 7 % 40)])
    direct, _ = enc.encode(ids, mask)
    assert e.shape == (int(mask.sum()), 2048) and torch.equal(e, direct[0, :e.shape[0]])
    assert e[:, 64:].abs().sum() == 0  # features past the encoder width are zero-padded to embed_dim
    assert enc.null().shape == (1, 1, 2048)


def test_ckpt_shard_clock(tmp_path, capsys):
    from nano_gpic_b200.tools.ckpt_shard_clock import main
    p = tmp_path / "last.ckpt"
    torch.save({"gpic_shard_clock": {"time": 12.5, "seed": "7", "step": 40}}, p)
    main([str(p)])
    assert capsys.readouterr().out.split() == ["12.5", "7", "40"]
