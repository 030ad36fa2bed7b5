"""Kernel microbenchmarks on one GPU: each hand-written kernel against its library counterpart (cuBLAS through
torch.matmul, SDPA, torch elementwise), timed with CUDA events after warm-up, inputs larger than L2 where the shape
allows, reported as TFLOP/s or GB/s and as a fraction of MEASURED_PEAKS.json.

    python -m nano_gpic_b200.tools.bench_kernels [--only gemm,fused,attn,mx,sample] [--d 1024] [--batch 128] [--json out.json]
"""
import argparse
import json
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["bf16_tflops"], d["hbm_gbs"], "measured"
    return 1590.0, 6650.0, "fallback"


def time_fn(fn, iters=20, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e-3


def bench_gemm(d, batch, rows):
    from nano_gpic_b200.ops import gemm
    M = batch * 256
    shapes = [("qkv_x", M, 3 * d, d), ("proj", M, d, d), ("w12", M, 8 * d, d), ("w3", M, d, 4 * d),
              ("kv_y", batch * 128, 2 * d, d)]
    pk, _, src = peaks()
    for name, m, n, k in shapes:
        x = torch.randn(m, k, device="cuda").bfloat16()
        w = (torch.randn(n, k, device="cuda") * 0.02).bfloat16()
        dy = torch.randn(m, n, device="cuda").bfloat16()
        fl = 2.0 * m * n * k
        from nano_gpic_b200._ext import ext
        res = {}
        for pair in (1, 0):  # CTA-pair (cta_group::2) tiles, then single-CTA tiles
            ext().gemm_set_pair(pair)
            sfx = "ours" if pair else "ours1cta"
            res["fwd_" + sfx] = time_fn(lambda: gemm.linear(x, w))
            res["dgrad_" + sfx] = time_fn(lambda: gemm.linear_dgrad(dy, w))
            res["wgrad_" + sfx] = time_fn(lambda: gemm.linear_wgrad(dy, x))
        ext().gemm_set_pair(1)
        res["fwd_cublas"] = time_fn(lambda: x @ w.t())
        res["dgrad_cublas"] = time_fn(lambda: dy @ w)
        res["wgrad_cublas"] = time_fn(lambda: dy.t() @ x)
        row = {"kernel": "gemm", "name": name, "M": m, "N": n, "K": k}
        for kk, v in res.items():
            row[kk + "_us"] = round(v * 1e6, 1)
            row[kk + "_tflops"] = round(fl / v / 1e12, 1)
            row[kk + "_frac_of_" + src] = round(fl / v / 1e12 / pk, 3)
        rows.append(row)
        print(json.dumps(row), flush=True)
        del x, w, dy


def bench_fused(d, batch, rows):
    """Fused-epilogue GEMMs against the plain GEMM of the same shape (the epilogue's cost is the difference)."""
    from nano_gpic_b200.ops import gemm
    M = batch * 256
    pk, _, src = peaks()
    r = lambda *s: (torch.randn(*s, device="cuda") * 0.5).bfloat16()
    x, w12, w3, pre, dy = r(M, d), r(8 * d, d), r(d, 4 * d), r(M, 8 * d), r(M, d)
    wp, res, mod = r(d, d), r(M, d), r(batch, 6 * d)
    bias = torch.zeros(d, device="cuda")
    cases = [("swiglu_fwd", lambda: gemm.swiglu_linear(x, w12), lambda: gemm.linear(x, w12), 2.0 * M * 8 * d * d),
             ("swiglu_bwd", lambda: gemm.swiglu_dgrad(dy, w3, pre), lambda: gemm.linear_dgrad(dy, w3), 2.0 * M * 4 * d * d),
             ("gated_proj", lambda: gemm.linear_gated_residual(x, wp, bias, res, mod[:, 2 * d:3 * d], 256),
              lambda: gemm.linear(x, wp), 2.0 * M * d * d)]
    for name, fused, plain, fl in cases:
        tf, tp = time_fn(fused), time_fn(plain)
        row = {"kernel": "gemm_fused", "name": name, "M": M, "d": d, "fused_us": round(tf * 1e6, 1),
               "plain_us": round(tp * 1e6, 1), "fused_tflops": round(fl / tf / 1e12, 1),
               "plain_tflops": round(fl / tp / 1e12, 1), "fused_frac_of_" + src: round(fl / tf / 1e12 / pk, 3)}
        rows.append(row)
        print(json.dumps(row), flush=True)


def bench_attn(d, batch, rows, T=128):
    """Image joint attention (256 queries, 256 image + T caption keys with random valid lengths): tcgen05 and
    mma.sync forward/backward, and torch SDPA with a boolean key mask (the reference's call) on the same problem."""
    from nano_gpic_b200.ops import attention as A
    H, L = d // 64, 256
    M = batch * L
    r = lambda *s: (torch.randn(*s, device="cuda")).bfloat16()
    qkv, kv = r(M, 3 * d), r(batch * T, 2 * d)
    lens = torch.randint(1, T + 1, (batch,), device="cuda", dtype=torch.int32)
    q, k0, v0, k1, v1 = qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:], kv[:, :d], kv[:, d:]
    o, lse = A.attn_fwd(q, L, k0, v0, L, L, k1, v1, T, lens)
    do = r(M, d)
    # FLOPs of the work that must be done: valid keys only
    keys = (L + lens.float()).sum().item()
    fl_fwd = 4.0 * L * keys * 64 * H
    res = {"tc_fwd": time_fn(lambda: A.attn_fwd(q, L, k0, v0, L, L, k1, v1, T, lens, impl="tc")),
           "tc2_fwd": time_fn(lambda: A.attn_fwd(q, L, k0, v0, L, L, k1, v1, T, lens, impl="tc2")),
           "tc1_fwd": time_fn(lambda: A.attn_fwd(q, L, k0, v0, L, L, k1, v1, T, lens, impl="tc1")),
           "mma_fwd": time_fn(lambda: A.attn_fwd(q, L, k0, v0, L, L, k1, v1, T, lens, impl="mma")),
           "tc_bwd": time_fn(lambda: A.attn_bwd(do, q, L, k0, v0, L, L, o, lse, k1, v1, T, lens, impl="tc")),
           "tc2_bwd": time_fn(lambda: A.attn_bwd(do, q, L, k0, v0, L, L, o, lse, k1, v1, T, lens, impl="tc2")),
           "tc1_bwd": time_fn(lambda: A.attn_bwd(do, q, L, k0, v0, L, L, o, lse, k1, v1, T, lens, impl="tc1")),
           "mma_bwd": time_fn(lambda: A.attn_bwd(do, q, L, k0, v0, L, L, o, lse, k1, v1, T, lens, impl="mma"))}
    Q = q.view(batch, L, H, 64).transpose(1, 2)
    K = torch.cat([k0.reshape(batch, L, H, 64), k1.reshape(batch, T, H, 64)], 1).transpose(1, 2)
    V = torch.cat([v0.reshape(batch, L, H, 64), v1.reshape(batch, T, H, 64)], 1).transpose(1, 2)
    mask = torch.cat([torch.ones(batch, L, dtype=torch.bool, device="cuda"),
                      torch.arange(T, device="cuda")[None] < lens[:, None]], 1)[:, None, None, :]
    sdpa = torch.nn.functional.scaled_dot_product_attention
    res["sdpa_fwd"] = time_fn(lambda: sdpa(Q, K, V, attn_mask=mask))
    Qg, Kg, Vg = (t.detach().clone().requires_grad_(True) for t in (Q, K, V))
    out = sdpa(Qg, Kg, Vg, attn_mask=mask)
    g = torch.randn_like(out)
    res["sdpa_bwd"] = time_fn(lambda: torch.autograd.grad(out, (Qg, Kg, Vg), g, retain_graph=True))
    row = {"kernel": "attention", "B": batch, "H": H, "Lq": L, "T": T}
    for k, v in res.items():
        row[k + "_us"] = round(v * 1e6, 1)
        row[k + "_tflops"] = round((fl_fwd if "fwd" in k else 2.5 * fl_fwd) / v / 1e12, 1)
    rows.append(row)
    print(json.dumps(row), flush=True)


def bench_mx(d, batch, rows):
    """The image block's forward GEMMs (qkv_x, proj + gated residual, w12 + SwiGLU, w3 + gated residual) in MXFP8 on
    the tcgen05 block-scaled kernel, against the bf16 kernel with the same epilogue and cuBLASLt's MXFP8 GEMM
    (torch._scaled_mm with the same e4m3 operands and E8M0 scale blocks, plain bf16 output), plus the quantizer."""
    from nano_gpic_b200.ops import gemm, mx
    M = batch * 256
    pk, _, src = peaks()
    r = lambda *s: (torch.randn(*s, device="cuda") * 0.5).bfloat16()
    res, mod = r(M, d), r(batch, 6 * d)
    cases = [("qkv_x", M, 3 * d, d, "lin"), ("proj", M, d, d, "gated"), ("w12", M, 8 * d, d, "swiglu"),
             ("w3", M, d, 4 * d, "gated")]
    for name, m, n, k, kind in cases:
        x, w = r(m, k), r(n, k)
        xq, wq = mx.quant(x), mx.quant(w)
        if kind == "lin":
            fb, fm = (lambda: gemm.linear(x, w)), (lambda: mx.linear(xq, wq))
        elif kind == "gated":
            g = mod[:, 2 * d:2 * d + n] if n == d else mod[:, :n]
            fb = lambda: gemm.linear_gated_residual(x, w, None, res, g, 256)
            fm = lambda: mx.linear_gated_residual(xq, wq, None, res, g, 256)
        else:
            fb, fm = (lambda: gemm.swiglu_linear(x, w)), (lambda: mx.swiglu_linear(xq, wq))
        fl = 2.0 * m * n * k
        tb, tm, tq = time_fn(fb), time_fn(fm), time_fn(lambda: mx.quant(x))
        row = {"kernel": "gemm_mxfp8", "name": name, "M": m, "N": n, "K": k, "epilogue": kind,
               "mx_us": round(tm * 1e6, 1), "bf16_us": round(tb * 1e6, 1), "quant_us": round(tq * 1e6, 1),
               "mx_tflops": round(fl / tm / 1e12, 1), "bf16_tflops": round(fl / tb / 1e12, 1),
               "mx_frac_of_" + src + "_bf16": round(fl / tm / 1e12 / pk, 3)}
        try:
            e8 = torch.float8_e8m0fnu
            a8, b8 = xq.q.view(torch.float8_e4m3fn), wq.q.view(torch.float8_e4m3fn)
            sa, sb = xq.sf.view(e8).flatten(), wq.sf.view(e8).flatten()
            tc = time_fn(lambda: torch._scaled_mm(a8, b8.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16))
            row["cublaslt_mx_us"] = round(tc * 1e6, 1)
            row["cublaslt_mx_tflops"] = round(fl / tc / 1e12, 1)
        except Exception as e:  # torch build without the MX path
            row["cublaslt_mx"] = f"unavailable: {type(e).__name__}: {str(e)[:120]}"
        rows.append(row)
        print(json.dumps(row), flush=True)


def bench_sample(d, batch, rows, steps=50, pred_batch=8):
    """Euler sampling (the predict path) at a small batch with classifier-free guidance: the denoiser's forward run
    eagerly and replayed from a CUDA graph (runtime/graphs.py). Reports images/s and ms per sampling step."""
    from nano_gpic_b200.config.ladder import SIZES
    from nano_gpic_b200.diffusion.sampling import EulerSamplerJiT
    from nano_gpic_b200.models.jit_t2i import JiT_T2I
    from nano_gpic_b200.runtime.graphs import GraphedCall
    size = next((k for k, v in SIZES.items() if v.width == d), "d12")
    s = SIZES[size]
    torch.manual_seed(0)
    net = JiT_T2I(input_size=256, in_channels=3, num_groups=d // 64, hidden_size=d, num_blocks=s.image_layers,
                  num_text_blocks=s.text_layers, patch_size=16, txt_embed_dim=2048, txt_max_length=320,
                  bottleneck_dim=128).cuda().eval()
    B, T = pred_batch, 128
    x = torch.randn(B, 3, 256, 256, device="cuda")
    y = torch.randn(B, T, 2048, device="cuda").bfloat16()
    m = torch.arange(T, device="cuda")[None] < torch.randint(16, T + 1, (B, 1), device="cuda")
    null = torch.zeros_like(m)
    null[:, 0] = True
    sampler = EulerSamplerJiT(num_steps=steps, guidance=2.0)
    row = {"kernel": "sample", "model": size, "batch": B, "steps": steps, "cfg": 2.0}
    for name, call in (("eager", lambda a, b_, c, e: net(a, b_, c, y_mask=e)),
                       ("graph", GraphedCall(lambda a, b_, c, e: net(a, b_, c, y_mask=e)))):
        f = lambda a, b_, c: call(a, b_, c, torch.cat([null, m]) if c.shape[0] == 2 * B else m)
        t = time_fn(lambda: sampler(f, x, y, torch.zeros_like(y)), iters=3, warmup=1)
        row[name + "_img_s"] = round(B / t, 2)
        row[name + "_ms_per_step"] = round(t / steps * 1e3, 3)
    rows.append(row)
    print(json.dumps(row), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm")
    ap.add_argument("--d", type=int, default=1024)
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    rows = []
    only = set(a.only.split(","))
    if "gemm" in only:
        bench_gemm(a.d, a.batch, rows)
    if "fused" in only:
        bench_fused(a.d, a.batch, rows)
    if "attn" in only:
        bench_attn(a.d, a.batch, rows)
    if "mx" in only:
        bench_mx(a.d, a.batch, rows)
    if "sample" in only:
        bench_sample(a.d, a.batch, rows)
    if a.json:
        with open(a.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
