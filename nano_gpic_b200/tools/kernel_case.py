"""Runs one kernel on one shape a few times: the target of ncu captures (small cases that end by themselves).

    python -m nano_gpic_b200.tools.kernel_case --case swiglu_fwd --m 8192 --d 1024 [--reps 3]
cases: linear_fwd, linear_dgrad, linear_wgrad, swiglu_fwd, swiglu_bwd, gated, attn_fwd, attn_bwd, rms_bwd, gate_bwd,
       qk_fwd, qk_bwd (per-head q norm + RoPE of the image rows)
"""
import argparse

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True)
    ap.add_argument("--m", type=int, default=8192, help="token rows (multiple of 256 for attention cases)")
    ap.add_argument("--d", type=int, default=1024)
    ap.add_argument("--t", type=int, default=128, help="caption length (attention cases)")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--impl", default=None, help="attention implementation (tc, tc2, tc1, mma)")
    ap.add_argument("--prof", action="store_true", help="attention backward: print the per-role cycle breakdown of the "
                                                         "profiled kernel instantiation (csrc/attn_tc.cu)")
    ap.add_argument("--time", action="store_true", help="also print the mean time per call (CUDA events, after the "
                                                          "--reps warm-up calls, 20 timed calls)")
    a = ap.parse_args()
    from nano_gpic_b200.ops import attention as A, gemm as G, norm as NR, status
    torch.manual_seed(0)
    M, d = a.m, a.d
    r = lambda *s: (torch.randn(*s, device="cuda") * 0.5).bfloat16()
    if a.case in ("linear_fwd", "linear_dgrad", "linear_wgrad"):
        x, w, dy = r(M, d), r(3 * d, d), r(M, 3 * d)
        fn = {"linear_fwd": lambda: G.linear(x, w), "linear_dgrad": lambda: G.linear_dgrad(dy, w),
              "linear_wgrad": lambda: G.linear_wgrad(dy, x)}[a.case]
    elif a.case == "swiglu_fwd":
        x, w12 = r(M, d), r(8 * d, d)
        fn = lambda: G.swiglu_linear(x, w12)
    elif a.case == "swiglu_bwd":
        dy, w3, pre = r(M, d), r(d, 4 * d), r(M, 8 * d)
        fn = lambda: G.swiglu_dgrad(dy, w3, pre)
    elif a.case == "gated":
        x, w, res, mod = r(M, d), r(d, d), r(M, d), r(M // 256, 6 * d)
        b = torch.zeros(d, device="cuda")
        fn = lambda: G.linear_gated_residual(x, w, b, res, mod[:, 2 * d:3 * d], 256)
    elif a.case in ("attn_fwd", "attn_bwd"):
        B, L, T = M // 256, 256, a.t
        qkv, kv = r(M, 3 * d), r(B * T, 2 * d)
        lens = torch.randint(1, T + 1, (B,), device="cuda", dtype=torch.int32)
        o, lse = A.attn_fwd(qkv[:, :d], L, qkv[:, d:2 * d], qkv[:, 2 * d:], L, L, kv[:, :d], kv[:, d:], T, lens)
        do = r(M, d)
        kw = {"impl": a.impl} if a.impl else {}
        if a.case == "attn_fwd":
            fn = lambda: A.attn_fwd(qkv[:, :d], L, qkv[:, d:2 * d], qkv[:, 2 * d:], L, L, kv[:, :d], kv[:, d:], T, lens,
                                    **kw)
        else:
            fn = lambda: A.attn_bwd(do, qkv[:, :d], L, qkv[:, d:2 * d], qkv[:, 2 * d:], L, L, o, lse, kv[:, :d],
                                    kv[:, d:], T, lens, **kw)
    elif a.case == "rms_bwd":
        x, dh = r(M, d), r(M, d)
        w = torch.ones(d, device="cuda")
        mod = r(M // 256, 6 * d)
        h, rstd = NR.rms_mod_fwd(x, w, mod[:, :d], mod[:, d:2 * d], 256)
        dw = torch.zeros(d, device="cuda")
        fn = lambda: NR.rms_mod_bwd(dh, x, rstd, w, mod[:, d:2 * d], 256, dres=dh, dw_acc=dw,
                                    dshift=dsh[:, :d], dscale=dsh[:, d:])
        dsh = torch.empty(M // 256, 2 * d, device="cuda")
    elif a.case in ("qk_fwd", "qk_bwd"):
        from nano_gpic_b200.models.layers import rope_tables
        from nano_gpic_b200.ops import qk as QK
        L = 256
        cos, sin = rope_tables(64, 16, 16, device="cuda")
        qkv, dq = r(M, 3 * d), r(M, d)
        w = torch.ones(64, device="cuda")
        q, rq = QK.qk_norm_fwd(qkv[:, :d], w, cos, sin, L)
        dsrc = torch.empty(M, d, device="cuda", dtype=torch.bfloat16)
        dw = torch.zeros(64, device="cuda")
        fn = (lambda: QK.qk_norm_fwd(qkv[:, :d], w, cos, sin, L)) if a.case == "qk_fwd" else \
            (lambda: QK.qk_norm_bwd(dq, qkv[:, :d], rq, w, cos, sin, L, dsrc=dsrc, dw_acc=dw))
    elif a.case == "gate_bwd":
        from nano_gpic_b200.ops import elementwise as E
        dout, y, mod = r(M, d), r(M, d), r(M // 256, 6 * d)
        dg = torch.empty(M // 256, d, device="cuda")
        fn = lambda: E.gate_bwd(dout, y, mod[:, 5 * d:], 256, dgate=dg)
    else:
        raise SystemExit(f"unknown case {a.case}")
    for _ in range(a.reps):
        fn()
    torch.cuda.synchronize()
    status.check()
    print(f"{a.case} ok", flush=True)
    if a.prof:
        from nano_gpic_b200._ext import ext
        cnt = torch.zeros(20, dtype=torch.int64, device="cuda")
        ext().attn_prof_set(cnt)
        fn()
        torch.cuda.synchronize()
        ext().attn_prof_set(None)
        c = cnt.tolist()
        names = ["compute: wait S", "compute: load+exp", "compute: wait products", "compute: store P/dS",
                 "compute: wait dK/dV", "compute: dK/dV out", "compute: wait dQ", "compute: dQ out",
                 "compute: total", "mma: wait Q/dO", "mma: wait K/V", "mma: wait S free", "mma: wait P/dS",
                 "mma: wait epilogue", "mma: total", "tma: waits", "compute: wait Q/dO", "compute: item setup",
                 "mma: issue S", "mma: issue products"]
        tot_c, tot_m = max(c[8], 1), max(c[14], 1)
        for i, (n, v) in enumerate(zip(names, c)):
            base = tot_m if 9 <= i <= 15 or i >= 18 else tot_c
            print(f"  {n:26s} {v:16d}  {100.0 * v / base:6.1f} %", flush=True)
    if a.time:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(20):
            fn()
        e.record()
        torch.cuda.synchronize()
        print(f"{a.case} m={M} d={d}: {s.elapsed_time(e) / 20 * 1000:.1f} us per call", flush=True)


if __name__ == "__main__":
    main()
