"""GPU health gate: every visible GPU runs a bf16 GEMM loop at the same time (shared load, as in a data-parallel job),
then each GPU's throughput, SM clock and throttle reasons are compared (reference tools/gpu_health.py:1-123).
A GPU below --min-frac of the median throughput, or with a thermal / hardware slowdown reason active under load, fails
the gate: exit 1, and with --verdict FILE a line "FAIL ..." (main.py then exits 98); otherwise "OK ...".

    python -m nano_gpic_b200.tools.gpu_health [--seconds 8] [--min-frac 0.85] [--verdict FILE]

The GEMM is this package's tcgen05 kernel (nano_gpic_b200.ops.gemm.linear), 8192^3 bf16. Clocks and reasons are READ
through NVML (pynvml); nothing is changed on the GPU.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

# NVML clock-event reason bits that mean the GPU is not healthy under load
BAD_REASONS = {0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake"}


def sample_nvml(index, nvml=None):
    """(sm clock MHz, temperature C, clock-event reasons bitmask) of GPU `index`, read through NVML."""
    if nvml is None:
        import pynvml as nvml
        nvml.nvmlInit()
    h = nvml.nvmlDeviceGetHandleByIndex(index)
    clock = nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM)
    temp = nvml.nvmlDeviceGetTemperature(h, nvml.NVML_TEMPERATURE_GPU)
    reasons = nvml.nvmlDeviceGetCurrentClocksEventReasons(h)
    return clock, temp, reasons


def worker(seconds, index, nvml=None):
    import torch
    from nano_gpic_b200.ops import gemm as G
    n = 8192
    a = torch.randn(n, n, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(n, n, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(n, n, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        G.linear(a, b, out=out)
    torch.cuda.synchronize()
    t0, iters, samples = time.time(), 0, []
    while time.time() - t0 < seconds:
        for _ in range(20):
            G.linear(a, b, out=out)
        torch.cuda.synchronize()
        iters += 20
        if time.time() - t0 > seconds / 2:  # under load, after the warm-up half
            samples.append(sample_nvml(index, nvml))
    dt = time.time() - t0
    reasons = 0
    for s in samples:
        reasons |= s[2]
    return {"tflops": 2 * n ** 3 * iters / dt / 1e12,
            "clock": statistics.median(s[0] for s in samples) if samples else 0,
            "temp": max(s[1] for s in samples) if samples else 0, "reasons": reasons}


def judge(results, min_frac=0.85):
    """results {gpu: {tflops, clock, temp, reasons} | {error}} -> (ok, lines, bad gpus). A worker error says nothing
    about the hardware: the gate fails without naming a bad GPU."""
    errors = {g: r["error"] for g, r in results.items() if "error" in r}
    if errors:
        return False, [f"GPU {g}: worker failed: {e}" for g, e in errors.items()] + ["check failed, node unknown"], []
    med = statistics.median(r["tflops"] for r in results.values())
    lines, bad = [], []
    for g, r in sorted(results.items()):
        flags = [name for bit, name in BAD_REASONS.items() if r["reasons"] & bit]
        slow = r["tflops"] < min_frac * med
        lines.append(f"GPU {g}: {r['tflops']:.0f} TFLOP/s, {r['clock']:.0f} MHz, {r['temp']} C, reasons "
                     f"0x{r['reasons']:x} {' '.join(flags)}{'  SLOW' if slow else ''}")
        if slow or flags:
            bad.append(g)
    lines.append(f"median {med:.0f} TFLOP/s; " + (f"UNHEALTHY GPUs {','.join(map(str, bad))}" if bad else "healthy"))
    return not bad, lines, bad


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--seconds", type=float, default=8)
    ap.add_argument("--min-frac", type=float, default=0.85)
    ap.add_argument("--verdict", default=None)
    ap.add_argument("--worker", type=int, default=None)
    a = ap.parse_args(argv)
    if a.worker is not None:
        print(json.dumps(worker(a.seconds, a.worker)), flush=True)
        return 0
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        gpus = [int(x) for x in vis.split(",") if x.strip()]
    else:
        import pynvml
        pynvml.nvmlInit()
        gpus = list(range(pynvml.nvmlDeviceGetCount()))
    procs = {}
    for g in gpus:
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(g))
        procs[g] = subprocess.Popen([sys.executable, "-m", "nano_gpic_b200.tools.gpu_health", "--worker", str(g),
                                     "--seconds", str(a.seconds)], env=env, stdout=subprocess.PIPE,
                                    stderr=subprocess.PIPE, text=True)
    res = {}
    for g, p in procs.items():
        out, err = p.communicate()
        try:
            res[g] = json.loads(out.strip().splitlines()[-1])
        except Exception:
            res[g] = {"error": (err or out)[-400:]}
    ok, lines, _ = judge(res, a.min_frac)
    for ln in lines:
        print(ln, flush=True)
    if a.verdict:
        with open(a.verdict + ".tmp", "w") as f:
            f.write(("OK " if ok else "FAIL ") + lines[-1] + "\n")
        os.replace(a.verdict + ".tmp", a.verdict)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
