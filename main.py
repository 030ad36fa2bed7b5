"""Training / prediction entry point with the reference's command line (baselines/PixelGen/main.py):

    python main.py fit --config configs/lite_ladder.yaml --config configs/muon_ladder.yaml [--a.b.c VALUE ...]
    torchrun --nproc-per-node 8 main.py fit ...
    python main.py predict --config configs/lite_ladder_sample.yaml --ckpt_path RUN/ms-step=040192.ckpt
    python main.py fit --config ... --print_config

Exit codes: 0 done; 98 the GPU-health gate failed (GPIC_HEALTH_FILE holds a failing verdict); 1 an exception escaped
(fail-fast: the traceback, at most GPIC_FAIL_EXIT_HOOKS_S seconds of exit hooks, then os._exit, never waiting on
peers in torch.distributed's shutdown; GPIC_FAIL_FAST=0 re-raises instead).
"""
import os
import sys


def _health_gate():
    """Before fit: when GPIC_HEALTH_FILE is set, wait (up to GPIC_HEALTH_WAIT_S) for the health check's verdict and
    exit 98 on a failure (reference main.py before_fit, tools/gpu_health.py)."""
    path = os.environ.get("GPIC_HEALTH_FILE")
    if not path:
        return
    import time
    deadline = time.time() + float(os.environ.get("GPIC_HEALTH_WAIT_S", 600))
    while not os.path.exists(path) and time.time() < deadline:
        time.sleep(1)
    if os.path.exists(path):
        with open(path) as f:
            verdict = f.read().strip()
        if verdict.startswith("FAIL"):
            print(f"[main] GPU health: {verdict}; exiting 98", flush=True)
            os._exit(98)


def exit_after_failure(exc, status=1):
    """Fail fast (GPIC_FAIL_FAST=1, the default; the role of reference main.py:128-183): after an exception escapes
    fit, a normal interpreter exit runs torch.distributed's shutdown, which can wait for good on peers that sit in a
    collective. Instead: print the traceback, run the other exit hooks (checkpoint writer, data workers) in a daemon
    thread for at most GPIC_FAIL_EXIT_HOOKS_S (30) seconds, then leave with `status` through os._exit. The launch
    guard (nano_gpic_b200.train.launch_guard) then ends the other ranks of the launch."""
    import atexit
    import threading
    import time
    import traceback
    traceback.print_exception(type(exc), exc, exc.__traceback__)
    sys.stderr.flush()
    limit = float(os.environ.get("GPIC_FAIL_EXIT_HOOKS_S", 30))
    t0 = time.time()
    hooks = threading.Thread(target=atexit._run_exitfuncs, name="exit-hooks", daemon=True)
    hooks.start()
    hooks.join(limit)
    late = " (exit hooks still running)" if hooks.is_alive() else ""
    print(f"[main] {type(exc).__name__}: leaving with status {status} after {time.time() - t0:.1f} s of exit hooks"
          f"{late}", file=sys.stderr, flush=True)
    os._exit(status)


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "fit":
        _health_gate()
    from nano_gpic_b200.config.cli import main
    try:
        rc = main()
    except SystemExit:  # a status chosen on purpose (argument errors, the health gate's 98)
        raise
    except BaseException as e:  # noqa: BLE001 -- every other failure leaves without waiting on peers
        if os.environ.get("GPIC_FAIL_FAST", "1") != "1":
            raise
        exit_after_failure(e)
    sys.exit(rc)
