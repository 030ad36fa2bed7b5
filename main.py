"""Training / prediction entry point with the reference's command line (baselines/PixelGen/main.py):

    python main.py fit --config configs/lite_ladder.yaml --config configs/muon_ladder.yaml [--a.b.c VALUE ...]
    torchrun --nproc-per-node 8 main.py fit ...
    python main.py predict --config configs/lite_ladder_sample.yaml --ckpt_path RUN/ms-step=040192.ckpt
    python main.py fit --config ... --print_config

Exit codes: 0 done; 98 the GPU-health gate failed (GPIC_HEALTH_FILE holds a failing verdict).
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


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "fit":
        _health_gate()
    from nano_gpic_b200.config.cli import main
    sys.exit(main())
