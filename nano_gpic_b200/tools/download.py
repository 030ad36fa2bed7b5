"""Fetch the GPIC dataset files from the Hugging Face hub (the role of the reference's tools/download_lite.py:1-36 and
tools/download_full.py:1-36).

    python -m nano_gpic_b200.tools.download lite OUT_DIR [--workers 8]
    python -m nano_gpic_b200.tools.download full OUT_DIR [--first 801] [--last 7999] [--workers 8]

lite: train shards 0-800, the 32 validation shards, the test / validation prompt files, the README and the reference
statistics of test, val and lite (the small files first, so an evaluation can start before the shards finish). full:
the full set's reference statistics and train shards first..last (the lite shards are 0-800). Needs network access;
every file is fetched by huggingface_hub's hf_hub_download into OUT_DIR under its repository path, which skips files
already complete, so a run that stopped resumes where it was. A failed file is retried with a growing wait; files that
still fail are listed at the end and the exit status is 1.
"""
import argparse
import os
import sys
import time
from concurrent.futures import ThreadPoolExecutor, as_completed

REPO = "stanford-vision-lab/gpic"
LITE_TRAIN_SHARDS = 801
VAL_SHARDS = 32


def lite_files():
    small = ["gpic_test_50k.jsonl", "gpic_val_50k.jsonl", "README.md"] + \
        [f"reference_stats/{w}_stats.npz" for w in ("test", "val", "lite")]
    shards = [f"train/gpic_train_{i:05d}.tar" for i in range(LITE_TRAIN_SHARDS)] + \
        [f"val/gpic_val_{i:05d}.tar" for i in range(VAL_SHARDS)]
    return small + shards


def full_files(first=LITE_TRAIN_SHARDS, last=7999):
    return ["reference_stats/full_stats.npz"] + [f"train/gpic_train_{i:05d}.tar" for i in range(first, last + 1)]


def hub_fetch(repo, out):
    """The network fetch: hf_hub_download of one file of the dataset repo into `out` (imported only when used)."""
    from huggingface_hub import hf_hub_download

    def fetch(name):
        return hf_hub_download(repo, name, repo_type="dataset", local_dir=out)
    return fetch


def with_retries(fetch, tries=6, first_wait=10.0, max_wait=600.0, sleep=time.sleep, log=print):
    """fetch(name) retried up to `tries` times, the wait doubling from first_wait (capped at max_wait)."""
    def run(name):
        wait = first_wait
        for attempt in range(tries):
            try:
                return fetch(name)
            except Exception as e:  # network errors of any kind: retried, then reported
                if attempt == tries - 1:
                    raise
                log(f"retry {name} ({attempt + 1}/{tries - 1}): {type(e).__name__}: {e}")
                sleep(wait)
                wait = min(max_wait, 2 * wait)
    return run


def download(files, fetch, workers=8, log=print):
    """Fetches every file with `workers` threads; returns the names that failed after their retries."""
    t0, done, failed = time.time(), 0, []
    with ThreadPoolExecutor(max(1, workers)) as ex:
        futs = {ex.submit(fetch, f): f for f in files}
        for fu in as_completed(futs):
            done += 1
            try:
                fu.result()
            except Exception as e:
                failed.append(futs[fu])
                log(f"FAILED {futs[fu]}: {type(e).__name__}: {e}")
            if done % 25 == 0 or done == len(files):
                log(f"{done}/{len(files)} files, {time.time() - t0:.0f} s")
    return sorted(failed)


def main(argv=None, fetch_factory=hub_fetch):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("what", choices=["lite", "full"])
    ap.add_argument("out")
    ap.add_argument("--first", type=int, default=LITE_TRAIN_SHARDS)
    ap.add_argument("--last", type=int, default=7999)
    ap.add_argument("--workers", type=int, default=int(os.environ.get("NW", 8)))
    ap.add_argument("--repo", default=REPO)
    ap.add_argument("--tries", type=int, default=6)
    a = ap.parse_args(argv)
    files = lite_files() if a.what == "lite" else full_files(a.first, a.last)
    os.makedirs(a.out, exist_ok=True)
    log = lambda m: print(m, flush=True)
    failed = download(files, with_retries(fetch_factory(a.repo, a.out), tries=a.tries, log=log), a.workers, log)
    log("DONE" if not failed else f"DONE, {len(failed)} failed: {failed[:20]}")
    return 1 if failed else 0


if __name__ == "__main__":
    sys.exit(main())
