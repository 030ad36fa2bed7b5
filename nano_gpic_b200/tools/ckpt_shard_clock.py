"""Prints a checkpoint's data-shard clock as `time seed step` ("-" for a missing seed), for the launch script's shard
log filtering (reference tools/ckpt_shard_clock.py:1-20).

    python -m nano_gpic_b200.tools.ckpt_shard_clock RUN/last.ckpt
"""
import sys

from ..train.checkpoint import read_shard_clock


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    clock = read_shard_clock(argv[0]) or {}
    seed = clock.get("seed")
    print(f"{clock.get('time', 0)} {seed if seed not in (None, '') else '-'} {clock.get('step', 0)}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
