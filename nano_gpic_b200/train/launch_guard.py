"""Launch guard: runs one training launch (a torchrun command line) and keeps it from hanging or leaking processes.

    python -m nano_gpic_b200.train.launch_guard --run RUN_DIR [--start-timeout 1500] [--retries 2] [--retry-wait 60]
        [--kill-after 30] -- torchrun ... main.py fit ...

The role of the reference's launch logic in jobs/train_ladder.sh:212-262 (first-step watchdog, killing what a launch
leaves behind) and :356-382 (retries before the first step), as a small state machine of its own:

  * Every process of the launch carries GPIC_LAUNCH_ID=<id> in its environment (ranks, data workers, the checkpoint
    writer inherit it). Whatever the outcome, processes of this user that still carry the id when the launch ends are
    killed, so a failed rank cannot leave a data worker holding a GPU's memory.
  * Start watchdog: until rank 0 writes GPIC_FIRST_STEP_FILE (train.callbacks.FirstStepMarker) the launch must show
    progress within --start-timeout seconds; the clock restarts whenever <file>.progress is touched (the warm-up
    callback touches it after each caption length). When it runs out, the launch's process group gets TERM, then KILL
    after --kill-after seconds, and the launch counts as failed with status 125.
  * Retries: a launch that fails before its first step (the watchdog, a crash, a lost rank) is started again after
    --retry-wait seconds, at most --retries times. Exit status 98 (the GPU-health gate refused the node) is final: a
    retry on the same node would fail the same way. After the first step there are no retries: a failure then is
    the job's to handle (it resumes from the last checkpoint).

Every decision is appended to RUN_DIR/launches.txt. The exit status is the launch's (or 125 for the watchdog).
"""
import argparse
import os
import signal
import subprocess
import sys
import time

WATCHDOG_STATUS = 125
HEALTH_STATUS = 98


def _log(run, msg):
    line = f"{time.strftime('%Y-%m-%dT%H:%M:%SZ', time.gmtime())} launch_guard: {msg}"
    print(line, flush=True)
    if run:
        os.makedirs(run, exist_ok=True)
        with open(os.path.join(run, "launches.txt"), "a") as f:
            f.write(line + "\n")


def processes_with(launch_id, skip=()):
    """PIDs of this user's processes whose environment holds GPIC_LAUNCH_ID=launch_id (read from /proc)."""
    key = f"GPIC_LAUNCH_ID={launch_id}".encode()
    uid, found = os.getuid(), []
    for name in os.listdir("/proc"):
        if not name.isdigit() or int(name) in skip:
            continue
        try:
            if os.stat(f"/proc/{name}").st_uid != uid:
                continue
            with open(f"/proc/{name}/environ", "rb") as f:
                if key in f.read().split(b"\0"):
                    found.append(int(name))
        except OSError:  # ended meanwhile, or not readable
            continue
    return found


def kill_leftovers(launch_id, sig=signal.SIGKILL):
    pids = processes_with(launch_id, skip={os.getpid()})
    for pid in pids:
        try:
            os.kill(pid, sig)
        except OSError:
            pass
    return pids


class Attempt:
    """One start of the command, in its own process group."""

    def __init__(self, cmd, env):
        self.proc = subprocess.Popen(cmd, env=env, start_new_session=True)
        self.started = time.time()

    def signal_group(self, sig):
        try:
            os.killpg(self.proc.pid, sig)
        except OSError:
            pass

    def wait_for(self, seconds):
        try:
            return self.proc.wait(timeout=seconds)
        except subprocess.TimeoutExpired:
            return None


def first_step_seen(marker):
    return bool(marker) and os.path.exists(marker)


def last_progress(marker, since):
    """The later of `since` and the mtime of <marker>.progress."""
    try:
        return max(since, os.path.getmtime(marker + ".progress"))
    except OSError:
        return since


def run_once(cmd, env, run, start_timeout, kill_after, poll=0.5):
    """Runs the command once. Returns (status, started): started tells whether the first step was reached."""
    marker = env.get("GPIC_FIRST_STEP_FILE")
    att = Attempt(cmd, env)
    while True:
        rc = att.wait_for(poll)
        if rc is not None:
            return rc, first_step_seen(marker)
        if start_timeout > 0 and marker and not first_step_seen(marker):
            quiet = time.time() - last_progress(marker, att.started)
            if quiet >= start_timeout:
                _log(run, f"no first step and no progress for {quiet:.0f} s (limit {start_timeout} s): TERM, KILL "
                          f"after {kill_after} s")
                att.signal_group(signal.SIGTERM)
                if att.wait_for(kill_after) is None:
                    att.signal_group(signal.SIGKILL)
                    att.wait_for(10)
                return WATCHDOG_STATUS, False


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if "--" not in argv:
        raise SystemExit("usage: launch_guard [options] -- command ...")
    k = argv.index("--")
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--run", default=None, help="run directory (launches.txt, the first-step marker)")
    ap.add_argument("--start-timeout", type=float, default=float(os.environ.get("GPIC_LAUNCH_START_TIMEOUT_S", 1500)))
    ap.add_argument("--retries", type=int, default=int(os.environ.get("GPIC_LAUNCH_RETRIES", 2)))
    ap.add_argument("--retry-wait", type=float, default=float(os.environ.get("GPIC_LAUNCH_RETRY_WAIT_S", 60)))
    ap.add_argument("--kill-after", type=float, default=float(os.environ.get("GPIC_LAUNCH_WATCHDOG_KILL_S", 30)))
    a = ap.parse_args(argv[:k])
    cmd = argv[k + 1:]
    if not cmd:
        raise SystemExit("launch_guard: no command after --")
    attempt, status = 0, 1
    while True:
        launch_id = f"{os.getpid()}-{time.time_ns()}"
        env = dict(os.environ, GPIC_LAUNCH_ID=launch_id)
        marker = os.path.join(a.run, f"first_step_{launch_id}.txt") if a.run else None
        if marker:
            env["GPIC_FIRST_STEP_FILE"] = marker
        _log(a.run, f"attempt {attempt} id={launch_id} start_timeout={a.start_timeout:g} retries={a.retries}")
        try:
            status, started = run_once(cmd, env, a.run, a.start_timeout, a.kill_after)
        finally:
            left = kill_leftovers(launch_id)
            if left:
                _log(a.run, f"killed {len(left)} leftover process(es) of launch {launch_id}")
        _log(a.run, f"attempt {attempt} ended with status {status}, first step {'reached' if started else 'not reached'}")
        if status == 0 or started or status == HEALTH_STATUS or attempt >= a.retries:
            return status
        attempt += 1
        _log(a.run, f"retrying in {a.retry_wait:g} s")
        time.sleep(a.retry_wait)


if __name__ == "__main__":
    sys.exit(main())
