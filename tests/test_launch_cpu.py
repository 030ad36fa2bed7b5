"""Launch guards on CPU with stub programs instead of training: the first-step watchdog (TERM, then KILL, status 125),
its clock restarting on warm-up progress, retries before the first step only, no retry after the health gate's 98,
leftover processes of a launch killed by launch id, and main.py's fail-fast exit that does not wait for a hung exit
hook (the role of the reference's jobs/train_ladder.sh:212-262,356-382 and PG/main.py:128-183)."""
import os
import subprocess
import sys
import textwrap
import time

from nano_gpic_b200.train import launch_guard as LG

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _stub(tmp_path, name, body):
    p = tmp_path / name
    p.write_text(textwrap.dedent(body))
    return [sys.executable, str(p)]


def _guard(tmp_path, cmd, run="run", **kw):
    args = ["--run", str(tmp_path / run), "--retry-wait", "0.1", "--kill-after", "1"]
    for k, v in kw.items():
        args += [f"--{k.replace('_', '-')}", str(v)]
    t0 = time.time()
    rc = LG.main(args + ["--"] + cmd)
    return rc, time.time() - t0, (tmp_path / run / "launches.txt").read_text()


def test_watchdog_ends_a_launch_without_first_step(tmp_path):
    """A launch that never writes its first step (nor progress) is ended after the start timeout: status 125, and a
    child it left behind (same launch id in its environment) is killed too."""
    pidfile = tmp_path / "child.pid"
    cmd = _stub(tmp_path, "hang.py", f"""
        import subprocess, sys, time
        child = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(600)"], start_new_session=True)
        open({str(pidfile)!r}, "w").write(str(child.pid))
        time.sleep(600)
    """)
    rc, dt, log = _guard(tmp_path, cmd, start_timeout=2, retries=0)
    assert rc == LG.WATCHDOG_STATUS and dt < 30, (rc, dt)
    assert "no first step" in log
    pid = int(pidfile.read_text())
    time.sleep(0.2)
    try:
        os.kill(pid, 0)
        alive = open(f"/proc/{pid}/stat").read().split()[2] != "Z"
    except OSError:
        alive = False
    assert not alive, "the launch's own child (its new session escapes the group) is killed by launch id"


def test_progress_restarts_the_clock(tmp_path):
    """Warm-up progress (touching <first step file>.progress) keeps a slow start alive past the timeout; the first
    step then ends the watchdog's duty."""
    cmd = _stub(tmp_path, "slow.py", """
        import os, time
        m = os.environ["GPIC_FIRST_STEP_FILE"]
        for _ in range(5):
            time.sleep(1.0)
            open(m + ".progress", "a").close(); os.utime(m + ".progress", None)
        open(m, "w").write("1")
        time.sleep(2.5)
    """)
    rc, dt, log = _guard(tmp_path, cmd, start_timeout=2, retries=0)
    assert rc == 0 and dt > 6, (rc, dt, log)
    assert "no first step" not in log


def test_retry_before_the_first_step_only(tmp_path):
    """A crash before the first step is retried (here the second attempt succeeds); a crash after the first step is
    not; the health gate's 98 is final."""
    count = tmp_path / "count"
    cmd = _stub(tmp_path, "flaky.py", f"""
        import os, sys
        p = {str(count)!r}
        n = int(open(p).read()) if os.path.exists(p) else 0
        open(p, "w").write(str(n + 1))
        if n == 0:
            sys.exit(3)
        open(os.environ["GPIC_FIRST_STEP_FILE"], "w").write("1")
    """)
    rc, _, log = _guard(tmp_path, cmd, start_timeout=30, retries=2)
    assert rc == 0 and count.read_text() == "2" and "retrying" in log
    cmd = _stub(tmp_path, "late.py", """
        import os, sys
        open(os.environ["GPIC_FIRST_STEP_FILE"], "w").write("1")
        sys.exit(7)
    """)
    rc, _, log = _guard(tmp_path, cmd, run="late", start_timeout=30, retries=2)
    assert rc == 7 and log.count("attempt 1 ") == 0
    cmd = _stub(tmp_path, "gate.py", "import sys; sys.exit(98)")
    rc, _, log = _guard(tmp_path, cmd, run="gate", start_timeout=30, retries=2)
    assert rc == 98 and "retrying" not in log


def test_fail_fast_does_not_wait_for_hung_exit_hooks(tmp_path):
    """An exception that escapes fit leaves with status 1 after at most GPIC_FAIL_EXIT_HOOKS_S of exit hooks, even
    when a hook would wait for good (as a process-group destroy waiting on absent peers does)."""
    stub = tmp_path / "failing_main.py"
    stub.write_text(textwrap.dedent(f"""
        import atexit, os, sys, time
        sys.path.insert(0, {HERE!r})
        import importlib.util
        spec = importlib.util.spec_from_file_location("ng_main", os.path.join({HERE!r}, "main.py"))
        m = importlib.util.module_from_spec(spec); spec.loader.exec_module(m)
        atexit.register(lambda: time.sleep(600))   # a hook that never returns
        try:
            raise RuntimeError("boom in fit")
        except RuntimeError as e:
            m.exit_after_failure(e)
    """))
    t0 = time.time()
    r = subprocess.run([sys.executable, str(stub)], capture_output=True, text=True, timeout=120,
                       env=dict(os.environ, GPIC_FAIL_EXIT_HOOKS_S="1"))
    assert r.returncode == 1 and time.time() - t0 < 60, (r.returncode, r.stderr[-500:])
    assert "boom in fit" in r.stderr and "leaving with status 1" in r.stderr
