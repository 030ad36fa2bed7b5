"""Dataset download and pre-publication scan tools on CPU (no network): the lite / full file lists of the reference's
tools/download_lite.py and download_full.py, retries with a growing wait and the failure report with a stand-in fetch;
the secret scan over every blob of a temporary git repository, history included."""
import os
import subprocess

from nano_gpic_b200.tools import download as D
from nano_gpic_b200.tools import secret_scan as S


def test_file_lists():
    lite = D.lite_files()
    assert lite[:3] == ["gpic_test_50k.jsonl", "gpic_val_50k.jsonl", "README.md"]  # small files first
    assert "train/gpic_train_00000.tar" in lite and "train/gpic_train_00800.tar" in lite
    assert "train/gpic_train_00801.tar" not in lite and "val/gpic_val_00031.tar" in lite
    assert len(lite) == 6 + 801 + 32
    full = D.full_files(801, 805)
    assert full == ["reference_stats/full_stats.npz"] + [f"train/gpic_train_{i:05d}.tar" for i in range(801, 806)]


def test_retries_and_failures(tmp_path):
    calls, waits = {}, []

    def fetch_factory(repo, out):
        def fetch(name):
            calls[name] = calls.get(name, 0) + 1
            if name.endswith("00001.tar") and calls[name] < 3:
                raise OSError("connection reset")
            if name.endswith("00002.tar"):
                raise OSError("gone")
            open(os.path.join(out, name.replace("/", "_")), "w").write("x")
            return name
        return fetch

    fetch = D.with_retries(fetch_factory("r", str(tmp_path)), tries=4, first_wait=1.0, max_wait=3.0,
                           sleep=waits.append, log=lambda m: None)
    failed = D.download(D.full_files(0, 3)[1:], fetch, workers=2, log=lambda m: None)
    assert failed == ["train/gpic_train_00002.tar"]
    assert calls["train/gpic_train_00001.tar"] == 3 and calls["train/gpic_train_00002.tar"] == 4
    assert sorted(waits) == [1.0, 1.0, 2.0, 2.0, 3.0]  # 00001: 1, 2; 00002: 1, 2, 3 (capped)
    rc = D.main(["full", str(tmp_path / "o"), "--first", "0", "--last", "1", "--workers", "1", "--tries", "3"],
                fetch_factory=lambda repo, out: (lambda name: name))
    assert rc == 0


def _git(repo, *args):
    subprocess.run(["git", "-C", str(repo), *args], check=True, capture_output=True,
                   env=dict(os.environ, GIT_AUTHOR_NAME="t", GIT_AUTHOR_EMAIL="t@example.org",
                            GIT_COMMITTER_NAME="t", GIT_COMMITTER_EMAIL="t@example.org"))


def test_secret_scan_sees_history(tmp_path):
    repo = tmp_path / "r"
    repo.mkdir()
    _git(repo, "init", "-q")
    (repo / "a.py").write_text("token = 'hf_" + "A" * 34 + "'\nprint('hi')\n")
    (repo / "b.bin").write_bytes(b"\x00\x01hf_" + b"B" * 34)
    _git(repo, "add", "-A")
    _git(repo, "commit", "-qm", "one")
    (repo / "a.py").write_text("print('clean')\nroot = '/scratch/cluster9/me'\n")  # the token is gone from HEAD
    _git(repo, "add", "-A")
    _git(repo, "commit", "-qm", "two")
    hits, n = S.scan(str(repo), forbid=[r"cluster9"])
    assert n >= 3
    assert any("a.py" in h for h in hits["hf_token"])  # found in the first commit's blob
    assert not any("b.bin" in h for v in hits.values() for h in v)  # binary blobs are skipped
    assert hits["forbidden_0"] and all("..." in h for v in hits.values() for h in v)  # masked
    assert S.main([str(repo)]) == 1
    clean = tmp_path / "c"
    clean.mkdir()
    _git(clean, "init", "-q")
    (clean / "x.txt").write_text("nothing to see\n")
    _git(clean, "add", "-A")
    _git(clean, "commit", "-qm", "c")
    assert S.scan(str(clean))[0] == {} and S.main([str(clean)]) == 0
