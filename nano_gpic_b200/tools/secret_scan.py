"""Scan every file version reachable from a git repository's refs for credentials and private identifiers before the
repository is published (the role of the reference's tools/pub_scan.py:1-59).

    python -m nano_gpic_b200.tools.secret_scan REPO [REF ...] [--forbid REGEX ...] [--emails]

Every blob reachable from the given refs (all refs when none) is read once through one `git cat-file --batch`
process; binary blobs are skipped. Built-in rules match the published formats of API tokens (Hugging Face, GitHub,
Slack, AWS access keys, OpenAI / Anthropic keys, Google API keys, a W&B key assignment or .netrc entry), PEM private
keys, credentials embedded in URLs and `password = ...`-style assignments; --forbid adds patterns of your own (a
cluster name, user names, internal paths); --emails also reports e-mail addresses. Hits are printed masked (first six
and last four characters) with the file path; the exit status is 1 when anything matched.
"""
import argparse
import collections
import re
import subprocess
import sys
import threading

RULES = {
    "hf_token": r"\bhf_[A-Za-z0-9]{30,}",
    "github_token": r"\b(?:ghp|gho|ghu|ghs|ghr)_[A-Za-z0-9]{30,}|\bgithub_pat_[A-Za-z0-9_]{40,}",
    "slack_token": r"\bxox[abprs]-[A-Za-z0-9-]{10,}",
    "aws_access_key": r"\bAKIA[0-9A-Z]{16}\b",
    "openai_key": r"\bsk-(?:proj-)?[A-Za-z0-9_-]{20,}",
    "anthropic_key": r"\bsk-ant-[A-Za-z0-9_-]{20,}",
    "google_api_key": r"\bAIza[0-9A-Za-z_-]{35}",
    "wandb_key": r"(?i)wandb[_ ]?api[_ ]?key\s*[=:]\s*['\"]?[0-9a-f]{40}|machine\s+api\.wandb\.ai\s+\S+\s+\S+\s+password\s+[0-9a-f]{40}",
    "private_key": r"-----BEGIN (?:[A-Z]+ )?PRIVATE KEY-----",
    "url_credentials": r"[a-z][a-z0-9+.-]*://[^/\s:@'\"]+:[^@\s/'\"]{6,}@",
    "password_assignment": r"(?i)\b(?:password|passwd|secret|api[_-]?key|access[_-]?token|auth[_-]?token)\b\s*[=:]\s*['\"]?[^\s'\"]{8,}",
}
EMAIL = r"\b[A-Za-z0-9._%+-]+@[A-Za-z0-9.-]+\.[A-Za-z]{2,}\b"


def mask(s):
    s = s.replace("\n", " ")
    return s[:6] + "..." + (s[-4:] if len(s) > 12 else "")


def blobs(repo, refs):
    """{sha: first path} of every blob reachable from refs."""
    out = subprocess.run(["git", "-C", repo, "rev-list", "--objects", *(refs or ["--all"])], capture_output=True,
                         text=True, check=True).stdout.splitlines()
    paths = {}
    for line in out:
        sha, _, path = line.partition(" ")
        if path:
            paths.setdefault(sha, path)
    kinds = subprocess.run(["git", "-C", repo, "cat-file", "--batch-check=%(objectname) %(objecttype)"],
                           input="".join(s + "\n" for s in paths), capture_output=True, text=True,
                           check=True).stdout.split()
    return {kinds[i]: paths[kinds[i]] for i in range(0, len(kinds) - 1, 2) if kinds[i + 1] == "blob"}


def read_blobs(repo, shas):
    """Yields (sha, bytes) through one cat-file process; the requests are written by a thread, so neither side of the
    two pipes can fill up and stall the other."""
    proc = subprocess.Popen(["git", "-C", repo, "cat-file", "--batch"], stdin=subprocess.PIPE, stdout=subprocess.PIPE)

    def feed():
        for s in shas:
            proc.stdin.write((s + "\n").encode())
        proc.stdin.close()
    t = threading.Thread(target=feed, daemon=True)
    t.start()
    for sha in shas:
        head = proc.stdout.readline().split()
        size = int(head[2])
        data = proc.stdout.read(size)
        proc.stdout.read(1)
        yield sha, data
    t.join()
    proc.wait()


def scan(repo, refs=(), forbid=(), emails=False):
    """{rule: sorted masked hits 'path :: text'} and the number of blobs read."""
    rules = {k: re.compile(v) for k, v in RULES.items()}
    for i, f in enumerate(forbid):
        rules[f"forbidden_{i}"] = re.compile(f)
    if emails:
        rules["email"] = re.compile(EMAIL)
    paths = blobs(repo, list(refs))
    hits = collections.defaultdict(set)
    n = 0
    for sha, data in read_blobs(repo, list(paths)):
        n += 1
        if b"\x00" in data[:8000]:
            continue
        text = data.decode("utf-8", "replace")
        for name, rx in rules.items():
            for m in rx.finditer(text):
                hits[name].add(f"{paths[sha]} :: {mask(m.group(0))}")
    return {k: sorted(v) for k, v in hits.items()}, n


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("repo")
    ap.add_argument("refs", nargs="*")
    ap.add_argument("--forbid", action="append", default=[], help="an extra pattern that must not appear")
    ap.add_argument("--emails", action="store_true")
    a = ap.parse_args(argv)
    hits, n = scan(a.repo, a.refs, a.forbid, a.emails)
    print(f"{n} blobs scanned")
    for name, hs in sorted(hits.items()):
        print(f"== {name}: {len(hs)}")
        for h in hs[:12]:
            print("   ", h)
    return 1 if hits else 0


if __name__ == "__main__":
    sys.exit(main())
