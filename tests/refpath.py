"""Locates the reference source tree for oracle tests: baseline/_ref (an unmodified copy of wenhaochai/nano-gpic),
or the directory named by the environment variable NG_REFERENCE_ROOT."""
import contextlib
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def ref_root():
    for c in (os.path.join(ROOT, "baseline", "_ref"), os.environ.get("NG_REFERENCE_ROOT")):
        if not c:
            continue
        if os.path.isdir(os.path.join(c, "baselines", "PixelGen", "src")):
            return c
    return None


@contextlib.contextmanager
def reference_imports():
    """sys.path with the reference's PixelGen directory first (its package is named `src`); restores afterwards."""
    root = ref_root()
    if root is None:
        import pytest
        pytest.skip("reference tree not available")
    pg = os.path.join(root, "baselines", "PixelGen")
    saved = {k: v for k, v in sys.modules.items() if k == "src" or k.startswith("src.")}
    for k in saved:
        del sys.modules[k]
    sys.path.insert(0, pg)
    try:
        yield pg
    finally:
        sys.path.remove(pg)
        for k in [k for k in sys.modules if k == "src" or k.startswith("src.")]:
            del sys.modules[k]
        sys.modules.update(saved)
