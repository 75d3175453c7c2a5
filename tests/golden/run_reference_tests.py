"""Runs the reference project's OWN test files for the row-reduction path against this package.

The reference's tests (tests/test_rmsnorm.py, test_layernorm.py, test_softmax.py,
test_cross_entropy.py, test_topk.py, test_linear_cross_entropy.py) import ``quack.*``; with this
repository's root first on ``sys.path`` those imports resolve to the sm_100a implementation, so
the unmodified files act as acceptance tests of the drop-in boundary.  The files are not part of
this repository: point the script at a checkout of the reference (or at a copy of its test files).

    python tests/golden/run_reference_tests.py --tests-dir <reference>/tests [-k EXPR] [--compile]

By default the ``use_compile=True`` parametrisations are deselected (torch.compile of several
hundred shape variants takes tens of minutes and exercises PyTorch, not the kernels); pass
``--compile`` to include them.  Further deselections, each with its reason, are in DESELECT.
Needs a CUDA device.
"""

from __future__ import annotations

import argparse
import sys
import tempfile
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[2]
FILES = ("test_rmsnorm.py", "test_layernorm.py", "test_softmax.py", "test_cross_entropy.py",
         "test_topk.py", "test_linear_cross_entropy.py")

# test id substring -> reason (filled in only for tests that probe internals of the reference's
# JIT cache / autotuner, which do not exist here)
DESELECT = {}


class _Plugin:
    def __init__(self, with_compile: bool):
        self.with_compile = with_compile
        self.deselected = []

    def pytest_collection_modifyitems(self, config, items):
        keep = []
        for it in items:
            reason = next((r for k, r in DESELECT.items() if k in it.nodeid), None)
            if reason is None and not self.with_compile and "use_compile" in getattr(it, "fixturenames", ()):  # noqa: E501
                if it.callspec.params.get("use_compile"):
                    reason = "use_compile=True (pass --compile to include)"
            if reason:
                self.deselected.append((it.nodeid, reason))
            else:
                keep.append(it)
        config.hook.pytest_deselected(items=[it for it in items if it not in keep])
        items[:] = keep


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--tests-dir", required=True, help="directory holding the reference's test files")
    ap.add_argument("-k", default=None)
    ap.add_argument("--compile", action="store_true", help="include the use_compile=True cases")
    ap.add_argument("--files", nargs="*", default=list(FILES))
    args, extra = ap.parse_known_args()
    src = Path(args.tests_dir)
    missing = [f for f in args.files if not (src / f).exists()]
    if missing:
        ap.error(f"not found under {src}: {missing}")
    sys.path.insert(0, str(ROOT))
    # Run from a scratch rootdir so that neither this repository's nor the reference's conftest.py
    # (which starts compile-worker pools for the reference's JIT) is picked up.
    with tempfile.TemporaryDirectory() as tmp:
        links = []
        for f in args.files:
            dst = Path(tmp) / f
            dst.write_bytes((src / f).read_bytes())
            links.append(str(dst))
        plugin = _Plugin(args.compile)
        argv = ["-q", "--rootdir", tmp, "-p", "no:cacheprovider", *links, *extra]
        if args.k:
            argv += ["-k", args.k]
        rc = pytest.main(argv, plugins=[plugin])
    by_reason = {}
    for nodeid, reason in plugin.deselected:
        by_reason.setdefault(reason, []).append(nodeid)
    for reason, ids in by_reason.items():
        print(f"deselected {len(ids)}: {reason}")
    return int(rc)


if __name__ == "__main__":
    sys.exit(main())
