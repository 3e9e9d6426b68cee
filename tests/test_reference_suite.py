"""The reference's own CPU test suite, run against this repository's packages.

The reference's tests import ``genesis.*`` and ``olympus.*`` by name; a child
interpreter puts this repository first on ``sys.path`` (and checks that the
imports resolve here), then runs the reference's ``tests/`` directory with
``-m "not gpu"``.  Every test must pass: the public and the test-visible
private API of the reference is reproduced.  The reference's source tree is
read from ``LRB_REFERENCE_DIR`` (its ``tests/`` directory is not part of the
installed package); skipped when that variable is unset or has no tests.
"""

from __future__ import annotations

import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE_TESTS = os.path.join(os.environ.get("LRB_REFERENCE_DIR", os.path.join(REPO, "baseline", "_ref")), "tests")

_RUNNER = r"""
import sys
repo, tests = sys.argv[1], sys.argv[2]
sys.path.insert(0, repo)
import genesis, olympus
assert genesis.__file__.startswith(repo), genesis.__file__
assert olympus.__file__.startswith(repo), olympus.__file__
import pytest
sys.exit(pytest.main([tests, "-q", "-p", "no:cacheprovider", "--import-mode=importlib", "-m", "not gpu",
                      "--timeout=300", "-W", "ignore"]))
"""


@pytest.mark.skipif(not os.path.isdir(REFERENCE_TESTS), reason="reference sources not present")
def test_reference_suite_passes_on_this_framework(tmp_path):
    proc = subprocess.run([sys.executable, "-c", _RUNNER, REPO, REFERENCE_TESTS], cwd=str(tmp_path),
                          capture_output=True, text=True, timeout=900)
    tail = "\n".join((proc.stdout + proc.stderr).splitlines()[-30:])
    assert proc.returncode == 0, tail
    assert " passed" in tail and "failed" not in tail, tail
