"""The drop-in proper: B200Device registered with the reference's own runtime.

tests/dropin_reference_child.py imports the reference package ``sf`` (an
offline install of it under baseline/_ref, or the directory named by
SF_REFERENCE_SITE), registers B200Device with ``sf.register_device`` and runs
the reference's own array API, ``sf.matmul`` (chain and wide) and its
``torch.compile(backend="superfloat")`` with ``default_device="b200"``, then
compares codes, SFStatus and float outputs with the reference's host path
and its flagged mock target.  It runs as a child process because the
reference and this package both register a TorchDynamo backend named
``superfloat``.  Skipped where the reference is not installed.
"""
import json
import os
import subprocess
import sys

import pytest

from conftest import REPO

CHILD = os.path.join(REPO, "tests", "dropin_reference_child.py")


def _reference_site():
    for d in (os.environ.get("SF_REFERENCE_SITE"), os.path.join(REPO, "baseline", "_ref")):
        if d and os.path.isfile(os.path.join(d, "sf", "__init__.py")):
            return d
    pytest.skip("the reference package is not installed (baseline/_ref or SF_REFERENCE_SITE)")


def _run_child(device, tmp_path):
    env = dict(os.environ, SF_CACHE_DIR=str(tmp_path / "sf_cache"))
    p = subprocess.run([sys.executable, CHILD, _reference_site(), REPO, device], capture_output=True, text=True,
                       timeout=900, env=env, cwd=str(tmp_path))
    assert p.returncode == 0, p.stderr[-3000:]
    return json.loads(p.stdout.strip().splitlines()[-1])


@pytest.mark.gpu
def test_b200_plugged_into_the_reference_runtime(gpu, tmp_path):
    r = _run_child("b200", tmp_path)
    assert r["mismatches"] == [], r["mismatches"]
    assert len(r["checks"]) == 43, r["checks"]          # the flagged mock's 37 plus codes and status of div at 3 widths
    assert r["launches"] > 100                           # every heavy op and converted layer reached the B200


def test_the_child_checks_itself_with_the_references_flagged_mock(tmp_path):
    """No GPU: the same script with the reference's own ``atreides-flags``
    mock as the target (it has no divider, so the div checks drop out)."""
    r = _run_child("atreides-flags", tmp_path)
    assert r["mismatches"] == [] and len(r["checks"]) == 37
