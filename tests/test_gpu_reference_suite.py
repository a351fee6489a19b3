"""The reference's own attention test-suite, run against ``ATTENTION=cuda`` on the GPU.

The reference package (``baseline/_ref``) is copied to a temporary directory and given the
INTEGRATION.md section 1 dispatcher patch; its unchanged ``tests/test_paged_attention.py``
(all 13 tests, including the dispatcher's unknown-value error and the arity check at
``:192-204``) and ``tests/test_paged_attention_triton.py`` (the CPU mirror tier and the
CUDA tier ``:165-230``, retargeted from the Triton kernel to this library) then run in a
child pytest with ``ATTENTION=cuda`` and the ``_retarget_cuda`` plugin.  The child must
pass every test it collects, and its report must show that the CUDA path served the
redirected calls.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

import _reference

pytestmark = pytest.mark.gpu
TESTS_DIR = Path(__file__).resolve().parent


@pytest.fixture(scope="module")
def patched(tmp_path_factory):
    _reference.require()
    return _reference.make_patched_copy(tmp_path_factory.mktemp("ref_patched"))


def _run_child(patched: Path, files: list[str], tmp_path: Path) -> tuple[subprocess.CompletedProcess, dict]:
    report = tmp_path / "retarget.json"
    env = dict(os.environ)
    env.update(ATTENTION="cuda", DEVICE="cuda", PA_RETARGET_REPORT=str(report),
               PYTHONPATH=os.pathsep.join([str(patched), str(TESTS_DIR), str(TESTS_DIR.parent),
                                           env.get("PYTHONPATH", "")]))
    cmd = [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-p", "_retarget_cuda",
           "-rs", *[str(patched / "reference_tests" / f) for f in files]]
    r = subprocess.run(cmd, cwd=patched / "reference_tests", env=env, capture_output=True, text=True, timeout=600)
    stats = json.loads(report.read_text()) if report.exists() else {}
    return r, stats


def test_reference_paged_attention_suite_on_cuda(patched, tmp_path):
    r, stats = _run_child(patched, ["test_paged_attention.py"], tmp_path)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    # 13 test functions, 27 items with their parametrisations; none skipped.
    assert stats.get("testscollected") == 27 and stats.get("testsfailed") == 0, (stats, r.stdout[-2000:])
    assert " skipped" not in r.stdout.splitlines()[-1], r.stdout[-2000:]
    assert stats["tests_redirected"] == 27
    # Every call that computes attention (25: the padding test runs three seeds, the two
    # contract tests raise before computing) went through the CUDA dispatcher branch.
    assert stats["cuda_calls"] == 25, stats
    assert stats["launch_bits"] != 0, stats


def test_reference_triton_suite_cuda_tier_on_cuda(patched, tmp_path):
    r, stats = _run_child(patched, ["test_paged_attention_triton.py"], tmp_path)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    # The CUDA tier runs here (triton imports and a GPU is present), so only the
    # "fails loudly without triton or CUDA" test is skipped, by the file's own condition.
    last = r.stdout.strip().splitlines()[-1]
    assert stats.get("testsfailed") == 0 and "1 skipped" in last, r.stdout[-3000:]
    assert stats["cuda_calls"] >= 10, stats
    assert stats["launch_bits"] != 0, stats
