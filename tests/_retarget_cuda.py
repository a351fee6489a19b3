"""pytest plugin that runs the reference's own attention tests against ``ATTENTION=cuda``.

Loaded with ``-p _retarget_cuda`` by ``test_gpu_reference_suite.py`` when it runs, in a
child process, the reference's ``tests/test_paged_attention.py`` and
``tests/test_paged_attention_triton.py`` (unchanged copies from ``baseline/_ref``) over
the reference package with the INTEGRATION.md dispatcher patch applied.  Nothing in the
test files is edited; two module globals are redirected for the duration of each test:

* ``test_paged_attention.paged_attention_gather`` — the function under test there, always
  called with CPU tensors — becomes: copy the inputs to ``cuda``, call the patched
  dispatcher ``inference_server.core.attention.paged_attention`` with
  ``CONFIG.attention == "cuda"``, copy the output back.  The dense reference those tests
  compare with is computed inside the test file and is not redirected.
* ``test_paged_attention_triton.paged_attention_triton`` — the CUDA tier's function under
  test — becomes ``paged_attention_cuda``; the gather path it is compared with is left
  alone.

Every redirected call is counted; the count and the kernels the library launched are
written to ``$PA_RETARGET_REPORT`` at the end, so the parent test can check the CUDA path
really ran.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import pytest
import torch

_ROOT = Path(__file__).resolve().parents[1]
if str(_ROOT) not in sys.path:
    sys.path.insert(0, str(_ROOT))

from __graft_entry__ import import_package  # noqa: E402

_pkg = import_package()
_STATS = {"cuda_calls": 0, "launch_bits": 0, "tests_redirected": 0}


def _note_call():
    _STATS["cuda_calls"] += 1
    _STATS["launch_bits"] |= int(_pkg._lib.lib().pa_last_launches())


def _via_dispatcher(query, k_pool, v_pool, block_tables, context_lens, query_lens, scale):
    from inference_server.config import CONFIG
    from inference_server.core.attention import paged_attention

    assert CONFIG.attention == "cuda", CONFIG.attention
    dev = torch.device("cuda")
    args = [t.to(dev) for t in (query, k_pool, v_pool, block_tables, context_lens, query_lens)]
    out = paged_attention(*args, scale)
    _note_call()
    return out.to(query.device)


def _direct(query, k_pool, v_pool, block_tables, context_lens, query_lens, scale):
    out = _pkg.paged_attention_cuda(query, k_pool, v_pool, block_tables, context_lens, query_lens, scale)
    _note_call()
    return out


@pytest.fixture(autouse=True)
def _retarget_to_cuda(request, monkeypatch):
    mod = request.module
    name = mod.__name__.rsplit(".", 1)[-1]
    if name == "test_paged_attention":
        monkeypatch.setattr(mod, "paged_attention_gather", _via_dispatcher)
        _STATS["tests_redirected"] += 1
    elif name == "test_paged_attention_triton":
        monkeypatch.setattr(mod, "paged_attention_triton", _direct)
        _STATS["tests_redirected"] += 1
    yield


def pytest_sessionfinish(session, exitstatus):
    path = os.environ.get("PA_RETARGET_REPORT")
    if path:
        Path(path).write_text(json.dumps({**_STATS, "exitstatus": int(exitstatus),
                                          "testscollected": session.testscollected,
                                          "testsfailed": session.testsfailed}))
