"""CPU checks of the maintainer's patch on the installed
reference (``baseline/_ref``): it applies to the unmodified ``core/attention.py``, keeps
the gather path's seven-parameter signature, keeps the unknown-value ``ValueError``, and
``ATTENTION=cuda`` on a machine without a GPU raises ``NotImplementedError`` naming the
reason instead of falling back to the gather path (the rule the reference sets for its
Triton path, tests/test_paged_attention_triton.py:151-161)."""

from __future__ import annotations

import inspect

import pytest
import torch

import _reference


@pytest.fixture(scope="module")
def patched_attention(tmp_path_factory, pkg):
    _reference.require()
    dest = _reference.make_patched_copy(tmp_path_factory.mktemp("ref_cpu"))
    mod = _reference.import_patched(dest)
    import importlib

    return importlib.import_module(f"{mod.__name__}.core.attention"), importlib.import_module(f"{mod.__name__}.config")


def _case():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(5, 3, 8, generator=g)
    pool = torch.randn(8, 4, 3, 8, generator=g)
    return q, pool, pool.clone(), torch.tensor([[3, 1]]), torch.tensor([5]), torch.tensor([5])


def test_patch_keeps_the_signature(patched_attention, pkg):
    attention, _ = patched_attention
    params = list(inspect.signature(attention.paged_attention).parameters)
    assert params == list(inspect.signature(attention.paged_attention_gather).parameters)
    assert params == list(inspect.signature(pkg.paged_attention_cuda).parameters)


def test_gather_value_is_unchanged(patched_attention, monkeypatch):
    attention, config = patched_attention
    monkeypatch.setattr(config.CONFIG, "attention", "gather")
    args = _case()
    torch.testing.assert_close(attention.paged_attention(*args, 0.5), attention.paged_attention_gather(*args, 0.5))


def test_cuda_value_without_a_gpu_fails_loudly(patched_attention, monkeypatch):
    attention, config = patched_attention
    monkeypatch.setattr(config.CONFIG, "attention", "cuda")
    with pytest.raises(NotImplementedError, match="ATTENTION=cuda"):
        attention.paged_attention(*_case(), 0.5)


def test_unknown_value_still_rejected(patched_attention, monkeypatch):
    attention, config = patched_attention
    monkeypatch.setattr(config.CONFIG, "attention", "cuda-graphs")
    with pytest.raises(ValueError, match="ATTENTION"):
        attention.paged_attention(*_case(), 0.5)

