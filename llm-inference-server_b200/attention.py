"""The attention seam, ``ATTENTION=cuda``: same call signature as the reference's gather
path (inference_server/core/attention.py:73-88, 92-100), backed by the sm_100a kernels.

    paged_attention_cuda(query, k_pool, v_pool, block_tables, context_lens, query_lens, scale)

Contract (inference_server/core/attention.py:19-58): query ``[T, Hq, D]`` with any
strides, pools ``[NB, BS, Hkv, D]``, ``block_tables [B, W]`` 0-padded, ``context_lens``
counting this pass's tokens, ``sum(query_lens) == T``; token t of sequence i attends to
keys ``0 .. ctx_i - q_i + t``; returns a fresh ``[T, Hq, D]`` in the query's dtype.

Failure is loud: a non-CUDA tensor or a missing library raises ``NotImplementedError``
naming the reason; contract violations raise ``ValueError`` with the reference's texts.
There is no CPU fallback.
"""

from __future__ import annotations

import os

import torch

from . import _lib
from .metadata import StepMetadata, attached, prefill_tile_tokens, sm_count

_DTYPE_CODE = {torch.float32: _lib.PA_DTYPE_F32, torch.float16: _lib.PA_DTYPE_F16,
               torch.bfloat16: _lib.PA_DTYPE_BF16}

_WORKSPACE: dict[int, torch.Tensor] = {}


def attention_mode() -> str:
    """The ``ATTENTION`` setting, read per call like the reference's dispatcher."""
    return os.environ.get("ATTENTION", "cuda")


def paged_attention(query, k_pool, v_pool, block_tables, context_lens, query_lens, scale):
    """Dispatcher in the shape of inference_server/core/attention.py:73-88.  This package
    supplies the ``cuda`` value; any other value is rejected with the reference's
    message shape (the reference's own dispatcher keeps ``gather`` and ``triton``)."""
    mode = attention_mode()
    if mode == "cuda":
        return paged_attention_cuda(query, k_pool, v_pool, block_tables, context_lens, query_lens, scale)
    raise ValueError(f"unknown ATTENTION={mode!r}; expected 'cuda'")


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Grow-only per-device workspace (split-K partials and the device error word)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WORKSPACE.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACE[idx] = ws
    return ws


def read_device_error(device=None, clear: bool = True) -> int:
    """The device error word of ``device``'s workspace (0 = no kernel reported a
    problem).  Synchronises the current stream."""
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WORKSPACE.get(idx)
    if ws is None:
        return 0
    word = _lib.ctypes.c_int32(0)
    _lib.check(_lib.lib().pa_read_device_error(ws.data_ptr(), int(clear), _lib.ctypes.byref(word),
                                               torch.cuda.current_stream(device).cuda_stream))
    return int(word.value)


def _check_tensors(query, k_pool, v_pool) -> None:
    """Shape checks of attention.py:205-208 plus what the kernels need."""
    if query.dim() != 3:
        raise ValueError(f"query must be [num_tokens, heads, dim], got {tuple(query.shape)}")
    if k_pool.dim() != 4:
        raise ValueError(f"k_pool must be [blocks, block_size, kv_heads, dim], got {tuple(k_pool.shape)}")
    if k_pool.shape != v_pool.shape:
        raise ValueError(f"k_pool {tuple(k_pool.shape)} and v_pool {tuple(v_pool.shape)} differ")
    if query.device.type != "cuda":
        raise NotImplementedError(
            f"ATTENTION=cuda: the sm_100a kernels need a CUDA device, got {query.device}. "
            "There is no CPU fallback.")
    for name, t in (("k_pool", k_pool), ("v_pool", v_pool)):
        if t.device != query.device:
            raise ValueError(f"{name} is on {t.device}, query is on {query.device}")
        if t.dtype != query.dtype:
            raise ValueError(f"{name} is {t.dtype}, query is {query.dtype}")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous [blocks, block_size, kv_heads, dim]")
    if query.dtype not in _DTYPE_CODE:
        raise NotImplementedError(f"ATTENTION=cuda: dtype {query.dtype} is not float32, float16 or bfloat16")
    heads, kv_heads = query.shape[1], k_pool.shape[2]
    if query.shape[2] != k_pool.shape[3]:
        raise ValueError(f"query head_dim {query.shape[2]} != pool head_dim {k_pool.shape[3]}")
    if heads % kv_heads:
        raise ValueError(f"{heads} query heads not divisible by {kv_heads} kv heads")


def step_metadata_for(query, k_pool, block_tables, context_lens, query_lens) -> StepMetadata:
    """The step's planned metadata: the one the executor attached to ``block_tables`` if it
    matches, else planned here from host copies of the arguments (one device->host
    synchronisation, as the reference's per-call ``_check`` costs)."""
    num_blocks, block_size, kv_heads = k_pool.shape[0], k_pool.shape[1], k_pool.shape[2]
    meta = attached(block_tables) if isinstance(block_tables, torch.Tensor) else None
    if meta is not None and meta.matches(query.shape[0], block_size, num_blocks) and meta.device_buffer is not None:
        return meta
    return StepMetadata.build(context_lens, query_lens, block_tables, num_tokens=query.shape[0],
                              pool_num_blocks=num_blocks, block_size=block_size, num_kv_heads=kv_heads,
                              device=query.device,
                              prefill_tile_tokens=prefill_tile_tokens(query.shape[1], kv_heads, query.shape[2]))


def paged_attention_cuda(query, k_pool, v_pool, block_tables, context_lens, query_lens, scale):
    """Causal paged attention on the sm_100a kernels; drop-in for
    ``paged_attention_gather`` (inference_server/core/attention.py:92-187)."""
    _check_tensors(query, k_pool, v_pool)
    lib = _lib.lib()
    meta = step_metadata_for(query, k_pool, block_tables, context_lens, query_lens)
    num_tokens, num_heads, head_dim = query.shape
    num_blocks, block_size, kv_heads, _ = k_pool.shape
    out = torch.empty((num_tokens, num_heads, head_dim), dtype=query.dtype, device=query.device)
    if num_tokens == 0:
        return out
    plan = meta.plan
    ws_bytes = int(lib.pa_workspace_bytes(_lib.ctypes.byref(plan), num_heads, head_dim))
    ws = _workspace(query.device, ws_bytes)
    stream = torch.cuda.current_stream(query.device).cuda_stream
    rc = lib.pa_paged_attention_fwd(
        query.data_ptr(), query.stride(0), query.stride(1), query.stride(2), num_tokens, num_heads, head_dim,
        k_pool.data_ptr(), v_pool.data_ptr(), num_blocks, block_size, kv_heads, _DTYPE_CODE[query.dtype],
        float(scale), _lib.ctypes.byref(plan), meta.device_buffer.data_ptr(), out.data_ptr(), out.stride(0),
        out.stride(1), ws.data_ptr(), ws.numel(), stream)
    _lib.check(rc)
    return out
