"""Fused KV append into the block-major pool (replaces the two ``index_copy_`` calls of
inference_server/core/paged_executor.py:116-125), and pool allocation in the
reference's layout (inference_server/core/kv_pool.py:106-125)."""

from __future__ import annotations

import torch

from . import _lib
from .attention import _DTYPE_CODE


def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                      slot_mapping: torch.Tensor) -> None:
    """Write ``key``/``value`` ``[T, Hkv, D]`` (unit stride along D, any other strides)
    into both pools at flat slots ``slot_mapping [T]`` (``block * block_size + offset``).
    One kernel launch for K and V together; the pool bytes after the call equal the
    reference's ``pool.view(-1, Hkv, D).index_copy_(0, slots, k)``."""
    if key.device.type != "cuda":
        raise NotImplementedError(f"ATTENTION=cuda: the KV append kernel needs a CUDA device, got {key.device}")
    if key.dim() != 3 or value.shape != key.shape:
        raise ValueError(f"key/value must both be [tokens, kv_heads, dim], got {tuple(key.shape)} and "
                         f"{tuple(value.shape)}")
    if k_pool.dim() != 4 or k_pool.shape != v_pool.shape:
        raise ValueError("k_pool and v_pool must both be [blocks, block_size, kv_heads, dim]")
    num_blocks, block_size, kv_heads, dim = k_pool.shape
    if key.shape[1:] != (kv_heads, dim):
        raise ValueError(f"key rows {tuple(key.shape[1:])} do not match the pool's {(kv_heads, dim)}")
    for t in (value, k_pool, v_pool):
        if t.dtype != key.dtype or t.device != key.device:
            raise ValueError("key, value and both pools must share dtype and device")
    if key.dtype not in _DTYPE_CODE:
        raise NotImplementedError(f"ATTENTION=cuda: dtype {key.dtype} is not float32, float16 or bfloat16")
    if key.stride(2) != 1 or value.stride(2) != 1:
        key, value = key.contiguous(), value.contiguous()
    if not (k_pool.is_contiguous() and v_pool.is_contiguous()):
        raise ValueError("pools must be contiguous")
    if slot_mapping.shape != (key.shape[0],):
        raise ValueError(f"slot_mapping must be [{key.shape[0]}], got {tuple(slot_mapping.shape)}")
    if slot_mapping.dtype != torch.int32:
        slot_mapping = slot_mapping.to(torch.int32)
    if slot_mapping.device != key.device:
        slot_mapping = slot_mapping.to(key.device, non_blocking=True)
    slot_mapping = slot_mapping.contiguous()
    _lib.check(_lib.lib().pa_reshape_and_cache(
        key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(), value.stride(0), value.stride(1),
        key.shape[0], kv_heads, dim, _DTYPE_CODE[key.dtype], k_pool.data_ptr(), v_pool.data_ptr(), num_blocks,
        block_size, slot_mapping.data_ptr(), torch.cuda.current_stream(key.device).cuda_stream))


def allocate_pool(num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                  dtype: torch.dtype, device) -> tuple[list[torch.Tensor], list[torch.Tensor]]:
    """Per-layer zero-initialised K and V pools ``[num_blocks, block_size, Hkv, D]``, the
    layout of inference_server/core/kv_pool.py:120-125."""
    shape = (num_blocks, block_size, num_kv_heads, head_dim)
    k = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
    v = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
    return k, v


class KVPool:
    """Per-layer K and V pools in the reference's layout with the attributes its executor
    reads (inference_server/core/kv_pool.py:106-139): ``k``/``v`` lists of
    ``[num_blocks, block_size, Hkv, D]`` zero-initialised tensors, ``num_blocks``,
    ``block_size``."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device) -> None:
        self.num_blocks, self.block_size = num_blocks, block_size
        self.num_kv_heads, self.head_dim, self.dtype = num_kv_heads, head_dim, dtype
        self.k, self.v = allocate_pool(num_layers, num_blocks, block_size, num_kv_heads, head_dim, dtype, device)

    @classmethod
    def from_model(cls, model, num_blocks: int, block_size: int = 16, dtype=None, device=None) -> "KVPool":
        """Sizes read off the model config the way ``ModelDims.from_model`` does
        (kv_pool.py:47-61): ``num_key_value_heads`` when present, else full multi-head."""
        cfg = model.config
        heads = getattr(cfg, "num_attention_heads", None) or cfg.n_head
        hidden = getattr(cfg, "hidden_size", None) or cfg.n_embd
        layers = getattr(cfg, "num_hidden_layers", None) or cfg.n_layer
        kv_heads = getattr(cfg, "num_key_value_heads", None) or heads
        head_dim = getattr(cfg, "head_dim", None) or hidden // heads
        p = next(model.parameters())
        return cls(layers, num_blocks, block_size, kv_heads, head_dim, dtype or p.dtype, device or p.device)

    @property
    def num_slots(self) -> int:
        return self.num_blocks * self.block_size

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)
