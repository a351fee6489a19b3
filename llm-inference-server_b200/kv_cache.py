"""Fused KV append into the block-major pool (replaces the two ``index_copy_`` calls of
inference_server/core/paged_executor.py:116-125), pool allocation in the reference's
layout (inference_server/core/kv_pool.py:106-125), and whole-block moves: copy-on-write
copies (paged_executor.py:265-270) and swap-out / swap-in (kv_pool.py:142-182), each one
kernel launch over every layer."""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

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


def _pool_args(k_pools, v_pools):
    """(ctypes K pointer array, V pointer array, layers, blocks, bytes per block, device)
    after checking every layer has the reference layout."""
    if len(k_pools) != len(v_pools) or not k_pools:
        raise ValueError("need one K and one V pool per layer")
    ref = k_pools[0]
    if ref.dim() != 4:
        raise ValueError("pools must be [blocks, block_size, kv_heads, dim]")
    if ref.device.type != "cuda":
        raise NotImplementedError(f"ATTENTION=cuda: block moves need CUDA pools, got {ref.device}")
    for t in list(k_pools) + list(v_pools):
        if t.shape != ref.shape or t.dtype != ref.dtype or t.device != ref.device or not t.is_contiguous():
            raise ValueError("every layer's K and V pool must be contiguous with the same shape, dtype and device")
    arr = ctypes.c_void_p * len(k_pools)
    kp = arr(*[t.data_ptr() for t in k_pools])
    vp = arr(*[t.data_ptr() for t in v_pools])
    block_bytes = ref[0].numel() * ref.element_size()
    return kp, vp, len(k_pools), ref.shape[0], block_bytes, ref.device


def _block_ids(ids, num_blocks: int, what: str) -> list[int]:
    out = [int(b) for b in ids]
    for b in out:
        if not 0 <= b < num_blocks:
            raise ValueError(f"{what}: block {b} is outside the pool of {num_blocks} blocks")
    return out


def _upload_ids(ids: list[int], device) -> torch.Tensor:
    return torch.tensor(ids, dtype=torch.int32).pin_memory().to(device, non_blocking=True)


def _error_word(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def copy_blocks(k_pools, v_pools, pairs, error_word: torch.Tensor | None = None) -> torch.Tensor:
    """``pool[dst] = pool[src]`` in every layer's K and V pool for each ``(src, dst)``
    pair, one launch (the reference moves one block of one layer per ``copy_``,
    paged_executor.py:265-270).  Destinations must be distinct and none may also be a
    source.  Returns the device error word the kernel reports bad ids in."""
    kp, vp, layers, nb, block_bytes, dev = _pool_args(k_pools, v_pools)
    flat = []
    for src, dst in pairs:
        flat += _block_ids((src, dst), nb, "copy_blocks")
    dsts = flat[1::2]
    if len(set(dsts)) != len(dsts) or set(dsts) & set(flat[0::2]):
        raise ValueError("copy_blocks: destination blocks must be distinct and not also sources")
    err = _error_word(dev) if error_word is None else error_word
    if not flat:
        return err
    ids = _upload_ids(flat, dev)
    _lib.check(_lib.lib().pa_copy_blocks(kp, vp, layers, nb, block_bytes, ids.data_ptr(), len(dsts),
                                         err.data_ptr(), torch.cuda.current_stream(dev).cuda_stream))
    return err


def gather_blocks(k_pools, v_pools, blocks, staging: torch.Tensor, error_word: torch.Tensor) -> None:
    """Copy ``blocks`` of every layer into ``staging`` laid out [layer][K, V][n][block]."""
    kp, vp, layers, nb, block_bytes, dev = _pool_args(k_pools, v_pools)
    ids = _block_ids(blocks, nb, "gather_blocks")
    if staging.numel() * staging.element_size() < layers * 2 * len(ids) * block_bytes:
        raise ValueError("gather_blocks: staging buffer too small")
    if ids:
        _lib.check(_lib.lib().pa_gather_blocks(kp, vp, layers, nb, block_bytes, _upload_ids(ids, dev).data_ptr(),
                                               len(ids), staging.data_ptr(), error_word.data_ptr(),
                                               torch.cuda.current_stream(dev).cuda_stream))


def scatter_blocks(k_pools, v_pools, blocks, staging: torch.Tensor, error_word: torch.Tensor) -> None:
    """Inverse of :func:`gather_blocks`; the blocks must be distinct."""
    kp, vp, layers, nb, block_bytes, dev = _pool_args(k_pools, v_pools)
    ids = _block_ids(blocks, nb, "scatter_blocks")
    if len(set(ids)) != len(ids):
        raise ValueError("scatter_blocks: blocks must be distinct")
    if staging.numel() * staging.element_size() < layers * 2 * len(ids) * block_bytes:
        raise ValueError("scatter_blocks: staging buffer too small")
    if ids:
        _lib.check(_lib.lib().pa_scatter_blocks(kp, vp, layers, nb, block_bytes, _upload_ids(ids, dev).data_ptr(),
                                                len(ids), staging.data_ptr(), error_word.data_ptr(),
                                                torch.cuda.current_stream(dev).cuda_stream))


@dataclass
class HostBlocks:
    """A sequence's blocks parked in host memory while it is swapped out, in the
    reference's form (inference_server/core/kv_pool.py:80-102): per-layer tensors
    ``[n, block_size, Hkv, D]`` for K and for V.  Produced by :meth:`KVPool.swap_out`
    they are views of one pinned buffer (``flat``, [layer][K, V][n][block]), which
    :meth:`KVPool.swap_in` moves back with a single copy."""

    k: list[torch.Tensor]
    v: list[torch.Tensor]
    flat: torch.Tensor | None = field(default=None, repr=False)

    def __len__(self) -> int:
        return int(self.k[0].shape[0]) if self.k else 0

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)


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

    # ------------------------------------------------------------ block moves
    def _staging(self, nbytes: int) -> torch.Tensor:
        buf = getattr(self, "_stage", None)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=self.k[0].device)
            self._stage = buf
        return buf

    def _err(self) -> torch.Tensor:
        if getattr(self, "_err_word", None) is None:
            self._err_word = _error_word(self.k[0].device)
        return self._err_word

    def read_error(self, clear: bool = True) -> int:
        """Error bits block moves reported since the last clear (1 = a bad block id).
        Synchronises the device."""
        word = int(self._err().item())
        if clear and word:
            self._err().zero_()
        return word

    def copy_blocks(self, pairs) -> None:
        """Copy-on-write moves ``pool[dst] = pool[src]`` for every layer, one launch."""
        copy_blocks(self.k, self.v, pairs, self._err())

    def swap_out(self, blocks) -> HostBlocks:
        """Copy the named blocks of every layer to pinned host memory (kv_pool.py:142-166):
        one gather launch into a device staging buffer, one device-to-host copy.  Does
        not free anything; returns when the host copy is complete."""
        n = len(blocks)
        shape = (len(self.k), 2, n) + tuple(self.k[0].shape[1:])
        flat = torch.empty(shape, dtype=self.dtype, pin_memory=True)
        if n:
            block_bytes = self.k[0][0].numel() * self.k[0].element_size()
            stage = self._staging(len(self.k) * 2 * n * block_bytes)
            gather_blocks(self.k, self.v, blocks, stage, self._err())
            flat.copy_(stage[:flat.numel() * flat.element_size()].view(self.dtype).view(shape))
            if self.read_error():
                raise RuntimeError("swap_out: the gather kernel met a block id outside the pool")
        return HostBlocks(k=[flat[l, 0] for l in range(len(self.k))], v=[flat[l, 1] for l in range(len(self.v))],
                          flat=flat)

    def swap_in(self, host: HostBlocks, blocks) -> None:
        """Copy a host copy back into ``blocks``, which need not be the ones it left
        (kv_pool.py:168-182).  Asynchronous on the current stream, like the reference's
        non-blocking copies."""
        if len(blocks) != len(host):
            raise ValueError(f"swap_in: {len(host)} host blocks into {len(blocks)} device blocks")
        n = len(blocks)
        if n == 0:
            return
        shape = (len(self.k), 2, n) + tuple(self.k[0].shape[1:])
        block_bytes = self.k[0][0].numel() * self.k[0].element_size()
        stage = self._staging(len(self.k) * 2 * n * block_bytes)
        view = stage[:len(self.k) * 2 * n * block_bytes].view(self.dtype).view(shape)
        if host.flat is not None and tuple(host.flat.shape) == shape and host.flat.dtype == self.dtype:
            view.copy_(host.flat, non_blocking=True)
        else:
            if len(host.k) != len(self.k) or len(host.v) != len(self.v):
                raise ValueError(f"swap_in: host copy has {len(host.k)} layers, the pool {len(self.k)}")
            for l in range(len(self.k)):
                view[l, 0].copy_(host.k[l], non_blocking=True)
                view[l, 1].copy_(host.v[l], non_blocking=True)
        scatter_blocks(self.k, self.v, blocks, stage, self._err())

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)
