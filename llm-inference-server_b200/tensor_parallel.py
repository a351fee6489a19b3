"""KV-head tensor parallelism for the large-GQA configurations (Llama-3-70B shape: 64
query heads, 8 KV heads).

Rank r of a tensor-parallel group of size tp holds KV heads ``[r*Hkv/tp, (r+1)*Hkv/tp)``
and the ``Hq/tp`` query heads that read them, so its KV pool is
``[num_blocks, 16, Hkv/tp, D]`` and every rank shares the same block tables (each rank
runs the same deterministic scheduler on the same requests).  Per layer a rank appends its
heads' new K/V, runs paged attention over its heads, multiplies by its row slice of the
output projection, and one all-reduce (NCCL over NVLink on GPUs) sums the partial
projections.  The reference has no multi-GPU path (its design notes name it a non-goal);
the arithmetic here is the single-device layer's, split by heads.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist


def kv_head_shard(num_heads: int, num_kv_heads: int, rank: int, world: int) -> tuple[slice, slice]:
    """(query-head slice, KV-head slice) owned by ``rank``.  KV heads split evenly; each
    KV head keeps its whole GQA group of query heads on the same rank."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a group of {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads cannot be split across {world} ranks")
    if num_heads % num_kv_heads:
        raise ValueError(f"{num_heads} query heads not divisible by {num_kv_heads} kv heads")
    kv = num_kv_heads // world
    group = num_heads // num_kv_heads
    return slice(rank * kv * group, (rank + 1) * kv * group), slice(rank * kv, (rank + 1) * kv)


def o_proj_shard(weight: torch.Tensor, num_heads: int, head_dim: int, rank: int, world: int,
                 num_kv_heads: int) -> torch.Tensor:
    """Rows of the output projection this rank multiplies, as an ``[in, out]`` matrix.

    ``weight`` is a ``torch.nn.Linear`` weight ``[d_model_out, num_heads * head_dim]``; the
    rank's query heads select a contiguous block of its input columns."""
    qs, _ = kv_head_shard(num_heads, num_kv_heads, rank, world)
    cols = slice(qs.start * head_dim, qs.stop * head_dim)
    return weight[:, cols].t().contiguous()


def _map_peers(buf: torch.Tensor, group, world: int, rank: int, device: torch.device):
    """Export ``buf`` through CUDA IPC (the C ABI's ``pa_ipc_export``) and open every peer's
    buffer on this rank's device.  Returns the ctypes array of all ranks' base pointers
    (this rank's own buffer at ``rank``) and the ``(pointer, offset)`` pairs opened here,
    which ``pa_ipc_close`` releases.  With one rank nothing is mapped."""
    from . import _lib

    torch.cuda.synchronize(device)
    if world == 1:
        return (ctypes.c_void_p * 1)(buf.data_ptr()), []
    lib = _lib.lib()
    handle = ctypes.create_string_buffer(64)
    offset = ctypes.c_int64()
    with torch.cuda.device(device):
        _lib.check(lib.pa_ipc_export(buf.data_ptr(), handle, ctypes.byref(offset)))
        handles = [None] * world
        dist.all_gather_object(handles, (handle.raw, offset.value), group=group)
        ptrs, opened = [], []
        for r, (h, off) in enumerate(handles):
            if r == rank:
                ptrs.append(buf.data_ptr())
                continue
            ptr = ctypes.c_void_p()
            _lib.check(lib.pa_ipc_open(h, off, ctypes.byref(ptr)))  # mapped on this rank's device
            ptrs.append(ptr.value)
            opened.append((ptr.value, off))
    return (ctypes.c_void_p * world)(*ptrs), opened


class PeerAllReduce:
    """In-place sum across the ranks of one node over NVLink peer memory (the C ABI's
    ``pa_peer_allreduce``): the replacement for NCCL after the row-split o_proj.

    Each rank allocates one buffer with ``SLOTS`` data slots of ``max_count`` elements and
    a flag area, and maps every peer's buffer through CUDA IPC (plain peer loads and
    stores; no multicast object is created).  A call works on the next slot in turn:
    :meth:`slot` hands out that slot as a tensor the o_proj GEMM writes its partial into,
    :meth:`all_reduce_` sums it across ranks in place.  A result stays valid until
    ``SLOTS`` more calls have been made.  All ranks must make the same sequence of calls.
    After a barrier wait runs out (a peer did not join within ``timeout_s``),
    :meth:`check` raises and the object must be discarded."""

    SLOTS = 2
    FLAG_BYTES = 128

    def __init__(self, max_count: int, dtype: torch.dtype, group=None, device=None, timeout_s: float = 2.0):
        from . import _lib
        from .attention import _DTYPE_CODE

        self._lib = _lib
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError(f"peer all-reduce spans at most 8 ranks of one node, got {self.world}")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dtype, self.code = dtype, _DTYPE_CODE[dtype]
        self.max_count = int(max_count)
        es = torch.empty(0, dtype=dtype).element_size()
        self.slot_bytes = -(-self.max_count * es // 256) * 256
        self.flags_offset = self.SLOTS * self.slot_bytes
        self.buf = torch.zeros(self.flags_offset + self.FLAG_BYTES, dtype=torch.uint8, device=self.device)
        self.bases, self._opened = _map_peers(self.buf, group, self.world, self.rank, self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.timeout_s = float(timeout_s)
        self._slot = 0
        dist.barrier(group=group)

    def slot(self, shape) -> torch.Tensor:
        """The next data slot as a contiguous ``shape`` tensor of this collective's dtype."""
        n = 1
        for d in shape:
            n *= int(d)
        if n > self.max_count:
            raise ValueError(f"{n} elements exceed the collective's {self.max_count}")
        off = self._slot * self.slot_bytes
        es = torch.empty(0, dtype=self.dtype).element_size()
        return self.buf[off:off + n * es].view(self.dtype).view(*shape)

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        """Sum ``t`` (the tensor :meth:`slot` returned for this call) across the ranks in place."""
        off = t.data_ptr() - self.buf.data_ptr()
        if t.dtype != self.dtype or not t.is_contiguous() or off != self._slot * self.slot_bytes:
            raise ValueError("all_reduce_ expects the tensor slot() handed out for this call")
        self._lib.check(self._lib.lib().pa_peer_allreduce(
            self.bases, self.world, self.rank, off, self.flags_offset, t.numel(), self.code, self.timeout_s,
            self.err.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream))
        self._slot = (self._slot + 1) % self.SLOTS
        return t

    def close(self) -> None:
        """Unmap the peers' buffers (after the last call has completed on every rank)."""
        torch.cuda.synchronize(self.device)
        for ptr, off in getattr(self, "_opened", []):
            self._lib.check(self._lib.lib().pa_ipc_close(ptr, off))
        self._opened = []

    def check(self) -> None:
        """Raise if a barrier wait of any call so far ran out (synchronises the device)."""
        if int(self.err.item()):
            raise RuntimeError(f"peer all-reduce: rank {self.rank} gave up waiting for its peers "
                               f"(timeout {self.timeout_s} s); discard this collective")


class FusedOProjAllReduce:
    """The row-split o_proj GEMM and its all-reduce as one collective over NVLink peer
    memory (the C ABI's ``pa_oproj_allreduce``): every rank gets ``sum_r a_r @ w_r``.

    The GEMM (tcgen05, 128 x 256 output tiles) stores each finished tile straight into the
    staging area of the rank that owns those columns, so the reduce-scatter rides on the
    GEMM's epilogue; each owner then sums its columns over the ranks' partials in rank
    order (float32) and stores them into every rank's output.  Every access to another
    GPU's memory is a plain store.  Each rank allocates one buffer (the staging area of
    ``max_rows * n`` elements, ``SLOTS`` output slots and a flag area) that every peer maps
    through CUDA IPC; no multicast object is created.  Without an initialised process group
    it runs on one GPU (the GEMM alone, through the same kernels).

    A call's output stays valid until ``SLOTS`` more calls.  All ranks make the same
    sequence of calls with the same ``rows``, ``k`` and ``n``.  After a wait for a peer runs
    out (``timeout_s``), :meth:`check` raises and the object must be discarded."""

    SLOTS = 2
    FLAG_BYTES = 128

    def __init__(self, max_rows: int, n: int, dtype: torch.dtype, group=None, device=None, timeout_s: float = 2.0):
        from . import _lib
        from .attention import _DTYPE_CODE

        if dtype not in (torch.bfloat16, torch.float16):
            raise NotImplementedError(f"fused o_proj all-reduce: {dtype} (bf16 or fp16 only)")
        self._lib = _lib
        self.group = group
        distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        if self.world > 8:
            raise ValueError(f"peer collectives span at most 8 ranks of one node, got {self.world}")
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype, self.code = dtype, _DTYPE_CODE[dtype]
        self.max_rows, self.n = int(max_rows), int(n)
        es = torch.empty(0, dtype=dtype).element_size()
        self.area_bytes = -(-self.max_rows * self.n * es // 256) * 256
        self.flags_offset = (1 + self.SLOTS) * self.area_bytes     # staging, then the output slots
        self.buf = torch.zeros(self.flags_offset + self.FLAG_BYTES, dtype=torch.uint8, device=self.device)
        self.bases, self._opened = _map_peers(self.buf, group, self.world, self.rank, self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.timeout_s = float(timeout_s)
        self._slot = 0
        if distributed:
            dist.barrier(group=group)

    def __call__(self, a: torch.Tensor, w_nk: torch.Tensor) -> torch.Tensor:
        """``a [rows, k]`` (unit column stride) times the K-major o_proj slice ``w_nk [n, k]``
        (``w_o.t().contiguous()``), summed over the ranks: ``[rows, n]`` in this call's
        output slot."""
        if a.dim() != 2 or w_nk.dim() != 2 or a.dtype != self.dtype or w_nk.dtype != self.dtype:
            raise ValueError(f"fused o_proj: a {tuple(a.shape)} {a.dtype} and w {tuple(w_nk.shape)} {w_nk.dtype}; "
                             f"expected 2-D {self.dtype}")
        rows, k = a.shape
        if w_nk.shape != (self.n, k) or not w_nk.is_contiguous() or a.stride(1) != 1:
            raise ValueError(f"fused o_proj: w must be a contiguous [{self.n}, {k}] (K-major) slice and a row-major")
        if rows > self.max_rows:
            raise ValueError(f"fused o_proj: {rows} rows exceed the collective's {self.max_rows}")
        if a.device != self.device or w_nk.device != self.device:
            raise ValueError(f"fused o_proj: tensors must be on {self.device}")
        off = (1 + self._slot) * self.area_bytes
        self._lib.check(self._lib.lib().pa_oproj_allreduce(
            a.data_ptr(), a.stride(0), rows, k, w_nk.data_ptr(), self.n, self.code, self.bases, self.world, self.rank,
            0, off, self.flags_offset, self.timeout_s, self.err.data_ptr(),
            torch.cuda.current_stream(self.device).cuda_stream))
        self._slot = (self._slot + 1) % self.SLOTS
        es = torch.empty(0, dtype=self.dtype).element_size()
        return self.buf[off:off + rows * self.n * es].view(self.dtype).view(rows, self.n)

    def close(self) -> None:
        """Unmap the peers' buffers (after the last call has completed on every rank)."""
        torch.cuda.synchronize(self.device)
        for ptr, off in getattr(self, "_opened", []):
            self._lib.check(self._lib.lib().pa_ipc_close(ptr, off))
        self._opened = []

    def check(self) -> None:
        """Raise if a wait of any call so far ran out (synchronises the device)."""
        if int(self.err.item()):
            raise RuntimeError(f"fused o_proj all-reduce: rank {self.rank} gave up waiting for its peers "
                               f"(timeout {self.timeout_s} s) or a pipeline wait ran out; discard this collective")


@dataclass
class KVHeadParallelAttention:
    """One layer's attention hot path on one tensor-parallel rank.

    ``attention`` and ``append`` default to the sm_100a kernels (``paged_attention_cuda``,
    ``reshape_and_cache``); they are parameters so the host logic — sharding, the o_proj
    split and the collective — can be exercised with other implementations of the same
    signatures."""

    w_o: torch.Tensor                 # [Hq_local * D, d_model]
    group: object = None              # torch.distributed process group (None = default)
    attention: object = None
    append: object = None
    reducer: object = None            # PeerAllReduce: sum over NVLink peer memory instead of NCCL
    fused: object = None              # FusedOProjAllReduce: the GEMM and its all-reduce in one collective

    def __post_init__(self):
        if self.fused is not None:
            self._w_nk = self.w_o.t().contiguous()   # K-major [d_model, Hq_local * D] for the fused GEMM
        if self.attention is None:
            from .attention import paged_attention_cuda

            self.attention = paged_attention_cuda
        if self.append is None:
            from .kv_cache import reshape_and_cache

            self.append = reshape_and_cache

    def __call__(self, q, k_new, v_new, k_pool, v_pool, block_tables, context_lens, query_lens, scale,
                 slot_mapping) -> torch.Tensor:
        """q ``[T, Hq/tp, D]``, new K/V ``[T, Hkv/tp, D]`` -> the all-reduced o_proj output
        ``[T, d_model]`` (identical on every rank)."""
        self.append(k_new, v_new, k_pool, v_pool, slot_mapping)
        attn = self.attention(q, k_pool, v_pool, block_tables, context_lens, query_lens, scale)
        a2 = attn.reshape(attn.shape[0], -1).to(self.w_o.dtype)
        if self.fused is not None:         # GEMM epilogue pushes tiles to their owners, owners sum
            return self.fused(a2, self._w_nk)
        if self.reducer is not None:       # the GEMM writes straight into the peer-mapped slot
            partial = torch.matmul(a2, self.w_o, out=self.reducer.slot((a2.shape[0], self.w_o.shape[1])))
            return self.reducer.all_reduce_(partial)
        partial = a2 @ self.w_o
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        return partial
