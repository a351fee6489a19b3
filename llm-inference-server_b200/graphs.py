"""CUDA-graph capture of decode steps: the per-step host work of the hot path reduced to
one metadata copy and one graph launch.

The reference pays a Python dispatch per layer per step (inference_server/core/
paged_executor.py:134-156 calls the attention seam once per layer); the eager CUDA path
here still pays a library call per kernel.  A :class:`DecodeStepGraph` captures
``layers x (fused K/V append + paged attention)`` of an all-decode step for a fixed
batch once, then each step only plans on the host (into a pinned buffer), copies that
metadata into the same device buffer and replays the graph.

Replaying needs every launch parameter to stay fixed, so the step is planned with
``pa_plan_decode_padded``: a fixed split size, block tables ``width`` wide, and decode-
item / combine lists padded with null entries to the worst case for that width
(``batch * ceil(width / split)`` items, ``batch`` combines).  Any step whose contexts
fit ``width * block_size`` tokens replays the same graph; a longer one raises
:class:`BucketOverflow` and the caller builds a wider graph.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .attention import _DTYPE_CODE
from .metadata import StepMetadata, attach, sm_count

BucketOverflow = _lib.BucketOverflow


class DecodeStepGraph:
    """One captured decode step over ``len(k_pools)`` layers for ``batch`` sequences.

    Inputs are the static tensors ``q [L, B, Hq, D]``, ``k_new`` / ``v_new``
    ``[L, B, Hkv, D]`` (write them before :meth:`replay`); outputs land in ``out
    [L, B, Hq, D]``.  ``width`` (blocks per table row) fixes the bucket."""

    def __init__(self, k_pools, v_pools, num_heads: int, scale: float, batch: int, width: int,
                 split_blocks: int | None = None, device=None):
        self.k_pools, self.v_pools = list(k_pools), list(v_pools)
        ref = self.k_pools[0]
        if ref.device.type != "cuda":
            raise NotImplementedError(f"ATTENTION=cuda: decode graphs need CUDA pools, got {ref.device}")
        self.device = torch.device(device) if device is not None else ref.device
        self.L = len(self.k_pools)
        self.NB, self.BS, self.Hkv, self.D = (int(x) for x in ref.shape)
        self.Hq, self.B, self.width, self.scale = int(num_heads), int(batch), int(width), float(scale)
        self.dtype = ref.dtype
        if split_blocks is None:   # the eager planner's choice for a batch of full-width contexts
            probe = StepMetadata.plan_host(np.full(self.B, self.width * self.BS, np.int64), np.ones(self.B, np.int64),
                                           np.zeros((self.B, self.width), np.int64), num_tokens=self.B,
                                           pool_num_blocks=self.NB, block_size=self.BS, num_kv_heads=self.Hkv,
                                           sm=sm_count(self.device))
            split_blocks = int(probe.plan.split_blocks)
        self.split = int(split_blocks)
        self.items = self.B * (-(-self.width // self.split))
        self.combine = self.B
        shape_q, shape_kv = (self.L, self.B, self.Hq, self.D), (self.L, self.B, self.Hkv, self.D)
        self.q = torch.zeros(shape_q, dtype=self.dtype, device=self.device)
        self.k_new = torch.zeros(shape_kv, dtype=self.dtype, device=self.device)
        self.v_new = torch.zeros(shape_kv, dtype=self.dtype, device=self.device)
        self.out = torch.zeros(shape_q, dtype=self.dtype, device=self.device)
        # plan the bucket's shape once (any in-bucket contexts give the same counts / offsets)
        probe = StepMetadata.plan_decode_padded(np.ones(self.B, np.int64), np.zeros((self.B, 1), np.int64),
                                                **self._caps())
        self.plan = probe.plan
        self.words = int(self.plan.words)
        self._host_t = torch.zeros(self.words, dtype=torch.int32, pin_memory=True)
        self._host = self._host_t.numpy()
        self.meta = torch.zeros(self.words, dtype=torch.int32, device=self.device)
        ws_bytes = int(_lib.lib().pa_workspace_bytes(ctypes.byref(self.plan), self.Hq, self.D))
        self.workspace = torch.zeros(ws_bytes + 256, dtype=torch.uint8, device=self.device)
        self._copied = torch.cuda.Event()
        self._copied.record(torch.cuda.current_stream(self.device))
        self.graph = None
        self._planned = False

    def _caps(self) -> dict:
        return dict(pool_num_blocks=self.NB, block_size=self.BS, num_kv_heads=self.Hkv, split_blocks=self.split,
                    width=self.width, items=self.items, combine=self.combine)

    # ---------------------------------------------------------------- per step
    def set_step(self, context_lens, block_tables) -> None:
        """Plan this step's metadata into the pinned buffer (contexts count the new
        token).  Raises BucketOverflow when a context needs more than ``width`` blocks."""
        self._copied.synchronize()           # the previous step's copy has left the buffer
        meta = StepMetadata.plan_decode_padded(context_lens, block_tables, host=self._host, **self._caps())
        if int(meta.plan.words) != self.words or int(meta.plan.num_decode_items) != self.items:
            raise RuntimeError("padded plan changed shape inside its bucket")
        self._planned = True

    def _upload(self, stream) -> None:
        self.meta.copy_(self._host_t, non_blocking=True)
        self._copied.record(stream)

    def _launch_layers(self, stream_handle: int) -> None:
        lib, code = _lib.lib(), _DTYPE_CODE[self.dtype]
        slots = self.meta.data_ptr() + 4 * int(self.plan.off_slot_mapping)
        ws = (self.workspace.data_ptr() + 255) // 256 * 256
        ws_bytes = self.workspace.numel() - (ws - self.workspace.data_ptr())
        for l in range(self.L):
            kn, vn, q, out = self.k_new[l], self.v_new[l], self.q[l], self.out[l]
            _lib.check(lib.pa_reshape_and_cache(kn.data_ptr(), kn.stride(0), kn.stride(1), vn.data_ptr(), vn.stride(0),
                                                vn.stride(1), self.B, self.Hkv, self.D, code,
                                                self.k_pools[l].data_ptr(), self.v_pools[l].data_ptr(), self.NB,
                                                self.BS, slots, stream_handle))
            _lib.check(lib.pa_paged_attention_fwd(q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), self.B,
                                                  self.Hq, self.D, self.k_pools[l].data_ptr(),
                                                  self.v_pools[l].data_ptr(), self.NB, self.BS, self.Hkv, code,
                                                  self.scale, ctypes.byref(self.plan), self.meta.data_ptr(),
                                                  out.data_ptr(), out.stride(0), out.stride(1), ws, ws_bytes,
                                                  stream_handle))

    def run_eager(self) -> None:
        """The same launches without the graph (for comparison)."""
        if not self._planned:
            raise RuntimeError("set_step() first")
        stream = torch.cuda.current_stream(self.device)
        self._upload(stream)
        self._launch_layers(stream.cuda_stream)

    def capture(self) -> None:
        """Capture the step's launches (call after set_step; runs them once eagerly
        first so every kernel is configured before capture)."""
        self.run_eager()
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            with torch.cuda.graph(self.graph, stream=side):
                self._launch_layers(side.cuda_stream)
        torch.cuda.current_stream(self.device).wait_stream(side)

    def replay(self) -> None:
        """Copy this step's metadata to the device and launch the captured step."""
        if self.graph is None:
            raise RuntimeError("capture() first")
        stream = torch.cuda.current_stream(self.device)
        self._upload(stream)
        self.graph.replay()

    def read_error(self, clear: bool = True) -> int:
        word = ctypes.c_int32(0)
        ws = (self.workspace.data_ptr() + 255) // 256 * 256
        _lib.check(_lib.lib().pa_read_device_error(ws, int(clear), ctypes.byref(word),
                                                   torch.cuda.current_stream(self.device).cuda_stream))
        return int(word.value)


class ModelDecodeGraph:
    """One captured all-decode pass of a whole model for a bucket of ``batch`` rows and
    ``width`` table blocks: the HF forward with this library's paged attention and fused
    append (the executor's two hooks), then the greedy argmax.  A step only plans its
    metadata on the host (into a pinned buffer), copies it and the token ids into the
    graph's static buffers and replays; the per-layer Python and library dispatch of the
    eager pass is gone.

    Rows past the step's real sequences repeat its last row: the same token at the same
    position writes the same K/V bytes into the same slot and its output is dropped, so
    the padding needs no spare pool block.  The plan is padded as in
    :class:`DecodeStepGraph` (fixed split size, decode-item and combine lists padded with
    null entries), so every launch parameter inside the graph stays fixed."""

    def __init__(self, executor, batch: int, width: int):
        ex = executor
        self.ex, self.B, self.width = ex, int(batch), int(width)
        dev = ex.device
        NB, BS, Hkv = ex.num_blocks, ex.block_size, ex.num_kv_heads
        probe = StepMetadata.plan_host(np.full(self.B, self.width * BS, np.int64), np.ones(self.B, np.int64),
                                       np.zeros((self.B, self.width), np.int64), num_tokens=self.B,
                                       pool_num_blocks=NB, block_size=BS, num_kv_heads=Hkv, sm=sm_count(dev))
        split = int(probe.plan.split_blocks)
        self.caps = dict(pool_num_blocks=NB, block_size=BS, num_kv_heads=Hkv, split_blocks=split,
                         width=self.width, items=self.B * (-(-self.width // split)), combine=self.B)
        shape = StepMetadata.plan_decode_padded(np.ones(self.B, np.int64), np.zeros((self.B, 1), np.int64),
                                                **self.caps)
        self.words, self.items = int(shape.plan.words), int(shape.plan.num_decode_items)
        self._host_t = torch.zeros(self.words, dtype=torch.int32, pin_memory=True)
        self.meta = StepMetadata(shape.plan, self._host_t.numpy(), NB)
        self.meta.device_buffer = torch.zeros(self.words, dtype=torch.int32, device=dev)
        self._ids_host = torch.zeros(1, self.B, dtype=torch.long, pin_memory=True)
        self.ids = torch.zeros(1, self.B, dtype=torch.long, device=dev)
        self._copied = torch.cuda.Event()
        self._copied.record(torch.cuda.current_stream(dev))
        self.graph = None
        self.tokens = None

    def set_step(self, context_lens, block_tables, token_ids) -> None:
        """Plan this step (contexts count the new token) and stage its token ids."""
        self._copied.synchronize()           # the previous step's copies have left the buffers
        meta = StepMetadata.plan_decode_padded(context_lens, block_tables, host=self.meta.host, **self.caps)
        if int(meta.plan.words) != self.words or int(meta.plan.num_decode_items) != self.items:
            raise RuntimeError("padded plan changed shape inside its bucket")
        self._ids_host[0].copy_(torch.as_tensor(token_ids, dtype=torch.long))

    def _forward(self):
        from .executor import StepContext   # the executor module imports this one

        buf, plan = self.meta.device_buffer, self.meta.plan
        ctx = StepContext(meta=self.meta, block_tables=attach(torch.empty(0, dtype=torch.long, device=buf.device),
                                                              self.meta),
                          context_lens=buf[plan.off_context_lens:plan.off_context_lens + self.B],
                          query_lens=buf[plan.off_query_lens:plan.off_query_lens + self.B], pool=self.ex.pool)
        logits = self.ex._forward(self.ids, self.meta.q_pos().unsqueeze(0), ctx)
        return logits[0].argmax(-1)

    def run(self) -> torch.Tensor:
        """Upload the staged step and run it (capturing it the first time); returns the
        greedy token of every row (device tensor, valid until the next run)."""
        dev = self.ex.device
        stream = torch.cuda.current_stream(dev)
        self.meta.device_buffer.copy_(self._host_t, non_blocking=True)
        self.ids.copy_(self._ids_host, non_blocking=True)
        self._copied.record(stream)
        if self.graph is None:
            self.tokens = self._forward()    # eager once: configures every kernel, sizes the workspace
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side), torch.cuda.graph(self.graph, stream=side):
                self.tokens = self._forward()
            stream.wait_stream(side)
        self.graph.replay()
        return self.tokens
