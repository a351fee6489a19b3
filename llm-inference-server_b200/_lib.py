"""ctypes binding of ``libpaged_attn_b200.so`` (the C ABI in include/paged_attention_b200.h).

The library is built in-tree by ``build.py``.  Loading never falls back to anything:
if the library is missing the CUDA path raises ``NotImplementedError`` naming the
reason, exactly as the reference's Triton path does when it cannot run
(inference_server/core/attention_triton.py:250-264).
"""

from __future__ import annotations

import ctypes
import re
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_uint64, c_void_p
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libpaged_attn_b200.so"
HEADER = PKG.parent / "include" / "paged_attention_b200.h"

PA_OK = 0
PA_ERR_INVALID_ARGUMENT = 1
PA_ERR_UNSUPPORTED = 2
PA_ERR_CUDA = 3
PA_ERR_BUFFER_TOO_SMALL = 4

PA_DTYPE_F32 = 0
PA_DTYPE_F16 = 1
PA_DTYPE_BF16 = 2

PA_NOALLOC_SCRATCH_BYTES = 32 << 20

PA_LAUNCH_DECODE_MMA = 1
PA_LAUNCH_DECODE_SIMT = 2
PA_LAUNCH_COMBINE = 4
PA_LAUNCH_PREFILL_TC = 8
PA_LAUNCH_GENERIC = 16
PA_LAUNCH_PREFILL_PAIR = 32
PA_LAUNCH_PREFILL_PERSIST = 64

ABI_VERSION = 7


class StepPlan(ctypes.Structure):
    """Mirror of ``pa_step_plan``."""

    _fields_ = [
        ("num_seqs", c_int32),
        ("num_tokens", c_int32),
        ("table_width", c_int32),
        ("block_size", c_int32),
        ("num_decode_seqs", c_int32),
        ("num_prefill_seqs", c_int32),
        ("num_prefill_tokens", c_int32),
        ("split_blocks", c_int32),
        ("num_decode_items", c_int32),
        ("num_combine_seqs", c_int32),
        ("max_context", c_int32),
        ("max_query_len", c_int32),
        ("prefill_tile_tokens", c_int32),
        ("num_prefill_tiles", c_int32),
        ("total_context", c_int64),
        ("off_block_tables", c_int64),
        ("off_context_lens", c_int64),
        ("off_query_lens", c_int64),
        ("off_cu_query_lens", c_int64),
        ("off_seq_idx", c_int64),
        ("off_q_pos", c_int64),
        ("off_slot_mapping", c_int64),
        ("off_decode_items", c_int64),
        ("off_combine", c_int64),
        ("off_prefill_tiles", c_int64),
        ("words", c_int64),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


_SIGNATURES = {
    "pa_abi_version": (c_int32, []),
    "pa_prefill_tile_rows": (c_int32, [c_int32]),
    "pa_last_launches": (c_int32, []),
    "pa_last_error": (c_char_p, []),
    "pa_plan_words_bound": (c_int64, [c_int32, c_int32, c_int32]),
    "pa_plan_step": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_int64, c_int32, c_int32, c_int64,
                               c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, POINTER(StepPlan)]),
    "pa_workspace_bytes": (c_uint64, [POINTER(StepPlan), c_int32, c_int32]),
    "pa_paged_attention_fwd": (c_int32, [c_void_p, c_int64, c_int64, c_int64, c_int32, c_int32, c_int32,
                                         c_void_p, c_void_p, c_int64, c_int32, c_int32, c_int32, c_float,
                                         POINTER(StepPlan), c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                         c_uint64, c_void_p]),
    "pa_reshape_and_cache": (c_int32, [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int32,
                                       c_int32, c_int32, c_int32, c_void_p, c_void_p, c_int64, c_int32,
                                       c_void_p, c_void_p]),
    "pa_read_device_error": (c_int32, [c_void_p, c_int32, POINTER(c_int32), c_void_p]),
    "pa_paged_attention_fwd_noalloc": (c_int32, [c_void_p, c_int64, c_int64, c_int64, c_int32, c_int32, c_int32,
                                                 c_void_p, c_void_p, c_int64, c_int32, c_int32, c_int32, c_float,
                                                 POINTER(StepPlan), c_void_p, c_void_p, c_int64, c_int64,
                                                 c_void_p]),
    "pa_noalloc_read_device_error": (c_int32, [c_int32, POINTER(c_int32), c_void_p]),
    "pa_copy_blocks": (c_int32, [POINTER(c_void_p), POINTER(c_void_p), c_int32, c_int64, c_int64, c_void_p, c_int32,
                                 c_void_p, c_void_p]),
    "pa_gather_blocks": (c_int32, [POINTER(c_void_p), POINTER(c_void_p), c_int32, c_int64, c_int64, c_void_p,
                                   c_int32, c_void_p, c_void_p, c_void_p]),
    "pa_scatter_blocks": (c_int32, [POINTER(c_void_p), POINTER(c_void_p), c_int32, c_int64, c_int64, c_void_p,
                                    c_int32, c_void_p, c_void_p, c_void_p]),
    "pa_peer_allreduce": (c_int32, [POINTER(c_void_p), c_int32, c_int32, c_int64, c_int64, c_int64, c_int32,
                                    ctypes.c_double, c_void_p, c_void_p]),
    "pa_ipc_export": (c_int32, [c_void_p, c_void_p, POINTER(c_int64)]),
    "pa_ipc_open": (c_int32, [c_void_p, c_int64, POINTER(c_void_p)]),
    "pa_ipc_close": (c_int32, [c_void_p, c_int64]),
    "pa_oproj_allreduce": (c_int32, [c_void_p, c_int64, c_int32, c_int32, c_void_p, c_int32, c_int32,
                                     POINTER(c_void_p), c_int32, c_int32, c_int64, c_int64, c_int64, ctypes.c_double,
                                     c_void_p, c_void_p]),
    "pa_plan_decode_padded": (c_int32, [c_void_p, c_int32, c_void_p, c_int64, c_int32, c_int64, c_int32, c_int32,
                                        c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, POINTER(StepPlan)]),
}

_lib = None


def lib():
    """The loaded library (loaded once).  Raises NotImplementedError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise NotImplementedError(
            f"ATTENTION=cuda: the sm_100a library {LIB_PATH.name} is not built; run "
            "`python llm-inference-server_b200/build.py` (or __graft_entry__.build())"
        )
    handle = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    if handle.pa_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{LIB_PATH.name} has ABI {handle.pa_abi_version()}, this binding expects {ABI_VERSION}")
    _lib = handle
    return _lib


def declared_symbols() -> list[str]:
    """Every function the public header declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(pa_\w+)\s*\(", text, flags=re.M)))


def last_launches() -> set[str]:
    """Names of the kernels the calling thread's last attention call launched."""
    mask = lib().pa_last_launches()
    names = {PA_LAUNCH_DECODE_MMA: "decode_mma", PA_LAUNCH_DECODE_SIMT: "decode_simt",
             PA_LAUNCH_COMBINE: "combine", PA_LAUNCH_PREFILL_TC: "prefill_tc", PA_LAUNCH_GENERIC: "generic",
             PA_LAUNCH_PREFILL_PAIR: "prefill_pair", PA_LAUNCH_PREFILL_PERSIST: "prefill_persist"}
    return {n for bit, n in names.items() if mask & bit}


class BucketOverflow(ValueError):
    """A step does not fit the fixed shape of a padded (CUDA-graph) plan."""


def check(rc: int) -> None:
    """Map a C return code to the reference's exception types."""
    if rc == PA_OK:
        return
    msg = lib().pa_last_error().decode(errors="replace")
    if rc == PA_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if rc == PA_ERR_UNSUPPORTED:
        raise NotImplementedError(f"ATTENTION=cuda: {msg}")
    if rc == PA_ERR_BUFFER_TOO_SMALL and msg.startswith("bucket"):
        raise BucketOverflow(msg)
    raise RuntimeError(msg)
