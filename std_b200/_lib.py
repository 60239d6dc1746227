"""ctypes binding of libstd_b200.so (the C ABI declared in include/std_b200.h).

This is the same binding a maintainer of the reference would add next to
std_repro/triton_attention.py: plain pointers, sizes and a cudaStream_t.  Any
nonzero status raises RuntimeError, matching the reference's error style
(std_qwen25vl.py:379-380, :401-402).  There is no fallback: if the library is
missing the import fails loudly.
"""

from __future__ import annotations

import ctypes
import os
from typing import Dict

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libstd_b200.so")

P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_longlong
SZ = ctypes.c_size_t
F = ctypes.c_float
PI32 = ctypes.c_void_p
PF = ctypes.c_void_p

# name -> (restype, argtypes); the single source of truth for the ABI surface
SIGNATURES: Dict[str, tuple] = {
    "std_version": (I, []),
    "std_get_device_error": (I, [P]),
    "std_device_supported": (I, []),
    "std_draft_attn_workspace_bytes": (SZ, [I, I, I, I, I]),
    "std_draft_attn": (I, [P, P, P, PI32, I, I, I, I, I, I, P, PF, P, SZ, I, P]),
    "std_draft_attn_indexed": (I, [P, P, P, I, PI32, I, P, P, I, PI32, I, I, I, I, I, P, PF, P]),
    "std_verify_attn_workspace_bytes": (SZ, [I, I, I]),
    "std_verify_attn": (I, [P, P, P, PI32, I, I, I, I, I, I, I, I, P, PF, P, SZ, P]),
    "std_verify_attn_noalloc": (I, [P, P, P, PI32, I, I, I, I, I, I, I, I, P, PF, P]),
    "std_merge_partials": (I, [P, PF, I, I, I, P, PF, P]),
    "std_verify_attn_partial": (I, [P, P, P, PI32, I, I, I, I, I, I, I, I, PF, PF, P, SZ, P]),
    "std_merge_partials_f32": (I, [PF, I64, I, I, I, P, PF, P]),
    "std_ipc_handle_bytes": (SZ, []),
    "std_device_alloc": (I, [SZ, P]),
    "std_device_free": (I, [P]),
    "std_ipc_handle": (I, [P, P]),
    "std_ipc_open": (I, [P, P]),
    "std_ipc_close": (I, [P]),
    "std_p2p_post": (I, [P, P, SZ, P, I, P, P]),
    "std_p2p_wait": (I, [P, I, P, P]),
    "std_merge_partials_f32_list": (I, [P, I, I, I, P, PF, P]),
    "std_select_workspace_bytes": (SZ, [I, I, I]),
    "std_select_scores": (I, [P, P, I64, I, I, I, I, I, I, F, PF, I, P, SZ, P]),
    "std_select_probs_view": (I, [I, I, I, P]),
    "std_topk_select": (I, [PF, I64, I, PI32, I, I, PI32, P]),
    "std_compact_gather": (I, [P, P, I, I, I, I, I, I, I, PI32, I, PI32, I, P]),
    "std_gemm_workspace_bytes": (SZ, [I, I, I]),
    "std_gemm_bf16": (I, [P, P, P, P, I, I, I, P, SZ, P]),
    "std_gemm_epilogue_workspace_bytes": (SZ, [I, I, I]),
    "std_gemm_add_rmsnorm": (I, [P, P, P, P, P, F, P, I, I, I, P, SZ, P]),
    "std_gemm_silu_mul": (I, [P, P, I, I, I, P, P, SZ, P]),
    "std_gemm_argmax": (I, [P, P, I, I, I, I, I, I, I, PI32, PF, P, P, SZ, P]),
    "std_gemm_rope_append": (I, [P, P, P, I, I, I, I, I, I, P, I, P, I, P, P, I, P, P, P, I, P, SZ, P]),
    "std_embed": (I, [P, I, I, PI32, I, I, I, I, P, P]),
    "std_gemm_set_smem_budget": (I, [I]),
    "std_collect_workspace_bytes": (SZ, [I, I, I, I]),
    "std_collect_relevance": (I, [P, P, PI32, I, I, I, I, I, I, I, PF, I64, P, SZ, P]),
    "std_gemm_plan": (I, [I, I, P]),
    "std_verify_policy": (I, [I, I, I, PI32, I, PI32, I, PI32, I, PI32, PI32, PI32, PF, F, I, I, I, PI32, PI32, PI32, PF,
                              I, PI32, ctypes.c_ulonglong, I, P]),
    "std_graph_cond_handle": (I, [P, P]),
    "std_capture_if_begin": (I, [P, P, ctypes.c_ulonglong]),
    "std_capture_if_end": (I, [P]),
    "std_stream_create": (I, [P]),
    "std_rmsnorm": (I, [P, P, F, I, I, P, P]),
    "std_add_rmsnorm": (I, [P, P, P, F, I, I, P, P]),
    "std_rope_append": (I, [P, I, I, I, I, I, PI32, I, PI32, I, P, P, I, P, P, P, I, P]),
    "std_silu_mul": (I, [P, I, I, I, P, P]),
    "std_add": (I, [P, P, SZ, P, P]),
    "std_argmax_rows": (I, [P, I, I, I, I, I, PI32, P]),
    "std_accept_commit": (I, [I, I, I, PI32, I, PI32, I, PI32, I, I, I, PI32, PI32, PI32, PI32, PI32, PI32, PI32,
                              PI32, I, P]),
    "std_ar_commit": (I, [I, I, I, I, I, PI32, PI32, PI32, PI32, PI32, P]),
    "std_ar_advance": (I, [I, PI32, PI32, PI32, I, PI32, PI32, P]),
    "std_capture_while_begin": (I, [P, P, PI32, I, PI32, P, P]),
    "std_capture_while_end": (I, [P, ctypes.c_ulonglong, PI32, I, PI32, I]),
    "std_launch_count": (I64, []),
}

_STATUS = {1: "bad shape or argument", 2: "capacity exceeded", 3: "unsupported device or driver entry point",
           4: "CUDA launch error", 5: "workspace missing or too small"}

_lib = None


_CAPTURE_STREAMS: Dict[tuple, object] = {}


def capture_stream(role: str):
    """A dedicated CUDA stream (torch.cuda.ExternalStream) per (role, device)
    for capturing conditional-node bodies; created once by the library."""
    import torch

    key = (role, torch.cuda.current_device())
    st = _CAPTURE_STREAMS.get(key)
    if st is None:
        ptr = ctypes.c_void_p(0)
        call("std_stream_create", ctypes.byref(ptr))
        st = torch.cuda.ExternalStream(ptr.value)
        _CAPTURE_STREAMS[key] = st
    return st


def load() -> ctypes.CDLL:
    """Load the in-tree library (building it first if sources are newer)."""
    global _lib
    if _lib is None:
        from . import build as _build

        if _build.needs_build():
            _build.build()
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def call(name: str, *args) -> int:
    rc = getattr(load(), name)(*args)
    if rc != 0:
        raise RuntimeError(f"{name} failed with status {rc} ({_STATUS.get(rc, 'unknown')})")
    return rc


def query(name: str, *args):
    return getattr(load(), name)(*args)


def device_error() -> int:
    code = ctypes.c_int(0)
    call("std_get_device_error", ctypes.byref(code))
    return int(code.value)
