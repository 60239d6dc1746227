"""torch-facing wrappers over the C ABI (one call per kernel entry point).

PyTorch only supplies device memory and the current CUDA stream here; every
call goes through libstd_b200.so.  Tensors must be CUDA, contiguous and of the
documented dtype -- there is no CPU path and no fallback.
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch

from . import _lib

_WS: Dict[Tuple[str, int], torch.Tensor] = {}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (no CPU path)")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def workspace(kind: str, nbytes: int, device: torch.device) -> torch.Tensor:
    """Scratch buffer, grown on demand, one per (kind, device).

    Allocation happens outside graph capture: call each op once eagerly before
    capturing it.
    """
    key = (kind, device.index if device.index is not None else torch.cuda.current_device())
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


# ----------------------------------------------------------------------------
# attention
# ----------------------------------------------------------------------------

def draft_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lens: torch.Tensor,
                    len_offset: int = 0, out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
                    after_append: bool = False):
    """q [B, Hq, D] bf16; caches [B, Hkv, cap, D] bf16; lens [B] int32 (device).

    after_append=True (STD_DRAFT_AFTER_APPEND): the previous launch on the
    stream writes only q and each request's newest K/V row, so the kernel may
    start reading the older rows before it finishes."""
    B, Hq, D = q.shape
    _, Hkv, cap, _ = k_cache.shape
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _check(t, torch.bfloat16, n)
    _check(lens, torch.int32, "lens")
    if out is None:
        out = torch.empty_like(q)
    nb = _lib.query("std_draft_attn_workspace_bytes", B, Hq, Hkv, D, cap)
    ws = workspace("draft", nb, q.device)
    _lib.call("std_draft_attn", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), lens.data_ptr(), int(len_offset),
              B, Hq, Hkv, D, cap, out.data_ptr(), _p(lse), ws.data_ptr(), ws.numel(), 1 if after_append else 0,
              _stream())
    return out


def draft_attention_indexed(q: torch.Tensor, dense_k: torch.Tensor, dense_v: torch.Tensor, idx: torch.Tensor,
                            tail_k: torch.Tensor, tail_v: torch.Tensor, lens: torch.Tensor, len_offset: int = 0,
                            out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None):
    """Draft attention over dense-cache rows idx [B, Hkv, n_idx] (int32,
    ascending) followed by the tail [B, Hkv, tail_cap, D]; keys per request =
    lens[b] + len_offset."""
    B, Hq, D = q.shape
    _, Hkv, cap_d, _ = dense_k.shape
    for t, n in ((q, "q"), (dense_k, "dense_k"), (dense_v, "dense_v"), (tail_k, "tail_k"), (tail_v, "tail_v")):
        _check(t, torch.bfloat16, n)
    _check(idx, torch.int32, "idx")
    _check(lens, torch.int32, "lens")
    if idx.shape[:2] != (B, Hkv):
        raise ValueError("idx must be [B, Hkv, n_idx]")
    if out is None:
        out = torch.empty_like(q)
    _lib.call("std_draft_attn_indexed", q.data_ptr(), dense_k.data_ptr(), dense_v.data_ptr(), cap_d, idx.data_ptr(),
              idx.shape[2], tail_k.data_ptr(), tail_v.data_ptr(), tail_k.shape[2], lens.data_ptr(), int(len_offset),
              B, Hq, Hkv, D, out.data_ptr(), _p(lse), _stream())
    return out


def verify_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lens: torch.Tensor,
                     len_offset: int, causal: bool = True, out: Optional[torch.Tensor] = None,
                     lse: Optional[torch.Tensor] = None):
    """q [B, nq, Hq, D] bf16; caches [B, Hkv, cap, D]; keys = lens[b] + len_offset."""
    B, nq, Hq, D = q.shape
    _, Hkv, cap, _ = k_cache.shape
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _check(t, torch.bfloat16, n)
    _check(lens, torch.int32, "lens")
    if out is None:
        out = torch.empty_like(q)
    nb = _lib.query("std_verify_attn_workspace_bytes", B, Hkv, cap)
    ws = workspace("verify", nb, q.device)
    _lib.call("std_verify_attn", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), lens.data_ptr(),
              int(len_offset), nq, 1 if causal else 0, B, Hq, Hkv, D, cap, out.data_ptr(), _p(lse), ws.data_ptr(),
              ws.numel(), _stream())
    return out


def verify_attention_partial(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lens: torch.Tensor,
                             len_offset: int, causal: bool, out_f32: torch.Tensor, lse: torch.Tensor):
    """verify_attention with an fp32 output and its LSE (one key range's
    partial of a sequence-sharded verify)."""
    B, nq, Hq, D = q.shape
    _, Hkv, cap, _ = k_cache.shape
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _check(t, torch.bfloat16, n)
    _check(out_f32, torch.float32, "out_f32")
    _check(lse, torch.float32, "lse")
    nb = _lib.query("std_verify_attn_workspace_bytes", B, Hkv, cap)
    ws = workspace("verify", nb, q.device)
    _lib.call("std_verify_attn_partial", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), lens.data_ptr(),
              int(len_offset), nq, 1 if causal else 0, B, Hq, Hkv, D, cap, out_f32.data_ptr(), lse.data_ptr(),
              ws.data_ptr(), ws.numel(), _stream())
    return out_f32


def merge_partials_f32(parts: torch.Tensor, rows: int, D: int, out: torch.Tensor,
                       lse_out: Optional[torch.Tensor] = None):
    """parts [n, stride] fp32, each [rows*D O | rows LSE] -> out [rows, D] bf16."""
    n, stride = parts.shape
    _check(parts, torch.float32, "parts")
    _lib.call("std_merge_partials_f32", parts.data_ptr(), stride, n, rows, D, out.data_ptr(), _p(lse_out), _stream())
    return out


def merge_partials(o_parts: torch.Tensor, lse_parts: torch.Tensor, out: Optional[torch.Tensor] = None,
                   lse_out: Optional[torch.Tensor] = None):
    """o_parts [n, rows, D] bf16, lse_parts [n, rows] fp32 -> out [rows, D]."""
    n, rows, D = o_parts.shape
    _check(o_parts, torch.bfloat16, "o_parts")
    _check(lse_parts, torch.float32, "lse_parts")
    if out is None:
        out = torch.empty((rows, D), dtype=torch.bfloat16, device=o_parts.device)
    _lib.call("std_merge_partials", o_parts.data_ptr(), lse_parts.data_ptr(), n, rows, D, out.data_ptr(),
              _p(lse_out), _stream())
    return out


def collect_relevance(q: torch.Tensor, k_cache: torch.Tensor, visual_pos: torch.Tensor, rel_out: torch.Tensor):
    """Collector v1 for one layer: rel_out [B, Hkv, P] fp32 at the visual
    positions gets sum over the verify rows of softmax over the visual keys of
    (group-mean query . k) / sqrt(D).  q [B, nq, Hq, D] bf16; k_cache [B, Hkv,
    cap, D] bf16; visual_pos [V] int32."""
    B, nq, Hq, D = q.shape
    _, Hkv, cap, _ = k_cache.shape
    _check(q, torch.bfloat16, "q")
    _check(k_cache, torch.bfloat16, "k_cache")
    _check(visual_pos, torch.int32, "visual_pos")
    _check(rel_out, torch.float32, "rel_out")
    V = visual_pos.numel()
    ws = workspace("collect", _lib.query("std_collect_workspace_bytes", B, Hkv, nq, V), q.device)
    _lib.call("std_collect_relevance", q.data_ptr(), k_cache.data_ptr(), visual_pos.data_ptr(), V, B, nq, Hq, Hkv, D,
              cap, rel_out.data_ptr(), rel_out.shape[-1], ws.data_ptr(), ws.numel(), _stream())
    return rel_out


# ----------------------------------------------------------------------------
# selection
# ----------------------------------------------------------------------------

def select_scores(q_text: torch.Tensor, k_rows: torch.Tensor, P: int, q_start: int,
                  scores: Optional[torch.Tensor] = None, write_probs: bool = False, scale: Optional[float] = None):
    """q_text [T, Hq, D] bf16; k_rows [Hkv, kstride, D] bf16 -> scores [Hkv, P] fp32.

    With write_probs, also returns the fp16 probabilities view [Hq, T, P].
    """
    T, Hq, D = q_text.shape
    Hkv, kstride, _ = k_rows.shape
    _check(q_text, torch.bfloat16, "q_text")
    _check(k_rows, torch.bfloat16, "k_rows")
    if scores is None:
        scores = torch.empty((Hkv, P), dtype=torch.float32, device=q_text.device)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    nb = _lib.query("std_select_workspace_bytes", T, Hq, P)
    ws = workspace("select", nb, q_text.device)
    _lib.call("std_select_scores", q_text.data_ptr(), k_rows.data_ptr(), kstride, T, Hq, Hkv, D, P, q_start,
              float(scale), scores.data_ptr(), 1 if write_probs else 0, ws.data_ptr(), ws.numel(), _stream())
    if not write_probs:
        return scores
    import ctypes

    ps = ctypes.c_longlong(0)
    _lib.call("std_select_probs_view", T, Hq, P, ctypes.byref(ps))
    probs = ws[: Hq * T * ps.value * 2].view(torch.float16).view(Hq, T, ps.value)[:, :, :P]
    return scores, probs


def topk_select(scores: torch.Tensor, visual_pos: torch.Tensor, k: int, out: Optional[torch.Tensor] = None):
    """scores [n_seg, P] fp32; visual_pos [V] int32 ascending -> [n_seg, k] int32 ascending."""
    n_seg, P = scores.shape
    _check(scores, torch.float32, "scores")
    _check(visual_pos, torch.int32, "visual_pos")
    if out is None:
        out = torch.empty((n_seg, k), dtype=torch.int32, device=scores.device)
    _lib.call("std_topk_select", scores.data_ptr(), P, n_seg, visual_pos.data_ptr(), visual_pos.numel(), k,
              out.data_ptr(), _stream())
    return out


def compact_gather(dense_cache: torch.Tensor, sparse_cache: torch.Tensor, b: int, non_visual: torch.Tensor,
                   topk: torch.Tensor):
    """caches [layers, 2, B, Hkv, cap, D]; non_visual [NV] int32; topk [layers, Hkv, K] int32."""
    layers, _, B, Hkv, cap_d, D = dense_cache.shape
    cap_s = sparse_cache.shape[4]
    _check(dense_cache, torch.bfloat16, "dense_cache")
    _check(sparse_cache, torch.bfloat16, "sparse_cache")
    _check(non_visual, torch.int32, "non_visual")
    _check(topk, torch.int32, "topk")
    _lib.call("std_compact_gather", dense_cache.data_ptr(), sparse_cache.data_ptr(), layers, B, b, Hkv, D, cap_d,
              cap_s, non_visual.data_ptr(), non_visual.numel(), topk.data_ptr(), topk.shape[-1], _stream())


# ----------------------------------------------------------------------------
# decoder pieces
# ----------------------------------------------------------------------------

def embed(table: torch.Tensor, tok: torch.Tensor, tok_start: int, n: int, out: torch.Tensor):
    B, stride = tok.shape
    _lib.call("std_embed", table.data_ptr(), table.shape[0], table.shape[1], tok.data_ptr(), stride, tok_start, n, B,
              out.data_ptr(), _stream())
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor):
    H = x.shape[-1]
    M = x.numel() // H
    _lib.call("std_rmsnorm", x.data_ptr(), w.data_ptr(), float(eps), M, H, out.data_ptr(), _stream())
    return out


def gemm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, bias: Optional[torch.Tensor] = None):
    """out[M, N] = x[M, K] @ w[N, K]^T (+ bias) on the tcgen05 weight-streaming GEMM (M <= 256)."""
    M, K = x.shape
    N = w.shape[0]
    _check(x, torch.bfloat16, "x")
    _check(w, torch.bfloat16, "w")
    _check(out, torch.bfloat16, "out")
    nb = _lib.query("std_gemm_workspace_bytes", M, N, K)
    ws = workspace("gemm", nb, x.device) if nb > 0 else None
    _lib.call("std_gemm_bf16", x.data_ptr(), w.data_ptr(), _p(bias), out.data_ptr(), M, N, K, _p(ws),
              0 if ws is None else ws.numel(), _stream())
    return out


def gemm_add_rmsnorm(x: torch.Tensor, w: torch.Tensor, resid: torch.Tensor, norm_w: Optional[torch.Tensor],
                     eps: float, out: Optional[torch.Tensor], bias: Optional[torch.Tensor] = None):
    """resid <- bf16(resid + x @ w^T (+ bias)); out = rmsnorm(resid) * norm_w (norm_w None: add only).

    One GEMM plus one fused epilogue kernel; equal to gemm() then add_rmsnorm()."""
    M, K = x.shape
    N = w.shape[0]
    for t, n in ((x, "x"), (w, "w"), (resid, "resid")):
        _check(t, torch.bfloat16, n)
    nb = _lib.query("std_gemm_epilogue_workspace_bytes", M, N, K)
    ws = workspace("gemm", nb, x.device)
    _lib.call("std_gemm_add_rmsnorm", x.data_ptr(), w.data_ptr(), _p(bias), resid.data_ptr(), _p(norm_w), float(eps),
              _p(out), M, N, K, ws.data_ptr(), ws.numel(), _stream())
    return out


def gemm_argmax(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, rows_out: Optional[int] = None, n: int = 1,
                out_stride: int = 1, out_start: int = 0, margin_out: Optional[torch.Tensor] = None):
    """Greedy argmax of x @ w^T's bf16 rows (lm_head + argmax) without storing the logits.

    Result t (< rows_out, default all rows) goes to out[(t//n)*out_stride + out_start + t%n];
    with margin_out (fp32, same indexing) also the row's top-1 minus top-2 logit."""
    M, K = x.shape
    N = w.shape[0]
    _check(x, torch.bfloat16, "x")
    _check(w, torch.bfloat16, "w")
    _check(out, torch.int32, "out")
    rows_out = M if rows_out is None else rows_out
    keys = workspace("argmax_keys", M * 8, x.device)  # zero-initialised, left zero by every call
    nb = _lib.query("std_gemm_epilogue_workspace_bytes", M, N, K)
    ws = workspace("gemm", nb, x.device)
    if margin_out is not None:
        _check(margin_out, torch.float32, "margin_out")
    _lib.call("std_gemm_argmax", x.data_ptr(), w.data_ptr(), M, N, K, rows_out, n, out_stride, out_start,
              out.data_ptr(), _p(margin_out), keys.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    return out


def gemm_rope_append(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], B: int, n: int, Hq: int,
                     Hkv: int, D: int, pos_base: torch.Tensor, pos_off: int, slot_base: torch.Tensor, slot_off: int,
                     cos_t: torch.Tensor, sin_t: torch.Tensor, q_out: torch.Tensor, k_cache: torch.Tensor,
                     v_cache: torch.Tensor):
    """qkv = x @ w^T + bias, then rope_append on it, as one GEMM + one fused epilogue kernel."""
    M, K = x.shape
    N = w.shape[0]
    if M != B * n or N != (Hq + 2 * Hkv) * D:
        raise ValueError("gemm_rope_append: x rows must be B*n and w rows (Hq + 2 Hkv) * D")
    _check(x, torch.bfloat16, "x")
    _check(w, torch.bfloat16, "w")
    cap = k_cache.shape[-2]
    nb = _lib.query("std_gemm_epilogue_workspace_bytes", M, N, K)
    ws = workspace("gemm", nb, x.device)
    _lib.call("std_gemm_rope_append", x.data_ptr(), w.data_ptr(), _p(bias), K, B, n, Hq, Hkv, D, pos_base.data_ptr(),
              int(pos_off), slot_base.data_ptr(), int(slot_off), cos_t.data_ptr(), sin_t.data_ptr(), cos_t.shape[0],
              q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), cap, ws.data_ptr(), ws.numel(), _stream())
    return q_out


def add_rmsnorm(x: torch.Tensor, delta: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor):
    """x <- x + delta (bf16, in place); out = rmsnorm(x) * w."""
    H = x.shape[-1]
    M = x.numel() // H
    _lib.call("std_add_rmsnorm", x.data_ptr(), delta.data_ptr(), w.data_ptr(), float(eps), M, H, out.data_ptr(),
              _stream())
    return out


def rope_append(qkv: torch.Tensor, B: int, n: int, Hq: int, Hkv: int, D: int, pos_base: torch.Tensor, pos_off: int,
                slot_base: torch.Tensor, slot_off: int, cos_t: torch.Tensor, sin_t: torch.Tensor,
                q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor):
    cap = k_cache.shape[-2]
    _lib.call("std_rope_append", qkv.data_ptr(), B, n, Hq, Hkv, D, pos_base.data_ptr(), int(pos_off),
              slot_base.data_ptr(), int(slot_off), cos_t.data_ptr(), sin_t.data_ptr(), cos_t.shape[0],
              q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), cap, _stream())
    return q_out


def silu_mul(gu: torch.Tensor, out: torch.Tensor, interleaved: bool = False):
    """out = silu(gate) * up; gu columns [gate | up] or 64-feature [gate | up] blocks (interleaved)."""
    I2 = gu.shape[-1]
    M = gu.numel() // I2
    _lib.call("std_silu_mul", gu.data_ptr(), M, I2 // 2, 1 if interleaved else 0, out.data_ptr(), _stream())
    return out


def gemm_silu_mul(x: torch.Tensor, w_gu: torch.Tensor, out: torch.Tensor):
    """out[M, I] = silu(x @ gate^T) * (x @ up^T) with w_gu [2I, K] in 64-row [gate | up] blocks."""
    M, K = x.shape
    N = w_gu.shape[0]
    _check(x, torch.bfloat16, "x")
    _check(w_gu, torch.bfloat16, "w_gu")
    _check(out, torch.bfloat16, "out")
    nb = _lib.query("std_gemm_epilogue_workspace_bytes", M, N, K)
    ws = workspace("gemm", nb, x.device)
    _lib.call("std_gemm_silu_mul", x.data_ptr(), w_gu.data_ptr(), M, N // 2, K, out.data_ptr(), ws.data_ptr(),
              ws.numel(), _stream())
    return out


def add(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor):
    _lib.call("std_add", a.data_ptr(), b.data_ptr(), a.numel(), out.data_ptr(), _stream())
    return out


def argmax_rows(logits: torch.Tensor, out: torch.Tensor, n: int = 1, out_stride: int = 1, out_start: int = 0):
    V = logits.shape[-1]
    rows = logits.numel() // V
    _lib.call("std_argmax_rows", logits.data_ptr(), rows, V, n, out_stride, out_start, out.data_ptr(), _stream())
    return out


def device_error() -> int:
    return _lib.device_error()
