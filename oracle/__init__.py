"""CPU oracle for the STD sparse-to-dense decode path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only as the checker or as the timed CPU restatement.  The product
path (``std_b200``) never imports it and has no CPU fallback.

What is restated here (reference file:line in brackets):

* selection scores and top-K            [modeling_qwen2_5_vl.py:966-995,
                                          std_qwen25vl.py:175-231]
  -> C code in ``std_oracle.c`` (bit-exact specification, see that header).
* compaction indices                    [std_qwen25vl.py:265-298]
* draft attention (q_len=1, GQA)        [std_qwen25vl.py:406-417]
* parallel-verify attention (causal)    [modeling_qwen2_5_vl.py:65-101,
                                          :1096-1133]
* greedy acceptance / commit / rollback [std_qwen25vl.py:806-815, :910-931]
* verification collector v1             [dynamic_selection.py:290-308]

Parity status: the selection restatement is pinned against the reference's
own functions run on CPU (tests/golden/make_golden.py); attention against the
reference's SDPA call paths; acceptance against a recorded reference decode
trace.
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import List, Optional, Sequence, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile ``std_oracle.c`` into ``oracle/liboracle.so`` (gcc, no fast-math)."""
    import subprocess

    src = os.path.join(_HERE, "std_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        cmd = [
            "gcc", "-O2", "-mfma", "-ffp-contract=off", "-fno-fast-math", "-fopenmp",
            "-shared", "-fPIC", "-o", _LIB_PATH, src, "-lm",
        ]
        subprocess.check_call(cmd)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I = ctypes.c_int
        I64 = ctypes.c_int64
        F = ctypes.c_float
        L.oracle_exp.argtypes = [P, P, I64]
        L.oracle_f32_to_f16.argtypes = [P, P, I64]
        L.oracle_f32_to_bf16.argtypes = [P, P, I64]
        L.oracle_select_logits.argtypes = [P, P, I, I, I, I, I, I64, I, F, P]
        L.oracle_select_row_stats.argtypes = [P, I64, I, P, P]
        L.oracle_select_colsum.argtypes = [P, P, P, I, I, I, I, P]
        L.oracle_select_scores.argtypes = [P, P, I, I, I, I, I, I64, I, F, P, P, P, P]
        L.oracle_topk_lowest.argtypes = [P, I, I, P, I, I, P]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ----------------------------------------------------------------------------
# bf16 / fp16 helpers (numpy has no bf16: bf16 values travel as uint16 bits)
# ----------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_bf16(_ptr(x), _ptr(out), x.size)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_f16(_ptr(x), _ptr(out), x.size)
    return out


def std_exp(x: np.ndarray) -> np.ndarray:
    """The exp() used by the selection chain on both CPU and GPU."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().oracle_exp(_ptr(x), _ptr(y), x.size)
    return y


SELECT_SCALE = np.float32(1.0 / math.sqrt(128.0))


# ----------------------------------------------------------------------------
# (a) selection
# ----------------------------------------------------------------------------

def select_scores(q_bits: np.ndarray, k_bits: np.ndarray, q_start: int, P: int,
                  scale: Optional[float] = None, return_logits: bool = False):
    """Selection scores for one layer.

    q_bits: [T, Hq, D] bf16 bits; k_bits: [Hkv, >=P, D] bf16 bits.
    Row t sits at absolute position q_start + t and sees keys 0..q_start+t.
    Returns scores [Hkv, P] fp32 (and logits [Hq, T, P] fp16 bits, row m, row l).
    Follows modeling_qwen2_5_vl.py:983-992 and std_qwen25vl.py:214-218.
    """
    q_bits = np.ascontiguousarray(q_bits, dtype=np.uint16)
    k_bits = np.ascontiguousarray(k_bits, dtype=np.uint16)
    T, Hq, D = q_bits.shape
    Hkv, kstride, D2 = k_bits.shape
    assert D == D2 and Hq % Hkv == 0 and P <= kstride and D <= 512
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    logits = np.empty((Hq, T, P), dtype=np.uint16)
    m = np.empty((Hq * T,), dtype=np.float32)
    l = np.empty((Hq * T,), dtype=np.float32)
    scores = np.empty((Hkv, P), dtype=np.float32)
    lib().oracle_select_scores(_ptr(q_bits), _ptr(k_bits), T, Hq, Hkv, D, P, kstride, q_start,
                               float(np.float32(scale)), _ptr(logits), _ptr(m), _ptr(l), _ptr(scores))
    if return_logits:
        return scores, logits, m.reshape(Hq, T), l.reshape(Hq, T)
    return scores


def selection_budget(prompt_len: int, text_start: int, visual_len: int, target_k_plus_text: int = 1024,
                     explicit_k: Optional[int] = None) -> int:
    """k = K+text - text_len clamped to [1, visual_len]  (std_qwen25vl.py:190-195)."""
    text_len = max(1, prompt_len - int(text_start))
    k = int(explicit_k) if explicit_k is not None else max(1, int(target_k_plus_text) - text_len)
    return min(k, int(visual_len))


def topk_lowest(scores: np.ndarray, visual_pos: np.ndarray, k: int) -> np.ndarray:
    """Per KV head: k largest visual scores, ties to the lowest position; ascending.

    Mirrors std_qwen25vl.py:219-222 (index_select, topk, map, sort) with the
    tie rule made explicit.  scores [H, P] fp32, visual_pos [V] ascending.
    """
    scores = np.ascontiguousarray(scores, dtype=np.float32)
    vp = np.ascontiguousarray(visual_pos, dtype=np.int32)
    H, P = scores.shape
    out = np.empty((H, k), dtype=np.int32)
    lib().oracle_topk_lowest(_ptr(scores), H, P, _ptr(vp), vp.size, k, _ptr(out))
    return out


def compact_indices(non_visual: np.ndarray, topk_pos: np.ndarray) -> np.ndarray:
    """idx[h] = unique(sorted(non_visual U topk[h]))  (std_qwen25vl.py:283-288)."""
    rows = []
    for h in range(topk_pos.shape[0]):
        idx = np.unique(np.concatenate([non_visual.astype(np.int64), topk_pos[h].astype(np.int64)]))
        rows.append(idx)
    n = {r.size for r in rows}
    if len(n) != 1:
        raise RuntimeError("Compacted sparse KV produced an unexpected length.")
    return np.stack(rows).astype(np.int32)


# ----------------------------------------------------------------------------
# (b)/(c) attention
# ----------------------------------------------------------------------------

def draft_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, lens: Sequence[int]):
    """q [B, Hq, D]; k, v [B, Hkv, cap, D]; keys 0..lens[b]-1, no mask.

    Same op as F.scaled_dot_product_attention(q, k, v, enable_gqa=True) with
    q_len=1 (std_qwen25vl.py:409-417).  float64 math; returns (o, lse).
    """
    B, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    o = np.zeros((B, Hq, D), dtype=np.float64)
    lse = np.zeros((B, Hq), dtype=np.float64)
    scale = 1.0 / math.sqrt(D)
    for b in range(B):
        L = int(lens[b])
        for h in range(Hq):
            kk = k[b, h // G, :L].astype(np.float64)
            vv = v[b, h // G, :L].astype(np.float64)
            s = kk @ q[b, h].astype(np.float64) * scale
            mx = s.max()
            e = np.exp(s - mx)
            o[b, h] = e @ vv / e.sum()
            lse[b, h] = mx + math.log(e.sum())
    return o, lse


def verify_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, lens_after: Sequence[int],
                     kv_begin: int = 0, kv_end: Optional[int] = None):
    """q [B, nq, Hq, D]; k, v [B, Hkv, cap, D]; query t sees keys <= lens-nq+t.

    Same op as repeat_kv + F.sdpa(attn_mask=_make_causal_mask(...)) in the
    dense forward (modeling_qwen2_5_vl.py:65-101, :1096-1133).  Optionally
    restricted to keys [kv_begin, kv_end) to model one sequence shard; rows
    that see no key in the range get o = 0, lse = -inf.  float64.
    """
    B, nq, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    o = np.zeros((B, nq, Hq, D), dtype=np.float64)
    lse = np.full((B, nq, Hq), -np.inf, dtype=np.float64)
    scale = 1.0 / math.sqrt(D)
    for b in range(B):
        L = int(lens_after[b])
        for t in range(nq):
            hi = min(L - nq + t + 1, kv_end if kv_end is not None else L)
            lo = kv_begin
            if hi <= lo:
                continue
            for h in range(Hq):
                kk = k[b, h // G, lo:hi].astype(np.float64)
                vv = v[b, h // G, lo:hi].astype(np.float64)
                s = kk @ q[b, t, h].astype(np.float64) * scale
                mx = s.max()
                e = np.exp(s - mx)
                o[b, t, h] = e @ vv / e.sum()
                lse[b, t, h] = mx + math.log(e.sum())
    return o, lse


def collect_relevance(q: np.ndarray, k: np.ndarray, visual_pos: np.ndarray) -> np.ndarray:
    """RuntimeVerificationCollector._hook (dynamic_selection.py:290-308) in
    fp64: q [B, Hq, nq, D], k [B, Hkv, P, D] (any float dtype) ->
    [B, Hkv, V] = sum over the nq rows of softmax over the visual keys of
    (mean of the group's query heads . k) / sqrt(D)."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    B, Hq, nq, D = q.shape
    Hkv = k.shape[1]
    qk = q.reshape(B, Hkv, Hq // Hkv, nq, D).mean(axis=2)              # [B, Hkv, nq, D]
    kv = k[:, :, np.asarray(visual_pos, dtype=np.int64)]              # [B, Hkv, V, D]
    logits = np.einsum("bhtd,bhvd->bhtv", qk, kv) / math.sqrt(D)
    logits -= logits.max(axis=-1, keepdims=True)
    w = np.exp(logits)
    w /= w.sum(axis=-1, keepdims=True)
    return w.sum(axis=2)


def merge_partials(o_parts: Sequence[np.ndarray], lse_parts: Sequence[np.ndarray]):
    """Exact log-sum-exp merge of attention partials over disjoint key ranges."""
    lse_stack = np.stack(lse_parts)
    mx = np.max(lse_stack, axis=0)
    safe = np.where(np.isfinite(mx), mx, 0.0)
    w = np.where(np.isfinite(lse_stack), np.exp(lse_stack - safe), 0.0)
    tot = w.sum(axis=0)
    o = sum(wi[..., None] * oi for wi, oi in zip(w, o_parts)) / np.where(tot > 0, tot, 1.0)[..., None]
    lse = np.where(tot > 0, safe + np.log(np.where(tot > 0, tot, 1.0)), -np.inf)
    return o, lse


# ----------------------------------------------------------------------------
# (d) greedy acceptance, commit and rollback
# ----------------------------------------------------------------------------

def accept_round(draft: Sequence[int], verify_argmax: Sequence[int], dense_next: int, has_pending: bool,
                 remaining: int, eos_token_id: int, ignore_eos: bool):
    """One STD round's acceptance and commit (std_qwen25vl.py:806-815, :910-921).

    ``draft`` holds the proposed tokens (length propose_len = min(gamma,
    remaining)); ``verify_argmax`` the dense argmax of every verify row.
    Returns (accept_len, bonus, appended_tokens, finished).
    """
    if has_pending:
        preds = [int(x) for x in verify_argmax]
    else:
        preds = [int(dense_next)] + [int(x) for x in verify_argmax]
    accept = 0
    while accept < len(draft) and int(draft[accept]) == preds[accept]:
        accept += 1
    bonus = preds[accept]
    full = [int(x) for x in draft[:accept]] + [bonus]
    if not ignore_eos:
        for i, tok in enumerate(full):
            if tok == eos_token_id:
                full = full[: i + 1]
                break
    to_append = full[:remaining]
    reached_limit = len(to_append) >= remaining
    reached_eos = bool(not ignore_eos and to_append and to_append[-1] == eos_token_id)
    return accept, bonus, to_append, bool(reached_limit or reached_eos)


def rollback_lengths(dense_cached_len: int, pending_len: int, sparse_prev_len: int, accept: int):
    """Cache lengths kept after a round (std_qwen25vl.py:923-929)."""
    return dense_cached_len + pending_len + accept, sparse_prev_len + accept


def replay_std_rounds(drafts: List[List[int]], verify_preds: List[List[int]], dense_next: int,
                      max_new_tokens: int, gamma: int, eos_token_id: int, ignore_eos: bool):
    """Replay the STD commit logic over recorded (draft, verify) pairs.

    Returns (generated tokens, accept lengths, pending lengths).
    """
    generated: List[int] = []
    accepts: List[int] = []
    pendings: List[int] = []
    pending: List[int] = []
    for draft, preds in zip(drafts, verify_preds):
        remaining = max_new_tokens - len(generated)
        assert len(draft) == min(gamma, remaining)
        pendings.append(len(pending))
        acc, bonus, app, fin = accept_round(draft, preds, dense_next, bool(pending), remaining,
                                            eos_token_id, ignore_eos)
        accepts.append(acc)
        generated.extend(app)
        if fin:
            break
        pending = [bonus]
    return generated, accepts, pendings
