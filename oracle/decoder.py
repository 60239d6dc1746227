"""CPU (numpy fp32) restatement of the STD decode loop -- the timed CPU baseline.

TEST / BASELINE INFRASTRUCTURE ONLY (see oracle/__init__.py).  bench.py's
``--impl reference`` arm and its ``cpu_baseline`` leg run this on the host
cores; the product path never imports it.

It restates, for one request, the reference's decode round
(std_qwen25vl.py:766-940): gamma sparse draft forwards over the compacted
sparse cache (_draft_tokens :531-550, draft attention :406-417), one parallel
dense verify forward over the full cache (:795-806, causal mask
modeling_qwen2_5_vl.py:65-101), greedy acceptance (:806-815) and the bonus
sparse forward (:931-939), through a Qwen2.5-VL decoder layer
(modeling_qwen2_5_vl.py:1156-1221: RMSNorm, q/k/v projections with bias,
RoPE, GQA attention, o_proj, SwiGLU MLP).

Bounded sample: prefill is not part of the metric (decoding_time,
std_qwen25vl.py:762-763), so the caches start from a seeded synthetic state of
the workload's lengths, and -- to keep host memory to a few GB -- all
`num_layers` decoder layers share one set of random fp32 weights (same
arithmetic and memory traffic per token as distinct layers; values differ).
"""

from __future__ import annotations

import math
import time
from typing import Dict, List, Optional

import numpy as np

from . import accept_round


def _rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    var = np.mean(x * x, axis=-1, keepdims=True)
    return (x / np.sqrt(var + eps)) * w


def _rope(x: np.ndarray, pos: np.ndarray, inv_freq: np.ndarray) -> np.ndarray:
    # x [S, H, D], pos [S]
    ang = pos[:, None].astype(np.float32) * inv_freq[None, :]
    c = np.cos(np.concatenate([ang, ang], -1))[:, None, :]
    s = np.sin(np.concatenate([ang, ang], -1))[:, None, :]
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], -1)
    return x * c + rot * s


class NumpySTD:
    """One request's STD decode on CPU, fp32."""

    def __init__(self, hidden=3584, inter=18944, layers=28, heads=28, kv_heads=4, vocab=152064, L_dense=32896,
                 L_sparse=1024, max_new=128, gamma=9, seed=0, eps=1e-6, theta=1e6):
        rng = np.random.default_rng(seed)
        D = hidden // heads
        self.H, self.I, self.layers, self.Hq, self.Hkv, self.D = hidden, inter, layers, heads, kv_heads, D
        self.vocab, self.gamma, self.eps = vocab, gamma, eps
        std = np.float32(0.02)

        def normal(*shape):
            return rng.standard_normal(shape, dtype=np.float32) * std

        # embedding / lm_head rows repeat one random block (their values do not
        # change the cost; generating 2 x 545M normals would dominate setup)
        blk = normal(min(vocab, 8192), hidden)
        reps = -(-vocab // blk.shape[0])
        self.embed = np.ascontiguousarray(np.tile(blk, (reps, 1))[:vocab])
        self.w_qkv = normal((heads + 2 * kv_heads) * D, hidden)
        self.b_qkv = np.zeros((heads + 2 * kv_heads) * D, np.float32)
        self.w_o = normal(hidden, hidden)
        self.w_gu = normal(2 * inter, hidden)
        self.w_down = normal(hidden, inter)
        self.lm_head = np.ascontiguousarray(np.tile(normal(min(vocab, 8192), hidden), (reps, 1))[:vocab])
        self.inv_freq = (1.0 / theta ** (np.arange(0, D, 2, dtype=np.float32) / D)).astype(np.float32)
        cap_d, cap_s = L_dense + max_new + gamma + 2, L_sparse + max_new + gamma + 2
        # one synthetic K/V per cache, shared by every layer (cost-equivalent)
        self.kd = np.zeros((kv_heads, cap_d, D), np.float32)
        self.vd = np.zeros_like(self.kd)
        self.ks = np.zeros((kv_heads, cap_s, D), np.float32)
        self.vs = np.zeros_like(self.ks)
        self.kd[:, :L_dense] = rng.standard_normal((kv_heads, L_dense, D), dtype=np.float32)
        self.vd[:, :L_dense] = rng.standard_normal((kv_heads, L_dense, D), dtype=np.float32)
        self.ks[:, :L_sparse] = self.kd[:, L_dense - L_sparse:L_dense]
        self.vs[:, :L_sparse] = self.vd[:, L_dense - L_sparse:L_dense]
        self.dense_len, self.sparse_len, self.ctx = L_dense, L_sparse, L_dense

    # ---------------------------------------------------------------- forward
    def _attend(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, L: int, causal_n: int) -> np.ndarray:
        # q [S, Hq, D]; keys 0..L-1; causal over the last causal_n rows (0 = none)
        S = q.shape[0]
        G = self.Hq // self.Hkv
        out = np.empty_like(q)
        scale = np.float32(1.0 / math.sqrt(self.D))
        for kv in range(self.Hkv):
            qg = q[:, kv * G:(kv + 1) * G].reshape(S * G, self.D)
            s = (qg @ k[kv, :L].T) * scale
            if causal_n:
                lim = L - causal_n + np.repeat(np.arange(S), G)
                s = np.where(np.arange(L)[None, :] <= lim[:, None], s, -np.inf)
            s = s - s.max(-1, keepdims=True)
            e = np.exp(s)
            o = (e @ v[kv, :L]) / e.sum(-1, keepdims=True)
            out[:, kv * G:(kv + 1) * G] = o.reshape(S, G, self.D)
        return out

    def forward(self, tokens: List[int], pos0: int, sparse: bool) -> np.ndarray:
        """Append `tokens` at positions pos0.. and return their greedy argmax."""
        S = len(tokens)
        x = self.embed[np.asarray(tokens)]
        k, v = (self.ks, self.vs) if sparse else (self.kd, self.vd)
        slot = self.sparse_len if sparse else self.dense_len
        pos = pos0 + np.arange(S)
        Hq, Hkv, D = self.Hq, self.Hkv, self.D
        for _ in range(self.layers):
            h = _rmsnorm(x, 1.0, self.eps)
            qkv = h @ self.w_qkv.T + self.b_qkv
            q = _rope(qkv[:, : Hq * D].reshape(S, Hq, D), pos, self.inv_freq)
            kk = _rope(qkv[:, Hq * D:(Hq + Hkv) * D].reshape(S, Hkv, D), pos, self.inv_freq)
            k[:, slot:slot + S] = kk.transpose(1, 0, 2)
            v[:, slot:slot + S] = qkv[:, (Hq + Hkv) * D:].reshape(S, Hkv, D).transpose(1, 0, 2)
            a = self._attend(q, k, v, slot + S, 0 if sparse else S)
            x = x + a.reshape(S, Hq * D) @ self.w_o.T
            h = _rmsnorm(x, 1.0, self.eps)
            gu = h @ self.w_gu.T
            g = gu[:, : self.I]
            x = x + ((g / (1.0 + np.exp(-g))) * gu[:, self.I:]) @ self.w_down.T
        logits = _rmsnorm(x, 1.0, self.eps) @ self.lm_head.T
        return logits.argmax(-1)

    # ---------------------------------------------------------------- decode
    def std_round(self, sparse_next: int, pending: List[int], dense_next: int, remaining: int):
        """One round; returns (appended tokens, accept_len, new sparse_next, new pending)."""
        gamma = min(self.gamma, remaining)
        draft, tok = [], sparse_next
        s0 = self.sparse_len
        for i in range(gamma):
            draft.append(int(tok))
            tok = int(self.forward([tok], self.ctx + i, sparse=True)[0])
            self.sparse_len += 1
        self.sparse_len = s0
        preds = self.forward(pending + draft, self.ctx - len(pending), sparse=False).tolist()
        acc, bonus, app, _ = accept_round(draft, preds, dense_next, bool(pending), remaining, -1, True)
        self.dense_len += len(pending) + acc
        self.sparse_len = s0 + acc
        self.ctx += len(app)
        nxt = int(self.forward([bonus], self.ctx - 1, sparse=True)[0])
        self.sparse_len += 1
        return app, acc, nxt, [bonus]


def run_cpu_std(rounds: int, warmup: int = 1, **shape) -> Dict[str, float]:
    """Time `rounds` STD rounds on the host cores; returns tokens, seconds, cores."""
    try:
        from threadpoolctl import threadpool_info

        cores = max([int(i.get("num_threads", 1)) for i in threadpool_info()] or [1])
    except Exception:  # pragma: no cover
        import os

        cores = os.cpu_count() or 1
    m = NumpySTD(**shape)
    max_new = shape.get("max_new", 128)
    tok, pending, dense_next, gen = 1, [], 1, 0
    for _ in range(warmup):
        app, _, tok, pending = m.std_round(tok, pending, dense_next, max_new - gen)
        gen += len(app)
    t0 = time.perf_counter()
    n_tok = 0
    accepts = []
    for _ in range(rounds):
        app, acc, tok, pending = m.std_round(tok, pending, dense_next, max(1, max_new - gen))
        n_tok += len(app)
        gen += len(app)
        accepts.append(acc)
    dt = time.perf_counter() - t0
    return {"tokens": n_tok, "seconds": dt, "cores": cores, "rounds": rounds, "accepts": accepts}
