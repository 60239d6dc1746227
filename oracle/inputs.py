"""Seeded synthetic inputs for the single-layer STD op.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The reference defines no draw order for these tensors.  This build fixes it:
one ``torch.Generator().manual_seed(seed)`` on CPU, fp32 N(0,1) draws in the
order q_text -> k -> v -> q_draft -> q_verify.  The text query rows are the
last ``T`` prompt rows (the reference's selection queries are the prompt's text
suffix, std_qwen25vl.py:689 and :204-222); visual tokens occupy positions
0..V-1 and text tokens V..P-1, so text_start = V.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np
import torch

VIDEO_TOKEN_ID = 151656


@dataclass
class LayerCase:
    name: str
    V: int            # visual tokens (positions 0..V-1)
    text: int         # text tokens after the video
    T: int            # selection query rows (last T prompt rows)
    k_plus_text: int  # target K+text
    nq_verify: int = 10

    @property
    def P(self) -> int:
        return self.V + self.text

    @property
    def text_start(self) -> int:
        return self.V

    @property
    def q_start(self) -> int:
        return self.P - self.T

    @property
    def k(self) -> int:
        return min(max(1, self.k_plus_text - self.text), self.V)


CONFIG0 = LayerCase("config0", V=8192, text=256, T=64, k_plus_text=1024)
SMALL = LayerCase("small", V=512, text=32, T=16, k_plus_text=128)
# configs[3] selection sizes for one layer: 131072 visual + 128 text keys,
# 64 text query rows (the last prompt rows), K = 4096 - 128 = 3968
CONFIG3_LAYER = LayerCase("config3", V=131072, text=128, T=64, k_plus_text=4096)


def make_layer_inputs(case: LayerCase, seed: int = 0, Hq: int = 28, Hkv: int = 4, D: int = 128):
    g = torch.Generator().manual_seed(seed)
    q_text = torch.randn(1, Hq, case.T, D, generator=g)
    k = torch.randn(1, Hkv, case.P, D, generator=g)
    v = torch.randn(1, Hkv, case.P, D, generator=g)
    q_draft = torch.randn(1, Hq, 1, D, generator=g)
    q_verify = torch.randn(1, Hq, case.nq_verify, D, generator=g)
    return dict(q_text=q_text, k=k, v=v, q_draft=q_draft, q_verify=q_verify)


def input_ids_for(case: LayerCase) -> torch.Tensor:
    ids = torch.arange(case.P, dtype=torch.long) % 1000 + 1000
    ids[: case.V] = VIDEO_TOKEN_ID
    return ids.view(1, -1)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 bit pattern (uint16) of a tensor, after an RNE cast to bf16."""
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]
