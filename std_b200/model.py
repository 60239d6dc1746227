"""Qwen2.5-VL-7B-shaped language decoder for the STD decode path.

Mirrors the reference's Qwen2.5-VL language model (modeling_qwen2_5_vl.py:
Qwen2_5_VLModel.forward :1301-1469, Qwen2_5_VLDecoderLayer :1156-1221,
Qwen2_5_VLSdpaAttention :1007-1140, Qwen2MLP :674-687, Qwen2RMSNorm :183-197)
with the vision tower left out: visual positions take precomputed embeddings.
Positions are 1-D (the fork disables get_rope_index, :2074-2105), so M-RoPE
reduces to ordinary RoPE with theta = 1e6.

Compute split:
  * decode forwards: every kernel is from libstd_b200.so -- the tcgen05
    weight-streaming GEMM for projections, MLP and lm_head, RMSNorm (fused
    with the residual add and the split-K sum), RoPE + KV append (fused with
    the split-K sum), draft / verify attention, SiLU*up, lm_head fused with
    the greedy argmax;
  * prefill (thousands of rows): cuBLAS GEMMs through torch and torch SDPA
    attention (library flash/efficient kernels), as the reference does.
Dense decode forwards (AR steps and verify) always run their GEMMs on the same
padded row count, and every other kernel on the decode path is row
independent, so a token gets bit-identical logits whether it is verified in a
block of gamma+1 or decoded alone -- the property STD == AR relies on.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn.functional as F

from . import ops


@dataclass
class DecoderConfig:
    vocab_size: int = 152064
    hidden_size: int = 3584
    intermediate_size: int = 18944
    num_hidden_layers: int = 28
    num_attention_heads: int = 28
    num_key_value_heads: int = 4
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    initializer_range: float = 0.02
    mrope_section: tuple = (16, 24, 24)

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def qkv_size(self) -> int:
        return (self.num_attention_heads + 2 * self.num_key_value_heads) * self.head_dim


QWEN25_VL_7B = DecoderConfig()
# smallest decoder the kernels accept (7 query heads per KV head, head_dim 128)
TINY = DecoderConfig(vocab_size=1024, hidden_size=896, intermediate_size=1536, num_hidden_layers=2,
                     num_attention_heads=7, num_key_value_heads=1)


class LayerWeights:
    __slots__ = ("w_in", "w_qkv", "b_qkv", "w_o", "w_post", "w_gu", "w_down")


class Qwen25VLDecoder:
    """Random-init decoder weights (HF init: N(0, std) linears/embeddings, zero
    biases, unit norms) generated on the GPU from one seed."""

    def __init__(self, config: DecoderConfig = QWEN25_VL_7B, seed: int = 2, device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16):
        if config.num_attention_heads != 7 * config.num_key_value_heads or config.head_dim != 128:
            raise ValueError("the STD kernels are built for 7 query heads per KV head and head_dim 128")
        self.config = config
        self.device = torch.device(device)
        self.dtype = dtype
        c = config
        g = torch.Generator(device=self.device).manual_seed(seed)
        std = c.initializer_range

        def normal(*shape):
            return (torch.randn(*shape, generator=g, device=self.device, dtype=torch.float32) * std).to(dtype)

        self.embed = normal(c.vocab_size, c.hidden_size)
        self.layers: List[LayerWeights] = []
        H, I = c.hidden_size, c.intermediate_size
        for _ in range(c.num_hidden_layers):
            lw = LayerWeights()
            lw.w_in = torch.ones(H, device=self.device, dtype=dtype)
            lw.w_qkv = normal(c.qkv_size, H)
            lw.b_qkv = torch.zeros(c.qkv_size, device=self.device, dtype=dtype)
            lw.w_o = normal(H, H)
            lw.w_post = torch.ones(H, device=self.device, dtype=dtype)
            # gate_proj and up_proj rows interleaved in 64-row blocks
            # [gate 64 | up 64] (a checkpoint loader permutes them so), so one
            # 128-row GEMM tile yields both halves of 64 features
            lw.w_gu = normal(2 * I, H)
            lw.w_down = normal(H, I)
            self.layers.append(lw)
        self.norm = torch.ones(H, device=self.device, dtype=dtype)
        self.lm_head = normal(c.vocab_size, H)
        self._rope_len = 0
        self.cos_t = self.sin_t = None

    # ------------------------------------------------------------------ checkpoints
    @classmethod
    def from_state_dict(cls, config: DecoderConfig, state: dict, device: str = "cuda",
                        dtype: torch.dtype = torch.bfloat16) -> "Qwen25VLDecoder":
        """Build the decoder from a Qwen2.5-VL language-model state dict with
        the reference's parameter names (modeling_qwen2_5_vl.py: embed_tokens,
        layers.{i}.self_attn.{q,k,v,o}_proj, layers.{i}.mlp.{gate,up,down}_proj,
        layers.{i}.{input,post_attention}_layernorm, norm; lm_head), an
        optional "model." prefix allowed.  q/k/v are fused into one matrix
        (+ bias) and gate/up interleaved in 64-row [gate | up] blocks."""
        self = cls.__new__(cls)
        if config.num_attention_heads != 7 * config.num_key_value_heads or config.head_dim != 128:
            raise ValueError("the STD kernels are built for 7 query heads per KV head and head_dim 128")
        self.config, self.device, self.dtype = config, torch.device(device), dtype

        def get(name):
            for key in (name, "model." + name, "model.language_model." + name):
                if key in state:
                    return state[key].to(device=self.device, dtype=dtype).contiguous()
            raise KeyError(name)

        c = config
        I = c.intermediate_size
        self.embed = get("embed_tokens.weight")
        self.layers = []
        for i in range(c.num_hidden_layers):
            pre = f"layers.{i}."
            lw = LayerWeights()
            lw.w_in = get(pre + "input_layernorm.weight")
            lw.w_post = get(pre + "post_attention_layernorm.weight")
            att = pre + "self_attn."
            lw.w_qkv = torch.cat([get(att + "q_proj.weight"), get(att + "k_proj.weight"),
                                  get(att + "v_proj.weight")]).contiguous()
            lw.b_qkv = torch.cat([get(att + "q_proj.bias"), get(att + "k_proj.bias"), get(att + "v_proj.bias")])
            lw.w_o = get(att + "o_proj.weight")
            gate, up = get(pre + "mlp.gate_proj.weight"), get(pre + "mlp.up_proj.weight")
            lw.w_gu = torch.stack([gate.view(I // 64, 64, -1), up.view(I // 64, 64, -1)], 1).reshape(2 * I, -1)
            lw.w_gu = lw.w_gu.contiguous()
            lw.w_down = get(pre + "mlp.down_proj.weight")
            self.layers.append(lw)
        self.norm = get("norm.weight")
        self.lm_head = get("lm_head.weight") if any(k.endswith("lm_head.weight") for k in state) else self.embed
        self._rope_len = 0
        self.cos_t = self.sin_t = None
        return self

    # ------------------------------------------------------------------ rope
    def rope_tables(self, max_pos: int):
        """cos/sin [max_pos, D/2] bf16: inv_freq = theta^(-2i/D) (fp32), angle =
        pos * inv_freq (fp32), cast to bf16 (modeling_qwen2_5_vl.py:638-671)."""
        if self._rope_len < max_pos:
            D = self.config.head_dim
            inv = 1.0 / (self.config.rope_theta ** (torch.arange(0, D, 2, dtype=torch.int64, device=self.device)
                                                    .float() / D))
            ang = torch.arange(max_pos, device=self.device, dtype=torch.float32)[:, None] * inv[None, :]
            self.cos_t = ang.cos().to(self.dtype).contiguous()
            self.sin_t = ang.sin().to(self.dtype).contiguous()
            self._rope_len = max_pos
        return self.cos_t, self.sin_t

    def num_params(self) -> int:
        n = self.embed.numel() + self.norm.numel() + self.lm_head.numel()
        for lw in self.layers:
            n += sum(getattr(lw, s).numel() for s in LayerWeights.__slots__)
        return n


class Workspace:
    """Static activation buffers for decode forwards of up to `rows` tokens."""

    def __init__(self, model: Qwen25VLDecoder, rows: int):
        c = model.config
        d, dt = model.device, model.dtype
        self.rows = rows
        self.x = torch.zeros(rows, c.hidden_size, device=d, dtype=dt)
        self.h = torch.zeros(rows, c.hidden_size, device=d, dtype=dt)
        self.qkv = torch.zeros(rows, c.qkv_size, device=d, dtype=dt)
        self.q = torch.zeros(rows, c.num_attention_heads, c.head_dim, device=d, dtype=dt)
        self.attn = torch.zeros(rows, c.hidden_size, device=d, dtype=dt)
        self.o = torch.zeros(rows, c.hidden_size, device=d, dtype=dt)
        self.act = torch.zeros(rows, c.intermediate_size, device=d, dtype=dt)


def decode_forward(model: Qwen25VLDecoder, ws: Workspace, cache: torch.Tensor, *, B: int, n: int, rows: int,
                   tok: torch.Tensor, tok_start: int, pos_base: torch.Tensor, pos_off: int, slot_base: torch.Tensor,
                   slot_off: int, lens: torch.Tensor, len_offset: int, sparse: bool,
                   argmax_out: Optional[torch.Tensor], argmax_stride: int = 1, argmax_start: int = 0,
                   dense_attn=None, sparse_index=None, collector=None,
                   margin_out: Optional[torch.Tensor] = None) -> None:
    """One forward of n new tokens per request through all layers (graph-capturable).

    cache: [layers, 2, B, Hkv, cap, D].  sparse=True uses the draft kernel
    (q_len = 1, no mask); otherwise the verify kernel (causal over the n new
    tokens).  GEMMs run on `rows` >= B*n rows (the fixed padded count for dense
    forwards).  The argmax of each new token's logits goes to
    argmax_out[b*argmax_stride + argmax_start + j]; argmax_out=None skips the
    final norm and lm_head (a draft step whose prediction is never used).  dense_attn (a
    seq_shard.ShardExchange on the owner rank) replaces the local verify
    kernel by the sequence-sharded attention over every rank's key range.
    sparse_index = (dense cache, selection [layers, B, Hkv, n_idx] int32):
    the draft reads its prompt rows from the dense cache by position and
    `cache` holds only the generated tokens' draft-path K/V (the tail).
    collector(li, q [B, n, Hq, D]) observes each layer's queries of a dense
    forward (verification-guided re-selection).  margin_out (fp32, indexed
    like argmax_out) receives each row's top-1 minus top-2 logit.
    """
    c = model.config
    M = B * n
    Hq, Hkv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
    eps = c.rms_norm_eps
    cos_t, sin_t = model.cos_t, model.sin_t
    x, h = ws.x[:rows], ws.h[:rows]
    if dense_attn is not None and not sparse:
        dense_attn.begin(n)
    # Eight launches per layer: QKV GEMM -> [split-K sum + bias + RoPE + KV
    # append] -> attention -> O GEMM -> [split-K sum + residual + RMSNorm] ->
    # gate/up GEMM with SiLU*up in its epilogue -> down GEMM -> [split-K sum +
    # residual + the next RMSNorm]; the bracketed steps are one small kernel
    # each, reading the GEMM's split partials from L2.
    ops.embed(model.embed, tok, tok_start, n, ws.x[:M])
    ops.rmsnorm(x, model.layers[0].w_in, eps, h)
    n_layers = len(model.layers)
    for li, lw in enumerate(model.layers):
        kc, vc = cache[li, 0], cache[li, 1]
        if rows == M:
            ops.gemm_rope_append(h, lw.w_qkv, lw.b_qkv, B, n, Hq, Hkv, D, pos_base, pos_off, slot_base, slot_off,
                                 cos_t, sin_t, ws.q[:M], kc, vc)
        else:  # padded rows: the GEMM runs on `rows`, RoPE on the M real ones
            ops.gemm(h, lw.w_qkv, ws.qkv[:rows], lw.b_qkv)
            ops.rope_append(ws.qkv[:M], B, n, Hq, Hkv, D, pos_base, pos_off, slot_base, slot_off, cos_t, sin_t,
                            ws.q[:M], kc, vc)
        if sparse and sparse_index is not None:
            dense, sel = sparse_index
            ops.draft_attention_indexed(ws.q[:M], dense[li, 0], dense[li, 1], sel[li], kc, vc, lens, len_offset,
                                        out=ws.attn[:M].view(B, Hq, D))
        elif sparse:
            ops.draft_attention(ws.q[:M], kc, vc, lens, len_offset, out=ws.attn[:M].view(B, Hq, D),
                                after_append=True)
        elif dense_attn is not None:
            dense_attn.attend(li, ws.q[:M].view(B, n, Hq, D), kc, vc, lens, len_offset, ws.attn[:M].view(B, n, Hq, D))
        else:
            ops.verify_attention(ws.q[:M].view(B, n, Hq, D), kc, vc, lens, len_offset,
                                 out=ws.attn[:M].view(B, n, Hq, D))
        if collector is not None and not sparse:
            collector(li, ws.q[:M].view(B, n, Hq, D))
        ops.gemm_add_rmsnorm(ws.attn[:rows], lw.w_o, x, lw.w_post, eps, h)
        ops.gemm_silu_mul(h, lw.w_gu, ws.act[:rows])
        if li + 1 < n_layers:
            next_norm = model.layers[li + 1].w_in
        else:  # the final norm feeds lm_head; a draft step without lm_head only adds
            next_norm = model.norm if argmax_out is not None else None
        ops.gemm_add_rmsnorm(ws.act[:rows], lw.w_down, x, next_norm, eps, h)
    if argmax_out is None:
        return
    ops.gemm_argmax(h, model.lm_head, argmax_out, rows_out=M, n=n, out_stride=argmax_stride, out_start=argmax_start,
                    margin_out=margin_out)


# ---------------------------------------------------------------------- prefill
def _sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, mask: Optional[torch.Tensor]):
    # q [S, Hq, D], k/v [Hkv, L, D] -> [S, Hq, D]
    G = q.shape[1] // k.shape[0]
    qh = q.permute(1, 0, 2).unsqueeze(0)
    kh = k.repeat_interleave(G, dim=0).unsqueeze(0)
    vh = v.repeat_interleave(G, dim=0).unsqueeze(0)
    o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, is_causal=causal)
    return o[0].permute(1, 0, 2)


def prefill_segment(model: Qwen25VLDecoder, cache: torch.Tensor, b: int, x: torch.Tensor, start: int,
                    selection: Optional[dict] = None, chunk: int = 8192) -> torch.Tensor:
    """Run rows [start, start+S) of request b's prompt through the decoder.

    x [S, H] bf16 holds the input embeddings (consumed).  K/V of the segment
    land in cache[..., b, :, start:start+S].  Attention: causal over keys
    0..start+row (the reference's _make_causal_mask with past length `start`,
    modeling_qwen2_5_vl.py:65-101).  With `selection` (the STD selection
    branch, std_qwen25vl.py:689 + modeling_qwen2_5_vl.py:1115-1123) each
    layer's scores are computed from the segment's queries with the custom
    precision chain (ops.select_scores) into selection["scores"][layer], and the
    attention output is probs @ V from those fp16 probabilities.
    Returns the final hidden state of the last row (normed), [1, H].
    """
    c = model.config
    S = x.shape[0]
    Hq, Hkv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
    dev = model.device
    cos_t, sin_t = model.rope_tables(max(model._rope_len, start + S + 1))
    zero = torch.zeros(1, dtype=torch.int32, device=dev)
    L = start + S
    for li, lw in enumerate(model.layers):
        kc = cache[li, 0, b:b + 1]
        vc = cache[li, 1, b:b + 1]
        h = torch.empty_like(x)
        ops.rmsnorm(x, lw.w_in, c.rms_norm_eps, h)
        q = torch.empty(S, Hq, D, device=dev, dtype=model.dtype)
        for s0 in range(0, S, chunk):
            s1 = min(S, s0 + chunk)
            qkv = torch.addmm(lw.b_qkv, h[s0:s1], lw.w_qkv.t())
            ops.rope_append(qkv, 1, s1 - s0, Hq, Hkv, D, zero, start + s0, zero, start + s0, cos_t, sin_t,
                            q[s0:s1], kc, vc)
        del h
        k_all = kc[0, :, :L]
        v_all = vc[0, :, :L]
        if selection is not None:
            sc, probs = ops.select_scores(q, cache[li, 0, b], L, start, scores=selection["scores"][li],
                                          write_probs=True)
            if selection.get("observe") is not None:  # (layer, post-RoPE text queries, K rows, keys, first query pos)
                selection["observe"](li, q, cache[li, 0, b], L, start)
            G = Hq // Hkv
            # probs [Hq, S, L] fp16 @ V [Hkv, L, D] in fp32: one batched matmul
            # over the KV groups (the G heads of a group share its V)
            pr = probs.float().reshape(Hkv, G * S, L)
            o = torch.bmm(pr, v_all.float())                 # [Hkv, G*S, D]
            attn = o.view(Hq, S, D).permute(1, 0, 2).to(model.dtype).contiguous()
        elif start == 0:
            attn = _sdpa(q, k_all, v_all, causal=True, mask=None)
        else:
            keep = torch.arange(L, device=dev)[None, :] <= (start + torch.arange(S, device=dev))[:, None]
            attn = _sdpa(q, k_all, v_all, causal=False, mask=keep)
        del q
        o = attn.reshape(S, c.hidden_size) @ lw.w_o.t()
        x = x + o
        del attn, o
        h = torch.empty_like(x)
        ops.rmsnorm(x, lw.w_post, c.rms_norm_eps, h)
        for s0 in range(0, S, chunk):
            s1 = min(S, s0 + chunk)
            gu = h[s0:s1] @ lw.w_gu.t()
            act = torch.empty(s1 - s0, c.intermediate_size, device=dev, dtype=model.dtype)
            ops.silu_mul(gu, act, interleaved=True)
            x[s0:s1] = x[s0:s1] + act @ lw.w_down.t()
            del gu, act
        del h
    last = torch.empty(1, c.hidden_size, device=dev, dtype=model.dtype)
    ops.rmsnorm(x[-1:].contiguous(), model.norm, c.rms_norm_eps, last)
    return last


def prefill_request(model: Qwen25VLDecoder, cache: torch.Tensor, b: int, embeds: torch.Tensor, text_start: int,
                    scores_out: Optional[torch.Tensor] = None, observe=None) -> int:
    """Two-stage prefill of one request (std_qwen25vl.py:670-707).

    1. video prefix rows [0, text_start) -> cache;
    2. if scores_out [layers, Hkv, P] is given: the selection branch over the
       text suffix (its K/V are written to the cache and then overwritten);
    3. the dense branch over the text suffix (the canonical verifier KV).
    observe(layer, q_text, k_rows, P, q_start), if given, sees each layer's
    selection inputs right after its scores are computed (for parity checks).
    Returns the prefill's greedy next token (dense_next).
    """
    P = embeds.shape[0]
    prefill_segment(model, cache, b, embeds[:text_start].clone(), 0)
    if scores_out is not None:
        prefill_segment(model, cache, b, embeds[text_start:].clone(), text_start,
                        selection={"scores": scores_out, "observe": observe})
    last = prefill_segment(model, cache, b, embeds[text_start:].clone(), text_start)
    logits = last @ model.lm_head.t()
    out = torch.empty(1, dtype=torch.int32, device=model.device)
    ops.argmax_rows(logits.contiguous(), out)
    return int(out.item())
