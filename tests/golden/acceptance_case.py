"""The reduced random-init decoder and inputs of the acceptance comparison.

TEST INFRASTRUCTURE.  make_acceptance.py loads these weights into the
reference's own Qwen2.5-VL modules and records what its STD / AR decoding
does on CPU (fixture acceptance_reduced.npz); tests/test_decode_gpu.py runs
the B200 path on the same weights and inputs and compares.

The decoder has the 7B's per-layer geometry where the kernels need it (7
query heads per KV head, head_dim 128, the real vocabulary) at reduced depth
and width, random init std 0.02 as in the configs (HF init: zero biases, unit
norms).  The prompt keeps configs[4]'s ratio of selected to visual tokens:
K = 112 of 4096 visual (configs[4]: 896 of 32768), 128 text tokens, so
K+text = 240.  Draw order: one torch CPU generator per tensor group, seeded
from SEED, in the order listed in state_dict()."""

from __future__ import annotations

import torch

SEED = 7
LAYERS, HIDDEN, INTER, HEADS, KV_HEADS, VOCAB = 4, 896, 4864, 7, 1, 152064
VISUAL, TEXT, K_PLUS_TEXT, GAMMA, MAX_NEW = 4096, 128, 240, 9, 32
REQUEST_SEEDS = (600, 601)
VIDEO_TOKEN_ID = 151656
STD = 0.02


def decoder_config():
    from std_b200.model import DecoderConfig

    return DecoderConfig(vocab_size=VOCAB, hidden_size=HIDDEN, intermediate_size=INTER, num_hidden_layers=LAYERS,
                         num_attention_heads=HEADS, num_key_value_heads=KV_HEADS)


def state_dict():
    """Reference-named weights (fp32, CPU)."""
    g = torch.Generator().manual_seed(SEED)
    D = HIDDEN // HEADS

    def normal(*shape):
        return torch.randn(*shape, generator=g) * STD

    sd = {"model.embed_tokens.weight": normal(VOCAB, HIDDEN)}
    for i in range(LAYERS):
        p = f"model.layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = normal(HEADS * D, HIDDEN)
        sd[p + "self_attn.k_proj.weight"] = normal(KV_HEADS * D, HIDDEN)
        sd[p + "self_attn.v_proj.weight"] = normal(KV_HEADS * D, HIDDEN)
        sd[p + "self_attn.o_proj.weight"] = normal(HIDDEN, HEADS * D)
        sd[p + "mlp.gate_proj.weight"] = normal(INTER, HIDDEN)
        sd[p + "mlp.up_proj.weight"] = normal(INTER, HIDDEN)
        sd[p + "mlp.down_proj.weight"] = normal(HIDDEN, INTER)
        for n, k in (("q", HEADS * D), ("k", KV_HEADS * D), ("v", KV_HEADS * D)):
            sd[p + f"self_attn.{n}_proj.bias"] = torch.zeros(k)
        sd[p + "input_layernorm.weight"] = torch.ones(HIDDEN)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(HIDDEN)
    sd["model.norm.weight"] = torch.ones(HIDDEN)
    sd["lm_head.weight"] = normal(VOCAB, HIDDEN)
    return sd


def request(i: int):
    """(input_ids [1, P] int64, visual embeddings [V, H] fp32) of request i."""
    g = torch.Generator().manual_seed(REQUEST_SEEDS[i])
    ids = torch.full((1, VISUAL + TEXT), VIDEO_TOKEN_ID, dtype=torch.long)
    ids[0, VISUAL:] = torch.randint(0, 151643, (TEXT,), generator=g)
    vis = torch.randn(VISUAL, HIDDEN, generator=g)
    return ids, vis
