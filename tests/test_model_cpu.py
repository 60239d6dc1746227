"""CPU: the decoder's checkpoint loader maps the reference's Qwen2.5-VL
parameter names onto the fused layouts the decode kernels read (q/k/v fused
with their biases, gate/up interleaved in 64-row blocks)."""
import torch

from std_b200.model import DecoderConfig, Qwen25VLDecoder


def _state(c, g):
    H, I = c.hidden_size, c.intermediate_size
    qd, kd = c.num_attention_heads * c.head_dim, c.num_key_value_heads * c.head_dim
    sd = {"embed_tokens.weight": torch.randn(c.vocab_size, H, generator=g), "norm.weight": torch.rand(H, generator=g),
          "lm_head.weight": torch.randn(c.vocab_size, H, generator=g)}
    for i in range(c.num_hidden_layers):
        p = f"model.layers.{i}."
        for n, sh in [("self_attn.q_proj", (qd, H)), ("self_attn.k_proj", (kd, H)), ("self_attn.v_proj", (kd, H)),
                      ("self_attn.o_proj", (H, qd)), ("mlp.gate_proj", (I, H)), ("mlp.up_proj", (I, H)),
                      ("mlp.down_proj", (H, I))]:
            sd[p + n + ".weight"] = torch.randn(*sh, generator=g)
        for n, k in [("self_attn.q_proj", qd), ("self_attn.k_proj", kd), ("self_attn.v_proj", kd)]:
            sd[p + n + ".bias"] = torch.randn(k, generator=g)
        sd[p + "input_layernorm.weight"] = torch.rand(H, generator=g)
        sd[p + "post_attention_layernorm.weight"] = torch.rand(H, generator=g)
    return sd


def test_from_state_dict_layouts():
    c = DecoderConfig(vocab_size=64, hidden_size=896, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=7, num_key_value_heads=1)
    sd = _state(c, torch.Generator().manual_seed(0))
    m = Qwen25VLDecoder.from_state_dict(c, sd, device="cpu", dtype=torch.float32)
    x = torch.randn(3, c.hidden_size)
    for i, lw in enumerate(m.layers):
        p = f"model.layers.{i}."
        qkv = x @ lw.w_qkv.t() + lw.b_qkv
        want = torch.cat([x @ sd[p + f"self_attn.{n}_proj.weight"].t() + sd[p + f"self_attn.{n}_proj.bias"]
                          for n in ("q", "k", "v")], -1)
        assert torch.allclose(qkv, want, atol=1e-4)
        gu = (x @ lw.w_gu.t()).view(3, c.intermediate_size // 64, 2, 64)
        assert torch.allclose(gu[:, :, 0].reshape(3, -1), x @ sd[p + "mlp.gate_proj.weight"].t(), atol=1e-4)
        assert torch.allclose(gu[:, :, 1].reshape(3, -1), x @ sd[p + "mlp.up_proj.weight"].t(), atol=1e-4)
        assert torch.equal(lw.w_in, sd[p + "input_layernorm.weight"])
        assert torch.equal(lw.w_down, sd[p + "mlp.down_proj.weight"])
    assert torch.equal(m.lm_head, sd["lm_head.weight"]) and torch.equal(m.norm, sd["norm.weight"])
