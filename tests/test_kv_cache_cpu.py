"""Reference-shaped KV cache views (kv_cache.py:6-165) over the B200 cache
layout [layers, 2, B, Hkv, cap, D], on CPU."""
import types

import torch

from std_b200.model import TINY
from std_b200.std_qwen25vl import KVCache, allocate_kv_cache, initialize_past_key_values, kv_cache_views


def _fake_model():
    return types.SimpleNamespace(config=TINY, device=torch.device("cpu"), dtype=torch.bfloat16)


def test_views_share_the_cache_and_track_lengths():
    m = _fake_model()
    cache = allocate_kv_cache(m, 2, 64)
    pkv, data_list, cur = kv_cache_views(cache)
    assert len(pkv) == TINY.num_hidden_layers and all(len(p) == 2 for p in pkv)
    assert data_list[0].shape == (2 * TINY.num_hidden_layers, 2, TINY.num_key_value_heads, 64, TINY.head_dim)
    assert cur.dtype == torch.long and cur.device.type == "cpu" and cur.numel() == 2 * TINY.num_hidden_layers
    k1 = pkv[1][0]
    assert k1.shape == (2, TINY.num_key_value_heads, 0, TINY.head_dim)
    new = torch.randn(2, TINY.num_key_value_heads, 5, TINY.head_dim).to(torch.bfloat16)
    out = k1.cat(new)
    assert out.shape[2] == 5 and k1.shape[2] == 5 and int(cur[2]) == 5
    assert torch.equal(cache[1, 0, :, :, :5], new)          # the view writes the decode cache itself
    more = torch.randn(2, TINY.num_key_value_heads, 3, TINY.head_dim).to(torch.bfloat16)
    k1.cat(more)
    assert torch.equal(cache[1, 0, :, :, 5:8], more) and k1.shape[2] == 8


def test_copy_moves_selected_rows_and_sets_length():
    m = _fake_model()
    cache = allocate_kv_cache(m, 1, 32)
    pkv, _, cur = kv_cache_views(cache)
    v0 = pkv[0][1]
    rows = torch.randn(1, TINY.num_key_value_heads, 10, TINY.head_dim).to(torch.bfloat16)
    v0.cat(rows)
    v0.copy(torch.tensor([7, 2, 9]), prev_length=4)   # rollback-and-append (kv_cache.py:40-52)
    assert v0.shape[2] == 7 and int(cur[1]) == 7
    assert torch.equal(cache[0, 1, :, :, 4:7], rows[:, :, [7, 2, 9]])
    assert torch.equal(cache[0, 1, :, :, :4], rows[:, :, :4])


def test_initialize_past_key_values_defaults(monkeypatch):
    m = _fake_model()
    monkeypatch.setenv("SPECVLM_MAX_CACHE_LEN", "48")
    pkv, data_list, cur = initialize_past_key_values(m)
    assert data_list[0].shape[3] == 48 and data_list[0].shape[1] == 1
    assert isinstance(pkv[0][0], KVCache)
    pkv, data_list, _ = initialize_past_key_values(m, batch_size=3, max_cache_len=16)
    assert data_list[0].shape[1] == 3 and data_list[0].shape[3] == 16


def test_topk_intersection_counts_matches_sets():
    from std_b200.std_qwen25vl import topk_intersection_counts

    g = torch.Generator().manual_seed(0)
    a = torch.stack([torch.randperm(300, generator=g)[:40].sort().values for _ in range(12)]).view(3, 4, 40)
    b = torch.stack([torch.randperm(300, generator=g)[:40].sort().values for _ in range(12)]).view(3, 4, 40)
    b[0, 0] = a[0, 0]                      # identical selections
    got = topk_intersection_counts(a.to(torch.int32), b.to(torch.int32))
    for i in range(3):
        for j in range(4):
            assert int(got[i, j]) == len(set(a[i, j].tolist()) & set(b[i, j].tolist()))
    assert int(got[0, 0]) == 40


def test_benchmark_cli_flags():
    """The reference CLI's decode flags parse; paths this build lacks are rejected."""
    import pytest

    from std_b200.benchmark_std import _agreement, _args

    a = _args(["--gamma", "5", "--target-k-plus-text", "512", "--k", "100", "--verify-mode", "sequential",
               "--ignore-eos", "--strict-equality", "--sparse-attn-mode", "b200"])
    assert a.gamma == 5 and a.k == 100 and a.verify_mode == "sequential" and a.ignore_eos and a.strict_equality
    for bad in (["--sparse-attn-mode", "triton_gqa"], ["--verify-fallback", "sequential_guard"],
                ["--verify-attn-backend", "math"], ["--dataset", "Video-MME"]):
        with pytest.raises(SystemExit):
            _args(bad)
    ag = _agreement(torch.tensor([1, 2, 3, 4]), torch.tensor([1, 2, 9, 4, 5]))
    assert ag["common_prefix_length"] == 2 and abs(ag["token_level_agreement"] - (1 - 2 / 5)) < 1e-9
