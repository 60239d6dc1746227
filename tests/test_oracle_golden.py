"""CPU: pin the oracle against the reference's own outputs (tests/golden/)."""
import os

import numpy as np
import pytest

import oracle
from oracle.inputs import CONFIG0, SMALL, bf16_bits, digest, make_layer_inputs

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _sel_inputs(case):
    inp = make_layer_inputs(case, 0)
    qb = bf16_bits(inp["q_text"][0].permute(1, 0, 2).contiguous())
    kb = bf16_bits(inp["k"][0])
    return inp, qb, kb


@pytest.mark.parametrize("case", [SMALL, CONFIG0], ids=lambda c: c.name)
def test_selection_matches_reference(case):
    g = np.load(os.path.join(GOLDEN, f"selection_{case.name}.npz"))
    _, qb, kb = _sel_inputs(case)
    assert digest(qb) == str(g["q_digest"]) and digest(kb) == str(g["k_digest"]), "input RNG drifted"
    if "q_bits" in g:
        assert np.array_equal(g["q_bits"], qb) and np.array_equal(g["k_bits"], kb)
    scores = oracle.select_scores(qb, kb, case.q_start, case.P)
    ref = g["ref_scores"]
    # identical up to the reference's library matmul / softmax rounding
    assert np.abs(scores - ref).max() <= 1e-3 * np.abs(ref).max()
    assert (scores == ref).mean() > 0.85
    k = int(g["k"])
    assert k == case.k
    topk = oracle.topk_lowest(scores, np.arange(case.V, dtype=np.int32), k)
    for h in range(topk.shape[0]):
        assert set(topk[h].tolist()) == set(g["ref_topk"][h].tolist())
        assert np.all(np.diff(topk[h]) > 0)
    assert np.array_equal(g["non_visual"], np.arange(case.V, case.P))


def test_std_exp_error_bound():
    x = np.concatenate([-np.linspace(0, 104, 200001, dtype=np.float32),
                        np.array([-np.inf, -1e-30, -0.0], dtype=np.float32)])
    y = oracle.std_exp(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    normal = ref > 1.2e-38
    rel = np.abs(y[normal] - ref[normal]) / ref[normal]
    assert rel.max() < 4e-7  # about 3 ulp
    assert np.all(np.abs(y[~normal] - ref[~normal]) < 3e-45)
    assert y[-3] == 0.0 and y[-1] == 1.0


def test_fp16_bf16_rounding_matches_numpy():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 300,
                        rng.standard_normal(1000).astype(np.float32) * 1e-6,
                        np.array([65504, 65519.99, 65520, 1e-8, 6e-5, -0.0], dtype=np.float32)])
    h = oracle.f32_to_f16_bits(x)
    assert np.array_equal(h, x.astype(np.float16).view(np.uint16))
    import torch

    b = oracle.f32_to_bf16_bits(x)
    assert np.array_equal(b, torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))


def test_attention_oracle_matches_reference_sdpa():
    g = np.load(os.path.join(GOLDEN, "attention_config0.npz"))
    inp = make_layer_inputs(CONFIG0, 0)
    k = inp["k"][0].numpy()
    v = inp["v"][0].numpy()
    idx = g["compact_index"]
    kc = np.stack([k[h, idx[h]] for h in range(4)])[None]
    vc = np.stack([v[h, idx[h]] for h in range(4)])[None]
    o, _ = oracle.draft_attention(inp["q_draft"][0, :, 0].numpy()[None], kc, vc, [kc.shape[2]])
    assert np.abs(o[0] - g["draft_out"]).max() < 1e-5
    q = inp["q_verify"][0].permute(1, 0, 2).numpy()[None]
    o, _ = oracle.verify_attention(q, k[None], v[None], [k.shape[1]])
    assert np.abs(o[0] - g["verify_out"]).max() < 1e-5


def test_compact_indices_match_reference():
    g = np.load(os.path.join(GOLDEN, "attention_config0.npz"))
    s = np.load(os.path.join(GOLDEN, "selection_config0.npz"))
    idx = oracle.compact_indices(s["non_visual"], s["ref_topk"])
    assert np.array_equal(idx, g["compact_index"])
    assert idx.shape[1] == CONFIG0.k_plus_text


def test_verify_oracle_causal_invariants():
    """Invariants of the reference's tests/test_sparse_verify_spike.py:49-80."""
    rng = np.random.default_rng(7)
    q = rng.standard_normal((1, 3, 4, 8))
    k = rng.standard_normal((1, 2, 7, 8))
    v = rng.standard_normal((1, 2, 7, 8))
    batched, _ = oracle.verify_attention(q, k, v, [7])
    for i in range(3):
        one, _ = oracle.verify_attention(q[:, i:i + 1], k, v, [7 - 3 + i + 1])
        assert np.allclose(batched[:, i], one[:, 0], atol=1e-12)
    q2 = rng.standard_normal((1, 2, 2, 4))
    k2 = rng.standard_normal((1, 1, 5, 4))
    v2 = rng.standard_normal((1, 1, 5, 4))
    base, _ = oracle.verify_attention(q2, k2, v2, [5])
    ch = v2.copy()
    ch[:, :, -1] += 10000
    alt, _ = oracle.verify_attention(q2, k2, ch, [5])
    assert np.allclose(base[:, 0], alt[:, 0]) and not np.allclose(base[:, 1], alt[:, 1])


def test_sharded_merge_equals_unsharded():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((2, 10, 14, 16))
    k = rng.standard_normal((2, 2, 300, 16))
    v = rng.standard_normal((2, 2, 300, 16))
    full, lse = oracle.verify_attention(q, k, v, [300, 260])
    parts = [oracle.verify_attention(q, k, v, [300, 260], kv_begin=a, kv_end=b) for a, b in
             [(0, 100), (100, 200), (200, 300)]]
    o, l = oracle.merge_partials([p[0] for p in parts], [p[1] for p in parts])
    assert np.allclose(o, full, atol=1e-12) and np.allclose(l, lse, atol=1e-12)


def test_accept_replay_matches_reference_trace():
    t = np.load(os.path.join(GOLDEN, "std_trace_tiny.npz"))
    drafts = [[int(x) for x in row if x >= 0] for row in t["drafts"]]
    verifies = [[int(x) for x in row if x >= 0] for row in t["verifies"]]
    gen, acc, pend = oracle.replay_std_rounds(drafts, verifies, int(t["dense_next"]), int(t["max_new"]),
                                              int(t["gamma"]), int(t["eos"]), ignore_eos=True)
    assert gen == t["std_tokens"].tolist()
    assert acc == t["accept_lengths"].tolist()
    assert pend == t["pending_lengths"].tolist()
    assert t["std_tokens"].tolist() == t["ar_tokens"].tolist()
    assert 0 in acc and max(acc) == int(t["gamma"])  # the trace exercises rejection and full acceptance


def test_accept_round_edge_cases():
    # EOS inside the accepted prefix truncates; the limit cuts the bonus
    a, bonus, app, fin = oracle.accept_round([5, 2, 7], [5, 2, 7, 9], 0, True, 10, eos_token_id=2, ignore_eos=False)
    assert (a, bonus, app, fin) == (3, 9, [5, 2], True)
    a, bonus, app, fin = oracle.accept_round([5, 6], [5, 6, 9], 0, True, 2, eos_token_id=2, ignore_eos=True)
    assert (a, app, fin) == (2, [5, 6], True)
    # no pending: dense_next predicts draft[0]
    a, bonus, app, fin = oracle.accept_round([4, 8], [8, 1], 4, False, 10, eos_token_id=2, ignore_eos=True)
    assert (a, bonus, app) == (2, 1, [4, 8, 1])
    a, bonus, app, fin = oracle.accept_round([4, 8], [3, 1], 5, False, 10, eos_token_id=2, ignore_eos=True)
    assert (a, bonus, app) == (0, 5, [5])
    assert oracle.rollback_lengths(100, 1, 50, 3) == (104, 53)


@pytest.mark.parametrize("seed", [1, 2])
def test_selection_matches_reference_other_seeds(seed):
    """configs[0]-shaped selection with two more input seeds: the oracle's top-K
    sets equal the reference's on every head."""
    g = np.load(os.path.join(GOLDEN, f"selection_config0_seed{seed}.npz"))
    inp = make_layer_inputs(CONFIG0, seed)
    qb = bf16_bits(inp["q_text"][0].permute(1, 0, 2).contiguous())
    kb = bf16_bits(inp["k"][0])
    assert digest(qb) == str(g["q_digest"]) and digest(kb) == str(g["k_digest"]), "input RNG drifted"
    scores = oracle.select_scores(qb, kb, CONFIG0.q_start, CONFIG0.P)
    ref = g["ref_scores"]
    assert np.abs(scores - ref).max() <= 1e-3 * np.abs(ref).max()
    assert (scores == ref).mean() > 0.85
    k = int(g["k"])
    topk = oracle.topk_lowest(scores, np.arange(CONFIG0.V, dtype=np.int32), k)
    for h in range(topk.shape[0]):
        assert set(topk[h].tolist()) == set(g["ref_topk"][h].tolist())
    # the reference's own boundary is not a tie: its K-th score is unique
    assert np.all(g["tie_equal_to_kth"] == 1)


def test_selection_matches_reference_config3_sizes():
    """configs[3] sizes (131072 visual keys, K = 3968).  At this length the fp16
    softmax probabilities are coarsely quantised, so the K-th score of every
    head is an exact fp32 tie or a near tie.  The reference fills the last
    slots from such a tie class in torch.topk's own order, and its library
    rounding (CPU matmul order, vectorised exp) moves a few scores by one or
    two ulp relative to the restated chain.  Pinned here: the oracle's scores
    agree with the reference's at the K + 256 best positions, every position
    whose reference score is clearly above the boundary is selected by both,
    and the sets differ only inside a 5e-5 relative band around the K-th
    score (measured: 5 of 15872 selected positions, all of them there)."""
    from oracle.inputs import CONFIG3_LAYER as case

    g = np.load(os.path.join(GOLDEN, "selection_config3.npz"))
    inp = make_layer_inputs(case, 0)
    qb = bf16_bits(inp["q_text"][0].permute(1, 0, 2).contiguous())
    kb = bf16_bits(inp["k"][0])
    del inp
    assert digest(qb) == str(g["q_digest"]) and digest(kb) == str(g["k_digest"]), "input RNG drifted"
    scores = oracle.select_scores(qb, kb, case.q_start, case.P)
    k = int(g["k"])
    assert k == case.k == 3968
    pos, ref = g["boundary_pos"].astype(np.int64), g["boundary_scores"]
    mine = np.take_along_axis(scores, pos, axis=1)
    assert np.abs(mine - ref).max() <= 1e-3 * np.abs(ref).max()
    assert (mine == ref).mean() > 0.80
    vis = scores[:, : case.V].astype(np.float64).sum(axis=1)
    assert np.allclose(vis, g["score_sums"], rtol=1e-5)
    topk = oracle.topk_lowest(scores, np.arange(case.V, dtype=np.int32), k)
    band = 5e-5
    n_diff = 0
    for h in range(topk.shape[0]):
        mine_set, ref_set = set(topk[h].tolist()), set(g["ref_topk"][h].tolist())
        kth = float(g["tie_kth"][h])
        ref_score = dict(zip(pos[h].tolist(), ref[h].tolist()))
        clearly_above = {p for p, v in ref_score.items() if v > kth * (1 + band)}
        assert clearly_above <= mine_set and clearly_above <= ref_set
        diff = mine_set ^ ref_set
        n_diff += len(diff)
        for p in diff:
            assert p in ref_score and abs(ref_score[p] - kth) <= band * kth, (h, p)
    assert n_diff <= 16  # a handful of boundary positions out of 4 x 3968


def test_collector_oracle_matches_reference():
    """The collector restatement (fp64) against the reference's own
    RuntimeVerificationCollector._hook (fp32 torch) on the same bf16 inputs."""
    import torch

    from oracle.inputs import bf16_bits, digest

    sys_path_golden = os.path.join(os.path.dirname(__file__), "golden")
    import sys

    sys.path.insert(0, sys_path_golden)
    from make_golden import collector_inputs

    g = np.load(os.path.join(GOLDEN, "collector_layer.npz"))
    q, k, vis = collector_inputs()
    assert digest(bf16_bits(q)) == str(g["q_digest"]) and digest(bf16_bits(k)) == str(g["k_digest"])
    rel = oracle.collect_relevance(q.float().numpy(), k.float().numpy(), vis.numpy())[0]
    ref = g["rel"]
    assert np.abs(rel - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())
    # the top of the ranking (what re-selection keeps) agrees
    for h in range(ref.shape[0]):
        assert set(np.argsort(-rel[h])[:64]) == set(np.argsort(-ref[h])[:64])
