"""CPU: the numpy STD decode restatement runs and keeps its caches consistent."""
from oracle.decoder import NumpySTD, run_cpu_std


def test_numpy_std_rounds_small():
    r = run_cpu_std(rounds=3, warmup=1, hidden=224, inter=512, layers=2, heads=14, kv_heads=2, vocab=300,
                    L_dense=200, L_sparse=64, max_new=32, gamma=4)
    assert r["tokens"] >= 3 and r["seconds"] > 0 and len(r["accepts"]) == 3


def test_numpy_std_cache_lengths():
    m = NumpySTD(hidden=224, inter=512, layers=1, heads=14, kv_heads=2, vocab=100, L_dense=50, L_sparse=20,
                 max_new=16, gamma=3)
    d0, s0, c0 = m.dense_len, m.sparse_len, m.ctx
    app, acc, nxt, pend = m.std_round(5, [], 5, 16)
    assert m.dense_len == d0 + acc and m.sparse_len == s0 + acc + 1 and m.ctx == c0 + len(app)
    assert app[:1] == [5] and pend == [app[-1]]
