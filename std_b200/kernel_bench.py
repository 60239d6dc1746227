"""Kernel microbenchmark: one STD kernel alone, timed with CUDA events.

    python -m std_b200.kernel_bench --kernel verify --B 8 --L 32906 --nq 10
    python -m std_b200.kernel_bench --kernel draft  --B 8 --L 1025
    python -m std_b200.kernel_bench --kernel gemm   --M 8 --N 4608 --K 3584 [--cublas]
    python -m std_b200.kernel_bench --kernel forward --B 8 --L 32906 [--gamma 9]
    python -m std_b200.kernel_bench --kernel select --L 32896 --text 128 --k 896

Each repetition cycles through `--caches` distinct K/V caches (default: as
many as keep the total above 256 MB, i.e. larger than the 126 MB L2), so the
number measures HBM, not L2.  The launches are captured into a CUDA graph and
timed over one replay (`--eager` times plain Python-level calls instead, which
adds the host cost of each call).  Prints achieved algorithmic GB/s:
  verify: B * (2048*L + 143360) bytes per launch  (K/V rows + q/out)
  draft:  B * (2048*L + 14336)  bytes per launch (launched as in a decode
          step, STD_DRAFT_AFTER_APPEND: the preceding draft launch writes none
          of its inputs)
  gemm:   2*N*K (weights) + 2*M*K + 2*M*N bytes per launch
  forward: one sparse (draft) forward and one dense verify forward of the
          7B-shaped decoder (random init) at B requests, as the decode loop
          runs them (CUDA graph, one launch sequence each), with sparse
          caches of L_s = K+text+1 keys and dense caches of L keys; the weight
          bytes (14.1 GB) dominate.
  select: the prefill-time selection of one request at the 7B shape -- per
          layer the score chain over its P keys (select_logits, row_stats,
          colsum; 2*T*Hq*P*D FMA flops on CUDA cores, fp16 probabilities
          written), then one top-K over all layers' heads and the gather into
          the sparse cache; eager, each piece timed alone.
This is also the target command of the ncu captures summarised in profiles/.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import ops
from .timing import graph_time_us


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", choices=["verify", "draft", "gemm", "forward", "select"], default="verify")
    ap.add_argument("--gamma", type=int, default=9)
    ap.add_argument("--sparse-len", type=int, default=1025)
    ap.add_argument("--only", choices=["sparse", "dense"], default=None, help="forward: time one of the two")
    ap.add_argument("--M", type=int, default=8)
    ap.add_argument("--N", type=int, default=4608)
    ap.add_argument("--K", type=int, default=3584)
    ap.add_argument("--cublas", action="store_true", help="time torch.mm (cuBLAS) on the same shapes instead")
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--L", type=int, default=32906, help="keys per request (including the nq new ones)")
    ap.add_argument("--nq", type=int, default=10)
    ap.add_argument("--caches", type=int, default=0)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--eager", action="store_true", help="time eager calls (includes host launch cost)")
    ap.add_argument("--text", type=int, default=128, help="select: text queries after the last video token")
    ap.add_argument("--k", type=int, default=896, help="select: visual keys kept per (layer, KV head)")
    a = ap.parse_args()

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if a.kernel == "gemm":
        return gemm_bench(a, dev)
    if a.kernel == "forward":
        return forward_bench(a, dev)
    if a.kernel == "select":
        return select_bench(a, dev)
    B, L = a.B, a.L
    cap = (L + 255) // 256 * 256
    per_cache = 2 * B * 4 * cap * 128 * 2
    n_caches = a.caches or max(1, min(28, (256 << 20) // per_cache + 1))
    g = torch.Generator(device=dev).manual_seed(0)
    ks = [torch.randn(B, 4, cap, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(n_caches)]
    vs = [torch.randn(B, 4, cap, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(n_caches)]
    if a.kernel == "verify":
        q = torch.randn(B, a.nq, 28, 128, generator=g, device=dev).to(torch.bfloat16)
        lens = torch.full((B,), L - a.nq, dtype=torch.int32, device=dev)

        def run(i):
            ops.verify_attention(q, ks[i], vs[i], lens, a.nq)

        nbytes = B * (2048 * L + 143360)
    else:
        q = torch.randn(B, 28, 128, generator=g, device=dev).to(torch.bfloat16)
        lens = torch.full((B,), L, dtype=torch.int32, device=dev)

        def run(i):
            ops.draft_attention(q, ks[i], vs[i], lens, 0, after_append=True)

        nbytes = B * (2048 * L + 14336)
    us = _time(a, run, n_caches)
    assert ops.device_error() == 0
    print(json.dumps({"kernel": a.kernel, "B": B, "L": L, "nq": a.nq if a.kernel == "verify" else 1,
                      "caches": n_caches, "launch_us": us, "algorithmic_bytes": nbytes,
                      "achieved_gbs": nbytes / us / 1e3}))


def _time(a, run, n_bufs: int) -> float:
    """Microseconds per launch, cycling through `n_bufs` buffer sets."""
    if not a.eager:
        rounds = max(1, (a.reps + n_bufs - 1) // n_bufs)
        return graph_time_us([lambda i=i: run(i) for i in range(n_bufs)], rounds=rounds)
    for i in range(max(a.warmup, 2)):
        run(i % n_bufs)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(a.reps, n_bufs)
    e0.record()
    for i in range(reps):
        run(i % n_bufs)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / reps


def gemm_bench(a, dev) -> None:
    M, N, K = a.M, a.N, a.K
    per = N * K * 2
    n_w = a.caches or max(2, min(64, (512 << 20) // per + 1))
    g = torch.Generator(device=dev).manual_seed(0)
    ws = [(torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(n_w)]
    x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)

    def run(i):
        if a.cublas:
            torch.mm(x, ws[i].t(), out=y)
        else:
            ops.gemm(x, ws[i], y)

    us = _time(a, run, n_w)
    nbytes = 2 * N * K + 2 * M * K + 2 * M * N
    print(json.dumps({"kernel": "cublas" if a.cublas else "gemm", "M": M, "N": N, "K": K, "weights": n_w,
                      "launch_us": us, "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / us / 1e3}))


def forward_bench(a, dev) -> None:
    """Graph-timed sparse (draft) and dense (verify) decode forwards."""
    from .model import QWEN25_VL_7B, Qwen25VLDecoder, Workspace, decode_forward

    c = QWEN25_VL_7B
    B, L, gamma = a.B, a.L, a.gamma
    model = Qwen25VLDecoder(c, seed=2, device=str(dev))
    Hkv, D = c.num_key_value_heads, c.head_dim
    cap_s = (a.sparse_len + gamma + 64 + 63) // 64 * 64
    cap_d = (L + gamma + 2 + 127) // 128 * 128
    g = torch.Generator(device=dev).manual_seed(0)
    sparse = torch.randn(c.num_hidden_layers, 2, B, Hkv, cap_s, D, generator=g, device=dev).to(torch.bfloat16)
    dense = torch.empty(c.num_hidden_layers, 2, B, Hkv, cap_d, D, device=dev, dtype=torch.bfloat16)
    dense.normal_(generator=g)
    model.rope_tables(cap_d + 2)
    rows = (B * (gamma + 1) + 15) // 16 * 16
    ws = Workspace(model, rows)
    i32 = dict(dtype=torch.int32, device=dev)
    tok = torch.randint(0, 1000, (B, gamma + 2), generator=g, device=dev, dtype=torch.int32)
    s_len = torch.full((B,), a.sparse_len - 1, **i32)
    d_len = torch.full((B,), L - gamma - 1, **i32)
    ctx = torch.full((B,), L - gamma - 1, **i32)
    out = torch.zeros(B * (gamma + 2), **i32)

    def sparse_fwd():
        decode_forward(model, ws, sparse, B=B, n=1, rows=B, tok=tok, tok_start=1, pos_base=ctx, pos_off=0,
                       slot_base=s_len, slot_off=0, lens=s_len, len_offset=1, sparse=True, argmax_out=out,
                       argmax_stride=gamma + 2, argmax_start=2)

    def dense_fwd():
        decode_forward(model, ws, dense, B=B, n=gamma + 1, rows=rows, tok=tok, tok_start=0, pos_base=d_len, pos_off=0,
                       slot_base=d_len, slot_off=0, lens=d_len, len_offset=gamma + 1, sparse=False, argmax_out=out,
                       argmax_stride=gamma + 2, argmax_start=0)

    res = {}
    for name, fn in (("sparse_forward", sparse_fwd), ("dense_forward", dense_fwd)):
        if a.only is None or name.startswith(a.only):
            res[name + "_us"] = graph_time_us([fn], rounds=4)
    wbytes = 2 * model.num_params() - 2 * c.vocab_size * c.hidden_size  # the embedding table is not streamed
    res.update(B=B, L=L, sparse_len=a.sparse_len, gamma=gamma, weight_bytes=wbytes,
               weight_stream_us=wbytes / 6548.5e3)
    assert ops.device_error() == 0
    print(json.dumps(res))


def _event_us(fn, reps: int) -> float:
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / reps


def select_bench(a, dev) -> None:
    """Selection of one request: 28 layers' score chains, the top-K, the gather."""
    from .model import QWEN25_VL_7B

    c = QWEN25_VL_7B
    Lyr, Hq, Hkv, D = c.num_hidden_layers, c.num_attention_heads, c.num_key_value_heads, c.head_dim
    P, T, K = a.L, a.text, a.k
    V = P - T  # visual keys first, the text (queries) last
    cap = (P + 127) // 128 * 128
    cap_s = (T + K + 64 + 63) // 64 * 64
    g = torch.Generator(device=dev).manual_seed(0)
    dense = torch.randn(Lyr, 2, 1, Hkv, cap, D, generator=g, device=dev).to(torch.bfloat16)
    sparse = torch.zeros(Lyr, 2, 1, Hkv, cap_s, D, device=dev, dtype=torch.bfloat16)
    q = torch.randn(Lyr, T, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    scores = torch.empty(Lyr, Hkv, P, device=dev, dtype=torch.float32)
    visual_pos = torch.arange(V, device=dev, dtype=torch.int32)
    non_visual = torch.arange(V, P, device=dev, dtype=torch.int32)
    topk = torch.empty(Lyr, Hkv, K, device=dev, dtype=torch.int32)

    def scores_all():
        for li in range(Lyr):
            ops.select_scores(q[li], dense[li, 0, 0], P, P - T, scores=scores[li], write_probs=True)

    reps = max(1, a.reps // 5)
    us_scores = _event_us(scores_all, reps)
    us_topk = _event_us(lambda: ops.topk_select(scores.view(Lyr * Hkv, P), visual_pos, K, out=topk.view(-1, K)),
                        a.reps)
    us_gather = _event_us(lambda: ops.compact_gather(dense, sparse, 0, non_visual, topk), a.reps)
    assert ops.device_error() == 0
    flops = 2.0 * T * Hq * P * D * Lyr
    probs_bytes = 2.0 * Hq * T * P * Lyr
    gather_bytes = 2.0 * Lyr * 2 * Hkv * (T + K) * D * 2  # read + write of the kept rows
    print(json.dumps({"kernel": "select", "P": P, "T": T, "K": K, "layers": Lyr,
                      "scores_us": us_scores, "scores_tflops": flops / us_scores / 1e6,
                      "probs_write_gbs": probs_bytes / us_scores / 1e3,
                      "topk_us": us_topk, "topk_read_gbs": 4.0 * Lyr * Hkv * P / us_topk / 1e3,
                      "gather_us": us_gather, "gather_gbs": gather_bytes / us_gather / 1e3,
                      "total_ms": (us_scores + us_topk + us_gather) / 1e3}))


if __name__ == "__main__":
    main()
