"""Microbenchmark of the sequence-sharded exchange (std_b200/seq_shard.py):
per-layer cost of one dense forward's attention with the key range split
over the ranks, against the owner's own key range alone.

    torchrun --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 --master-port 29519 \\
        -m std_b200.exchange_bench [--keys 4096 131072] [--transport p2p]

One request, the 7B attention shape (28 query heads, 4 KV heads, D = 128),
one query token per forward (an AR step), 28 layers.  For each key count the
owner (rank N-1) times, over 20 forwards captured in a CUDA graph and
replayed: `local_us` = its own key range's partial alone, `exchange_us` =
the whole exchange (announce, per layer the queries out, every rank's
partial, the merge).  Timing is CUDA events on the owner's stream; the
servers answer through ShardExchange.serve.  Rank N-1 prints one JSON line
per key count.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from . import ops
from .seq_shard import ShardExchange, ShardPlan

B, HQ, HKV, D, LAYERS = 1, 28, 4, 128, 28


def _time_graph(g: torch.cuda.CUDAGraph, reps: int, before=None) -> float:
    for _ in range(3):
        if before:
            before()
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        if before:
            before()
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / reps


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--keys", type=int, nargs="+", default=[4096, 131072])
    ap.add_argument("--transport", choices=["p2p", "collective"], default="p2p")
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    nq = 1
    try:
        for keys in a.keys:
            cap = keys + 256
            plan = ShardPlan.make(keys, cap, world)
            ex = ShardExchange(plan, rank, B, HQ, D, 10, dev, transport=a.transport)
            g = torch.Generator(device=dev).manual_seed(5 + rank)
            kv = torch.randn(LAYERS, 2, B, HKV, plan.local_cap(rank), D, device=dev, generator=g).to(torch.bfloat16)
            if not ex.is_owner:
                ex.serve(kv, LAYERS)
                ex.release()
                continue
            q = torch.randn(B, nq, HQ, D, device=dev, generator=g).to(torch.bfloat16)
            out = torch.empty(B, nq, HQ, D, device=dev, dtype=torch.bfloat16)
            lens = torch.full((B,), keys - plan.key_range(rank)[0], dtype=torch.int32, device=dev)
            o32 = torch.empty(B, nq, HQ, D, device=dev)
            lse = torch.empty(B, nq, HQ, device=dev)

            def local_only():
                for li in range(LAYERS):
                    ops.verify_attention_partial(q, kv[li, 0], kv[li, 1], lens, nq, True, o32, lse)

            def forward():
                ex.begin(nq)
                for li in range(LAYERS):
                    ex.attend(li, q, kv[li, 0], kv[li, 1], lens, nq, out)

            local_only()
            forward()  # eager once: workspaces, and the servers answer it
            torch.cuda.synchronize()
            g_local = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_local):
                local_only()
            t_local = _time_graph(g_local, a.reps)
            if ex.capturable:
                g_ex = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g_ex):
                    forward()
                t_ex = _time_graph(g_ex, a.reps, before=lambda: ex.announce(nq))
                del g_ex
            else:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(a.reps):
                    forward()
                e1.record()
                torch.cuda.synchronize()
                t_ex = e0.elapsed_time(e1) * 1000.0 / a.reps
            err = ops.device_error()
            ex.close()
            ex.release()
            print(json.dumps({"bench": "seq_shard_exchange", "transport": a.transport, "world": world,
                              "keys": keys, "owner_keys": int(lens[0].item()), "server_keys": plan.shard,
                              "nq": nq, "layers": LAYERS, "local_us_per_layer": t_local / LAYERS,
                              "exchange_us_per_layer": t_ex / LAYERS,
                              "graph": bool(ex.capturable), "device_error": err}), flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
