"""Sequence-sharded verify on 2 GPUs: STD == AR token for token when the
dense cache is split across ranks (the owner holds the tail and runs the
model, the other rank serves its key range every dense forward), with the
per-layer exchange over peer memory (p2p: IPC-mapped buffers, epoch flags,
the owner's rounds captured in CUDA graphs) and over NCCL collectives.

Needs two visible GPUs; skipped otherwise (the protocol itself is covered on
CPU by test_seq_shard_cpu.py)."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

VIDEO = 7


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, B, gamma, max_new, transport, q):
    import torch.distributed as dist

    from std_b200 import ops
    from std_b200.model import TINY, Qwen25VLDecoder
    from std_b200.seq_shard import ShardExchange, ShardPlan
    from std_b200.std_qwen25vl import STDRunner, _prepare, selection_budget

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        V, T = 1200, 40
        P = V + T
        cap = STDRunner.dense_capacity(P, max_new, gamma)
        plan = ShardPlan.make(P, cap, world)
        ex = ShardExchange(plan, rank, B, TINY.num_attention_heads, TINY.head_dim, gamma + 1, dev, transport=transport)
        if not ex.is_owner:
            local = torch.zeros(TINY.num_hidden_layers, 2, B, TINY.num_key_value_heads, plan.local_cap(rank),
                                TINY.head_dim, dtype=torch.bfloat16, device=dev)
            ex.distribute(None, local, P)
            served = ex.serve(local, TINY.num_hidden_layers)
            ex.release()
            q.put(("served", rank, served, ops.device_error()))
            return
        g = torch.Generator().manual_seed(31)
        ids = torch.randint(10, TINY.vocab_size, (B, P), generator=g)
        ids[:, :V] = VIDEO
        vis = torch.randn(B, V, TINY.hidden_size, generator=g).to(torch.bfloat16)
        model = Qwen25VLDecoder(TINY, seed=2, device=str(dev))
        _, layout, embeds = _prepare(model, {"input_ids": ids, "visual_embeds": vis}, VIDEO)
        k = selection_budget(layout.prompt_len, layout.text_start, V, 200, None)
        runner = STDRunner(model, B, layout, max_new, gamma=gamma, k=k, ignore_eos=True, shard=ex)
        runner.prefill(embeds, with_selection=True)
        runner.run_std()
        std_tokens = runner.out_tokens.cpu().clone()
        st = runner.std_stats()
        runner.run_ar()
        ar_tokens = runner.out_tokens.cpu().clone()
        ex.close()
        ex.release()
        torch.cuda.synchronize()
        q.put(("owner", bool(torch.equal(std_tokens, ar_tokens)), int(runner.n_gen.min()), sum(st["rounds"]),
               ops.device_error()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,B,gamma,transport",
                         [(2, 1, 9, "p2p"), (2, 2, 5, "p2p"), (2, 2, 5, "collective"), (4, 2, 5, "p2p")])
def test_sharded_std_equals_ar(world, B, gamma, transport):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    max_new = 24
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, gamma, max_new, transport, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    msgs = [q.get(timeout=5) for _ in range(world)]
    owner = [m for m in msgs if m[0] == "owner"][0]
    servers = [m for m in msgs if m[0] == "served"]
    assert sorted(m[1] for m in servers) == list(range(world - 1))
    _, equal, n_min, rounds, err = owner
    assert err == 0
    assert equal, "sharded STD tokens differ from sharded AR tokens"
    assert n_min == max_new
    # every STD round has one verify forward and every AR step one dense
    # forward; each of them reached the server
    for served in servers:
        assert served[2] >= max_new + 1
        assert served[3] == 0
