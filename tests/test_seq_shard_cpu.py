"""Sequence-sharded dense attention: shard plan, prefill hand-out and the
per-layer exchange protocol, on CPU ranks over gloo (world sizes 2 and 3).

The attention partial and the merge are torch fp32 stand-ins of the verify
kernel's fp32 partial and std_merge_partials_f32 (same conventions: keys L =
lens[b] + len_offset, causal row t sees keys <= L - nq + t, natural-log LSE,
one packed [O | LSE] buffer per rank); the collective order, buffers and rank
roles are the product code's."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from std_b200.seq_shard import ShardExchange, ShardPlan

B, HQ, HKV, D, LAYERS = 2, 7, 1, 128, 3


def ref_partial(q4, kc, vc, lens, len_offset, causal, out, lse):
    Bq, nq, Hq, Dq = q4.shape
    G = Hq // kc.shape[1]
    for b in range(Bq):
        L = int(lens[b]) + len_offset
        k = kc[b, :, :L].float().repeat_interleave(G, 0)   # [Hq, L, D]
        v = vc[b, :, :L].float().repeat_interleave(G, 0)
        q = q4[b].float().permute(1, 0, 2)                  # [Hq, nq, D]
        s = q @ k.transpose(1, 2) / Dq ** 0.5               # [Hq, nq, L]
        if causal:
            keep = torch.arange(L)[None, :] <= (L - nq + torch.arange(nq))[:, None]
            s = s.masked_fill(~keep, float("-inf"))
        m = torch.logsumexp(s, dim=-1)                      # [Hq, nq]
        o = torch.softmax(s, dim=-1) @ v                    # [Hq, nq, D]
        out[b] = o.permute(1, 0, 2).to(out.dtype)
        lse[b] = m.transpose(0, 1)


def ref_merge(parts, rows, D, out):
    o_parts = parts[:, : rows * D].view(-1, rows, D)
    lse_parts = parts[:, rows * D: rows * (D + 1)]
    mx = lse_parts.max(dim=0).values
    w = torch.exp(lse_parts - mx)
    w = torch.where(torch.isfinite(lse_parts), w, torch.zeros_like(w))
    o = (w[..., None] * o_parts.float()).sum(0) / w.sum(0)[..., None]
    out.copy_(o.to(out.dtype))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, prompt, cap, nqs, q_out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = ShardPlan.make(prompt, cap, world, align=16)
        ex = ShardExchange(plan, rank, B, HQ, D, max_nq=max(nqs), device="cpu", partial_fn=ref_partial,
                           merge_fn=ref_merge)
        g = torch.Generator().manual_seed(0)
        full = (torch.randn(LAYERS, 2, B, HKV, cap, D, generator=g)).to(torch.bfloat16)
        local = torch.zeros(LAYERS, 2, B, HKV, plan.local_cap(rank), D, dtype=torch.bfloat16)
        ex.distribute(full if ex.is_owner else None, local, prompt)
        b0, _ = plan.key_range(rank)
        n_check = min(prompt, b0 + local.shape[-2]) - b0
        assert torch.equal(local[..., :n_check, :], full[..., b0:b0 + n_check, :]), "prefill range"
        if not ex.is_owner:
            served = ex.serve(local, LAYERS)
            q_out.put(("served", rank, served))
            return
        # owner: the decode appends new tokens at the end of its local range
        dense_len = torch.full((B,), prompt, dtype=torch.int32)
        shift = b0
        for nq in nqs:
            local[..., prompt - shift:prompt - shift + nq, :] = full[..., prompt:prompt + nq, :]
            q = torch.randn(B, nq, HQ, D, generator=g).to(torch.bfloat16)
            ex.begin(nq)
            worst = 0.0
            for li in range(LAYERS):
                out = torch.empty(B, nq, HQ, D, dtype=torch.bfloat16)
                ex.attend(li, q, local[li, 0], local[li, 1], dense_len, nq - shift, out)
                want = torch.empty_like(out)
                lse = torch.empty(B, nq, HQ)
                ref_partial(q, full[li, 0], full[li, 1], dense_len, nq, True, want, lse)
                worst = max(worst, (out.float() - want.float()).abs().max().item())
            q_out.put(("owner", nq, worst))
        ex.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_attention_protocol(world):
    prompt, cap, nqs = 200, 256, [10, 1, 4]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, prompt, cap, nqs, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    msgs = [q.get(timeout=5) for _ in range(len(nqs) + world - 1)]
    served = [m for m in msgs if m[0] == "served"]
    owner = [m for m in msgs if m[0] == "owner"]
    assert sorted(m[1] for m in served) == list(range(world - 1))
    assert all(m[2] == len(nqs) for m in served)
    assert [m[1] for m in owner] == nqs
    for _, nq, worst in owner:
        assert worst <= 2e-2, (nq, worst)   # fp32 partials merged, bf16 output


def test_shard_plan():
    p = ShardPlan.make(131200, 131456, 4)
    assert p.shard == 32768 and p.owner == 3
    assert p.key_range(0) == (0, 32768) and p.key_range(2) == (65536, 98304)
    assert p.key_range(3) == (98304, 131456) and p.local_cap(3) == 131456 - 98304
    with pytest.raises(ValueError):
        ShardPlan.make(100, 256, 4)
    with pytest.raises(ValueError):
        ShardPlan.make(1000, 1024, 1)


def test_transport_choice():
    plan = ShardPlan.make(200, 256, 2)
    ex = ShardExchange(plan, 0, 1, 4, 8, 2, "cpu", partial_fn=lambda *a: None, merge_fn=lambda *a: None)
    assert ex.transport == "collective" and not ex.capturable  # CPU: only the collective exchange
    with pytest.raises(ValueError):
        ShardExchange(plan, 0, 1, 4, 8, 2, "cpu", transport="p2p")
    with pytest.raises(ValueError):
        ShardExchange(plan, 0, 1, 4, 8, 2, "cpu", transport="shm")
