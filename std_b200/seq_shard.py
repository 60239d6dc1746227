"""Sequence-sharded dense attention for very long caches.

The reference keeps one dense KV cache on one device (kv_cache.py:72-165,
capacity from SPECVLM_MAX_CACHE_LEN) and verifies with repeat_kv + SDPA over
all of it (modeling_qwen2_5_vl.py:1096-1133).  Here the dense cache of a long
request is split by sequence position across the ranks of one node:

  rank r < N-1 (a "shard server") holds keys [r*S, (r+1)*S) of every layer --
      prompt keys only, so every verify query sees all of them;
  rank N-1 (the "owner") holds keys [(N-1)*S, cap): the rest of the prompt
      and every token appended while decoding; it also holds the weights, the
      sparse cache and runs the draft steps.

A dense forward on the owner (a verify block or an AR step) exchanges, per
layer: the owner broadcasts the layer's queries, every rank computes the
(O, LSE) partial of its key range with the verify kernel in fp32 (the owner
causal over its local keys, the servers non-causal) into one packed buffer
[O | LSE], the packed partials are all-gathered in one collective and the
owner merges them in rank order with std_merge_partials_f32: two collectives
per layer.  Attention over disjoint key ranges combines exactly through LSE,
so the only difference from the unsharded result is fp32 rounding at fixed
boundaries -- identical for a token verified in a block and the same token
decoded alone, which keeps STD == AR.

Each forward starts with a 2-int header broadcast ([1, nq]); [0, 0] ends the
servers' loop.  The collectives run on NCCL over NVLink (gloo on CPU for the
protocol tests); every rank issues them in the same order.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class ShardPlan:
    world: int
    shard: int      # keys per server shard
    cap: int        # global dense capacity (keys)

    @property
    def owner(self) -> int:
        return self.world - 1

    def key_range(self, rank: int):
        if rank < self.owner:
            return rank * self.shard, (rank + 1) * self.shard
        return self.owner * self.shard, self.cap

    def local_cap(self, rank: int) -> int:
        b, e = self.key_range(rank)
        return e - b

    @staticmethod
    def make(prompt_len: int, cap: int, world: int, align: int = 64) -> "ShardPlan":
        """Server shards are equal, `align`-multiple and filled by the prompt."""
        if world < 2:
            raise ValueError("sequence sharding needs at least 2 ranks")
        s = (prompt_len // world) // align * align
        if s < align:
            raise ValueError(f"prompt of {prompt_len} keys is too short for {world} shards")
        return ShardPlan(world=world, shard=s, cap=cap)


def _verify_partial(q4, kc, vc, lens, len_offset, causal, out_f32, lse):
    from . import ops

    ops.verify_attention_partial(q4, kc, vc, lens, len_offset, causal, out_f32, lse)


def _merge(parts, rows, D, out):
    from . import ops

    ops.merge_partials_f32(parts, rows, D, out)


class ShardExchange:
    """Buffers and collective steps shared by the owner and the shard servers.

    partial_fn / merge_fn default to the CUDA kernels; the CPU protocol tests
    pass torch stand-ins and run over gloo."""

    def __init__(self, plan: ShardPlan, rank: int, B: int, Hq: int, D: int, max_nq: int, device,
                 group=None, partial_fn: Optional[Callable] = None, merge_fn: Optional[Callable] = None):
        self.plan, self.rank, self.group = plan, rank, group
        self.B, self.Hq, self.D, self.max_nq = B, Hq, D, max_nq
        self.device = torch.device(device)
        self.partial_fn = partial_fn or _verify_partial
        self.merge_fn = merge_fn or _merge
        N = plan.world
        rows = B * max_nq * Hq
        self.q = torch.zeros(rows * D, dtype=torch.bfloat16, device=self.device)
        # packed fp32 partial of this rank, [rows * D O | rows LSE], and all ranks'
        self.part = torch.zeros(rows * (D + 1), dtype=torch.float32, device=self.device)
        self.parts = torch.zeros(N * rows * (D + 1), dtype=torch.float32, device=self.device)
        self.hdr = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.is_owner = rank == plan.owner

    # ------------------------------------------------------------ collectives
    def _bcast(self, t: torch.Tensor) -> None:
        dist.broadcast(t, src=self.plan.owner, group=self.group)

    def _all_gather(self, out_flat: torch.Tensor, inp: torch.Tensor) -> None:
        if out_flat.is_cuda:
            dist.all_gather_into_tensor(out_flat, inp, group=self.group)
        else:  # gloo (CPU protocol tests)
            dist.all_gather(list(out_flat.chunk(self.plan.world)), inp, group=self.group)

    def _exchange(self, nq: int, q4: torch.Tensor, kc, vc, lens, len_offset: int, causal: bool,
                  out4: Optional[torch.Tensor]) -> None:
        B, Hq, D, N = self.B, self.Hq, self.D, self.plan.world
        rows = B * nq * Hq
        n = rows * (D + 1)
        self._bcast(q4)
        part = self.part[:n]
        self.partial_fn(q4, kc, vc, lens, len_offset, causal, part[: rows * D].view(B, nq, Hq, D),
                        part[rows * D:].view(B, nq, Hq))
        parts = self.parts[: N * n]
        self._all_gather(parts, part)
        if out4 is not None:
            self.merge_fn(parts.view(N, n), rows, D, out4.view(rows, D))

    # ------------------------------------------------------------ owner side
    def begin(self, nq: int) -> None:
        """Owner: announce a dense forward of nq tokens per request."""
        if not 1 <= nq <= self.max_nq:
            raise ValueError(f"nq={nq} outside [1, {self.max_nq}]")
        self.hdr.copy_(torch.tensor([1, nq], dtype=torch.int32))
        self._bcast(self.hdr)

    def attend(self, li: int, q4: torch.Tensor, kc, vc, lens, len_offset: int, out4: torch.Tensor) -> None:
        """Owner: one layer's dense attention over all shards into out4 [B, nq, Hq, D]."""
        self._exchange(q4.shape[1], q4.contiguous(), kc, vc, lens, len_offset, True, out4)

    def close(self) -> None:
        """Owner: end the servers' loop."""
        self.hdr.zero_()
        self._bcast(self.hdr)

    # ------------------------------------------------------------ server side
    def serve(self, cache: torch.Tensor, n_layers: int) -> int:
        """Shard server: answer dense forwards until the owner closes.

        cache [layers, 2, B, Hkv, S, D] holds this rank's key range; every
        query sees all S keys.  Returns the number of forwards served."""
        lens = torch.full((self.B,), self.plan.shard, dtype=torch.int32, device=self.device)
        served = 0
        while True:
            self._bcast(self.hdr)
            op, nq = (int(v) for v in self.hdr.tolist())
            if op == 0:
                return served
            q4 = self.q[: self.B * nq * self.Hq * self.D].view(self.B, nq, self.Hq, self.D)
            for li in range(n_layers):
                self._exchange(nq, q4, cache[li, 0], cache[li, 1], lens, 0, False, None)
            served += 1

    # ------------------------------------------------------------ prefill
    def distribute(self, full: Optional[torch.Tensor], local: torch.Tensor, filled: int) -> None:
        """Move each rank's key range of the owner's prefilled cache to it.

        full [layers, 2, B, Hkv, cap, D] exists on the owner only; `filled` =
        prompt keys written.  Servers receive into `local`; the owner copies
        its own range.  Point-to-point, once per prefill."""
        own_b, _ = self.plan.key_range(self.plan.owner)
        if self.is_owner:
            for r in range(self.plan.owner):
                b, e = self.plan.key_range(r)
                dist.send(full[..., b:e, :].contiguous(), dst=r, group=self.group)
            n = filled - own_b
            local[..., :n, :].copy_(full[..., own_b:filled, :])
        else:
            buf = torch.empty_like(local)
            dist.recv(buf, src=self.plan.owner, group=self.group)
            local.copy_(buf)
