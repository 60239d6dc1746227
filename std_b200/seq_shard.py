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
layer: every rank computes the (O, LSE) partial of its key range for the
owner's queries with the verify kernel in fp32 (the owner causal over its
local keys, the servers non-causal), and the owner merges the partials in
rank order (std_merge_partials_f32 / _list).  Attention over disjoint key
ranges combines exactly through LSE, so the only difference from the
unsharded result is fp32 rounding at fixed boundaries -- identical for a
token verified in a block and the same token decoded alone, which keeps
STD == AR.

Each forward starts with a 2-int header broadcast ([1, nq]); [0, 0] ends the
servers' loop.

Two transports carry the per-layer exchange:

  "p2p" (GPUs of one node, the default on CUDA): no collective inside a
      forward.  The ranks map each other's exported buffers with CUDA IPC
      (std_b200/csrc/p2p.cu): the owner copies the layer's queries into its
      exported query buffer and posts an epoch flag to every server; a server
      waits for it, runs the verify kernel on the queries read straight from
      the owner's memory over NVLink, storing its fp32 partial into its slot
      of the owner's exported inbox, and posts its flag; the owner waits for
      every server and merges from its own memory.  Waits are bounded (about
      a second).  The owner's layer steps
      are kernels and copies only, so its dense forward can be captured in a
      CUDA graph: begin() announces a forward only outside capture, and a
      caller replaying such a graph calls announce(nq) first.
  "collective" (any backend; gloo on CPU for the protocol tests): the owner
      broadcasts the queries, every rank computes its partial into one packed
      buffer [O | LSE], and one all-gather moves them; every rank issues the
      collectives in the same order.
"""

from __future__ import annotations

import ctypes
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
    """Buffers and exchange steps shared by the owner and the shard servers.

    partial_fn / merge_fn default to the CUDA kernels; the CPU protocol tests
    pass torch stand-ins and run over gloo with the collective transport."""

    def __init__(self, plan: ShardPlan, rank: int, B: int, Hq: int, D: int, max_nq: int, device,
                 group=None, partial_fn: Optional[Callable] = None, merge_fn: Optional[Callable] = None,
                 transport: Optional[str] = None):
        self.plan, self.rank, self.group = plan, rank, group
        self.B, self.Hq, self.D, self.max_nq = B, Hq, D, max_nq
        self.device = torch.device(device)
        self.partial_fn = partial_fn or _verify_partial
        self.merge_fn = merge_fn or _merge
        if transport is None:
            transport = "p2p" if self.device.type == "cuda" and partial_fn is None and merge_fn is None \
                else "collective"
        if transport not in ("p2p", "collective"):
            raise ValueError(f"unknown transport {transport!r}")
        if transport == "p2p" and self.device.type != "cuda":
            raise ValueError("the p2p transport maps GPU memory: it needs a CUDA device")
        self.transport = transport
        N = plan.world
        rows = B * max_nq * Hq
        self.hdr = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.is_owner = rank == plan.owner
        if transport == "p2p":
            self._p2p_setup(rows)
            return
        self.q = torch.zeros(rows * D, dtype=torch.bfloat16, device=self.device)
        # packed fp32 partial of this rank, [rows * D O | rows LSE], and all ranks'
        self.part = torch.zeros(rows * (D + 1), dtype=torch.float32, device=self.device)
        self.parts = torch.zeros(N * rows * (D + 1), dtype=torch.float32, device=self.device)

    # ------------------------------------------------------------ p2p set-up
    def _p2p_setup(self, rows: int) -> None:
        """Export this rank's buffers, map the peers' (one GPU per rank, one node)."""
        from . import _lib

        N, D = self.plan.world, self.D
        if N > 8:
            raise ValueError("the p2p transport takes at most 8 ranks")
        ids = [None] * N
        dist.all_gather_object(ids, str(torch.cuda.get_device_properties(self.device).uuid), group=self.group)
        if len(set(ids)) != N:
            raise RuntimeError("the p2p transport needs every rank on its own GPU of one node")
        hb = int(_lib.query("std_ipc_handle_bytes"))

        def alloc(nbytes: int) -> int:
            ptr = ctypes.c_void_p(0)
            _lib.call("std_device_alloc", int(nbytes), ctypes.byref(ptr))
            self._allocs.append(ptr.value)
            return ptr.value

        def export(ptr: int) -> bytes:
            buf = ctypes.create_string_buffer(hb)
            _lib.call("std_ipc_handle", ptr, buf)
            return buf.raw

        def open_peer(handle: bytes) -> int:
            ptr = ctypes.c_void_p(0)
            _lib.call("std_ipc_open", ctypes.create_string_buffer(handle, hb), ctypes.byref(ptr))
            self._opened.append(ptr.value)
            return ptr.value

        # one server's [O | LSE] partial in the owner's inbox, 256-byte aligned slots
        self._slot_bytes = (rows * (D + 1) * 4 + 255) // 256 * 256
        self._allocs, self._opened = [], []
        with torch.cuda.device(self.device):
            self._ctr = alloc(16)  # [query epoch, partial epoch] of this rank
            if self.is_owner:
                self._q_ipc = alloc(rows * D * 2)                       # the layer's queries, read by the servers
                self._pflags = alloc(4 * max(1, N - 1))                 # slot r: server r's partial epoch
                self._inbox = alloc(max(1, N - 1) * self._slot_bytes)   # slot r: server r's partial
                exports = (export(self._q_ipc), export(self._pflags), export(self._inbox))
            else:
                self._qflag = alloc(16)  # the owner's query epoch
                exports = (export(self._qflag),)
            every = [None] * N
            dist.all_gather_object(every, exports, group=self.group)
            if self.is_owner:
                self._peer_qflags = [open_peer(every[r][0]) for r in range(self.plan.owner)]
                self._own_part = torch.zeros(rows * (D + 1), dtype=torch.float32, device=self.device)
            else:
                owner = every[self.plan.owner]
                self._peer_q = open_peer(owner[0])
                self._peer_pflag = open_peer(owner[1]) + 4 * self.rank
                self._peer_slot = open_peer(owner[2]) + self.rank * self._slot_bytes
            self.q = None
        dist.barrier(group=self.group)

    def release(self) -> None:
        """Unmap the peers' buffers and free this rank's exported ones (p2p);
        every rank calls it after the servers' loop has ended."""
        if self.transport != "p2p":
            return
        from . import _lib

        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                _lib.call("std_ipc_close", ptr)
            self._opened = []
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for ptr in self._allocs:
                _lib.call("std_device_free", ptr)
            self._allocs = []

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
    @property
    def capturable(self) -> bool:
        """The owner's dense forward can be captured in a CUDA graph (p2p)."""
        return self.transport == "p2p"

    def announce(self, nq: int) -> None:
        """Owner: tell the servers that a dense forward of nq tokens per request follows."""
        if not 1 <= nq <= self.max_nq:
            raise ValueError(f"nq={nq} outside [1, {self.max_nq}]")
        self.hdr.copy_(torch.tensor([1, nq], dtype=torch.int32))
        self._bcast(self.hdr)

    def begin(self, nq: int) -> None:
        """Owner: announce a dense forward of nq tokens per request (the start
        of decode_forward).  Under graph capture (p2p) nothing is sent: the
        caller announces before each replay."""
        if self.capturable and self.device.type == "cuda" and torch.cuda.is_current_stream_capturing():
            if not 1 <= nq <= self.max_nq:
                raise ValueError(f"nq={nq} outside [1, {self.max_nq}]")
            return
        self.announce(nq)

    def attend(self, li: int, q4: torch.Tensor, kc, vc, lens, len_offset: int, out4: torch.Tensor) -> None:
        """Owner: one layer's dense attention over all shards into out4 [B, nq, Hq, D]."""
        if self.transport == "p2p":
            self._attend_p2p(q4.contiguous(), kc, vc, lens, len_offset, out4)
            return
        self._exchange(q4.shape[1], q4.contiguous(), kc, vc, lens, len_offset, True, out4)

    def _attend_p2p(self, q4: torch.Tensor, kc, vc, lens, len_offset: int, out4: torch.Tensor) -> None:
        from . import _lib

        B, nq, Hq, D = q4.shape
        rows = B * nq * Hq
        N = self.plan.world
        s = torch.cuda.current_stream().cuda_stream
        # queries -> the exported buffer, then epoch -> every server
        flags = (ctypes.c_ulonglong * (N - 1))(*self._peer_qflags)
        _lib.call("std_p2p_post", q4.data_ptr(), self._q_ipc, rows * D * 2, flags, N - 1, self._ctr, s)
        part = self._own_part[: rows * (D + 1)]
        self.partial_fn(q4, kc, vc, lens, len_offset, True, part[: rows * D].view(B, nq, Hq, D),
                        part[rows * D:].view(B, nq, Hq))
        _lib.call("std_p2p_wait", self._pflags, N - 1, self._ctr + 4, s)
        # rank order: the servers' inbox slots, then the owner's own partial
        parts = (ctypes.c_ulonglong * N)(*[self._inbox + r * self._slot_bytes for r in range(N - 1)], part.data_ptr())
        _lib.call("std_merge_partials_f32_list", parts, N, rows, D, out4.data_ptr(), None, s)

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
            if self.transport == "p2p":
                for li in range(n_layers):
                    self._serve_layer_p2p(nq, cache[li, 0], cache[li, 1], lens)
            else:
                q4 = self.q[: self.B * nq * self.Hq * self.D].view(self.B, nq, self.Hq, self.D)
                for li in range(n_layers):
                    self._exchange(nq, q4, cache[li, 0], cache[li, 1], lens, 0, False, None)
            served += 1

    def _serve_layer_p2p(self, nq: int, kc: torch.Tensor, vc: torch.Tensor, lens: torch.Tensor) -> None:
        """Wait for the owner's queries, compute this key range's partial from
        them (read in the owner's memory) into this rank's slot of the owner's
        inbox, post it."""
        from . import _lib, ops

        B, Hq, D = self.B, self.Hq, self.D
        _, Hkv, cap, _ = kc.shape
        rows = B * nq * Hq
        s = torch.cuda.current_stream().cuda_stream
        _lib.call("std_p2p_wait", self._qflag, 1, self._ctr, s)
        nb = _lib.query("std_verify_attn_workspace_bytes", B, Hkv, cap)
        ws = ops.workspace("verify", nb, self.device)
        _lib.call("std_verify_attn_partial", self._peer_q, kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), 0, nq, 0,
                  B, Hq, Hkv, D, cap, self._peer_slot, self._peer_slot + rows * D * 4, ws.data_ptr(), ws.numel(), s)
        flags = (ctypes.c_ulonglong * 1)(self._peer_pflag)
        _lib.call("std_p2p_post", None, None, 0, flags, 1, self._ctr + 4, s)

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
