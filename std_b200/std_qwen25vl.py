"""Sparse-to-Dense (STD) and AR greedy decoding on B200 -- the public API.

Keeps the reference's entry points and result types (std_qwen25vl.py):
  ar_generate_qwen25vl   (:553-606)   vanilla greedy decoding, the oracle STD must equal
  std_generate_qwen25vl  (:609-978)   STD: sparse drafting, parallel dense verify
  build_sparse_selection (:175-231)   per-layer / per-KV-head top-K visual selection
  compact_sparse_prompt_cache (:265-298)
  SparseSelection (:41-50), GenerateResult (:53-89), generated_suffix / tokens_equal (:981-986)

What changes is underneath: both caches live on the device with device-resident
lengths ([layers, 2, B, Hkv, cap, D] bf16), selection/compaction/attention/
acceptance run as libstd_b200.so kernels, and a whole STD round (gamma draft
steps, the dense verify, the fused accept/rollback, the bonus sparse step) is
one CUDA graph; the host reads one 4-byte "all done" flag per round instead of
gamma+1 .item() syncs.  Requests are batched (the reference is batch 1): every
request keeps its own lengths and finishes independently.
"""

from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import ops
from .model import Qwen25VLDecoder, Workspace, decode_forward, prefill_request

SPARSE_ATTN_MODES = ("b200",)
# "compact": the selected prompt rows are copied into a per-request sparse
# cache (the reference's copy + compaction, std_qwen25vl.py:265-320);
# "indexed": the draft reads them in place from the dense cache by position
# (the reference's gather variant, :323-351) and only generated tokens get
# sparse-path K/V rows.
SPARSE_CACHE_MODES = ("compact", "indexed")
# Visual selection across rounds (dynamic_selection.py:176-240): "static"
# keeps S_0; "previous_verify_topk" sets S_{t+1} = TopK(A_t), A_t being round
# t's dense-verification visual relevance (collector v1, :241-308).
SELECTION_POLICIES = ("static", "previous_verify_topk")


def _lib_capture_stream(role: str):
    from . import _lib

    return _lib.capture_stream(role)


def topk_intersection_counts(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a ∩ b| over the last dim of two selections of unique, ascending
    positions (dynamic_selection.py:85-101), on the selections' device."""
    k = a.shape[-1]
    pos = torch.searchsorted(b.contiguous(), a.contiguous()).clamp(max=k - 1)
    return ((b.gather(-1, pos) == a)).sum(dim=-1)
VERIFY_MODES = ("parallel", "sequential")
# verify_fallback values (std_qwen25vl.py:637-647) -> the policy kernel's mode
VERIFY_FALLBACKS = {"none": 0, "sequential_on_reject": 1, "sequential_on_low_accept": 2,
                    "sequential_on_low_margin": 3, "sequential_guard": 4}
VERIFY_ATTN_BACKENDS = ("default", "math", "math_on_full_accept")


@dataclass
class SparseSelection:
    """Per-layer sparse visual KV choices (std_qwen25vl.py:41-50)."""

    topk_positions: List[torch.Tensor]   # per layer [Hkv, k] int64 (CPU), ascending
    non_visual_positions: torch.Tensor   # [NV] int64 (CPU)
    prompt_len: int
    visual_len: int
    text_len: int
    k: int


@dataclass
class GenerateResult:
    """Same fields as the reference's GenerateResult (std_qwen25vl.py:53-89)."""

    output_ids: torch.Tensor
    decoding_time: float
    inference_time: float
    generate_len: int
    accepted_draft_tokens: int = 0
    proposed_draft_tokens: int = 0
    mean_accept_length: float = 0.0
    decode_rounds: int = 0
    final_gamma: int = 0
    fallback_count: int = 0
    fallback_accepted_extra: int = 0
    verify_margin_reruns: int = 0
    min_verify_margin: float = 0.0
    gamma_history: List[int] = field(default_factory=list)
    proposed_lengths: List[int] = field(default_factory=list)
    accept_lengths: List[int] = field(default_factory=list)
    pending_lengths: List[int] = field(default_factory=list)
    draft_time: float = 0.0
    verify_time: float = 0.0
    bonus_time: float = 0.0
    cache_adjust_time: float = 0.0
    cache_init_time: float = 0.0
    prefill_time: float = 0.0
    selection_prefill_time: float = 0.0
    selection_time: float = 0.0
    dense_prefill_time: float = 0.0
    sparse_cache_time: float = 0.0
    # B200 batch extension: the per-round lists above concatenate every
    # request's rounds in request order; these keep them per request
    request_accept_lengths: List[List[int]] = field(default_factory=list)
    request_generate_lens: List[int] = field(default_factory=list)

    @property
    def acceptance_rate(self) -> float:
        if self.proposed_draft_tokens == 0:
            return 0.0
        return self.accepted_draft_tokens / self.proposed_draft_tokens


def generated_suffix(output_ids: torch.Tensor, prompt_len: int) -> torch.Tensor:
    return output_ids[:, prompt_len:]


def tokens_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    return a.shape == b.shape and bool(torch.equal(a.detach().cpu(), b.detach().cpu()))


def get_last_video_idx(input_ids: Sequence[int], video_token_id: int) -> int:
    """Last position of video_token_id, or -1 (utils.py:8-15)."""
    for i in range(len(input_ids) - 1, -1, -1):
        if int(input_ids[i]) == video_token_id:
            return i
    return -1


def selection_budget(prompt_len: int, text_start: int, visual_len: int, target_k_plus_text: int,
                     explicit_k: Optional[int]) -> int:
    """k = K+text - text_len, clamped to [1, visual_len] (std_qwen25vl.py:190-195)."""
    text_len = max(1, prompt_len - int(text_start))
    k = int(explicit_k) if explicit_k is not None else max(1, int(target_k_plus_text) - text_len)
    return min(k, int(visual_len))


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass
class PromptLayout:
    prompt_len: int
    text_start: int
    visual_pos: torch.Tensor     # [V] int32 device, ascending
    non_visual: torch.Tensor     # [NV] int32 device, ascending

    @staticmethod
    def from_ids(ids: torch.Tensor, video_token_id: int, device) -> "PromptLayout":
        ids_cpu = ids.detach().cpu().view(-1)
        last = get_last_video_idx(ids_cpu.tolist(), video_token_id)
        if last < 0:
            raise ValueError("No video token found in the prompt; STD visual KV selection requires video input.")
        vis = torch.nonzero(ids_cpu == video_token_id).flatten().to(torch.int32)
        nv = torch.nonzero(ids_cpu != video_token_id).flatten().to(torch.int32)
        return PromptLayout(int(ids_cpu.numel()), last + 1, vis.to(device), nv.to(device))


def allocate_kv_cache(model: Qwen25VLDecoder, batch_size: int, max_cache_len: int) -> torch.Tensor:
    """One preallocated cache [layers, 2, B, Hkv, cap, D] bf16 -- the memory
    layout of the reference's past_key_values_data [2*layers, B, Hkv, cap, D]
    (kv_cache.py:72-165), with every layer's K and V slices contiguous."""
    c = model.config
    return torch.zeros(c.num_hidden_layers, 2, batch_size, c.num_key_value_heads, max_cache_len, c.head_dim,
                       device=model.device, dtype=model.dtype)


class KVCache:
    """One (layer, K or V) slice of a decode cache with the reference's
    interface (kv_cache.py:6-69): data [B, Hkv, cap, D], current_length a 0-d
    int64 tensor; shape reports the filled length, cat appends along dim 2,
    copy moves rows selected by indices to prev_length.  The B200 decode loop
    keeps its lengths on the device instead (STDRunner); this view is for
    callers written against the reference's cache objects."""

    def __init__(self, data: torch.Tensor, current_length: torch.Tensor):
        self.data = data
        self.current_length = current_length

    @property
    def shape(self):
        return (self.data.shape[0], self.data.shape[1], int(self.current_length.item()), self.data.shape[3])

    def copy(self, indices: torch.Tensor, prev_length: int, dim: int = 2) -> None:
        tgt = self.data.index_select(dim, indices.to(self.data.device))
        self.data.narrow(dim, prev_length, tgt.shape[dim]).copy_(tgt, non_blocking=True)
        self.current_length.fill_(prev_length + tgt.shape[dim])

    def cat(self, tensor: torch.Tensor, dim: int = 2) -> torch.Tensor:
        n = int(self.current_length.item())
        self.data.narrow(dim, n, tensor.shape[dim]).copy_(tensor)
        self.current_length.add_(tensor.shape[dim])
        return torch.narrow(self.data, 2, 0, n + tensor.shape[dim])


def kv_cache_views(cache: torch.Tensor, current_length_data: Optional[torch.Tensor] = None):
    """Reference-shaped views of an allocate_kv_cache tensor: (past_key_values
    [[KVCache K, KVCache V] per layer], [data as [2*layers, B, Hkv, cap, D]],
    current_length_data [2*layers] int64 on the CPU)."""
    L = cache.shape[0]
    data = cache.view(2 * L, *cache.shape[2:])
    if current_length_data is None:
        current_length_data = torch.zeros(2 * L, dtype=torch.long, device="cpu")
    pkv = [[KVCache(data[2 * i + j], current_length_data[2 * i + j]) for j in range(2)] for i in range(L)]
    return pkv, [data], current_length_data


def initialize_past_key_values(model: Qwen25VLDecoder, batch_size: int = 1, max_cache_len: Optional[int] = None):
    """kv_cache.py:72-165: (past_key_values, past_key_values_data_list,
    current_length_data) over one zeroed cache.  Capacity: max_cache_len, else
    SPECVLM_MAX_CACHE_LEN, else 16384 (the reference's default for this
    model).  All layers live on the model's device."""
    if max_cache_len is None:
        max_cache_len = int(os.environ.get("SPECVLM_MAX_CACHE_LEN", 16384))
    return kv_cache_views(allocate_kv_cache(model, batch_size, max_cache_len))


def build_sparse_selection(scores: torch.Tensor, layout: PromptLayout, k: int) -> torch.Tensor:
    """scores [layers, Hkv, P] fp32 -> top-k visual positions [layers, Hkv, k] int32 (device).

    std_qwen25vl.py:204-222 on the device, ties to the lowest position."""
    layers, Hkv, P = scores.shape
    return ops.topk_select(scores.view(layers * Hkv, P), layout.visual_pos, k).view(layers, Hkv, k)


def compact_sparse_prompt_cache(dense_cache: torch.Tensor, sparse_cache: torch.Tensor, b: int, layout: PromptLayout,
                                topk: torch.Tensor) -> int:
    """Gather sorted(non_visual U topk[layer, head]) rows of request b into the
    sparse cache (std_qwen25vl.py:265-298); returns compact_len."""
    ops.compact_gather(dense_cache, sparse_cache, b, layout.non_visual, topk)
    return int(layout.non_visual.numel() + topk.shape[-1])


class STDRunner:
    """Device state, caches and CUDA graphs for one batch of same-length requests."""

    def __init__(self, model: Qwen25VLDecoder, batch_size: int, layout: PromptLayout, max_new_tokens: int,
                 gamma: int = 9, k: int = 896, eos_token_id: int = -1, ignore_eos: bool = False,
                 use_graphs: bool = True, verify_mode: str = "parallel", shard=None,
                 sparse_cache: str = "compact", selection_policy: str = "static",
                 selection_update_interval: int = 1, min_selection_change_ratio: float = 0.0,
                 device_loop: bool = True, verify_fallback: str = "none",
                 verify_margin_threshold: Optional[float] = None, sequential_fallback_max_accept: int = 1,
                 verify_attn_backend: str = "default"):
        c = model.config
        if gamma < 1 or 7 * (gamma + 1) > 126:
            raise ValueError("gamma must be in [1, 17]")
        if verify_mode not in VERIFY_MODES:
            raise ValueError(f"verify_mode must be one of {VERIFY_MODES}")
        if sparse_cache not in SPARSE_CACHE_MODES:
            raise ValueError(f"sparse_cache must be one of {SPARSE_CACHE_MODES}")
        if sparse_cache == "indexed" and shard is not None:
            raise ValueError("an indexed sparse cache reads the dense prompt rows, which a sharded owner does not hold")
        if selection_policy not in SELECTION_POLICIES:
            raise ValueError(f"selection_policy must be one of {SELECTION_POLICIES}")
        if selection_policy != "static" and sparse_cache != "indexed":
            raise ValueError("dynamic re-selection needs sparse_cache='indexed' (a selection change is an index update)")
        if selection_update_interval < 1 or not 0.0 <= min_selection_change_ratio <= 1.0:
            raise ValueError("selection_update_interval must be >= 1 and min_selection_change_ratio in [0, 1]")
        if verify_fallback not in VERIFY_FALLBACKS:
            raise ValueError(f"verify_fallback must be one of {tuple(VERIFY_FALLBACKS)}")
        if sequential_fallback_max_accept < 0:
            raise ValueError("sequential_fallback_max_accept must be non-negative.")
        if verify_fallback == "sequential_on_low_margin" and verify_margin_threshold is None:
            raise ValueError("sequential_on_low_margin requires verify_margin_threshold.")
        if verify_margin_threshold is not None and verify_margin_threshold < 0:
            raise ValueError("verify_margin_threshold must be non-negative.")
        if verify_attn_backend not in VERIFY_ATTN_BACKENDS:
            raise ValueError(f"verify_attn_backend must be one of {VERIFY_ATTN_BACKENDS}")
        self.verify_mode = verify_mode
        # verification policies of a parallel verify (std_qwen25vl.py:816-884);
        # every re-verification is the exact one-token-at-a-time replay
        self.policy_mode = VERIFY_FALLBACKS[verify_fallback]
        self.margin_threshold = verify_margin_threshold
        self.max_accept = int(sequential_fallback_max_accept)
        self.math_on_full_accept = verify_attn_backend == "math_on_full_accept"
        self.policy_active = verify_mode == "parallel" and (
            self.policy_mode != 0 or verify_margin_threshold is not None or self.math_on_full_accept)
        self.sparse_cache = sparse_cache
        self.dynamic = selection_policy == "previous_verify_topk"
        self.update_interval = selection_update_interval
        self.min_change = float(min_selection_change_ratio)
        self.model, self.B, self.layout = model, batch_size, layout
        self.gamma, self.k, self.max_new = gamma, k, max_new_tokens
        self.eos, self.ignore_eos, self.use_graphs = eos_token_id, ignore_eos, use_graphs
        P = layout.prompt_len
        self.compact_len = int(layout.non_visual.numel()) + k
        self.cap_d = self.dense_capacity(P, max_new_tokens, gamma)
        self.cap_s = _round_up(self.compact_len + max_new_tokens + gamma + 2, 64)
        dev = model.device
        # With a seq_shard.ShardExchange this rank is the owner of a sequence-
        # sharded dense cache: it stores keys [dense_shift, cap_d) locally and
        # every dense forward attends over all ranks' ranges.
        self.shard = shard
        self.dense_shift = 0
        if shard is not None:
            if shard.plan.cap != self.cap_d or not shard.is_owner:
                raise ValueError("the shard plan must be built for this runner's dense capacity, on the owner rank")
            self.dense_shift = shard.plan.key_range(shard.plan.owner)[0]
        self.dense = allocate_kv_cache(model, batch_size, self.cap_d - self.dense_shift)
        if sparse_cache == "indexed":
            # tail: draft-path K/V of generated tokens; prompt rows by position
            self.sparse_shift = self.compact_len
            self.sparse = allocate_kv_cache(model, batch_size, _round_up(max_new_tokens + gamma + 2, 64))
            self.sel_idx = torch.zeros(c.num_hidden_layers, batch_size, c.num_key_value_heads, self.compact_len,
                                       dtype=torch.int32, device=model.device)
            sel_shape = (c.num_hidden_layers, batch_size, c.num_key_value_heads, k)
            self.topk_init = torch.zeros(sel_shape, dtype=torch.int32, device=model.device)
            self.topk_cur = torch.zeros_like(self.topk_init)
        else:
            self.sparse_shift = 0
            self.sparse = allocate_kv_cache(model, batch_size, self.cap_s)
            self.sel_idx = None
        model.rope_tables(self.cap_d + 2)
        self.dense_rows = _round_up(batch_size * (gamma + 1), 16)
        if self.dense_rows > 128:
            raise ValueError("requests x (gamma + 1) must be <= 128 (the fused decode GEMMs' row limit)")
        self.ws = Workspace(model, max(self.dense_rows, batch_size))
        B = batch_size
        i32 = dict(dtype=torch.int32, device=dev)
        self.tok_stride = gamma + 2
        self.tok = torch.zeros(B, self.tok_stride, **i32)
        self.vpred = torch.zeros(B, gamma + 1, **i32)
        self.ctx_len = torch.zeros(B, **i32)
        self.dense_len = torch.zeros(B, **i32)
        self.sparse_len = torch.zeros(B, **i32)
        self.n_gen = torch.zeros(B, **i32)
        self.done = torch.zeros(B, **i32)
        self.active = torch.zeros(B, **i32)
        self.next_tok = torch.zeros(B, **i32)
        self.dense_next = torch.zeros(B, **i32)
        self.out_tokens = torch.zeros(B, max_new_tokens, **i32)
        self.stats = torch.zeros(B, 4, **i32)
        self.hist_cap = max_new_tokens + 1
        self.accept_hist = torch.zeros(B, self.hist_cap, **i32)
        self.all_done = torch.zeros(1, **i32)
        # verification policy state
        self.vmargin = torch.zeros(B, gamma + 1, dtype=torch.float32, device=dev)
        self.rerun = torch.zeros(B, **i32)
        self.first_accept = torch.zeros(B, **i32)
        self.pol_counters = torch.zeros(B, 3, **i32)  # margin reruns, fallbacks, accepted extra
        self.margin_hist = torch.full((B, self.hist_cap), float("nan"), dtype=torch.float32, device=dev)
        self.any_rerun = torch.zeros(1, **i32)
        self._if_stream: Optional[torch.cuda.Stream] = None
        self.all_done_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.topk = torch.zeros(c.num_hidden_layers, c.num_key_value_heads, k, **i32)
        self.topk_per_request: List[torch.Tensor] = []
        self._graphs: Dict[str, torch.cuda.CUDAGraph] = {}
        self.loop_counter = torch.zeros(1, **i32)
        self._loop_launches: Dict[str, Dict[str, int]] = {}
        self._body_stream: Optional[torch.cuda.Stream] = None
        # decode loops as one graph each (a WHILE node around a round / AR
        # step): no host round trip between rounds.  The host-driven loop
        # remains for dynamic re-selection (its update allocates) and for a
        # sequence-sharded owner (its collectives run outside graphs).
        self.device_loop = device_loop and use_graphs and shard is None and not self.dynamic
        self.prefill_done = False
        if self.dynamic:
            # relevance over prompt positions (only visual ones are ranked)
            self.relevance = torch.zeros(c.num_hidden_layers, batch_size, c.num_key_value_heads, P,
                                         dtype=torch.float32, device=dev)
            self.sel_stats = torch.zeros(batch_size, 2, dtype=torch.float32, device=dev)  # updates, changed sum
            self.update_flag = torch.zeros(batch_size, dtype=torch.bool, device=dev)

    @staticmethod
    def dense_capacity(prompt_len: int, max_new_tokens: int, gamma: int) -> int:
        return _round_up(prompt_len + max_new_tokens + gamma + 2, 128)

    # ------------------------------------------------------------------ prefill
    def prefill(self, embeds: Sequence[torch.Tensor], with_selection: bool = True, observe=None) -> Dict[str, float]:
        """Prefill every request (embeds[b]: [P, H] bf16) and, for STD, select and compact.

        observe(b, layer, q_text, k_rows, P, q_start, scores) sees every
        layer's selection inputs and scores (parity checks)."""
        c = self.model.config
        L, Hkv, P = c.num_hidden_layers, c.num_key_value_heads, self.layout.prompt_len
        t = {"prefill_time": 0.0, "selection_time": 0.0, "sparse_cache_time": 0.0}
        scores = torch.empty(L, Hkv, P, dtype=torch.float32, device=self.model.device) if with_selection else None
        self.topk_per_request = []
        dn = []
        # a sharded owner prefills into a whole-length cache, then hands out the ranges
        full = self.dense if self.shard is None else allocate_kv_cache(self.model, self.B, self.cap_d)
        for b in range(self.B):
            torch.cuda.synchronize()
            t0 = time.time()
            obs = None
            if observe is not None and with_selection:
                obs = (lambda li, q, k, P_, s0, b=b: observe(b, li, q, k, P_, s0, scores[li]))
            dn.append(prefill_request(self.model, full, b, embeds[b], self.layout.text_start, scores, obs))
            torch.cuda.synchronize()
            t1 = time.time()
            t["prefill_time"] += t1 - t0
            if with_selection:
                topk = build_sparse_selection(scores, self.layout, self.k)
                torch.cuda.synchronize()
                t2 = time.time()
                if self.sel_idx is not None:
                    self.topk_init[:, b] = topk
                    self.topk_cur[:, b] = topk
                    self._rebuild_selection()
                else:
                    compact_sparse_prompt_cache(full, self.sparse, b, self.layout, topk)
                torch.cuda.synchronize()
                t["selection_time"] += t2 - t1
                t["sparse_cache_time"] += time.time() - t2
                self.topk_per_request.append(topk.clone())
        if self.shard is not None:
            torch.cuda.synchronize()
            t0 = time.time()
            self.shard.distribute(full, self.dense, P)
            del full
            torch.cuda.synchronize()
            t["shard_distribute_time"] = time.time() - t0
        self.dense_next.copy_(torch.tensor(dn, dtype=torch.int32))
        self.prefill_done = True
        return t

    # ------------------------------------------------------------------ state
    def reset(self) -> None:
        P = self.layout.prompt_len
        self.ctx_len.fill_(P)
        self.dense_len.fill_(P)
        self.sparse_len.fill_(self.compact_len)
        self.n_gen.zero_()
        self.done.zero_()
        self.active.zero_()
        self.stats.zero_()
        self.accept_hist.zero_()
        self.out_tokens.zero_()
        self.tok.zero_()
        self.tok[:, 0] = self.dense_next   # AR: current token
        self.tok[:, 1] = self.dense_next   # STD: sparse_next = dense_next (copy_sparse_prefill)
        self.all_done.zero_()
        self.pol_counters.zero_()
        self.margin_hist.fill_(float("nan"))
        if self.dynamic:  # every decode starts from the static selection S_0
            self.topk_cur.copy_(self.topk_init)
            self._rebuild_selection()
            self.relevance.zero_()
            self.sel_stats.zero_()

    def _rebuild_selection(self) -> None:
        """sel_idx = sorted(non_visual ∪ topk_cur) per (layer, request, KV head)."""
        L, B, H, _ = self.topk_cur.shape
        nv = self.layout.non_visual.view(1, 1, 1, -1).expand(L, B, H, -1)
        self.sel_idx.copy_(torch.cat([nv, self.topk_cur], dim=-1).sort(dim=-1).values)

    def _collect(self, li: int, q4: torch.Tensor) -> None:
        """Collector v1 (dynamic_selection.py:290-308) for layer li of a verify
        forward, on the device in fp32 (libstd_b200 collect.cu): A[b, h, v] =
        sum over the verify queries of softmax over the visual keys of
        (group-mean query . k_v) / sqrt(D), written at the visual positions."""
        ops.collect_relevance(q4, self.dense[li, 0], self.layout.visual_pos, self.relevance[li])

    def _update_selection(self) -> None:
        """S_{t+1} = TopK(A_t) per (layer, request, KV head), applied to request
        b when its selection changed by at least min_selection_change_ratio
        (Jaccard distance averaged over layers and heads,
        dynamic_selection.py:55-83)."""
        L, B, H, k = self.topk_cur.shape
        P = self.relevance.shape[-1]
        new = ops.topk_select(self.relevance.view(L * B * H, P), self.layout.visual_pos, k).view(L, B, H, k)
        inter = topk_intersection_counts(new, self.topk_cur).float()
        jac = (inter / (2 * k - inter).clamp(min=1)).mean(dim=(0, 2))  # [B]
        changed = 1.0 - jac
        torch.ge(changed, self.min_change, out=self.update_flag)
        self.topk_cur.copy_(torch.where(self.update_flag.view(1, B, 1, 1), new, self.topk_cur))
        self._rebuild_selection()
        self.sel_stats[:, 0] += self.update_flag.float()
        self.sel_stats[:, 1] += changed

    # ------------------------------------------------------------------ steps
    def _sparse_index(self):
        return None if self.sel_idx is None else (self.dense, self.sel_idx)

    def _draft_step(self, i: int) -> None:
        last = i == self.gamma - 1
        decode_forward(self.model, self.ws, self.sparse, B=self.B, n=1, rows=self.B, tok=self.tok, tok_start=1 + i,
                       pos_base=self.ctx_len, pos_off=i, slot_base=self.sparse_len, slot_off=i - self.sparse_shift,
                       lens=self.sparse_len, len_offset=i + 1, sparse=True,
                       argmax_out=None if last else self.tok.view(-1), argmax_stride=self.tok_stride,
                       argmax_start=2 + i, sparse_index=self._sparse_index())

    def _verify(self, pending: int) -> None:
        nq = self.gamma + pending
        sh = self.dense_shift
        decode_forward(self.model, self.ws, self.dense, B=self.B, n=nq, rows=self.dense_rows, tok=self.tok,
                       tok_start=1 - pending, pos_base=self.dense_len, pos_off=0, slot_base=self.dense_len,
                       slot_off=-sh, lens=self.dense_len, len_offset=nq - sh, sparse=False,
                       argmax_out=self.vpred.view(-1), argmax_stride=self.gamma + 1, argmax_start=0,
                       dense_attn=self.shard, collector=self._collect if self.dynamic else None,
                       margin_out=self.vmargin.view(-1) if self.margin_threshold is not None else None)

    def _verify_sequential(self, pending: int) -> None:
        """verify_mode="sequential" (std_qwen25vl.py:504-528, :775-781, :885-893):
        the pending bonus and every draft token go through the dense model one
        token at a time (q_len = 1, the AR step's kernels and padded row
        count), each prediction landing in the same slot as the parallel
        block's.  The reference stops at the first mismatch; here the tokens
        after it are still run (no host round trip per token), but they cannot
        change the accepted prefix or the bonus -- both are functions of the
        predictions up to the first mismatch -- and their cache rows lie past
        the rolled-back dense length, so they are overwritten next round."""
        nq = self.gamma + pending
        sh = self.dense_shift
        for j in range(nq):
            decode_forward(self.model, self.ws, self.dense, B=self.B, n=1, rows=self.dense_rows, tok=self.tok,
                           tok_start=1 - pending + j, pos_base=self.dense_len, pos_off=j, slot_base=self.dense_len,
                           slot_off=j - sh, lens=self.dense_len, len_offset=j + 1 - sh, sparse=False,
                           argmax_out=self.vpred.view(-1), argmax_stride=self.gamma + 1, argmax_start=j,
                           dense_attn=self.shard)

    def _accept(self, pending: int) -> None:
        from . import _lib

        _lib.call("std_accept_commit", self.B, self.gamma, pending, self.tok.data_ptr(), self.tok_stride,
                  self.vpred.data_ptr(), self.gamma + 1, self.dense_next.data_ptr(), self.max_new, self.eos,
                  1 if self.ignore_eos else 0, self.ctx_len.data_ptr(), self.dense_len.data_ptr(),
                  self.sparse_len.data_ptr(), self.n_gen.data_ptr(), self.done.data_ptr(),
                  self.out_tokens.data_ptr(), self.stats.data_ptr(), self.accept_hist.data_ptr(), self.hist_cap,
                  torch.cuda.current_stream().cuda_stream)

    def _bonus_step(self) -> None:
        decode_forward(self.model, self.ws, self.sparse, B=self.B, n=1, rows=self.B, tok=self.tok, tok_start=0,
                       pos_base=self.ctx_len, pos_off=-1, slot_base=self.sparse_len, slot_off=-1 - self.sparse_shift,
                       lens=self.sparse_len, len_offset=0, sparse=True, argmax_out=self.tok.view(-1),
                       argmax_stride=self.tok_stride, argmax_start=1, sparse_index=self._sparse_index())

    def _drafts(self) -> None:
        for i in range(self.gamma):
            self._draft_step(i)

    def _verify_phase(self, pending: int) -> None:
        if self.verify_mode == "sequential":
            self._verify_sequential(pending)
        else:
            self._verify(pending)
            if self.policy_active:
                self._policy(pending)

    def _policy_call(self, pending: int, cond: int, after: int) -> None:
        from . import _lib

        thr = float("nan") if self.margin_threshold is None else float(self.margin_threshold)
        _lib.call("std_verify_policy", self.B, self.gamma, pending, self.tok.data_ptr(), self.tok_stride,
                  self.vpred.data_ptr(), self.gamma + 1, self.dense_next.data_ptr(), self.max_new,
                  self.n_gen.data_ptr(), self.done.data_ptr(), self.stats.data_ptr(), self.vmargin.data_ptr(), thr,
                  self.policy_mode, self.max_accept, 1 if self.math_on_full_accept else 0, self.rerun.data_ptr(),
                  self.first_accept.data_ptr(), self.pol_counters.data_ptr(), self.margin_hist.data_ptr(),
                  self.hist_cap, self.any_rerun.data_ptr(), cond, after, torch.cuda.current_stream().cuda_stream)

    def _policy(self, pending: int) -> None:
        """Decide, per request, whether this round's parallel verify is
        re-verified (margin check, math_on_full_accept, verify_fallback), and
        if any request asks, replay the round's dense predictions one token at
        a time (the sequential verify) before the accept kernel commits.
        Under graph capture the decision is an IF node whose condition the
        policy kernel sets on the device; eagerly the host reads it."""
        import ctypes

        from . import _lib

        if torch.cuda.is_current_stream_capturing():
            s = torch.cuda.current_stream()
            h = ctypes.c_ulonglong(0)
            _lib.call("std_graph_cond_handle", s.cuda_stream, ctypes.byref(h))
            self._policy_call(pending, h.value, 0)
            if self._if_stream is None:
                raise RuntimeError("capture() creates the replay stream before capturing")
            _lib.call("std_capture_if_begin", s.cuda_stream, self._if_stream.cuda_stream, h.value)
            with torch.cuda.stream(self._if_stream):
                self._verify_sequential(pending)
                self._policy_call(pending, 0, 1)
            _lib.call("std_capture_if_end", self._if_stream.cuda_stream)
            return
        self._policy_call(pending, 0, 0)
        if int(self.any_rerun.item()):
            self._verify_sequential(pending)
            self._policy_call(pending, 0, 1)

    def _post(self, pending: int, update: bool = False) -> None:
        self._accept(pending)
        if update:  # before the bonus append, which already uses S_{t+1}
            self._update_selection()
        self._bonus_step()
        torch.amin(self.done, dim=0, keepdim=True, out=self.all_done)

    def std_round(self, first: bool, update: bool = False) -> None:
        pending = 0 if first else 1
        self._drafts()
        self._verify_phase(pending)
        self._post(pending, update)

    def ar_step(self) -> None:
        from . import _lib

        s = torch.cuda.current_stream().cuda_stream
        _lib.call("std_ar_commit", self.B, self.tok_stride, self.max_new, self.eos, 1 if self.ignore_eos else 0,
                  self.tok.data_ptr(), self.n_gen.data_ptr(), self.done.data_ptr(), self.out_tokens.data_ptr(),
                  self.active.data_ptr(), s)
        sh = self.dense_shift
        decode_forward(self.model, self.ws, self.dense, B=self.B, n=1, rows=self.dense_rows, tok=self.tok,
                       tok_start=0, pos_base=self.dense_len, pos_off=0, slot_base=self.dense_len, slot_off=-sh,
                       lens=self.dense_len, len_offset=1 - sh, sparse=False, argmax_out=self.next_tok,
                       dense_attn=self.shard)
        _lib.call("std_ar_advance", self.B, self.active.data_ptr(), self.next_tok.data_ptr(), self.tok.data_ptr(),
                  self.tok_stride, self.dense_len.data_ptr(), self.ctx_len.data_ptr(), s)
        torch.amin(self.done, dim=0, keepdim=True, out=self.all_done)

    # ------------------------------------------------------------------ graphs
    def capture(self, mode: str = "all") -> None:
        """Capture the CUDA graphs a decode of `mode` ("std", "ar" or "all") replays.

        Device loop: one graph per mode (std_loop / ar_loop).  Host-driven
        loop: the round-1, steady-state (and selection-update) round graphs
        and the AR-step graph; a sequence-sharded owner captures only its
        local phases.  Each step runs once eagerly first (allocating
        workspaces and setting kernel attributes outside capture); state is
        reset afterwards."""
        if not self.use_graphs:
            return
        if self.policy_active and self._if_stream is None:
            self._if_stream = _lib_capture_stream("if_body")
        want_std, want_ar = mode in ("std", "all"), mode in ("ar", "all")
        if self.shard is not None and not self._shard_rounds_captured():
            # collectives stay outside the graphs: the dense forwards (verify,
            # AR steps) run eagerly between captured local phases
            steps = [("drafts", self._drafts), ("post_first", lambda: self._post(0)), ("post", lambda: self._post(1))]
        elif self.device_loop:
            steps = []
            if want_std and "std_loop" not in self._graphs:
                steps += [("std_first", lambda: self.std_round(True)), ("std", lambda: self.std_round(False))]
            if want_ar and "ar_loop" not in self._graphs:
                steps += [("ar", self.ar_step)]
        else:
            steps = []
            if want_std:
                steps += [("std_first", lambda: self.std_round(True)), ("std", lambda: self.std_round(False))]
                if self.dynamic:
                    steps += [("std_first_upd", lambda: self.std_round(True, True)),
                              ("std_upd", lambda: self.std_round(False, True))]
            if want_ar:
                steps += [("ar", self.ar_step)]
        for name, fn in steps:
            if name in self._graphs:
                continue
            self.reset()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                fn()
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            if self.device_loop:
                continue  # eager warm-up only: the loop graphs below hold these steps
            self.reset()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            self._graphs[name] = g
        if self.device_loop:
            self._capture_loops(want_std, want_ar)
        self.reset()
        torch.cuda.synchronize()

    def _capture_loops(self, want_std: bool, want_ar: bool) -> None:
        """std_loop: round 1, then a WHILE node around steady-state rounds;
        ar_loop: a WHILE node around AR steps.  The loop condition is set on
        the device from the done flags (libstd_b200 graph_loop.cu), bounded by
        max_new_tokens + 1 iterations.  Every step already ran eagerly in
        capture(), so nothing allocates while the body is captured."""
        import ctypes

        from . import _lib

        if self._body_stream is None:
            self._body_stream = _lib_capture_stream("while_body")
        body_stream = self._body_stream
        limit = self.max_new + 1

        def launches() -> int:
            return int(_lib.query("std_launch_count"))

        def loop(body) -> None:
            h = ctypes.c_ulonglong(0)
            counts["outer"] = launches() - counts["start"] + 1  # + the loop's init kernel
            _lib.call("std_capture_while_begin", torch.cuda.current_stream().cuda_stream, body_stream.cuda_stream,
                      self.done.data_ptr(), self.B, self.loop_counter.data_ptr(), ctypes.byref(h), None)
            n0 = launches()
            with torch.cuda.stream(body_stream):
                body()
            counts["body"] = launches() - n0 + 1  # + the loop's condition update
            _lib.call("std_capture_while_end", body_stream.cuda_stream, h.value, self.done.data_ptr(), self.B,
                      self.loop_counter.data_ptr(), limit)

        loops = []
        if want_std:
            loops.append(("std_loop", lambda: (self.std_round(True), loop(lambda: self.std_round(False)))))
        if want_ar:
            loops.append(("ar_loop", lambda: loop(self.ar_step)))
        for name, fn in loops:
            if name in self._graphs:
                continue
            self.reset()
            torch.cuda.synchronize()
            counts = {"start": launches()}
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            self._graphs[name] = g
            self._loop_launches[name] = {"outer": counts["outer"], "body": counts["body"]}

    def launch_counts(self, name: str) -> Dict[str, int]:
        """This library's kernel launches in one replay of loop graph `name`
        ("std_loop" / "ar_loop"): "outer" run once per decode (round 1 and the
        loop's init kernel), "body" once per loop iteration (a round or an AR
        step, and the condition update).  Counted from the library's launch
        counter while the graph was captured."""
        return dict(self._loop_launches[name])

    def _all_done(self) -> bool:
        self.all_done_host.copy_(self.all_done, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return bool(self.all_done_host.item())

    # ------------------------------------------------------------------ loops
    def run_std(self, device_loop: Optional[bool] = None) -> float:
        """STD decode of every request from the post-prefill state; returns seconds (device time).

        With the device loop the whole decode is one graph launch and one
        synchronisation; otherwise (device_loop=False, or a runner built
        without it) the host launches a round graph and reads the 4-byte
        all-done flag after each round."""
        if device_loop is False and self.device_loop:
            return self._without_device_loop(self.run_std)
        self.capture("std")
        self.reset()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        loop = self._graphs.get("std_loop")
        if loop is not None:
            start.record()
            loop.replay()
            end.record()
            end.synchronize()
            if not bool(self.done.all().item()):
                raise RuntimeError("STD decode did not terminate within max_new_tokens + 1 rounds")
            return start.elapsed_time(end) / 1000.0
        start.record()
        self._round(True, self._update_due(1))
        rounds = 1
        while not self._all_done():
            if rounds > self.max_new + 1:
                raise RuntimeError("STD decode did not terminate")
            rounds += 1
            self._round(False, self._update_due(rounds))
        end.record()
        end.synchronize()
        return start.elapsed_time(end) / 1000.0

    def _without_device_loop(self, fn):
        """Run fn with the host-driven loop (per-round graphs) on this runner."""
        saved = {k: self._graphs.pop(k) for k in ("std_loop", "ar_loop") if k in self._graphs}
        self.device_loop = False
        try:
            return fn()
        finally:
            self.device_loop = True
            self._graphs.update(saved)

    def run_ar(self, device_loop: Optional[bool] = None) -> float:
        if device_loop is False and self.device_loop:
            return self._without_device_loop(self.run_ar)
        self.capture("ar")
        self.reset()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        loop = self._graphs.get("ar_loop")
        if loop is not None:
            start.record()
            loop.replay()
            end.record()
            end.synchronize()
            if not bool(self.done.all().item()):
                raise RuntimeError("AR decode did not terminate within max_new_tokens + 1 steps")
            return start.elapsed_time(end) / 1000.0
        start.record()
        steps = 0
        while True:
            self._replay_or_run("ar", self.ar_step, 1)
            steps += 1
            if steps >= self.max_new:
                if self._all_done():
                    break
            elif steps % 16 == 0 and self._all_done():
                break
        end.record()
        end.synchronize()
        return start.elapsed_time(end) / 1000.0

    def run_std_profiled(self) -> Dict[str, float]:
        """STD decode with per-phase device timers (profile_decode=True; the
        reference's _profile_mark stages, std_qwen25vl.py:771-939, and
        decode_profiler.py:85-145).  Each round runs as four graphs -- the
        gamma draft steps, the dense verify, the fused accept/rollback, the
        bonus sparse step -- with CUDA events between them, and the host
        reads the all-done flag after every round as the reference does.
        Returns seconds per phase: draft_time, verify_time, cache_adjust_time
        (accept + cache-length rollback), bonus_time, and decoding_time."""
        if self.shard is not None or self.dynamic:
            raise ValueError("profiled decode covers the single-GPU static-selection runner")
        phases = {"drafts": self._drafts, "verify_first": lambda: self._verify_phase(0),
                  "verify": lambda: self._verify_phase(1), "accept_first": lambda: self._accept_and_flag(0),
                  "accept": lambda: self._accept_and_flag(1), "bonus": self._bonus_step}
        if self.policy_active and self._if_stream is None:
            self._if_stream = _lib_capture_stream("if_body")
        if self.use_graphs and any("phase_" + name not in self._graphs for name in phases):
            # Warm up with whole rounds (workspaces, kernel attributes), never
            # with a phase out of its round: a bonus step run straight after
            # reset() would write its K/V row over the last prompt row of the
            # sparse cache.  Capturing a phase runs nothing.
            self.reset()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self.std_round(True)
                self.std_round(False)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            for name, fn in phases.items():
                key = "phase_" + name
                if key in self._graphs:
                    continue
                self.reset()
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    fn()
                self._graphs[key] = g
        self.reset()
        torch.cuda.synchronize()
        marks = []
        rounds = 0
        t0 = torch.cuda.Event(enable_timing=True)
        t0.record()
        while True:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
            first = rounds == 0
            ev[0].record()
            self._replay_or_run("phase_drafts", phases["drafts"])
            ev[1].record()
            name = "verify_first" if first else "verify"
            self._replay_or_run("phase_" + name, phases[name])
            ev[2].record()
            name = "accept_first" if first else "accept"
            self._replay_or_run("phase_" + name, phases[name])
            ev[3].record()
            self._replay_or_run("phase_bonus", phases["bonus"])
            ev[4].record()
            marks.append(ev)
            rounds += 1
            if self._all_done():
                break
            if rounds > self.max_new + 1:
                raise RuntimeError("STD decode did not terminate")
        t1 = torch.cuda.Event(enable_timing=True)
        t1.record()
        t1.synchronize()
        out = {"draft_time": 0.0, "verify_time": 0.0, "cache_adjust_time": 0.0, "bonus_time": 0.0}
        for ev in marks:
            out["draft_time"] += ev[0].elapsed_time(ev[1]) / 1000.0
            out["verify_time"] += ev[1].elapsed_time(ev[2]) / 1000.0
            out["cache_adjust_time"] += ev[2].elapsed_time(ev[3]) / 1000.0
            out["bonus_time"] += ev[3].elapsed_time(ev[4]) / 1000.0
        out["decoding_time"] = t0.elapsed_time(t1) / 1000.0
        return out

    def _accept_and_flag(self, pending: int) -> None:
        self._accept(pending)
        torch.amin(self.done, dim=0, keepdim=True, out=self.all_done)

    def _update_due(self, round_id: int) -> bool:
        """Selection updates run after rounds round_id % interval == 0 (one-based)."""
        return self.dynamic and round_id % self.update_interval == 0

    def _shard_rounds_captured(self) -> bool:
        """A sequence-sharded owner whose exchange runs over peer memory
        (kernels only) captures whole rounds and AR steps like an unsharded
        runner, announcing each replay's one dense forward to the shard
        servers first.  Rounds whose number of dense forwards is decided on
        the device (policy re-verifies) or that run several (sequential
        verify) keep the eager dense forwards."""
        return (self.shard is not None and self.shard.capturable and self.verify_mode == "parallel"
                and not self.policy_active and not self.dynamic)

    def _round(self, first: bool, update: bool = False) -> None:
        pending = 0 if first else 1
        if self.shard is None or self._shard_rounds_captured():
            name = ("std_first" if first else "std") + ("_upd" if update else "")
            self._replay_or_run(name, lambda: self.std_round(first, update), self.gamma + pending)
            return
        self._replay_or_run("drafts", self._drafts)
        self._verify_phase(pending)
        self._replay_or_run("post_first" if first else "post", lambda: self._post(pending))

    def _replay_or_run(self, name: str, fn, dense_nq: int = 0) -> None:
        """Replay graph `name` (announcing its dense forward of dense_nq
        tokens to the shard servers first, when sharded) or run fn eagerly."""
        g = self._graphs.get(name)
        if g is not None:
            if self.shard is not None and dense_nq:
                self.shard.announce(dense_nq)
            g.replay()
        else:
            fn()

    # ------------------------------------------------------------------ results
    def generated(self) -> torch.Tensor:
        return self.out_tokens[:, : int(self.n_gen.max().item())].to(torch.int64).cpu()

    def selection_stats(self) -> Dict[str, object]:
        """Dynamic re-selection bookkeeping of the last decode, per request."""
        if not self.dynamic:
            return {"policy": "static", "updates": [0] * self.B, "mean_changed_ratio": [0.0] * self.B}
        st = self.sel_stats.cpu()
        rounds = self.stats[:, 0].cpu().clamp(min=1).float()
        return {"policy": "previous_verify_topk", "updates": st[:, 0].int().tolist(),
                "mean_changed_ratio": (st[:, 1] / rounds).tolist()}

    def std_stats(self) -> Dict[str, object]:
        """Per-request round records of the last STD decode.  proposed_lengths
        and pending_lengths follow the reference's per-round bookkeeping
        (std_qwen25vl.py:783-793): a round proposes min(gamma, remaining)
        drafts, and every round after the first carries one pending bonus."""
        st = self.stats.cpu()
        hist = self.accept_hist.cpu()
        rounds = st[:, 0].tolist()
        accept = [hist[b, : rounds[b]].tolist() for b in range(self.B)]
        proposed = []
        for b in range(self.B):
            n_gen, props = 0, []
            for a in accept[b]:
                remaining = self.max_new - n_gen
                props.append(min(self.gamma, remaining))
                n_gen += min(a + 1, remaining)
            proposed.append(props)
        pc = self.pol_counters.cpu()
        mh = self.margin_hist.cpu()
        margins = [[float(m) for m in mh[b, : rounds[b]].tolist() if m == m] for b in range(self.B)]
        return {
            "rounds": rounds,
            "accepted": st[:, 1].tolist(),
            "proposed": st[:, 2].tolist(),
            "accept_lengths": accept,
            "proposed_lengths": proposed,
            "pending_lengths": [[0] + [1] * (r - 1) if r > 0 else [] for r in rounds],
            "verify_margin_reruns": pc[:, 0].tolist(),
            "fallback_count": pc[:, 1].tolist(),
            "fallback_accepted_extra": pc[:, 2].tolist(),
            "verify_margins": margins,
        }


# ----------------------------------------------------------------------------
# reference-shaped entry points
# ----------------------------------------------------------------------------

def _std_result(runner: STDRunner, ids: torch.Tensor, decoding_time: float, t0: float, tp: Dict[str, float],
                gamma: int, prof: Optional[Dict[str, float]] = None) -> GenerateResult:
    """GenerateResult of an STD decode over every request of the batch: counts
    are summed, the per-round lists concatenate the requests' rounds in
    request order, and mean_accept_length is accepted drafts per round over
    all requests' rounds (for one request: the reference's definition,
    std_qwen25vl.py:943)."""
    gen = runner.generated()
    out = torch.cat([ids.cpu().long(), gen], dim=1) if ids.shape[0] == gen.shape[0] else gen
    st = runner.std_stats()
    acc = [a for r in st["accept_lengths"] for a in r]
    prof = prof or {}
    return GenerateResult(
        output_ids=out, decoding_time=decoding_time, inference_time=time.time() - t0,
        generate_len=int(runner.n_gen.sum().item()), accepted_draft_tokens=int(sum(st["accepted"])),
        proposed_draft_tokens=int(sum(st["proposed"])), mean_accept_length=(sum(acc) / len(acc)) if acc else 0.0,
        decode_rounds=int(max(st["rounds"])), final_gamma=gamma, gamma_history=[gamma] * int(max(st["rounds"])),
        accept_lengths=acc, proposed_lengths=[p for r in st["proposed_lengths"] for p in r],
        pending_lengths=[p for r in st["pending_lengths"] for p in r],
        fallback_count=int(sum(st["fallback_count"])), fallback_accepted_extra=int(sum(st["fallback_accepted_extra"])),
        verify_margin_reruns=int(sum(st["verify_margin_reruns"])),
        min_verify_margin=min((m for r in st["verify_margins"] for m in r), default=0.0),
        draft_time=prof.get("draft_time", 0.0), verify_time=prof.get("verify_time", 0.0),
        bonus_time=prof.get("bonus_time", 0.0), cache_adjust_time=prof.get("cache_adjust_time", 0.0),
        prefill_time=tp["prefill_time"], selection_time=tp["selection_time"],
        sparse_cache_time=tp["sparse_cache_time"], request_accept_lengths=st["accept_lengths"],
        request_generate_lens=runner.n_gen.cpu().tolist())


def _prepare(model: Qwen25VLDecoder, inputs: Dict[str, torch.Tensor], video_token_id: int):
    ids = inputs["input_ids"]
    if ids.dim() == 1:
        ids = ids.view(1, -1)
    B, P = ids.shape
    layout = PromptLayout.from_ids(ids[0], video_token_id, model.device)
    for b in range(1, B):
        if not torch.equal((ids[b] == video_token_id).cpu(), (ids[0] == video_token_id).cpu()):
            raise ValueError("all requests of a batch must share the video/text layout")
    vis = inputs["visual_embeds"]
    if vis.dim() == 2:
        vis = vis.unsqueeze(0)
    ids_dev = ids.to(model.device, non_blocking=True)
    vis_dev = vis.to(model.device, non_blocking=True)
    embeds = []
    vpos = layout.visual_pos.long()
    for b in range(B):
        e = model.embed[ids_dev[b].clamp(0, model.config.vocab_size - 1)]
        e[vpos] = vis_dev[b].to(model.dtype)
        embeds.append(e)
    return ids, layout, embeds


@torch.inference_mode()
def ar_generate_qwen25vl(model: Qwen25VLDecoder, inputs: Dict[str, torch.Tensor], video_token_id: int,
                         eos_token_id: int, max_new_tokens: int = 256, output_attentions: bool = False,
                         profile_prefill: bool = False, ignore_eos: bool = False,
                         runner: Optional[STDRunner] = None) -> GenerateResult:
    """Vanilla greedy decoding with the same two-stage prefill as STD (std_qwen25vl.py:553-606).

    inputs: {"input_ids": [B, P], "visual_embeds": [B, V, H]} -- the visual
    rows replace the embeddings of the video-token positions (the vision tower
    is outside this path)."""
    torch.cuda.synchronize()
    t0 = time.time()
    ids, layout, embeds = _prepare(model, inputs, video_token_id)
    if runner is None:
        runner = STDRunner(model, ids.shape[0], layout, max_new_tokens, gamma=9, k=1, eos_token_id=eos_token_id,
                           ignore_eos=ignore_eos)
    tp = runner.prefill(embeds, with_selection=False)
    dec = runner.run_ar()
    torch.cuda.synchronize()
    gen = runner.generated()
    out = torch.cat([ids.cpu().long(), gen], dim=1) if ids.shape[0] == gen.shape[0] else gen
    return GenerateResult(out, dec, time.time() - t0, int(runner.n_gen.sum().item()),
                          prefill_time=tp["prefill_time"])


@torch.inference_mode()
def std_generate_qwen25vl(model: Qwen25VLDecoder, inputs: Dict[str, torch.Tensor], video_token_id: int,
                          eos_token_id: int, max_new_tokens: int = 256, gamma: int = 9,
                          target_k_plus_text: int = 1024, explicit_k: Optional[int] = None,
                          verify_mode: str = "parallel", verify_fallback: str = "none",
                          sequential_fallback_max_accept: int = 1, profile_decode: bool = False,
                          sparse_attn_mode: str = "b200", adaptive_gamma_min: Optional[int] = None,
                          adaptive_gamma_mode: str = "accept_len", copy_sparse_prefill: bool = True,
                          profile_prefill: bool = False, verify_attn_backend: str = "default",
                          verify_margin_threshold: Optional[float] = None, use_compile: bool = False,
                          ignore_eos: bool = False, runner: Optional[STDRunner] = None,
                          sparse_cache: str = "compact") -> Tuple[GenerateResult, SparseSelection]:
    """Sparse-to-Dense greedy decoding (std_qwen25vl.py:609-978).

    Implemented: verify_mode "parallel" | "sequential"; every verify_fallback
    mode, verify_margin_threshold (with min_verify_margin and
    verify_margin_reruns) and verify_attn_backend "default" | "math" |
    "math_on_full_accept", decided per request on the device; a
    re-verification (the reference's math-backend rerun or sequential
    fallback) is the exact one-token-at-a-time replay of the round's dense
    predictions.  The verify kernel is the only attention backend, so "math"
    runs it too (it is already exact: a verify row equals the AR step's row bit
    for bit).  sparse_attn_mode="b200", copy_sparse_prefill=True, fixed gamma;
    adaptive gamma and torch.compile raise ValueError.  profile_decode=True
    fills draft_time / verify_time / cache_adjust_time / bonus_time from CUDA
    events between the round's phases.  B200 extension: sparse_cache=
    "indexed" reads the selected prompt rows in place from the dense cache
    instead of compacting a copy (same tokens)."""
    if verify_mode not in VERIFY_MODES:
        raise ValueError(f"Unsupported verify_mode={verify_mode!r}; expected one of {VERIFY_MODES}.")
    if sparse_attn_mode not in SPARSE_ATTN_MODES:
        raise ValueError(f"Unsupported sparse_attn_mode={sparse_attn_mode!r}; expected 'b200'.")
    if adaptive_gamma_min is not None or use_compile or not copy_sparse_prefill:
        raise ValueError("adaptive gamma, torch.compile and a separate sparse prefill are not part of the B200 path.")
    torch.cuda.synchronize()
    t0 = time.time()
    ids, layout, embeds = _prepare(model, inputs, video_token_id)
    k = selection_budget(layout.prompt_len, layout.text_start, int(layout.visual_pos.numel()), target_k_plus_text,
                         explicit_k)
    if runner is None:
        runner = STDRunner(model, ids.shape[0], layout, max_new_tokens, gamma=gamma, k=k, eos_token_id=eos_token_id,
                           ignore_eos=ignore_eos, verify_mode=verify_mode, sparse_cache=sparse_cache,
                           verify_fallback=verify_fallback, verify_margin_threshold=verify_margin_threshold,
                           sequential_fallback_max_accept=sequential_fallback_max_accept,
                           verify_attn_backend=verify_attn_backend)
    elif (runner.verify_mode != verify_mode or runner.policy_mode != VERIFY_FALLBACKS.get(verify_fallback)
          or runner.margin_threshold != verify_margin_threshold):
        raise ValueError("the runner was built for a different verify_mode / verification policy")
    tp = runner.prefill(embeds, with_selection=True)
    prof = None
    if profile_decode and runner.shard is None:
        prof = runner.run_std_profiled()
        dec = prof["decoding_time"]
    else:
        dec = runner.run_std()
    torch.cuda.synchronize()
    result = _std_result(runner, ids, dec, t0, tp, gamma, prof)
    topk0 = runner.topk_per_request[0].cpu().long()
    selection = SparseSelection(topk_positions=[topk0[l] for l in range(topk0.shape[0])],
                                non_visual_positions=layout.non_visual.cpu().long(), prompt_len=layout.prompt_len,
                                visual_len=int(layout.visual_pos.numel()),
                                text_len=max(1, layout.prompt_len - layout.text_start), k=k)
    return result, selection


@torch.inference_mode()
def dynamic_std_generate_qwen25vl(model: Qwen25VLDecoder, inputs: Dict[str, torch.Tensor], video_token_id: int,
                                  eos_token_id: int, max_new_tokens: int = 256, gamma: int = 9,
                                  target_k_plus_text: int = 1024, explicit_k: Optional[int] = None,
                                  policy: str = "previous_verify_topk", profile_decode: bool = False,
                                  profile_prefill: bool = False, sparse_attn_mode: str = "b200",
                                  copy_sparse_prefill: bool = True, ignore_eos: bool = False,
                                  collector_version: str = "v1", refresh_mode: str = "incremental",
                                  selection_update_interval: int = 1, min_selection_change_ratio: float = 0.05,
                                  bootstrap_mode: str = "attention", verify_fallback: str = "none",
                                  runner: Optional[STDRunner] = None):
    """Verification-guided STD (dynamic_std_qwen25vl.py:109-530): the static
    prefill selection S_0, then after round t's verification S_{t+1} =
    TopK(A_t) from collector v1.  With the index-based sparse cache a refresh
    is an update of the position lists (both refresh_mode values), so the
    selected K/V rows are never copied.  Returns (result, selection, stats).
    Implemented: policy static / previous_verify_topk, collector_version
    "v1", bootstrap_mode "attention"; other research knobs raise ValueError."""
    if policy not in SELECTION_POLICIES:
        raise ValueError(f"Unsupported policy={policy!r}; expected one of {SELECTION_POLICIES}.")
    if collector_version != "v1":
        raise ValueError("collector_version: this build implements 'v1' (RuntimeVerificationCollector).")
    if refresh_mode not in ("full", "incremental"):
        raise ValueError(f"Unsupported refresh_mode={refresh_mode!r}; expected 'full' or 'incremental'.")
    if bootstrap_mode != "attention" or verify_fallback != "none":
        raise ValueError("bootstrap_mode must be 'attention' and verify_fallback 'none' in the B200 path.")
    if sparse_attn_mode not in SPARSE_ATTN_MODES or not copy_sparse_prefill:
        raise ValueError("sparse_attn_mode must be 'b200' with copy_sparse_prefill=True.")
    torch.cuda.synchronize()
    t0 = time.time()
    ids, layout, embeds = _prepare(model, inputs, video_token_id)
    k = selection_budget(layout.prompt_len, layout.text_start, int(layout.visual_pos.numel()), target_k_plus_text,
                         explicit_k)
    if runner is None:
        runner = STDRunner(model, ids.shape[0], layout, max_new_tokens, gamma=gamma, k=k, eos_token_id=eos_token_id,
                           ignore_eos=ignore_eos, sparse_cache="indexed", selection_policy=policy,
                           selection_update_interval=selection_update_interval,
                           min_selection_change_ratio=min_selection_change_ratio)
    tp = runner.prefill(embeds, with_selection=True)
    dec = runner.run_std()
    torch.cuda.synchronize()
    result = _std_result(runner, ids, dec, t0, tp, gamma)
    topk0 = runner.topk_cur[:, 0].cpu().long()
    selection = SparseSelection(topk_positions=[topk0[l] for l in range(topk0.shape[0])],
                                non_visual_positions=layout.non_visual.cpu().long(), prompt_len=layout.prompt_len,
                                visual_len=int(layout.visual_pos.numel()),
                                text_len=max(1, layout.prompt_len - layout.text_start), k=k)
    stats = dict(runner.selection_stats(), collector_version="v1", refresh_mode=refresh_mode,
                 selection_update_interval=selection_update_interval,
                 min_selection_change_ratio=min_selection_change_ratio)
    return result, selection, stats
