// decode_ops.cu -- per-token decoder kernels and (d) the fused greedy accept.
//
// Decoder pieces of the Qwen2.5-VL language model that sit between the
// library GEMMs (modeling_qwen2_5_vl.py):
//   embed        nn.Embedding lookup                     (:1336)
//   rmsnorm      Qwen2RMSNorm                            (:183-197)
//   rope_append  apply_multimodal_rotary_pos_emb with 1-D positions (:690-732,
//                positions :1368-1384) fused with KVCache.cat (kv_cache.py:54-69)
//   silu_mul     Qwen2MLP act_fn(gate) * up              (:674-687)
//   add          residual adds                           (:1200-1221)
//   argmax_rows  torch.argmax over the vocabulary, first index on ties
//                (std_qwen25vl.py:98-99, :806)
// Every kernel processes a row independently with a fixed operation order, so
// a token's result does not depend on how many tokens share the launch (AR
// rows and verify rows agree bit for bit).
//
// (d) accept_commit replaces the host-side acceptance and rollback of one STD
// round (std_qwen25vl.py:806-815 acceptance, :910-921 commit/EOS/limit,
// :923-929 cache-length rollback, :931-939 pending bonus) with one kernel over
// device-resident state, so a round needs no device->host synchronisation.
#include "common.cuh"

namespace stdb {

// ------------------------------- embed -------------------------------------
// out[b*n + j] = table[tok[b*tok_stride + tok_start + j]]
__global__ void embed_kernel(const __nv_bfloat16* table, int vocab, int H, const int32_t* tok, int tok_stride,
                             int tok_start, int n, __nv_bfloat16* out) {
  pdl_launch_dependents();  // followed by the first RMSNorm, which reads after its wait
  pdl_wait();
  const int row = blockIdx.x;
  const int b = row / n, j = row % n;
  int id = tok[b * tok_stride + tok_start + j];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) std_set_error(STD_DEVERR_BOUNDS);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(id) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// ------------------------------- RMSNorm -----------------------------------
// One block per row, one thread per 8 consecutive elements (H % 8 == 0,
// H/8 <= 512): every input is loaded once into registers before any store.
// Sum of squares: per-thread sequential over its 8 values, xor tree inside
// each warp, then warps in order -- the same order for every row count.
STD_DEV float block_sum_ordered(float s, float* s_part) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = s;
  __syncthreads();
  float tot = 0.f;
  const int nw = (blockDim.x + 31) >> 5;
  for (int i = 0; i < nw; ++i) tot = __fadd_rn(tot, s_part[i]);
  return tot;
}

STD_DEV void load8(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

STD_DEV void store8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Row sources: 8 consecutive columns of one row as floats.  Bf16Rows reads a
// bf16 matrix; NoRows is the absent operand.  gemm.cu adds GemmOut (a GEMM's
// bf16 result assembled from its split-K partials), so a GEMM epilogue can be
// fused into the kernels below with the same arithmetic as the unfused pair.
struct NoRows {
  static constexpr bool kActive = false;
  STD_DEV void load8(size_t, int, float*) const {}
};
struct Bf16Rows {
  static constexpr bool kActive = true;
  const __nv_bfloat16* p;
  int ld;
  STD_DEV void load8(size_t row, int col, float* v) const { ::stdb::load8(p + row * ld + col, v); }
};

// y = bf16( w * bf16( x * rsqrt(mean(x^2) + eps) ) );  with an active delta,
// first x <- bf16(x + delta) (the residual add), written back in place.
// w == null: only the residual add (no norm, `out` untouched).
template <class Delta>
__global__ void __launch_bounds__(512) rmsnorm_kernel(__nv_bfloat16* __restrict__ x, const Delta delta,
                                                       const __nv_bfloat16* __restrict__ w, float eps, int H,
                                                       __nv_bfloat16* __restrict__ out) {
  __shared__ float s_part[32];
  pdl_launch_dependents();  // the following GEMM may start streaming its weights
  pdl_wait();
  const size_t row = blockIdx.x;
  const int c = threadIdx.x * 8;
  const bool act = c < H;
  float v[8], wv[8];
  if (act) {
    load8(x + row * H + c, v);
    if (w != nullptr) load8(w + c, wv);
    if (Delta::kActive) {
      float dv[8];
      delta.load8(row, c, dv);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = bf16_round(__fadd_rn(v[j], dv[j]));
      store8(x + row * H + c, v);
    }
  }
  if (w == nullptr) return;  // uniform across the block
  float s = 0.f;
  if (act) {
#pragma unroll
    for (int j = 0; j < 8; ++j) s = __fmaf_rn(v[j], v[j], s);
  }
  const float tot = block_sum_ordered(s, s_part);
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(H)), eps));
  if (act) {
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(wv[j], bf16_round(__fmul_rn(v[j], inv)));
    store8(out + row * H + c, y);
  }
}

// ------------------------------- RoPE + KV append --------------------------
// qkv rows (b, j): [Hq*D | Hkv*D | Hkv*D].  q -> q_out [b*n+j, Hq, D];
// k, v -> cache slot slot_base[b] + slot_off + j of [B, Hkv, cap, D].
// position = pos_base[b] + pos_off + j; cos/sin tables [max_pos, D/2] bf16.
// One block per token row; a thread owns 8 dims of the first half of one head
// and the matching 8 of the second half (rotate_half pairs d and d + D/2).
struct RopeParams {
  int n, Hq, Hkv, D, cap, max_pos;
  const int32_t* pos_base;
  int pos_off;
  const int32_t* slot_base;
  int slot_off;
  const __nv_bfloat16* cos_t;
  const __nv_bfloat16* sin_t;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
};

template <class Src>  // qkv rows [B*n, (Hq + 2 Hkv) * D]
__global__ void __launch_bounds__(512) rope_append_kernel(const Src qkv, const RopeParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int b = row / p.n, j = row % p.n;
  const int heads = p.Hq + 2 * p.Hkv;
  const int half = p.D / 2;
  const int per_head = half / 8;
  const int h = threadIdx.x / per_head, c = (threadIdx.x % per_head) * 8;
  int pos = p.pos_base[b] + p.pos_off + j;
  const int slot = p.slot_base[b] + p.slot_off + j;
  const bool slot_ok = slot >= 0 && slot < p.cap;
  if (pos < 0 || pos >= p.max_pos) {
    if (threadIdx.x == 0) std_set_error(STD_DEVERR_BOUNDS);
    pos = pos < 0 ? 0 : p.max_pos - 1;
  }
  if (!slot_ok && threadIdx.x == 0) std_set_error(STD_DEVERR_LENGTH);
  if (h >= heads) return;
  float lo[8], hi[8];
  qkv.load8(row, h * p.D + c, lo);
  qkv.load8(row, h * p.D + half + c, hi);
  __nv_bfloat16* dst;
  if (h < p.Hq) {
    dst = p.q_out + (static_cast<size_t>(row) * p.Hq + h) * p.D;
  } else if (h < p.Hq + p.Hkv) {
    if (!slot_ok) return;
    dst = p.k_cache + ((static_cast<size_t>(b) * p.Hkv + (h - p.Hq)) * p.cap + slot) * p.D;
  } else {
    if (!slot_ok) return;
    dst = p.v_cache + ((static_cast<size_t>(b) * p.Hkv + (h - p.Hq - p.Hkv)) * p.cap + slot) * p.D;
    store8(dst + c, lo);
    store8(dst + half + c, hi);
    return;
  }
  float cs[8], sn[8];
  load8(p.cos_t + static_cast<size_t>(pos) * half + c, cs);
  load8(p.sin_t + static_cast<size_t>(pos) * half + c, sn);
  float ylo[8], yhi[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    // q*cos + rotate_half(q)*sin, each product and the sum rounded to bf16
    ylo[k] = bf16_round(__fadd_rn(bf16_round(__fmul_rn(lo[k], cs[k])), bf16_round(__fmul_rn(-hi[k], sn[k]))));
    yhi[k] = bf16_round(__fadd_rn(bf16_round(__fmul_rn(hi[k], cs[k])), bf16_round(__fmul_rn(lo[k], sn[k]))));
  }
  store8(dst + c, ylo);
  store8(dst + half + c, yhi);
}

// ------------------------------- SiLU * up ---------------------------------
// out = bf16( bf16(silu(gate)) * up ), 8 features per thread.  gu rows hold
// 2I columns: [gate (I) | up (I)], or with `interleaved` 64-feature blocks
// [gate 64 | up 64] (the layout that lets the gate/up GEMM finish SiLU in its
// own epilogue: one 128-row weight tile = 64 gate + 64 up rows).
STD_DEV float silu_times(float g, float u) {
  const float sg = bf16_round(__fdiv_rn(g, __fadd_rn(1.0f, __expf(-g))));
  return __fmul_rn(sg, u);
}

template <class Src>
__global__ void silu_mul_kernel(const Src gu, int I, int interleaved, size_t total8, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int I8 = I / 8;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total8;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = idx / I8;
    const int c = static_cast<int>(idx % I8) * 8;
    const int gc = interleaved ? (c >> 6) * 128 + (c & 63) : c;
    const int uc = interleaved ? gc + 64 : I + c;
    float g[8], u[8], y[8];
    gu.load8(row, gc, g);
    gu.load8(row, uc, u);
#pragma unroll
    for (int k = 0; k < 8; ++k) y[k] = silu_times(g[k], u[k]);
    store8(out + row * I + c, y);
  }
}

__global__ void add_kernel(const __nv_bfloat16* a, const __nv_bfloat16* b, size_t n, __nv_bfloat16* out) {
  pdl_wait();
  pdl_launch_dependents();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(a[i]), __bfloat162float(b[i])));
}

// ------------------------------- argmax ------------------------------------
// out[row] = first index of the maximum of the row's V bf16 logits (V % 8 ==
// 0), read 8 columns at a time from a row source (a logits matrix, or a
// GEMM's split-K partials).  Written to out[(row / n) * out_stride +
// out_start + row % n].
// With margin_out, also the row's largest minus second-largest logit (equal
// maxima give 0), written at the same index.
template <class Src>
__global__ void __launch_bounds__(1024) argmax_kernel(const Src logits, int V, int n, int out_stride, int out_start,
                                                      int32_t* out, float* margin_out) {
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  float best = -INFINITY, second = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
    float v8[8];
    logits.load8(row, c, v8);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      second = fmaxf(second, fminf(best, v8[k]));
      if (v8[k] > best || (v8[k] == best && c + k < bi)) {
        best = v8[k];
        bi = c + k;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const float os = __shfl_xor_sync(0xffffffffu, second, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    second = fmaxf(fmaxf(second, os), fminf(best, ov));
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float s_v[32], s_s[32];
  __shared__ int s_i[32];
  if ((threadIdx.x & 31) == 0) {
    s_v[threadIdx.x >> 5] = best;
    s_s[threadIdx.x >> 5] = second;
    s_i[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) {
      second = fmaxf(fmaxf(second, s_s[w]), fminf(best, s_v[w]));
      if (s_v[w] > best || (s_v[w] == best && s_i[w] < bi)) {
        best = s_v[w];
        bi = s_i[w];
      }
    }
    if (bi == 0x7fffffff) bi = 0;
    const size_t o = static_cast<size_t>(row / n) * out_stride + out_start + row % n;
    out[o] = bi;
    if (margin_out != nullptr) margin_out[o] = best - second;
  }
}

// ------------------------------- (d) accept / commit -----------------------
// Per-request device state (int32, [B] unless noted):
//   ctx_len     prompt_len + generated tokens (logical position of the next token)
//   dense_len   rows kept in the dense cache
//   sparse_len  rows kept in the sparse cache (incl. the pending bonus's row)
//   n_gen       generated tokens;  done  0/1
//   tok         [B, tok_stride]: tok[0] = pending bonus, tok[1..gamma] = drafts
//   vpred       [B, vstride]: dense argmax of each verify row
//   dense_next  [B] the prefill's argmax (used when no bonus is pending)
//   out_tokens  [B, max_new];  stats [B, 4] = rounds, accepted, proposed, last accept
//   accept_hist [B, hist_cap] per-round accept lengths (may be null)
struct AcceptParams {
  int B, gamma, pending, tok_stride, vstride, max_new, eos, ignore_eos, hist_cap;
  const int32_t* vpred;
  const int32_t* dense_next;
  int32_t* tok;
  int32_t* ctx_len;
  int32_t* dense_len;
  int32_t* sparse_len;
  int32_t* n_gen;
  int32_t* done;
  int32_t* out_tokens;
  int32_t* stats;
  int32_t* accept_hist;
};

__global__ void accept_commit_kernel(const AcceptParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= p.B || p.done[b]) return;
  const int32_t* draft = p.tok + static_cast<size_t>(b) * p.tok_stride + 1;
  const int32_t* vp = p.vpred + static_cast<size_t>(b) * p.vstride;
  const int ng = p.n_gen[b];
  const int remaining = p.max_new - ng;
  const int propose = min(p.gamma, remaining);
  // dense prediction for draft i: verify row i (pending) or [dense_next, row 0, ...]
  int accept = 0;
  while (accept < propose) {
    const int pred = p.pending ? vp[accept] : (accept == 0 ? p.dense_next[b] : vp[accept - 1]);
    if (draft[accept] != pred) break;
    ++accept;
  }
  const int bonus = p.pending ? vp[accept] : (accept == 0 ? p.dense_next[b] : vp[accept - 1]);
  // full_append = draft[:accept] + [bonus], cut after the first EOS, then at remaining
  int n_app = 0;
  bool hit_eos = false;
  int32_t* outp = p.out_tokens + static_cast<size_t>(b) * p.max_new + ng;
  for (int i = 0; i <= accept && n_app < remaining; ++i) {
    const int tk = i < accept ? draft[i] : bonus;
    outp[n_app++] = tk;
    if (!p.ignore_eos && tk == p.eos) {
      hit_eos = true;
      break;
    }
  }
  const int32_t rounds = p.stats[b * 4 + 0];
  if (p.accept_hist != nullptr && rounds < p.hist_cap) p.accept_hist[static_cast<size_t>(b) * p.hist_cap + rounds] = accept;
  p.stats[b * 4 + 0] = rounds + 1;
  p.stats[b * 4 + 1] += accept;
  p.stats[b * 4 + 2] += propose;
  p.stats[b * 4 + 3] = accept;
  p.n_gen[b] = ng + n_app;
  p.ctx_len[b] += n_app;
  if (hit_eos || ng + n_app >= p.max_new) {
    p.done[b] = 1;
    return;
  }
  // rollback: keep pending + accepted rows in the dense cache, accepted drafts
  // plus the bonus (appended by the next sparse step) in the sparse cache
  p.dense_len[b] += p.pending + accept;
  p.sparse_len[b] += accept + 1;
  p.tok[static_cast<size_t>(b) * p.tok_stride] = bonus;
}

// ------------------------------- verification policy ---------------------
// The reference's checks on a parallel verify (std_qwen25vl.py:816-884,
// verification_policy.py:29-67), per request, before the round is committed:
//   * margin check (verify_margin_threshold): the smallest top-1 minus top-2
//     logit over the committed predictions i = 0..accept (verify row i with a
//     pending bonus, i - 1 without; rows outside the block are skipped); a
//     margin below the threshold is a "margin rerun" unless the fallback mode
//     is sequential_on_low_margin;
//   * math_on_full_accept: a full accept is re-verified (a fallback);
//   * verify_fallback: sequential_guard always, sequential_on_reject when a
//     draft was rejected, sequential_on_low_accept when additionally accept <=
//     max_accept, sequential_on_low_margin on a low margin (a fallback, and a
//     margin rerun too).
// Every re-verification here is the exact replay of the round's dense
// predictions (one token at a time); rerun[b] marks the requests that asked
// for it, and the round's graph runs the replay when any request did.
struct PolicyParams {
  int B, gamma, pending, tok_stride, vstride, max_new, mode, max_accept, math_on_full_accept, hist_cap;
  float threshold;  // NaN: no margin check
  const int32_t* tok;
  const int32_t* vpred;
  const int32_t* dense_next;
  const int32_t* n_gen;
  const int32_t* done;
  const int32_t* stats;   // [B, 4]; stats[b][0] = rounds committed so far (this round's index)
  const float* margins;   // [B, vstride]
  int32_t* rerun;         // [B]
  int32_t* first_accept;  // [B]
  int32_t* counters;      // [B, 3]: margin reruns, fallbacks, accepted extra
  float* margin_hist;     // [B, hist_cap]: the round's smallest margin (NaN: none)
  int32_t* any_rerun;     // [1]
  unsigned long long cond;
};

STD_DEV int accepted_prefix(const int32_t* draft, const int32_t* vp, int pending, int dnext, int propose) {
  int accept = 0;
  while (accept < propose) {
    const int pred = pending ? vp[accept] : (accept == 0 ? dnext : vp[accept - 1]);
    if (draft[accept] != pred) break;
    ++accept;
  }
  return accept;
}

enum PolicyMode : int { POL_NONE = 0, POL_ON_REJECT = 1, POL_ON_LOW_ACCEPT = 2, POL_ON_LOW_MARGIN = 3, POL_GUARD = 4 };

__global__ void verify_policy_kernel(const PolicyParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = threadIdx.x;
  int rr = 0;
  if (b < p.B && !p.done[b]) {
    const int32_t* draft = p.tok + static_cast<size_t>(b) * p.tok_stride + 1;
    const int32_t* vp = p.vpred + static_cast<size_t>(b) * p.vstride;
    const int propose = min(p.gamma, p.max_new - p.n_gen[b]);
    const int accept = accepted_prefix(draft, vp, p.pending, p.dense_next[b], propose);
    p.first_accept[b] = accept;
    int32_t* cnt = p.counters + static_cast<size_t>(b) * 3;
    bool low_margin = false;
    if (!isnan(p.threshold)) {
      float mmin = INFINITY;
      bool any = false;
      const int nq = p.gamma + p.pending;
      for (int i = 0; i <= accept; ++i) {
        const int row = p.pending ? i : i - 1;
        if (row < 0 || row >= nq) continue;
        mmin = fminf(mmin, p.margins[static_cast<size_t>(b) * p.vstride + row]);
        any = true;
      }
      const int r = p.stats[b * 4];
      if (r < p.hist_cap) p.margin_hist[static_cast<size_t>(b) * p.hist_cap + r] = any ? mmin : NAN;
      low_margin = any && mmin < p.threshold;
      if (low_margin && p.mode != POL_ON_LOW_MARGIN) {
        cnt[0] += 1;
        rr = 1;
      }
    }
    if (p.math_on_full_accept && accept == propose) {
      cnt[1] += 1;
      rr = 1;
    }
    const bool seq = p.mode == POL_GUARD || (p.mode == POL_ON_LOW_MARGIN && low_margin) ||
                     (p.mode == POL_ON_REJECT && accept < propose) ||
                     (p.mode == POL_ON_LOW_ACCEPT && accept < propose && accept <= p.max_accept);
    if (seq) {
      cnt[1] += 1;
      if (low_margin && p.mode == POL_ON_LOW_MARGIN) cnt[0] += 1;
      rr = 1;
    }
  }
  if (b < p.B) p.rerun[b] = rr;
  const int any = __syncthreads_or(rr);
  if (threadIdx.x == 0) {
    *p.any_rerun = any;
    if (p.cond != 0ull) cudaGraphSetConditional(static_cast<cudaGraphConditionalHandle>(p.cond), any ? 1u : 0u);
  }
}

// After a replay: accepted-extra bookkeeping from the replayed predictions.
__global__ void verify_policy_after_kernel(const PolicyParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = threadIdx.x;
  if (b >= p.B || p.done[b] || !p.rerun[b]) return;
  const int32_t* draft = p.tok + static_cast<size_t>(b) * p.tok_stride + 1;
  const int32_t* vp = p.vpred + static_cast<size_t>(b) * p.vstride;
  const int propose = min(p.gamma, p.max_new - p.n_gen[b]);
  const int accept = accepted_prefix(draft, vp, p.pending, p.dense_next[b], propose);
  if (accept > p.first_accept[b]) p.counters[static_cast<size_t>(b) * 3 + 2] += accept - p.first_accept[b];
}

// AR step bookkeeping (std_qwen25vl.py:584-590).  ar_commit records cur =
// tok[b][0] as generated (active[b] = request still running before this
// step); the step's forward then appends cur's KV at dense_len and writes its
// argmax into next_tok[b]; ar_advance moves dense_len on and makes next_tok
// the new cur, for requests that were active.  A finished request's state is
// frozen, so a batch can keep stepping until its last request finishes.
__global__ void ar_commit_kernel(int B, int tok_stride, int max_new, int eos, int ignore_eos, const int32_t* tok,
                                 int32_t* n_gen, int32_t* done, int32_t* out_tokens, int32_t* active) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (done[b]) {
    active[b] = 0;
    return;
  }
  active[b] = 1;
  const int ng = n_gen[b];
  const int t = tok[static_cast<size_t>(b) * tok_stride];
  out_tokens[static_cast<size_t>(b) * max_new + ng] = t;
  n_gen[b] = ng + 1;
  if ((!ignore_eos && t == eos) || ng + 1 >= max_new) done[b] = 1;
}

__global__ void ar_advance_kernel(int B, const int32_t* active, const int32_t* next_tok, int32_t* tok, int tok_stride,
                                  int32_t* dense_len, int32_t* ctx_len) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B || !active[b]) return;
  dense_len[b] += 1;
  ctx_len[b] += 1;
  tok[static_cast<size_t>(b) * tok_stride] = next_tok[b];
}

}  // namespace stdb

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" int std_embed(const void* table, int vocab, int H, const int32_t* tok, int tok_stride, int tok_start, int n,
                         int B, void* out, void* stream) {
  if (H % 8 != 0 || n <= 0 || B <= 0) return 1;
  return launch_pdl(stdb::embed_kernel, dim3(B * n), dim3(128), 0, static_cast<cudaStream_t>(stream),
                    static_cast<const __nv_bfloat16*>(table), vocab, H, tok, tok_stride, tok_start, n,
                    static_cast<__nv_bfloat16*>(out)) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_rmsnorm(const void* x, const void* w, float eps, int M, int H, void* out, void* stream) {
  if (M <= 0 || H <= 0) return 1;
  if (H % 8 != 0 || H / 8 > 512) return 1;
  const int nt = ((H / 8 + 31) / 32) * 32;
  if (w == nullptr) return 1;
  return launch_pdl(stdb::rmsnorm_kernel<stdb::NoRows>, dim3(M), dim3(nt), 0, static_cast<cudaStream_t>(stream),
                    const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(x)), stdb::NoRows{},
                    static_cast<const __nv_bfloat16*>(w), eps, H, static_cast<__nv_bfloat16*>(out)) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_add_rmsnorm(void* x, const void* delta, const void* w, float eps, int M, int H, void* out,
                               void* stream) {
  if (M <= 0 || H <= 0) return 1;
  if (H % 8 != 0 || H / 8 > 512 || delta == nullptr || w == nullptr) return 1;
  const int nt = ((H / 8 + 31) / 32) * 32;
  return launch_pdl(stdb::rmsnorm_kernel<stdb::Bf16Rows>, dim3(M), dim3(nt), 0, static_cast<cudaStream_t>(stream),
                    static_cast<__nv_bfloat16*>(x), stdb::Bf16Rows{static_cast<const __nv_bfloat16*>(delta), H},
                    static_cast<const __nv_bfloat16*>(w), eps, H, static_cast<__nv_bfloat16*>(out)) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_rope_append(const void* qkv, int B, int n, int Hq, int Hkv, int D, const int32_t* pos_base,
                               int pos_off, const int32_t* slot_base, int slot_off, const void* cos_t,
                               const void* sin_t, int max_pos, void* q_out, void* k_cache, void* v_cache, int cap,
                               void* stream) {
  if (B <= 0 || n <= 0 || D % 16 != 0 || cap <= 0 || (Hq + 2 * Hkv) * (D / 16) > 512) return 1;
  stdb::RopeParams p;
  p.n = n;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.D = D;
  p.cap = cap;
  p.max_pos = max_pos;
  p.pos_base = pos_base;
  p.pos_off = pos_off;
  p.slot_base = slot_base;
  p.slot_off = slot_off;
  p.cos_t = static_cast<const __nv_bfloat16*>(cos_t);
  p.sin_t = static_cast<const __nv_bfloat16*>(sin_t);
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  const int nt = (((Hq + 2 * Hkv) * (D / 16) + 31) / 32) * 32;
  const stdb::Bf16Rows src{static_cast<const __nv_bfloat16*>(qkv), (Hq + 2 * Hkv) * D};
  return launch_pdl(stdb::rope_append_kernel<stdb::Bf16Rows>, dim3(B * n), dim3(nt), 0,
                    static_cast<cudaStream_t>(stream), src, p) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_silu_mul(const void* gu, int M, int I, int interleaved, void* out, void* stream) {
  if (M <= 0 || I <= 0 || I % 8 != 0 || (interleaved && I % 64 != 0)) return 1;
  const size_t total8 = static_cast<size_t>(M) * I / 8;
  const int blocks = static_cast<int>((total8 + 255) / 256 < 148 * 8 ? (total8 + 255) / 256 : 148 * 8);
  return launch_pdl(stdb::silu_mul_kernel<stdb::Bf16Rows>, dim3(blocks), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), stdb::Bf16Rows{static_cast<const __nv_bfloat16*>(gu), 2 * I},
                    I, interleaved ? 1 : 0, total8, static_cast<__nv_bfloat16*>(out)) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_add(const void* a, const void* b, size_t n, void* out, void* stream) {
  const int blocks = static_cast<int>((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  return launch_pdl(stdb::add_kernel, dim3(blocks > 0 ? blocks : 1), dim3(256), 0, static_cast<cudaStream_t>(stream),
                    static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b), n,
                    static_cast<__nv_bfloat16*>(out)) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_argmax_rows(const void* logits, int rows, int V, int n, int out_stride, int out_start, int32_t* out,
                               void* stream) {
  if (rows <= 0 || V <= 0 || n <= 0) return 1;
  if (V % 8 != 0) return 1;
  return launch_pdl(stdb::argmax_kernel<stdb::Bf16Rows>, dim3(rows), dim3(1024), 0, static_cast<cudaStream_t>(stream),
                    stdb::Bf16Rows{static_cast<const __nv_bfloat16*>(logits), V}, V, n, out_stride, out_start, out,
                    static_cast<float*>(nullptr)) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_accept_commit(int B, int gamma, int pending, int32_t* tok, int tok_stride, const int32_t* vpred,
                                 int vstride, const int32_t* dense_next, int max_new, int eos, int ignore_eos,
                                 int32_t* ctx_len, int32_t* dense_len, int32_t* sparse_len, int32_t* n_gen,
                                 int32_t* done, int32_t* out_tokens, int32_t* stats, int32_t* accept_hist,
                                 int hist_cap, void* stream) {
  if (B <= 0 || gamma <= 0 || tok_stride < gamma + 1 || vstride < gamma + pending) return 1;
  stdb::AcceptParams p;
  p.B = B;
  p.gamma = gamma;
  p.pending = pending;
  p.tok_stride = tok_stride;
  p.vstride = vstride;
  p.max_new = max_new;
  p.eos = eos;
  p.ignore_eos = ignore_eos;
  p.hist_cap = hist_cap;
  p.vpred = vpred;
  p.dense_next = dense_next;
  p.tok = tok;
  p.ctx_len = ctx_len;
  p.dense_len = dense_len;
  p.sparse_len = sparse_len;
  p.n_gen = n_gen;
  p.done = done;
  p.out_tokens = out_tokens;
  p.stats = stats;
  p.accept_hist = accept_hist;
  return launch_pdl(stdb::accept_commit_kernel, dim3((B + 127) / 128), dim3(128), 0,
                    static_cast<cudaStream_t>(stream), p) == cudaSuccess
             ? 0
             : 4;
}

static stdb::PolicyParams policy_params(int B, int gamma, int pending, const int32_t* tok, int tok_stride,
                                        const int32_t* vpred, int vstride, const int32_t* dense_next, int max_new,
                                        const int32_t* n_gen, const int32_t* done, const int32_t* stats,
                                        const float* margins, float threshold, int mode, int max_accept,
                                        int math_on_full_accept, int32_t* rerun, int32_t* first_accept,
                                        int32_t* counters, float* margin_hist, int hist_cap, int32_t* any_rerun,
                                        unsigned long long cond) {
  stdb::PolicyParams p;
  p.B = B;
  p.gamma = gamma;
  p.pending = pending;
  p.tok_stride = tok_stride;
  p.vstride = vstride;
  p.max_new = max_new;
  p.mode = mode;
  p.max_accept = max_accept;
  p.math_on_full_accept = math_on_full_accept;
  p.hist_cap = hist_cap;
  p.threshold = threshold;
  p.tok = tok;
  p.vpred = vpred;
  p.dense_next = dense_next;
  p.n_gen = n_gen;
  p.done = done;
  p.stats = stats;
  p.margins = margins;
  p.rerun = rerun;
  p.first_accept = first_accept;
  p.counters = counters;
  p.margin_hist = margin_hist;
  p.any_rerun = any_rerun;
  p.cond = cond;
  return p;
}

extern "C" int std_verify_policy(int B, int gamma, int pending, const int32_t* tok, int tok_stride, const int32_t* vpred,
                                 int vstride, const int32_t* dense_next, int max_new, const int32_t* n_gen,
                                 const int32_t* done, const int32_t* stats, const float* margins, float threshold,
                                 int mode, int max_accept, int math_on_full_accept, int32_t* rerun,
                                 int32_t* first_accept, int32_t* counters, float* margin_hist, int hist_cap,
                                 int32_t* any_rerun, unsigned long long cond, int after, void* stream) {
  if (B <= 0 || B > 1024 || gamma < 1 || (pending != 0 && pending != 1) || vstride < gamma + pending) return 1;
  if (mode < stdb::POL_NONE || mode > stdb::POL_GUARD || max_new <= 0 || hist_cap <= 0) return 1;
  if (tok == nullptr || vpred == nullptr || dense_next == nullptr || n_gen == nullptr || done == nullptr ||
      stats == nullptr || rerun == nullptr || first_accept == nullptr || counters == nullptr || any_rerun == nullptr)
    return 1;
  if (!isnan(threshold) && (margins == nullptr || margin_hist == nullptr)) return 1;
  const stdb::PolicyParams p =
      policy_params(B, gamma, pending, tok, tok_stride, vpred, vstride, dense_next, max_new, n_gen, done, stats,
                    margins, threshold, mode, max_accept, math_on_full_accept, rerun, first_accept, counters,
                    margin_hist, hist_cap, any_rerun, cond);
  const int threads = ((B + 31) / 32) * 32;
  return launch_pdl(after ? stdb::verify_policy_after_kernel : stdb::verify_policy_kernel, dim3(1), dim3(threads), 0,
                    static_cast<cudaStream_t>(stream), p) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_ar_commit(int B, int tok_stride, int max_new, int eos, int ignore_eos, const int32_t* tok,
                             int32_t* n_gen, int32_t* done, int32_t* out_tokens, int32_t* active, void* stream) {
  if (B <= 0 || tok_stride <= 0 || max_new <= 0) return 1;
  return launch_pdl(stdb::ar_commit_kernel, dim3((B + 127) / 128), dim3(128), 0, static_cast<cudaStream_t>(stream),
                    B, tok_stride, max_new, eos, ignore_eos, tok, n_gen, done, out_tokens, active) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_ar_advance(int B, const int32_t* active, const int32_t* next_tok, int32_t* tok, int tok_stride,
                              int32_t* dense_len, int32_t* ctx_len, void* stream) {
  if (B <= 0 || tok_stride <= 0) return 1;
  return launch_pdl(stdb::ar_advance_kernel, dim3((B + 127) / 128), dim3(128), 0, static_cast<cudaStream_t>(stream),
                    B, active, next_tok, tok, tok_stride, dense_len, ctx_len) == cudaSuccess
             ? 0
             : 4;
}
