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
// y = bf16( w * bf16( x * rsqrt(mean(x^2) + eps) ) ), per-thread strided sums
// then a fixed xor tree: the same order for every row count.
template <int NT>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(const __nv_bfloat16* x, const __nv_bfloat16* w, float eps, int H,
                                                     __nv_bfloat16* out) {
  const size_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  __shared__ float s_part[NT / 32];
  float s = 0.f;
  for (int i = threadIdx.x; i < H; i += NT) {
    const float v = __bfloat162float(xr[i]);
    s = __fmaf_rn(v, v, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = s;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) tot = __fadd_rn(tot, s_part[i]);
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(H)), eps));
  for (int i = threadIdx.x; i < H; i += NT) {
    const float v = bf16_round(__fmul_rn(__bfloat162float(xr[i]), inv));
    out[row * H + i] = __float2bfloat16_rn(__fmul_rn(__bfloat162float(w[i]), v));
  }
}

// ------------------------------- RoPE + KV append --------------------------
// qkv rows (b, j): [Hq*D | Hkv*D | Hkv*D].  q -> q_out [b*n+j, Hq, D];
// k, v -> cache slot slot_base[b] + slot_off + j of [B, Hkv, cap, D].
// position = pos_base[b] + pos_off + j; cos/sin tables [max_pos, D/2] bf16.
struct RopeParams {
  const __nv_bfloat16* qkv;
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

__global__ void rope_append_kernel(const RopeParams p) {
  const int row = blockIdx.x;
  const int b = row / p.n, j = row % p.n;
  const int heads = p.Hq + 2 * p.Hkv;
  const int half = p.D / 2;
  int pos = p.pos_base[b] + p.pos_off + j;
  int slot = p.slot_base[b] + p.slot_off + j;
  const bool slot_ok = slot >= 0 && slot < p.cap;
  if (pos < 0 || pos >= p.max_pos) {
    if (threadIdx.x == 0) std_set_error(STD_DEVERR_BOUNDS);
    pos = pos < 0 ? 0 : p.max_pos - 1;
  }
  if (!slot_ok && threadIdx.x == 0) std_set_error(STD_DEVERR_LENGTH);
  const __nv_bfloat16* src = p.qkv + static_cast<size_t>(row) * heads * p.D;
  const __nv_bfloat16* cr = p.cos_t + static_cast<size_t>(pos) * half;
  const __nv_bfloat16* sr = p.sin_t + static_cast<size_t>(pos) * half;
  for (int idx = threadIdx.x; idx < heads * p.D; idx += blockDim.x) {
    const int h = idx / p.D, d = idx % p.D;
    const float x = __bfloat162float(src[idx]);
    if (h < p.Hq + p.Hkv) {
      const float c = __bfloat162float(cr[d % half]);
      const float s = __bfloat162float(sr[d % half]);
      const float partner = __bfloat162float(src[h * p.D + (d < half ? d + half : d - half)]);
      const float rot = d < half ? -partner : partner;
      const float y = bf16_round(__fadd_rn(bf16_round(__fmul_rn(x, c)), bf16_round(__fmul_rn(rot, s))));
      if (h < p.Hq) {
        p.q_out[(static_cast<size_t>(row) * p.Hq + h) * p.D + d] = __float2bfloat16_rn(y);
      } else if (slot_ok) {
        const int kh = h - p.Hq;
        p.k_cache[((static_cast<size_t>(b) * p.Hkv + kh) * p.cap + slot) * p.D + d] = __float2bfloat16_rn(y);
      }
    } else if (slot_ok) {
      const int vh = h - p.Hq - p.Hkv;
      p.v_cache[((static_cast<size_t>(b) * p.Hkv + vh) * p.cap + slot) * p.D + d] = src[idx];
    }
  }
}

// ------------------------------- SiLU * up ---------------------------------
// gu rows: [gate (I) | up (I)]; out = bf16( bf16(silu(gate)) * up )
__global__ void silu_mul_kernel(const __nv_bfloat16* gu, int I, size_t total, __nv_bfloat16* out) {
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = idx / I, c = idx % I;
    const float g = __bfloat162float(gu[row * 2 * I + c]);
    const float u = __bfloat162float(gu[row * 2 * I + I + c]);
    const float sg = bf16_round(__fdiv_rn(g, __fadd_rn(1.0f, __expf(-g))));
    out[idx] = __float2bfloat16_rn(__fmul_rn(sg, u));
  }
}

__global__ void add_kernel(const __nv_bfloat16* a, const __nv_bfloat16* b, size_t n, __nv_bfloat16* out) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(a[i]), __bfloat162float(b[i])));
}

// ------------------------------- argmax ------------------------------------
// out[row] = first index of the maximum of logits[row, :V] (bf16).  Written to
// out[(row / n) * out_stride + out_start + row % n].
__global__ void __launch_bounds__(1024) argmax_kernel(const __nv_bfloat16* logits, int V, int n, int out_stride,
                                                      int out_start, int32_t* out) {
  const int row = blockIdx.x;
  const __nv_bfloat16* lr = logits + static_cast<size_t>(row) * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = __bfloat162float(lr[i]);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float s_v[32];
  __shared__ int s_i[32];
  if ((threadIdx.x & 31) == 0) {
    s_v[threadIdx.x >> 5] = best;
    s_i[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) {
      if (s_v[w] > best || (s_v[w] == best && s_i[w] < bi)) {
        best = s_v[w];
        bi = s_i[w];
      }
    }
    if (bi == 0x7fffffff) bi = 0;
    out[(row / n) * out_stride + out_start + row % n] = bi;
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

// AR step bookkeeping (std_qwen25vl.py:584-590).  ar_commit records cur =
// tok[b][0] as generated (active[b] = request still running before this
// step); the step's forward then appends cur's KV at dense_len and writes its
// argmax into next_tok[b]; ar_advance moves dense_len on and makes next_tok
// the new cur, for requests that were active.  A finished request's state is
// frozen, so a batch can keep stepping until its last request finishes.
__global__ void ar_commit_kernel(int B, int tok_stride, int max_new, int eos, int ignore_eos, const int32_t* tok,
                                 int32_t* n_gen, int32_t* done, int32_t* out_tokens, int32_t* active) {
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
  stdb::embed_kernel<<<B * n, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(table), vocab, H, tok, tok_stride, tok_start, n,
      static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int std_rmsnorm(const void* x, const void* w, float eps, int M, int H, void* out, void* stream) {
  if (M <= 0 || H <= 0) return 1;
  stdb::rmsnorm_kernel<256><<<M, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), eps, H,
      static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int std_rope_append(const void* qkv, int B, int n, int Hq, int Hkv, int D, const int32_t* pos_base,
                               int pos_off, const int32_t* slot_base, int slot_off, const void* cos_t,
                               const void* sin_t, int max_pos, void* q_out, void* k_cache, void* v_cache, int cap,
                               void* stream) {
  if (B <= 0 || n <= 0 || D % 2 != 0 || cap <= 0) return 1;
  stdb::RopeParams p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
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
  stdb::rope_append_kernel<<<B * n, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int std_silu_mul(const void* gu, int M, int I, void* out, void* stream) {
  if (M <= 0 || I <= 0) return 1;
  const size_t total = static_cast<size_t>(M) * I;
  const int blocks = static_cast<int>((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
  stdb::silu_mul_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gu), I, total, static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int std_add(const void* a, const void* b, size_t n, void* out, void* stream) {
  const int blocks = static_cast<int>((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  stdb::add_kernel<<<blocks > 0 ? blocks : 1, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b), n, static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int std_argmax_rows(const void* logits, int rows, int V, int n, int out_stride, int out_start, int32_t* out,
                               void* stream) {
  if (rows <= 0 || V <= 0 || n <= 0) return 1;
  stdb::argmax_kernel<<<rows, 1024, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const __nv_bfloat16*>(logits),
                                                                            V, n, out_stride, out_start, out);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
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
  stdb::accept_commit_kernel<<<(B + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int std_ar_commit(int B, int tok_stride, int max_new, int eos, int ignore_eos, const int32_t* tok,
                             int32_t* n_gen, int32_t* done, int32_t* out_tokens, int32_t* active, void* stream) {
  if (B <= 0 || tok_stride <= 0 || max_new <= 0) return 1;
  stdb::ar_commit_kernel<<<(B + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      B, tok_stride, max_new, eos, ignore_eos, tok, n_gen, done, out_tokens, active);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int std_ar_advance(int B, const int32_t* active, const int32_t* next_tok, int32_t* tok, int tok_stride,
                              int32_t* dense_len, int32_t* ctx_len, void* stream) {
  if (B <= 0 || tok_stride <= 0) return 1;
  stdb::ar_advance_kernel<<<(B + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(B, active, next_tok, tok,
                                                                                          tok_stride, dense_len,
                                                                                          ctx_len);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
