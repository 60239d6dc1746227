// gemm.cu -- weight-streaming skinny GEMM on tcgen05 for the decode forwards.
//
//   Y[M, N] = X[M, K] . W[N, K]^T (+ bias[N]),  bf16 in, fp32 accumulate, bf16 out
//
// Replaces the cuBLAS calls behind the decoder's nn.Linear layers during decode
// (modeling_qwen2_5_vl.py: q/k/v/o projections :778-781, Qwen2MLP :674-687,
// lm_head :1749) for M <= 256 tokens, where the op streams the weights once
// and is HBM-bound (a 7B forward reads 14.1 GB of weights).
//
// The weights are the MMA's M=128 operand (128 output features per CTA) and
// the tokens its N operand (padded to a multiple of 16), so the tensor-core
// work scales with the token count, not with a 128-row tile.  A TMA warp
// streams 128x64 weight tiles and nmma x 64 token tiles (128-B swizzle)
// through a ring of 2..8 stages (as many as fit two CTAs per SM); one thread issues tcgen05.mma (M128, N=nmma,
// K16) into a TMEM accumulator; then all four warps drain TMEM (one output
// feature per thread, tokens along the columns) with coalesced bf16 stores.
// K is split into `splits` contiguous ranges chosen from (N, K) alone; split
// partials (fp32) are summed by gemm_reduce_kernel in split order.
//
// Row invariance: a token's output depends only on its own X row, the weights,
// the (N, K)-fixed split and the MMA N (the padded token count) -- not on the
// other rows -- so callers that keep the padded count fixed (the dense decode
// forwards) get bit-identical rows for AR steps and verify blocks.
#include "common.cuh"

namespace stdb {

constexpr int GM_BM = 128;         // output features per CTA (MMA M)
constexpr int GM_BK = 64;          // K per stage (one 128-B swizzle row)
constexpr int GM_MAX_STAGES = 8;
constexpr uint32_t GM_SMEM_BUDGET = 104 * 1024;  // per CTA: two CTAs per SM
constexpr int GM_THREADS = 128;
constexpr uint32_t GM_WTILE = GM_BM * GM_BK * 2;  // 16 KB
constexpr int GM_SUM_BATCH = 8;                    // split partials loaded per batch by the epilogues

struct GemmParams {
  int M, N, K, nmma, splits, kblocks, stages;
  const __nv_bfloat16* bias;  // [N] or null
  __nv_bfloat16* y;           // [M, N]
  float* partial;             // [splits, M, N] (splits > 1)
  // fused greedy argmax (splits == 1): instead of storing y, fold each row's
  // bf16 values into amax_keys[t] (rows t < amax_rows) with atomicMax on
  // (order_key(value) << 32 | ~column): the maximum, first column on ties
  unsigned long long* amax_keys;
  int amax_rows;
  // with amax_keys: also the two largest values of each row within each warp's
  // 32 columns, amax_top2[(tile * 4 + warp) * M + t] (verify margins)
  float2* amax_top2;
  // fused SiLU * up (splits == 1; weights in 64-row [gate | up] blocks): tile
  // rows 0..63 are gate, 64..127 up of features 64*tile ..; writes
  // act[t][64*tile + r] = bf16(bf16(silu(gate)) * up) instead of y
  __nv_bfloat16* act;
};

// (a1, a2) <- the two largest of the (a1, a2) pairs of the warp's lanes
// (a2 <= a1 in every pair; equal maxima give a2 == a1).
STD_DEV void top2_merge(float& a1, float& a2, float b1, float b2) {
  const float hi = fmaxf(a1, b1), lo = fminf(a1, b1);
  a2 = fmaxf(lo, fmaxf(a2, b2));
  a1 = hi;
}
STD_DEV void top2_warp(float& a1, float& a2) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float b1 = __shfl_xor_sync(0xffffffffu, a1, o), b2 = __shfl_xor_sync(0xffffffffu, a2, o);
    top2_merge(a1, a2, b1, b2);
  }
}

__global__ void __launch_bounds__(GM_THREADS)
    gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                const GemmParams p) {
  const int tile = blockIdx.x, split = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kb0 = static_cast<int>((static_cast<long>(split) * p.kblocks) / p.splits);
  const int kb1 = static_cast<int>((static_cast<long>(split + 1) * p.kblocks) / p.splits);
  const int nkb = kb1 - kb0;
  const int n0 = tile * GM_BM;
  const uint32_t xtile = static_cast<uint32_t>(p.nmma) * GM_BK * 2;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint8_t* sW = smem;                 // [S][16 KB]
  uint8_t* sX = smem + S * GM_WTILE;  // [S][xtile]
  __shared__ __align__(8) uint64_t bar_full[GM_MAX_STAGES], bar_empty[GM_MAX_STAGES], bar_done;
  __shared__ uint32_t s_tmem;

  uint32_t ncols = 32;
  while (ncols < static_cast<uint32_t>(p.nmma)) ncols <<= 1;
  if (warp == 1) {
    tmem_alloc(&s_tmem, ncols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_empty[i], 1);
    }
    mbar_init(&bar_done, 1);
    fence_barrier_init();
    prefetch_tensormap(&tmW);
    prefetch_tensormap(&tmX);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  // Every kernel that follows a GEMM reads its inputs after its own wait (or,
  // a GEMM, only weights before it): let it be scheduled now, so it is
  // resident when this one completes.  After the TMEM allocation, so a
  // successor can never hold columns this CTA still needs.
  pdl_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    // The weights do not depend on the previous kernel: the first stages'
    // weight tiles are requested before waiting for it (programmatic
    // dependent launch), the token tiles only after.
    const uint64_t stream_policy = l2_policy_evict_first();  // each weight byte is read once per step
    const int pre = nkb < S ? nkb : S;
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&bar_full[i], GM_WTILE + xtile);
      tma_load_2d_hint(sW + i * GM_WTILE, &tmW, &bar_full[i], (kb0 + i) * GM_BK, n0, stream_policy);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i) tma_load_2d(sX + i * xtile, &tmX, &bar_full[i], (kb0 + i) * GM_BK, 0);
    int issued = pre;
    for (int i = pre; i < nkb; ++i) {
      const int st = i % S;
      if (!mbar_wait(&bar_empty[st], ((i / S) - 1) & 1)) break;
      mbar_arrive_expect_tx(&bar_full[st], GM_WTILE + xtile);
      const int kx = (kb0 + i) * GM_BK;
      tma_load_2d_hint(sW + st * GM_WTILE, &tmW, &bar_full[st], kx, n0, stream_policy);
      tma_load_2d(sX + st * xtile, &tmX, &bar_full[st], kx, 0);
      issued = i + 1;
    }
    for (int i = issued - S < 0 ? 0 : issued - S; i < issued; ++i) mbar_wait(&bar_full[i % S], (i / S) & 1);
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    const uint32_t idesc = idesc_bf16_f32(GM_BM, p.nmma, 0, 0);
    for (int i = 0; i < nkb; ++i) {
      const int st = i % S;
      if (!mbar_wait(&bar_full[st], (i / S) & 1)) break;
      tc_fence_after();
      const uint32_t aW = smem_u32(sW + st * GM_WTILE), aX = smem_u32(sX + st * xtile);
#pragma unroll
      for (int ks = 0; ks < GM_BK / 16; ++ks)
        umma_bf16(tmem, sdesc_sw128(aW + ks * 32u, 16, 1024), sdesc_sw128(aX + ks * 32u, 16, 1024), idesc,
                  (i > 0 || ks > 0) ? 1u : 0u);
      umma_commit(&bar_empty[st]);
    }
    umma_commit(&bar_done);
  }

  // ---- epilogue: thread = output feature, columns = tokens ----
  mbar_wait(&bar_done, 0);
  pdl_wait();  // every thread: the previous kernel is complete before any store
  __syncwarp();
  tc_fence_after();
  const int f = n0 + warp * 32 + lane;
  const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const float bias = (p.splits == 1 && p.bias != nullptr && f < p.N) ? __bfloat162float(p.bias[f]) : 0.f;
  // ncols is a power of two >= max(nmma, 32), so 32-column loads stay inside it
  for (int t0 = 0; p.amax_keys != nullptr && t0 < p.nmma; t0 += 32) {
    uint32_t v[32];
    tmem_ld32(trow + t0, v);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int t = t0 + j;
      unsigned long long key = 0ull;
      if (t < p.amax_rows && f < p.N)
        key = (static_cast<unsigned long long>(order_key(bf16_round(__uint_as_float(v[j]) + bias))) << 32) |
              (0xFFFFFFFFu - static_cast<uint32_t>(f));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if (lane == 0 && key != 0ull) atomicMax(&p.amax_keys[t], key);
      if (p.amax_top2 != nullptr && t < p.amax_rows) {
        float a1 = f < p.N ? bf16_round(__uint_as_float(v[j]) + bias) : -INFINITY, a2 = -INFINITY;
        top2_warp(a1, a2);
        if (lane == 0) p.amax_top2[static_cast<size_t>(tile * 4 + warp) * p.M + t] = make_float2(a1, a2);
      }
    }
  }
  if (p.act != nullptr) {
    // the stage buffers are free (every MMA retired): up rows go through smem
    // [token][64] so that the gate rows' threads can pair them
    __nv_bfloat16* s_up = reinterpret_cast<__nv_bfloat16*>(smem);
    const int r = warp * 32 + lane;
    if (warp >= 2) {
      for (int t0 = 0; t0 < p.nmma; t0 += 32) {
        uint32_t v[32];
        tmem_ld32(trow + t0, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) s_up[(t0 + j) * 64 + (r - 64)] = __float2bfloat16_rn(__uint_as_float(v[j]));
      }
    }
    __syncthreads();
    if (warp < 2) {
      const int I = p.N / 2;
      const int feat = tile * 64 + r;
      for (int t0 = 0; t0 < p.nmma; t0 += 32) {
        uint32_t v[32];
        tmem_ld32(trow + t0, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int t = t0 + j;
          if (t >= p.M) continue;
          const float g = bf16_round(__uint_as_float(v[j]));
          const float u = __bfloat162float(s_up[t * 64 + r]);
          p.act[static_cast<size_t>(t) * I + feat] = __float2bfloat16_rn(silu_times(g, u));
        }
      }
    }
  }
  for (int t0 = 0; p.amax_keys == nullptr && p.act == nullptr && t0 < p.nmma; t0 += 32) {
    uint32_t v[32];
    tmem_ld32(trow + t0, v);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int t = t0 + j;
      if (t >= p.M || f >= p.N) continue;
      const float acc = __uint_as_float(v[j]);
      if (p.splits == 1)
        p.y[static_cast<size_t>(t) * p.N + f] = __float2bfloat16_rn(acc + bias);
      else
        p.partial[(static_cast<size_t>(split) * p.M + t) * p.N + f] = acc;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

// y[t, f] = bf16( sum_s partial[s, t, f] + bias[f] ), splits in order
__global__ void gemm_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N,
                                   const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ y) {
  pdl_launch_dependents();  // followed by RoPE + append or a norm: both read after their wait
  pdl_wait();
  const size_t total = static_cast<size_t>(M) * N / 4;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < splits; s0 += GM_SUM_BATCH) {  // batched loads, adds in split order
      float4 b[GM_SUM_BATCH];
#pragma unroll
      for (int j = 0; j < GM_SUM_BATCH; ++j)
        if (s0 + j < splits) b[j] = reinterpret_cast<const float4*>(partial + static_cast<size_t>(s0 + j) * M * N)[i];
#pragma unroll
      for (int j = 0; j < GM_SUM_BATCH; ++j) {
        if (s0 + j == 0) {
          a = b[0];
        } else if (s0 + j < splits) {
          a.x += b[j].x;
          a.y += b[j].y;
          a.z += b[j].z;
          a.w += b[j].w;
        }
      }
    }
    const int f = static_cast<int>((i * 4) % N);
    if (bias != nullptr) {
      a.x += __bfloat162float(bias[f]);
      a.y += __bfloat162float(bias[f + 1]);
      a.z += __bfloat162float(bias[f + 2]);
      a.w += __bfloat162float(bias[f + 3]);
    }
    uint2 u;
    u.x = pack_bf16x2(a.x, a.y);
    u.y = pack_bf16x2(a.z, a.w);
    reinterpret_cast<uint2*>(y)[i] = u;
  }
}

// The GEMM's bf16 result read 8 columns at a time by a fused epilogue (the
// rmsnorm and rope_append kernels of decode_ops.cu): split partials summed in
// split order, + bias, rounded to bf16 -- the same operations, in the same
// order, as gemm_reduce_kernel -- or, when K was not split, the GEMM's own
// bf16 output (bias already applied).
struct GemmOut {
  static constexpr bool kActive = true;
  const float* partial;        // [splits, M, N]  (splits > 1)
  const __nv_bfloat16* y;      // [M, N]          (splits == 1)
  const __nv_bfloat16* bias;   // [N] or null     (splits > 1)
  int splits, M, N;
  STD_DEV void load8(size_t row, int col, float* v) const {
    if (splits <= 1) {
      ::stdb::load8(y + row * N + col, v);
      return;
    }
    const size_t off = row * N + col;
    const size_t MN = static_cast<size_t>(M) * N;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    // the splits in batches of GM_SUM_BATCH: every load of a batch is issued
    // before the first add (one L2 latency per batch), then the adds run in
    // split order, so the sum is the same as a one-at-a-time loop
    for (int s0 = 0; s0 < splits; s0 += GM_SUM_BATCH) {
      float4 c[GM_SUM_BATCH], d[GM_SUM_BATCH];
#pragma unroll
      for (int j = 0; j < GM_SUM_BATCH; ++j) {
        if (s0 + j < splits) {
          const float* ps = partial + static_cast<size_t>(s0 + j) * MN + off;
          c[j] = __ldcg(reinterpret_cast<const float4*>(ps));
          d[j] = __ldcg(reinterpret_cast<const float4*>(ps + 4));
        }
      }
#pragma unroll
      for (int j = 0; j < GM_SUM_BATCH; ++j) {
        if (s0 + j == 0) {
          a = c[0];
          b = d[0];
        } else if (s0 + j < splits) {
          a.x += c[j].x;
          a.y += c[j].y;
          a.z += c[j].z;
          a.w += c[j].w;
          b.x += d[j].x;
          b.y += d[j].y;
          b.z += d[j].z;
          b.w += d[j].w;
        }
      }
    }
    float t[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (bias != nullptr) {
#pragma unroll
      for (int j = 0; j < 8; ++j) t[j] += __bfloat162float(bias[col + j]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = bf16_round(t[j]);
  }
};

// out[(t / n) * out_stride + out_start + t % n] = column of amax_keys[t]; the
// keys are cleared for the next call.
__global__ void argmax_keys_kernel(unsigned long long* keys, int rows, int n, int out_stride, int out_start,
                                   int32_t* out) {
  pdl_launch_dependents();  // followed by the embedding, the accept or the AR bookkeeping: read after their wait
  pdl_wait();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= rows) return;
  const unsigned long long k = keys[t];
  out[(t / n) * out_stride + out_start + t % n] =
      k == 0ull ? 0 : static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
  keys[t] = 0ull;
}

// As argmax_keys_kernel, plus each row's top-1 minus top-2 logit from the
// per-warp pairs in top2 [nsub, M] (one block per row):
// margin_out[(t / n) * out_stride + out_start + t % n].
__global__ void __launch_bounds__(256) argmax_margin_kernel(unsigned long long* keys, const float2* top2, int nsub,
                                                            int M, int n, int out_stride, int out_start, int32_t* out,
                                                            float* margin_out) {
  __shared__ float2 s_w[8];
  pdl_launch_dependents();  // followed by the accept or the AR bookkeeping: read after their wait
  pdl_wait();
  const int t = blockIdx.x;
  float a1 = -INFINITY, a2 = -INFINITY;
  for (int i = threadIdx.x; i < nsub; i += blockDim.x) {
    const float2 v = top2[static_cast<size_t>(i) * M + t];
    top2_merge(a1, a2, v.x, v.y);
  }
  top2_warp(a1, a2);
  if ((threadIdx.x & 31) == 0) s_w[threadIdx.x >> 5] = make_float2(a1, a2);
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) top2_merge(a1, a2, s_w[w].x, s_w[w].y);
    const unsigned long long k = keys[t];
    const size_t o = static_cast<size_t>(t / n) * out_stride + out_start + t % n;
    out[o] = k == 0ull ? 0 : static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
    margin_out[o] = a1 - a2;
    keys[t] = 0ull;
  }
}

}  // namespace stdb

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
// K splits from (N, K) only: fill whole waves of two resident CTAs per SM.
static int gemm_splits(int N, int K) {
  const long tiles = (N + stdb::GM_BM - 1) / stdb::GM_BM;
  const long kblocks = K / stdb::GM_BK;
  const long slots = 2L * 148;
  if (tiles >= slots / 2) return 1;  // enough tiles to stream the weights without splitting K
  long best = 1;
  double best_eff = -1.0;
  for (long s = 1; s <= kblocks / 2 && s <= 16; ++s) {
    const long ctas = tiles * s;
    const double eff = static_cast<double>(ctas) / (static_cast<double>((ctas + slots - 1) / slots) * slots);
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = s;
    }
  }
  return static_cast<int>(best);
}

static int gemm_nmma(int M) { return ((M + 15) / 16) * 16; }

extern "C" size_t std_gemm_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int s = gemm_splits(N, K);
  return s > 1 ? static_cast<size_t>(s) * M * N * 4 : 0;
}

// Launch gemm_kernel: with splits > 1 it writes fp32 partials to `partial`,
// otherwise bf16 y (+ bias).  Shapes are checked by the callers.
// Per-CTA shared-memory budget for the stage ring (the ring depth follows
// from it).  A smaller budget leaves room on each SM for the next kernel's
// CTAs, which then start streaming their weights before this one ends.
static std::atomic<uint32_t> g_gemm_smem_budget{stdb::GM_SMEM_BUDGET};

extern "C" int std_gemm_set_smem_budget(int bytes) {
  if (bytes < 40 * 1024 || bytes > 200 * 1024) return 1;
  g_gemm_smem_budget.store(static_cast<uint32_t>(bytes));
  return 0;
}

static int gemm_launch(const void* x, const void* w, const void* bias, void* y, float* partial, int M, int N, int K,
                       int splits, cudaStream_t s, unsigned long long* amax_keys = nullptr, int amax_rows = 0,
                       void* act = nullptr, void* amax_top2 = nullptr) {
  const int nmma = gemm_nmma(M);
  const uint32_t stage_bytes = stdb::GM_WTILE + static_cast<uint32_t>(nmma) * stdb::GM_BK * 2;
  int stages = static_cast<int>(g_gemm_smem_budget.load() / stage_bytes);
  stages = stages < 2 ? 2 : (stages > stdb::GM_MAX_STAGES ? stdb::GM_MAX_STAGES : stages);
  const size_t smem = static_cast<size_t>(stages) * stage_bytes + 1024;
  static SmemGrant grant;
  if (ensure_smem(stdb::gemm_kernel, grant, smem) != 0) return 3;
  CUtensorMap tw, tx;
  int rc = make_tmap_bf16_2d(&tw, w, static_cast<uint64_t>(N), static_cast<uint64_t>(K),
                             static_cast<uint64_t>(K) * 2, stdb::GM_BK, stdb::GM_BM);
  if (rc == 0)
    rc = make_tmap_bf16_2d(&tx, x, static_cast<uint64_t>(M), static_cast<uint64_t>(K), static_cast<uint64_t>(K) * 2,
                           stdb::GM_BK, static_cast<uint32_t>(nmma));
  if (rc != 0) return rc;
  stdb::GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.nmma = nmma;
  p.splits = splits;
  p.kblocks = K / stdb::GM_BK;
  p.stages = stages;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.partial = partial;
  p.amax_keys = amax_keys;
  p.amax_rows = amax_rows;
  p.act = static_cast<__nv_bfloat16*>(act);
  p.amax_top2 = static_cast<float2*>(amax_top2);
  // may begin while the previous kernel in the stream finishes: the weight
  // tiles of the first stages are requested before griddepcontrol.wait
  return launch_pdl(stdb::gemm_kernel, dim3((N + stdb::GM_BM - 1) / stdb::GM_BM, splits), dim3(stdb::GM_THREADS),
                    smem, s, tw, tx, p) == cudaSuccess
             ? 0
             : 4;
}

static bool gemm_shape_ok(const void* x, const void* w, int M, int N, int K, int n_align) {
  if (M <= 0 || M > 256 || N <= 0 || K <= 0 || K % stdb::GM_BK != 0 || N % n_align != 0) return false;
  if (x == nullptr || w == nullptr) return false;
  return ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) == 0;
}

extern "C" int std_gemm_bf16(const void* x, const void* w, const void* bias, void* y, int M, int N, int K,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (!gemm_shape_ok(x, w, M, N, K, 4) || y == nullptr) return 1;
  const int splits = gemm_splits(N, K);
  const size_t need = std_gemm_workspace_bytes(M, N, K);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need)) return 5;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = gemm_launch(x, w, bias, y, static_cast<float*>(workspace), M, N, K, splits, s);
  if (rc != 0 || splits == 1) return rc;
  const size_t total4 = static_cast<size_t>(M) * N / 4;
  const int blocks = static_cast<int>((total4 + 255) / 256 < 1184 ? (total4 + 255) / 256 : 1184);
  return launch_pdl(stdb::gemm_reduce_kernel, dim3(blocks), dim3(256), 0, s,
                    static_cast<const float*>(workspace), splits, M, N, static_cast<const __nv_bfloat16*>(bias),
                    static_cast<__nv_bfloat16*>(y)) == cudaSuccess
             ? 0
             : 4;
}

// Fused GEMM epilogues: the GEMM's output goes straight into the next decode
// op, through workspace (split partials, or the bf16 output when K is not split).
extern "C" size_t std_gemm_epilogue_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const size_t part = std_gemm_workspace_bytes(M, N, K);
  const size_t ybytes = static_cast<size_t>(M) * N * 2;
  // the argmax's margins: per-warp top-2 pairs [N/128 * 4, M] of float2
  const size_t top2 = static_cast<size_t>((N + stdb::GM_BM - 1) / stdb::GM_BM) * 4 * M * 8;
  size_t b = part > ybytes ? part : ybytes;
  b = b > top2 ? b : top2;
  return ((b + 255) / 256) * 256;
}

// The K split count of a GEMM on an [N, K] weight matrix.
extern "C" int std_gemm_plan(int N, int K, int* splits_out) {
  if (N <= 0 || K <= 0 || K % stdb::GM_BK != 0 || splits_out == nullptr) return 1;
  *splits_out = gemm_splits(N, K);
  return 0;
}

static stdb::GemmOut gemm_out_view(void* workspace, const void* bias, int splits, int M, int N) {
  stdb::GemmOut o;
  o.partial = splits > 1 ? static_cast<const float*>(workspace) : nullptr;
  o.y = splits > 1 ? nullptr : static_cast<const __nv_bfloat16*>(workspace);
  o.bias = splits > 1 ? static_cast<const __nv_bfloat16*>(bias) : nullptr;
  o.splits = splits;
  o.M = M;
  o.N = N;
  return o;
}

extern "C" int std_gemm_add_rmsnorm(const void* x, const void* w, const void* bias, void* resid, const void* norm_w,
                                    float eps, void* out, int M, int N, int K, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (!gemm_shape_ok(x, w, M, N, K, 8) || resid == nullptr || N / 8 > 512) return 1;
  if (norm_w != nullptr && out == nullptr) return 1;
  if (workspace == nullptr || workspace_bytes < std_gemm_epilogue_workspace_bytes(M, N, K)) return 5;
  const int splits = gemm_splits(N, K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = gemm_launch(x, w, bias, workspace, static_cast<float*>(workspace), M, N, K, splits, s);
  if (rc != 0) return rc;
  const int nt = ((N / 8 + 31) / 32) * 32;
  return launch_pdl(stdb::rmsnorm_kernel<stdb::GemmOut>, dim3(M), dim3(nt), 0, s, static_cast<__nv_bfloat16*>(resid),
                    gemm_out_view(workspace, bias, splits, M, N), static_cast<const __nv_bfloat16*>(norm_w), eps, N,
                    static_cast<__nv_bfloat16*>(out)) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_gemm_rope_append(const void* x, const void* w, const void* bias, int K, int B, int n, int Hq,
                                    int Hkv, int D, const int32_t* pos_base, int pos_off, const int32_t* slot_base,
                                    int slot_off, const void* cos_t, const void* sin_t, int max_pos, void* q_out,
                                    void* k_cache, void* v_cache, int cap, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  const int M = B * n, N = (Hq + 2 * Hkv) * D;
  if (B <= 0 || n <= 0 || D % 16 != 0 || cap <= 0 || (Hq + 2 * Hkv) * (D / 16) > 512) return 1;
  if (!gemm_shape_ok(x, w, M, N, K, 8)) return 1;
  if (workspace == nullptr || workspace_bytes < std_gemm_epilogue_workspace_bytes(M, N, K)) return 5;
  const int splits = gemm_splits(N, K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = gemm_launch(x, w, bias, workspace, static_cast<float*>(workspace), M, N, K, splits, s);
  if (rc != 0) return rc;
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
  return launch_pdl(stdb::rope_append_kernel<stdb::GemmOut>, dim3(M), dim3(nt), 0, s,
                    gemm_out_view(workspace, bias, splits, M, N), p) == cudaSuccess
             ? 0
             : 4;
}

// lm_head + greedy argmax: the argmax of each of the first `rows_out` rows of
// x . w^T (bf16 logits, first index on ties) without storing the logits.
extern "C" int std_gemm_argmax(const void* x, const void* w, int M, int N, int K, int rows_out, int n, int out_stride,
                               int out_start, int32_t* out, float* margin_out, unsigned long long* keys,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (!gemm_shape_ok(x, w, M, N, K, 8) || out == nullptr || keys == nullptr) return 1;
  if (rows_out <= 0 || rows_out > M || n <= 0) return 1;
  const int splits = gemm_splits(N, K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (splits == 1) {
    if (margin_out != nullptr) {  // per-warp top-2 pairs in the workspace, then one block per row
      if (workspace == nullptr || workspace_bytes < std_gemm_epilogue_workspace_bytes(M, N, K)) return 5;
      int rc = gemm_launch(x, w, nullptr, nullptr, nullptr, M, N, K, 1, s, keys, rows_out, nullptr, workspace);
      if (rc != 0) return rc;
      return launch_pdl(stdb::argmax_margin_kernel, dim3(rows_out), dim3(256), 0, s, keys,
                        static_cast<const float2*>(workspace), ((N + stdb::GM_BM - 1) / stdb::GM_BM) * 4, M, n,
                        out_stride, out_start, out, margin_out) == cudaSuccess
                 ? 0
                 : 4;
    }
    int rc = gemm_launch(x, w, nullptr, nullptr, nullptr, M, N, K, 1, s, keys, rows_out);
    if (rc != 0) return rc;
    return launch_pdl(stdb::argmax_keys_kernel, dim3((rows_out + 127) / 128), dim3(128), 0, s, keys, rows_out, n,
                      out_stride, out_start, out) == cudaSuccess
               ? 0
               : 4;
  }
  if (workspace == nullptr || workspace_bytes < std_gemm_epilogue_workspace_bytes(M, N, K)) return 5;
  int rc = gemm_launch(x, w, nullptr, workspace, static_cast<float*>(workspace), M, N, K, splits, s);
  if (rc != 0) return rc;
  return launch_pdl(stdb::argmax_kernel<stdb::GemmOut>, dim3(rows_out), dim3(1024), 0, s,
                    gemm_out_view(workspace, nullptr, splits, M, N), N, n, out_stride, out_start, out,
                    margin_out) == cudaSuccess
             ? 0
             : 4;
}

// Qwen2MLP's act_fn(gate_proj(x)) * up_proj(x) in one pass over the fused
// gate/up weights w [2I, K] stored as 64-row [gate | up] blocks.
extern "C" int std_gemm_silu_mul(const void* x, const void* w, int M, int I, int K, void* act, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  const int N = 2 * I;
  if (!gemm_shape_ok(x, w, M, N, K, 8) || act == nullptr || I % 64 != 0) return 1;
  const int splits = gemm_splits(N, K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (splits == 1) return gemm_launch(x, w, nullptr, nullptr, nullptr, M, N, K, 1, s, nullptr, 0, act);
  if (workspace == nullptr || workspace_bytes < std_gemm_epilogue_workspace_bytes(M, N, K)) return 5;
  int rc = gemm_launch(x, w, nullptr, workspace, static_cast<float*>(workspace), M, N, K, splits, s);
  if (rc != 0) return rc;
  const size_t total8 = static_cast<size_t>(M) * I / 8;
  const int blocks = static_cast<int>((total8 + 255) / 256 < 148 * 8 ? (total8 + 255) / 256 : 148 * 8);
  return launch_pdl(stdb::silu_mul_kernel<stdb::GemmOut>, dim3(blocks), dim3(256), 0, s,
                    gemm_out_view(workspace, nullptr, splits, M, N), I, 1, total8,
                    static_cast<__nv_bfloat16*>(act)) == cudaSuccess
             ? 0
             : 4;
}
