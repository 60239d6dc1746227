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
#include <map>
#include <tuple>

#include "common.cuh"

namespace stdb {

constexpr int GM_BM = 128;         // output features per CTA (MMA M)
constexpr int GM_BK = 64;          // K per stage (one 128-B swizzle row)
constexpr int GM_MAX_STAGES = 8;
constexpr uint32_t GM_SMEM_BUDGET = 104 * 1024;  // default per-CTA stage budget: two CTAs per SM
constexpr int GM_THREADS = 128;
constexpr uint32_t GM_WTILE = GM_BM * GM_BK * 2;  // 16 KB

// In-kernel epilogues that need the full K sum of a 128-feature tile.  With K
// split over several CTAs, each CTA stores its fp32 partial and counts itself
// in on the tile's arrival counter; the last CTA to arrive sums the partials
// in split order (the order gemm_reduce_kernel uses) and applies the epilogue
// for the whole tile.  No CTA waits for another.
enum GemmFixup : int {
  FIX_NONE = 0,
  FIX_ROPE = 1,   // QKV projection: bias, RoPE of q/k heads, q -> q_out, k/v -> the cache slot (one head per tile)
  FIX_RESID = 2,  // O / down projection: resid += y (bf16), and the tile's per-row sum of squares of the new resid
};

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
  // RMSNorm prologue (norm_w != null): X is a residual stream and each staged
  // X tile becomes bf16(norm_w[k] * bf16(x * inv[t])) before the MMA reads it,
  // inv[t] = rsqrt(sum_i norm_sumsq[i * M + t] / K + eps), i < K / 128 (the
  // per-tile sums of squares written by the producer of x)
  const float* norm_sumsq;
  const __nv_bfloat16* norm_w;
  float norm_eps;
  // split-K fixup (fixup != FIX_NONE; the splits of a tile form one cluster)
  int fixup;
  RopeParams rope;  // FIX_ROPE: rows t < rope_rows are real tokens (t = b * rope.n + j)
  int rope_rows;
  __nv_bfloat16* resid;  // FIX_RESID: [M, N]
  float* sumsq_out;      // FIX_RESID: [N / 128, M]
  // dependents are released only after this grid's own wait (a following
  // kernel that reads before its wait then sees every earlier kernel done)
  int late_trigger;
};

// Sum of 128 per-thread values (one per thread of a 128-thread block, warp w
// holding values 32w..32w+31): xor tree inside each warp, then the four warp
// sums in order.  The fixed order makes a tile's sum of squares identical
// wherever it is computed (GEMM fixup, embedding).
STD_DEV float tile_sum128(float v, float* s_part4, int slot) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) s_part4[slot * 4 + (threadIdx.x >> 5)] = v;
  return v;
}
STD_DEV float tile_sum128_finish(const float* s_part4, int slot) {
  return __fadd_rn(__fadd_rn(__fadd_rn(s_part4[slot * 4 + 0], s_part4[slot * 4 + 1]), s_part4[slot * 4 + 2]),
                   s_part4[slot * 4 + 3]);
}

// RMSNorm of staged X rows in place: the 128B-swizzled [rows][64] bf16 tile at
// `tile` holds columns k0..k0+63 (indices into w) of rows 0..nrows-1; rows >=
// M are left as loaded (zero fill).  Threads t, t + nthr, ... share the work.
STD_DEV void norm_x_tile(uint8_t* tile, int nrows, int M, int k0, const float* s_inv, const __nv_bfloat16* w,
                         int t, int nthr) {
  for (int i = t; i < nrows * 8; i += nthr) {
    const int r = i >> 3, pc = i & 7;
    if (r >= M) continue;
    const int c = pc ^ (r & 7);  // logical 16-byte chunk: columns k0 + 8c .. +7
    uint4* q = reinterpret_cast<uint4*>(tile + r * 128 + pc * 16);
    float v[8], wv[8], y[8];
    const uint4 u = *q;
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
    load8(w + k0 + 8 * c, wv);
    const float inv = s_inv[r];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(wv[j], bf16_round(__fmul_rn(v[j], inv)));
    uint4 o;
    o.x = pack_bf16x2(y[0], y[1]);
    o.y = pack_bf16x2(y[2], y[3]);
    o.z = pack_bf16x2(y[4], y[5]);
    o.w = pack_bf16x2(y[6], y[7]);
    *q = o;
  }
}

// Apply a split-K fixup epilogue to the tile's bf16 results y[t] (t < M) of
// feature f = n0 + thread.  `yv(t)` returns them; s_y (>= 32 x 128 bf16) and
// s_part (>= 4 x 32 floats) are free shared memory.
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

// ---- split-K fixup (FIX_ROPE / FIX_RESID) ----------------------------------
// The fixup of a tile runs on the tokens t = t_first + i * t_step (this
// cluster rank's share), FX_TB tokens at a time.  Every global and
// distributed-shared-memory read of a batch is issued before any of its
// results is used, so a batch costs about one memory latency, not one per
// token and split.
constexpr int FX_TB = 8;
constexpr int FX_MAX_SPLITS = 8;

// y[j] = bf16(sum over splits, in split order, of the tile's fp32 partial for
// token tt[j] and this thread's feature, + fb), j < n.  s_acc: this CTA's
// stage [M][128]; with splits > 1 the partials are read from every cluster
// rank's stage at the same offset (my_acc = this thread's column of s_acc).
STD_DEV void fixup_sums(const GemmParams& p, const float* s_acc, uint32_t my_acc, float fb, const int (&tt)[FX_TB],
                        int n, float (&y)[FX_TB]) {
  float v[FX_MAX_SPLITS][FX_TB];
  if (p.splits == 1) {
#pragma unroll
    for (int j = 0; j < FX_TB; ++j) v[0][j] = j < n ? s_acc[tt[j] * GM_BM + threadIdx.x] : 0.f;
  } else {
#pragma unroll
    for (int s2 = 0; s2 < FX_MAX_SPLITS; ++s2)
#pragma unroll
      for (int j = 0; j < FX_TB; ++j)
        v[s2][j] = (s2 < p.splits && j < n)
                       ? ld_dsmem_f32(mapa_rank(my_acc + static_cast<uint32_t>(tt[j]) * GM_BM * 4u, s2))
                       : 0.f;
  }
#pragma unroll
  for (int j = 0; j < FX_TB; ++j) {
    float a = v[0][j];
#pragma unroll
    for (int s2 = 1; s2 < FX_MAX_SPLITS; ++s2)
      if (s2 < p.splits) a += v[s2][j];
    y[j] = bf16_round(a + fb);
  }
}

// s_y: >= FX_TB x 128 bf16 of free shared memory; s_part: >= 4 x FX_TB floats;
// s_tok: >= 4 x FX_TB ints.
STD_DEV void gemm_fixup(const GemmParams& p, int tile, int n0, const float* s_acc, uint32_t my_acc, float fb,
                        __nv_bfloat16* s_y, float* s_part, int* s_tok, int t_first, int t_step) {
  const int tid = threadIdx.x;
  const int f = n0 + tid;
  const int rows = p.fixup == FIX_RESID ? p.M : p.rope_rows;
  const int mine = t_first < rows ? (rows - t_first + t_step - 1) / t_step : 0;
  if (p.fixup == FIX_RESID) {
    for (int i0 = 0; i0 < mine; i0 += FX_TB) {
      const int nt = mine - i0 < FX_TB ? mine - i0 : FX_TB;
      int tt[FX_TB];
      float xo[FX_TB], y[FX_TB];
#pragma unroll
      for (int j = 0; j < FX_TB; ++j) {
        tt[j] = t_first + (i0 + (j < nt ? j : 0)) * t_step;
        xo[j] = (j < nt && f < p.N) ? __bfloat162float(p.resid[static_cast<size_t>(tt[j]) * p.N + f]) : 0.f;
      }
      fixup_sums(p, s_acc, my_acc, fb, tt, nt, y);
#pragma unroll
      for (int j = 0; j < FX_TB; ++j) {
        if (j >= nt) break;
        float xn = 0.f;
        if (f < p.N) {
          xn = bf16_round(__fadd_rn(xo[j], y[j]));
          p.resid[static_cast<size_t>(tt[j]) * p.N + f] = __float2bfloat16_rn(xn);
        }
        tile_sum128(__fmul_rn(xn, xn), s_part, j);
      }
      __syncthreads();
      if (tid < nt) p.sumsq_out[static_cast<size_t>(tile) * p.M + t_first + (i0 + tid) * t_step] =
          tile_sum128_finish(s_part, tid);
      __syncthreads();
    }
    return;
  }
  // FIX_ROPE: one head per tile (D == 128); thread = dim d; rotate_half pairs d and d +- 64
  const RopeParams& r = p.rope;
  const int heads = r.Hq + 2 * r.Hkv;
  if (tile >= heads) return;
  const int d = tid, half = 64, c = d & 63;
  const bool is_q = tile < r.Hq, is_v = tile >= r.Hq + r.Hkv;
  int* s_pos = s_tok;
  int* s_slot = s_tok + FX_TB;
  int* s_b = s_tok + 2 * FX_TB;
  for (int i0 = 0; i0 < mine; i0 += FX_TB) {
    const int nt = mine - i0 < FX_TB ? mine - i0 : FX_TB;
    int tt[FX_TB];
    float y[FX_TB];
#pragma unroll
    for (int j = 0; j < FX_TB; ++j) tt[j] = t_first + (i0 + (j < nt ? j : 0)) * t_step;
    fixup_sums(p, s_acc, my_acc, fb, tt, nt, y);
#pragma unroll
    for (int j = 0; j < FX_TB; ++j)
      if (j < nt) s_y[j * 128 + d] = __float2bfloat16_rn(y[j]);
    if (d < nt) {  // the batch's positions and cache slots
      const int row = t_first + (i0 + d) * t_step;
      const int b = row / r.n, jj = row % r.n;
      int pos = r.pos_base[b] + r.pos_off + jj;
      const int slot = r.slot_base[b] + r.slot_off + jj;
      if (pos < 0 || pos >= r.max_pos) {
        std_set_error(STD_DEVERR_BOUNDS);
        pos = pos < 0 ? 0 : r.max_pos - 1;
      }
      const bool slot_ok = slot >= 0 && slot < r.cap;
      if (!slot_ok && !is_q) std_set_error(STD_DEVERR_LENGTH);
      s_pos[d] = pos;
      s_slot[d] = slot_ok ? slot : -1;
      s_b[d] = b;
    }
    __syncthreads();
    float cs[FX_TB], sn[FX_TB];
#pragma unroll
    for (int j = 0; j < FX_TB; ++j) {
      cs[j] = (j < nt && !is_v) ? __bfloat162float(r.cos_t[static_cast<size_t>(s_pos[j]) * half + c]) : 0.f;
      sn[j] = (j < nt && !is_v) ? __bfloat162float(r.sin_t[static_cast<size_t>(s_pos[j]) * half + c]) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < FX_TB; ++j) {
      if (j >= nt) break;
      const float lo = __bfloat162float(s_y[j * 128 + c]);
      const float hi = __bfloat162float(s_y[j * 128 + half + c]);
      __nv_bfloat16* dst;
      if (is_q) {
        dst = r.q_out + (static_cast<size_t>(tt[j]) * r.Hq + tile) * 128;
      } else {
        if (s_slot[j] < 0) continue;
        const int hk = is_v ? tile - r.Hq - r.Hkv : tile - r.Hq;
        dst = (is_v ? r.v_cache : r.k_cache) +
              ((static_cast<size_t>(s_b[j]) * r.Hkv + hk) * r.cap + s_slot[j]) * 128;
      }
      float out;
      if (is_v) {
        out = d < half ? lo : hi;  // v: no rotation
      } else {
        // q*cos + rotate_half(q)*sin, each product and the sum rounded to bf16
        out = d < half ? bf16_round(__fadd_rn(bf16_round(__fmul_rn(lo, cs[j])), bf16_round(__fmul_rn(-hi, sn[j]))))
                       : bf16_round(__fadd_rn(bf16_round(__fmul_rn(hi, cs[j])), bf16_round(__fmul_rn(lo, sn[j]))));
      }
      dst[d] = __float2bfloat16_rn(out);
    }
    __syncthreads();
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
  const bool norm = p.norm_w != nullptr;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint8_t* sW = smem;                 // [S][16 KB]
  uint8_t* sX = smem + S * GM_WTILE;  // [S][xtile]
  // norm prologue: the CTA's K range of the norm weight ([kmax] bf16, kmax =
  // the largest split's K range), then the sums of squares [K/128][M] fp32
  __nv_bfloat16* s_normw = reinterpret_cast<__nv_bfloat16*>(sX + S * xtile);
  float* s_ssq = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s_normw) +
                                          ((p.kblocks + p.splits - 1) / p.splits) * GM_BK * 2);
  __shared__ __align__(8) uint64_t bar_full[GM_MAX_STAGES], bar_empty[GM_MAX_STAGES], bar_xready[GM_MAX_STAGES],
      bar_done;
  __shared__ uint32_t s_tmem;
  __shared__ float s_inv[256];
  __shared__ float s_part[4 * 32];
  __shared__ int s_tok[4 * FX_TB];
  __shared__ int s_norm_ok[2][2];

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
      mbar_init(&bar_xready[i], 1);
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
  // successor can never hold columns this CTA still needs.  With late_trigger
  // the release waits for this grid's own predecessors (below).
  if (!p.late_trigger) pdl_launch_dependents();

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
    if (p.late_trigger) pdl_launch_dependents();
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
      if (!mbar_wait(norm ? &bar_xready[st] : &bar_full[st], (i / S) & 1)) break;
      tc_fence_after();
      const uint32_t aW = smem_u32(sW + st * GM_WTILE), aX = smem_u32(sX + st * xtile);
#pragma unroll
      for (int ks = 0; ks < GM_BK / 16; ++ks)
        umma_bf16(tmem, sdesc_sw128(aW + ks * 32u, 16, 1024), sdesc_sw128(aX + ks * 32u, 16, 1024), idesc,
                  (i > 0 || ks > 0) ? 1u : 0u);
      umma_commit(&bar_empty[st]);
    }
    umma_commit(&bar_done);
  } else if (norm && warp >= 2) {
    // ---- RMSNorm of the staged X tiles (warps 2-3) ----
    const int t = tid - 64;
    // Global reads here are batched (eight or sixteen independent loads per
    // thread before their stores): one memory latency per batch instead of
    // one per element.
    // this CTA's columns of the norm weight (constant: before the wait)
    const int nw16 = nkb * 8;
    const uint4* wsrc = reinterpret_cast<const uint4*>(p.norm_w + kb0 * GM_BK);
    for (int base = 0; base < nw16; base += 64 * 8) {
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = base + j * 64 + t;
        if (i < nw16) v[j] = wsrc[i];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = base + j * 64 + t;
        if (i < nw16) reinterpret_cast<uint4*>(s_normw)[i] = v[j];
      }
    }
    pdl_wait();
    if (p.late_trigger) pdl_launch_dependents();
    // per-tile sums of squares [K/128, M] -> shared; then each row adds its
    // tiles in order
    const int ntiles_in = p.K / GM_BM;
    const int nss = ntiles_in * p.M;
    for (int base = 0; base < nss; base += 64 * 16) {
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int i = base + j * 64 + t;
        v[j] = i < nss ? __ldcg(&p.norm_sumsq[i]) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int i = base + j * 64 + t;
        if (i < nss) s_ssq[i] = v[j];
      }
    }
    named_bar_sync(1, 64);
    for (int r = t; r < p.nmma; r += 64) {
      float inv = 0.f;
      if (r < p.M) {
        float ss = 0.f;
        for (int i = 0; i < ntiles_in; ++i) ss = __fadd_rn(ss, s_ssq[i * p.M + r]);
        inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(p.K)), p.norm_eps));
      }
      s_inv[r] = inv;
    }
    named_bar_sync(1, 64);
    for (int i = 0; i < nkb; ++i) {
      const int st = i % S;
      // a timed-out wait must end the loop in both warps together (the named
      // barrier counts 64 threads): vote per warp, then read both votes after
      // the barrier (double-buffered, so a warp that runs ahead never
      // overwrites a vote the other warp has yet to read)
      const bool ok_w = __all_sync(0xffffffffu, mbar_wait(&bar_full[st], (i / S) & 1));
      if (ok_w) norm_x_tile(sX + st * xtile, p.nmma, p.M, i * GM_BK, s_inv, s_normw, t, 64);
      fence_async_smem();
      if (lane == 0) s_norm_ok[i & 1][warp - 2] = ok_w ? 1 : 0;
      named_bar_sync(1, 64);
      if (t == 0) mbar_arrive(&bar_xready[st]);
      if (!(s_norm_ok[i & 1][0] && s_norm_ok[i & 1][1])) break;
    }
  }

  // ---- epilogue: thread = output feature, columns = tokens ----
  mbar_wait(&bar_done, 0);
  pdl_wait();  // every thread: the previous kernel is complete before any store
  if (p.late_trigger) pdl_launch_dependents();
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
  const bool fused = p.fixup != FIX_NONE;
  for (int t0 = 0; p.amax_keys == nullptr && p.act == nullptr && !fused && t0 < p.nmma; t0 += 32) {
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
  if (fused) {
    // The K splits of this tile are one thread-block cluster (rank = split).
    // Each CTA stages its fp32 accumulator [M][128] in its shared memory;
    // rank r then reduces tokens r, r + splits, ... by reading every rank's
    // stage in split order over distributed shared memory (the order
    // gemm_reduce_kernel adds global partials in) and applies the fixup.
    float* s_acc = reinterpret_cast<float*>(smem);
    for (int t0 = 0; t0 < p.nmma; t0 += 32) {
      uint32_t v[32];
      tmem_ld32(trow + t0, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (t0 + j < p.M) s_acc[(t0 + j) * GM_BM + tid] = __uint_as_float(v[j]);
    }
    if (p.splits > 1) {
      cluster_arrive_release();
      cluster_wait_acquire();
    } else {
      __syncthreads();
    }
    const float fb = (p.bias != nullptr && f < p.N) ? __bfloat162float(p.bias[f]) : 0.f;
    const uint32_t my_acc = smem_u32(s_acc) + static_cast<uint32_t>(tid) * 4u;
    gemm_fixup(p, tile, n0, s_acc, my_acc, fb,
               reinterpret_cast<__nv_bfloat16*>(smem + static_cast<size_t>(p.M) * GM_BM * 4), s_part, s_tok, split,
               p.splits);
    if (p.splits > 1) {  // no CTA leaves while another may still read its stage
      cluster_arrive_release();
      cluster_wait_acquire();
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

// Embedding rows for a decode forward, with each 128-column tile's sum of
// squares per row (sumsq [H/128, ld]) for the RMSNorm prologue of the first
// projection: out[b*n + j] = table[tok[b*tok_stride + tok_start + j]].
__global__ void __launch_bounds__(128) embed_sumsq_kernel(const __nv_bfloat16* table, int vocab, int H,
                                                          const int32_t* tok, int tok_stride, int tok_start, int n,
                                                          __nv_bfloat16* out, float* sumsq, int ld) {
  __shared__ float s_part[4];
  pdl_launch_dependents();  // followed by a GEMM, which reads this only after its own wait
  pdl_wait();
  const int row = blockIdx.x;
  const int b = row / n, j = row % n;
  int id = tok[b * tok_stride + tok_start + j];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) std_set_error(STD_DEVERR_BOUNDS);
    id = 0;
  }
  const __nv_bfloat16* src = table + static_cast<size_t>(id) * H;
  __nv_bfloat16* dst = out + static_cast<size_t>(row) * H;
  for (int t = 0; t < H / GM_BM; ++t) {
    const int c = t * GM_BM + threadIdx.x;
    const __nv_bfloat16 v = src[c];
    dst[c] = v;
    const float x = __bfloat162float(v);
    tile_sum128(__fmul_rn(x, x), s_part, 0);
    __syncthreads();
    if (threadIdx.x == 0) sumsq[static_cast<size_t>(t) * ld + row] = tile_sum128_finish(s_part, 0);
    __syncthreads();
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
    float4 a = reinterpret_cast<const float4*>(partial)[i];
    for (int s = 1; s < splits; ++s) {
      const float4 b = reinterpret_cast<const float4*>(partial + static_cast<size_t>(s) * M * N)[i];
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
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
    float4 a = __ldcg(reinterpret_cast<const float4*>(partial + off));
    float4 b = __ldcg(reinterpret_cast<const float4*>(partial + off + 4));
    for (int s = 1; s < splits; ++s) {
      const float* ps = partial + static_cast<size_t>(s) * M * N + off;
      const float4 c = __ldcg(reinterpret_cast<const float4*>(ps));
      const float4 d = __ldcg(reinterpret_cast<const float4*>(ps + 4));
      a.x += c.x;
      a.y += c.y;
      a.z += c.z;
      a.w += c.w;
      b.x += d.x;
      b.y += d.y;
      b.z += d.z;
      b.w += d.w;
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
  pdl_launch_dependents();
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

// How many clusters of `cluster` gemm_kernel CTAs (with `smem` bytes of
// dynamic shared memory) the current device runs at once; 0 when unknown.
// Clusters are placed within one GPC, so this can be well below
// (SMs x CTAs per SM) / cluster.  Cached per (device, cluster, smem).
static int gemm_active_clusters(int cluster, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, cluster, smem);
  std::lock_guard<std::mutex> lock(mu);
  const auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  static SmemGrant grant;
  int n = 0;
  if (ensure_smem(stdb::gemm_kernel, grant, smem) == 0) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = cluster;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, cluster);
    cfg.blockDim = dim3(stdb::GM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, stdb::gemm_kernel, &cfg) != cudaSuccess) n = 0;
    cudaGetLastError();
  }
  cache[key] = n;
  return n;
}

// Splits of a GEMM whose split-K sum is reduced inside one cluster (at most
// 8, the portable cluster size): the largest count whose clusters -- one per
// 128-feature tile -- all run in one wave; with none, the count of fewest
// waves.  Depends on (N, K) and the device only, so every call on a weight
// matrix (an AR step, a verify block) splits K the same way.
static int gemm_splits_cluster(int N, int K) {
  const int tiles = (N + stdb::GM_BM - 1) / stdb::GM_BM;
  const int kblocks = K / stdb::GM_BK;
  int s_max = gemm_splits(N, K);
  if (s_max > 8) s_max = 8;
  if (s_max <= 1) return 1;
  // shared memory of a two-CTA-per-SM launch (the ring budget; the norm
  // prologue's extra rows are a few KB within the same 2-per-SM bound)
  const size_t smem = static_cast<size_t>(stdb::GM_SMEM_BUDGET) + 1024;
  int best = s_max, best_waves = 1 << 30;
  for (int s = s_max; s >= 2; --s) {
    if (kblocks / s < 2) continue;
    const int active = gemm_active_clusters(s, smem);
    if (active <= 0) return s_max;  // occupancy unknown: keep the wave heuristic
    const int waves = (tiles + active - 1) / active;
    if (waves == 1) return s;
    if (waves < best_waves) {
      best_waves = waves;
      best = s;
    }
  }
  return best;
}

extern "C" size_t std_gemm_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int s = gemm_splits(N, K);
  return s > 1 ? static_cast<size_t>(s) * M * N * 4 : 0;
}

// Launch gemm_kernel: with splits > 1 it writes fp32 partials to `partial`,
// otherwise bf16 y (+ bias).  Shapes are checked by the callers.
// Fields of an in-kernel epilogue / prologue (norm, fixup) for gemm_launch.
struct GemmExtra {
  const float* norm_sumsq = nullptr;
  const void* norm_w = nullptr;
  float norm_eps = 0.f;
  int fixup = stdb::FIX_NONE;
  stdb::RopeParams rope = {};
  int rope_rows = 0;
  void* resid = nullptr;
  float* sumsq_out = nullptr;
  int late_trigger = 0;
  void* amax_top2 = nullptr;
};

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
                       void* act = nullptr, const GemmExtra* ext = nullptr) {
  const int nmma = gemm_nmma(M);
  const uint32_t stage_bytes = stdb::GM_WTILE + static_cast<uint32_t>(nmma) * stdb::GM_BK * 2;
  const uint32_t budget = g_gemm_smem_budget.load();
  int stages = static_cast<int>(budget / stage_bytes);
  stages = stages < 2 ? 2 : (stages > stdb::GM_MAX_STAGES ? stdb::GM_MAX_STAGES : stages);
  const bool norm = ext != nullptr && ext->norm_w != nullptr;
  const bool fused = ext != nullptr && ext->fixup != stdb::FIX_NONE;
  // norm prologue: the CTA's K range of the norm weight after the stages
  const uint32_t kmax = static_cast<uint32_t>((K / stdb::GM_BK + splits - 1) / splits) * stdb::GM_BK;
  const uint32_t normw_bytes =
      norm ? kmax * 2u + ((static_cast<uint32_t>(K / stdb::GM_BM) * static_cast<uint32_t>(M) * 4u + 15u) & ~15u) : 0u;
  if (norm) {
    stages = static_cast<int>((budget - normw_bytes) / stage_bytes);
    stages = stages < 2 ? 2 : (stages > stdb::GM_MAX_STAGES ? stdb::GM_MAX_STAGES : stages);
  }
  // a fused fixup stages the tile's fp32 accumulator ([M][128]) and a 32-row
  // RoPE exchange buffer in the (then idle) stage buffers
  const uint32_t fix_bytes = static_cast<uint32_t>(M) * 512u + 32u * 256u;
  while (fused && static_cast<uint32_t>(stages) * stage_bytes < fix_bytes) ++stages;
  if (stages > stdb::GM_MAX_STAGES) return 1;
  const size_t smem = static_cast<size_t>(stages) * stage_bytes + normw_bytes + 1024;
  if (smem > 227 * 1024) return 1;
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
  const GemmExtra none;
  const GemmExtra& e = ext != nullptr ? *ext : none;
  p.norm_sumsq = e.norm_sumsq;
  p.norm_w = static_cast<const __nv_bfloat16*>(e.norm_w);
  p.norm_eps = e.norm_eps;
  p.fixup = e.fixup;
  p.rope = e.rope;
  p.rope_rows = e.rope_rows;
  p.resid = static_cast<__nv_bfloat16*>(e.resid);
  p.sumsq_out = e.sumsq_out;
  p.late_trigger = e.late_trigger;
  p.amax_top2 = static_cast<float2*>(e.amax_top2);
  // may begin while the previous kernel in the stream finishes: the weight
  // tiles of the first stages are requested before griddepcontrol.wait
  const dim3 grid((N + stdb::GM_BM - 1) / stdb::GM_BM, splits);
  if (fused && splits > 1)  // the splits of a tile reduce in one cluster
    return launch_pdl_cluster(stdb::gemm_kernel, grid, dim3(stdb::GM_THREADS), dim3(1, splits, 1), smem, s, tw, tx,
                              p) == cudaSuccess
               ? 0
               : 4;
  return launch_pdl(stdb::gemm_kernel, grid, dim3(stdb::GM_THREADS), smem, s, tw, tx, p) == cudaSuccess ? 0 : 4;
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
    GemmExtra e;
    if (margin_out != nullptr) {  // per-warp top-2 pairs in the workspace
      if (workspace == nullptr || workspace_bytes < std_gemm_epilogue_workspace_bytes(M, N, K)) return 5;
      e.amax_top2 = workspace;
    }
    int rc = gemm_launch(x, w, nullptr, nullptr, nullptr, M, N, K, 1, s, keys, rows_out, nullptr, &e);
    if (rc != 0) return rc;
    if (margin_out != nullptr)
      return launch_pdl(stdb::argmax_margin_kernel, dim3(rows_out), dim3(256), 0, s, keys,
                        static_cast<const float2*>(workspace), ((N + stdb::GM_BM - 1) / stdb::GM_BM) * 4, M, n,
                        out_stride, out_start, out, margin_out) == cudaSuccess
                 ? 0
                 : 4;
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

// ---------------------------------------------------------------------------
// Decode-layer GEMMs with their neighbours folded in (one launch each):
// the RMSNorm in front of a projection runs on the staged X tiles, and the
// split-K reduction with the op after a projection runs inside the cluster
// formed by each 128-feature tile's K splits (distributed shared memory).
// Only the norm + SiLU / argmax ops take a workspace (split partials for
// their separate reduction kernel, used when K is split).
// ---------------------------------------------------------------------------
// The launch plan of a GEMM: split count (cluster size for the fused
// epilogues) and, for the plain one, of the unfused ops.
extern "C" int std_gemm_plan(int N, int K, int fused, int* splits_out, int* active_clusters_out) {
  if (N <= 0 || K <= 0 || K % stdb::GM_BK != 0 || splits_out == nullptr) return 1;
  const int s = fused ? gemm_splits_cluster(N, K) : gemm_splits(N, K);
  *splits_out = s;
  if (active_clusters_out != nullptr)
    *active_clusters_out = s > 1 ? gemm_active_clusters(s, static_cast<size_t>(stdb::GM_SMEM_BUDGET) + 1024) : 0;
  return 0;
}

extern "C" size_t std_gemm_fused_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  // split partials for the norm + SiLU / argmax ops, or the argmax margins' per-warp top-2 pairs
  const size_t part = std_gemm_workspace_bytes(M, N, K);
  const size_t top2 = static_cast<size_t>((N + stdb::GM_BM - 1) / stdb::GM_BM) * 4 * M * sizeof(float2);
  return part > top2 ? part : top2;
}

static bool fused_ws_ok(void* workspace, size_t workspace_bytes, int M, int N, int K) {
  return workspace != nullptr && workspace_bytes >= std_gemm_fused_workspace_bytes(M, N, K);
}

static bool norm_ok(const float* sumsq, const void* norm_w, int K) {
  return sumsq != nullptr && norm_w != nullptr && K % stdb::GM_BM == 0;
}

extern "C" int std_embed_sumsq(const void* table, int vocab, int H, const int32_t* tok, int tok_stride, int tok_start,
                               int n, int B, void* out, float* sumsq, int ld, void* stream) {
  if (table == nullptr || tok == nullptr || out == nullptr || sumsq == nullptr || vocab <= 0 || H <= 0 ||
      H % stdb::GM_BM != 0 || n <= 0 || B <= 0 || ld < B * n)
    return 1;
  return launch_pdl(stdb::embed_sumsq_kernel, dim3(B * n), dim3(128), 0, static_cast<cudaStream_t>(stream),
                    static_cast<const __nv_bfloat16*>(table), vocab, H, tok, tok_stride, tok_start, n,
                    static_cast<__nv_bfloat16*>(out), sumsq, ld) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_gemm_norm_rope_append(const void* x, const float* sumsq, const void* norm_w, float eps,
                                         const void* w, const void* bias, int M, int K, int B, int n, int Hq, int Hkv,
                                         int D, const int32_t* pos_base, int pos_off, const int32_t* slot_base,
                                         int slot_off, const void* cos_t, const void* sin_t, int max_pos, void* q_out,
                                         void* k_cache, void* v_cache, int cap, void* stream) {
  const int N = (Hq + 2 * Hkv) * D;
  if (D != stdb::GM_BM || B <= 0 || n <= 0 || B * n > M || M > 128 || cap <= 0 || max_pos <= 0) return 1;
  if (!gemm_shape_ok(x, w, M, N, K, 8) || !norm_ok(sumsq, norm_w, K)) return 1;
  if (q_out == nullptr || k_cache == nullptr || v_cache == nullptr || pos_base == nullptr || slot_base == nullptr ||
      cos_t == nullptr || sin_t == nullptr)
    return 1;
  GemmExtra e;
  e.norm_sumsq = sumsq;
  e.norm_w = norm_w;
  e.norm_eps = eps;
  e.fixup = stdb::FIX_ROPE;
  e.rope.n = n;
  e.rope.Hq = Hq;
  e.rope.Hkv = Hkv;
  e.rope.D = D;
  e.rope.cap = cap;
  e.rope.max_pos = max_pos;
  e.rope.pos_base = pos_base;
  e.rope.pos_off = pos_off;
  e.rope.slot_base = slot_base;
  e.rope.slot_off = slot_off;
  e.rope.cos_t = static_cast<const __nv_bfloat16*>(cos_t);
  e.rope.sin_t = static_cast<const __nv_bfloat16*>(sin_t);
  e.rope.q_out = static_cast<__nv_bfloat16*>(q_out);
  e.rope.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  e.rope.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  e.rope_rows = B * n;
  // the draft kernel that follows reads older K/V rows and the lengths before
  // its own wait: release it only once this grid's predecessors are done
  e.late_trigger = 1;
  return gemm_launch(x, w, bias, nullptr, nullptr, M, N, K, gemm_splits_cluster(N, K),
                     static_cast<cudaStream_t>(stream), nullptr, 0, nullptr, &e);
}

extern "C" int std_gemm_residual(const void* a, const void* w, const void* bias, void* resid, float* sumsq_out, int M,
                                 int N, int K, void* stream) {
  if (!gemm_shape_ok(a, w, M, N, K, stdb::GM_BM) || M > 128 || resid == nullptr || sumsq_out == nullptr) return 1;
  GemmExtra e;
  e.fixup = stdb::FIX_RESID;
  e.resid = resid;
  e.sumsq_out = sumsq_out;
  return gemm_launch(a, w, bias, nullptr, nullptr, M, N, K, gemm_splits_cluster(N, K),
                     static_cast<cudaStream_t>(stream), nullptr, 0, nullptr, &e);
}

extern "C" int std_gemm_norm_silu_mul(const void* x, const float* sumsq, const void* norm_w, float eps,
                                      const void* w, int M, int I, int K, void* act, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  const int N = 2 * I;
  if (!gemm_shape_ok(x, w, M, N, K, 8) || act == nullptr || I % 64 != 0 || !norm_ok(sumsq, norm_w, K)) return 1;
  GemmExtra e;
  e.norm_sumsq = sumsq;
  e.norm_w = norm_w;
  e.norm_eps = eps;
  const int splits = gemm_splits(N, K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (splits == 1) return gemm_launch(x, w, nullptr, nullptr, nullptr, M, N, K, 1, s, nullptr, 0, act, &e);
  if (!fused_ws_ok(workspace, workspace_bytes, M, N, K)) return 5;
  float* partial = static_cast<float*>(workspace);
  int rc = gemm_launch(x, w, nullptr, partial, partial, M, N, K, splits, s, nullptr, 0, nullptr, &e);
  if (rc != 0) return rc;
  const size_t total8 = static_cast<size_t>(M) * I / 8;
  const int blocks = static_cast<int>((total8 + 255) / 256 < 148 * 8 ? (total8 + 255) / 256 : 148 * 8);
  return launch_pdl(stdb::silu_mul_kernel<stdb::GemmOut>, dim3(blocks), dim3(256), 0, s,
                    gemm_out_view(partial, nullptr, splits, M, N), I, 1, total8,
                    static_cast<__nv_bfloat16*>(act)) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_gemm_norm_argmax(const void* x, const float* sumsq, const void* norm_w, float eps, const void* w,
                                    int M, int N, int K, int rows_out, int n, int out_stride, int out_start,
                                    int32_t* out, float* margin_out, unsigned long long* keys, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (!gemm_shape_ok(x, w, M, N, K, 8) || out == nullptr || keys == nullptr || !norm_ok(sumsq, norm_w, K)) return 1;
  if (rows_out <= 0 || rows_out > M || n <= 0) return 1;
  GemmExtra e;
  e.norm_sumsq = sumsq;
  e.norm_w = norm_w;
  e.norm_eps = eps;
  const int splits = gemm_splits(N, K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (splits == 1) {
    if (margin_out != nullptr) {
      if (!fused_ws_ok(workspace, workspace_bytes, M, N, K)) return 5;
      e.amax_top2 = workspace;
    }
    int rc = gemm_launch(x, w, nullptr, nullptr, nullptr, M, N, K, 1, s, keys, rows_out, nullptr, &e);
    if (rc != 0) return rc;
    if (margin_out != nullptr)
      return launch_pdl(stdb::argmax_margin_kernel, dim3(rows_out), dim3(256), 0, s, keys,
                        static_cast<const float2*>(workspace), ((N + stdb::GM_BM - 1) / stdb::GM_BM) * 4, M, n,
                        out_stride, out_start, out, margin_out) == cudaSuccess
                 ? 0
                 : 4;
    return launch_pdl(stdb::argmax_keys_kernel, dim3((rows_out + 127) / 128), dim3(128), 0, s, keys, rows_out, n,
                      out_stride, out_start, out) == cudaSuccess
               ? 0
               : 4;
  }
  if (!fused_ws_ok(workspace, workspace_bytes, M, N, K)) return 5;
  float* partial = static_cast<float*>(workspace);
  int rc = gemm_launch(x, w, nullptr, partial, partial, M, N, K, splits, s, nullptr, 0, nullptr, &e);
  if (rc != 0) return rc;
  return launch_pdl(stdb::argmax_kernel<stdb::GemmOut>, dim3(rows_out), dim3(1024), 0, s,
                    gemm_out_view(partial, nullptr, splits, M, N), N, n, out_stride, out_start, out,
                    margin_out) == cudaSuccess
             ? 0
             : 4;
}
