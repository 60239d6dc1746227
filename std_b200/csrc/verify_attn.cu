// verify_attn.cu -- (c) parallel dense verify attention on tcgen05 / TMEM.
//
// Replaces the dense attention of the verify forward
//   std_qwen25vl.py:797-803          model(input_ids=[pending + draft], dense_pkv)
//   modeling_qwen2_5_vl.py:1096-1133 repeat_kv + F.sdpa(attn_mask=causal)
//   modeling_qwen2_5_vl.py:65-101    _make_causal_mask (row i sees keys <= past+i)
// and, with nq = 1, the dense attention of AR decoding
//   std_qwen25vl.py:584-590          ar_generate_qwen25vl loop.
//
// One CTA = one (request, KV head, split of split_keys keys).  The 7 query
// heads of the group times nq tokens form the rows of a 128-row tile
// (row = t*7 + g, zero-padded), so each K/V byte is read once for all 7 heads:
//   S_c  = Q K_c^T    tcgen05.mma M=128 N=64 K=128 (8 x K16), fp32 in TMEM;
//                     Q is the A operand held in TMEM (stored there once)
//   P_c  = exp2(S_c*scale*log2e - m_row), bf16, written into TMEM
//   O   += P_c V_c    tcgen05.mma with P as the A operand in TMEM, V MN-major
//                     from shared memory
// Only K and V cross shared memory.  Two threads issue the MMAs: one the S
// MMAs, one the P.V MMAs (P has its own TMEM columns, so the chains share no
// operand).  A tcgen05.mma costs its issuing thread ~100 cycles; from one
// thread the 12 MMAs of a 64-key chunk and the wait for P serialised into
// ~1670 cycles per chunk.  The softmax waits for P_{c-2} V_{c-2} (its
// group's previous P.V) before it rescales O or rewrites P.
// m_row is a running row max; O is rescaled in TMEM only when a chunk raises
// the max by more than 2^8 (lazy rescale), so the softmax threads normally
// touch TMEM once per chunk.  Warp roles: two softmax warpgroups (warps 0-3 and
// 4-7, one row per thread, chunks alternating); warp 8 lane 0 issues TMA (a
// 6-stage K/V ring); warp 9 allocates TMEM and lane 0 issues the S MMAs;
// warp 10 lane 0 issues the P.V MMAs.  Splits write (O, m, l) partials that a
// second kernel combines; a request whose keys fit one split writes its output
// directly.
//
// Row invariance.  Chunk boundaries (64 keys) and split boundaries
// (split_keys, a function of the cache shape only) sit at fixed absolute key
// positions, and every per-row decision (running max, rescale, masking) uses
// only that row's scores; fully masked chunks and splits contribute exact
// zeros.  A row's result therefore depends only on its query, its visible
// keys and these boundaries -- not on nq or on the other rows.  AR (nq = 1)
// and verify rows (nq = gamma+1) are bit-identical, which STD's
// token-exactness against AR relies on.
#include "common.cuh"

namespace stdb {

constexpr int VF_D = 128;
constexpr int VF_CHUNK = 64;       // keys per chunk (MMA N of S, K of P V)
constexpr int VF_STAGES = 6;       // K/V ring depth
constexpr int VF_THREADS = 352;    // 2 softmax warpgroups + TMA warp + S-MMA warp + PV-MMA warp
constexpr int VF_G = 7;
constexpr uint32_t VF_KV = 16384;     // one K or V chunk: 64 keys x 256 B (two 8 KB d-blocks)
constexpr uint32_t VF_SMEM = 2 * VF_STAGES * VF_KV + 1024;
// TMEM columns (all 512): S[w] (w = chunk & 1) at 64 w; O[w] at 128 + 128 w;
// Q (128 d as 64 bf16 pairs) at 384; P[w] (64 keys as 32 bf16 pairs) at 448 + 32 w
constexpr uint32_t VF_TQ = 384;
constexpr uint32_t VF_TP = 448;
constexpr float VF_RESCALE = 8.0f;    // log2 units

struct VerifyParams {
  const __nv_bfloat16* q;  // [B, nq, Hq, D]
  const int32_t* lens;     // [B]
  int len_offset;          // keys L = lens[b] + len_offset (incl. the nq new keys)
  int nq, cap, Hq, Hkv;
  int causal;              // 1: row t sees keys <= L-nq+t ; 0: every row sees all L keys
  float scale_log2;
  __nv_bfloat16* out;      // [B, nq, Hq, D]
  float* out_f32;          // non-null: fp32 output [B, nq, Hq, D] instead of out (sharded partials)
  float* lse;              // [B, nq, Hq] natural log, may be null
  float* ws_ml;            // [B, Hkv, max_splits, 128, 2]
  float* ws_o;             // [B, Hkv, max_splits, 128, D]
  int max_splits;
  int split_keys;          // keys per split: a multiple of VF_CHUNK fixed by (B, Hkv, cap)
};

STD_DEV int verify_len(const VerifyParams& p, int b) {
  int L = p.lens[b] + p.len_offset;
  if (L > p.cap) L = p.cap;
  if (L < p.nq) L = p.nq;
  return L;
}

// Chunk c of a split goes to softmax warpgroup / TMEM accumulator (c & 1);
// S buffer (c & 1), P buffer (c & 1), K/V stage (c % 4).
__global__ void __launch_bounds__(VF_THREADS, 1)
    verify_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const VerifyParams p) {
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  const int Lraw = p.lens[b] + p.len_offset;
  if ((Lraw > p.cap || Lraw < p.nq) && split == 0 && tid == 0) std_set_error(STD_DEVERR_LENGTH);
  const int L = verify_len(p, b);
  const int n_splits = (L + p.split_keys - 1) / p.split_keys;
  if (split >= n_splits || split >= p.max_splits) {
    pdl_launch_dependents();
    return;
  }
  const int k0 = split * p.split_keys;
  const int k1 = min(k0 + p.split_keys, L);
  const int nchunks = (k1 - k0 + VF_CHUNK - 1) / VF_CHUNK;
  const int nrows = VF_G * p.nq;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;                                  // [VF_STAGES][VF_KV]
  uint8_t* sV = sK + VF_STAGES * VF_KV;                // [VF_STAGES][VF_KV]

  __shared__ __align__(8) uint64_t bar_q, bar_kv_full[VF_STAGES], bar_kv_empty[VF_STAGES], bar_s_full[2],
      bar_s_free[2], bar_p_full[2], bar_pv_done[2], bar_mma_done;
  __shared__ uint32_t s_tmem;
  __shared__ float s_mB[128], s_lB[128];

  if (warp == 9) {
    tmem_alloc(&s_tmem, 512);
    tmem_relinquish();
  }
  if (tid == 256) {
    mbar_init(&bar_q, 128);
    for (int i = 0; i < VF_STAGES; ++i) {
      mbar_init(&bar_kv_full[i], 1);
      mbar_init(&bar_kv_empty[i], 1);
    }
    // only the warps that hold query rows take part in the softmax handshakes
    const uint32_t live_threads = 32u * static_cast<uint32_t>(min(4, (nrows + 31) / 32));
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_s_full[i], 1);
      mbar_init(&bar_s_free[i], live_threads);
      mbar_init(&bar_p_full[i], live_threads);
      mbar_init(&bar_pv_done[i], 1);
    }
    mbar_init(&bar_mma_done, 1);
    fence_barrier_init();
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Dependents may launch only once this CTA holds its TMEM: a successor that
  // allocates TMEM before its own griddepcontrol.wait can then never take
  // columns this CTA still needs.
  pdl_launch_dependents();
  const uint32_t tmem = s_tmem;  // S[w]: cols 64w .. 64w+63; O[w]: cols 128 + 128w
  const int row0 = (b * p.Hkv + kvh) * p.cap;

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();  // each K/V row is read once per forward
      int issued = 0;
      for (int c = 0; c < nchunks; ++c) {
        const int st = c % VF_STAGES;
        if (c >= VF_STAGES && !mbar_wait(&bar_kv_empty[st], ((c / VF_STAGES) - 1) & 1)) break;
        mbar_arrive_expect_tx(&bar_kv_full[st], 2 * VF_KV);
        const int y = row0 + k0 + c * VF_CHUNK;
        uint8_t* kd = sK + st * VF_KV;
        uint8_t* vd = sV + st * VF_KV;
        tma_load_2d_hint(kd, &tmK, &bar_kv_full[st], 0, y, pol);
        tma_load_2d_hint(kd + VF_KV / 2, &tmK, &bar_kv_full[st], 64, y, pol);
        tma_load_2d_hint(vd, &tmV, &bar_kv_full[st], 0, y, pol);
        tma_load_2d_hint(vd + VF_KV / 2, &tmV, &bar_kv_full[st], 64, y, pol);
        issued = c + 1;
      }
      // never leave a copy in flight: wait for the last load of each stage
      for (int c = issued - VF_STAGES < 0 ? 0 : issued - VF_STAGES; c < issued; ++c)
        mbar_wait(&bar_kv_full[c % VF_STAGES], (c / VF_STAGES) & 1);
    }
  } else if (warp == 9) {
    // ---------------- S issuer: S_c = Q K_c^T into S[c & 1] ----------------
    if (lane == 0) {
      const uint32_t idS = idesc_bf16_f32(128, VF_CHUNK, 0, 0);
      bool ok = mbar_wait(&bar_q, 0);
      tc_fence_after();
      for (int c = 0; ok && c < nchunks; ++c) {
        const int st = c % VF_STAGES, w = c & 1;
        // K_c landed; S[w] read by the softmax of chunk c - 2
        if (!mbar_wait(&bar_kv_full[st], (c / VF_STAGES) & 1)) break;
        if (c >= 2 && !mbar_wait(&bar_s_free[w], ((c >> 1) - 1) & 1)) break;
        tc_fence_after();
        const uint32_t aK = smem_u32(sK + st * VF_KV);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t offK = (ks >> 2) * (VF_KV / 2) + (ks & 3) * 32u;
          umma_bf16_ts(tmem + w * VF_CHUNK, tmem + VF_TQ + ks * 8, sdesc_sw128(aK + offK, 16, 1024), idS,
                       ks > 0 ? 1u : 0u);
        }
        umma_commit(&bar_s_full[w]);
      }
    }
  } else if (warp == 10) {
    // ---------------- P.V issuer: O[c & 1] += P_c V_c ----------------
    if (lane == 0) {
      const uint32_t idO = idesc_bf16_f32(128, VF_D, 0, 1);
      for (int c = 0; c < nchunks; ++c) {
        const int st = c % VF_STAGES, w = c & 1;
        if (!mbar_wait(&bar_p_full[w], (c >> 1) & 1)) break;
        tc_fence_after();
        const uint32_t aV = smem_u32(sV + st * VF_KV);
#pragma unroll
        for (int ks = 0; ks < VF_CHUNK / 16; ++ks) {
          umma_bf16_ts(tmem + 128 + 128 * w, tmem + VF_TP + w * 32 + ks * 8,
                       sdesc_sw128(aV + ks * 2048u, VF_KV / 2, 1024), idO, (c >= 2 || ks > 0) ? 1u : 0u);
        }
        // S_c retired before P_c existed, so both halves of the stage are free
        umma_commit(&bar_kv_empty[st]);
        umma_commit(&bar_pv_done[w]);
      }
      // the last P V retires after every S (each P needs its S)
      umma_commit(&bar_mma_done);
    }
  } else {
    // ---------------- softmax warpgroups: thread = row ----------------
    const int wg = warp >> 2;          // 0 or 1
    const int r = tid & 127;
    const int t = r / VF_G, g = r % VF_G;
    const bool valid_row = r < nrows;
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    if (wg == 0) {
      // this row's query (zero for padding rows) into the Q columns of TMEM
      const uint4* src = reinterpret_cast<const uint4*>(
          p.q + ((static_cast<size_t>(b) * p.nq + (valid_row ? t : 0)) * p.Hq + kvh * VF_G + g) * VF_D);
      uint32_t qw[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = valid_row ? src[half * 8 + c] : make_uint4(0, 0, 0, 0);
          qw[4 * c] = v.x;
          qw[4 * c + 1] = v.y;
          qw[4 * c + 2] = v.z;
          qw[4 * c + 3] = v.w;
        }
        tmem_st32(trow + VF_TQ + half * 32, qw);
      }
      if (warp * 32 >= nrows) {
        // an all-padding warp never writes P: zero its rows of both P buffers
#pragma unroll
        for (int j = 0; j < 32; ++j) qw[j] = 0u;
        tmem_st32(trow + VF_TP, qw);
        tmem_st32(trow + VF_TP + 32, qw);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_q);
    }
    const int limit = min(p.causal ? (L - p.nq + t) : (L - 1), k1 - 1);  // last visible key
    const uint32_t tO = trow + 128 + 128 * wg;
    const float sc = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    uint32_t s[VF_CHUNK];
    // a warp whose 32 rows are all padding (rows >= 7*nq) skips the softmax
    const bool live = (warp & 3) * 32 < nrows;

    for (int c = wg; live && c < nchunks; c += 2) {
      const int kk = c >> 1;
      if (ok) ok = mbar_wait(&bar_s_full[wg], kk & 1);  // S_c in TMEM
      __syncwarp();
      tc_fence_after();
      tmem_ld32(trow + wg * VF_CHUNK, s);
      tmem_ld32(trow + wg * VF_CHUNK + 32, s + 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bar_s_free[wg]);
      const int nvis = limit - (k0 + c * VF_CHUNK) + 1;  // visible keys of this chunk
      float mraw = -INFINITY;
      if (nvis >= VF_CHUNK) {
#pragma unroll
        for (int j = 0; j < VF_CHUNK; ++j) mraw = fmaxf(mraw, __uint_as_float(s[j]));
      } else {
#pragma unroll
        for (int j = 0; j < VF_CHUNK; ++j)
          if (j < nvis) mraw = fmaxf(mraw, __uint_as_float(s[j]));
      }
      const float m_c = mraw * sc;  // scale > 0: max commutes with the scaling
      // O[wg] and P[wg] are free once this group's previous P V has retired
      if (c >= 2 && ok) ok = mbar_wait(&bar_pv_done[wg], ((c >> 1) - 1) & 1);
      __syncwarp();
      tc_fence_after();
      const bool need = (m_run != -INFINITY) && (m_c > m_run + VF_RESCALE);
      if (__any_sync(0xffffffffu, need)) {
        const float alpha = need ? exp2f(m_run - m_c) : 1.0f;
        uint32_t o[32];
#pragma unroll
        for (int piece = 0; piece < 4; ++piece) {
          tmem_ld32(tO + piece * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
          tmem_st32(tO + piece * 32, o);
        }
        tmem_wait_st();
        if (need) {
          l_run *= alpha;
          m_run = m_c;
        }
      }
      if (m_run == -INFINITY) m_run = m_c;
      const float nm = -m_run;
      const bool any = m_run != -INFINITY;
      // P as bf16 pairs (keys j, j+1 in column j/2) over S's first 32 columns
      uint32_t pk[VF_CHUNK / 2];
#pragma unroll
      for (int j = 0; j < VF_CHUNK; j += 2) {
        float e0 = (any && j < nvis) ? ex2_approx(fmaf(__uint_as_float(s[j]), sc, nm)) : 0.f;
        float e1 = (any && j + 1 < nvis) ? ex2_approx(fmaf(__uint_as_float(s[j + 1]), sc, nm)) : 0.f;
        l_run += e0 + e1;
        pk[j / 2] = pack_bf16x2(e0, e1);
      }
      tmem_st32(trow + VF_TP + wg * 32, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_p_full[wg]);
    }
    // ---- combine the two accumulators (row-local), write output or partial ----
    if (ok) ok = mbar_wait(&bar_mma_done, 0);
    __syncwarp();
    tc_fence_after();
    if (wg == 1) {
      s_mB[r] = m_run;
      s_lB[r] = l_run;
    }
    named_bar_sync(1, 256);
    if (wg == 0) {
      const float mB = s_mB[r], lB = s_lB[r];
      const bool hasA = m_run != -INFINITY && l_run > 0.f, hasB = mB != -INFINITY && lB > 0.f;
      const float m = hasA ? (hasB ? fmaxf(m_run, mB) : m_run) : (hasB ? mB : -INFINITY);
      const float wa = hasA ? exp2f(m_run - m) : 0.f, wb = hasB ? exp2f(mB - m) : 0.f;
      const float l = (hasA ? l_run * wa : 0.f) + (hasB ? lB * wb : 0.f);
      const bool single = n_splits == 1;
      const float inv = (single && l > 0.f) ? 1.f / l : 1.f;
      uint32_t oa[32], ob[32];
#pragma unroll
      for (int piece = 0; piece < 4; ++piece) {
        tmem_ld32(trow + 128 + piece * 32, oa);
        tmem_ld32(trow + 256 + piece * 32, ob);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float x = hasA ? __uint_as_float(oa[j]) * wa : 0.f;
          if (hasB) x += __uint_as_float(ob[j]) * wb;
          v[j] = x * inv;
        }
        if (valid_row) {
          if (single && p.out_f32 != nullptr) {
            float4* dst = reinterpret_cast<float4*>(
                p.out_f32 + ((static_cast<size_t>(b) * p.nq + t) * p.Hq + kvh * VF_G + g) * VF_D + piece * 32);
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) dst[c4] = make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
          } else if (single) {
            uint4* dst = reinterpret_cast<uint4*>(
                p.out + ((static_cast<size_t>(b) * p.nq + t) * p.Hq + kvh * VF_G + g) * VF_D + piece * 32);
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
              dst[c4] = make_uint4(pack_bf16x2(v[8 * c4], v[8 * c4 + 1]), pack_bf16x2(v[8 * c4 + 2], v[8 * c4 + 3]),
                                   pack_bf16x2(v[8 * c4 + 4], v[8 * c4 + 5]), pack_bf16x2(v[8 * c4 + 6], v[8 * c4 + 7]));
          } else {
            const size_t slot = ((static_cast<size_t>(b) * p.Hkv + kvh) * p.max_splits + split) * 128 + r;
            float4* dst = reinterpret_cast<float4*>(p.ws_o + slot * VF_D + piece * 32);
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) dst[c4] = make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
          }
        }
      }
      if (valid_row) {
        if (single) {
          if (p.lse != nullptr)
            p.lse[(static_cast<size_t>(b) * p.nq + t) * p.Hq + kvh * VF_G + g] =
                l > 0.f ? (m + log2f(l)) * 0.69314718055994530942f : -INFINITY;
        } else {
          const size_t slot = ((static_cast<size_t>(b) * p.Hkv + kvh) * p.max_splits + split) * 128 + r;
          p.ws_ml[slot * 2 + 0] = l > 0.f ? m : -INFINITY;
          p.ws_ml[slot * 2 + 1] = l;
        }
      }
    }
  }

  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Combine split partials: m = max_s m_s, w_s = exp2(m_s - m) (0 for splits a
// row cannot see), out = (sum_s w_s o_s) / (sum_s w_s l_s).  One block of nw
// warps per query row (nw = ceil(max_splits / VM_PER), at most VM_WARPS: a
// function of the cache shape); requests whose keys fit one split are skipped
// (the split kernel wrote them).  At small batches this kernel is a chain of
// dependent memory round trips, so it is laid out for latency: warp w takes
// splits w, w + nw, ... (lane = 4 dims) and loads its first VM_PER of them
// while the block reduces the split maxima, so up to nw * VM_PER splits cost
// one round trip; the warps' sums are added in warp order -- a fixed order,
// so the result depends only on the split boundaries (an AR step and a
// verify block on the same cache combine identically).
constexpr int VM_WARPS = 8, VM_PER = 8;

__global__ void __launch_bounds__(VM_WARPS * 32) verify_merge_kernel(const VerifyParams p) {
  pdl_launch_dependents();  // followed by the O projection GEMM (weights before its wait)
  pdl_wait();
  const int r = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int L = verify_len(p, b);
  const int n_splits = (L + p.split_keys - 1) / p.split_keys;
  if (n_splits <= 1 || r >= VF_G * p.nq) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  const size_t slot0 = (static_cast<size_t>(b) * p.Hkv + kvh) * p.max_splits * 128 + r;
  const float2* ml = reinterpret_cast<const float2*>(p.ws_ml) + slot0;                  // split s: ml[s * 128]
  const float4* os = reinterpret_cast<const float4*>(p.ws_o) + slot0 * (VF_D / 4) + lane;  // split s: os[s * 4096]
  float2 mlv[VM_PER];
  float4 ov[VM_PER];
#pragma unroll
  for (int j = 0; j < VM_PER; ++j) {
    const int s = warp + nw * j;
    mlv[j] = s < n_splits ? __ldcg(ml + static_cast<size_t>(s) * 128) : make_float2(-INFINITY, 0.f);
    ov[j] = s < n_splits ? __ldcg(os + static_cast<size_t>(s) * 128 * (VF_D / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __shared__ float s_m[VM_WARPS];
  __shared__ float s_l[VM_WARPS];
  __shared__ float4 s_a[VM_WARPS][32];
  float m = -INFINITY;
  for (int s = tid; s < n_splits; s += nw * 32) m = fmaxf(m, __ldcg(&ml[static_cast<size_t>(s) * 128].x));
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, sh));
  if (lane == 0) s_m[warp] = m;
  __syncthreads();
  m = s_m[0];
  for (int w = 1; w < nw; ++w) m = fmaxf(m, s_m[w]);
  float l = 0.f;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < n_splits; s0 += nw * VM_PER) {
    if (s0 > 0) {
#pragma unroll
      for (int j = 0; j < VM_PER; ++j) {
        const int s = s0 + warp + nw * j;
        mlv[j] = s < n_splits ? __ldcg(ml + static_cast<size_t>(s) * 128) : make_float2(-INFINITY, 0.f);
        ov[j] = s < n_splits ? __ldcg(os + static_cast<size_t>(s) * 128 * (VF_D / 4))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int j = 0; j < VM_PER; ++j) {
      // past the last split, or a split the row cannot see (m_s = -inf, l_s =
      // 0, o_s = 0: the split kernel writes every row): weight 0 adds +-0 to
      // sums that start at +0
      const bool live = mlv[j].x != -INFINITY;
      const float w = live ? exp2f(mlv[j].x - m) : 0.f;
      l += w * mlv[j].y;
      a.x += w * ov[j].x;
      a.y += w * ov[j].y;
      a.z += w * ov[j].z;
      a.w += w * ov[j].w;
    }
  }
  s_a[warp][lane] = a;
  if (lane == 0) s_l[warp] = l;
  __syncthreads();
  if (warp != 0) return;
  a = s_a[0][lane];
  l = s_l[0];
  for (int w = 1; w < nw; ++w) {
    const float4 t = s_a[w][lane];
    a.x += t.x;
    a.y += t.y;
    a.z += t.z;
    a.w += t.w;
    l += s_l[w];
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  const int t = r / VF_G, g = r % VF_G;
  const size_t o = ((static_cast<size_t>(b) * p.nq + t) * p.Hq + kvh * VF_G + g) * VF_D + 4 * lane;
  if (p.out_f32 != nullptr) {
    *reinterpret_cast<float4*>(p.out_f32 + o) = make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
  } else {
    uint2 pk;
    pk.x = pack_bf16x2(a.x * inv, a.y * inv);
    pk.y = pack_bf16x2(a.z * inv, a.w * inv);
    *reinterpret_cast<uint2*>(p.out + o) = pk;
  }
  if (lane == 0 && p.lse != nullptr)
    p.lse[(static_cast<size_t>(b) * p.nq + t) * p.Hq + kvh * VF_G + g] =
        l > 0.f ? (m + log2f(l)) * 0.69314718055994530942f : -INFINITY;
}

}  // namespace stdb

// ---------------------------------------------------------------------------
// host: tensor maps and C ABI
// ---------------------------------------------------------------------------
// Keys per split, fixed by the cache shape alone (so two calls on the same
// cache -- an AR step and a verify block -- use the same split boundaries).
// The split count per (request, head) is chosen so the CTAs fill whole waves of
// the 148 SMs (one CTA per SM) as evenly as possible, preferring fewer waves.
static int verify_split_keys(int B, int Hkv, int cap) {
  const long heads = static_cast<long>(B) * Hkv;
  const long max_ns = (cap + 2 * stdb::VF_CHUNK - 1) / (2 * stdb::VF_CHUNK);  // >= 2 chunks per split
  long best_ns = 1;
  double best_eff = -1.0;
  for (long waves = 1; waves <= 4; ++waves) {
    long ns = waves * 148 / heads;
    if (ns < 1) ns = 1;
    if (ns > max_ns) ns = max_ns;
    const long ctas = heads * ns;
    const double eff = static_cast<double>(ctas) / (static_cast<double>((ctas + 147) / 148) * 148.0);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best_ns = ns;
    }
  }
  long keys = (cap + best_ns - 1) / best_ns;
  keys = ((keys + stdb::VF_CHUNK - 1) / stdb::VF_CHUNK) * stdb::VF_CHUNK;
  if (keys < stdb::VF_CHUNK) keys = stdb::VF_CHUNK;
  return static_cast<int>(keys);
}

extern "C" size_t std_verify_attn_workspace_bytes(int B, int Hkv, int cap) {
  if (B <= 0 || Hkv <= 0 || cap <= 0) return 0;
  const int split_keys = verify_split_keys(B, Hkv, cap);
  const size_t max_splits = (cap + split_keys - 1) / split_keys;
  const size_t n = static_cast<size_t>(B) * Hkv;
  size_t bytes = n * max_splits * 128 * 2 * 4;
  bytes = ((bytes + 255) / 256) * 256;
  bytes += n * max_splits * 128 * stdb::VF_D * 4;
  return bytes;
}

static int verify_launch(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens, int len_offset,
                         int nq, int causal, int B, int Hq, int Hkv, int D, int cap, void* out, float* out_f32,
                         float* lse, void* workspace, size_t workspace_bytes, void* stream);

extern "C" int std_verify_attn(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens,
                               int len_offset, int nq, int causal, int B, int Hq, int Hkv, int D, int cap, void* out,
                               float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  if (out == nullptr) return 1;
  return verify_launch(q, k_cache, v_cache, lens, len_offset, nq, causal, B, Hq, Hkv, D, cap, out, nullptr, lse,
                       workspace, workspace_bytes, stream);
}

extern "C" int std_verify_attn_partial(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens,
                                       int len_offset, int nq, int causal, int B, int Hq, int Hkv, int D, int cap,
                                       float* out_f32, float* lse, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  if (out_f32 == nullptr || lse == nullptr) return 1;
  return verify_launch(q, k_cache, v_cache, lens, len_offset, nq, causal, B, Hq, Hkv, D, cap, nullptr, out_f32, lse,
                       workspace, workspace_bytes, stream);
}

static int verify_launch(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens, int len_offset,
                         int nq, int causal, int B, int Hq, int Hkv, int D, int cap, void* out, float* out_f32,
                         float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  if (D != stdb::VF_D || Hq != Hkv * stdb::VF_G || nq < 1 || stdb::VF_G * nq > 128 || B <= 0 || cap <= 0) return 1;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || lens == nullptr) return 1;
  if (((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(q)) &
       15) != 0)
    return 1;
  if (workspace == nullptr || workspace_bytes < std_verify_attn_workspace_bytes(B, Hkv, cap)) return 5;
  static SmemGrant grant;
  if (ensure_smem(stdb::verify_attn_kernel, grant, stdb::VF_SMEM) != 0) return 3;
  CUtensorMap tk, tv;
  const uint64_t rows = static_cast<uint64_t>(B) * Hkv * cap;
  int rc = make_tmap_bf16_2d(&tk, k_cache, rows, 128, 256, 64, stdb::VF_CHUNK);
  if (rc == 0) rc = make_tmap_bf16_2d(&tv, v_cache, rows, 128, 256, 64, stdb::VF_CHUNK);
  if (rc != 0) return rc;
  stdb::VerifyParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.lens = lens;
  p.len_offset = len_offset;
  p.nq = nq;
  p.cap = cap;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.causal = causal;
  p.scale_log2 = (1.0f / sqrtf(static_cast<float>(D))) * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_f32 = out_f32;
  p.lse = lse;
  p.split_keys = verify_split_keys(B, Hkv, cap);
  p.max_splits = (cap + p.split_keys - 1) / p.split_keys;
  const size_t n = static_cast<size_t>(B) * Hkv;
  char* ws = static_cast<char*>(workspace);
  p.ws_ml = reinterpret_cast<float*>(ws);
  size_t off = n * p.max_splits * 128 * 2 * 4;
  off = ((off + 255) / 256) * 256;
  p.ws_o = reinterpret_cast<float*>(ws + off);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(p.max_splits, Hkv, B);
  if (launch_pdl(stdb::verify_attn_kernel, grid, dim3(stdb::VF_THREADS), stdb::VF_SMEM, s, tk, tv, p) != cudaSuccess)
    return 4;
  if (p.max_splits > 1) {
    dim3 mgrid(stdb::VF_G * nq, Hkv, B);  // one block per row
    const int nw = std::min<int>(stdb::VM_WARPS, (p.max_splits + stdb::VM_PER - 1) / stdb::VM_PER);
    if (launch_pdl(stdb::verify_merge_kernel, mgrid, dim3(32 * nw), 0, s, p) != cudaSuccess) return 4;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

// ---------------------------------------------------------------------------
// std_verify_attn_noalloc: the verify entry point for callers that cannot
// allocate device memory.
//
// Some callers of this path are not allowed to call cudaMalloc at all: a
// serving process that reserves the whole GPU for its own memory pool and
// does not let plugins allocate outside it; a foreign-language host (an FFI
// or ctypes caller without torch) that has no device allocator of its own; a
// latency-critical loop where an allocation, which may synchronise the
// device, is not acceptable.  For them the split-partial scratch of the
// verify kernel lives in a fixed file-scope __device__ array instead of a
// caller workspace.  Every GPU that loads this library holds that array
// (STD_VERIFY_NOALLOC_SCRATCH_BYTES) until the process exits.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(32) << 20;  // == STD_VERIFY_NOALLOC_SCRATCH_BYTES
__device__ __align__(256) unsigned char g_verify_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[STD_MAX_DEVICES] = {};  // device address of the array, per device ordinal

// On the host, g_verify_noalloc_scratch only stands in for the symbol; its
// device address is looked up once per device, with that device current.
int noalloc_scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 4;
  if (dev < 0 || dev >= STD_MAX_DEVICES) return 3;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_verify_noalloc_scratch) != cudaSuccess || p == nullptr) return 4;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}
}  // namespace

extern "C" int std_verify_attn_noalloc(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens,
                                       int len_offset, int nq, int causal, int B, int Hq, int Hkv, int D, int cap,
                                       void* out, float* lse, void* stream) {
  // argument errors (status 1) take precedence over the capacity check (status 2)
  if (D != stdb::VF_D || Hkv <= 0 || Hq != Hkv * stdb::VF_G || nq < 1 || stdb::VF_G * nq > 128 || B <= 0 || cap <= 0)
    return 1;
  if (std_verify_attn_workspace_bytes(B, Hkv, cap) > kNoAllocScratchBytes) return 2;
  void* scratch = nullptr;
  const int rc = noalloc_scratch_for_current_device(&scratch);
  if (rc != 0) return rc;
  // Nothing in the scratch has to start at zero: every partial the merge
  // reads was written by the split kernel of the same call.
  return std_verify_attn(q, k_cache, v_cache, lens, len_offset, nq, causal, B, Hq, Hkv, D, cap, out, lse, scratch,
                         kNoAllocScratchBytes, stream);
}
