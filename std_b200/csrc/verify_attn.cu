// verify_attn.cu -- (c) parallel dense verify attention on tcgen05 / TMEM.
//
// Replaces the dense attention of the verify forward
//   std_qwen25vl.py:797-803          model(input_ids=[pending + draft], dense_pkv)
//   modeling_qwen2_5_vl.py:1096-1133 repeat_kv + F.sdpa(attn_mask=causal)
//   modeling_qwen2_5_vl.py:65-101    _make_causal_mask (row i sees keys <= past+i)
// and, with nq = 1, the dense attention of AR decoding
//   std_qwen25vl.py:584-590          ar_generate_qwen25vl loop.
//
// One CTA = one (request, KV head, split of 512 keys).  The 7 query heads of
// the group times nq tokens form the rows of a 128-row tile (row = t*7 + g,
// zero-padded), so each K/V byte is read once for all 7 heads:
//   S_c  = Q K_c^T   tcgen05.mma M=128 N=128 K=128 (8 x K16), fp32 in TMEM
//   P_c  = exp2(S_c*scale*log2e - rowmax_c), bf16, written to smem (SW128)
//   O_c  = P_c V_c   tcgen05.mma M=128 N=128 K=128, V as an MN-major operand
// Warp roles: warps 0-3 own TMEM lanes 0-127 (one row per thread: softmax,
// chunk merge, epilogue); warp 4 lane 0 issues TMA (K/V chunks, 2 stages);
// warp 5 allocates TMEM and lane 0 issues the MMAs.
//
// Canonical reduction tree.  Chunk boundaries (128 keys) and split boundaries
// (512 keys) sit at fixed absolute key positions; each chunk is normalised to
// its own max and chunk partials are merged in key order, fully masked chunks
// are skipped, and splits are merged in split order the same way.  A row's
// result therefore depends only on its query, its visible keys and these
// boundaries -- not on nq or on the other rows.  AR (nq = 1) and verify rows
// (nq = gamma+1) through this kernel are bit-identical, which STD's
// token-exactness against AR relies on.
#include "common.cuh"

namespace stdb {

constexpr int VF_D = 128;
constexpr int VF_CHUNK = 128;
constexpr int VF_SPLIT = 512;
constexpr int VF_THREADS = 192;
constexpr int VF_G = 7;
constexpr uint32_t VF_TILE = 32768;  // 128 rows x 256 B
constexpr uint32_t VF_SMEM = 6 * VF_TILE + 1024;

struct VerifyParams {
  const __nv_bfloat16* q;  // [B, nq, Hq, D]
  const int32_t* lens;     // [B]
  int len_offset;          // keys L = lens[b] + len_offset (incl. the nq new keys)
  int nq, cap, Hq, Hkv;
  int causal;              // 1: row t sees keys <= L-nq+t ; 0: every row sees all L keys
  float scale_log2;
  __nv_bfloat16* out;      // [B, nq, Hq, D]
  float* lse;              // [B, nq, Hq] natural log, may be null
  int* counters;           // [B, Hkv]
  float* ws_ml;            // [B, Hkv, max_splits, 128, 2]
  float* ws_o;             // [B, Hkv, max_splits, 128, D]
  int max_splits;
};

STD_DEV void merge_chunk(float* acc, float& m_run, float& l_run, const uint32_t* oc, int base, float m_c,
                         float l_c, float& a_out, float& b_out) {
  (void)acc;
  (void)oc;
  (void)base;
  if (m_c == -INFINITY) {
    a_out = 1.f;
    b_out = 0.f;
    return;
  }
  if (m_run == -INFINITY) {
    a_out = 0.f;
    b_out = 1.f;
    m_run = m_c;
    l_run = l_c;
    return;
  }
  const float mn = fmaxf(m_run, m_c);
  a_out = exp2f(m_run - mn);
  b_out = exp2f(m_c - mn);
  l_run = l_run * a_out + l_c * b_out;
  m_run = mn;
}

__global__ void __launch_bounds__(VF_THREADS, 1)
    verify_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const VerifyParams p) {
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int L = p.lens[b] + p.len_offset;
  if (L > p.cap || L < p.nq) {
    if (split == 0 && tid == 0) std_set_error(STD_DEVERR_LENGTH);
    L = L > p.cap ? p.cap : p.nq;
  }
  const int n_splits = (L + VF_SPLIT - 1) / VF_SPLIT;
  if (split >= n_splits || split >= p.max_splits) return;
  const int k0 = split * VF_SPLIT;
  const int k1 = min(k0 + VF_SPLIT, L);
  const int nchunks = (k1 - k0 + VF_CHUNK - 1) / VF_CHUNK;
  const int nrows = VF_G * p.nq;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK[2] = {smem + VF_TILE, smem + 2 * VF_TILE};
  uint8_t* sV[2] = {smem + 3 * VF_TILE, smem + 4 * VF_TILE};
  uint8_t* sP = smem + 5 * VF_TILE;

  __shared__ __align__(8) uint64_t bar_q, bar_kv_full[2], bar_kv_empty[2], bar_s_full[2], bar_s_free[2], bar_p_full,
      bar_o_full, bar_mma_done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_ticket;

  if (warp == 5) {
    tmem_alloc(&s_tmem, 512);
    tmem_relinquish();
  }
  if (tid == 128) {
    mbar_init(&bar_q, 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_kv_full[i], 1);
      mbar_init(&bar_kv_empty[i], 1);
      mbar_init(&bar_s_full[i], 1);
      mbar_init(&bar_s_free[i], 128);
    }
    mbar_init(&bar_p_full, 128);
    mbar_init(&bar_o_full, 1);
    mbar_init(&bar_mma_done, 1);
    fence_barrier_init();
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int row0 = (b * p.Hkv + kvh) * p.cap;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int c = 0; c < nchunks; ++c) {
        const int st = c & 1;
        if (c >= 2 && !mbar_wait(&bar_kv_empty[st], ((c >> 1) - 1) & 1)) break;
        mbar_arrive_expect_tx(&bar_kv_full[st], 4 * 16384);
        const int y = row0 + k0 + c * VF_CHUNK;
        tma_load_2d(sK[st], &tmK, &bar_kv_full[st], 0, y);
        tma_load_2d(sK[st] + 16384, &tmK, &bar_kv_full[st], 64, y);
        tma_load_2d(sV[st], &tmV, &bar_kv_full[st], 0, y);
        tma_load_2d(sV[st] + 16384, &tmV, &bar_kv_full[st], 64, y);
        issued = c + 1;
      }
      // never leave a copy in flight: wait for the last load of each stage
      for (int c = issued - 2 < 0 ? 0 : issued - 2; c < issued; ++c) mbar_wait(&bar_kv_full[c & 1], (c >> 1) & 1);
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idS = idesc_bf16_f32(128, 128, 0, 0);
      const uint32_t idO = idesc_bf16_f32(128, 128, 0, 1);
      const uint32_t aQ = smem_u32(sQ), aP = smem_u32(sP);
      bool ok = mbar_wait(&bar_q, 0);
      tc_fence_after();
      auto issue_S = [&](int c) -> bool {
        const int st = c & 1;
        if (!mbar_wait(&bar_kv_full[st], (c >> 1) & 1)) return false;
        if (c >= 2 && !mbar_wait(&bar_s_free[st], ((c >> 1) - 1) & 1)) return false;
        tc_fence_after();
        const uint32_t aK = smem_u32(sK[st]);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (ks >> 2) * 16384u + (ks & 3) * 32u;
          umma_bf16(tmem + st * 128, sdesc_sw128(aQ + off, 16, 1024), sdesc_sw128(aK + off, 16, 1024), idS,
                    ks > 0 ? 1u : 0u);
        }
        umma_commit(&bar_s_full[st]);
        return true;
      };
      if (ok) ok = issue_S(0);
      for (int c = 0; ok && c < nchunks; ++c) {
        if (c + 1 < nchunks && !issue_S(c + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&bar_p_full, c & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t aV = smem_u32(sV[c & 1]);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t offP = (ks >> 2) * 16384u + (ks & 3) * 32u;
          umma_bf16(tmem + 256, sdesc_sw128(aP + offP, 16, 1024), sdesc_sw128(aV + ks * 2048u, 16384, 1024), idO,
                    ks > 0 ? 1u : 0u);
        }
        umma_commit(&bar_o_full);
        umma_commit(&bar_kv_empty[c & 1]);
      }
      umma_commit(&bar_mma_done);
      mbar_wait(&bar_mma_done, 0);
    }
  } else {
    // ---------------- softmax / merge / epilogue: thread = row ----------------
    const int r = tid;
    const int t = r / VF_G, g = r % VF_G;
    const bool valid_row = r < nrows;
    {
      const uint4* src = reinterpret_cast<const uint4*>(
          p.q + ((static_cast<size_t>(b) * p.nq + (valid_row ? t : 0)) * p.Hq + kvh * VF_G + g) * VF_D);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 v = valid_row ? src[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sQ + (c >> 3) * 16384u + sw128_offset(r, c & 7)) = v;
      }
    }
    fence_async_smem();
    mbar_arrive(&bar_q);

    const int limit = p.causal ? (L - p.nq + t) : (L - 1);  // last visible key
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float acc[VF_D];
#pragma unroll
    for (int d = 0; d < VF_D; ++d) acc[d] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    float m_prev = -INFINITY, l_prev = 0.f;
    bool ok = true;
    uint32_t v[32];

    auto merge_o = [&](float m_c, float l_c) {
      float a, bb;
      merge_chunk(acc, m_run, l_run, nullptr, 0, m_c, l_c, a, bb);
#pragma unroll
      for (int piece = 0; piece < 4; ++piece) {
        tmem_ld32(trow + 256 + piece * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float oc = __uint_as_float(v[j]);
          float& x = acc[piece * 32 + j];
          if (bb == 1.f && a == 0.f)
            x = oc;
          else if (bb != 0.f)
            x = x * a + oc * bb;
        }
      }
    };

    for (int c = 0; c < nchunks; ++c) {
      const int sb = c & 1;
      if (ok) ok = mbar_wait(&bar_s_full[sb], (c >> 1) & 1);
      tc_fence_after();
      const int key0 = k0 + c * VF_CHUNK;
      float m_c = -INFINITY;
#pragma unroll
      for (int piece = 0; piece < 4; ++piece) {
        tmem_ld32(trow + sb * 128 + piece * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int key = key0 + piece * 32 + j;
          if (key <= limit && key < k1) m_c = fmaxf(m_c, __uint_as_float(v[j]) * p.scale_log2);
        }
      }
      if (c > 0) {
        if (ok) ok = mbar_wait(&bar_o_full, (c - 1) & 1);
        tc_fence_after();
        merge_o(m_prev, l_prev);
      }
      float l_c = 0.f;
#pragma unroll
      for (int piece = 0; piece < 4; ++piece) {
        tmem_ld32(trow + sb * 128 + piece * 32, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float e[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int jj = 2 * j + h;
            const int key = key0 + piece * 32 + jj;
            float pe = 0.f;
            if (m_c != -INFINITY && key <= limit && key < k1)
              pe = bf16_round(exp2f(__uint_as_float(v[jj]) * p.scale_log2 - m_c));
            e[h] = pe;
            l_c += pe;
          }
          pk[j] = pack_bf16x2(e[0], e[1]);
        }
        // keys piece*32 .. +31 -> K-block piece/2, 16-B chunks (piece%2)*4 .. +3
        uint8_t* base = sP + (piece >> 1) * 16384u;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          *reinterpret_cast<uint4*>(base + sw128_offset(r, (piece & 1) * 4 + q4)) =
              make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&bar_s_free[sb]);
      fence_async_smem();
      mbar_arrive(&bar_p_full);
      m_prev = m_c;
      l_prev = l_c;
    }
    if (ok) ok = mbar_wait(&bar_o_full, (nchunks - 1) & 1);
    tc_fence_after();
    merge_o(m_prev, l_prev);

    if (valid_row) {
      if (n_splits == 1) {
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(
            p.out + ((static_cast<size_t>(b) * p.nq + t) * p.Hq + kvh * VF_G + g) * VF_D);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          uint4 w;
          w.x = pack_bf16x2(acc[8 * c + 0] * inv, acc[8 * c + 1] * inv);
          w.y = pack_bf16x2(acc[8 * c + 2] * inv, acc[8 * c + 3] * inv);
          w.z = pack_bf16x2(acc[8 * c + 4] * inv, acc[8 * c + 5] * inv);
          w.w = pack_bf16x2(acc[8 * c + 6] * inv, acc[8 * c + 7] * inv);
          dst[c] = w;
        }
        if (p.lse != nullptr)
          p.lse[(static_cast<size_t>(b) * p.nq + t) * p.Hq + kvh * VF_G + g] =
              l_run > 0.f ? (m_run + log2f(l_run)) * 0.69314718055994530942f : -INFINITY;
      } else {
        const size_t slot = ((static_cast<size_t>(b) * p.Hkv + kvh) * p.max_splits + split) * 128 + r;
        float4* dst = reinterpret_cast<float4*>(p.ws_o + slot * VF_D);
#pragma unroll
        for (int c = 0; c < 32; ++c) dst[c] = make_float4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
        p.ws_ml[slot * 2 + 0] = m_run;
        p.ws_ml[slot * 2 + 1] = l_run;
      }
    }
  }

  // ---------------- teardown + cross-split merge ----------------
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (n_splits == 1) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_ticket = atomicAdd(&p.counters[b * p.Hkv + kvh], 1);
  __syncthreads();
  if (s_ticket != n_splits - 1) return;
  __threadfence();
  const size_t slot0 = (static_cast<size_t>(b) * p.Hkv + kvh) * p.max_splits * 128;
  for (int idx = tid; idx < nrows * VF_D; idx += VF_THREADS) {
    const int r = idx / VF_D, d = idx % VF_D;
    float m = -INFINITY, l = 0.f, a = 0.f;
    for (int s = 0; s < n_splits; ++s) {
      const size_t sl = slot0 + static_cast<size_t>(s) * 128 + r;
      const float ms = __ldcg(&p.ws_ml[sl * 2]);
      const float ls = __ldcg(&p.ws_ml[sl * 2 + 1]);
      const float os = __ldcg(&p.ws_o[sl * VF_D + d]);
      if (ms == -INFINITY) continue;
      if (m == -INFINITY) {
        m = ms;
        l = ls;
        a = os;
        continue;
      }
      const float mn = fmaxf(m, ms);
      const float x = exp2f(m - mn), y = exp2f(ms - mn);
      a = a * x + os * y;
      l = l * x + ls * y;
      m = mn;
    }
    const int t = r / VF_G, g = r % VF_G;
    const float inv = l > 0.f ? 1.f / l : 0.f;
    p.out[((static_cast<size_t>(b) * p.nq + t) * p.Hq + kvh * VF_G + g) * VF_D + d] = __float2bfloat16_rn(a * inv);
    if (d == 0 && p.lse != nullptr)
      p.lse[(static_cast<size_t>(b) * p.nq + t) * p.Hq + kvh * VF_G + g] =
          l > 0.f ? (m + log2f(l)) * 0.69314718055994530942f : -INFINITY;
  }
  if (tid == 0) p.counters[b * p.Hkv + kvh] = 0;
}

}  // namespace stdb

// ---------------------------------------------------------------------------
// host: tensor maps and C ABI
// ---------------------------------------------------------------------------
typedef CUresult (*PFN_tmapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                        const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                        CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                        CUtensorMapFloatOOBfill);

static PFN_tmapEncodeTiled tmap_encoder() {
  static PFN_tmapEncodeTiled fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_tmapEncodeTiled>(ptr);
  }
  return fn;
}

// 2-D bf16 tensor [rows, cols] (row pitch = cols*2 bytes), box = box_cols x box_rows,
// 128-byte swizzle.  box_cols*2 must be 128.
static int make_tmap_bf16_2d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t row_pitch_bytes,
                             uint32_t box_cols, uint32_t box_rows) {
  PFN_tmapEncodeTiled enc = tmap_encoder();
  if (enc == nullptr) return 3;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 4;
}

extern "C" size_t std_verify_attn_workspace_bytes(int B, int Hkv, int cap) {
  const size_t max_splits = (cap + stdb::VF_SPLIT - 1) / stdb::VF_SPLIT;
  const size_t n = static_cast<size_t>(B) * Hkv;
  size_t bytes = ((n * 4 + 255) / 256) * 256;
  bytes += n * max_splits * 128 * 2 * 4;
  bytes = ((bytes + 255) / 256) * 256;
  bytes += n * max_splits * 128 * stdb::VF_D * 4;
  return bytes;
}

extern "C" int std_verify_attn(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens,
                               int len_offset, int nq, int causal, int B, int Hq, int Hkv, int D, int cap, void* out,
                               float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  if (D != stdb::VF_D || Hq != Hkv * stdb::VF_G || nq < 1 || stdb::VF_G * nq > 128 || B <= 0 || cap <= 0) return 1;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || lens == nullptr || out == nullptr) return 1;
  if (((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(q)) &
       15) != 0)
    return 1;
  if (workspace == nullptr || workspace_bytes < std_verify_attn_workspace_bytes(B, Hkv, cap)) return 5;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(stdb::verify_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, stdb::VF_SMEM) !=
        cudaSuccess)
      return 3;
    attr_set = true;
  }
  CUtensorMap tk, tv;
  const uint64_t rows = static_cast<uint64_t>(B) * Hkv * cap;
  int rc = make_tmap_bf16_2d(&tk, k_cache, rows, 128, 256, 64, 128);
  if (rc == 0) rc = make_tmap_bf16_2d(&tv, v_cache, rows, 128, 256, 64, 128);
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
  p.lse = lse;
  p.max_splits = (cap + stdb::VF_SPLIT - 1) / stdb::VF_SPLIT;
  const size_t n = static_cast<size_t>(B) * Hkv;
  char* ws = static_cast<char*>(workspace);
  p.counters = reinterpret_cast<int*>(ws);
  size_t off = ((n * 4 + 255) / 256) * 256;
  p.ws_ml = reinterpret_cast<float*>(ws + off);
  off += n * p.max_splits * 128 * 2 * 4;
  off = ((off + 255) / 256) * 256;
  p.ws_o = reinterpret_cast<float*>(ws + off);
  dim3 grid(p.max_splits, Hkv, B);
  stdb::verify_attn_kernel<<<grid, stdb::VF_THREADS, stdb::VF_SMEM, static_cast<cudaStream_t>(stream)>>>(tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
