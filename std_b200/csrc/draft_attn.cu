// draft_attn.cu -- (b) sparse GQA draft attention, q_len = 1.
//
// Replaces the reference's sparse draft attention
//   std_qwen25vl.py:406-417  F.scaled_dot_product_attention(q, k, v, enable_gqa=True)
//   triton_attention.py:13-112  _gqa_single_query_kernel (one program per q head)
// over the compacted sparse cache (no mask: the draft query sees every cached
// key, std_qwen25vl.py:400-417).
//
// Design (HBM-bound, ~7 flop/B): split-KV flash-decoding.
//   grid = (max_splits, Hkv, B); one CTA = one chunk of CHUNK keys of one
//   (request, KV head) and all G = 7 query heads of that group, so every K/V
//   byte is read from HBM exactly once (the Triton kernel re-reads each KV head
//   for each of its 7 query heads).  The chunk's K and V rows are contiguous
//   in the cache ([B, Hkv, cap, D]) and arrive by two cp.async.bulk copies.
//   The number of live splits comes from the device-resident length, so the
//   launch is graph-capturable while lengths change between replays.
//   Each CTA writes (m, l, O) partials; the last CTA of a (request, head)
//   (atomic ticket) merges the splits in split order and writes out / lse.
#include "common.cuh"

namespace stdb {

constexpr int DR_D = 128;
constexpr int DR_G = 7;
constexpr int DR_THREADS = 128;

struct DraftParams {
  const __nv_bfloat16* q;   // [B, Hq, D]
  const __nv_bfloat16* k;   // [B, Hkv, cap, D]
  const __nv_bfloat16* v;   // [B, Hkv, cap, D]
  const int32_t* lens;      // [B] device lengths
  int len_offset;           // live keys = lens[b] + len_offset
  int cap;
  int Hq, Hkv;
  float scale_log2;         // (1/sqrt(D)) * log2(e)
  __nv_bfloat16* out;       // [B, Hq, D]
  float* lse;               // [B, Hq] natural-log LSE, may be null
  int* counters;            // [B, Hkv] zero-initialised tickets
  float* ws_ml;             // [B, Hkv, max_splits, G, 2]
  float* ws_o;              // [B, Hkv, max_splits, G, D]
  int max_splits;
};

template <int CHUNK>
__global__ void __launch_bounds__(DR_THREADS) draft_attn_kernel(const DraftParams p) {
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int L = p.lens[b] + p.len_offset;
  if (L > p.cap || L < 0) {
    if (split == 0 && tid == 0) std_set_error(STD_DEVERR_LENGTH);
    L = L < 0 ? 0 : p.cap;
  }
  const int n_splits = (L + CHUNK - 1) / CHUNK;
  if (split >= n_splits || split >= p.max_splits) return;
  const int k0 = split * CHUNK;
  const int nk = min(CHUNK, L - k0);

  __shared__ __align__(128) __nv_bfloat16 sK[CHUNK * DR_D];
  __shared__ __align__(128) __nv_bfloat16 sV[CHUNK * DR_D];
  __shared__ float sQ[DR_G][DR_D];
  __shared__ float sP[DR_G][CHUNK];
  __shared__ float sM[DR_G], sL[DR_G];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int s_ticket;

  const size_t head_off = (static_cast<size_t>(b) * p.Hkv + kvh) * p.cap;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t bytes = static_cast<uint32_t>(nk) * DR_D * 2;
    mbar_arrive_expect_tx(&bar, 2 * bytes);
    bulk_load(sK, p.k + (head_off + k0) * DR_D, bytes, &bar);
    bulk_load(sV, p.v + (head_off + k0) * DR_D, bytes, &bar);
  }
  // q for the G heads of this group (fp32 in smem)
  for (int i = tid; i < DR_G * DR_D; i += DR_THREADS) {
    const int g = i / DR_D, d = i % DR_D;
    sQ[g][d] = __bfloat162float(p.q[(static_cast<size_t>(b) * p.Hq + kvh * DR_G + g) * DR_D + d]);
  }
  __syncthreads();
  const bool loaded = mbar_wait(&bar, 0);

  // ---- scores: 8 lanes per key, 16 d-elements per lane ----
  {
    const int sub = lane >> 3;   // key slot within the warp (0..3)
    const int part = lane & 7;   // d segment [16*part, 16*part+16)
    float qr[DR_G][16];
#pragma unroll
    for (int g = 0; g < DR_G; ++g)
#pragma unroll
      for (int j = 0; j < 16; ++j) qr[g][j] = sQ[g][part * 16 + j];
    for (int kb = warp * 4 + sub; kb < CHUNK; kb += 16) {
      float acc[DR_G];
#pragma unroll
      for (int g = 0; g < DR_G; ++g) acc[g] = 0.f;
      if (kb < nk) {
        const uint4* kr = reinterpret_cast<const uint4*>(sK + kb * DR_D + part * 16);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint4 u = kr[h];
          const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float2 f = __bfloat1622float2(e[j]);
#pragma unroll
            for (int g = 0; g < DR_G; ++g) {
              acc[g] = fmaf(qr[g][h * 8 + 2 * j], f.x, acc[g]);
              acc[g] = fmaf(qr[g][h * 8 + 2 * j + 1], f.y, acc[g]);
            }
          }
        }
      }
#pragma unroll
      for (int g = 0; g < DR_G; ++g) {
        float v = acc[g];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        if (part == 0) sP[g][kb] = (kb < nk && loaded) ? v * p.scale_log2 : -INFINITY;
      }
    }
  }
  __syncthreads();

  // ---- per-head softmax over the chunk (log2 domain) ----
  for (int g = warp; g < DR_G; g += 4) {
    float m = -INFINITY;
    for (int j = lane; j < CHUNK; j += 32) m = fmaxf(m, sP[g][j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < CHUNK; j += 32) {
      const float e = (m == -INFINITY) ? 0.f : exp2f(sP[g][j] - m);
      sP[g][j] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      sM[g] = m;
      sL[g] = l;
    }
  }
  __syncthreads();

  // ---- O = P V : thread = d ----
  float o[DR_G];
#pragma unroll
  for (int g = 0; g < DR_G; ++g) o[g] = 0.f;
  {
    const int d = tid;
    for (int j = 0; j < nk; ++j) {
      const float vv = __bfloat162float(sV[j * DR_D + d]);
#pragma unroll
      for (int g = 0; g < DR_G; ++g) o[g] = fmaf(sP[g][j], vv, o[g]);
    }
  }

  const int Hq = p.Hq;
  if (n_splits == 1) {
#pragma unroll
    for (int g = 0; g < DR_G; ++g) {
      const float l = sL[g];
      p.out[(static_cast<size_t>(b) * Hq + kvh * DR_G + g) * DR_D + tid] =
          __float2bfloat16_rn(l > 0.f ? o[g] / l : 0.f);
    }
    if (p.lse != nullptr && tid < DR_G) {
      const float l = sL[tid];
      p.lse[static_cast<size_t>(b) * Hq + kvh * DR_G + tid] =
          l > 0.f ? (sM[tid] + log2f(l)) * 0.69314718055994530942f : -INFINITY;
    }
    return;
  }

  // ---- multi-split: publish partials, last CTA merges ----
  const size_t slot = (static_cast<size_t>(b) * p.Hkv + kvh) * p.max_splits;
#pragma unroll
  for (int g = 0; g < DR_G; ++g) p.ws_o[((slot + split) * DR_G + g) * DR_D + tid] = o[g];
  if (tid < DR_G) {
    p.ws_ml[((slot + split) * DR_G + tid) * 2 + 0] = sM[tid];
    p.ws_ml[((slot + split) * DR_G + tid) * 2 + 1] = sL[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_ticket = atomicAdd(&p.counters[b * p.Hkv + kvh], 1);
  __syncthreads();
  if (s_ticket != n_splits - 1) return;
  __threadfence();
  const int d = tid;
#pragma unroll 1
  for (int g = 0; g < DR_G; ++g) {
    float m = -INFINITY, l = 0.f, acc = 0.f;
    for (int s = 0; s < n_splits; ++s) {
      const float ms = __ldcg(&p.ws_ml[((slot + s) * DR_G + g) * 2 + 0]);
      const float ls = __ldcg(&p.ws_ml[((slot + s) * DR_G + g) * 2 + 1]);
      const float os = __ldcg(&p.ws_o[((slot + s) * DR_G + g) * DR_D + d]);
      if (ms == -INFINITY) continue;
      if (m == -INFINITY) {
        m = ms;
        l = ls;
        acc = os;
        continue;
      }
      const float mn = fmaxf(m, ms);
      const float a = exp2f(m - mn), c = exp2f(ms - mn);
      acc = acc * a + os * c;
      l = l * a + ls * c;
      m = mn;
    }
    p.out[(static_cast<size_t>(b) * Hq + kvh * DR_G + g) * DR_D + d] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
    if (p.lse != nullptr && d == 0)
      p.lse[static_cast<size_t>(b) * Hq + kvh * DR_G + g] =
          l > 0.f ? (m + log2f(l)) * 0.69314718055994530942f : -INFINITY;
  }
  if (tid == 0) p.counters[b * p.Hkv + kvh] = 0;
}

}  // namespace stdb

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
static int draft_chunk_for(int B, int Hkv, int cap) {
  const long ctas64 = static_cast<long>(B) * Hkv * ((cap + 63) / 64);
  return ctas64 >= 2 * 148 ? 64 : 32;
}

extern "C" size_t std_draft_attn_workspace_bytes(int B, int Hq, int Hkv, int D, int cap) {
  (void)Hq;
  (void)D;
  const int chunk = draft_chunk_for(B, Hkv, cap);
  const size_t max_splits = (cap + chunk - 1) / chunk;
  const size_t n = static_cast<size_t>(B) * Hkv;
  size_t bytes = ((n * 4 + 255) / 256) * 256;
  bytes += n * max_splits * stdb::DR_G * 2 * 4;
  bytes = ((bytes + 255) / 256) * 256;
  bytes += n * max_splits * stdb::DR_G * stdb::DR_D * 4;
  return bytes;
}

extern "C" int std_draft_attn(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens,
                              int len_offset, int B, int Hq, int Hkv, int D, int cap, void* out, float* lse,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (D != stdb::DR_D || Hq != Hkv * stdb::DR_G || B <= 0 || cap <= 0) return 1;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || lens == nullptr || out == nullptr) return 1;
  if (workspace == nullptr || workspace_bytes < std_draft_attn_workspace_bytes(B, Hq, Hkv, D, cap)) return 5;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) return 1;
  const int chunk = draft_chunk_for(B, Hkv, cap);
  stdb::DraftParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k_cache);
  p.v = static_cast<const __nv_bfloat16*>(v_cache);
  p.lens = lens;
  p.len_offset = len_offset;
  p.cap = cap;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = (1.0f / sqrtf(static_cast<float>(D))) * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.max_splits = (cap + chunk - 1) / chunk;
  const size_t n = static_cast<size_t>(B) * Hkv;
  char* ws = static_cast<char*>(workspace);
  p.counters = reinterpret_cast<int*>(ws);
  size_t off = ((n * 4 + 255) / 256) * 256;
  p.ws_ml = reinterpret_cast<float*>(ws + off);
  off += n * p.max_splits * stdb::DR_G * 2 * 4;
  off = ((off + 255) / 256) * 256;
  p.ws_o = reinterpret_cast<float*>(ws + off);
  dim3 grid(p.max_splits, Hkv, B);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (chunk == 64)
    stdb::draft_attn_kernel<64><<<grid, stdb::DR_THREADS, 0, s>>>(p);
  else
    stdb::draft_attn_kernel<32><<<grid, stdb::DR_THREADS, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
