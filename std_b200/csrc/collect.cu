// collect.cu -- verification-guided visual relevance (collector v1).
//
// Replaces RuntimeVerificationCollector._hook (dynamic_selection.py:290-308),
// which during each dense verify forward turns every layer's verify queries
// into a per-(KV head) visual relevance:
//   q_kv[t]  = mean over the G query heads of the group of q[t]   (fp32)
//   l[t, v]  = q_kv[t] . k[vis[v]] / sqrt(D)                      (fp32)
//   A[v]     = sum_t softmax_v(l[t, :])[v]                        (fp32)
// for the verify rows t < nq and the visual keys vis[0..V) of the dense
// cache.  Everything is fp32, as in the reference (which computes it with
// torch fp32 matmul + softmax on the gathered keys).
//
// Two kernels per (request, KV head, block of 256 visual keys):
//   collect_logits_kernel  stages the block's K rows (coalesced 16-byte loads,
//       XOR-swizzled so each key's row is read without bank conflicts), one
//       thread per key computes its nq dot products with q_kv (held in shared
//       memory), writes l[t, v] to scratch and the block's per-row max and
//       sum of exp to a partial table;
//   collect_finish_kernel  merges the partials of every block in block order
//       (max first, then rescaled sums) and writes A[v] = sum_t exp(l[t,v] -
//       M_t) / L_t to rel_out[b][h][vis[v]] (a row indexed by prompt position).
// The row maxima and sums are combined in a fixed order, so the result does
// not depend on scheduling.
#include "common.cuh"

namespace stdb {

constexpr int CL_KEYS = 256;    // visual keys per block (one per thread)
constexpr int CL_D = 128;
constexpr int CL_MAXQ = 32;     // verify rows per call

struct CollectParams {
  const __nv_bfloat16* q;       // [B, nq, Hq, D]
  const __nv_bfloat16* k;       // [B, Hkv, cap, D]
  const int32_t* vis;           // [V] key positions
  int B, nq, Hq, Hkv, cap, V, nblk;
  float scale;                  // 1/sqrt(D)
  float* logits;                // scratch [B, Hkv, nq, V]
  float* part;                  // scratch [B, Hkv, nblk, nq, 2] (max, sum of exp)
  float* rel;                   // out [B, Hkv, rel_stride]
  long long rel_stride;
};

__global__ void __launch_bounds__(CL_KEYS) collect_logits_kernel(const CollectParams p) {
  extern __shared__ uint8_t cl_smem_raw[];
  uint4* sK = reinterpret_cast<uint4*>(cl_smem_raw);                   // [CL_KEYS][16] swizzled
  float* sQ = reinterpret_cast<float*>(cl_smem_raw + CL_KEYS * 256);   // [nq][CL_D]
  __shared__ float s_red[CL_KEYS / 32][CL_MAXQ];
  pdl_wait();
  pdl_launch_dependents();
  const int blk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.Hq / p.Hkv;
  // q_kv: fp32 mean of the group's query heads (sum in head order, then / G)
  for (int i = tid; i < p.nq * CL_D; i += CL_KEYS) {
    const int t = i / CL_D, d = i % CL_D;
    const __nv_bfloat16* qr = p.q + ((static_cast<size_t>(b) * p.nq + t) * p.Hq + h * G) * CL_D + d;
    float s = 0.f;
    for (int g = 0; g < G; ++g) s += __bfloat162float(qr[g * CL_D]);
    sQ[i] = s / static_cast<float>(G);
  }
  // this block's K rows: chunk c of key j at slot j*16 + (c ^ (j & 15))
  const int v0 = blk * CL_KEYS;
  const int nk = min(CL_KEYS, p.V - v0);
  for (int i = tid; i < nk * 16; i += CL_KEYS) {
    const int j = i >> 4, c = i & 15;
    int pos = p.vis[v0 + j];
    if (pos < 0 || pos >= p.cap) {
      if (c == 0) std_set_error(STD_DEVERR_BOUNDS);
      pos = 0;
    }
    sK[j * 16 + (c ^ (j & 15))] =
        reinterpret_cast<const uint4*>(p.k + ((static_cast<size_t>(b) * p.Hkv + h) * p.cap + pos) * CL_D)[c];
  }
  __syncthreads();
  float acc[CL_MAXQ];
#pragma unroll
  for (int t = 0; t < CL_MAXQ; ++t) acc[t] = 0.f;
  const int j = tid;
  if (j < nk) {
    for (int c = 0; c < 16; ++c) {
      const uint4 u = sK[j * 16 + (c ^ (j & 15))];
      const __nv_bfloat162* hk = reinterpret_cast<const __nv_bfloat162*>(&u);
      float kv[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(hk[e]);
        kv[2 * e] = f.x;
        kv[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int t = 0; t < CL_MAXQ; ++t) {
        if (t >= p.nq) break;
        const float* qd = sQ + t * CL_D + c * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[t] = fmaf(qd[e], kv[e], acc[t]);
      }
    }
  }
  float* lg = p.logits + (static_cast<size_t>(b) * p.Hkv + h) * p.nq * p.V;
  float* pt = p.part + ((static_cast<size_t>(b) * p.Hkv + h) * p.nblk + blk) * p.nq * 2;
  for (int t = 0; t < p.nq; ++t) {
    const float l = acc[t] * p.scale;
    if (j < nk) lg[static_cast<size_t>(t) * p.V + v0 + j] = l;
    // block max, then block sum of exp(l - max), in a fixed order
    float m = j < nk ? l : -INFINITY;
    m = warp_max(m);
    if (lane == 0) s_red[warp][t] = m;
    __syncthreads();
    float bm = -INFINITY;
    for (int w = 0; w < CL_KEYS / 32; ++w) bm = fmaxf(bm, s_red[w][t]);
    __syncthreads();
    float e = j < nk ? expf(l - bm) : 0.f;
    e = warp_sum(e);
    if (lane == 0) s_red[warp][t] = e;
    __syncthreads();
    if (tid == 0) {
      float bs = 0.f;
      for (int w = 0; w < CL_KEYS / 32; ++w) bs += s_red[w][t];
      pt[t * 2 + 0] = bm;
      pt[t * 2 + 1] = bs;
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(CL_KEYS) collect_finish_kernel(const CollectParams p) {
  __shared__ float s_M[CL_MAXQ], s_invL[CL_MAXQ];
  pdl_wait();
  pdl_launch_dependents();
  const int blk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const float* pt = p.part + (static_cast<size_t>(b) * p.Hkv + h) * p.nblk * p.nq * 2;
  if (tid < p.nq) {
    const int t = tid;
    float M = -INFINITY;
    for (int i = 0; i < p.nblk; ++i) M = fmaxf(M, pt[(i * p.nq + t) * 2]);
    float L = 0.f;
    for (int i = 0; i < p.nblk; ++i) L += pt[(i * p.nq + t) * 2 + 1] * expf(pt[(i * p.nq + t) * 2] - M);
    s_M[t] = M;
    s_invL[t] = L > 0.f ? 1.f / L : 0.f;
  }
  __syncthreads();
  const int v = blk * CL_KEYS + tid;
  if (v >= p.V) return;
  const float* lg = p.logits + (static_cast<size_t>(b) * p.Hkv + h) * p.nq * p.V;
  float a = 0.f;
  for (int t = 0; t < p.nq; ++t) a += expf(lg[static_cast<size_t>(t) * p.V + v] - s_M[t]) * s_invL[t];
  int pos = p.vis[v];
  if (pos < 0 || pos >= p.rel_stride) return;
  p.rel[(static_cast<size_t>(b) * p.Hkv + h) * p.rel_stride + pos] = a;
}

}  // namespace stdb

extern "C" size_t std_collect_workspace_bytes(int B, int Hkv, int nq, int V) {
  if (B <= 0 || Hkv <= 0 || nq <= 0 || V <= 0) return 0;
  const size_t nblk = (V + stdb::CL_KEYS - 1) / stdb::CL_KEYS;
  const size_t logits = static_cast<size_t>(B) * Hkv * nq * V * 4;
  const size_t part = static_cast<size_t>(B) * Hkv * nblk * nq * 2 * 4;
  return ((logits + 255) / 256) * 256 + part;
}

extern "C" int std_collect_relevance(const void* q, const void* k_cache, const int32_t* visual_pos, int V, int B,
                                     int nq, int Hq, int Hkv, int D, int cap, float* rel_out, long long rel_stride,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  if (q == nullptr || k_cache == nullptr || visual_pos == nullptr || rel_out == nullptr) return 1;
  if (D != stdb::CL_D || B <= 0 || Hkv <= 0 || Hq % Hkv != 0 || nq < 1 || nq > stdb::CL_MAXQ || V <= 0 || cap <= 0 ||
      rel_stride <= 0)
    return 1;
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache)) & 15) != 0) return 1;
  if (workspace == nullptr || workspace_bytes < std_collect_workspace_bytes(B, Hkv, nq, V)) return 5;
  stdb::CollectParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k_cache);
  p.vis = visual_pos;
  p.B = B;
  p.nq = nq;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.cap = cap;
  p.V = V;
  p.nblk = (V + stdb::CL_KEYS - 1) / stdb::CL_KEYS;
  p.scale = 1.0f / sqrtf(static_cast<float>(D));
  char* ws = static_cast<char*>(workspace);
  p.logits = reinterpret_cast<float*>(ws);
  const size_t logits = static_cast<size_t>(B) * Hkv * nq * V * 4;
  p.part = reinterpret_cast<float*>(ws + ((logits + 255) / 256) * 256);
  p.rel = rel_out;
  p.rel_stride = rel_stride;
  const size_t smem = stdb::CL_KEYS * 256 + static_cast<size_t>(nq) * stdb::CL_D * 4;
  static SmemGrant grant;
  if (ensure_smem(stdb::collect_logits_kernel, grant, smem) != 0) return 3;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(p.nblk, Hkv, B);
  if (launch_pdl(stdb::collect_logits_kernel, grid, dim3(stdb::CL_KEYS), smem, s, p) != cudaSuccess) return 4;
  return launch_pdl(stdb::collect_finish_kernel, grid, dim3(stdb::CL_KEYS), 0, s, p) == cudaSuccess ? 0 : 4;
}
