// draft_attn.cu -- (b) sparse GQA draft attention, q_len = 1.
//
// Replaces the reference's sparse draft attention
//   std_qwen25vl.py:406-417  F.scaled_dot_product_attention(q, k, v, enable_gqa=True)
//   triton_attention.py:13-112  _gqa_single_query_kernel (one program per q head)
// over the compacted sparse cache (no mask: the draft query sees every cached
// key, std_qwen25vl.py:400-417).
//
// Design (HBM-bound, ~7 flop/B, and at batch 1 latency-bound): split-KV
// flash-decoding inside one thread-block cluster per (request, KV head).
//   grid = (DR_CLUSTER, Hkv, B), cluster = (DR_CLUSTER, 1, 1).  CTA rank i
//   streams keys [i*per, (i+1)*per) of the request's live length through a
//   two-stage cp.async.bulk ring (K and V rows are contiguous in the
//   [B, Hkv, cap, D] cache), computing all G = 7 query heads of the group with
//   an online softmax, so every K/V byte is read from HBM once (the Triton
//   kernel re-reads each KV head for each of its 7 query heads).  The CTAs of
//   the cluster then combine their (m, l, O) partials through distributed
//   shared memory -- four ranks each read a quarter of the outputs from all
//   eight ranks' smem -- so there is one launch,
//   no global scratch and no second kernel.  Lengths come from device memory,
//   so the launch is graph-capturable while they change between replays.
#include <cooperative_groups.h>

#include "common.cuh"

namespace stdb {

constexpr int DR_D = 128;
constexpr int DR_G = 7;
constexpr int DR_THREADS = 256;
constexpr int DR_SUB = 64;      // keys per pipeline stage
constexpr int DR_CLUSTER = 8;   // CTAs per (request, KV head)
constexpr uint32_t DR_STAGE_BYTES = DR_SUB * DR_D * 2;  // one K (or V) stage
constexpr uint32_t DR_SMEM = 4 * DR_STAGE_BYTES + 128;  // 2 stages x (K, V) + alignment

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
};

__global__ void __cluster_dims__(DR_CLUSTER, 1, 1) __launch_bounds__(DR_THREADS, 2)
    draft_attn_kernel(const DraftParams p) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  extern __shared__ uint8_t dsmem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem_raw) + 127) & ~uintptr_t(127));
  __nv_bfloat16* sK[2] = {reinterpret_cast<__nv_bfloat16*>(sbase),
                          reinterpret_cast<__nv_bfloat16*>(sbase + DR_STAGE_BYTES)};
  __nv_bfloat16* sV[2] = {reinterpret_cast<__nv_bfloat16*>(sbase + 2 * DR_STAGE_BYTES),
                          reinterpret_cast<__nv_bfloat16*>(sbase + 3 * DR_STAGE_BYTES)};
  __shared__ float sQ[DR_G][DR_D];
  __shared__ float sS[DR_G][DR_SUB];
  __shared__ float sAlpha[DR_G];
  // partials published to the cluster
  __shared__ float pm[DR_G], pl[DR_G];
  __shared__ __align__(16) float po[DR_G][DR_D];
  __shared__ __align__(8) uint64_t bar[2];

  int L = p.lens[b] + p.len_offset;
  if (L > p.cap || L < 0) {
    if (rank == 0 && tid == 0) std_set_error(STD_DEVERR_LENGTH);
    L = L < 0 ? 0 : p.cap;
  }
  int per = (L + DR_CLUSTER - 1) / DR_CLUSTER;
  per = (per + 15) & ~15;
  const int k0 = min(L, rank * per);
  const int k1 = min(L, k0 + per);
  const int nsub = (k1 - k0 + DR_SUB - 1) / DR_SUB;
  const size_t head_off = (static_cast<size_t>(b) * p.Hkv + kvh) * p.cap;

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int i) {
    const int st = i & 1;
    const int a = k0 + i * DR_SUB;
    const uint32_t bytes = static_cast<uint32_t>(min(DR_SUB, k1 - a)) * DR_D * 2;
    mbar_arrive_expect_tx(&bar[st], 2 * bytes);
    bulk_load(sK[st], p.k + (head_off + a) * DR_D, bytes, &bar[st]);
    bulk_load(sV[st], p.v + (head_off + a) * DR_D, bytes, &bar[st]);
  };
  if (tid == 0) {
    if (nsub > 0) issue(0);
    if (nsub > 1) issue(1);
  }
  for (int i = tid; i < DR_G * DR_D; i += DR_THREADS) {
    const int g = i / DR_D, d = i % DR_D;
    sQ[g][d] = __bfloat162float(p.q[(static_cast<size_t>(b) * p.Hq + kvh * DR_G + g) * DR_D + d]);
  }
  __syncthreads();

  // scores: 16 lanes per key, lane part owns dims [8*part, 8*part+8) (16 B of
  // the 256-B key row: a half-warp reads one row without bank conflicts)
  const int slot = lane >> 4, part = lane & 15;
  float qr[DR_G][8];
#pragma unroll
  for (int g = 0; g < DR_G; ++g)
#pragma unroll
    for (int j = 0; j < 8; ++j) qr[g][j] = sQ[g][part * 8 + j];
  // PV: thread owns dims (2*dp, 2*dp+1) of heads hg and hg+4
  const int dp = tid & 63, hg = tid >> 6;
  float o[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  float m_run = -INFINITY, l_run = 0.f;  // meaningful in warp g's lanes (softmax of head g)
  bool ok = true;

  for (int i = 0; i < nsub; ++i) {
    const int st = i & 1;
    const int nk = min(DR_SUB, k1 - (k0 + i * DR_SUB));
    if (ok) ok = mbar_wait(&bar[st], (i >> 1) & 1);
#pragma unroll 1
    for (int kb = warp * 2 + slot; kb < DR_SUB; kb += 16) {
      float acc[DR_G];
#pragma unroll
      for (int g = 0; g < DR_G; ++g) acc[g] = 0.f;
      if (kb < nk) {
        const uint4 u = *reinterpret_cast<const uint4*>(sK[st] + kb * DR_D + part * 8);
        const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(e[j]);
#pragma unroll
          for (int g = 0; g < DR_G; ++g) {
            acc[g] = fmaf(qr[g][2 * j], f.x, acc[g]);
            acc[g] = fmaf(qr[g][2 * j + 1], f.y, acc[g]);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < DR_G; ++g) {
        float x = acc[g];
        x += __shfl_xor_sync(0xffffffffu, x, 1);
        x += __shfl_xor_sync(0xffffffffu, x, 2);
        x += __shfl_xor_sync(0xffffffffu, x, 4);
        x += __shfl_xor_sync(0xffffffffu, x, 8);
        if (part == 0) sS[g][kb] = (kb < nk && ok) ? x * p.scale_log2 : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax, warp g owns head g
    if (warp < DR_G) {
      const int g = warp;
      const float a0 = sS[g][lane], a1 = sS[g][lane + 32];
      const float mc = warp_max(fmaxf(a0, a1));
      const float mn = fmaxf(m_run, mc);
      const float alpha = (m_run == -INFINITY) ? 0.f : exp2f(m_run - mn);
      const float e0 = (mn == -INFINITY) ? 0.f : exp2f(a0 - mn);
      const float e1 = (mn == -INFINITY) ? 0.f : exp2f(a1 - mn);
      sS[g][lane] = e0;
      sS[g][lane + 32] = e1;
      l_run = l_run * alpha + warp_sum(e0 + e1);
      m_run = mn;
      if (lane == 0) sAlpha[g] = alpha;
    }
    __syncthreads();
    // O = O * alpha + P V
    {
      const bool h1 = hg + 4 < DR_G;
      const float a0 = sAlpha[hg], a1 = h1 ? sAlpha[hg + 4] : 0.f;
      o[0][0] *= a0;
      o[0][1] *= a0;
      o[1][0] *= a1;
      o[1][1] *= a1;
      const __nv_bfloat162* vcol = reinterpret_cast<const __nv_bfloat162*>(sV[st]) + dp;
      const float* p0 = sS[hg];
      const float* p1 = sS[h1 ? hg + 4 : hg];
#pragma unroll 4
      for (int j = 0; j < nk; ++j) {
        const float2 vv = __bfloat1622float2(vcol[j * (DR_D / 2)]);
        const float w0 = p0[j], w1 = p1[j];
        o[0][0] = fmaf(w0, vv.x, o[0][0]);
        o[0][1] = fmaf(w0, vv.y, o[0][1]);
        o[1][0] = fmaf(w1, vv.x, o[1][0]);
        o[1][1] = fmaf(w1, vv.y, o[1][1]);
      }
    }
    __syncthreads();  // stage st and sS free
    if (tid == 0 && i + 2 < nsub) issue(i + 2);
  }

  // publish this CTA's partial to the cluster
  po[hg][2 * dp] = o[0][0];
  po[hg][2 * dp + 1] = o[0][1];
  if (hg + 4 < DR_G) {
    po[hg + 4][2 * dp] = o[1][0];
    po[hg + 4][2 * dp + 1] = o[1][1];
  }
  if (warp < DR_G && lane == 0) {
    pm[warp] = (l_run > 0.f) ? m_run : -INFINITY;
    pl[warp] = l_run;
  }
  cluster.sync();
  // Combine: output element idx = rank * DR_THREADS + tid (ranks 0..3 cover the
  // 7 x 128 outputs); the 8 ranks' partials are read over DSMEM, loads unrolled.
  {
    const int idx = rank * DR_THREADS + tid;
    if (idx < DR_G * DR_D) {
      const int g = idx / DR_D, d = idx % DR_D;
      float mr[DR_CLUSTER], lr[DR_CLUSTER], orr[DR_CLUSTER];
#pragma unroll
      for (int r = 0; r < DR_CLUSTER; ++r) {
        mr[r] = *cluster.map_shared_rank(&pm[g], r);
        lr[r] = *cluster.map_shared_rank(&pl[g], r);
        orr[r] = *cluster.map_shared_rank(&po[g][d], r);
      }
      float m = -INFINITY;
#pragma unroll
      for (int r = 0; r < DR_CLUSTER; ++r) m = fmaxf(m, mr[r]);
      float l = 0.f, acc = 0.f;
#pragma unroll
      for (int r = 0; r < DR_CLUSTER; ++r) {
        if (mr[r] == -INFINITY) continue;
        const float w = exp2f(mr[r] - m);
        l += w * lr[r];
        acc += w * orr[r];
      }
      p.out[(static_cast<size_t>(b) * p.Hq + kvh * DR_G + g) * DR_D + d] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
      if (d == 0 && p.lse != nullptr)
        p.lse[static_cast<size_t>(b) * p.Hq + kvh * DR_G + g] =
            l > 0.f ? (m + log2f(l)) * 0.69314718055994530942f : -INFINITY;
    }
  }
  cluster.sync();  // keep every CTA's smem alive until the others have read it
}

}  // namespace stdb

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" size_t std_draft_attn_workspace_bytes(int B, int Hq, int Hkv, int D, int cap) {
  (void)B;
  (void)Hq;
  (void)Hkv;
  (void)D;
  (void)cap;
  return 0;  // partials are combined in distributed shared memory
}

extern "C" int std_draft_attn(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens,
                              int len_offset, int B, int Hq, int Hkv, int D, int cap, void* out, float* lse,
                              void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (D != stdb::DR_D || Hq != Hkv * stdb::DR_G || B <= 0 || cap <= 0) return 1;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || lens == nullptr || out == nullptr) return 1;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) return 1;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(stdb::draft_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, stdb::DR_SMEM) !=
            cudaSuccess ||
        cudaFuncSetAttribute(stdb::draft_attn_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return 3;
    attr_set = true;
  }
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
  dim3 grid(stdb::DR_CLUSTER, Hkv, B);
  stdb::draft_attn_kernel<<<grid, stdb::DR_THREADS, stdb::DR_SMEM, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
