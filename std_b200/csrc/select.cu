// select.cu -- (a) prefill-time sparse KV selection.
//
// Replaces
//   modeling_qwen2_5_vl.py:966-995  custom scaled_dot_product_attention (the
//       output_attentions=True path): bf16 QK^T, bf16 scale, fp16 cast,
//       causal fp16 bias, fp16 softmax, materialised [Hq, T, P] weights;
//   std_qwen25vl.py:204-222         build_sparse_selection: fp32 sum over the
//       G query heads of a KV head and all text rows, index_select of the
//       visual columns, torch.topk, sort, .cpu();
//   std_qwen25vl.py:265-298         compact_sparse_prompt_cache: per head
//       unique(sorted(non_visual U topk)), gather into the sparse cache
//       (and copy_prompt_cache, :301-320, which the gather makes unnecessary).
//
// The arithmetic is the bit-exact specification in oracle/std_oracle.c:
//   logits  : acc = fmaf chain over d = 0..D-1 (fp32), s1 = bf16(acc),
//             s2 = bf16(s1 * scale), s3 = fp16(s2); masked -> -inf
//   row stat: m = max; l = 32-lane strided sums + xor butterfly 16..1
//   colsum  : fp32, g outer, t inner, p = fp16(std_exp(s3 - m) / l)
//   top-K   : K largest scores, ties to the lowest position, ascending output
// The logits are CUDA-core FMA (not tensor cores) because the fp32 fmaf order
// is what makes the scores reproducible bit for bit; they are materialised as
// fp16 (the same size the reference's own weights tensor has) and read twice.
#include "common.cuh"

namespace stdb {

// ------------------------------- logits ------------------------------------
constexpr int SL_RT = 128;  // rows per block
constexpr int SL_KT = 128;  // keys per block
constexpr int SL_DC = 16;   // d per smem stage

struct SelLogitsParams {
  const __nv_bfloat16* q;  // [T, Hq, D]
  const __nv_bfloat16* k;  // [Hkv, kstride, D]
  long long kstride;
  int T, Hq, Hkv, D, P, q_start, pstride;
  float scale;
  __half* logits;          // [Hq, T, pstride]
};

__global__ void __launch_bounds__(256) select_logits_kernel(const SelLogitsParams p) {
  const int kt = blockIdx.x, rt = blockIdx.y, kvh = blockIdx.z;
  const int G = p.Hq / p.Hkv;
  const int R = G * p.T;  // rows of this KV head: r = g*T + t
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;  // key group, row group
  __shared__ __align__(16) float sQ[SL_DC][SL_RT];
  __shared__ __align__(16) float sK[SL_DC][SL_KT];
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int lr = tid >> 1, lh = tid & 1;  // loader: row/key lr, 8 d-elements at 8*lh
  const int rrow = rt * SL_RT + lr;
  const int key = kt * SL_KT + lr;
  const __nv_bfloat16* qsrc = nullptr;
  if (rrow < R) {
    const int g = rrow / p.T, t = rrow % p.T;
    qsrc = p.q + (static_cast<size_t>(t) * p.Hq + kvh * G + g) * p.D;
  }
  const __nv_bfloat16* ksrc = (key < p.P) ? p.k + (static_cast<size_t>(kvh) * p.kstride + key) * p.D : nullptr;

  for (int d0 = 0; d0 < p.D; d0 += SL_DC) {
    {
      uint4 u = qsrc ? *reinterpret_cast<const uint4*>(qsrc + d0 + 8 * lh) : make_uint4(0, 0, 0, 0);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) sQ[8 * lh + j][lr] = __bfloat162float(e[j]);
      uint4 w = ksrc ? *reinterpret_cast<const uint4*>(ksrc + d0 + 8 * lh) : make_uint4(0, 0, 0, 0);
      const __nv_bfloat16* f = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
      for (int j = 0; j < 8; ++j) sK[8 * lh + j][lr] = __bfloat162float(f[j]);
    }
    __syncthreads();
#pragma unroll
    for (int d = 0; d < SL_DC; ++d) {
      const float4 a0 = *reinterpret_cast<const float4*>(&sQ[d][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&sQ[d][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&sK[d][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&sK[d][64 + tx * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(a[i], bb[j], acc[i][j]);
    }
    __syncthreads();
  }

  // thread owns rows {ty*4+i, 64+ty*4+i} and keys {tx*4+j, 64+tx*4+j}, i, j < 4
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = rt * SL_RT + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (r >= R) continue;
    const int g = r / p.T, t = r % p.T;
    const int lim = p.q_start + t;
    __half* dst = p.logits + (static_cast<size_t>(kvh * G + g) * p.T + t) * p.pstride;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      __align__(8) __half hv[4];
      const int pk0 = kt * SL_KT + half * 64 + tx * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float s1 = bf16_round(acc[i][half * 4 + j]);
        const float s2 = bf16_round(__fmul_rn(s1, p.scale));
        hv[j] = (pk0 + j > lim) ? __ushort_as_half(0xfc00u) : __float2half_rn(s2);
      }
      if (pk0 + 4 <= p.pstride) *reinterpret_cast<uint2*>(dst + pk0) = *reinterpret_cast<const uint2*>(hv);
    }
  }
}

// ------------------------------- row stats ---------------------------------
__global__ void __launch_bounds__(256) select_row_stats_kernel(const __half* logits, int rows, int P, int pstride,
                                                               float* row_m, float* row_l) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const __half* row = logits + static_cast<size_t>(warp) * pstride;
  float m = -INFINITY;
  for (int i = lane; i < P; i += 32) m = fmaxf(m, __half2float(row[i]));
  m = warp_max(m);
  float s = 0.f;
  for (int i = lane; i < P; i += 32) s = __fadd_rn(s, std_exp(__fsub_rn(__half2float(row[i]), m)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  if (lane == 0) {
    row_m[warp] = m;
    row_l[warp] = s;
  }
}

// ------------------------------- column sums -------------------------------
__global__ void __launch_bounds__(256) select_colsum_kernel(__half* logits, const float* row_m, const float* row_l,
                                                            int T, int Hq, int Hkv, int P, int pstride, float* scores,
                                                            int write_probs) {
  const int pcol = blockIdx.x * blockDim.x + threadIdx.x;
  const int kvh = blockIdx.y;
  if (pcol >= P) return;
  const int G = Hq / Hkv;
  float acc = 0.f;
  for (int g = 0; g < G; ++g) {
    const int h = kvh * G + g;
    for (int t = 0; t < T; ++t) {
      const int r = h * T + t;
      __half* ptr = logits + static_cast<size_t>(r) * pstride + pcol;
      const float e = std_exp(__fsub_rn(__half2float(*ptr), __ldg(&row_m[r])));
      const __half pr = __float2half_rn(__fdiv_rn(e, __ldg(&row_l[r])));
      acc = __fadd_rn(acc, __half2float(pr));
      if (write_probs) *ptr = pr;
    }
  }
  scores[static_cast<size_t>(kvh) * P + pcol] = acc;
}

// ------------------------------- top-K -------------------------------------
constexpr int TK_THREADS = 1024;

STD_DEV int block_exclusive_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = (lane < (blockDim.x >> 5)) ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  const int warp_prefix = warp > 0 ? s_warp[warp - 1] : 0;
  total = s_warp[(blockDim.x >> 5) - 1];
  __syncthreads();
  return warp_prefix + x - v;
}

__global__ void __launch_bounds__(TK_THREADS) topk_lowest_kernel(const float* scores, long long seg_stride,
                                                                 const int32_t* visual_pos, int V, int K,
                                                                 int32_t* out) {
  const int seg = blockIdx.x;
  const float* sc = scores + static_cast<size_t>(seg) * seg_stride;
  __shared__ int hist[256];
  __shared__ int s_warp[32];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ int s_need;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_need = K;
  }
  __syncthreads();
  for (int digit = 3; digit >= 0; --digit) {
    for (int i = tid; i < 256; i += TK_THREADS) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int i = tid; i < V; i += TK_THREADS) {
      const uint32_t key = order_key(sc[visual_pos[i]]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> (8 * digit)) & 255u], 1);
    }
    __syncthreads();
    if (tid == 0) {
      int need = s_need, cum = 0, chosen = 0;
      for (int bkt = 255; bkt >= 0; --bkt) {
        if (cum + hist[bkt] >= need) {
          chosen = bkt;
          need -= cum;
          break;
        }
        cum += hist[bkt];
      }
      s_need = need;
      s_prefix = prefix | (static_cast<uint32_t>(chosen) << (8 * digit));
      s_mask = mask | (255u << (8 * digit));
    }
    __syncthreads();
  }
  const uint32_t thr = s_prefix;
  const int need_eq = s_need;  // how many elements equal to thr are taken
  int eq_base = 0, out_base = 0;
  for (int base = 0; base < V; base += TK_THREADS) {
    const int i = base + tid;
    uint32_t key = 0;
    if (i < V) key = order_key(sc[visual_pos[i]]);
    const int gt = (i < V && key > thr) ? 1 : 0;
    const int eq = (i < V && key == thr) ? 1 : 0;
    int eq_tot;
    const int eq_rank = eq_base + block_exclusive_scan(eq, s_warp, eq_tot);
    const int take = gt || (eq && eq_rank < need_eq);
    int take_tot;
    const int slot = out_base + block_exclusive_scan(take, s_warp, take_tot);
    if (take && slot < K) out[static_cast<size_t>(seg) * K + slot] = visual_pos[i];
    eq_base += eq_tot;
    out_base += take_tot;
  }
}

// ------------------------------- compaction --------------------------------
STD_DEV int count_less(const int32_t* a, int n, int x) {  // a ascending
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < x)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

struct CompactParams {
  const __nv_bfloat16* dense;  // [layers, 2, B, Hkv, cap_d, D]
  __nv_bfloat16* sparse;       // [layers, 2, B, Hkv, cap_s, D]
  const int32_t* non_visual;   // [NV] ascending
  const int32_t* topk;         // [layers, Hkv, K] ascending per row
  int NV, K, B, b, Hkv, D, cap_d, cap_s, layers;
};

// one warp per (layer, head, output slot source element); copies the K and V rows
__global__ void __launch_bounds__(256) compact_gather_kernel(const CompactParams p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int kvh = blockIdx.y, layer = blockIdx.z;
  const int n = p.NV + p.K;
  if (warp >= n) return;
  const int32_t* tk = p.topk + (static_cast<size_t>(layer) * p.Hkv + kvh) * p.K;
  int pos, slot;
  if (warp < p.NV) {
    pos = p.non_visual[warp];
    slot = warp + count_less(tk, p.K, pos);
  } else {
    const int j = warp - p.NV;
    pos = tk[j];
    slot = j + count_less(p.non_visual, p.NV, pos);
  }
  if (pos < 0 || pos >= p.cap_d || slot >= p.cap_s) {
    if (lane == 0) std_set_error(STD_DEVERR_BOUNDS);
    return;
  }
  const int D8 = p.D / 8;  // uint4 per row
  for (int kv = 0; kv < 2; ++kv) {
    const size_t dhead = ((static_cast<size_t>(layer) * 2 + kv) * p.B + p.b) * p.Hkv + kvh;
    const uint4* src = reinterpret_cast<const uint4*>(p.dense + (dhead * p.cap_d + pos) * p.D);
    uint4* dst = reinterpret_cast<uint4*>(p.sparse + (dhead * p.cap_s + slot) * p.D);
    for (int i = lane; i < D8; i += 32) dst[i] = src[i];
  }
}

}  // namespace stdb

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
static int select_pstride(int P) { return (P + 7) & ~7; }  // multiple of 8 -> 4-key stores stay in the row

extern "C" size_t std_select_workspace_bytes(int T, int Hq, int P) {
  const size_t rows = static_cast<size_t>(Hq) * T;
  size_t bytes = rows * select_pstride(P) * 2;
  bytes = ((bytes + 255) / 256) * 256;
  bytes += 2 * ((rows * 4 + 255) / 256) * 256;
  return bytes;
}

// Scores of one layer (and, if probs_out is requested, the fp16 probabilities
// left in the workspace at [Hq, T, pstride] for the selection-branch output).
extern "C" int std_select_scores(const void* q_text, const void* k_cache, long long kstride, int T, int Hq, int Hkv,
                                 int D, int P, int q_start, float scale, float* scores, int write_probs,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  if (D % 16 != 0 || Hq % Hkv != 0 || T <= 0 || P <= 0 || q_start < 0 || q_start + T > P || kstride < P) return 1;
  if (workspace == nullptr || workspace_bytes < std_select_workspace_bytes(T, Hq, P)) return 5;
  if (((reinterpret_cast<uintptr_t>(q_text) | reinterpret_cast<uintptr_t>(k_cache)) & 15) != 0) return 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int pstride = select_pstride(P);
  const size_t rows = static_cast<size_t>(Hq) * T;
  char* ws = static_cast<char*>(workspace);
  __half* logits = reinterpret_cast<__half*>(ws);
  size_t off = ((rows * pstride * 2 + 255) / 256) * 256;
  float* row_m = reinterpret_cast<float*>(ws + off);
  off += ((rows * 4 + 255) / 256) * 256;
  float* row_l = reinterpret_cast<float*>(ws + off);

  stdb::SelLogitsParams lp;
  lp.q = static_cast<const __nv_bfloat16*>(q_text);
  lp.k = static_cast<const __nv_bfloat16*>(k_cache);
  lp.kstride = kstride;
  lp.T = T;
  lp.Hq = Hq;
  lp.Hkv = Hkv;
  lp.D = D;
  lp.P = P;
  lp.q_start = q_start;
  lp.pstride = pstride;
  lp.scale = scale;
  lp.logits = logits;
  const int G = Hq / Hkv;
  dim3 g1((P + stdb::SL_KT - 1) / stdb::SL_KT, (G * T + stdb::SL_RT - 1) / stdb::SL_RT, Hkv);
  count_launch();
  stdb::select_logits_kernel<<<g1, 256, 0, s>>>(lp);
  count_launch();
  stdb::select_row_stats_kernel<<<(static_cast<unsigned>(rows) * 32 + 255) / 256, 256, 0, s>>>(logits, rows, P,
                                                                                              pstride, row_m, row_l);
  dim3 g3((P + 255) / 256, Hkv);
  count_launch();
  stdb::select_colsum_kernel<<<g3, 256, 0, s>>>(logits, row_m, row_l, T, Hq, Hkv, P, pstride, scores, write_probs);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int std_select_probs_view(int T, int Hq, int P, long long* pstride_out) {
  if (T <= 0 || Hq <= 0 || P <= 0 || pstride_out == nullptr) return 1;
  *pstride_out = select_pstride(P);
  return 0;
}

extern "C" int std_topk_select(const float* scores, long long seg_stride, int n_seg, const int32_t* visual_pos, int V,
                               int K, int32_t* out, void* stream) {
  if (n_seg <= 0 || V <= 0 || K <= 0 || K > V || scores == nullptr || visual_pos == nullptr || out == nullptr) return 1;
  count_launch();
  stdb::topk_lowest_kernel<<<n_seg, stdb::TK_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(scores, seg_stride,
                                                                                             visual_pos, V, K, out);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int std_compact_gather(const void* dense_cache, void* sparse_cache, int layers, int B, int b, int Hkv, int D,
                                  int cap_dense, int cap_sparse, const int32_t* non_visual, int NV,
                                  const int32_t* topk, int K, void* stream) {
  if (layers <= 0 || B <= 0 || b < 0 || b >= B || Hkv <= 0 || D % 8 != 0 || NV < 0 || K <= 0) return 1;
  if (NV + K > cap_sparse) return 2;
  stdb::CompactParams p;
  p.dense = static_cast<const __nv_bfloat16*>(dense_cache);
  p.sparse = static_cast<__nv_bfloat16*>(sparse_cache);
  p.non_visual = non_visual;
  p.topk = topk;
  p.NV = NV;
  p.K = K;
  p.B = B;
  p.b = b;
  p.Hkv = Hkv;
  p.D = D;
  p.cap_d = cap_dense;
  p.cap_s = cap_sparse;
  p.layers = layers;
  const int n = NV + K;
  dim3 grid((n * 32 + 255) / 256, Hkv, layers);
  count_launch();
  stdb::compact_gather_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
