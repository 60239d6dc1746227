// merge.cu -- exact (O, LSE) merge of attention partials over disjoint key
// ranges: the exchange step of sequence-sharded verify.  The reference has no
// sequence parallelism (its long-context path preallocates a larger cache,
// kv_cache.py:104-105); this is the combine that makes a sharded verify equal
// to the unsharded one up to fp32 rounding.
#include "common.cuh"

namespace stdb {

// one warp per row: lse_max over parts, weights exp(lse_i - lse_max),
// out = sum_i w_i o_i / sum_i w_i, parts in index order.
__global__ void merge_partials_kernel(const __nv_bfloat16* o_parts, const float* lse_parts, int n_parts, int rows,
                                      int D, __nv_bfloat16* out, float* lse_out) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float mx = -INFINITY;
  for (int i = 0; i < n_parts; ++i) mx = fmaxf(mx, lse_parts[static_cast<size_t>(i) * rows + row]);
  float tot = 0.f;
  for (int i = 0; i < n_parts; ++i) {
    const float l = lse_parts[static_cast<size_t>(i) * rows + row];
    tot += (l == -INFINITY) ? 0.f : __expf(l - mx);
  }
  const float inv = tot > 0.f ? 1.f / tot : 0.f;
  for (int d = lane; d < D; d += 32) {
    float acc = 0.f;
    for (int i = 0; i < n_parts; ++i) {
      const float l = lse_parts[static_cast<size_t>(i) * rows + row];
      if (l == -INFINITY) continue;
      acc += __expf(l - mx) * __bfloat162float(o_parts[(static_cast<size_t>(i) * rows + row) * D + d]);
    }
    out[static_cast<size_t>(row) * D + d] = __float2bfloat16_rn(acc * inv);
  }
  if (lse_out != nullptr && lane == 0) lse_out[row] = tot > 0.f ? mx + logf(tot) : -INFINITY;
}

// The same merge over fp32 partials packed one per part: part i is
// [rows * D fp32 O | rows fp32 LSE] at parts + i * part_stride (floats).
__global__ void merge_partials_f32_kernel(const float* parts, size_t part_stride, int n_parts, int rows, int D,
                                          __nv_bfloat16* out, float* lse_out) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const size_t lse_off = static_cast<size_t>(rows) * D;
  float mx = -INFINITY;
  for (int i = 0; i < n_parts; ++i) mx = fmaxf(mx, parts[i * part_stride + lse_off + row]);
  float tot = 0.f;
  for (int i = 0; i < n_parts; ++i) {
    const float l = parts[i * part_stride + lse_off + row];
    tot += (l == -INFINITY) ? 0.f : __expf(l - mx);
  }
  const float inv = tot > 0.f ? 1.f / tot : 0.f;
  for (int d = lane; d < D; d += 32) {
    float acc = 0.f;
    for (int i = 0; i < n_parts; ++i) {
      const float l = parts[i * part_stride + lse_off + row];
      if (l == -INFINITY) continue;
      acc += __expf(l - mx) * parts[i * part_stride + static_cast<size_t>(row) * D + d];
    }
    out[static_cast<size_t>(row) * D + d] = __float2bfloat16_rn(acc * inv);
  }
  if (lse_out != nullptr && lane == 0) lse_out[row] = tot > 0.f ? mx + logf(tot) : -INFINITY;
}

}  // namespace stdb

extern "C" int std_merge_partials(const void* o_parts, const float* lse_parts, int n_parts, int rows, int D, void* out,
                                  float* lse_out, void* stream) {
  if (n_parts <= 0 || rows <= 0 || D <= 0) return 1;
  count_launch();
  stdb::merge_partials_kernel<<<(rows * 32 + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(o_parts), lse_parts, n_parts, rows, D, static_cast<__nv_bfloat16*>(out),
      lse_out);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

extern "C" int std_merge_partials_f32(const float* parts, long long part_stride, int n_parts, int rows, int D,
                                      void* out, float* lse_out, void* stream) {
  if (parts == nullptr || out == nullptr || n_parts <= 0 || rows <= 0 || D <= 0) return 1;
  if (part_stride < static_cast<long long>(rows) * (D + 1)) return 1;
  count_launch();
  stdb::merge_partials_f32_kernel<<<(rows * 32 + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      parts, static_cast<size_t>(part_stride), n_parts, rows, D, static_cast<__nv_bfloat16*>(out), lse_out);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
