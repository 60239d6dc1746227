// p2p.cu -- peer-memory exchange of the sequence-sharded verify (one node,
// NVLink / NVSwitch): the ranks map each other's buffers with CUDA IPC and
// order their accesses with epoch flags instead of collectives.
//
// Per dense-forward layer, with rank N-1 the owner:
//   owner : p2p_post   copies the layer's queries into its exported query
//                      buffer and publishes epoch e to every server's flag;
//   server: p2p_wait   waits for e, then its verify kernel reads the queries
//                      from the owner's memory over NVLink and stores its
//                      (O, LSE) partial into its slot of the owner's inbox;
//           p2p_post   publishes e to its slot of the owner's flag array;
//   owner : p2p_wait   waits for every server's e, then the list merge reads
//                      every partial from its own memory.
// Loads cross NVLink only for the queries (a few round trips at the start of
// the verify kernel); the partials cross as stores, which do not stall the
// writer.  A buffer is rewritten only after the peer that reads it has
// signalled a later step (the owner posts the next layer's queries after
// merging this layer's partials, which the servers stored after reading
// these queries), so reuse needs no extra handshake.
// Epochs are device-side counters advanced by the kernels, so the steps can
// be captured in a CUDA graph and replayed.  Waits give up after about one
// second (STD_DEVERR_WAIT_TIMEOUT) instead of spinning for ever.
#include <cstring>

#include "common.cuh"

namespace stdb {

constexpr int P2P_MAX_PEERS = 8;

struct P2PFlags {
  int* flag[P2P_MAX_PEERS];
  int n;
};

STD_DEV int ld_relaxed_sys(const int* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
STD_DEV void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
STD_DEV void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The three kernels are launched with programmatic dependent launch: each
// lets its successor be scheduled early and waits (pdl_wait) for its
// predecessor before it touches anything that predecessor wrote, and before
// it completes, so stream order holds transitively.

// dst <- src (n16 16-byte vectors, one block), then epoch = ++*counter is
// published to every flag.  The barrier orders the block's copies before the
// publishing thread's system-scope release stores (release is cumulative), and
// pdl_wait has ordered everything the stream wrote before this kernel (the
// partial a server's verify stored into the owner's memory) before it too.
__global__ void __launch_bounds__(1024) p2p_post_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                        size_t n16, P2PFlags flags, int* counter) {
  pdl_wait();
  pdl_launch_dependents();
  for (size_t i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    const int e = *counter + 1;
    *counter = e;
    for (int i = 0; i < flags.n; ++i) st_release_sys(flags.flag[i], e);
  }
}

// Wait until flags[0..n) all reach epoch = *counter + 1, then advance the
// counter.  Bounded: after ~1 s the error word is set and the kernel returns.
// Launched early, it starts polling once its predecessor has finished
// (pdl_wait: the counter was written by an earlier kernel of this stream), so
// its successor sees both the peers' data and the predecessor's.  Polls are
// relaxed loads; one acquire fence after the last orders what follows.
__global__ void p2p_wait_kernel(const int* flags, int n, int* counter) {
  pdl_launch_dependents();
  if (threadIdx.x != 0) return;
  pdl_wait();
  const uint64_t t0 = globaltimer_ns();
  const int e = *counter + 1;
  bool timed_out = false;
  for (int i = 0; i < n && !timed_out; ++i) {
    uint32_t polls = 0;
    while (ld_relaxed_sys(flags + i) < e) {
      if ((++polls & 255u) == 0u && globaltimer_ns() - t0 > 1000000000ull) {
        std_set_error(STD_DEVERR_WAIT_TIMEOUT);
        timed_out = true;
        break;
      }
    }
  }
  fence_acq_rel_sys();  // with the relaxed polls above: acquire of every flag seen
  *counter = e;
}

struct PartList {
  const float* part[P2P_MAX_PEERS];  // each [rows * D fp32 O | rows fp32 LSE]
};

// merge_partials_f32_kernel with the parts behind a pointer list (they live
// in different GPUs' memories): same operations, same order, same bytes.
__global__ void merge_partials_list_kernel(PartList parts, int n_parts, int rows, int D, __nv_bfloat16* out,
                                           float* lse_out) {
  pdl_wait();
  pdl_launch_dependents();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const size_t lse_off = static_cast<size_t>(rows) * D;
  float mx = -INFINITY;
  for (int i = 0; i < n_parts; ++i) mx = fmaxf(mx, parts.part[i][lse_off + row]);
  float tot = 0.f;
  for (int i = 0; i < n_parts; ++i) {
    const float l = parts.part[i][lse_off + row];
    tot += (l == -INFINITY) ? 0.f : __expf(l - mx);
  }
  const float inv = tot > 0.f ? 1.f / tot : 0.f;
  for (int d = lane; d < D; d += 32) {
    float acc = 0.f;
    for (int i = 0; i < n_parts; ++i) {
      const float l = parts.part[i][lse_off + row];
      if (l == -INFINITY) continue;
      acc += __expf(l - mx) * parts.part[i][static_cast<size_t>(row) * D + d];
    }
    out[static_cast<size_t>(row) * D + d] = __float2bfloat16_rn(acc * inv);
  }
  if (lse_out != nullptr && lane == 0) lse_out[row] = tot > 0.f ? mx + logf(tot) : -INFINITY;
}

}  // namespace stdb

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
extern "C" size_t std_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int std_device_alloc(size_t bytes, void** ptr_out) {
  if (bytes == 0 || ptr_out == nullptr) return 1;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return 4;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return 4;
  }
  *ptr_out = p;
  return 0;
}

extern "C" int std_device_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? 0 : 4; }

extern "C" int std_ipc_handle(const void* base, void* handle_out) {
  if (base == nullptr || handle_out == nullptr) return 1;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(base)) != cudaSuccess) return 4;
  memcpy(handle_out, &h, sizeof(h));
  return 0;
}

extern "C" int std_ipc_open(const void* handle, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr) return 1;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? 0 : 4;
}

extern "C" int std_ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? 0 : 4; }

extern "C" int std_p2p_post(const void* src, void* dst, size_t bytes, const unsigned long long* flags, int n_flags,
                            int* counter, void* stream) {
  if (n_flags < 0 || n_flags > stdb::P2P_MAX_PEERS || counter == nullptr || bytes % 16 != 0) return 1;
  if (bytes > 0 && (src == nullptr || dst == nullptr)) return 1;
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) != 0) return 1;
  stdb::P2PFlags f = {};
  for (int i = 0; i < n_flags; ++i) {
    if (flags == nullptr || flags[i] == 0) return 1;
    f.flag[i] = reinterpret_cast<int*>(flags[i]);
  }
  f.n = n_flags;
  return launch_pdl(stdb::p2p_post_kernel, dim3(1), dim3(1024), 0, static_cast<cudaStream_t>(stream),
                    static_cast<const uint4*>(src), static_cast<uint4*>(dst), bytes / 16, f, counter) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_p2p_wait(const int* flags, int n_flags, int* counter, void* stream) {
  if (flags == nullptr || counter == nullptr || n_flags <= 0) return 1;
  return launch_pdl(stdb::p2p_wait_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), flags, n_flags,
                    counter) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_merge_partials_f32_list(const unsigned long long* parts, int n_parts, int rows, int D, void* out,
                                           float* lse_out, void* stream) {
  if (parts == nullptr || out == nullptr || n_parts <= 0 || n_parts > stdb::P2P_MAX_PEERS || rows <= 0 || D <= 0)
    return 1;
  stdb::PartList pl = {};
  for (int i = 0; i < n_parts; ++i) {
    if (parts[i] == 0) return 1;
    pl.part[i] = reinterpret_cast<const float*>(parts[i]);
  }
  return launch_pdl(stdb::merge_partials_list_kernel, dim3((rows * 32 + 255) / 256), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), pl, n_parts, rows, D, static_cast<__nv_bfloat16*>(out),
                    lse_out) == cudaSuccess
             ? 0
             : 4;
}
