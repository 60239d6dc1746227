// common.cuh -- shared device helpers for the STD B200 kernels (sm_100a).
//
// * bounded mbarrier waits (every spin has a ~1 s wall-clock limit; on expiry
//   the kernel records an error code in the library's device error word and
//   returns through its normal exit path);
// * TMA (cp.async.bulk / cp.async.bulk.tensor) wrappers -- never multicast;
// * tcgen05 wrappers: TMEM alloc/dealloc, UMMA smem/instruction descriptors,
//   tcgen05.mma kind::f16 (bf16 x bf16 -> fp32), commit, tcgen05.ld;
// * the selection chain's exp (std_exp), identical to oracle/std_oracle.c.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <utility>

#define STD_DEV __device__ __forceinline__

// ---------------------------------------------------------------------------
// library-wide device error word (one translation unit: std_b200.cu)
// ---------------------------------------------------------------------------
__device__ int g_std_error;

enum StdDeviceError : int {
  STD_DEVERR_NONE = 0,
  STD_DEVERR_WAIT_TIMEOUT = 1,  // an mbarrier wait exceeded its limit
  STD_DEVERR_BOUNDS = 2,        // an index outside its buffer was skipped
  STD_DEVERR_LENGTH = 3,        // a device-resident length exceeded capacity
};

STD_DEV void std_set_error(int code) { atomicCAS(&g_std_error, 0, code); }

STD_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

STD_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
STD_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
STD_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
STD_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
STD_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Distributed shared memory: the shared::cluster address of the object at
// shared::cta address `local` in cluster rank `rank`, and asynchronous stores
// into it that complete transaction bytes on that rank's mbarrier (so the
// receiver learns of their arrival by waiting on its own barrier).
STD_DEV uint32_t mapa_rank(uint32_t local, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
STD_DEV void st_async_f32(uint32_t remote, float v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(remote),
               "r"(__float_as_uint(v)), "r"(remote_bar)
               : "memory");
}
STD_DEV void st_async_v2f32(uint32_t remote, float a, float b, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(remote),
               "r"(__float_as_uint(a)), "r"(__float_as_uint(b)), "r"(remote_bar)
               : "memory");
}
STD_DEV void st_async_v4f32(uint32_t remote, float4 v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   remote),
               "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)), "r"(__float_as_uint(v.z)),
               "r"(__float_as_uint(v.w)), "r"(remote_bar)
               : "memory");
}
STD_DEV void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
STD_DEV void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
STD_DEV void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

STD_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of the same condition (for loops that poll several
// barriers and must not be parked on one of them).
STD_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up after about
// one second (or 2^26 polls), records STD_DEVERR_WAIT_TIMEOUT and returns false.
STD_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && globaltimer_ns() - t0 > 1000000000ull) break;
  }
  std_set_error(STD_DEVERR_WAIT_TIMEOUT);
  return false;
}

// ---------------------------------------------------------------------------
// TMA / bulk copies (global -> shared, completion counted on an mbarrier)
// ---------------------------------------------------------------------------
STD_DEV void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

STD_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// The same 2-D tile load with an L2 eviction-priority hint (a policy from
// l2_policy_evict_first): for data read once per step, so that it does not
// push out lines another kernel is about to read.
STD_DEV void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
STD_DEV uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

STD_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// generic-proxy smem writes -> visible to the async proxy (TMA / tcgen05.mma)
STD_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05 (5th-gen tensor cores, TMEM accumulators)
// ---------------------------------------------------------------------------
STD_DEV void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
STD_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
STD_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
STD_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
STD_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulate.
STD_DEV void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A read from tensor memory (lane = row,
// 32-bit column c = K elements 2c, 2c+1), so that only B crosses shared memory.
STD_DEV void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// mbarrier arrives once every tcgen05.mma issued so far by this thread retires.
STD_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle, version 1 (sm_100).
//   K-major operand : rows of 128 B (64 bf16 of K), 8-row atoms SBO = 1024 B apart.
//   MN-major operand: 64 MN-elements per 128 B row, K-rows 128 B apart,
//                     8-row K groups SBO apart, 64-element MN blocks LBO apart.
STD_DEV uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, A=B=bf16, D=fp32, dense.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn_major) << 15) |
         (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// 32 lanes x 32 consecutive 32-bit TMEM columns; thread i gets lane (base+i).
STD_DEV void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
STD_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
STD_DEV void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
STD_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }


// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a 128B-swizzled tile
// whose rows are 128 bytes (the layout TMA SWIZZLE_128B produces).
STD_DEV uint32_t sw128_offset(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

// ---------------------------------------------------------------------------
// numeric helpers
// ---------------------------------------------------------------------------
// exp(x) for x <= 88, 0 for x < -104 -- the selection chain's exp.  Same
// operation sequence as std_exp() in oracle/std_oracle.c (Cody-Waite
// reduction, degree-7 Taylor polynomial, exponent construction), written with
// explicit round-to-nearest intrinsics so nvcc cannot contract or reorder.
STD_DEV float std_exp(float x) {
  if (x < -104.0f) return 0.0f;
  float t = __fmaf_rn(x, 1.44269504088896340736f, 12582912.0f);
  float n = __fsub_rn(t, 12582912.0f);
  float r = __fmaf_rn(n, -0.693145751953125f, x);
  r = __fmaf_rn(n, -1.42860682030941723212e-6f, r);
  float p = 0.000198412698412698412698f;
  p = __fmaf_rn(p, r, 0.00138888888888888888889f);
  p = __fmaf_rn(p, r, 0.00833333333333333333333f);
  p = __fmaf_rn(p, r, 0.0416666666666666666667f);
  p = __fmaf_rn(p, r, 0.166666666666666666667f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ni = static_cast<int>(n);
  if (ni < -125) {
    p = __fmul_rn(p, 5.42101086242752217004e-20f);
    ni += 64;
  }
  return __fmul_rn(p, __uint_as_float(static_cast<uint32_t>(ni + 127) << 23));
}


// 2^x on the SFU (approximate, denormal results flushed to zero).
STD_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue (launch_dependents), and wait for the previous kernel's completion
// and memory (wait; a no-op when the launch had no programmatic dependency).
// The next kernel is scheduled once every CTA of this one has triggered (or
// exited), so an early trigger never keeps this kernel's own CTAs from
// starting.  A kernel triggers before its own wait only where each kernel
// that can follow it reads nothing before its own wait but data no decode
// kernel writes (the GEMMs prefetch weights there); kernels followed by a
// reader of earlier results before its wait (RoPE + KV append before the
// draft's early reads; the accept and AR bookkeeping) trigger after it.
STD_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
STD_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier over the first `nthreads` threads of the block (id 1..15).
STD_DEV void named_bar_sync(int id, int nthreads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory"); }

STD_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

STD_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ---------------------------------------------------------------------------
// warp-level tensor-core tiles (for skinny, bandwidth-bound contractions whose
// M is a handful of query heads: too small for a 64/128-row tcgen05 tile)
// ---------------------------------------------------------------------------
// Four 8x8 b16 matrices from shared memory; lane i gives the address of row
// i%8 of matrix i/8.  Without .trans lane t receives (row t/4, cols 2(t%4)..+1)
// of each matrix, with .trans (rows 2(t%4)..+1, col t/4).
STD_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
STD_DEV void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
// Transpose of an 8x8 b16 matrix held one 32-bit pair per lane (lane 4r+c
// holds row r, columns 2c and 2c+1) into the same layout.
STD_DEV uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}
// c[16x8 fp32] += a[16x16 bf16, row-major] * b[16x16 -> 16x8 bf16, col-major]
STD_DEV void mma_bf16_16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Order-preserving float -> uint32 key (larger float, larger key).
STD_DEV uint32_t order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

STD_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
STD_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// host: launches with programmatic dependent launch.  The kernel may be
// scheduled while the previous kernel in the stream is still running; every
// kernel launched this way executes pdl_wait() in every CTA before it reads
// anything the stream wrote before it, so the result is that of a plain
// stream-ordered launch, minus the launch gap.
// ---------------------------------------------------------------------------
// Host-side count of kernel launches this library has enqueued (including
// launches recorded into a CUDA graph under stream capture): launch
// accounting for callers, read with std_launch_count().
static std::atomic<long long> g_std_launches{0};
static inline void count_launch() { g_std_launches.fetch_add(1, std::memory_order_relaxed); }

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  count_launch();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// host: dynamic shared-memory limits, per device.  cudaFuncSetAttribute
// applies to the current device only, so the grant is recorded per device
// ordinal: a process that drives several GPUs sets it on each of them.  The
// fast path is one atomic load; setting it takes a lock, so host threads
// launching on the same device concurrently are safe.
// ---------------------------------------------------------------------------
constexpr int STD_MAX_DEVICES = 128;

struct SmemGrant {
  std::atomic<size_t> bytes[STD_MAX_DEVICES];
  std::mutex mu;
  SmemGrant() {
    for (auto& b : bytes) b.store(0, std::memory_order_relaxed);
  }
};

// Ensure `kernel` may use `smem` bytes of dynamic shared memory on the current
// device (and, with max_carveout, prefers the largest shared-memory carveout).
// Returns 0, or 3 when the device or the attribute call fails.
template <typename Kernel>
static int ensure_smem(Kernel kernel, SmemGrant& grant, size_t smem, bool max_carveout = false) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= STD_MAX_DEVICES) return 3;
  if (grant.bytes[dev].load(std::memory_order_acquire) >= smem) return 0;
  std::lock_guard<std::mutex> lock(grant.mu);
  if (grant.bytes[dev].load(std::memory_order_relaxed) >= smem) return 0;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return 3;
  if (max_carveout &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
          cudaSuccess)
    return 3;
  grant.bytes[dev].store(smem, std::memory_order_release);
  return 0;
}

// ---------------------------------------------------------------------------
// host: TMA tensor maps (cuTensorMapEncodeTiled through the runtime's driver
// entry point, so the library needs no link against libcuda)
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

// 2-D bf16 tensor [rows, cols] (row pitch in bytes), box = box_cols x box_rows,
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
