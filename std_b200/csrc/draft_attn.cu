// draft_attn.cu -- (b) sparse GQA draft attention, q_len = 1.
//
// Replaces the reference's sparse draft attention
//   std_qwen25vl.py:406-417  F.scaled_dot_product_attention(q, k, v, enable_gqa=True)
//   triton_attention.py:13-112  _gqa_single_query_kernel (one program per q head)
// over the compacted sparse cache (no mask: the draft query sees every cached
// key, std_qwen25vl.py:400-417).
//
// Design.  The op reads 2048 B of K/V per key and does ~7 flop per byte, so it
// is HBM-bound -- provided the math keeps up: at 6.5 TB/s the 7 query heads of
// a KV group need ~45 TFLOP/s, more than fp32 CUDA cores sustain once the
// conversions and reductions are counted.  So the two contractions run on the
// tensor cores as warp-level m16n8k16 bf16 tiles (the 7 heads padded to the
// 16-row tile), which leaves the kernel bound by the K/V stream alone.
//
//   grid = (DR_CLUSTER, Hkv, B), cluster = (DR_CLUSTER, 1, 1), 4 warps/CTA.
//   CTA rank i owns keys [i*per, (i+1)*per) of the request's live length
//   (per = ceil(L/8) rounded up to 16).  TMA (2-D tensor maps, 128-byte
//   swizzle, 16-row boxes, no multicast) streams its K and V rows through a
//   three-stage ring of 64-key sub-tiles; only the boxes that hold live keys are
//   fetched.  Each warp takes 16 keys of every sub-tile: S = Q K^T from
//   ldmatrix'd K fragments, an online softmax on the accumulator registers,
//   then O += P V with P reused from registers as the A operand and V
//   fragments from ldmatrix.trans.  Every K/V byte is read from HBM once (the
//   Triton kernel re-reads each KV head for each of its 7 query heads).
//   The 4 warp partials are combined in shared memory; each CTA then pushes
//   its partial of output slice q into rank q's shared memory (DSMEM stores),
//   one cluster barrier later every rank finishes its 112 of the 7 x 128
//   outputs from local data -- one launch, no global scratch, no second
//   kernel, one cluster barrier.  Lengths come from device memory, so the
//   launch is graph-capturable while they change between replays.
#include <cooperative_groups.h>

#include "common.cuh"

namespace stdb {

constexpr int DR_D = 128;
constexpr int DR_G = 7;
constexpr int DR_WARPS = 4;
constexpr int DR_THREADS = DR_WARPS * 32;
constexpr int DR_SUB = 64;     // keys per pipeline stage, 16 per warp
constexpr int DR_BOX = 16;     // rows per TMA box
constexpr int DR_STAGES = 3;
constexpr int DR_CLUSTER = 8;  // CTAs per (request, KV head)
constexpr uint32_t DR_HALF_BYTES = DR_SUB * 64 * 2;                // 64 keys x 64 dims (one 128-B swizzle span)
constexpr uint32_t DR_STAGE_BYTES = 4 * DR_HALF_BYTES;             // K lo, K hi, V lo, V hi
constexpr uint32_t DR_SMEM = DR_STAGES * DR_STAGE_BYTES + 1024;    // + alignment slack (swizzle atoms: 1 KB)
constexpr int DR_OSTRIDE = DR_D + 4;                               // fp32 row of a warp partial (bank skew)
constexpr int DR_OUT_PER_RANK = DR_G * DR_D / DR_CLUSTER;          // 112
static_assert(DR_WARPS * 8 * DR_OSTRIDE * 4 + 2 * DR_WARPS * 8 * 4 <= DR_STAGES * DR_STAGE_BYTES,
              "warp partials alias the stage buffers");

struct DraftParams {
  const __nv_bfloat16* q;   // [B, Hq, D]
  const int32_t* lens;      // [B] device lengths
  int len_offset;           // live keys = lens[b] + len_offset
  int cap;
  int Hq, Hkv;
  float scale_log2;         // (1/sqrt(D)) * log2(e)
  __nv_bfloat16* out;       // [B, Hq, D]
  float* lse;               // [B, Hq] natural-log LSE, may be null
  int flags;                // STD_DRAFT_AFTER_APPEND: see the C ABI below
};

// Byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled half tile.
STD_DEV uint32_t dr_sw(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Q of KV group kvh as the m16n8k16 A operand: row gid = query head kvh*7 +
// gid (row 7 and rows 8..15 are zero padding), k-step ks covers dims
// [16ks, 16ks+16).
STD_DEV void draft_load_q(const DraftParams& p, int b, int kvh, int gid, int tig, uint32_t (&qa)[8][2]) {
  const bool hv = gid < DR_G;
  const __nv_bfloat16* qrow = p.q + (static_cast<size_t>(b) * p.Hq + kvh * DR_G + (hv ? gid : 0)) * DR_D;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    qa[ks][0] = hv ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 2 * tig) : 0u;
    qa[ks][1] = hv ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 8 + 2 * tig) : 0u;
  }
}

// One warp's 16 keys (kw .. kw+15 of the sub-tile in sK / sV, nvalid of them
// live) folded into its online softmax state (o, m_run, l_run of row gid).
STD_DEV void draft_subtile(const uint8_t* sK, const uint8_t* sV, int kw, int nvalid, const uint32_t (&qa)[8][2],
                           float sc, int lane, float (&o)[16][4], float& m_run, float& l_run) {
  const int tig = lane & 3;
  // S[16 x 16 keys] = Q K^T, even and odd k-steps in separate
  // accumulators (four independent MMA chains instead of two)
  float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  float s2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const int mi = lane >> 3;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int key = kw + (mi >> 1) * 8 + (lane & 7);
    const int ch = (ks & 3) * 2 + (mi & 1);
    uint32_t b0, b1, b2, b3;
    ldsm_x4(smem_u32(sK + (ks >> 2) * DR_HALF_BYTES + dr_sw(key, ch)), b0, b1, b2, b3);
    float* d0 = (ks & 1) ? s2[0] : s[0];
    float* d1 = (ks & 1) ? s2[1] : s[1];
    mma_bf16_16816(d0, qa[ks][0], 0u, qa[ks][1], 0u, b0, b1);
    mma_bf16_16816(d1, qa[ks][0], 0u, qa[ks][1], 0u, b2, b3);
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    s[0][e] += s2[0][e];
    s[1][e] += s2[1][e];
  }
  // online softmax on row gid (keys 2tig, 2tig+1, 8+2tig, 9+2tig)
  float x[4];
  x[0] = (2 * tig < nvalid) ? s[0][0] * sc : -INFINITY;
  x[1] = (2 * tig + 1 < nvalid) ? s[0][1] * sc : -INFINITY;
  x[2] = (8 + 2 * tig < nvalid) ? s[1][0] * sc : -INFINITY;
  x[3] = (9 + 2 * tig < nvalid) ? s[1][1] * sc : -INFINITY;
  float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  const float mn = fmaxf(m_run, mx);  // finite: key kw is live
  const float alpha = ex2_approx(m_run - mn);
  float pr[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) pr[e] = ex2_approx(x[e] - mn);
  l_run = l_run * alpha + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
  m_run = mn;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    o[j][0] *= alpha;
    o[j][1] *= alpha;
  }
  const uint32_t pa0 = pack_bf16x2(pr[0], pr[1]), pa2 = pack_bf16x2(pr[2], pr[3]);
  // O[16 x 128] += P[16 x 16 keys] V[16 keys x 128]
#pragma unroll
  for (int jj = 0; jj < 8; ++jj) {
    const int key = kw + (mi & 1) * 8 + (lane & 7);
    const int ch = (2 * jj & 7) + (mi >> 1);
    uint32_t v0, v1, v2, v3;
    ldsm_x4_trans(smem_u32(sV + (jj >> 2) * DR_HALF_BYTES + dr_sw(key, ch)), v0, v1, v2, v3);
    mma_bf16_16816(o[2 * jj], pa0, 0u, pa2, 0u, v0, v1);
    mma_bf16_16816(o[2 * jj + 1], pa0, 0u, pa2, 0u, v2, v3);
  }
}

// Combine the 4 warp partials of this CTA, push them to the ranks that finish
// each output slice, and finish this rank's slice (one cluster barrier).
STD_DEV void draft_finish(cooperative_groups::cluster_group& cluster, int rank, int b, int kvh, uint8_t* sbase,
                          const DraftParams& p, float (&o)[16][4], float m_run, float l_run, bool ok,
                          float (&r_o)[DR_CLUSTER][DR_OUT_PER_RANK], float (&r_m)[DR_CLUSTER][DR_G],
                          float (&r_l)[DR_CLUSTER][DR_G]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  // warp partials -> shared memory (the stage buffers are free now)
  float* wo = reinterpret_cast<float*>(sbase);  // [warp][8 rows][DR_OSTRIDE]
  float* wm = wo + DR_WARPS * 8 * DR_OSTRIDE;   // [warp][8]
  float* wl = wm + DR_WARPS * 8;                // [warp][8]
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (gid < DR_G) {
    float* row = wo + (warp * 8 + gid) * DR_OSTRIDE;
#pragma unroll
    for (int j = 0; j < 16; ++j) *reinterpret_cast<float2*>(row + 8 * j + 2 * tig) = make_float2(o[j][0], o[j][1]);
    if (tig == 0) {
      wm[warp * 8 + gid] = (l_run > 0.f && ok) ? m_run : -INFINITY;
      wl[warp * 8 + gid] = ok ? l_run : 0.f;
    }
  }
  __syncthreads();
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  // CTA partial: thread tid owns dim tid of all 7 heads
#pragma unroll
  for (int h = 0; h < DR_G; ++h) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < DR_WARPS; ++w) M = fmaxf(M, wm[w * 8 + h]);
    float acc = 0.f, lsum = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < DR_WARPS; ++w) {
        const float mw = wm[w * 8 + h];
        if (mw == -INFINITY) continue;
        const float wt = ex2_approx(mw - M);
        acc += wt * wo[(w * 8 + h) * DR_OSTRIDE + tid];
        lsum += wt * wl[w * 8 + h];
      }
    }
    // push output h*128 + tid to the rank that finishes it (DSMEM store)
    const int idx = h * DR_D + tid;
    *cluster.map_shared_rank(&r_o[rank][idx % DR_OUT_PER_RANK], idx / DR_OUT_PER_RANK) = acc;
    if (tid == 0) {
      for (int q = (h * DR_D) / DR_OUT_PER_RANK; q <= (h * DR_D + DR_D - 1) / DR_OUT_PER_RANK; ++q) {
        *cluster.map_shared_rank(&r_m[rank][h], q) = M;
        *cluster.map_shared_rank(&r_l[rank][h], q) = lsum;
      }
    }
  }
  // One cluster barrier: every push has landed (release/acquire), and after it
  // no CTA touches another's shared memory, so none has to wait for the
  // others before exiting.
  cluster.sync();
  // Rank r finishes outputs [112 r, 112 r + 112) of the group's 7 x 128 from
  // the 8 partials in its own shared memory.
  if (tid < DR_OUT_PER_RANK) {
    const int idx = rank * DR_OUT_PER_RANK + tid;
    const int g = idx / DR_D, d = idx % DR_D;
    float mr[DR_CLUSTER], lr[DR_CLUSTER], orr[DR_CLUSTER];
#pragma unroll
    for (int r = 0; r < DR_CLUSTER; ++r) {
      mr[r] = r_m[r][g];
      lr[r] = r_l[r][g];
      orr[r] = r_o[r][tid];
    }
    float m = -INFINITY;
#pragma unroll
    for (int r = 0; r < DR_CLUSTER; ++r) m = fmaxf(m, mr[r]);
    float l = 0.f, acc = 0.f;
#pragma unroll
    for (int r = 0; r < DR_CLUSTER; ++r) {
      if (mr[r] == -INFINITY) continue;
      const float w = ex2_approx(mr[r] - m);
      l += w * lr[r];
      acc += w * orr[r];
    }
    p.out[(static_cast<size_t>(b) * p.Hq + kvh * DR_G + g) * DR_D + d] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
    if (d == 0 && p.lse != nullptr)
      p.lse[static_cast<size_t>(b) * p.Hq + kvh * DR_G + g] =
          l > 0.f ? (m + log2f(l)) * 0.69314718055994530942f : -INFINITY;
  }
}

__global__ void __cluster_dims__(DR_CLUSTER, 1, 1) __launch_bounds__(DR_THREADS, 2)
    draft_attn_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                      const DraftParams p) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  // Every CTA of the cluster must be running before another writes into its
  // shared memory: arrive now, wait just before the first push (by then the
  // wait returns at once).
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  // After an append (the decode step's RoPE + KV-append kernel, which writes
  // only q and the K/V row at position L-1): the lengths and every older K/V
  // row are read while that kernel may still run; q and row L-1 only after
  // griddepcontrol.wait.  Otherwise nothing is read before the wait.
  const bool early = (p.flags & 1) != 0;
  if (!early) {
    pdl_wait();
    pdl_launch_dependents();
  }

  extern __shared__ uint8_t dsmem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bar[DR_STAGES];
  // partials pushed here by every rank r of the cluster for the 112 outputs
  // this CTA finishes (and, per head it covers, their m and l)
  __shared__ __align__(16) float r_o[DR_CLUSTER][DR_OUT_PER_RANK];
  __shared__ float r_m[DR_CLUSTER][DR_G], r_l[DR_CLUSTER][DR_G];

  int L = p.lens[b] + p.len_offset;
  if (L > p.cap || L < 0) {
    if (rank == 0 && tid == 0) std_set_error(STD_DEVERR_LENGTH);
    L = L < 0 ? 0 : p.cap;
  }
  int per = (L + DR_CLUSTER - 1) / DR_CLUSTER;
  per = (per + 15) & ~15;
  const int k0 = min(L, rank * per);
  const int k1 = min(L, k0 + per);
  const int nkeys = k1 - k0;
  const int nsub = (nkeys + DR_SUB - 1) / DR_SUB;
  const int row0 = (b * p.Hkv + kvh) * p.cap + k0;  // first tensor-map row of this CTA
  // early mode: the 16-row box holding row L-1 waits for the append
  int defer_i = -1, defer_j = -1;
  if (early && L - 1 >= k0 && L - 1 < k1) {
    defer_i = (L - 1 - k0) / DR_SUB;
    defer_j = ((L - 1 - k0) % DR_SUB) / DR_BOX;
  }

  if (tid == 0) {
    prefetch_tensormap(&tk);
    prefetch_tensormap(&tv);
#pragma unroll
    for (int s = 0; s < DR_STAGES; ++s) mbar_init(&bar[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  // Sub-tile i is issued by the 32 lanes of warp 0 together: lane 4j+part
  // copies box j (16 rows) of K lo/hi (part 0/1) or V lo/hi (part 2/3).
  // mode 0: the whole sub-tile; 1: all but the deferred box; 2: only that box
  auto issue = [&](int i, int mode) {
    const int st = i % DR_STAGES;
    const int a = i * DR_SUB;
    const int nbox = (min(DR_SUB, nkeys - a) + DR_BOX - 1) / DR_BOX;
    uint8_t* s = sbase + st * DR_STAGE_BYTES;
    if (mode != 2) {
      if (lane == 0) mbar_arrive_expect_tx(&bar[st], static_cast<uint32_t>(nbox) * 4u * DR_BOX * 128u);
      __syncwarp();
    }
    const int j = lane >> 2, part = lane & 3;
    const bool is_deferred = i == defer_i && j == defer_j;
    if (lane < 4 * nbox && (mode == 0 || (mode == 1) != is_deferred)) {
      const uint32_t off = j * DR_BOX * 128 + (part & 1) * DR_HALF_BYTES + (part >> 1) * 2 * DR_HALF_BYTES;
      tma_load_2d(s + off, part < 2 ? &tk : &tv, &bar[st], (part & 1) * 64, row0 + a + j * DR_BOX);
    }
  };
  // sub-tiles issued so far: the same value in every thread (warp 0 issues),
  // so the block-wide barriers below that depend on it are uniform
  int issued = min(DR_STAGES, nsub);
  if (warp == 0) {
    for (int i = 0; i < issued; ++i) issue(i, early ? 1 : 0);
  }
  if (early) {
    pdl_wait();
    pdl_launch_dependents();
    if (warp == 0 && defer_i >= 0 && defer_i < issued) issue(defer_i, 2);
  }

  uint32_t qa[8][2];
  draft_load_q(p, b, kvh, gid, tig, qa);

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // row gid of this warp, identical across the quad
  bool ok = true;
  const float sc = p.scale_log2;

  for (int i = 0; i < nsub; ++i) {
    const int st = i % DR_STAGES;
    const int nk = min(DR_SUB, nkeys - i * DR_SUB);
    if (ok) ok = mbar_wait(&bar[st], (i / DR_STAGES) & 1);
    ok = __all_sync(0xffffffffu, ok);  // warp-uniform: guards warp-collective code below
    uint8_t* sK = sbase + st * DR_STAGE_BYTES;
    uint8_t* sV = sK + 2 * DR_HALF_BYTES;
    const int kw = warp * 16;
    const int nvalid = min(16, nk - kw);
    if (nvalid > 0 && ok) {
      if (nvalid < 16) {
        // Rows past the live length inside the last box hold whatever the
        // cache holds there; zero their V so that P = 0 times them stays 0.
        for (int e = lane; e < (16 - nvalid) * 16; e += 32) {
          const int r = kw + nvalid + (e >> 4), c = e & 15;
          *reinterpret_cast<uint4*>(sV + (c >> 3) * DR_HALF_BYTES + r * 128 + ((c & 7) << 4)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        fence_async_smem();
        __syncwarp();
      }
      draft_subtile(sK, sV, kw, nvalid, qa, sc, lane, o, m_run, l_run);
    }
    if (issued < nsub) {  // uniform: a refill follows
      __syncthreads();    // every warp is done with stage st
      if (warp == 0 && __all_sync(0xffffffffu, ok)) issue(issued, 0);
      ++issued;
    }
  }
  if (tid == 0) {
    // Normally a no-op (every issued phase has completed).  If a wait gave up,
    // let the loads still in flight land before the stage buffers are reused
    // or the CTA exits; these waits are bounded too.
    for (int i = max(0, issued - DR_STAGES); i < issued; ++i) mbar_wait(&bar[i % DR_STAGES], (i / DR_STAGES) & 1);
  }
  __syncthreads();

  draft_finish(cluster, rank, b, kvh, sbase, p, o, m_run, l_run, ok, r_o, r_m, r_l);
}
// ---------------------------------------------------------------------------
// Index-based sparse cache: the draft reads the selected prompt rows straight
// from the dense cache through a per-(request, KV head) position list, and the
// generated tokens' sparse-path K/V from a small tail buffer -- no compacted
// copy of the prompt.  Key j of request b, head h is dense row idx[b][h][j]
// for j < n_idx (positions ascending, as compaction would order them), else
// tail row j - n_idx; keys, chunking and arithmetic are those of the
// compacted-cache kernel, so both give the same bytes.  The rows are gathered
// with 16-byte cp.async into the same 128-byte-swizzled stage layout (a
// 256-byte K or V row is two swizzle rows); rows past the live length are
// zero-filled.
// ---------------------------------------------------------------------------
struct DraftIndex {
  const int32_t* idx;        // [B, Hkv, n_idx] dense-cache positions
  int n_idx;
  const __nv_bfloat16* dk;   // dense cache of this layer [B, Hkv, cap_d, D]
  const __nv_bfloat16* dv;
  int cap_d;
  const __nv_bfloat16* tk;   // tail of this layer [B, Hkv, tail_cap, D]
  const __nv_bfloat16* tv;
  int tail_cap;
};

STD_DEV void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
STD_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
STD_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __cluster_dims__(DR_CLUSTER, 1, 1) __launch_bounds__(DR_THREADS, 2)
    draft_attn_indexed_kernel(const DraftParams p, const DraftIndex ix) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  pdl_wait();
  pdl_launch_dependents();

  extern __shared__ uint8_t dsmem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(16) float r_o[DR_CLUSTER][DR_OUT_PER_RANK];
  __shared__ float r_m[DR_CLUSTER][DR_G], r_l[DR_CLUSTER][DR_G];

  int L = p.lens[b] + p.len_offset;
  if (L > p.cap || L < 0) {
    if (rank == 0 && tid == 0) std_set_error(STD_DEVERR_LENGTH);
    L = L < 0 ? 0 : p.cap;
  }
  int per = (L + DR_CLUSTER - 1) / DR_CLUSTER;
  per = (per + 15) & ~15;
  const int k0 = min(L, rank * per);
  const int k1 = min(L, k0 + per);
  const int nkeys = k1 - k0;
  const int nsub = (nkeys + DR_SUB - 1) / DR_SUB;
  const size_t head = static_cast<size_t>(b) * p.Hkv + kvh;

  // thread t gathers half (t & 1) of row t >> 1 of a 64-row sub-tile, K and V
  auto issue = [&](int i) {
    if (i >= nsub) return;
    const int st = i % DR_STAGES;
    const int r = tid >> 1, hf = tid & 1;
    const int rel = i * DR_SUB + r;
    const __nv_bfloat16* srcK = ix.dk;  // any valid address when zero-filling
    const __nv_bfloat16* srcV = ix.dv;
    uint32_t nbytes = 0;
    if (rel < nkeys) {
      const int j = k0 + rel;
      if (j < ix.n_idx) {
        const int row = ix.idx[head * ix.n_idx + j];
        if (row >= 0 && row < ix.cap_d) {
          srcK = ix.dk + (head * ix.cap_d + row) * DR_D;
          srcV = ix.dv + (head * ix.cap_d + row) * DR_D;
          nbytes = 16;
        } else {
          std_set_error(STD_DEVERR_BOUNDS);
        }
      } else {
        srcK = ix.tk + (head * ix.tail_cap + (j - ix.n_idx)) * DR_D;
        srcV = ix.tv + (head * ix.tail_cap + (j - ix.n_idx)) * DR_D;
        nbytes = 16;
      }
    }
    uint8_t* sK = sbase + st * DR_STAGE_BYTES;
    uint8_t* sV = sK + 2 * DR_HALF_BYTES;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint32_t off = hf * DR_HALF_BYTES + dr_sw(r, c);
      cp_async16(sK + off, srcK + hf * 64 + c * 8, nbytes);
      cp_async16(sV + off, srcV + hf * 64 + c * 8, nbytes);
    }
  };
#pragma unroll
  for (int i = 0; i < DR_STAGES; ++i) {
    issue(i);
    cp_async_commit();
  }

  uint32_t qa[8][2];
  draft_load_q(p, b, kvh, gid, tig, qa);
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;

  for (int i = 0; i < nsub; ++i) {
    cp_async_wait<DR_STAGES - 1>();  // this thread's copies of sub-tile i have landed
    __syncthreads();                 // ... and every other thread's
    const int st = i % DR_STAGES;
    const uint8_t* sK = sbase + st * DR_STAGE_BYTES;
    const uint8_t* sV = sK + 2 * DR_HALF_BYTES;
    const int kw = warp * 16;
    const int nvalid = min(16, min(DR_SUB, nkeys - i * DR_SUB) - kw);
    if (nvalid > 0) draft_subtile(sK, sV, kw, nvalid, qa, p.scale_log2, lane, o, m_run, l_run);
    __syncthreads();  // stage st is free
    issue(i + DR_STAGES);
    cp_async_commit();
  }
  cp_async_wait<0>();  // nothing in flight into the stage buffers
  __syncthreads();
  draft_finish(cluster, rank, b, kvh, sbase, p, o, m_run, l_run, true, r_o, r_m, r_l);
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
                              void* workspace, size_t workspace_bytes, int flags, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (D != stdb::DR_D || Hq != Hkv * stdb::DR_G || B <= 0 || cap <= 0) return 1;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || lens == nullptr || out == nullptr) return 1;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) return 1;
  if ((reinterpret_cast<uintptr_t>(q) & 3) != 0) return 1;
  const long long rows = static_cast<long long>(B) * Hkv * cap;
  if (rows + stdb::DR_SUB >= (1ll << 31)) return 1;  // tensor-map row coordinates are 32-bit
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(stdb::draft_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, stdb::DR_SMEM) !=
            cudaSuccess ||
        cudaFuncSetAttribute(stdb::draft_attn_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return 3;
    attr_set = true;
  }
  CUtensorMap tk, tv;
  int rc = make_tmap_bf16_2d(&tk, k_cache, static_cast<uint64_t>(rows), 128, 256, 64, stdb::DR_BOX);
  if (rc == 0) rc = make_tmap_bf16_2d(&tv, v_cache, static_cast<uint64_t>(rows), 128, 256, 64, stdb::DR_BOX);
  if (rc != 0) return rc;
  stdb::DraftParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.lens = lens;
  p.len_offset = len_offset;
  p.cap = cap;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = (1.0f / sqrtf(static_cast<float>(D))) * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.flags = flags & 1;
  dim3 grid(stdb::DR_CLUSTER, Hkv, B);
  return launch_pdl(stdb::draft_attn_kernel, grid, dim3(stdb::DR_THREADS), stdb::DR_SMEM,
                    static_cast<cudaStream_t>(stream), tk, tv, p) == cudaSuccess
             ? 0
             : 4;
}

extern "C" int std_draft_attn_indexed(const void* q, const void* dense_k, const void* dense_v, int cap_dense,
                                      const int32_t* idx, int n_idx, const void* tail_k, const void* tail_v,
                                      int tail_cap, const int32_t* lens, int len_offset, int B, int Hq, int Hkv,
                                      int D, void* out, float* lse, void* stream) {
  if (D != stdb::DR_D || Hq != Hkv * stdb::DR_G || B <= 0 || cap_dense <= 0 || n_idx < 0 || tail_cap < 0) return 1;
  if (q == nullptr || dense_k == nullptr || dense_v == nullptr || lens == nullptr || out == nullptr) return 1;
  if (n_idx > 0 && idx == nullptr) return 1;
  if (tail_cap > 0 && (tail_k == nullptr || tail_v == nullptr)) return 1;
  if (((reinterpret_cast<uintptr_t>(dense_k) | reinterpret_cast<uintptr_t>(dense_v) |
        reinterpret_cast<uintptr_t>(tail_k) | reinterpret_cast<uintptr_t>(tail_v)) & 15) != 0)
    return 1;
  if ((reinterpret_cast<uintptr_t>(q) & 3) != 0) return 1;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(stdb::draft_attn_indexed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             stdb::DR_SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(stdb::draft_attn_indexed_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return 3;
    attr_set = true;
  }
  stdb::DraftParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.lens = lens;
  p.len_offset = len_offset;
  p.cap = n_idx + tail_cap;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = (1.0f / sqrtf(static_cast<float>(D))) * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.flags = 0;
  stdb::DraftIndex ix;
  ix.idx = idx;
  ix.n_idx = n_idx;
  ix.dk = static_cast<const __nv_bfloat16*>(dense_k);
  ix.dv = static_cast<const __nv_bfloat16*>(dense_v);
  ix.cap_d = cap_dense;
  ix.tk = static_cast<const __nv_bfloat16*>(tail_k);
  ix.tv = static_cast<const __nv_bfloat16*>(tail_v);
  ix.tail_cap = tail_cap;
  dim3 grid(stdb::DR_CLUSTER, Hkv, B);
  return launch_pdl(stdb::draft_attn_indexed_kernel, grid, dim3(stdb::DR_THREADS), stdb::DR_SMEM,
                    static_cast<cudaStream_t>(stream), p, ix) == cudaSuccess
             ? 0
             : 4;
}
