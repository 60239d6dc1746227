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
// tensor cores as warp-level m16n8k16 bf16 tiles, in transposed form so that
// the 7 heads (plus one zero pad) are the N = 8 side of both tiles:
// S^T = K Q^T puts 16 keys on M, and O^T += V^T P^T puts 16 dims on M, with P^T
// moved from the accumulator layout to the operand layout by movmatrix.  A
// 16-key unit then costs 8 + 8 MMAs and the output accumulator is 32 fp32
// registers per thread (the untransposed form pads 7 heads to 16 rows: twice
// the MMAs and registers).
//
//   grid = (DR_CLUSTER, Hkv, B), cluster = (DR_CLUSTER, 1, 1), 8 warps/CTA.
//   CTA rank i owns keys [i*per, (i+1)*per) of the request's live length,
//   the last rank also the remainder (per a multiple of 16, draft_split).  TMA (2-D tensor maps, 128-byte
//   swizzle, no multicast; 64-row boxes for a full sub-tile, 16-row boxes for
//   a partial one) streams its K and V rows through a three-stage ring of
//   64-key sub-tiles; only rows of boxes that hold live keys are fetched.  The
//   two warp groups take alternate sub-tiles (group g: sub-tiles g, g+2, ...;
//   an odd count ends with group 0 folding two in one step) and each warp 16
//   keys of a sub-tile: S^T from ldmatrix'd K
//   fragments and the q fragments held in registers, an online softmax on the
//   accumulator registers, then O^T += V^T P^T with V^T from ldmatrix.trans.
//   Every K/V byte is read from HBM once (the Triton kernel re-reads each KV
//   head for each of its 7 query heads).  The 8 warp partials are combined in
//   shared memory; each CTA then pushes its partial of output slice q into
//   rank q's shared memory with st.async (asynchronous DSMEM stores that
//   complete bytes on rank q's mbarrier), and every rank finishes its 112 of
//   the 7 x 128 outputs from local data once its barrier completes -- one
//   launch, no global scratch, no second kernel, and no cluster barrier after
//   the pushes.  Lengths come from device memory, so the launch is
//   graph-capturable while they change between replays.
#include <cooperative_groups.h>

#include "common.cuh"

namespace stdb {

constexpr int DR_D = 128;
constexpr int DR_G = 7;
constexpr int DR_WARPS = 8;    // two groups of 4, alternate sub-tiles
constexpr int DR_THREADS = DR_WARPS * 32;
constexpr int DR_SUB = 64;     // keys per pipeline stage, 16 per warp of a group
constexpr int DR_BOX = 16;     // rows per TMA box
constexpr int DR_STAGES = 3;
constexpr int DR_CLUSTER = 8;  // CTAs per (request, KV head)
// The thread that issues every K/V copy: lane 0 of the last warp, which never
// takes the extra unit of an odd sub-tile count (group 0's first warp does),
// so that the busiest warp is not held back loading q while copies are issued.
constexpr int DR_ISSUER = (DR_WARPS - 1) * 32;
constexpr uint32_t DR_HALF_BYTES = DR_SUB * 64 * 2;                // 64 keys x 64 dims (one 128-B swizzle span)
constexpr uint32_t DR_STAGE_BYTES = 4 * DR_HALF_BYTES;             // K lo, K hi, V lo, V hi
constexpr uint32_t DR_SMEM = DR_STAGES * DR_STAGE_BYTES + 1024;    // + alignment slack (swizzle atoms: 1 KB)
constexpr int DR_OSTRIDE = DR_D + 4;                               // fp32 row of a warp partial (bank skew)
constexpr int DR_OUT_PER_RANK = DR_G * DR_D / DR_CLUSTER;          // 112
static_assert(DR_WARPS * 8 * DR_OSTRIDE * 4 + 3 * DR_WARPS * 8 * 4 + 16 * 4 <= DR_STAGES * DR_STAGE_BYTES,
              "warp partials alias the stage buffers");
static_assert(DR_OUT_PER_RANK % 4 == 0 && DR_D % 4 == 0, "pushes are 4-output vectors of one rank and one head");

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

// Q^T of KV group kvh as the m16n8k16 B operand (k = dim, n = head): lane
// (gid, tig) holds head kvh*7 + gid, dims 16ks + 2tig (+1) and 16ks + 8 + 2tig
// (+1); head 7 of the tile is zero padding.
STD_DEV void draft_load_q(const DraftParams& p, int b, int kvh, int gid, int tig, uint32_t (&qb)[8][2]) {
  const bool hv = gid < DR_G;
  const __nv_bfloat16* qrow = p.q + (static_cast<size_t>(b) * p.Hq + kvh * DR_G + (hv ? gid : 0)) * DR_D;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    qb[ks][0] = hv ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 2 * tig) : 0u;
    qb[ks][1] = hv ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 8 + 2 * tig) : 0u;
  }
}

// NU (1 or 2) 16-key units of one warp -- rows kw .. kw+15 of the sub-tiles in
// sK[u] / sV[u], nvalid[u] of them live -- folded into the warp's online
// softmax state in one step (two units share one max, one rescale and
// interleaved MMA chains, so a pair costs little more latency than one).  Lane
// (gid, tig) keeps heads 2tig and 2tig+1: m_run / l_run per head (l_run over
// this lane's keys only; the lanes of a head are summed at the end) and
// o[mt] = O^T rows (dims) 16mt + gid and 16mt + gid + 8 of those two heads.
template <int NU>
STD_DEV void draft_units(const uint8_t* const (&sK)[NU], const uint8_t* const (&sV)[NU], const int (&nvalid)[NU],
                         int kw, const uint32_t (&qb)[8][2], float sc, int lane, float (&o)[8][4], float (&m_run)[2],
                         float (&l_run)[2]) {
  constexpr int NCH = 4 / NU;  // independent MMA chains per unit for S
  const int gid = lane >> 2, mi = lane >> 3;
  // S^T[16 keys x 8 heads] = K Q^T per unit; A = K rows (matrices: keys lo/hi x dims lo/hi)
  float s[NU][NCH][4];
#pragma unroll
  for (int u = 0; u < NU; ++u)
#pragma unroll
    for (int c = 0; c < NCH; ++c) s[u][c][0] = s[u][c][1] = s[u][c][2] = s[u][c][3] = 0.f;
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    uint32_t ka[8][4];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int key = kw + (mi & 1) * 8 + (lane & 7);
      const int c = 2 * ks + (mi >> 1);
      ldsm_x4(smem_u32(sK[u] + (c >> 3) * DR_HALF_BYTES + dr_sw(key, c & 7)), ka[ks][0], ka[ks][1], ka[ks][2],
              ka[ks][3]);
    }
#pragma unroll
    for (int ks = 0; ks < 8; ++ks)
      mma_bf16_16816(s[u][ks % NCH], ka[ks][0], ka[ks][1], ka[ks][2], ka[ks][3], qb[ks][0], qb[ks][1]);
  }
  // V^T fragments of unit 0 (A operand of O^T += V^T P^T: dims x keys), loaded
  // before the softmax so their latency overlaps it
  uint32_t va[8][4];
  auto load_v = [&](int u) {
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int key = kw + (mi >> 1) * 8 + (lane & 7);
      const int c = 2 * mt + (mi & 1);
      ldsm_x4_trans(smem_u32(sV[u] + (c >> 3) * DR_HALF_BYTES + dr_sw(key, c & 7)), va[mt][0], va[mt][1],
                    va[mt][2], va[mt][3]);
    }
  };
  load_v(0);
  // online softmax: x[u][0], x[u][1] = key kw+gid of unit u, heads 2tig, 2tig+1;
  // x[u][2], x[u][3] = key kw+gid+8
  float x[NU][4];
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    float t[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      t[e] = s[u][0][e];
#pragma unroll
      for (int c = 1; c < NCH; ++c) t[e] += s[u][c][e];
    }
    x[u][0] = gid < nvalid[u] ? t[0] * sc : -INFINITY;
    x[u][1] = gid < nvalid[u] ? t[1] * sc : -INFINITY;
    x[u][2] = gid + 8 < nvalid[u] ? t[2] * sc : -INFINITY;
    x[u][3] = gid + 8 < nvalid[u] ? t[3] * sc : -INFINITY;
    mx0 = fmaxf(mx0, fmaxf(x[u][0], x[u][2]));
    mx1 = fmaxf(mx1, fmaxf(x[u][1], x[u][3]));
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);  // finite: key kw of unit 0 is live
  const float al0 = ex2_approx(m_run[0] - mn0), al1 = ex2_approx(m_run[1] - mn1);
  float ps0 = 0.f, ps1 = 0.f;
  uint32_t pb[NU][2];
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const float p0 = ex2_approx(x[u][0] - mn0), p1 = ex2_approx(x[u][1] - mn1);
    const float p2 = ex2_approx(x[u][2] - mn0), p3 = ex2_approx(x[u][3] - mn1);
    ps0 += p0 + p2;
    ps1 += p1 + p3;
    // P^T (k = key, n = head) as the B operand: transpose the
    // accumulator-layout 8x8 blocks (keys lo, keys hi)
    pb[u][0] = movmatrix_trans(pack_bf16x2(p0, p1));
    pb[u][1] = movmatrix_trans(pack_bf16x2(p2, p3));
  }
  l_run[0] = l_run[0] * al0 + ps0;
  l_run[1] = l_run[1] * al1 + ps1;
  m_run[0] = mn0;
  m_run[1] = mn1;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    o[mt][0] *= al0;
    o[mt][1] *= al1;
    o[mt][2] *= al0;
    o[mt][3] *= al1;
  }
  // O^T += V^T P^T
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    if (u > 0) load_v(u);
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
      mma_bf16_16816(o[mt], va[mt][0], va[mt][1], va[mt][2], va[mt][3], pb[u][0], pb[u][1]);
  }
}

// Rows past the live length inside a sub-tile's last box hold whatever the
// cache holds there: zero V rows kw+nvalid .. kw+15 so that P = 0 times them
// stays 0.
STD_DEV void draft_zero_tail_v(uint8_t* sV, int kw, int nvalid, int lane) {
  for (int e = lane; e < (16 - nvalid) * 16; e += 32) {
    const int r = kw + nvalid + (e >> 4), c = e & 15;
    *reinterpret_cast<uint4*>(sV + (c >> 3) * DR_HALF_BYTES + r * 128 + ((c & 7) << 4)) = make_uint4(0u, 0u, 0u, 0u);
  }
  fence_async_smem();
  __syncwarp();
}

// The units a warp of group grp folds in at loop step i0 (sub-tiles are taken
// in pairs: group g takes i0 + g), except that an odd count of sub-tiles ends
// with three, of which group 0 takes the first and the third together.
// Returns the second sub-tile of that pair, or -1.
STD_DEV int draft_pair_of(int nsub, int i0, int grp) { return (nsub - i0 == 3 && grp == 0) ? i0 + 2 : -1; }

// What every rank of a cluster receives from the others: its output slice of
// each rank's CTA partial, and (m, l) of the heads that slice covers.  The
// senders write it with st.async, which completes transaction bytes on `bar`,
// so the receiver learns of its arrival by waiting on its own barrier.
struct DraftRecv {
  float o[DR_CLUSTER][DR_OUT_PER_RANK];
  float ml[DR_CLUSTER][DR_G][2];
  uint64_t bar;
};

// Keys [k0, k1) of cluster rank `rank`: shares of `per` keys, a multiple of
// 16 (the TMA box height), the last rank also taking the remainder; `per` is
// floor(L/8) rounded down or up to 16, whichever gives the smaller largest
// share (L = 1025: 7 x 128 + 129 rather than 7 x 144 + 17).
STD_DEV void draft_split(int L, int rank, int& k0, int& k1) {
  const int dn = (L / DR_CLUSTER) & ~15, up = dn + 16;
  const int load_dn = dn > 0 ? max(dn, L - (DR_CLUSTER - 1) * dn) : L;
  const int per = (dn > 0 && load_dn <= up) ? dn : up;
  k0 = min(L, rank * per);
  k1 = rank == DR_CLUSTER - 1 ? L : min(L, k0 + per);
}

// heads whose 128 outputs overlap output slice q ([112 q, 112 q + 112))
STD_DEV int draft_slice_head0(int q) { return (q * DR_OUT_PER_RANK) / DR_D; }
STD_DEV int draft_slice_head1(int q) { return (q * DR_OUT_PER_RANK + DR_OUT_PER_RANK - 1) / DR_D; }

// Thread 0, before the cluster's first barrier arrive: the receive barrier
// expects one slice and its heads' (m, l) from each of the DR_CLUSTER ranks.
STD_DEV void draft_recv_init(DraftRecv& rv, int rank) {
  const int nh = draft_slice_head1(rank) - draft_slice_head0(rank) + 1;
  mbar_init(&rv.bar, 1);
  mbar_arrive_expect_tx(&rv.bar, static_cast<uint32_t>(DR_CLUSTER * (DR_OUT_PER_RANK * 4 + nh * 8)));
}

// Combine the 8 warp partials of this CTA, push them to the ranks that finish
// each output slice (asynchronous DSMEM stores), and finish this rank's slice
// once every rank's push has landed.
STD_DEV void draft_finish(int rank, int b, int kvh, uint8_t* sbase, const DraftParams& p, float (&o)[8][4],
                          float (&m_run)[2], float (&l_run)[2], bool ok, DraftRecv& rv) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  // warp partials -> shared memory (the stage buffers are free now)
  float* wo = reinterpret_cast<float*>(sbase);  // [warp][8 heads][DR_OSTRIDE]
  float* wm = wo + DR_WARPS * 8 * DR_OSTRIDE;   // [warp][8]
  float* wl = wm + DR_WARPS * 8;                // [warp][8]
#pragma unroll
  for (int e = 0; e < 2; ++e) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], off);
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int h = 2 * tig + e;
    if (h < DR_G) {
      float* row = wo + (warp * 8 + h) * DR_OSTRIDE;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        row[16 * mt + gid] = o[mt][e];
        row[16 * mt + gid + 8] = o[mt][2 + e];
      }
      if (gid == 0) {
        wm[warp * 8 + h] = (l_run[e] > 0.f && ok) ? m_run[e] : -INFINITY;
        wl[warp * 8 + h] = ok ? l_run[e] : 0.f;
      }
    }
  }
  __syncthreads();
  // per head: M = max over warps, the warps' weights exp2(m_w - M) and the
  // weighted sum of their l
  float* wt = wl + DR_WARPS * 8;  // [warp][8]
  float* hm = wt + DR_WARPS * 8;  // [0, 8): M, [8, 16): l
  if (tid < DR_G) {
    const int h = tid;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < DR_WARPS; ++w) M = fmaxf(M, wm[w * 8 + h]);
    float lsum = 0.f;
#pragma unroll
    for (int w = 0; w < DR_WARPS; ++w) {
      const float x = M == -INFINITY ? 0.f : ex2_approx(wm[w * 8 + h] - M);  // 0 for a warp without keys
      wt[w * 8 + h] = x;
      lsum += x * wl[w * 8 + h];
    }
    hm[h] = M;
    hm[8 + h] = lsum;
  }
  __syncthreads();
  // every rank has initialised its receive barrier (it arrived after that)
  cluster_wait_acquire();
  const uint32_t bar_local = smem_u32(&rv.bar);
  // CTA partial of outputs idx .. idx+3 (idx = 4 tid = h*128 + d), pushed as
  // one vector to the rank that finishes them; (M, l) of head h to each rank
  // whose slice covers part of h (at most two)
  if (tid < DR_G * DR_D / 4) {
    const int idx = 4 * tid, h = idx / DR_D, d = idx % DR_D;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < DR_WARPS; ++w) {
      const float x = wt[w * 8 + h];
      const float4 v = *reinterpret_cast<const float4*>(wo + (w * 8 + h) * DR_OSTRIDE + d);
      acc.x += x * v.x;
      acc.y += x * v.y;
      acc.z += x * v.z;
      acc.w += x * v.w;
    }
    const int q = idx / DR_OUT_PER_RANK;
    st_async_v4f32(mapa_rank(smem_u32(&rv.o[rank][idx % DR_OUT_PER_RANK]), q), acc, mapa_rank(bar_local, q));
  } else if (tid < DR_G * DR_D / 4 + 2 * DR_G) {
    const int h = (tid - DR_G * DR_D / 4) >> 1;
    const int t = h * DR_D / DR_OUT_PER_RANK + ((tid - DR_G * DR_D / 4) & 1);
    if (t <= (h * DR_D + DR_D - 1) / DR_OUT_PER_RANK)
      st_async_v2f32(mapa_rank(smem_u32(&rv.ml[rank][h][0]), t), hm[h], hm[8 + h], mapa_rank(bar_local, t));
  }
  // Rank r finishes outputs [112 r, 112 r + 112) of the group's 7 x 128 from
  // the 8 partials in its own shared memory.  No rank exits before its own
  // barrier completes, i.e. before every store into its memory has landed.
  if (tid < DR_OUT_PER_RANK) {
    mbar_wait(&rv.bar, 0);
    const int idx = rank * DR_OUT_PER_RANK + tid;
    const int g = idx / DR_D, d = idx % DR_D;
    float mr[DR_CLUSTER], lr[DR_CLUSTER], orr[DR_CLUSTER];
#pragma unroll
    for (int r = 0; r < DR_CLUSTER; ++r) {
      mr[r] = rv.ml[r][g][0];
      lr[r] = rv.ml[r][g][1];
      orr[r] = rv.o[r][tid];
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
    draft_attn_kernel(const __grid_constant__ CUtensorMap tk64, const __grid_constant__ CUtensorMap tv64,
                      const __grid_constant__ CUtensorMap tk16, const __grid_constant__ CUtensorMap tv16,
                      const DraftParams p) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  extern __shared__ uint8_t dsmem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bar[DR_STAGES];
  __shared__ __align__(16) DraftRecv rv;
  // After an append (the decode step's RoPE + KV-append kernel, which writes
  // only q and the K/V row at position L-1): the lengths and every older K/V
  // row are read while that kernel may still run; q and row L-1 only after
  // griddepcontrol.wait.  Otherwise nothing is read before the wait.
  const bool early = (p.flags & 1) != 0;
  int L = early ? p.lens[b] + p.len_offset : 0;
  if (tid == 0) {
    prefetch_tensormap(&tk64);
    prefetch_tensormap(&tv64);
    prefetch_tensormap(&tk16);
    prefetch_tensormap(&tv16);
#pragma unroll
    for (int s = 0; s < DR_STAGES; ++s) mbar_init(&bar[s], 1);
    draft_recv_init(rv, rank);
    fence_barrier_init();
  }
  // Every CTA of the cluster must have initialised its receive barrier before
  // another pushes into it: arrive now (relaxed: the init fence above orders
  // the initialisation), wait just before the first push (by then the wait
  // returns at once).
  cluster_arrive_relaxed();
  if (!early) {
    pdl_wait();
    pdl_launch_dependents();
    L = p.lens[b] + p.len_offset;
  }
  if (L > p.cap || L < 0) {
    if (rank == 0 && tid == 0) std_set_error(STD_DEVERR_LENGTH);
    L = L < 0 ? 0 : p.cap;
  }
  int k0, k1;
  draft_split(L, rank, k0, k1);
  const int nkeys = k1 - k0;
  const int nsub = (nkeys + DR_SUB - 1) / DR_SUB;
  const int row0 = (b * p.Hkv + kvh) * p.cap + k0;  // first tensor-map row of this CTA
  // early mode: the 16-row box holding row L-1 waits for the append
  int defer_i = -1, defer_j = -1;
  if (early && L - 1 >= k0 && L - 1 < k1) {
    defer_i = (L - 1 - k0) / DR_SUB;
    defer_j = ((L - 1 - k0) % DR_SUB) / DR_BOX;
  }

  __syncthreads();  // the stage barriers are initialised
  // Sub-tile i is issued by thread DR_ISSUER: a full sub-tile (64 live keys) as one
  // 64-row box per K/V half, a partial one -- or the one holding the deferred
  // row -- as 16-row boxes (both give the same shared-memory layout).  One
  // thread with few large boxes: a copy instruction with per-lane coordinates
  // issues its lanes one after another.
  // mode 0: the whole sub-tile; 1: all but the deferred box; 2: only that box
  auto issue = [&](int i, int mode) {
    const int st = i % DR_STAGES;
    const int a = i * DR_SUB;
    const int nk = min(DR_SUB, nkeys - a);
    const int nbox = (nk + DR_BOX - 1) / DR_BOX;
    uint8_t* s = sbase + st * DR_STAGE_BYTES;
    const uint64_t pol = l2_policy_evict_first();  // each K/V row is read once per forward
    if (mode != 2) mbar_arrive_expect_tx(&bar[st], static_cast<uint32_t>(nbox) * 4u * DR_BOX * 128u);
    if (nk == DR_SUB && i != defer_i) {
      if (mode != 2) {
#pragma unroll
        for (int part = 0; part < 4; ++part)
          tma_load_2d_hint(s + (part & 1) * DR_HALF_BYTES + (part >> 1) * 2 * DR_HALF_BYTES,
                           part < 2 ? &tk64 : &tv64, &bar[st], (part & 1) * 64, row0 + a, pol);
      }
      return;
    }
    for (int j = 0; j < nbox; ++j) {
      const bool is_deferred = i == defer_i && j == defer_j;
      if (mode == 0 || (mode == 1) != is_deferred) {
#pragma unroll
        for (int part = 0; part < 4; ++part)
          tma_load_2d_hint(s + j * DR_BOX * 128 + (part & 1) * DR_HALF_BYTES + (part >> 1) * 2 * DR_HALF_BYTES,
                           part < 2 ? &tk16 : &tv16, &bar[st], (part & 1) * 64, row0 + a + j * DR_BOX, pol);
      }
    }
  };
  // sub-tiles issued so far: the same value in every thread (the issuer
  // issues), so the block-wide barriers below that depend on it are uniform
  int issued = min(DR_STAGES, nsub);
  int issued_real = issued;  // what the issuer really issued (differs only after a wait gave up)
  if (tid == DR_ISSUER) {
    for (int i = 0; i < issued; ++i) issue(i, early ? 1 : 0);
  }
  if (early) {
    pdl_launch_dependents();  // the decode step's O projection GEMM: weights before its wait
    pdl_wait();
    if (tid == DR_ISSUER && defer_i >= 0 && defer_i < issued) issue(defer_i, 2);
  }

  uint32_t qb[8][2];
  draft_load_q(p, b, kvh, gid, tig, qb);

  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  bool ok = true;
  const float sc = p.scale_log2;
  const int grp = warp >> 2, kw = (warp & 3) * 16;

  // Iteration j: group 0 takes sub-tile 2j, group 1 sub-tile 2j+1; then the
  // two stages they free are refilled with the next two sub-tiles.  A stage's
  // previous phase was consumed before the refill that reuses it, so a wait can
  // never see the parity of a phase older than the one it waits for.  An odd
  // count ends with three sub-tiles in one iteration (draft_pair_of).
  for (int i0 = 0; i0 < nsub; i0 += 2) {
    const int i = i0 + grp;
    if (i < nsub) {
      const int ib = draft_pair_of(nsub, i0, grp);
      if (ok) ok = mbar_wait(&bar[i % DR_STAGES], (i / DR_STAGES) & 1);
      if (ok && ib >= 0) ok = mbar_wait(&bar[ib % DR_STAGES], (ib / DR_STAGES) & 1);
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform: guards warp-collective code below
      uint8_t* sK0 = sbase + (i % DR_STAGES) * DR_STAGE_BYTES;
      const int nv0 = min(16, min(DR_SUB, nkeys - i * DR_SUB) - kw);
      const int nv1 = ib >= 0 ? min(16, min(DR_SUB, nkeys - ib * DR_SUB) - kw) : 0;
      if (nv0 > 0 && ok) {
        if (nv0 < 16) draft_zero_tail_v(sK0 + 2 * DR_HALF_BYTES, kw, nv0, lane);
        if (nv1 > 0) {
          uint8_t* sK1 = sbase + (ib % DR_STAGES) * DR_STAGE_BYTES;
          if (nv1 < 16) draft_zero_tail_v(sK1 + 2 * DR_HALF_BYTES, kw, nv1, lane);
          const uint8_t* const k2[2] = {sK0, sK1};
          const uint8_t* const v2[2] = {sK0 + 2 * DR_HALF_BYTES, sK1 + 2 * DR_HALF_BYTES};
          const int n2[2] = {nv0, nv1};
          draft_units<2>(k2, v2, n2, kw, qb, sc, lane, o, m_run, l_run);
        } else {
          const uint8_t* const k1[1] = {sK0};
          const uint8_t* const v1[1] = {sK0 + 2 * DR_HALF_BYTES};
          const int n1[1] = {nv0};
          draft_units<1>(k1, v1, n1, kw, qb, sc, lane, o, m_run, l_run);
        }
      }
    }
    if (nsub - i0 == 3) break;  // uniform: the last three sub-tiles are consumed
    if (issued < nsub) {        // uniform: a refill follows
      __syncthreads();          // both groups are done with their stages
      if (warp == DR_ISSUER / 32) {
        const bool warp_ok = __all_sync(0xffffffffu, ok);
        if (lane == 0 && warp_ok) {
          issue(issued, 0);
          if (issued + 1 < nsub) issue(issued + 1, 0);
          issued_real = min(nsub, issued + 2);
        }
      }
      issued = min(nsub, issued + 2);
    }
  }
  if (!__syncthreads_and(ok)) {
    // A wait gave up: let the loads still in flight land before the stage
    // buffers are reused or the CTA exits; these waits are bounded too.
    if (tid == DR_ISSUER) {
      for (int i = max(0, issued_real - DR_STAGES); i < issued_real; ++i)
        mbar_wait(&bar[i % DR_STAGES], (i / DR_STAGES) & 1);
    }
    __syncthreads();
  }

  draft_finish(rank, b, kvh, sbase, p, o, m_run, l_run, ok, rv);
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
  extern __shared__ uint8_t dsmem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(16) DraftRecv rv;
  if (tid == 0) {
    draft_recv_init(rv, rank);
    fence_barrier_init();
  }
  cluster_arrive_relaxed();
  pdl_wait();
  pdl_launch_dependents();

  int L = p.lens[b] + p.len_offset;
  if (L > p.cap || L < 0) {
    if (rank == 0 && tid == 0) std_set_error(STD_DEVERR_LENGTH);
    L = L < 0 ? 0 : p.cap;
  }
  int k0, k1;
  draft_split(L, rank, k0, k1);
  const int nkeys = k1 - k0;
  const int nsub = (nkeys + DR_SUB - 1) / DR_SUB;
  const size_t head = static_cast<size_t>(b) * p.Hkv + kvh;

  // thread t gathers chunks 4(t&3) .. 4(t&3)+3 (of the 16 per 256-byte row) of
  // row t >> 2 of a 64-row sub-tile, K and V
  auto issue = [&](int i) {
    if (i >= nsub) return;
    const int st = i % DR_STAGES;
    const int r = tid >> 2, qd = tid & 3;
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
    for (int e = 0; e < 4; ++e) {
      const int c = 4 * qd + e;  // 16-byte chunk of the row: half c >> 3
      const uint32_t off = (c >> 3) * DR_HALF_BYTES + dr_sw(r, c & 7);
      cp_async16(sK + off, srcK + c * 8, nbytes);
      cp_async16(sV + off, srcV + c * 8, nbytes);
    }
  };
#pragma unroll
  for (int i = 0; i < DR_STAGES; ++i) {
    issue(i);
    cp_async_commit();
  }

  uint32_t qb[8][2];
  draft_load_q(p, b, kvh, gid, tig, qb);
  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int grp = warp >> 2, kw = (warp & 3) * 16;

  // Iteration j: group 0 takes sub-tile 2j, group 1 sub-tile 2j+1 (the
  // assignment of the TMA kernel, so both give the same bytes).  Groups of
  // copies are committed one per sub-tile: before iteration j, sub-tiles up
  // to 2j+2 are committed and 2j, 2j+1 must have landed.
  for (int i0 = 0; i0 < nsub; i0 += 2) {
    const bool last3 = nsub - i0 == 3;  // uniform
    if (last3)
      cp_async_wait<0>();  // this thread's copies of sub-tiles i0 .. i0+2 have landed
    else
      cp_async_wait<1>();  // this thread's copies of sub-tiles i0, i0+1 have landed
    __syncthreads();       // ... and every other thread's
    const int i = i0 + grp;
    if (i < nsub) {
      const int ib = draft_pair_of(nsub, i0, grp);
      const uint8_t* sK0 = sbase + (i % DR_STAGES) * DR_STAGE_BYTES;
      const int nv0 = min(16, min(DR_SUB, nkeys - i * DR_SUB) - kw);
      const int nv1 = ib >= 0 ? min(16, min(DR_SUB, nkeys - ib * DR_SUB) - kw) : 0;
      if (nv0 > 0 && nv1 > 0) {
        const uint8_t* sK1 = sbase + (ib % DR_STAGES) * DR_STAGE_BYTES;
        const uint8_t* const k2[2] = {sK0, sK1};
        const uint8_t* const v2[2] = {sK0 + 2 * DR_HALF_BYTES, sK1 + 2 * DR_HALF_BYTES};
        const int n2[2] = {nv0, nv1};
        draft_units<2>(k2, v2, n2, kw, qb, p.scale_log2, lane, o, m_run, l_run);
      } else if (nv0 > 0) {
        const uint8_t* const k1[1] = {sK0};
        const uint8_t* const v1[1] = {sK0 + 2 * DR_HALF_BYTES};
        const int n1[1] = {nv0};
        draft_units<1>(k1, v1, n1, kw, qb, p.scale_log2, lane, o, m_run, l_run);
      }
    }
    if (last3) break;
    __syncthreads();  // stages of i0, i0+1 are free
    issue(i0 + DR_STAGES);
    cp_async_commit();
    issue(i0 + DR_STAGES + 1);
    cp_async_commit();
  }
  cp_async_wait<0>();  // nothing in flight into the stage buffers
  __syncthreads();
  draft_finish(rank, b, kvh, sbase, p, o, m_run, l_run, true, rv);
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
  static SmemGrant grant;
  if (ensure_smem(stdb::draft_attn_kernel, grant, stdb::DR_SMEM, true) != 0) return 3;
  CUtensorMap tk64, tv64, tk16, tv16;
  int rc = make_tmap_bf16_2d(&tk64, k_cache, static_cast<uint64_t>(rows), 128, 256, 64, stdb::DR_SUB);
  if (rc == 0) rc = make_tmap_bf16_2d(&tv64, v_cache, static_cast<uint64_t>(rows), 128, 256, 64, stdb::DR_SUB);
  if (rc == 0) rc = make_tmap_bf16_2d(&tk16, k_cache, static_cast<uint64_t>(rows), 128, 256, 64, stdb::DR_BOX);
  if (rc == 0) rc = make_tmap_bf16_2d(&tv16, v_cache, static_cast<uint64_t>(rows), 128, 256, 64, stdb::DR_BOX);
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
                    static_cast<cudaStream_t>(stream), tk64, tv64, tk16, tv16, p) == cudaSuccess
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
  static SmemGrant grant;
  if (ensure_smem(stdb::draft_attn_indexed_kernel, grant, stdb::DR_SMEM, true) != 0) return 3;
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
