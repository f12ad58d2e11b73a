// Single-query attention for the decode step, split over a thread-block
// cluster (split-K flash decode) with the reference's rounding points.
//
// One cluster of C CTAs serves one (row, head); CTA `rank` takes keys
// [rank*chunk, min(L, (rank+1)*chunk)).  The reference evaluates
// (engine.py:286-292)
//     s = bf16(q . k) * 1/8            (bf16 matmul, then a bf16 scale)
//     p = bf16(softmax_fp32(s + bias))
//     o = bf16(sum_j p_j v_j)          (fp32 accumulation)
// so a split must know the global max and sum before rounding p.  The CTAs
// exchange their partial max and partial sum through distributed shared
// memory (two cluster barriers), then each accumulates p v over its keys and
// rank 0 adds the C partial outputs in rank order.  Keys beyond the visible
// length are never read; the reference masks them with -inf, which gives the
// same softmax.
//   self  (engine.py:303-312): keys 0..position of the slot, paged pool
//   cross (engine.py:134,208-209,313): the slot's first `frames` encoder frames
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace s2r {

namespace cg = cooperative_groups;

struct AttnArgs {
  int M, H;
  RowMap rm;
  SlotState st;
  const bf16* q;  // [M, ldq]
  int ldq;
  bf16* out;  // [M, ldo]
  int ldo;
  int cross;
  const bf16* k;  // self: paged pool [pages, H, 64, 64]; cross: [batch, H, frames_cap, 64]
  const bf16* v;
  int pages_per_slot;
  int frames_cap;
  int chunk_cap;  // score buffer length per CTA
  int splits;     // CTAs per (row, head): the cluster size the launch must have
  int* err;       // device error word: set (and the work skipped) on a broken invariant
  const int32_t* order;  // [M] row of each grid z index (longest first), or null: identity
};

constexpr int kErrAttnCluster = 1;  // launched without the expected cluster shape
constexpr int kErrAttnChunk = 2;    // a row's keys do not fit the score buffer

constexpr int kAttnThreads = 256;
constexpr int kAttnGroups = kAttnThreads / 8;  // 8 lanes x 16 bytes per key row
constexpr int kAttnUnroll = 4;

__device__ __forceinline__ const bf16* attn_row(const AttnArgs& a, const bf16* base, int slot, int h, int j) {
  if (a.cross) return base + (((size_t)slot * a.H + h) * a.frames_cap + j) * kHeadDim;
  return base + paged_offset(a.st.page_table, a.pages_per_slot, a.H, slot, h, j);
}

// kPrefetch: the first pass of keys and values (kAttnGroups * kAttnUnroll
// keys of the CTA's range) is loaded into registers before the kernel waits
// for the previous kernel, except the keys written during the launch's own
// step (the rows' own positions).  That is safe because the first kernel of
// every decode step and prefill chunk starts only after everything before it
// has completed.  Used by engines below 16 slots, whose CTAs see one or two
// passes of keys; the batched engines keep the registers for occupancy.
template <bool kPrefetch>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnArgs a) {
  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.dim_blocks().x;
  const int rank = (int)cluster.block_rank();
  const int h = blockIdx.y, m = a.order ? a.order[blockIdx.z] : (int)blockIdx.z;
  extern __shared__ __align__(16) float smem_f[];
  float* sc = smem_f;                                 // [chunk_cap] scores, then exp values
  float* part = smem_f + ((a.chunk_cap + 3) & ~3);    // [kAttnGroups][64] partial outputs
  __shared__ float red[2];                            // this CTA's max and sum
  __shared__ float wred[kAttnThreads / 32];
  __shared__ float ovec[kHeadDim];

  pdl_launch_dependents();
  const int tid = threadIdx.x, grp = tid >> 3, sub = tid & 7;
  const int lane = tid & 31, warp = tid >> 5;
  // The whole cluster sees the same row and the same launch shape, so every
  // early return below is taken by all of its CTAs together.
  if (C != a.splits) {
    if (threadIdx.x == 0) atomicExch(a.err, kErrAttnCluster);
    return;
  }
  // the slot state read here was written before the step began
  if (!row_active(a.rm, a.st, m)) return;
  const int slot = row_slot(a.rm, m);
  const int L = a.cross ? a.st.frames[slot] : row_pos(a.rm, a.st, m) + 1;
  const int chunk = (L + C - 1) / C;
  if (chunk > a.chunk_cap) {
    if (threadIdx.x == 0) atomicExch(a.err, kErrAttnChunk);
    return;
  }
  const int j0 = min(L, rank * chunk), j1 = min(L, j0 + chunk);
  // keys at or after `fresh` are written during this step (the rows' own positions)
  const int fresh = a.cross ? L : (a.rm.prefill ? a.rm.pos0 : row_pos(a.rm, a.st, m));
  uint4 kpre[kAttnUnroll], vpre[kAttnUnroll];
  if constexpr (kPrefetch) {
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const int j = j0 + grp + u * kAttnGroups;
      const bool ok = j < j1 && j < fresh;
      kpre[u] = ok ? ld_stream(attn_row(a, a.k, slot, h, j) + sub * 8) : make_uint4(0, 0, 0, 0);
      vpre[u] = ok ? ld_stream(attn_row(a, a.v, slot, h, j) + sub * 8) : make_uint4(0, 0, 0, 0);
    }
  }
  pdl_wait();

  const uint4 qraw = *reinterpret_cast<const uint4*>(a.q + (size_t)m * a.ldq + h * kHeadDim + sub * 8);

  // ---- scores and local max
  float lmax = -INFINITY;
  // The loop bound is uniform across the block (the shuffles below need all lanes).
  for (int base = j0; base < j1; base += kAttnGroups * kAttnUnroll) {
    const int jb = base + grp;
    uint4 kv[kAttnUnroll];
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const int j = jb + u * kAttnGroups;
      if (kPrefetch && base == j0 && j < fresh)
        kv[u] = kpre[u];
      else
        kv[u] = j < j1 ? ld_stream(attn_row(a, a.k, slot, h, j) + sub * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const int j = jb + u * kAttnGroups;
      float s = bf_lo(kv[u].x) * bf_lo(qraw.x);
      s = fmaf(bf_hi(kv[u].x), bf_hi(qraw.x), s);
      s = fmaf(bf_lo(kv[u].y), bf_lo(qraw.y), s);
      s = fmaf(bf_hi(kv[u].y), bf_hi(qraw.y), s);
      s = fmaf(bf_lo(kv[u].z), bf_lo(qraw.z), s);
      s = fmaf(bf_hi(kv[u].z), bf_hi(qraw.z), s);
      s = fmaf(bf_lo(kv[u].w), bf_lo(qraw.w), s);
      s = fmaf(bf_hi(kv[u].w), bf_hi(qraw.w), s);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      if (j < j1) {
        s = round_bf16(s) * 0.125f;  // head_dim ** -0.5 for head_dim 64
        if (sub == 0) sc[j - j0] = s;
        lmax = fmaxf(lmax, s);
      }
    }
  }
  lmax = warp_max(lmax);
  if (lane == 0) wred[warp] = lmax;
  __syncthreads();
  if (tid == 0) {
    float v = wred[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) v = fmaxf(v, wred[w]);
    red[0] = v;
  }
  cluster.sync();
  float gmax = -INFINITY;
  for (int r = 0; r < C; ++r) gmax = fmaxf(gmax, *cluster.map_shared_rank(&red[0], r));

  // ---- exp and local sum
  float lsum = 0.f;
  for (int j = j0 + tid; j < j1; j += kAttnThreads) {
    const float e = expf(sc[j - j0] - gmax);
    sc[j - j0] = e;
    lsum += e;
  }
  lsum = warp_sum(lsum);
  if (lane == 0) wred[warp] = lsum;
  __syncthreads();
  if (tid == 0) {
    float v = 0.f;
    for (int w = 0; w < kAttnThreads / 32; ++w) v += wred[w];
    red[1] = v;
  }
  cluster.sync();
  float gsum = 0.f;
  for (int r = 0; r < C; ++r) gsum += *cluster.map_shared_rank(&red[1], r);

  // ---- p = bf16(e / sum), partial p.V
  float acc[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) acc[t] = 0.f;
  for (int base = j0; base < j1; base += kAttnGroups * kAttnUnroll) {
    const int jb = base + grp;
    uint4 vv[kAttnUnroll];
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const int j = jb + u * kAttnGroups;
      if (kPrefetch && base == j0 && j < fresh)
        vv[u] = vpre[u];
      else
        vv[u] = j < j1 ? ld_stream(attn_row(a, a.v, slot, h, j) + sub * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const int j = jb + u * kAttnGroups;
      const float p = j < j1 ? round_bf16(sc[j - j0] / gsum) : 0.f;
      acc[0] = fmaf(p, bf_lo(vv[u].x), acc[0]);
      acc[1] = fmaf(p, bf_hi(vv[u].x), acc[1]);
      acc[2] = fmaf(p, bf_lo(vv[u].y), acc[2]);
      acc[3] = fmaf(p, bf_hi(vv[u].y), acc[3]);
      acc[4] = fmaf(p, bf_lo(vv[u].z), acc[4]);
      acc[5] = fmaf(p, bf_hi(vv[u].z), acc[5]);
      acc[6] = fmaf(p, bf_lo(vv[u].w), acc[6]);
      acc[7] = fmaf(p, bf_hi(vv[u].w), acc[7]);
    }
  }
#pragma unroll
  for (int t = 0; t < 8; ++t) part[grp * kHeadDim + sub * 8 + t] = acc[t];
  __syncthreads();
  if (tid < kHeadDim) {
    float o = 0.f;
    for (int g = 0; g < kAttnGroups; ++g) o += part[g * kHeadDim + tid];
    ovec[tid] = o;
  }
  cluster.sync();
  if (rank == 0 && tid < kHeadDim) {
    float o = 0.f;
    for (int r = 0; r < C; ++r) o += cluster.map_shared_rank(ovec, r)[tid];
    a.out[(size_t)m * a.ldo + h * kHeadDim + tid] = __float2bfloat16_rn(o);
  }
  cluster.sync();  // peers keep their shared memory until rank 0 has read it
}

}  // namespace s2r
