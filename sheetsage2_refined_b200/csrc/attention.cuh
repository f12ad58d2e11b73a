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
  // kFuseOut: the out-projection, residual and LayerNorm that follow the attention
  int D;
  const bf16* wo;            // out-projection weight [D, D]
  const bf16* bo;            // its bias [D]
  const float *ln_g, *ln_b;  // the LayerNorm after the residual sum
  float* part;               // [H][M][D] out-projection partial sums by head
  unsigned* ticket;          // [M] arrivals per row, zero between launches
  float* x;                  // [M][D] float32: residual input, then the LayerNorm output
  bf16* xn;                  // [M][D] the LayerNorm output in bf16 (the next projection's input)
};

constexpr int kAttnOutPrefetch = 4;  // out-projection passes (32 features each) loaded before the wait

constexpr int kErrAttnCluster = 1;  // launched without the expected cluster shape
constexpr int kErrAttnChunk = 2;    // a row's keys do not fit the score buffer

constexpr int kAttnThreads = 256;
constexpr int kAttnGroups = kAttnThreads / 8;  // 8 lanes x 16 bytes per key row
constexpr int kAttnUnroll = 4;

__device__ __forceinline__ uint32_t pack_bf16_pair(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

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
//
// kFuseOut (engines below 16 slots): the kernel also runs what follows the
// attention in the reference (engine.py:312-313):
//     r = x + bf16(o @ Wo^T + bo),   x = LayerNorm(r)
// Every CTA of the head's cluster adds the C partial outputs in rank order
// (the same o in each), then computes its 1/C of the output features of the
// head's share of the out-projection, sum_d Wo[n][64h + d] o[d], as a float32
// partial sum over the head (the weights are loaded before the PDL wait).  The
// last CTA of the row (a ticket counter) adds the partials of all heads in
// head order, the bias and the residual, rounds as the reference does, and
// writes the LayerNorm output as float32 (the next residual input) and bf16
// (the next projection's input).
template <bool kPrefetch, bool kFuseOut>
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
  __shared__ float ohead[kHeadDim];                   // kFuseOut: the head's output, bf16-rounded
  __shared__ int is_last;

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
  // kFuseOut: this CTA's out-projection features and their weights for head h
  const int per = kFuseOut ? (a.D + C - 1) / C : 0, n0 = rank * per;
  uint4 wpre[kAttnOutPrefetch];
  if constexpr (kFuseOut) {
#pragma unroll
    for (int p = 0; p < kAttnOutPrefetch; ++p) {
      const int i = p * kAttnGroups + grp, n = n0 + i;
      wpre[p] = (i < per && n < a.D) ? ld_stream(a.wo + (size_t)n * a.D + h * kHeadDim + sub * 8) : make_uint4(0, 0, 0, 0);
    }
  }
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
  if constexpr (!kFuseOut) {
    if (rank == 0 && tid < kHeadDim) {
      float o = 0.f;
      for (int r = 0; r < C; ++r) o += cluster.map_shared_rank(ovec, r)[tid];
      a.out[(size_t)m * a.ldo + h * kHeadDim + tid] = __float2bfloat16_rn(o);
    }
    cluster.sync();  // peers keep their shared memory until rank 0 has read it
  } else {
    if (tid < kHeadDim) {
      float o = 0.f;
      for (int r = 0; r < C; ++r) o += cluster.map_shared_rank(ovec, r)[tid];
      ohead[tid] = round_bf16(o);  // the attention output is bf16 (engine.py:292)
    }
    cluster.sync();  // every CTA has its o; peers may leave
    float oh[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) oh[t] = ohead[sub * 8 + t];
    auto emit = [&](int p, uint4 w) {  // features of pass p: 32 of them, one per group of 8 lanes
      const int i = p * kAttnGroups + grp, n = n0 + i;
      float d = bf_lo(w.x) * oh[0];
      d = fmaf(bf_hi(w.x), oh[1], d);
      d = fmaf(bf_lo(w.y), oh[2], d);
      d = fmaf(bf_hi(w.y), oh[3], d);
      d = fmaf(bf_lo(w.z), oh[4], d);
      d = fmaf(bf_hi(w.z), oh[5], d);
      d = fmaf(bf_lo(w.w), oh[6], d);
      d = fmaf(bf_hi(w.w), oh[7], d);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      if (i < per && n < a.D && sub == 0) a.part[((size_t)h * a.M + m) * a.D + n] = d;
    };
    // pass counts are uniform across the block: the shuffles need every lane
#pragma unroll
    for (int p = 0; p < kAttnOutPrefetch; ++p)
      if (p * kAttnGroups < per) emit(p, wpre[p]);
    for (int p = kAttnOutPrefetch; p * kAttnGroups < per; ++p) {
      const int i = p * kAttnGroups + grp, n = n0 + i;
      emit(p, (i < per && n < a.D) ? ld_stream(a.wo + (size_t)n * a.D + h * kHeadDim + sub * 8) : make_uint4(0, 0, 0, 0));
    }
    // ---- the last CTA of the row: residual sum and LayerNorm
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(a.ticket + m, 1u) == (unsigned)(a.H * C) - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    if (tid == 0) a.ticket[m] = 0u;
    constexpr int kCols = 16;  // columns per thread (width <= 4096)
    float r[kCols];
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < kCols / 4; ++c) {
      const int col = c * 4 * kAttnThreads + tid * 4;
      float4 v4 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (col < a.D) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int hh = 0; hh < a.H; ++hh) {
          const float4 p4 = __ldcg(reinterpret_cast<const float4*>(a.part + ((size_t)hh * a.M + m) * a.D + col));
          acc.x += p4.x;
          acc.y += p4.y;
          acc.z += p4.z;
          acc.w += p4.w;
        }
        const float4 x4 = *reinterpret_cast<const float4*>(a.x + (size_t)m * a.D + col);
        v4.x = x4.x + round_bf16(acc.x + __bfloat162float(a.bo[col + 0]));
        v4.y = x4.y + round_bf16(acc.y + __bfloat162float(a.bo[col + 1]));
        v4.z = x4.z + round_bf16(acc.z + __bfloat162float(a.bo[col + 2]));
        v4.w = x4.w + round_bf16(acc.w + __bfloat162float(a.bo[col + 3]));
      }
      r[c * 4 + 0] = v4.x;
      r[c * 4 + 1] = v4.y;
      r[c * 4 + 2] = v4.z;
      r[c * 4 + 3] = v4.w;
      sum += (v4.x + v4.y) + (v4.z + v4.w);
    }
    // LayerNorm (two-pass, biased variance), block sums in fixed warp order
    sum = warp_sum(sum);
    if (lane == 0) wred[warp] = sum;
    __syncthreads();
    float mean = 0.f;
    for (int w = 0; w < kAttnThreads / 32; ++w) mean += wred[w];
    mean /= (float)a.D;
    __syncthreads();
    float sq = 0.f;
#pragma unroll
    for (int c = 0; c < kCols / 4; ++c) {
      if (c * 4 * kAttnThreads + tid * 4 < a.D) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float d = r[c * 4 + j] - mean;
          sq = fmaf(d, d, sq);
        }
      }
    }
    sq = warp_sum(sq);
    if (lane == 0) wred[warp] = sq;
    __syncthreads();
    float var = 0.f;
    for (int w = 0; w < kAttnThreads / 32; ++w) var += wred[w];
    const float rstd = rsqrtf(var / (float)a.D + kLnEps);
#pragma unroll
    for (int c = 0; c < kCols / 4; ++c) {
      const int col = c * 4 * kAttnThreads + tid * 4;
      if (col < a.D) {
        float y[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) y[j] = (r[c * 4 + j] - mean) * rstd * a.ln_g[col + j] + a.ln_b[col + j];
        *reinterpret_cast<float4*>(a.x + (size_t)m * a.D + col) = make_float4(y[0], y[1], y[2], y[3]);
        *reinterpret_cast<uint2*>(a.xn + (size_t)m * a.D + col) =
            make_uint2(pack_bf16_pair(y[0], y[1]), pack_bf16_pair(y[2], y[3]));
      }
    }
  }
}

}  // namespace s2r
