// One decode step as ONE persistent kernel, for up to 8 live rows.
//
// At batch 1 the multi-kernel step is bound by launch and dependency latency
// (97 kernels that each move 2-8 MB).  Here a grid of clusters of 4 CTAs (one
// CTA per SM) runs the whole step with three grid barriers per layer, the
// minimum for this decoder: every LayerNorm and every projection input needs
// the whole residual vector, and the residual needs every head or every FFN
// unit.  Inside a phase the exchanges stay in a cluster (distributed shared
// memory and cluster barriers):
//
//   phase A (cluster per head h): combine the previous FFN partial sums into
//     the residual, LayerNorm, the 192 q/k/v rows of head h, K/V append, self
//     attention of head h split over the cluster, and head h's share of the
//     out-projection, written as a partial sum over the head.
//   phase B (cluster per head h): combine the out-projection partials,
//     residual + self_attn_norm, cross q of head h, cross attention, cross
//     out-projection partial.
//   phase C (every CTA): combine, residual + cross_attn_norm, a slice of fc1
//     units + GELU, their fc2 contribution, reduced inside the cluster.
//   logits (every CTA): combine, residual + final_norm, a slice of the
//     vocabulary, grammar mask, argmax keys; the last CTA commits the step.
//
// Rounding follows the reference's CUDA path (engine.py:286-315) exactly as
// the multi-kernel path does; only float32 summation orders differ, and they
// are fixed, so the step is deterministic and a row's result does not depend
// on the other rows of the launch.
//
// Every wait is bounded.  A grid barrier that has not completed after 2 s
// records an error word; from then on no barrier waits (each sees the error
// word), the CTAs run the remaining phases without waiting and the commit is
// skipped, so every CTA takes the same cluster barriers and the kernel ends.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"
#include "logits.cuh"
#include "proj.cuh"

namespace s2r {

namespace cg = cooperative_groups;

constexpr int kPClus = 4;                      // CTAs per cluster (one head per cluster)
constexpr int kPThreads = 256;
constexpr int kPWarps = kPThreads / 32;
constexpr int kPMaxRows = 8;
constexpr int kQkvLocal = 3 * kHeadDim / kPClus;  // q/k/v rows of a head per CTA (48)
constexpr int kDimsLocal = kHeadDim / kPClus;     // head dims per CTA (16)
constexpr int kErrBarrier = 3;                    // a grid barrier timed out
constexpr unsigned long long kSpinNs = 2000000000ull;

struct PLayer {
  const bf16 *wqkv, *bqkv;  // [3D, D], [3D]
  const bf16 *woT, *bo;     // out-projection transposed [D_in, D_out]
  const bf16 *wcq, *bcq;    // [D, D]
  const bf16 *wcoT, *bco;   // cross out-projection transposed
  const bf16 *w1, *b1;      // [F, D]
  const bf16 *w2T, *b2;     // fc2 transposed [F, D]
  const float *ln_self_g, *ln_self_b, *ln_cross_g, *ln_cross_b, *ln_final_g, *ln_final_b;
  bf16 *kpool, *vpool;
  const bf16 *ck, *cv;
};

struct PArgs {
  int M;
  RowMap rm;
  SlotState st;
  Grammar gr;
  int D, H, FFN, V, L, T, F, pps;
  int units;       // fc1 units per CTA (phase C)
  int chunk_cap;   // attention scores per row per CTA
  int logits;      // 1: decode step (logits + commit); 0: prefill (K/V only)
  const PLayer* layers;
  const float *tok_emb, *pos_emb, *emb_g, *emb_b;
  const bf16* emb;
  const float* bias;
  float *part_o, *part_c, *part_f;  // [H][M][D], [H][M][D], [clusters][M][D]
  unsigned* bar;                    // [0] arrivals, [1] exits
  unsigned long long* keys;
  unsigned* counter;
  int* err;
  const int64_t* forced;
  float* logits_out;
  int64_t* greedy_out;
  int prefetch;      // issue next-phase L2 prefetches
  long long* trace;  // optional clock64 marks (rank 0 of the first kTraceCtas clusters)
};

constexpr int kTraceSlots = 512;
constexpr int kTraceCtas = 16;

__device__ __forceinline__ void trace_mark(const PArgs& a, int idx) {
  if (a.trace == nullptr || threadIdx.x != 0 || idx < 0 || idx >= kTraceSlots) return;
  const int b = blockIdx.x;
  const int which = (b % kPClus == 0 && b / kPClus < kTraceCtas) ? b / kPClus : -1;
  if (which >= 0) a.trace[which * kTraceSlots + idx] = clock64();
}

// L2-coherent loads (data written earlier in this launch by other SMs) and
// read-only weight loads.
__device__ __forceinline__ uint4 ld_cg(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ float4 ld_cg_f4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ uint4 ld_w(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void prefetch_bulk_l2(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Shared memory of one CTA (dynamic); sizes mirror persistent_smem() on the host.
struct PSmem {
  float* xk;    // [MR][D]  residual-stream value after LayerNorm (fp32)
  bf16* xs;     // [MR][KP] the same rounded to bf16, GEMV input
  float* y;     // [MR][D]  partial sums exchanged inside the cluster
  float* sc;    // [MR][chunk_cap] attention scores
  float* qh;    // [MR][64] the head's query
  float* kn;    // [MR][64] the head's new key (decode rows)
  float* vn;    // [MR][64] the head's new value
  float* loc;   // [MR][48] this CTA's q/k/v rows
  float* ov;    // [MR][64] partial attention output
  float* stat;  // [MR][2]  local max and sum
  float* av;    // [MR][16] this CTA's dims of the attention output
  float* hid;   // [MR][units] fc1 outputs
  float* red;   // [8][64]  reduction scratch
};

// Grid barrier: every CTA arrives on one counter and waits for all (bounded).
// Returns false once any CTA has recorded an error.
__device__ __forceinline__ bool grid_barrier(const PArgs& a, unsigned& target) {
  __shared__ int ok_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    __threadfence();
    atomicAdd(a.bar, 1u);
    int ok = 1;
    const unsigned long long t0 = global_ns();
    while (ld_acquire(a.bar) < target) {
      if (*(volatile int*)a.err != 0) {
        ok = 0;
        break;
      }
      if (global_ns() - t0 > kSpinNs) {
        atomicExch(a.err, kErrBarrier);
        ok = 0;
        break;
      }
      __nanosleep(20);
    }
    if (ok && *(volatile int*)a.err != 0) ok = 0;
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

// Sum v[m] over the block (fixed order: warps 0..7); every thread gets the totals.
template <int MR>
__device__ __forceinline__ void block_sum(float (&v)[MR], float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    const float t = warp_sum(v[m]);
    if (lane == 0) red[warp * MR + m] = t;
  }
  __syncthreads();
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kPWarps; ++w) t += red[w * MR + m];
    v[m] = t;
  }
  __syncthreads();
}

// Residual stream update at the start of a phase, identically in every CTA:
// r = xk + bf16(sum_p part[p][m][:] + bias) (the embedding for layer 0),
// then x = LayerNorm(r) (two-pass, biased variance) into xk / xs.  Thread t
// owns columns 4t..4t+3 (width <= 1024).
template <int KCH, int MR>
__device__ void combine_ln(const PArgs& a, PSmem& s, const float* part, int nparts, const bf16* pbias,
                           const float* g, const float* b, bool embed) {
  constexpr int KP = KCH * 256;
  const int D = a.D;
  const int col = threadIdx.x * 4;
  const bool own = col < D;
  float4 r[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    r[m] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (m >= a.M || !own) continue;
    if (embed) {
      const float4 t = *reinterpret_cast<const float4*>(a.tok_emb + (size_t)row_token(a.rm, a.st, m) * D + col);
      const float4 p = *reinterpret_cast<const float4*>(a.pos_emb + (size_t)(row_pos(a.rm, a.st, m) + 2) * D + col);
      r[m] = make_float4(t.x + p.x, t.y + p.y, t.z + p.z, t.w + p.w);  // POSITION_OFFSET 2
    } else {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 16
      for (int q = 0; q < nparts; ++q) {
        const float4 p = ld_cg_f4(part + ((size_t)q * a.M + m) * D + col);
        acc.x += p.x;
        acc.y += p.y;
        acc.z += p.z;
        acc.w += p.w;
      }
      const float4 x = *reinterpret_cast<const float4*>(s.xk + (size_t)m * D + col);
      const uint2 bb = *reinterpret_cast<const uint2*>(pbias + col);
      r[m].x = x.x + round_bf16(acc.x + bf_lo(bb.x));
      r[m].y = x.y + round_bf16(acc.y + bf_hi(bb.x));
      r[m].z = x.z + round_bf16(acc.z + bf_lo(bb.y));
      r[m].w = x.w + round_bf16(acc.w + bf_hi(bb.y));
    }
  }
  float sum[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) sum[m] = (r[m].x + r[m].y) + (r[m].z + r[m].w);
  block_sum<MR>(sum, s.red);
  float mean[MR], sq[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    mean[m] = sum[m] / (float)D;
    if (own) {
      const float d0 = r[m].x - mean[m], d1 = r[m].y - mean[m], d2 = r[m].z - mean[m], d3 = r[m].w - mean[m];
      sq[m] = (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
    } else {
      sq[m] = 0.f;
    }
  }
  block_sum<MR>(sq, s.red);
  if (col < KP) {
    float4 gg = make_float4(0.f, 0.f, 0.f, 0.f), bb = gg;
    if (own) {
      gg = *reinterpret_cast<const float4*>(g + col);
      bb = *reinterpret_cast<const float4*>(b + col);
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      if (m >= a.M) continue;
      uint2 packed = make_uint2(0, 0);
      if (own) {
        const float rstd = rsqrtf(sq[m] / (float)D + kLnEps);
        float4 y;
        y.x = (r[m].x - mean[m]) * rstd * gg.x + bb.x;
        y.y = (r[m].y - mean[m]) * rstd * gg.y + bb.y;
        y.z = (r[m].z - mean[m]) * rstd * gg.z + bb.z;
        y.w = (r[m].w - mean[m]) * rstd * gg.w + bb.w;
        *reinterpret_cast<float4*>(s.xk + (size_t)m * D + col) = y;
        packed = make_uint2(pack_bf16(y.x, y.y), pack_bf16(y.z, y.w));
      }
      *reinterpret_cast<uint2*>(s.xs + (size_t)m * KP + col) = packed;
    }
  }
  __syncthreads();
}

// Dot products of weight rows against the staged rows: warp w takes rows
// r0 + w, r0 + w + 8, ... < r1 (four per pass, all loads in flight together)
// and calls epi(m, row, acc) on lane m.
template <int KCH, int MR, typename Epi>
__device__ __forceinline__ void gemv_rows(const bf16* W, int K, int r0, int r1, const bf16* xs, int M, Epi epi) {
  constexpr int KP = KCH * 256;
  constexpr int RP = 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = r0 + warp; r < r1; r += RP * kPWarps) {
    uint4 w[RP][KCH];
#pragma unroll
    for (int k = 0; k < RP; ++k) {
      const int row = r + k * kPWarps;
#pragma unroll
      for (int c = 0; c < KCH; ++c) {
        const int col = c * 256 + lane * 8;
        w[k][c] = (col < K && row < r1) ? ld_w(W + (size_t)row * K + col) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float acc[RP];
#pragma unroll
      for (int k = 0; k < RP; ++k) acc[k] = 0.f;
#pragma unroll
      for (int c = 0; c < KCH; ++c) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + (size_t)m * KP + c * 256 + lane * 8);
#pragma unroll
        for (int k = 0; k < RP; ++k) acc[k] += dot8(w[k][c], xv);
      }
#pragma unroll
      for (int k = 0; k < RP; ++k) {
        acc[k] = warp_sum(acc[k]);
        if (lane == m && m < M && r + k * kPWarps < r1) epi(m, r + k * kPWarps, acc[k]);
      }
    }
  }
}

// y[m][n] = sum_j s[m][j] * WT[j0 + j][n] for every n (rows of a transposed
// weight).  Thread t owns 4 columns; the loads of 16 rows are issued before
// any is used, and j is summed in order.
template <int MR>
__device__ __forceinline__ void axpy_rows(const bf16* WT, int D, int j0, int J, const float* sv, int lds, int M,
                                          float* y) {
  constexpr int JB = 32;
  for (int n = threadIdx.x * 4; n < D; n += kPThreads * 4) {
    float acc[MR][4];
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int t = 0; t < 4; ++t) acc[m][t] = 0.f;
    for (int jb = 0; jb < J; jb += JB) {
      uint2 w[JB];
#pragma unroll
      for (int u = 0; u < JB; ++u)
        w[u] = jb + u < J ? __ldg(reinterpret_cast<const uint2*>(WT + (size_t)(j0 + jb + u) * D + n)) : make_uint2(0, 0);
#pragma unroll
      for (int u = 0; u < JB; ++u) {
        if (jb + u < J) {
          const float w0 = bf_lo(w[u].x), w1 = bf_hi(w[u].x), w2 = bf_lo(w[u].y), w3 = bf_hi(w[u].y);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            const float sj = m < M ? sv[m * lds + jb + u] : 0.f;
            acc[m][0] = fmaf(sj, w0, acc[m][0]);
            acc[m][1] = fmaf(sj, w1, acc[m][1]);
            acc[m][2] = fmaf(sj, w2, acc[m][2]);
            acc[m][3] = fmaf(sj, w3, acc[m][3]);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m)
      if (m < M) *reinterpret_cast<float4*>(y + (size_t)m * D + n) = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
  }
}

// Sum the cluster's y[m][n] over this CTA's column range, in rank order, into dst[m][n].
template <int MR>
__device__ __forceinline__ void cluster_reduce_y(cg::cluster_group& cluster, PSmem& s, int D, int M, float* dst) {
  const int rank = (int)cluster.block_rank();
  const int per = D / kPClus;
  const int n0 = rank * per;
  for (int idx = threadIdx.x * 4; idx < M * per; idx += kPThreads * 4) {
    const int m = idx / per, n = n0 + idx % per;
    float4 v[kPClus];
#pragma unroll
    for (int r = 0; r < kPClus; ++r)
      v[r] = *reinterpret_cast<const float4*>(cluster.map_shared_rank(s.y, r) + (size_t)m * D + n);
    float4 acc = v[0];
#pragma unroll
    for (int r = 1; r < kPClus; ++r) {
      acc.x += v[r].x;
      acc.y += v[r].y;
      acc.z += v[r].z;
      acc.w += v[r].w;
    }
    *reinterpret_cast<float4*>(dst + (size_t)m * D + n) = acc;
  }
}

struct KeySrc {
  bool cross;
  bool own_last;  // the last key/value of each row come from s.kn / s.vn
  const bf16* k;
  const bf16* v;
  const int32_t* page_table;
  int pps, H, F;
  __device__ __forceinline__ const bf16* krow(int slot, int h, int j) const {
    return cross ? k + (((size_t)slot * H + h) * F + j) * kHeadDim : k + paged_offset(page_table, pps, H, slot, h, j);
  }
  __device__ __forceinline__ const bf16* vrow(int slot, int h, int j) const {
    return cross ? v + (((size_t)slot * H + h) * F + j) * kHeadDim : v + paged_offset(page_table, pps, H, slot, h, j);
  }
};

__device__ __forceinline__ uint4 pack8(const float* p) {
  return make_uint4(pack_bf16(p[0], p[1]), pack_bf16(p[2], p[3]), pack_bf16(p[4], p[5]), pack_bf16(p[6], p[7]));
}

// Attention of head h for every active row, keys split over the cluster.
// Leaves this CTA's kDimsLocal output dims (bf16-rounded) in s.av.  Two
// cluster barriers.
template <int MR>
__device__ void cluster_attention(const PArgs& a, cg::cluster_group& cluster, PSmem& s, const KeySrc& src, int h) {
  const int rank = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = tid >> 3, sub = tid & 7;
  constexpr int G = kPThreads / 8;
  __shared__ float wred[kPWarps];
  for (int m = 0; m < a.M; ++m) {
    float* sc = s.sc + (size_t)m * a.chunk_cap;
    const bool active = row_active(a.rm, a.st, m);
    const int slot = row_slot(a.rm, m);
    const int L = !active ? 0 : src.cross ? a.st.frames[slot] : row_pos(a.rm, a.st, m) + 1;
    const int chunk = (L + kPClus - 1) / kPClus;
    const int j0 = min(L, rank * chunk), j1 = min(L, j0 + chunk);
    const int jown = src.own_last ? L - 1 : -1;
    float q[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) q[t] = s.qh[m * kHeadDim + sub * 8 + t];
    float lmax = -INFINITY;
    for (int base = j0; base < j1; base += G * 4) {
      uint4 kv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = base + grp + u * G;
        kv[u] = (j < j1 && j != jown) ? ld_cg(src.krow(slot, h, j) + sub * 8) : make_uint4(0, 0, 0, 0);
        if (j == jown) kv[u] = pack8(s.kn + m * kHeadDim + sub * 8);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = base + grp + u * G;
        float d = bf_lo(kv[u].x) * q[0];
        d = fmaf(bf_hi(kv[u].x), q[1], d);
        d = fmaf(bf_lo(kv[u].y), q[2], d);
        d = fmaf(bf_hi(kv[u].y), q[3], d);
        d = fmaf(bf_lo(kv[u].z), q[4], d);
        d = fmaf(bf_hi(kv[u].z), q[5], d);
        d = fmaf(bf_lo(kv[u].w), q[6], d);
        d = fmaf(bf_hi(kv[u].w), q[7], d);
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        d += __shfl_xor_sync(0xffffffffu, d, 4);
        if (j < j1) {
          d = round_bf16(d) * 0.125f;  // head_dim ** -0.5
          if (sub == 0) sc[j - j0] = d;
          lmax = fmaxf(lmax, d);
        }
      }
    }
    lmax = warp_max(lmax);
    if (lane == 0) wred[warp] = lmax;
    __syncthreads();
    float bm = wred[0];
#pragma unroll
    for (int w = 1; w < kPWarps; ++w) bm = fmaxf(bm, wred[w]);
    __syncthreads();
    float lsum = 0.f;
    for (int j = j0 + tid; j < j1; j += kPThreads) lsum += expf(sc[j - j0] - bm);
    lsum = warp_sum(lsum);
    if (lane == 0) wred[warp] = lsum;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kPWarps; ++w) t += wred[w];
      s.stat[m * 2 + 0] = bm;
      s.stat[m * 2 + 1] = t;
    }
    __syncthreads();
  }
  cluster.sync();  // (1) every CTA's local max and sum are visible
  for (int m = 0; m < a.M; ++m) {
    float* sc = s.sc + (size_t)m * a.chunk_cap;
    const bool active = row_active(a.rm, a.st, m);
    const int slot = row_slot(a.rm, m);
    const int L = !active ? 0 : src.cross ? a.st.frames[slot] : row_pos(a.rm, a.st, m) + 1;
    const int chunk = (L + kPClus - 1) / kPClus;
    const int j0 = min(L, rank * chunk), j1 = min(L, j0 + chunk);
    const int jown = src.own_last ? L - 1 : -1;
    // global max and sum of exp(s - max) over the cluster (softmax, engine.py:291)
    float mx[kPClus], sm[kPClus];
#pragma unroll
    for (int r = 0; r < kPClus; ++r) {
      const float* st = cluster.map_shared_rank(s.stat, r) + m * 2;
      mx[r] = st[0];
      sm[r] = st[1];
    }
    float gmax = mx[0];
#pragma unroll
    for (int r = 1; r < kPClus; ++r) gmax = fmaxf(gmax, mx[r]);
    float gsum = 0.f;
#pragma unroll
    for (int r = 0; r < kPClus; ++r)
      if (sm[r] > 0.f) gsum += sm[r] * expf(mx[r] - gmax);
    float acc[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = 0.f;
    for (int base = j0; base < j1; base += G * 4) {
      uint4 vv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = base + grp + u * G;
        vv[u] = (j < j1 && j != jown) ? ld_cg(src.vrow(slot, h, j) + sub * 8) : make_uint4(0, 0, 0, 0);
        if (j == jown) vv[u] = pack8(s.vn + m * kHeadDim + sub * 8);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = base + grp + u * G;
        const float p = j < j1 ? round_bf16(expf(sc[j - j0] - gmax) / gsum) : 0.f;
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
    for (int t = 0; t < 8; ++t) {
      acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], 8);
      acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], 16);
    }
    if (lane < 8) {
#pragma unroll
      for (int t = 0; t < 8; ++t) s.red[warp * kHeadDim + lane * 8 + t] = acc[t];
    }
    __syncthreads();
    if (tid < kHeadDim) {
      float o = 0.f;
#pragma unroll
      for (int w = 0; w < kPWarps; ++w) o += s.red[w * kHeadDim + tid];
      s.ov[m * kHeadDim + tid] = o;
    }
    __syncthreads();
  }
  cluster.sync();  // (2) partial outputs visible
  for (int idx = threadIdx.x; idx < a.M * kDimsLocal; idx += kPThreads) {
    const int m = idx / kDimsLocal, d = rank * kDimsLocal + idx % kDimsLocal;
    float v[kPClus];
#pragma unroll
    for (int r = 0; r < kPClus; ++r) v[r] = cluster.map_shared_rank(s.ov, r)[m * kHeadDim + d];
    float o = v[0];
#pragma unroll
    for (int r = 1; r < kPClus; ++r) o += v[r];
    s.av[m * kDimsLocal + idx % kDimsLocal] = round_bf16(o);
  }
  __syncthreads();
}

// L2 prefetches for what this CTA reads in its next phase (weights and the
// K/V of positions already cached), so that HBM streams them while the grid
// barrier resolves.  phase: 0 = A of `layer`, 1 = B, 2 = C, 3 = logits.
static __device__ void prefetch_phase(const PArgs& a, int phase, int layer, int rank, int ci, unsigned nclusters) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane != 0 || !a.prefetch) return;
  const int D = a.D, H = a.H;
  const size_t row_bytes = (size_t)D * sizeof(bf16);
  if (phase == 3) {
    for (int v = blockIdx.x * kPWarps + warp; v < a.V; v += gridDim.x * kPWarps)
      prefetch_bulk_l2(a.emb + (size_t)v * D, (unsigned)row_bytes);
    return;
  }
  const PLayer& W = a.layers[layer];
  if (phase == 2) {
    const int u0 = blockIdx.x * a.units, u1 = min(a.FFN, u0 + a.units);
    if (u1 <= u0) return;
    if (warp == 0) prefetch_bulk_l2(W.w1 + (size_t)u0 * D, (unsigned)((u1 - u0) * row_bytes));
    if (warp == 1) prefetch_bulk_l2(W.w2T + (size_t)u0 * D, (unsigned)((u1 - u0) * row_bytes));
    return;
  }
  for (int h = ci; h < H; h += nclusters) {
    if (phase == 0) {
      if (warp == 0) {  // this CTA's q/k/v rows, in up to two runs
        int li = rank * kQkvLocal;
        const int end = li + kQkvLocal;
        while (li < end) {
          const int part = li / kHeadDim, d0 = li % kHeadDim;
          const int n = min(end - li, kHeadDim - d0);
          prefetch_bulk_l2(W.wqkv + ((size_t)part * D + h * kHeadDim + d0) * D, (unsigned)(n * row_bytes));
          li += n;
        }
      }
      if (warp == 1)
        prefetch_bulk_l2(W.woT + (size_t)(h * kHeadDim + rank * kDimsLocal) * D, (unsigned)(kDimsLocal * row_bytes));
    } else {
      if (warp == 0)
        prefetch_bulk_l2(W.wcq + (size_t)(h * kHeadDim + rank * kDimsLocal) * D, (unsigned)(kDimsLocal * row_bytes));
      if (warp == 1)
        prefetch_bulk_l2(W.wcoT + (size_t)(h * kHeadDim + rank * kDimsLocal) * D, (unsigned)(kDimsLocal * row_bytes));
    }
    for (int m = warp; m < a.M; m += kPWarps) {
      if (!row_active(a.rm, a.st, m)) continue;
      const int slot = row_slot(a.rm, m);
      if (phase == 1) {
        const int L = a.st.frames[slot];
        const int chunk = (L + kPClus - 1) / kPClus;
        const int j0 = min(L, rank * chunk), j1 = min(L, j0 + chunk);
        if (j1 <= j0) continue;
        const size_t off = (((size_t)slot * H + h) * a.F + j0) * kHeadDim;
        prefetch_bulk_l2(W.ck + off, (unsigned)((j1 - j0) * kHeadDim * sizeof(bf16)));
        prefetch_bulk_l2(W.cv + off, (unsigned)((j1 - j0) * kHeadDim * sizeof(bf16)));
      } else {
        const int L = row_pos(a.rm, a.st, m);  // positions before the new token
        const int chunk = (L + 1 + kPClus - 1) / kPClus;
        const int j0 = min(L, rank * chunk), j1 = min(L, j0 + chunk);
        for (int t = j0; t < j1;) {
          const int n = min(j1 - t, kPageTokens - t % kPageTokens);
          const size_t off = paged_offset(a.st.page_table, a.pps, H, slot, h, t);
          prefetch_bulk_l2(W.kpool + off, (unsigned)(n * kHeadDim * sizeof(bf16)));
          prefetch_bulk_l2(W.vpool + off, (unsigned)(n * kHeadDim * sizeof(bf16)));
          t += n;
        }
      }
    }
  }
}

template <int KCH, int MR>
__global__ void __launch_bounds__(kPThreads, 1) step_persistent_kernel(const PArgs a) {
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int KP = KCH * 256;
  const int D = a.D, H = a.H;
  const int rank = (int)cluster.block_rank();
  const unsigned nclusters = gridDim.x / kPClus;
  const int ci = blockIdx.x / kPClus;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  PSmem s;
  {
    unsigned char* p = smem_raw;
    auto take = [&](size_t bytes) {
      unsigned char* q = p;
      p += (bytes + 15) & ~size_t(15);
      return q;
    };
    s.xk = reinterpret_cast<float*>(take(sizeof(float) * MR * D));
    s.xs = reinterpret_cast<bf16*>(take(sizeof(bf16) * MR * KP));
    s.y = reinterpret_cast<float*>(take(sizeof(float) * MR * D));
    s.sc = reinterpret_cast<float*>(take(sizeof(float) * MR * a.chunk_cap));
    s.qh = reinterpret_cast<float*>(take(sizeof(float) * MR * kHeadDim));
    s.kn = reinterpret_cast<float*>(take(sizeof(float) * MR * kHeadDim));
    s.vn = reinterpret_cast<float*>(take(sizeof(float) * MR * kHeadDim));
    s.loc = reinterpret_cast<float*>(take(sizeof(float) * MR * kQkvLocal));
    s.ov = reinterpret_cast<float*>(take(sizeof(float) * MR * kHeadDim));
    s.stat = reinterpret_cast<float*>(take(sizeof(float) * MR * 2));
    s.av = reinterpret_cast<float*>(take(sizeof(float) * MR * kDimsLocal));
    s.hid = reinterpret_cast<float*>(take(sizeof(float) * MR * a.units));
    s.red = reinterpret_cast<float*>(take(sizeof(float) * kPWarps * kHeadDim));
  }
  trace_mark(a, kTraceSlots - 1);
  prefetch_phase(a, 0, 0, rank, ci, nclusters);
  // Distributed shared memory is only touched after a cluster barrier.
  cluster.sync();
  unsigned target = 0;
  // A prefill chunk reads K/V that other CTAs of the cluster wrote in this
  // launch through global memory; a decode row only its own new key/value,
  // which travel through shared memory.
  const bool prefill = a.rm.prefill != 0;

  for (int l = 0; l < a.L; ++l) {
    const PLayer& W = a.layers[l];
    const bool kv_only = !a.logits && l == a.L - 1;
    const int tb = l * 40;
    trace_mark(a, tb + 0);
    // ---------------- phase A
    if (l == 0)
      combine_ln<KCH, MR>(a, s, nullptr, 0, nullptr, a.emb_g, a.emb_b, true);
    else
      combine_ln<KCH, MR>(a, s, a.part_f, nclusters, a.layers[l - 1].b2, a.layers[l - 1].ln_final_g,
                          a.layers[l - 1].ln_final_b, false);
    trace_mark(a, tb + 1);
    for (int h = ci; h < H; h += nclusters) {
      const int r0 = rank * kQkvLocal;
      // this CTA's 48 of the head's 192 rows (q 0-63, k 64-127, v 128-191):
      // warp w owns local rows w + 8k, all six loaded before any is used
      constexpr int RW = kQkvLocal / kPWarps;
      {
        const int pass = 0;
        uint4 w[RW][KCH];
        int rows[RW];
#pragma unroll
        for (int k = 0; k < RW; ++k) {
          const int li = r0 + warp + (pass * RW + k) * kPWarps;
          rows[k] = (li / kHeadDim) * D + h * kHeadDim + li % kHeadDim;
#pragma unroll
          for (int c = 0; c < KCH; ++c) {
            const int col = c * 256 + lane * 8;
            w[k][c] = col < D ? ld_w(W.wqkv + (size_t)rows[k] * D + col) : make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll
        for (int k = 0; k < RW; ++k) {
          const int i = warp + (pass * RW + k) * kPWarps;
          const int li = r0 + i;
          const int part = li / kHeadDim, d = li % kHeadDim;
          const float bias = __bfloat162float(W.bqkv[rows[k]]);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            float acc = 0.f;
#pragma unroll
            for (int c = 0; c < KCH; ++c)
              acc += dot8(w[k][c], *reinterpret_cast<const uint4*>(s.xs + (size_t)m * KP + c * 256 + lane * 8));
            acc = warp_sum(acc);
            if (lane == m && m < a.M) {
              const float val = round_bf16(acc + bias);
              s.loc[m * kQkvLocal + i] = val;
              if (part > 0 && row_active(a.rm, a.st, m)) {
                bf16* dst = part == 1 ? W.kpool : W.vpool;
                dst[paged_offset(a.st.page_table, a.pps, H, row_slot(a.rm, m), h, row_pos(a.rm, a.st, m)) + d] =
                    __float2bfloat16_rn(val);
              }
            }
          }
        }
      }
      if (prefill) __threadfence();
      cluster.sync();  // q, k, v rows of the cluster visible
      trace_mark(a, tb + 2);
      for (int idx = tid; idx < a.M * 3 * kHeadDim; idx += kPThreads) {
        const int m = idx / (3 * kHeadDim), li = idx % (3 * kHeadDim);
        const float v = cluster.map_shared_rank(s.loc, li / kQkvLocal)[m * kQkvLocal + li % kQkvLocal];
        float* dst = li < kHeadDim ? s.qh : li < 2 * kHeadDim ? s.kn : s.vn;
        dst[m * kHeadDim + li % kHeadDim] = v;
      }
      __syncthreads();
      if (kv_only) continue;
      KeySrc src{false, !prefill, W.kpool, W.vpool, a.st.page_table, a.pps, H, a.F};
      cluster_attention<MR>(a, cluster, s, src, h);
      trace_mark(a, tb + 3);
      axpy_rows<MR>(W.woT, D, h * kHeadDim + rank * kDimsLocal, kDimsLocal, s.av, kDimsLocal, a.M, s.y);
      cluster.sync();
      cluster_reduce_y<MR>(cluster, s, D, a.M, a.part_o + (size_t)h * a.M * D);
      cluster.sync();  // peers finished reading y and loc before they are reused
      trace_mark(a, tb + 4);
    }
    if (kv_only) break;
    prefetch_phase(a, 1, l, rank, ci, nclusters);
    grid_barrier(a, target);
    trace_mark(a, tb + 5);
    // ---------------- phase B
    combine_ln<KCH, MR>(a, s, a.part_o, H, W.bo, W.ln_self_g, W.ln_self_b, false);
    trace_mark(a, tb + 6);
    for (int h = ci; h < H; h += nclusters) {
      const int r0 = h * kHeadDim + rank * kDimsLocal;
      gemv_rows<KCH, MR>(W.wcq, D, r0, r0 + kDimsLocal, s.xs, a.M, [&](int m, int row, float acc) {
        s.loc[m * kQkvLocal + (row - r0)] = round_bf16(acc + __bfloat162float(W.bcq[row]));
      });
      cluster.sync();
      trace_mark(a, tb + 7);
      for (int idx = tid; idx < a.M * kHeadDim; idx += kPThreads) {
        const int m = idx / kHeadDim, d = idx % kHeadDim;
        s.qh[idx] = cluster.map_shared_rank(s.loc, d / kDimsLocal)[m * kQkvLocal + d % kDimsLocal];
      }
      __syncthreads();
      KeySrc src{true, false, W.ck, W.cv, a.st.page_table, a.pps, H, a.F};
      cluster_attention<MR>(a, cluster, s, src, h);
      trace_mark(a, tb + 8);
      axpy_rows<MR>(W.wcoT, D, h * kHeadDim + rank * kDimsLocal, kDimsLocal, s.av, kDimsLocal, a.M, s.y);
      cluster.sync();
      cluster_reduce_y<MR>(cluster, s, D, a.M, a.part_c + (size_t)h * a.M * D);
      cluster.sync();
      trace_mark(a, tb + 9);
    }
    prefetch_phase(a, 2, l, rank, ci, nclusters);
    grid_barrier(a, target);
    trace_mark(a, tb + 10);
    // ---------------- phase C
    combine_ln<KCH, MR>(a, s, a.part_c, H, W.bco, W.ln_cross_g, W.ln_cross_b, false);
    trace_mark(a, tb + 11);
    {
      const int u0 = blockIdx.x * a.units;
      const int u1 = min(a.FFN, u0 + a.units);
      for (int idx = tid; idx < MR * a.units; idx += kPThreads) s.hid[idx] = 0.f;
      __syncthreads();
      gemv_rows<KCH, MR>(W.w1, D, u0, u1, s.xs, a.M, [&](int m, int row, float acc) {
        const float v = round_bf16(acc + __bfloat162float(W.b1[row]));
        s.hid[m * a.units + (row - u0)] = round_bf16(gelu_erf(v));
      });
      __syncthreads();
      trace_mark(a, tb + 12);
      axpy_rows<MR>(W.w2T, D, u0, max(0, u1 - u0), s.hid, a.units, a.M, s.y);
      cluster.sync();
      cluster_reduce_y<MR>(cluster, s, D, a.M, a.part_f + (size_t)ci * a.M * D);
      cluster.sync();
    }
    trace_mark(a, tb + 13);
    if (l + 1 < a.L)
      prefetch_phase(a, 0, l + 1, rank, ci, nclusters);
    else if (a.logits)
      prefetch_phase(a, 3, l, rank, ci, nclusters);
    grid_barrier(a, target);
    trace_mark(a, tb + 14);
  }

  if (a.logits) {
    // ---------------- logits: residual + final_norm, vocabulary slice, grammar mask, argmax
    const PLayer& last = a.layers[a.L - 1];
    combine_ln<KCH, MR>(a, s, a.part_f, nclusters, last.b2, last.ln_final_g, last.ln_final_b, false);
    trace_mark(a, 40 * a.L);
    __shared__ uint32_t rule[kPMaxRows];
    __shared__ unsigned long long wbest[kPWarps][kPMaxRows];
    __shared__ int is_last;
    if (tid < MR) rule[tid] = tid < a.M ? (a.gr.kind == 1 ? (uint32_t)a.st.g[tid] : class_mask(a.st, tid)) : 0u;
    __syncthreads();
    unsigned long long best[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) best[m] = 0ull;
    for (int v0 = blockIdx.x * kPWarps + warp; v0 < a.V; v0 += 2 * gridDim.x * kPWarps) {
      const int v1 = v0 + gridDim.x * kPWarps;
      uint4 w[2][KCH];
#pragma unroll
      for (int c = 0; c < KCH; ++c) {
        const int col = c * 256 + lane * 8;
        w[0][c] = col < D ? ld_w(a.emb + (size_t)v0 * D + col) : make_uint4(0, 0, 0, 0);
        w[1][c] = (col < D && v1 < a.V) ? ld_w(a.emb + (size_t)v1 * D + col) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int v = k == 0 ? v0 : v1;
        if (v >= a.V) continue;
        const float bias = a.bias ? a.bias[v] : 0.f;
        const int cls = a.gr.kind == 1 ? 0 : a.gr.token_class[v];
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          float acc = 0.f;
#pragma unroll
          for (int c = 0; c < KCH; ++c)
            acc += dot8(w[k][c], *reinterpret_cast<const uint4*>(s.xs + (size_t)m * KP + c * 256 + lane * 8));
          acc = warp_sum(acc);
          if (m < a.M) {
            const float logit = round_bf16(acc);
            if (a.logits_out && lane == 0) a.logits_out[(size_t)m * a.V + v] = logit;
            const bool allowed =
                a.gr.kind == 1 ? a.gr.table[(size_t)rule[m] * a.V + v] != 0 : ((rule[m] >> cls) & 1u) != 0;
            if (allowed) {
              const unsigned long long key = argmax_key(logit + bias, v);
              best[m] = key > best[m] ? key : best[m];
            }
          }
        }
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < MR; ++m) wbest[warp][m] = best[m];
    }
    __syncthreads();
    if (tid < a.M) {
      unsigned long long k = 0ull;
      for (int w = 0; w < kPWarps; ++w) k = wbest[w][tid] > k ? wbest[w][tid] : k;
      if (k) atomicMax(a.keys + tid, k);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (is_last) {
      __threadfence();
      const bool failed = *(volatile int*)a.err != 0;  // a barrier gave up: leave the slots as they were
      for (int sl = tid; sl < a.M; sl += kPThreads) {
        const unsigned long long k = atomicExch(a.keys + sl, 0ull);
        if (failed) continue;
        const int64_t greedy = k ? (int64_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull)) : 0;
        if (a.greedy_out) a.greedy_out[sl] = greedy;
        const bool active = a.st.finished[sl] == 0;
        const int64_t tok = a.st.token[sl], pos = a.st.position[sl];
        int64_t choice = greedy;
        if (a.forced && a.forced[sl] >= 0) choice = a.forced[sl];
        if (!active) choice = tok;
        const int64_t new_pos = active ? pos + 1 : pos;
        if (active && new_pos < a.T) a.st.out[(size_t)sl * a.T + new_pos] = choice;
        grammar_update(a.gr, a.st, sl, choice, active, new_pos >= a.T - 1);
        a.st.token[sl] = choice;
        a.st.position[sl] = new_pos;
      }
      if (tid == 0) *a.counter = 0u;
    }
  }
  trace_mark(a, 40 * a.L + 2);
  // Leave: the last CTA out resets the barrier counters for the next launch.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(a.bar + 1, 1u) == gridDim.x - 1) {
      atomicExch(a.bar, 0u);
      atomicExch(a.bar + 1, 0u);
    }
  }
  cluster.sync();  // no CTA leaves while a peer may still read its shared memory
}

}  // namespace s2r
