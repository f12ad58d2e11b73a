// One decode step (or prefill chunk of up to 8 rows) as ONE persistent kernel
// whose weights and K/V stream through a shared-memory ring.
//
// At batch 1 the multi-kernel step is bound by launch and dependency latency
// (97 kernels that each move 2-8 MB).  Here one CTA per SM runs the whole
// step.  Each CTA has a producer warp and eight consumer warps:
//
//   * the producer walks the CTA's fixed sequence of pieces for the whole
//     step -- its slice of every weight matrix, and for attention CTAs the
//     K/V blocks of its key range -- and copies each piece (at most 16 KB)
//     into the next free stage of a ring in shared memory with 1-D bulk
//     copies.  Nothing it copies is written during the step (weights, cross
//     K/V, self K/V of earlier positions), so it runs ahead of the consumers
//     by the ring's depth, across grid barriers, and HBM streams while the
//     consumers wait;
//   * the consumers run the step in six phases per layer separated by grid
//     barriers, every matrix split by rows over all CTAs:
//       P1  r -> LayerNorm -> QKV rows (q to global, K/V appended to the cache)
//       P2  self-attention, one cluster of 4 CTAs per head (keys split over
//           the cluster, softmax statistics and outputs exchanged through
//           distributed shared memory), then the head's share of the
//           out-projection as a partial sum over the head
//       P3  r = x + bf16(sum over heads + bias) -> self_attn_norm -> cross q rows
//       P4  cross-attention as P2, with the cross out-projection
//       P5  r -> cross_attn_norm -> fc1 rows + GELU (to global)
//       P6  fc2 rows -> r = x + bf16(fc2 + bias) (to global)
//     then the logits phase: r -> final_norm -> a vocabulary slice, grammar
//     mask, argmax keys; the last CTA commits the step.
//
// Rounding follows the reference's CUDA path (engine.py:286-315) as the
// multi-kernel path does; float32 summation orders differ from it but are
// fixed, so the step is deterministic and a row's result does not depend on
// the other rows of the launch.
//
// Every wait is bounded.  A grid barrier, ring stage or cluster exchange that
// has not completed in time records an error word; from then on no wait
// blocks, the phases run on whatever data they have, the commit is skipped
// and every CTA still takes the same barriers, so the kernel ends.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"
#include "logits.cuh"
#include "mbarrier.cuh"
#include "proj.cuh"

namespace s2r {

namespace cg = cooperative_groups;

constexpr int kPClus = 4;                        // CTAs per cluster: one head's attention per cluster
constexpr int kPConsumers = 256;                 // eight consumer warps
constexpr int kPWarps = kPConsumers / 32;
constexpr int kPThreads = kPConsumers + 32;      // + the producer warp
constexpr int kPMaxRows = 8;
constexpr int kPStage = 16384;                   // bytes per ring stage
constexpr int kPKeys = kPStage / (kHeadDim * 2);  // K or V rows per stage (128)
constexpr int kPMaxStages = 12;
constexpr int kErrBarrier = 3;  // a grid barrier timed out
constexpr int kErrRing = 8;     // a ring stage or cluster exchange timed out
constexpr unsigned long long kSpinNs = 2000000000ull;
constexpr int kTraceSlots = 512;
constexpr int kTraceCtas = 16;

struct PLayer {
  const bf16 *wqkv, *bqkv;   // [3D, D], [3D]
  const bf16 *wo_hb, *bo;    // out-projection by head: wo_hb[h][n][d] = Wo[n][64h + d]
  const bf16 *wcq, *bcq;     // [D, D]
  const bf16 *wco_hb, *bco;  // cross out-projection by head
  const bf16 *w1, *b1;       // [F, D]
  const bf16 *w2, *b2;       // [D, F]
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
  int chunk_cap;  // attention keys per row per CTA
  int stages;     // ring stages
  int logits;     // 1: decode step (logits + commit); 0: prefill (K/V only)
  const PLayer* layers;
  const float *tok_emb, *pos_emb, *emb_g, *emb_b;
  const bf16* emb;
  const float* bias;
  float* r;                // [M][D] residual sums between phases
  bf16* q;                 // [M][D] queries (self, then cross)
  bf16* hid;               // [M][FFN] GELU outputs
  float *part_o, *part_c;  // [H][M][D] out-projection partial sums by head
  unsigned* bar;           // [0] arrivals, [1] exits
  unsigned long long* keys;
  unsigned* counter;
  int* err;
  const int64_t* forced;
  float* logits_out;
  int64_t* greedy_out;
  long long* trace;  // optional globaltimer marks (rank 0 of the first kTraceCtas clusters)
  Rescore rs;        // frame-head rescoring (rs.on == 0: none)
};

// ---------------------------------------------------------------- geometry
// The producer and the consumers derive the same piece sequence from these.

// Rows [r0, r1) of an N-row matrix owned by this CTA.
__device__ __forceinline__ void row_slice(int N, int& r0, int& r1) {
  r0 = (int)((long long)N * blockIdx.x / gridDim.x);
  r1 = (int)((long long)N * (blockIdx.x + 1) / gridDim.x);
}

__device__ __forceinline__ int rows_per_stage(int K) { return max(1, kPStage / (K * 2)); }

struct KeyRange {
  int slot, L, j0, j1, js;  // keys [j0, j1) of this CTA; [j0, js) stream through the ring
};

__device__ __forceinline__ KeyRange key_range(const PArgs& a, int m, bool cross, int rank) {
  KeyRange k{0, 0, 0, 0, 0};
  if (!row_active(a.rm, a.st, m)) return k;
  k.slot = row_slot(a.rm, m);
  k.L = cross ? a.st.frames[k.slot] : row_pos(a.rm, a.st, m) + 1;
  const int chunk = (k.L + kPClus - 1) / kPClus;
  k.j0 = min(k.L, rank * chunk);
  k.j1 = min(k.L, k.j0 + chunk);
  // keys written during this launch (the rows' own positions) are read from global memory
  const int fresh = cross ? k.L : (a.rm.prefill ? a.rm.pos0 : row_pos(a.rm, a.st, m));
  k.js = max(k.j0, min(k.j1, fresh));
  return k;
}

// Number of 128-key ring pieces of [j0, js).
__device__ __forceinline__ int key_blocks(const KeyRange& k) {
  return k.js > k.j0 ? (k.js - 1) / kPKeys - k.j0 / kPKeys + 1 : 0;
}

__device__ __forceinline__ void block_keys(const KeyRange& k, int b, int& lo, int& hi) {
  const int base = (k.j0 / kPKeys + b) * kPKeys;
  lo = max(k.j0, base);
  hi = min(k.js, base + kPKeys);
}

__device__ __forceinline__ const bf16* key_row(const PArgs& a, const PLayer& W, bool cross, bool value, int slot, int h,
                                               int j) {
  if (cross) return (value ? W.cv : W.ck) + (((size_t)slot * a.H + h) * a.F + j) * kHeadDim;
  return (value ? W.vpool : W.kpool) + paged_offset(a.st.page_table, a.pps, a.H, slot, h, j);
}

// ---------------------------------------------------------------- ring
struct Ring {
  unsigned char* buf;
  uint64_t* full;
  uint64_t* empty;
  int stages;
};

// Producer: request one piece into the next stage (waits, bounded, for it to be free).
struct Producer {
  const PArgs* a;
  Ring ring;
  int seq = 0;
  bool dead = false;
  __device__ __forceinline__ unsigned char* begin(unsigned bytes) {
    const int s = seq % ring.stages;
    if (!dead && seq >= ring.stages) {
      if (*(volatile int*)a->err != 0 || !mbar_wait(&ring.empty[s], ((seq / ring.stages) - 1) & 1)) {
        if (*(volatile int*)a->err == 0) atomicExch(a->err, kErrRing);
        dead = true;
      }
    }
    if (!dead) mbar_expect_tx(&ring.full[s], bytes);
    return ring.buf + (size_t)s * kPStage;
  }
  __device__ __forceinline__ void copy(unsigned char* dst, const void* src, unsigned bytes) {
    if (!dead) bulk_load(dst, src, bytes, &ring.full[seq % ring.stages]);
  }
  __device__ __forceinline__ void end() { ++seq; }
  // a run of rows [r0, r1) of a row-major [*, K] matrix, in pieces of rows_per_stage(K)
  __device__ __forceinline__ void rows(const bf16* W, int K, int r0, int r1) {
    const int rps = rows_per_stage(K);
    for (int p = r0; p < r1; p += rps) {
      const int n = min(rps, r1 - p);
      unsigned char* dst = begin((unsigned)(n * K * 2));
      copy(dst, W + (size_t)p * K, (unsigned)(n * K * 2));
      end();
    }
  }
  __device__ __forceinline__ void keys(const PLayer& W, bool cross, bool value, int h, const KeyRange& k) {
    const int nb = key_blocks(k);
    for (int b = 0; b < nb; ++b) {
      int lo, hi;
      block_keys(k, b, lo, hi);
      unsigned char* dst = begin((unsigned)((hi - lo) * kHeadDim * 2));
      for (int j = lo; j < hi;) {  // a self K/V page holds 64 consecutive keys of a head
        const int n = cross ? hi - j : min(hi - j, kPageTokens - j % kPageTokens);
        copy(dst + (size_t)(j - lo) * kHeadDim * 2, key_row(*a, W, cross, value, k.slot, h, j),
             (unsigned)(n * kHeadDim * 2));
        j += n;
      }
      end();
    }
  }
  // the last stages' copies land before the CTA leaves
  __device__ __forceinline__ void drain() {
    for (int i = max(0, seq - ring.stages); i < seq; ++i) mbar_wait(&ring.full[i % ring.stages], (i / ring.stages) & 1);
  }
};

// Consumers: wait (bounded) for the next piece, release it after use.
struct Consumer {
  const PArgs* a;
  Ring ring;
  int seq = 0;
  int* failed;  // shared flag
  __device__ __forceinline__ const unsigned char* wait() {
    const int s = seq % ring.stages;
    if (!*(volatile int*)failed && !mbar_wait(&ring.full[s], (seq / ring.stages) & 1)) {
      *(volatile int*)failed = 1;
      atomicExch(a->err, kErrRing);
    }
    return ring.buf + (size_t)s * kPStage;
  }
  __device__ __forceinline__ void release() {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&ring.empty[seq % ring.stages])) : "memory");
    ++seq;
  }
};

// ---------------------------------------------------------------- consumer helpers
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kPConsumers) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void trace_mark(const PArgs& a, int idx) {
  if (a.trace == nullptr || threadIdx.x != 0 || idx < 0 || idx >= kTraceSlots) return;
  const int b = blockIdx.x;
  const int which = (b % kPClus == 0 && b / kPClus < kTraceCtas) ? b / kPClus : -1;
  if (which >= 0) a.trace[which * kTraceSlots + idx] = (long long)global_ns();
}

// Grid barrier over the consumers of every CTA (bounded).  False once any
// CTA has recorded an error: from then on nobody waits.
__device__ __forceinline__ bool grid_barrier(const PArgs& a, unsigned& target, int* ok_s) {
  csync();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
    int ok = *(volatile int*)a.err == 0;
    const unsigned long long t0 = global_ns();
    while (ok && ld_acquire_u32(a.bar) < target) {
      if (*(volatile int*)a.err != 0) {
        ok = 0;
        break;
      }
      if (global_ns() - t0 > kSpinNs) {
        atomicExch(a.err, kErrBarrier);
        ok = 0;
        break;
      }
    }
    *ok_s = ok;
  }
  csync();
  return *ok_s != 0;
}

// Sum v[m] over the consumers (fixed order); every consumer gets the totals.
template <int MR>
__device__ __forceinline__ void consumer_sum(float (&v)[MR], float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    const float t = warp_sum(v[m]);
    if (lane == 0) red[warp * MR + m] = t;
  }
  csync();
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kPWarps; ++w) t += red[w * MR + m];
    v[m] = t;
  }
  csync();
}

struct PSmem {
  float* x;     // [MR][D]  the LayerNorm output (float32): the residual input of the next sum
  bf16* xs;     // [MR][KP] the same in bfloat16: GEMV input
  bf16* hs;     // [MR][FP] GELU outputs (fc2 input), shares space with sc
  float* sc;    // [MR][chunk_cap] attention scores
  float* qh;    // [MR][64] the head's query
  float* oh;    // [MR][64] the head's attention output (bf16-rounded)
  float* xch0;  // [2][kPClus][MR][2]  exchanged (max, sum) by use parity and source rank
  float* xch1;  // [2][kPClus][MR][64] exchanged partial outputs by use parity and source rank
  float* red;   // [8][64] reduction scratch
};

// r (from global, or the embedding for layer 0) -> LayerNorm into x / xs.
// with_part: r = x + bf16(sum_h part[h] + bias) first (the residual sum of an
// attention block).  Thread t owns columns 4t..4t+3.
template <int MR>
__device__ void combine_ln(const PArgs& a, PSmem& s, int KP, int mode, const float* part, const bf16* pbias,
                           const float* g, const float* b) {
  // mode 0: embedding; 1: r from global; 2: x + bf16(sum of head partials + bias)
  const int D = a.D;
  const int col = threadIdx.x * 4;
  const bool own = col < D;
  float4 r[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    r[m] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (m >= a.M || !own) continue;
    if (mode == 0) {
      const float4 t = *reinterpret_cast<const float4*>(a.tok_emb + (size_t)row_token(a.rm, a.st, m) * D + col);
      const float4 p = *reinterpret_cast<const float4*>(a.pos_emb + (size_t)(row_pos(a.rm, a.st, m) + 2) * D + col);
      r[m] = make_float4(t.x + p.x, t.y + p.y, t.z + p.z, t.w + p.w);  // POSITION_OFFSET 2
    } else if (mode == 1) {
      r[m] = __ldcg(reinterpret_cast<const float4*>(a.r + (size_t)m * D + col));
    } else {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int h = 0; h < a.H; ++h) {
        const float4 p = __ldcg(reinterpret_cast<const float4*>(part + ((size_t)h * a.M + m) * D + col));
        acc.x += p.x;
        acc.y += p.y;
        acc.z += p.z;
        acc.w += p.w;
      }
      const float4 x = *reinterpret_cast<const float4*>(s.x + (size_t)m * D + col);
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
  consumer_sum<MR>(sum, s.red);
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
  consumer_sum<MR>(sq, s.red);
  if (col < KP) {
    float4 gg = make_float4(0.f, 0.f, 0.f, 0.f), bb = gg;
    if (own) {
      gg = *reinterpret_cast<const float4*>(g + col);
      bb = *reinterpret_cast<const float4*>(b + col);
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      uint2 packed = make_uint2(0, 0);
      if (own && m < a.M) {
        const float rstd = rsqrtf(sq[m] / (float)D + kLnEps);
        float4 y;
        y.x = (r[m].x - mean[m]) * rstd * gg.x + bb.x;
        y.y = (r[m].y - mean[m]) * rstd * gg.y + bb.y;
        y.z = (r[m].z - mean[m]) * rstd * gg.z + bb.z;
        y.w = (r[m].w - mean[m]) * rstd * gg.w + bb.w;
        *reinterpret_cast<float4*>(s.x + (size_t)m * D + col) = y;
        packed = make_uint2(pack_bf16(y.x, y.y), pack_bf16(y.z, y.w));
      }
      *reinterpret_cast<uint2*>(s.xs + (size_t)m * KP + col) = packed;
    }
  }
  csync();
}

// Rows [r0, r1) of a [*, K] weight streamed through the ring, against the
// staged rows xs (stride KP, zero padded): warp w takes row w of every piece.
// Lane l holds columns c*256 + 8l .. 8l+7 of every 256-column chunk c, as in
// the multi-kernel projection.  epi(m, row, acc) runs on lane m.
template <int MR, typename Epi>
__device__ __forceinline__ void gemv_stream(Consumer& cs, int K, int r0, int r1, const bf16* xs, int KP, int M,
                                            Epi epi) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rps = rows_per_stage(K);
  const int nch = (K + 255) / 256;
  for (int p = r0; p < r1; p += rps) {
    const bf16* ws = reinterpret_cast<const bf16*>(cs.wait());
    const int n = min(rps, r1 - p);
    for (int i = warp; i < n; i += kPWarps) {
      float acc[MR];
#pragma unroll
      for (int m = 0; m < MR; ++m) acc[m] = 0.f;
      for (int c = 0; c < nch; ++c) {
        const int col = c * 256 + lane * 8;
        const uint4 w = col < K ? *reinterpret_cast<const uint4*>(ws + (size_t)i * K + col) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int m = 0; m < MR; ++m)
          acc[m] += dot8(w, *reinterpret_cast<const uint4*>(xs + (size_t)m * KP + col));
      }
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        acc[m] = warp_sum(acc[m]);
        if (lane == m && m < M) epi(m, p + i, acc[m]);
      }
    }
    cs.release();
  }
}

// Exchange `count` floats per source rank with the cluster: src (this CTA's
// values) go to slot [rank] (of `cap` floats) of every peer's buffer; returns (bounded) once
// every peer's values are in this CTA's buffer, which it returns.  xbar
// counts one arrival per rank.  Buffers alternate by use, so a peer that is
// one exchange ahead never overwrites values still being read.
__device__ __forceinline__ const float* cluster_exchange(const PArgs& a, cg::cluster_group& cluster, float* bufs,
                                                         const float* src, int count, int cap, uint64_t* xbar,
                                                         int& uses, int* failed) {
  const int rank = (int)cluster.block_rank();
  float* buf = bufs + (size_t)(uses & 1) * kPClus * cap;
  for (int idx = threadIdx.x; idx < kPClus * count; idx += kPConsumers) {
    const int peer = idx / count, i = idx % count;
    cluster.map_shared_rank(buf, peer)[rank * cap + i] = src[i];
  }
  csync();
  if (threadIdx.x == 0) {  // the release of each arrival covers the consumers' stores (ordered by csync)
    for (int peer = 0; peer < kPClus; ++peer) {
      uint32_t remote;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(xbar)), "r"(peer));
      asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
    }
  }
  const unsigned parity = uses & 1;
  ++uses;
  if (*(volatile int*)failed) return buf;
  const uint32_t addr = smem_u32(xbar);
  bool done = false;
  const unsigned long long t0 = global_ns();
  while (!done) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(addr), "r"(parity)
        : "memory");
    done = r != 0;
    if (!done && global_ns() - t0 > kMbarWaitNs) {
      *(volatile int*)failed = 1;
      atomicExch(a.err, kErrRing);
      break;
    }
  }
  return buf;
}

// Attention of head h for every active row (keys split over the cluster),
// then this CTA's quarter of the head's out-projection as a partial sum:
// part[h][m][n] = sum_d Who[h][n][d] * o[m][d] for n in the CTA's quarter.
template <int MR>
__device__ void head_attention(const PArgs& a, const PLayer& W, cg::cluster_group& cluster, PSmem& s, Consumer& cs,
                               bool cross, int h, float* part, uint64_t* xbar, int* uses) {
  const int rank = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = tid >> 3, sub = tid & 7;  // 32 groups of 8 lanes: one key row per group
  constexpr int G = kPConsumers / 8;
  // the head's query of every row (written in the previous phase)
  for (int idx = tid; idx < a.M * kHeadDim; idx += kPConsumers) {
    const int m = idx / kHeadDim, d = idx % kHeadDim;
    s.qh[idx] = __bfloat162float(__ldcg(a.q + (size_t)m * a.D + h * kHeadDim + d));
  }
  csync();
  float stat[MR][2];
  // ---- scores: streamed keys [j0, js), then the keys written in this launch [js, j1)
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    stat[m][0] = -INFINITY;
    stat[m][1] = 0.f;
    if (m >= a.M) continue;
    const KeyRange k = key_range(a, m, cross, rank);
    float* sc = s.sc + (size_t)m * a.chunk_cap;
    float q[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) q[t] = s.qh[m * kHeadDim + sub * 8 + t];
    float lmax = -INFINITY;
    auto score = [&](uint4 kv, int j) {
      float d = bf_lo(kv.x) * q[0];
      d = fmaf(bf_hi(kv.x), q[1], d);
      d = fmaf(bf_lo(kv.y), q[2], d);
      d = fmaf(bf_hi(kv.y), q[3], d);
      d = fmaf(bf_lo(kv.z), q[4], d);
      d = fmaf(bf_hi(kv.z), q[5], d);
      d = fmaf(bf_lo(kv.w), q[6], d);
      d = fmaf(bf_hi(kv.w), q[7], d);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      if (j >= 0) {
        d = round_bf16(d) * 0.125f;  // head_dim ** -0.5
        if (sub == 0) sc[j - k.j0] = d;
        lmax = fmaxf(lmax, d);
      }
    };
    const int nb = key_blocks(k);
    for (int b = 0; b < nb; ++b) {
      int lo, hi;
      block_keys(k, b, lo, hi);
      const unsigned char* st = cs.wait();
      for (int i = grp; i < kPKeys; i += G) {  // uniform trip count: shuffles need every lane
        const bool in = i < hi - lo;
        const uint4 kv = in ? *reinterpret_cast<const uint4*>(st + (size_t)i * 128 + sub * 16) : make_uint4(0, 0, 0, 0);
        score(kv, in ? lo + i : -1);
      }
      cs.release();
    }
    for (int base = k.js; base < k.j1; base += G) {
      const int j = base + grp;
      const bool in = j < k.j1;
      const uint4 kv = in ? __ldcg(reinterpret_cast<const uint4*>(key_row(a, W, cross, false, k.slot, h, j) + sub * 8))
                          : make_uint4(0, 0, 0, 0);
      score(kv, in ? j : -1);
    }
    lmax = warp_max(lmax);
    if (lane == 0) s.red[warp] = lmax;
    csync();
    float bm = s.red[0];
#pragma unroll
    for (int w = 1; w < kPWarps; ++w) bm = fmaxf(bm, s.red[w]);
    csync();
    float lsum = 0.f;
    for (int j = k.j0 + tid; j < k.j1; j += kPConsumers) lsum += expf(sc[j - k.j0] - bm);
    lsum = warp_sum(lsum);
    if (lane == 0) s.red[warp] = lsum;
    csync();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kPWarps; ++w) t += s.red[w];
    stat[m][0] = bm;
    stat[m][1] = t;
    csync();
  }
  // ---- softmax statistics of the whole head, through the cluster
  if (tid < a.M * 2) s.red[64 + tid] = stat[tid / 2][tid % 2];
  csync();
  const float* st0 = cluster_exchange(a, cluster, s.xch0, s.red + 64, a.M * 2, MR * 2, &xbar[0], uses[0], cs.failed);
  csync();
  // ---- p = bf16(exp(s - max) / sum), partial p.V
  float ov[MR][8];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
#pragma unroll
    for (int t = 0; t < 8; ++t) ov[m][t] = 0.f;
    if (m >= a.M) continue;
    const KeyRange k = key_range(a, m, cross, rank);
    const float* sc = s.sc + (size_t)m * a.chunk_cap;
    float gmax = -INFINITY;
#pragma unroll
    for (int r = 0; r < kPClus; ++r) gmax = fmaxf(gmax, st0[r * MR * 2 + m * 2]);
    float gsum = 0.f;
#pragma unroll
    for (int r = 0; r < kPClus; ++r) {
      const float sm = st0[r * MR * 2 + m * 2 + 1];
      if (sm > 0.f) gsum += sm * expf(st0[r * MR * 2 + m * 2] - gmax);
    }
    auto accum = [&](uint4 vv, int j) {
      const float p = j >= 0 ? round_bf16(expf(sc[j - k.j0] - gmax) / gsum) : 0.f;
      ov[m][0] = fmaf(p, bf_lo(vv.x), ov[m][0]);
      ov[m][1] = fmaf(p, bf_hi(vv.x), ov[m][1]);
      ov[m][2] = fmaf(p, bf_lo(vv.y), ov[m][2]);
      ov[m][3] = fmaf(p, bf_hi(vv.y), ov[m][3]);
      ov[m][4] = fmaf(p, bf_lo(vv.z), ov[m][4]);
      ov[m][5] = fmaf(p, bf_hi(vv.z), ov[m][5]);
      ov[m][6] = fmaf(p, bf_lo(vv.w), ov[m][6]);
      ov[m][7] = fmaf(p, bf_hi(vv.w), ov[m][7]);
    };
    const int nb = key_blocks(k);
    for (int b = 0; b < nb; ++b) {
      int lo, hi;
      block_keys(k, b, lo, hi);
      const unsigned char* st = cs.wait();
      for (int i = grp; i < hi - lo; i += G)
        accum(*reinterpret_cast<const uint4*>(st + (size_t)i * 128 + sub * 16), lo + i);
      cs.release();
    }
    for (int j = k.js + grp; j < k.j1; j += G)
      accum(__ldcg(reinterpret_cast<const uint4*>(key_row(a, W, cross, true, k.slot, h, j) + sub * 8)), j);
  }
  // this CTA's partial output per row: groups reduced in fixed order
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    if (m >= a.M) continue;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      ov[m][t] += __shfl_xor_sync(0xffffffffu, ov[m][t], 8);
      ov[m][t] += __shfl_xor_sync(0xffffffffu, ov[m][t], 16);
    }
    if (lane < 8) {
#pragma unroll
      for (int t = 0; t < 8; ++t) s.red[warp * kHeadDim + lane * 8 + t] = ov[m][t];
    }
    csync();
    if (tid < kHeadDim) {
      float o = 0.f;
#pragma unroll
      for (int w = 0; w < kPWarps; ++w) o += s.red[w * kHeadDim + tid];
      s.oh[m * kHeadDim + tid] = o;
    }
    csync();
  }
  const float* st1 =
      cluster_exchange(a, cluster, s.xch1, s.oh, a.M * kHeadDim, MR * kHeadDim, &xbar[1], uses[1], cs.failed);
  csync();
  // o = bf16(sum over ranks in order)
  for (int idx = tid; idx < a.M * kHeadDim; idx += kPConsumers) {
    float o = 0.f;
#pragma unroll
    for (int r = 0; r < kPClus; ++r) o += st1[r * MR * kHeadDim + idx];
    s.oh[idx] = round_bf16(o);
  }
  csync();
  // ---- out-projection partial of the CTA's quarter of the features
  const int per = a.D / kPClus, n0 = rank * per;
  for (int p = 0; p < per; p += kPKeys) {  // 128 features (x 64 inputs) per piece
    const unsigned char* st = cs.wait();
    const int n = min(kPKeys, per - p);
    for (int i = grp; i < kPKeys; i += G) {
      const bool in = i < n;
      const uint4 w = in ? *reinterpret_cast<const uint4*>(st + (size_t)i * 128 + sub * 16) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        if (m >= a.M) continue;
        const float* o = s.oh + m * kHeadDim + sub * 8;
        float d = bf_lo(w.x) * o[0];
        d = fmaf(bf_hi(w.x), o[1], d);
        d = fmaf(bf_lo(w.y), o[2], d);
        d = fmaf(bf_hi(w.y), o[3], d);
        d = fmaf(bf_lo(w.z), o[4], d);
        d = fmaf(bf_hi(w.z), o[5], d);
        d = fmaf(bf_lo(w.w), o[6], d);
        d = fmaf(bf_hi(w.w), o[7], d);
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        d += __shfl_xor_sync(0xffffffffu, d, 4);
        if (in && sub == 0) part[((size_t)h * a.M + m) * a.D + n0 + p + i] = d;
      }
    }
    cs.release();
  }
}

// ---------------------------------------------------------------- the kernel
template <int KCH, int MR>
__global__ void __launch_bounds__(kPThreads, 1) step_persistent_kernel(const PArgs a) {
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(128) unsigned char pst_smem[];
  constexpr int KP = KCH * 256;
  const int D = a.D, H = a.H;
  const int rank = (int)cluster.block_rank();
  const int nclusters = gridDim.x / kPClus;
  const int ci = blockIdx.x / kPClus;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int FP = (a.FFN + 255) / 256 * 256;

  __shared__ __align__(8) uint64_t full[kPMaxStages], empty[kPMaxStages], xbar[2];
  __shared__ int failed, ok_s, is_last;
  __shared__ uint32_t rule[kPMaxRows];
  __shared__ unsigned long long wbest[kPWarps][kPMaxRows];

  Ring ring;
  PSmem s;
  {
    unsigned char* p = pst_smem;
    auto take = [&](size_t bytes) {
      unsigned char* q = p;
      p += (bytes + 127) & ~size_t(127);
      return q;
    };
    ring.buf = take((size_t)a.stages * kPStage);
    s.x = reinterpret_cast<float*>(take(sizeof(float) * MR * D));
    s.xs = reinterpret_cast<bf16*>(take(sizeof(bf16) * MR * KP));
    unsigned char* shared_sc = take(max(sizeof(float) * MR * a.chunk_cap, sizeof(bf16) * MR * FP));
    s.sc = reinterpret_cast<float*>(shared_sc);
    s.hs = reinterpret_cast<bf16*>(shared_sc);
    s.qh = reinterpret_cast<float*>(take(sizeof(float) * MR * kHeadDim));
    s.oh = reinterpret_cast<float*>(take(sizeof(float) * MR * kHeadDim));
    s.xch0 = reinterpret_cast<float*>(take(sizeof(float) * 2 * kPClus * MR * 2));
    s.xch1 = reinterpret_cast<float*>(take(sizeof(float) * 2 * kPClus * MR * kHeadDim));
    s.red = reinterpret_cast<float*>(take(sizeof(float) * kPWarps * kHeadDim));
  }
  ring.full = full;
  ring.empty = empty;
  ring.stages = a.stages;
  if (tid == 0) {
    for (int i = 0; i < a.stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kPWarps);
    }
    mbar_init(&xbar[0], kPClus);
    mbar_init(&xbar[1], kPClus);
    failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  trace_mark(a, kTraceSlots - 1);
  cluster.sync();  // barriers initialised everywhere before any copy or remote arrival

  if (warp == kPWarps) {
    // ======================================================== producer warp
    if ((tid & 31) == 0) {
      Producer pr;
      pr.a = &a;
      pr.ring = ring;
      int r0, r1;
      for (int l = 0; l < a.L; ++l) {
        const PLayer& W = a.layers[l];
        const bool kv_only = !a.logits && l == a.L - 1;
        row_slice(3 * D, r0, r1);
        pr.rows(W.wqkv, D, r0, r1);
        if (kv_only) break;
        for (int phase = 0; phase < 2; ++phase) {
          const bool cross = phase == 1;
          for (int h = ci; h < H; h += nclusters) {
            for (int m = 0; m < a.M; ++m) pr.keys(W, cross, false, h, key_range(a, m, cross, rank));
            for (int m = 0; m < a.M; ++m) pr.keys(W, cross, true, h, key_range(a, m, cross, rank));
            const int per = D / kPClus;
            pr.rows((cross ? W.wco_hb : W.wo_hb) + (size_t)h * D * kHeadDim, kHeadDim, rank * per, rank * per + per);
          }
          if (!cross) {
            row_slice(D, r0, r1);
            pr.rows(W.wcq, D, r0, r1);
          }
        }
        row_slice(a.FFN, r0, r1);
        pr.rows(W.w1, D, r0, r1);
        row_slice(D, r0, r1);
        pr.rows(W.w2, a.FFN, r0, r1);
      }
      if (a.logits) {
        row_slice(a.V, r0, r1);
        pr.rows(a.emb, D, r0, r1);
      }
      pr.drain();
    }
    __syncwarp();
  } else {
    // ======================================================== consumer warps
    Consumer cs;
    cs.a = &a;
    cs.ring = ring;
    cs.failed = &failed;
    unsigned target = 0;
    int uses[2] = {0, 0};
    int r0, r1;
    for (int l = 0; l < a.L; ++l) {
      const PLayer& W = a.layers[l];
      const bool kv_only = !a.logits && l == a.L - 1;
      const int tb = l * 8;
      trace_mark(a, tb + 0);
      // ---------------- P1: (embedding) + LayerNorm, QKV rows, K/V append
      if (l == 0)
        combine_ln<MR>(a, s, KP, 0, nullptr, nullptr, a.emb_g, a.emb_b);
      else
        combine_ln<MR>(a, s, KP, 1, nullptr, nullptr, a.layers[l - 1].ln_final_g, a.layers[l - 1].ln_final_b);
      row_slice(3 * D, r0, r1);
      gemv_stream<MR>(cs, D, r0, r1, s.xs, KP, a.M, [&](int m, int row, float acc) {
        const float v = acc + __bfloat162float(W.bqkv[row]);
        if (row < D) {
          a.q[(size_t)m * D + row] = __float2bfloat16_rn(v);
        } else if (row_active(a.rm, a.st, m)) {
          const int c = row - D, which = c >= D, cc = which ? c - D : c;
          bf16* dst = which ? W.vpool : W.kpool;
          dst[paged_offset(a.st.page_table, a.pps, H, row_slot(a.rm, m), cc / kHeadDim, row_pos(a.rm, a.st, m)) +
              cc % kHeadDim] = __float2bfloat16_rn(v);
        }
      });
      grid_barrier(a, target, &ok_s);
      if (kv_only) break;
      trace_mark(a, tb + 1);
      // ---------------- P2: self-attention + out-projection partials
      for (int h = ci; h < H; h += nclusters)
        head_attention<MR>(a, W, cluster, s, cs, false, h, a.part_o, xbar, uses);
      grid_barrier(a, target, &ok_s);
      trace_mark(a, tb + 2);
      // ---------------- P3: residual + self_attn_norm, cross q rows
      combine_ln<MR>(a, s, KP, 2, a.part_o, W.bo, W.ln_self_g, W.ln_self_b);
      row_slice(D, r0, r1);
      gemv_stream<MR>(cs, D, r0, r1, s.xs, KP, a.M, [&](int m, int row, float acc) {
        a.q[(size_t)m * D + row] = __float2bfloat16_rn(acc + __bfloat162float(W.bcq[row]));
      });
      grid_barrier(a, target, &ok_s);
      trace_mark(a, tb + 3);
      // ---------------- P4: cross-attention + cross out-projection partials
      for (int h = ci; h < H; h += nclusters)
        head_attention<MR>(a, W, cluster, s, cs, true, h, a.part_c, xbar, uses);
      grid_barrier(a, target, &ok_s);
      trace_mark(a, tb + 4);
      // ---------------- P5: residual + cross_attn_norm, fc1 rows + GELU
      combine_ln<MR>(a, s, KP, 2, a.part_c, W.bco, W.ln_cross_g, W.ln_cross_b);
      row_slice(a.FFN, r0, r1);
      gemv_stream<MR>(cs, D, r0, r1, s.xs, KP, a.M, [&](int m, int row, float acc) {
        const float v = round_bf16(acc + __bfloat162float(W.b1[row]));
        a.hid[(size_t)m * a.FFN + row] = __float2bfloat16_rn(gelu_erf(v));
      });
      grid_barrier(a, target, &ok_s);
      trace_mark(a, tb + 5);
      // ---------------- P6: fc2 rows, r = x + bf16(fc2 + bias)
      for (int idx = tid; idx < MR * (FP / 8); idx += kPConsumers) {
        const int m = idx / (FP / 8), col = (idx % (FP / 8)) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (m < a.M && col < a.FFN) v = __ldcg(reinterpret_cast<const uint4*>(a.hid + (size_t)m * a.FFN + col));
        *reinterpret_cast<uint4*>(s.hs + (size_t)m * FP + col) = v;
      }
      csync();
      row_slice(D, r0, r1);
      gemv_stream<MR>(cs, a.FFN, r0, r1, s.hs, FP, a.M, [&](int m, int row, float acc) {
        a.r[(size_t)m * D + row] = s.x[(size_t)m * D + row] + round_bf16(acc + __bfloat162float(W.b2[row]));
      });
      grid_barrier(a, target, &ok_s);
      trace_mark(a, tb + 6);
    }

    if (a.logits) {
      // ---------------- logits: final_norm, vocabulary slice, grammar mask, argmax
      const PLayer& last = a.layers[a.L - 1];
      combine_ln<MR>(a, s, KP, 1, nullptr, nullptr, last.ln_final_g, last.ln_final_b);
      if (tid < MR) rule[tid] = tid < a.M ? row_rule(a.gr, a.st, tid) : 0u;
      csync();
      unsigned long long best[MR];
#pragma unroll
      for (int m = 0; m < MR; ++m) best[m] = 0ull;
      row_slice(a.V, r0, r1);
      gemv_stream<MR>(cs, D, r0, r1, s.xs, KP, a.M, [&](int m, int v, float acc) {
        const float logit = round_bf16(acc);
        if (a.logits_out) a.logits_out[(size_t)m * a.V + v] = logit;
        if (token_allowed(a.gr, rule[m], a.V, v)) {
          const unsigned long long key = argmax_key(rescore_logit(a.rs, a.st, m, v, logit + (a.bias ? a.bias[v] : 0.f)), v);
          best[m] = key > best[m] ? key : best[m];
        }
      });
      // lane m of each warp holds row m's best key
      const int lane = tid & 31;
#pragma unroll
      for (int m = 0; m < MR; ++m)
        if (lane == m) wbest[warp][m] = best[m];
      csync();
      if (tid < a.M) {
        unsigned long long k = 0ull;
        for (int w = 0; w < kPWarps; ++w) k = wbest[w][tid] > k ? wbest[w][tid] : k;
        if (k) atomicMax(a.keys + (size_t)tid * kKeyStride, k);
      }
      __threadfence();
      csync();
      if (tid == 0) is_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
      csync();
      if (is_last) {
        __threadfence();
        const bool bad = *(volatile int*)a.err != 0;  // a wait gave up: leave the slots as they were
        for (int sl = tid; sl < a.M; sl += kPConsumers) {
          const unsigned long long k = atomicExch(a.keys + (size_t)sl * kKeyStride, 0ull);
          if (bad) continue;
          const int64_t greedy = key_token(k);
          if (a.greedy_out) a.greedy_out[sl] = greedy;
          const bool active = a.st.finished[sl] == 0;
          const int64_t tok = a.st.token[sl], pos = a.st.position[sl];
          int64_t choice = greedy;
          if (a.forced && a.forced[sl] >= 0) choice = a.forced[sl];
          if (!active) choice = tok;
          const int64_t new_pos = active ? pos + 1 : pos;
          if (active && new_pos < a.T) a.st.out[(size_t)sl * a.T + new_pos] = choice;
          grammar_update(a.gr, a.st, sl, choice, active, new_pos >= a.T - 1);
          rescore_commit(a.rs, a.gr, sl, choice, active);
          a.st.token[sl] = choice;
          a.st.position[sl] = new_pos;
        }
        if (tid == 0) *a.counter = 0u;
      }
    }
    trace_mark(a, 8 * a.L + 1);
    // the last CTA out resets the barrier counters for the next launch
    csync();
    if (tid == 0) {
      __threadfence();
      if (atomicAdd(a.bar + 1, 1u) == gridDim.x - 1) {
        atomicExch(a.bar, 0u);
        atomicExch(a.bar + 1, 0u);
      }
    }
  }
  cluster.sync();  // no CTA leaves while a peer may still write into its shared memory
}

}  // namespace s2r
