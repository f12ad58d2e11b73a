// Tensor-core projection for many rows: D = W X^T with tcgen05 + TMA (sm_100a).
//
// The batched step (16 or more slots) and the prefill chunks of every engine
// multiply a weight matrix W [N, K] by tens to hundreds of activation rows
// X [R, K] (the per-window cross K/V projection has its own persistent kernel,
// crosskv.cuh).  The weights are the large operand, so they are
// the MMA's A operand (M = 128 output features per CTA) and the rows are its B
// operand (NB rows, 64..256): D[n][r] = sum_k W[n][k] X[r][k], both operands
// K-major, bf16 in, fp32 accumulated in tensor memory.
//
//   warp 0, one lane: TMA producer, a 4-stage ring of (W tile 128x64, X tile
//                     NBx64) in shared memory with the 128-byte swizzle;
//                     the first stages' weight tiles are requested before the
//                     kernel waits for the previous kernel (they do not depend
//                     on it), the activation tiles after;
//   warp 1, one lane: issues tcgen05.mma (4 per 64-wide K tile) and commits
//                     each stage back to the producer;
//   all 4 warps:      read the accumulator with tcgen05.ld (warp w owns
//                     features 32w..32w+31) and run the epilogue.
//
// Split-K: the S CTAs that share an output tile (S = 1, 2, 4 or 8, each over
// a contiguous slice of the K tiles) form one thread-block cluster.  Each
// writes its fp32 partial tile to its own shared memory; after a cluster
// barrier CTA s adds rows [s*NB/S, (s+1)*NB/S) of all S partials, in slice
// order, through distributed shared memory and runs the epilogue on them.  No
// partial leaves the cluster and the sum order is fixed.
//
// Epilogues: those of proj.cuh (bias, bf16 rounding, residual, GELU, paged K/V
// append; the same function the CUDA-core kernel runs) and
// EPI_LOGITS, the tied-embedding logits fused with the grammar mask, the mode
// bias and the greedy argmax of logits.cuh: per row a warp reduces its
// 64-bit (value, ~index) keys and publishes them with one atomicMax; the last
// CTA of the grid (a ticket counter) commits the step.
//
// Every mbarrier wait is bounded in time; on a timeout the CTA records an
// error word, stops issuing, waits (bounded) for the copies it issued, frees
// its tensor memory, still takes part in every cluster barrier and returns.
#pragma once

#include <cooperative_groups.h>
#include <cuda.h>

#include "common.cuh"
#include "logits.cuh"
#include "mbarrier.cuh"
#include "proj.cuh"

namespace s2r {

constexpr int kTcThreads = 128;
constexpr int kTcBlockN = 128;  // output features per CTA (MMA M)
constexpr int kTcBlockK = 64;   // K per stage: 128 bytes of bf16, one swizzle row
constexpr int kTcStages = 4;
constexpr int kErrGemmWait = 4;                          // an mbarrier wait of the tensor-core GEMM timed out

constexpr int EPI_LOGITS = 6;  // (after the EpiMode values) tied-embedding logits + grammar mask + greedy argmax (+ commit)
constexpr int kTcMaxSplits = 8;

struct TcArgs {
  ProjArgs p;  // shapes and epilogue pointers: p.M rows, p.N features, p.K
  int k_tiles_per_split;
  int* err;
  LogitsArgs lg;  // EPI_LOGITS only: rows, vocabulary, slot state, grammar, keys, ticket counter
};

__host__ __device__ constexpr size_t tc_smem_bytes(int nb) {
  return (size_t)kTcStages * (kTcBlockN + nb) * kTcBlockK * 2 + 1024;  // + slack for 1024-byte alignment
}

// 2-D tiled TMA load of the box at (x, y) into shared memory (x in elements, a
// multiple of 64 here, so 128-byte aligned); completion is counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B).
// Fields: start address >> 4 [0,14), leading byte offset >> 4 [16,30) (1 for
// swizzled K-major), stride byte offset >> 4 [32,46), version 1 [46,48),
// layout type [61,64) = 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* smem) {
  const uint64_t addr = smem_u32(smem);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: f32 accumulator [4,6)=1, A and B bf16
// [7,10)=1 and [10,13)=1, both K-major, N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int nb) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(nb >> 3) << 17) | ((uint32_t)(kTcBlockN >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma this thread issued has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's tensor-memory lane; complete
// after tmem_wait_ld().
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Split cluster barrier: arrive (release) now, wait (acquire) later.

// Epilogue of one output (m, n) (both in range) given accumulator + bias.
template <int EPI>
__device__ __forceinline__ void tc_store(const TcArgs& t, int m, int n, float v) {
  if constexpr (EPI != EPI_LOGITS) proj_epilogue_biased<EPI>(t.p, m, n, v);
}

// EPI_LOGITS: the logit of token n for row m (stored when requested) and its
// argmax key, 0 when the grammar masks the token.
__device__ __forceinline__ unsigned long long tc_logit_key(const TcArgs& t, uint32_t rule, const RescoreRow& rr, int m,
                                                           int n, float v, float bias) {
  const float logit = round_bf16(v);
  if (t.lg.logits_out) t.lg.logits_out[(size_t)m * t.lg.V + n] = logit;
  if (!token_allowed(t.lg.gr, rule, t.lg.V, n)) return 0ull;
  const float x = rescored_token(t.lg.rs, n) ? rescore_logit_call(t.lg.rs, rr, m, n, logit + bias) : logit + bias;
  return argmax_key(x, n);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long k) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
    k = other > k ? other : k;
  }
  return k;
}

template <int NB, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                   const __grid_constant__ TcArgs t) {
  static_assert(NB == 64 || NB == 128 || NB == 256, "NB: 64, 128 or 256 rows");
  constexpr uint32_t kBytesW = kTcBlockN * kTcBlockK * 2;
  constexpr uint32_t kBytesX = NB * kTcBlockK * 2;
  constexpr uint32_t kCols = NB;  // tensor-memory columns: one fp32 accumulator column per row
  static_assert((size_t)NB * kTcBlockN * 4 <= (size_t)kTcStages * (kBytesW + kBytesX), "partial tile fits the stages");
  extern __shared__ __align__(1024) unsigned char tc_smem[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem) + 1023) & ~uintptr_t(1023));
  unsigned char* sw = base;                        // [S][128 rows][128 B]
  unsigned char* sx = base + kTcStages * kBytesW;  // [S][NB rows][128 B]
  float* part = reinterpret_cast<float*>(base);    // [NB][128] after the MMAs: this CTA's partial tile
  __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], done;
  __shared__ uint32_t tmem_base;
  __shared__ int aborted, good, is_last;
  __shared__ uint32_t rule[EPI == EPI_LOGITS ? NB : 1];
  __shared__ unsigned long long row_best[EPI == EPI_LOGITS ? NB : 1];  // this CTA's best key per row
  __shared__ RescoreRow rrow[EPI == EPI_LOGITS ? NB : 1];              // rescoring state per row
  __shared__ float sbias[kTcBlockN];  // bias of this CTA's features (weights: read before the wait)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, splits = gridDim.x, n_tile = blockIdx.y, m_tile = blockIdx.z;
  const int n0 = n_tile * kTcBlockN, m0 = m_tile * NB;
  const int M = t.p.M, N = t.p.N;
  const int k_tiles = (t.p.K + kTcBlockK - 1) / kTcBlockK;
  const int kt0 = split * t.k_tiles_per_split;
  const int nk = max(0, min(k_tiles, kt0 + t.k_tiles_per_split) - kt0);

  if constexpr (EPI != EPI_LOGITS)
    sbias[threadIdx.x] = n0 + (int)threadIdx.x < N ? __bfloat162float(t.p.bias[n0 + threadIdx.x]) : 0.f;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    aborted = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_launch_dependents();

  int issued = 0;
  if (warp == 0 && lane == 0) {
    const int pre = min(nk, kTcStages);
    for (int i = 0; i < pre; ++i) {
      mbar_expect_tx(&full[i], kBytesW + kBytesX);
      tma_load_2d(sw + i * kBytesW, &map_w, (kt0 + i) * kTcBlockK, n0, &full[i]);
    }
    pdl_wait();  // the activation rows come from the previous kernel
    for (int i = 0; i < pre; ++i) tma_load_2d(sx + i * kBytesX, &map_x, (kt0 + i) * kTcBlockK, m0, &full[i]);
    issued = pre;
    for (int i = pre; i < nk; ++i) {
      const int s = i % kTcStages;
      if (!mbar_wait(&empty[s], ((i / kTcStages) - 1) & 1)) {
        atomicExch(t.err, kErrGemmWait);
        aborted = 1;
        break;
      }
      mbar_expect_tx(&full[s], kBytesW + kBytesX);
      tma_load_2d(sw + s * kBytesW, &map_w, (kt0 + i) * kTcBlockK, n0, &full[s]);
      tma_load_2d(sx + s * kBytesX, &map_x, (kt0 + i) * kTcBlockK, m0, &full[s]);
      issued = i + 1;
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = umma_idesc_bf16(NB);
    for (int i = 0; i < nk; ++i) {
      const int s = i % kTcStages;
      if (!mbar_wait(&full[s], (i / kTcStages) & 1)) {
        atomicExch(t.err, kErrGemmWait);
        aborted = 1;
        break;
      }
      tmem_fence_after();
      const uint64_t da = umma_desc_sw128(sw + s * kBytesW);
      const uint64_t db = umma_desc_sw128(sx + s * kBytesX);
#pragma unroll
      for (int k = 0; k < kTcBlockK / 16; ++k)  // K = 16 per MMA: +32 bytes, +2 in the address field
        umma_bf16(tmem, da + 2 * k, db + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
      umma_commit(&empty[s]);
    }
    umma_commit(&done);  // arrives at once when nothing was issued
  }
  __syncthreads();  // both roles have finished issuing
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait(&done, 0) && !aborted;
    if (!ok) {  // wait (bounded) for the copies still in flight before the shared memory is reused
      for (int i = max(0, issued - kTcStages); i < issued; ++i) mbar_wait(&full[i % kTcStages], (i / kTcStages) & 1);
    }
    good = ok;
  }
  __syncthreads();
  tmem_fence_after();
  pdl_wait();  // the previous kernel may read what the epilogue overwrites until it completes
  if constexpr (EPI == EPI_LOGITS) {
    for (int r = threadIdx.x; r < NB; r += kTcThreads) {
      rule[r] = m0 + r < M ? row_rule(t.lg.gr, t.lg.st, m0 + r) : 0u;
      rrow[r] = m0 + r < M ? rescore_row(t.lg.rs, t.lg.st, m0 + r) : RescoreRow{0, -1, 0, 0};
      row_best[r] = 0ull;
    }
    __syncthreads();
  }

  const int f_own = warp * 32 + lane;  // the feature (tensor-memory lane) this thread reads
  const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
  const bool have = good && nk > 0;
  if (splits == 1) {
    // ---- the accumulator is the result: epilogue straight from tensor memory
    const int n = n0 + f_own;
#pragma unroll 1
    for (int c = 0; c < NB; c += 32) {
      uint32_t r[32];
      if (have) {
        tmem_ld32(taddr + c, r);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
      if constexpr (EPI == EPI_LOGITS) {
        // the 32 rows' keys first (independent loads of the grammar and rescoring tables), then
        // the warp reductions
        const float bias = (n < N && t.lg.bias) ? t.lg.bias[n] : 0.f;
        unsigned long long key[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int m = m0 + c + j;
          key[j] = (m < M && n < N) ? tc_logit_key(t, rule[c + j], rrow[c + j], m, n, __uint_as_float(r[j]), bias) : 0ull;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const unsigned long long k = warp_max_u64(key[j]);
          if (lane == 0 && k) atomicMax(&row_best[c + j], k);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int m = m0 + c + j;
          if (m < M && n < N) tc_store<EPI>(t, m, n, __uint_as_float(r[j]) + sbias[f_own]);
        }
      }
    }
    tmem_fence_before();
    __syncthreads();
    if (warp == 0)
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
  } else {
    // ---- split-K over the cluster: every CTA writes its partial tile to its
    // own shared memory; after a cluster barrier CTA s adds rows
    // [s*R, (s+1)*R), R = NB/S, of the S partials in slice order through
    // distributed shared memory and runs the epilogue on them.
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
#pragma unroll 1
    for (int c = 0; c < NB; c += 32) {
      uint32_t r[32];
      if (have) {
        tmem_ld32(taddr + c, r);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) part[(c + j) * kTcBlockN + f_own] = __uint_as_float(r[j]);
    }
    tmem_fence_before();
    __syncthreads();
    if (warp == 0)
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
    cluster_arrive();
    cluster_wait();  // every partial tile of the cluster is in shared memory
    const int rows = NB / splits, r0 = split * rows;
    // 32 threads per row (4 features each): warp w takes rows r0 + w, r0 + w + 4, ...
    constexpr int kMaxIters = NB / 2 * (kTcBlockN / 4) / kTcThreads;  // rows <= NB/2 with 2+ slices
    float4 sums[kMaxIters];
#pragma unroll
    for (int it = 0; it < kMaxIters; ++it) {
      const int idx = threadIdx.x + it * kTcThreads;
      if (idx < rows * (kTcBlockN / 4)) {
        const int r = r0 + idx / (kTcBlockN / 4), f = (idx % (kTcBlockN / 4)) * 4;
        float4 acc = *reinterpret_cast<const float4*>(cluster.map_shared_rank(part, 0) + r * kTcBlockN + f);
#pragma unroll
        for (int sp = 1; sp < kTcMaxSplits; ++sp) {
          if (sp < splits) {
            const float4 x = *reinterpret_cast<const float4*>(cluster.map_shared_rank(part, sp) + r * kTcBlockN + f);
            acc.x += x.x;
            acc.y += x.y;
            acc.z += x.z;
            acc.w += x.w;
          }
        }
        sums[it] = acc;
      }
    }
    cluster_arrive();  // done reading the peers' shared memory; the epilogue overlaps the barrier
#pragma unroll
    for (int it = 0; it < kMaxIters; ++it) {
      const int idx = threadIdx.x + it * kTcThreads;
      if (idx < rows * (kTcBlockN / 4)) {
        const int r = r0 + idx / (kTcBlockN / 4), f = (idx % (kTcBlockN / 4)) * 4;
        const float a4[4] = {sums[it].x, sums[it].y, sums[it].z, sums[it].w};
        const int m = m0 + r;
        if constexpr (EPI == EPI_LOGITS) {
          unsigned long long key = 0ull;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (m < M && n0 + f + j < N) {
              const int n = n0 + f + j;
              const unsigned long long kj =
                  tc_logit_key(t, rule[r], rrow[r], m, n, a4[j], t.lg.bias ? t.lg.bias[n] : 0.f);
              key = kj > key ? kj : key;
            }
          }
          key = warp_max_u64(key);  // the warp covers the row's 128 features
          if (lane == 0 && key) atomicMax(&row_best[r], key);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (m < M && n0 + f + j < N) tc_store<EPI>(t, m, n0 + f + j, a4[j] + sbias[f + j]);
        }
      }
    }
    cluster_wait();  // peers keep their shared memory until every CTA has read it
  }

  if constexpr (EPI == EPI_LOGITS) {
    // ---- one global atomic per row and CTA (rows on separate lines), then the
    // last CTA of the grid commits the step
    __syncthreads();
    for (int r = threadIdx.x; r < NB; r += kTcThreads)
      if (row_best[r] && m0 + r < M) atomicMax(t.lg.keys + (size_t)(m0 + r) * kKeyStride, row_best[r]);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0)
      is_last = atomicAdd(t.lg.counter, 1u) == gridDim.x * gridDim.y * gridDim.z - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    commit_rows(t.lg);
    if (threadIdx.x == 0) *t.lg.counter = 0u;
  }
}

// LayerNorm (IN_LN) or embedding + LayerNorm (IN_EMBED) of rows [0, M) into
// bfloat16 rows of stride KCH*256 (the tensor-core GEMM's X operand), and the
// float32 rows into x_out.  One row per CTA, staged by all of its threads.
template <int KCH, int IN>
__global__ void __launch_bounds__(128) ln_rows_kernel(const ProjArgs a, bf16* __restrict__ xb) {
  pdl_launch_dependents();
  pdl_wait();
  // one row per CTA, staged by the whole block
  const int m = blockIdx.x;
  stage_ln_row_block<KCH, IN>(a, xb + (size_t)m * (KCH * 256), m, a.gamma, a.beta, true);
}

}  // namespace s2r
