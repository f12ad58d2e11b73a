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
// the C partial outputs are added in rank order.  Every exchange is a push:
// each CTA sends its value into its peers' shared memory with asynchronous
// remote stores that count their bytes on the receiver's mbarrier, so a CTA
// waits only for the values it needs and reads only its own shared memory.  Keys beyond the visible
// length are never read; the reference masks them with -inf, which gives the
// same softmax.
//   self  (engine.py:303-312): keys 0..position of the slot, paged pool
//   cross (engine.py:134,208-209,313): the slot's first `frames` encoder frames
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"
#include "mbarrier.cuh"
#include "proj.cuh"

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
  int stage_cap;  // kAttnPreStage: key and value rows per CTA held in shared memory
  int splits;     // CTAs per (row, head): the cluster size the launch must have
  int* err;       // device error word: set (and the work skipped) on a broken invariant
  const int32_t* order;  // [M] row of each grid z index (longest first), or null: identity
  // kAccOut (engines below 16 slots): the out-projection that follows the attention
  // (engine.py:292,312): every CTA adds its share of the head's contribution,
  // sum_d Wo[n][64h + d] o_h[d], to acc_out[m][n] as a fixed-point sum (acc_add);
  // the next launch adds the bias and the residual and normalises (IN_ACC)
  int D;
  const bf16* wo;                 // out-projection weight [D, D]
  unsigned long long* acc_out;    // [M][D]
  // fuse_q (cross attention, kAttnPreStage with kAccOut, 8 or 16 splits, D <= 1024): the kernel
  // forms its input row itself, x = LayerNorm(x_in + bf16(acc_in + bias_in)) (the previous
  // attention's residual sum and norm, engine.py:312), writes it to x_out once, and computes
  // its head's query rows from it, q = bf16(x Wq^T + bq), 64 / splits rows per CTA
  const unsigned long long* acc_in;  // [M][D]
  const bf16* bias_in;               // [D]
  const float* x_in;                 // [M][D]
  float* x_out;                      // [M][D]
  const float *ln_g, *ln_b;          // [D]
  const bf16* wq;  // [D, D]
  const bf16* bq;  // [D]
  int fuse_q;
  unsigned long long* zero;  // cleared after the wait (an accumulator the launch before has read)
  int zero_n;
  L2Ahead ahead;  // what the next kernel reads, prefetched into the L2 before the wait
};

constexpr int kAttnOutPrefetch = 4;  // out-projection passes (32 features each) loaded before the wait

constexpr int kErrAttnCluster = 1;  // launched without the expected cluster shape
constexpr int kErrAttnChunk = 2;    // a row's keys do not fit the score buffer
constexpr int kErrAttnStage = 5;    // a bulk copy into shared memory did not complete in time
constexpr int kErrAttnExchange = 6; // a value from a peer CTA did not arrive in time

// How a CTA gets its keys and values ahead of the PDL wait.
constexpr int kAttnPreNone = 0;   // read in the loops (batched engines, which keep occupancy)
constexpr int kAttnPreRegs = 1;   // the first pass of the CTA's earlier keys in registers
constexpr int kAttnPreStage = 2;  // all of them (up to stage_cap rows) bulk-copied to shared memory
// static shared memory of the kernel plus the 1 KB the SM reserves per CTA (upper bound)
constexpr size_t kAttnStaticSmem = 4096;
constexpr size_t kAttnStaticSmemWide = 8192;  // the same for the 16-split instantiations
// shared memory of an SM left to the projection kernels that run beside the attention
constexpr size_t kAttnOtherSmem = 32768;

constexpr int kAttnThreads = 256;
constexpr int kAttnMaxSplits = 16;  // CTAs per (row, head) at most (above 8: non-portable clusters)
constexpr int kAttnGroups = kAttnThreads / 8;  // 8 lanes x 16 bytes per key row
static_assert(kAttnThreads == 4 * kHeadDim && kAttnGroups % 4 == 0, "the partial-output sum takes 4 threads per dimension");
constexpr int kAttnUnroll = 4;  // keys per group and pass (kAttnPreNone / kAttnPreRegs)
constexpr int kAttnQRows = 8;  // fuse_q: query rows per CTA at most (64 / splits, one per warp)
constexpr int kAttnQLnGroups = 128;  // fuse_q: 8-column groups of the input row (D <= 1024)
constexpr int kAttnUnrollStaged = 8;  // the same from shared memory (kAttnPreStage): more keys in flight

__device__ __forceinline__ uint32_t pack_bf16_pair(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ const bf16* attn_row(const AttnArgs& a, const bf16* base, int slot, int h, int j) {
  if (a.cross) return base + (((size_t)slot * a.H + h) * a.frames_cap + j) * kHeadDim;
  return base + paged_offset(a.st.page_table, a.pages_per_slot, a.H, slot, h, j);
}

// Dynamic shared memory of one attention CTA: the score buffer, the partial
// outputs of the key groups and, for kAttnPreStage, the staged key and value
// rows and (with fuse_q) the input LayerNorm's parameters, the previous
// out-projection's bias, the CTA's query weight rows and the normalised input
// row.  Every part starts 16-byte aligned.
struct AttnSmem {
  size_t part, sk, sv, sg, sb, sbi, sw, sxq, total;
  __host__ __device__ AttnSmem(int chunk_cap, int stage_cap, int D, bool fuse_q) {
    const size_t dq = fuse_q ? (size_t)D : 0;
    part = (size_t)((chunk_cap + 3) & ~3) * 4;
    sk = part + (size_t)kAttnGroups * kHeadDim * 4;
    sv = sk + (size_t)stage_cap * kHeadDim * 2;
    sg = sv + (size_t)stage_cap * kHeadDim * 2;
    sb = sg + dq * 4;
    sbi = sb + dq * 4;
    sw = sbi + ((dq * 2 + 15) & ~(size_t)15);
    sxq = sw + dq * kAttnQRows * 2;
    total = sxq + ((dq * 2 + 15) & ~(size_t)15);
  }
};

// kPre says how the CTA's keys and values written before the step (every key
// of a cross-attention row; the keys before the row's own position of a self-
// attention row) reach it:
//   kAttnPreRegs  the first pass (kAttnGroups * kAttnUnroll keys) is loaded
//                 into registers before the PDL wait;
//   kAttnPreStage up to stage_cap rows are bulk-copied into shared memory
//                 before the wait, the keys of the step itself after it (plain
//                 loads into the same buffer), so both loops read shared memory.
// Reading before the wait is safe because the first kernel of every decode
// step and prefill chunk starts only after everything before it has completed.
// Engines below 16 slots use these; the batched engines keep shared memory and
// registers for occupancy.
//
// kAccOut (engines below 16 slots): the kernel also runs the out-projection
// that follows the attention in the reference (engine.py:292,312).  Every CTA
// of the head's cluster adds the C partial outputs in rank order (the same o
// in each), rounds the head's output to bf16 as the reference does, computes
// its 1/C of the output features of the head's share of the projection,
// sum_d Wo[n][64h + d] o[d] (the weights are loaded before the PDL wait), and
// adds it to acc_out[m][n] as a fixed-point sum: the totals do not depend on
// the order in which the H*C CTAs of a row arrive, and nothing waits for the
// last of them.  The next launch adds the bias and the residual and
// normalises the row (IN_ACC), as reference's self_attn_norm / cross_attn_norm.
// Register budget: the fused kernels (kAccOut) at most 104 a thread (two
// attention CTAs and a projection CTA share an SM's 64K), the batched one 48
// (five CTAs an SM).  Left to itself ptxas chose 80 for the fused kernels and
// spilled.
// kMaxSplits sizes the exchange arrays: 8, or 16 for the wide cross attention (an instantiation
// of its own, so that the 8-way kernels keep their shared memory).
template <int kPre, bool kAccOut, int kMaxSplits = 8>
__global__ void __maxnreg__(kAccOut ? 104 : 48) attn_kernel(const AttnArgs a) {
  constexpr bool kStage = kPre == kAttnPreStage;
  constexpr int kU = kStage ? kAttnUnrollStaged : kAttnUnroll;
  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.dim_blocks().x;
  const int rank = (int)cluster.block_rank();
  const int h = blockIdx.y, m = a.order ? a.order[blockIdx.z] : (int)blockIdx.z;
  extern __shared__ __align__(16) unsigned char attn_smem[];
  const bool fuse_q = kStage && kAccOut && a.fuse_q;
  const int qrows = fuse_q ? kHeadDim / C : 0;  // fuse_q: this CTA's query rows (8 or 4: 8 or 16 splits)
  const AttnSmem lay(a.chunk_cap, kStage ? a.stage_cap : 0, a.D, fuse_q);
  float* sc = reinterpret_cast<float*>(attn_smem);                // [chunk_cap] scores, then exp values
  float* part = reinterpret_cast<float*>(attn_smem + lay.part);   // [kAttnGroups][64] partial outputs
  bf16* sk = reinterpret_cast<bf16*>(attn_smem + lay.sk);         // kStage: [stage_cap][64] keys
  bf16* sv = reinterpret_cast<bf16*>(attn_smem + lay.sv);         //         [stage_cap][64] values
  float* sg = reinterpret_cast<float*>(attn_smem + lay.sg);       // fuse_q: input LayerNorm weight [D]
  float* sb = reinterpret_cast<float*>(attn_smem + lay.sb);       //         input LayerNorm bias [D]
  bf16* sbi = reinterpret_cast<bf16*>(attn_smem + lay.sbi);       //         previous out-projection bias [D]
  bf16* sw = reinterpret_cast<bf16*>(attn_smem + lay.sw);         //         this CTA's query weight rows [8][D]
  bf16* sxq = reinterpret_cast<bf16*>(attn_smem + lay.sxq);       //         the normalised input row [D]
  __shared__ float xred[2][kMaxSplits];          // every rank's partial max and sum
  __shared__ float xo[kMaxSplits][kHeadDim];      // every rank's partial output
  __shared__ float wmax[kAttnThreads / 32], wsum[kAttnThreads / 32];
  __shared__ __align__(16) bf16 sq[kHeadDim];  // kStage: the row's query for this head
  __shared__ __align__(8) uint64_t xbar[4];           // exchanges received: max, sum, output, query
  __shared__ float sqx[kHeadDim];                     // fuse_q: the head's query, from every rank
  __shared__ float ohead[kHeadDim];                   // kAccOut: the head's output, bf16-rounded
  __shared__ float ln_red[kAttnQLnGroups + 2];        // fuse_q: LayerNorm reductions
  __shared__ __align__(8) uint64_t bars[2];           // kStage: [0] key and value rows, [1] fuse_q operands

  pdl_launch_dependents();
  const int tid = threadIdx.x, grp = tid >> 3, sub = tid & 7;
  const int lane = tid & 31, warp = tid >> 5;
  // The whole cluster sees the same row and the same launch shape, so every
  // early return below is taken by all of its CTAs together.
  if (C != a.splits || C > kMaxSplits) {
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
  // kStage: rows [j0, js) are read from shared memory, [j0, jbulk) arrive by bulk copy
  const int js = kStage ? min(j1, j0 + a.stage_cap) : j0;
  const int jbulk = kStage ? max(j0, min(js, fresh)) : j0;
  uint4 kpre[kU], vpre[kU];  // kAttnPreRegs (kU == kAttnUnroll there)
  // kAccOut: this CTA's out-projection features and their weights for head h
  const int per = kAccOut ? (a.D + C - 1) / C : 0, n0 = rank * per;
  uint4 wpre[kAttnOutPrefetch];
  // every rank receives the C maxima and sums; the partial outputs go to every
  // rank with kAccOut, else to rank 0 alone
  const bool gets_o = kAccOut || rank == 0;
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&xbar[i], 1);
    if constexpr (kStage) {
      mbar_init(&bars[0], 1);
      mbar_init(&bars[1], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_expect_tx(&xbar[0], (unsigned)C * 4);
    mbar_expect_tx(&xbar[1], (unsigned)C * 4);
    mbar_expect_tx(&xbar[2], gets_o ? (unsigned)(C * kHeadDim * 4) : 0u);
    mbar_expect_tx(&xbar[3], fuse_q ? (unsigned)(kHeadDim * 4) : 0u);
  }
  if constexpr (kStage) {
    if (tid == 0) {
      mbar_expect_tx(&bars[0], (unsigned)(jbulk - j0) * (2 * kHeadDim * 2));
      mbar_expect_tx(&bars[1], fuse_q ? (unsigned)a.D * 10 + (unsigned)(qrows * a.D * 2) : 0u);
      if (fuse_q) {  // first: what the query rows need
        bulk_load(sg, a.ln_g, (unsigned)a.D * 4, &bars[1]);
        bulk_load(sb, a.ln_b, (unsigned)a.D * 4, &bars[1]);
        bulk_load(sbi, a.bias_in, (unsigned)a.D * 2, &bars[1]);
        // the CTA's 8 query rows of head h: contiguous in Wq
        bulk_load(sw, a.wq + (size_t)(h * kHeadDim + rank * qrows) * a.D, (unsigned)(qrows * a.D * 2),
                  &bars[1]);
      }
      // one copy per run of rows that is contiguous in memory (a page of the
      // self-attention pool; the whole range for cross-attention)
      for (int s = j0; s < jbulk;) {
        const int e = a.cross ? jbulk : min(jbulk, (s / kPageTokens + 1) * kPageTokens);
        const unsigned bytes = (unsigned)(e - s) * kHeadDim * 2;
        bulk_load(sk + (size_t)(s - j0) * kHeadDim, attn_row(a, a.k, slot, h, s), bytes, &bars[0]);
        bulk_load(sv + (size_t)(s - j0) * kHeadDim, attn_row(a, a.v, slot, h, s), bytes, &bars[0]);
        s = e;
      }
      // rows past the stage that were written before the step: into the L2
      // now, so that the loops' reads of them after the wait hit it
      const int jl = min(j1, fresh);
      for (int s = js; s < jl;) {
        const int e = a.cross ? jl : min(jl, (s / kPageTokens + 1) * kPageTokens);
        const uint64_t bytes = (uint64_t)(e - s) * kHeadDim * 2;
        l2_prefetch_bytes(attn_row(a, a.k, slot, h, s), bytes);
        l2_prefetch_bytes(attn_row(a, a.v, slot, h, s), bytes);
        s = e;
      }
    }
  }
  if constexpr (kAccOut) {
#pragma unroll
    for (int p = 0; p < kAttnOutPrefetch; ++p) {
      const int i = p * kAttnGroups + grp, n = n0 + i;
      wpre[p] = (i < per && n < a.D) ? ld_stream(a.wo + (size_t)n * a.D + h * kHeadDim + sub * 8) : make_uint4(0, 0, 0, 0);
    }
  }
  // fuse_q: the bias of this warp's query row
  const float qbias =
      fuse_q && lane == 0 && warp < qrows ? __bfloat162float(a.bq[h * kHeadDim + rank * qrows + warp]) : 0.f;
  if constexpr (kPre == kAttnPreRegs) {
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int j = j0 + grp + u * kAttnGroups;
      const bool ok = j < j1 && j < fresh;
      kpre[u] = ok ? ld_stream(attn_row(a, a.k, slot, h, j) + sub * 8) : make_uint4(0, 0, 0, 0);
      vpre[u] = ok ? ld_stream(attn_row(a, a.v, slot, h, j) + sub * 8) : make_uint4(0, 0, 0, 0);
    }
  }
  if (tid == 0)
    l2_ahead(a.ahead, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x, gridDim.x * gridDim.y * gridDim.z);
  // kStage: whether this thread saw the copies land (if not, it waits for them
  // again, bounded, before the CTA exits; the error word is set either way)
  bool staged = true, q_staged = true;
  __syncthreads();  // the barriers are initialised before anyone waits on them
  // First half of a barrier that proves every peer has started and initialised
  // its barriers before the first store into its shared memory (the wait comes
  // just before that store).
  cluster_arrive_relaxed();
  pdl_wait();
  if (a.zero) {
    const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    for (int i = cta * kAttnThreads + tid; i < a.zero_n; i += gridDim.x * gridDim.y * gridDim.z * kAttnThreads)
      a.zero[i] = 0ull;
  }

  const uint4 qraw = fuse_q ? make_uint4(0, 0, 0, 0)
                            : *reinterpret_cast<const uint4*>(a.q + (size_t)m * a.ldq + h * kHeadDim + sub * 8);
  if (fuse_q) {
    // The input row, LayerNorm(x_in + bf16(acc_in + bias_in)), by the whole
    // block in the order every LayerNorm of the step uses (thread t holds
    // columns 8t .. 8t+7); CTA (rank 0, head 0) keeps the float32 row.
    ProjArgs pa{};
    pa.K = a.D;
    pa.r = a.x_in;
    pa.acc = a.acc_in;
    pa.acc_bias = sbi;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const int col = tid * 8;
    q_staged = mbar_wait(&bars[1], 0);  // parameters, bias and weight rows
    if (!q_staged) atomicExch(a.err, kErrAttnStage);
    if (col < a.D) ln_inputs8<IN_ACC>(pa, m, col, v);
    const float2 st = block_ln_stats<kAttnQLnGroups / 32, kAttnThreads>(v, a.D, ln_red);
    if (col < a.D) {
      float y[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = ln_apply(v[j], st.x, st.y, sg[col + j], sb[col + j]);
      *reinterpret_cast<uint4*>(sxq + col) =
          make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
      if (rank == 0 && h == 0) {
        float* dst = a.x_out + (size_t)m * a.D + col;
        *reinterpret_cast<float4*>(dst) = make_float4(y[0], y[1], y[2], y[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(y[4], y[5], y[6], y[7]);
      }
    }
    __syncthreads();
    // This CTA's query rows of head h (8, or 4 with 16 splits), one per warp, with the projection
    // kernel's arithmetic (16-byte pieces of 8 products, pieces added in
    // order, then the warp butterfly; + bias, rounded to bf16), sent to
    // every rank of the cluster.
    const int kch = a.D / 256;
    const bf16* wrow = sw + (size_t)warp * a.D;
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (c >= kch) break;
      const uint4 w = *reinterpret_cast<const uint4*>(wrow + c * 256 + lane * 8);
      acc += dot8(w, *reinterpret_cast<const uint4*>(sxq + c * 256 + lane * 8));
    }
    acc = warp_sum(acc);
    cluster_wait();  // every peer has started: the first store into its shared memory follows
    if (lane == 0 && warp < qrows) {
      const float qb = round_bf16(acc + qbias);
      for (int r = 0; r < C; ++r) st_async_f32(&sqx[rank * qrows + warp], r, qb, &xbar[3]);
    }
  }
  if constexpr (kStage) {
    if (grp == 0 && !fuse_q) *reinterpret_cast<uint4*>(sq + sub * 8) = qraw;
    // the rows of this step's own positions: plain loads into the stage
    for (int j = jbulk + grp; j < js; j += kAttnGroups) {
      const uint4 kk = ld_stream(attn_row(a, a.k, slot, h, j) + sub * 8);
      const uint4 vv = ld_stream(attn_row(a, a.v, slot, h, j) + sub * 8);
      *reinterpret_cast<uint4*>(sk + (size_t)(j - j0) * kHeadDim + sub * 8) = kk;
      *reinterpret_cast<uint4*>(sv + (size_t)(j - j0) * kHeadDim + sub * 8) = vv;
    }
    staged = mbar_wait(&bars[0], 0);
    if (!staged) atomicExch(a.err, kErrAttnStage);
    if (fuse_q) {
      if (!mbar_wait(&xbar[3], 0)) atomicExch(a.err, kErrAttnExchange);
      if (tid < kHeadDim) sq[tid] = __float2bfloat16_rn(sqx[tid]);  // bf16 values already
    }
    __syncthreads();
  }
  // ---- scores and local max
  float lmax = -INFINITY;
  if constexpr (kStage) {
    // One key per thread.  The eight 8-dimension partial dot products are the
    // ones the 8-lane groups of the other paths form, added in the same
    // butterfly order, so the scores are bit-identical to theirs.  Each lane
    // starts at a different 16-byte piece, so the 8 lanes of a shared-memory
    // phase read 8 different banks.
    for (int j = j0 + tid; j < j1; j += kAttnThreads) {
      const bf16* krow = j < js ? sk + (size_t)(j - j0) * kHeadDim : attn_row(a, a.k, slot, h, j);
      float part8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c0 = 0; c0 < 8; ++c0) {
        const int c = (c0 + lane) & 7;
        const uint4 kk = j < js ? *reinterpret_cast<const uint4*>(krow + c * 8) : ld_stream(krow + c * 8);
        const uint4 qq = *reinterpret_cast<const uint4*>(sq + c * 8);
        float d = bf_lo(kk.x) * bf_lo(qq.x);
        d = fmaf(bf_hi(kk.x), bf_hi(qq.x), d);
        d = fmaf(bf_lo(kk.y), bf_lo(qq.y), d);
        d = fmaf(bf_hi(kk.y), bf_hi(qq.y), d);
        d = fmaf(bf_lo(kk.z), bf_lo(qq.z), d);
        d = fmaf(bf_hi(kk.z), bf_hi(qq.z), d);
        d = fmaf(bf_lo(kk.w), bf_lo(qq.w), d);
        d = fmaf(bf_hi(kk.w), bf_hi(qq.w), d);
#pragma unroll
        for (int t = 0; t < 8; ++t) part8[t] = t == c ? d : part8[t];  // static indices: registers
      }
      float s = ((part8[0] + part8[1]) + (part8[2] + part8[3])) + ((part8[4] + part8[5]) + (part8[6] + part8[7]));
      s = round_bf16(s) * 0.125f;  // head_dim ** -0.5 for head_dim 64
      sc[j - j0] = s;
      lmax = fmaxf(lmax, s);
    }
  }
  // The loop bound is uniform across the block (the shuffles below need all lanes).
  for (int base = j0; !kStage && base < j1; base += kAttnGroups * kU) {
    const int jb = base + grp;
    uint4 kv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int j = jb + u * kAttnGroups;
      if (kPre == kAttnPreRegs && base == j0 && j < fresh)
        kv[u] = kpre[u];
      else if (kStage && j < js)
        kv[u] = *reinterpret_cast<const uint4*>(sk + (size_t)(j - j0) * kHeadDim + sub * 8);
      else
        kv[u] = j < j1 ? ld_stream(attn_row(a, a.k, slot, h, j) + sub * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
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
  if (lane == 0) wmax[warp] = lmax;
  __syncthreads();
  if (!fuse_q) cluster_wait();  // (with fuse_q the query exchange waited already)
  if (tid < C) {  // thread r sends this CTA's max to rank r
    float v = wmax[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) v = fmaxf(v, wmax[w]);
    st_async_f32(&xred[0][rank], tid, v, &xbar[0]);
  }
  if (!mbar_wait(&xbar[0], 0)) atomicExch(a.err, kErrAttnExchange);
  float gmax = -INFINITY;
  for (int r = 0; r < C; ++r) gmax = fmaxf(gmax, xred[0][r]);

  // ---- exp and local sum
  float lsum = 0.f;
  for (int j = j0 + tid; j < j1; j += kAttnThreads) {
    const float e = expf(sc[j - j0] - gmax);
    sc[j - j0] = e;
    lsum += e;
  }
  lsum = warp_sum(lsum);
  if (lane == 0) wsum[warp] = lsum;
  __syncthreads();
  if (tid < C) {
    float v = 0.f;
    for (int w = 0; w < kAttnThreads / 32; ++w) v += wsum[w];
    st_async_f32(&xred[1][rank], tid, v, &xbar[1]);
  }
  if (!mbar_wait(&xbar[1], 0)) atomicExch(a.err, kErrAttnExchange);
  float gsum = 0.f;
  for (int r = 0; r < C; ++r) gsum += xred[1][r];
  // p = bf16(e / sum), once per key (each thread divides the values it wrote)
  for (int j = j0 + tid; j < j1; j += kAttnThreads) sc[j - j0] = round_bf16(sc[j - j0] / gsum);
  __syncthreads();

  // ---- partial p.V
  float acc[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) acc[t] = 0.f;
  for (int base = j0; base < j1; base += kAttnGroups * kU) {
    const int jb = base + grp;
    uint4 vv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int j = jb + u * kAttnGroups;
      if (kPre == kAttnPreRegs && base == j0 && j < fresh)
        vv[u] = vpre[u];
      else if (kStage && j < js)
        vv[u] = *reinterpret_cast<const uint4*>(sv + (size_t)(j - j0) * kHeadDim + sub * 8);
      else
        vv[u] = j < j1 ? ld_stream(attn_row(a, a.v, slot, h, j) + sub * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int j = jb + u * kAttnGroups;
      const float p = j < j1 ? sc[j - j0] : 0.f;
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
  {
    // The 32 groups' partial outputs of dimension d: thread 4d + q adds groups
    // q, q + 4, ..., q + 28 in order, then the four sums meet in a butterfly,
    // (s0 + s1) + (s2 + s3), in the lanes of one warp.
    const int d = tid >> 2, q = tid & 3;
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < kAttnGroups / 4; ++i) o += part[(q + 4 * i) * kHeadDim + d];
    o += __shfl_xor_sync(0xffffffffu, o, 1);
    o += __shfl_xor_sync(0xffffffffu, o, 2);
    if (q == 0) {
      if (kAccOut) {  // every rank needs the head's output
        for (int r = 0; r < C; ++r) st_async_f32(&xo[rank][d], r, o, &xbar[2]);
      } else {
        st_async_f32(&xo[rank][d], 0, o, &xbar[2]);
      }
    }
  }
  if (gets_o && !mbar_wait(&xbar[2], 0)) atomicExch(a.err, kErrAttnExchange);
  // Everything sent to this CTA has landed.  Every CTA waits at its exit for
  // the whole cluster to get here, so no CTA leaves while a store into it
  // could still be on its way.
  cluster_arrive_relaxed();
  if constexpr (!kAccOut) {
    if (rank == 0 && tid < kHeadDim) {
      float o = 0.f;
      for (int r = 0; r < C; ++r) o += xo[r][tid];
      a.out[(size_t)m * a.ldo + h * kHeadDim + tid] = __float2bfloat16_rn(o);
    }
    // no copy may still be landing in this CTA's shared memory when it exits (bounded waits)
    if (kStage && !staged) mbar_wait(&bars[0], 0);
    if (fuse_q && !q_staged) mbar_wait(&bars[1], 0);
    cluster_wait();
  } else {
    if (tid < kHeadDim) {
      float o = 0.f;
      for (int r = 0; r < C; ++r) o += xo[r][tid];
      ohead[tid] = round_bf16(o);  // the attention output is bf16 (engine.py:292)
    }
    __syncthreads();
    float oh[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) oh[t] = ohead[sub * 8 + t];
    bool in_range = true;
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
      if (i < per && n < a.D && sub == 0) in_range &= acc_add(a.acc_out + (size_t)m * a.D + n, d);
    };
    // pass counts are uniform across the block: the shuffles need every lane
#pragma unroll
    for (int p = 0; p < kAttnOutPrefetch; ++p)
      if (p * kAttnGroups < per) emit(p, wpre[p]);
    for (int p = kAttnOutPrefetch; p * kAttnGroups < per; ++p) {
      const int i = p * kAttnGroups + grp, n = n0 + i;
      emit(p, (i < per && n < a.D) ? ld_stream(a.wo + (size_t)n * a.D + h * kHeadDim + sub * 8) : make_uint4(0, 0, 0, 0));
    }
    if (!in_range) atomicExch(a.err, kErrAccRange);
    // no copy may still be landing in this CTA's shared memory when it exits (bounded waits)
    if (kStage && !staged) mbar_wait(&bars[0], 0);
    if (fuse_q && !q_staged) mbar_wait(&bars[1], 0);
    cluster_wait();
  }
}

}  // namespace s2r
