// Streaming projection kernel: y = x W^T + b for a handful of rows, weights
// read once from HBM at full width.
//
// One warp owns one output feature at a time and reads that feature's weight
// row with 16-byte loads (lane l holds columns c*256 + 8l .. 8l+7 of every
// 256-column chunk c), multiplies it against up to MC input rows staged in
// shared memory as bfloat16, and reduces across the warp.  The input rows are
// produced in the prologue, fused with what precedes the projection in the
// reference step (engine.py:298-314):
//   IN_EMBED  token + position embedding, then LayerNorm   (engine.py:298-302)
//   IN_LN     LayerNorm of the residual sum r              (decoder.py:78,81,84)
//   IN_BF16   bfloat16 rows (attention output, GELU hidden, encoder memory)
//   IN_F32    float32 rows rounded to bfloat16 (float32 encoder memory)
//   IN_ACC    LayerNorm of x + bf16(s + b), s the fixed-point out-projection sums
//             an attention launch accumulated (decoder.py:81-84 after the
//             attention, engine.py:312-313)
// and the epilogue applies what follows it:
//   EPI_QKV     q to a buffer, k/v appended to the paged self K/V cache (engine.py:310-311)
//   EPI_RESID   r = x + bf16(acc + b): the residual sum before the next LayerNorm
//   EPI_BF16    bf16(acc + b)
//   EPI_GELU    bf16(gelu(bf16(acc + b)))  (exact erf GELU on the bfloat16 value, decoder.py:83)
//   EPI_CROSSKV cross K/V of one slot's encoder frames (decoder.py:108-113)
//   EPI_SLICES  the fixed-point sum, over 32-column slices of K, of each
//               slice's float32 partial product (no bias): fc2 into the
//               accumulator the next LayerNorm reads (IN_ACC), so that the
//               fused FFN kernel, which adds the same slice partials with
//               integer atomics, gives the same bits
// Rounding follows the reference's CUDA autocast: the Linear input is the
// bfloat16 rounding of the float32 activation, accumulation is float32 and the
// output is rounded once after the bias is added.
#pragma once

#include "common.cuh"

namespace s2r {

enum InMode { IN_LN = 0, IN_EMBED = 1, IN_BF16 = 2, IN_F32 = 3, IN_ACC = 4 };

template <int IN>
__host__ __device__ constexpr bool ln_input() { return IN == IN_LN || IN == IN_EMBED || IN == IN_ACC; }
enum EpiMode { EPI_QKV = 0, EPI_RESID = 1, EPI_BF16 = 2, EPI_GELU = 3, EPI_CROSSKV = 4, EPI_SLICES = 5 };

constexpr int kSliceCols = 32;  // EPI_SLICES: columns of K per fixed-point partial (4 lanes x 8)

struct ProjArgs {
  int M, K, N;
  RowMap rm;
  SlotState st;
  // input
  const float* r;      // IN_LN: [M, K] residual sums; IN_ACC: [M, K] the residual input x
  const unsigned long long* acc;  // IN_ACC: [M, K] fixed-point out-projection sums (acc_add)
  const bf16* acc_bias;           // IN_ACC: [K] that projection's bias
  const float* gamma;  // IN_LN / IN_EMBED: LayerNorm weight [K]
  const float* beta;   //                   LayerNorm bias [K]
  const float* tok_emb;
  const float* pos_emb;
  const void* xin;  // IN_BF16 / IN_F32: [M, ldx]
  int ldx;
  float* x_out;  // IN_LN / IN_EMBED: the normalised float32 rows [M, K] (null: not kept)
  // weights [N, K] row-major and bias [N]
  const bf16* W;
  const bf16* bias;
  // epilogue
  bf16* out;
  int ldo;
  float* r_out;        // EPI_RESID [M, N]
  const float* x_res;  // EPI_RESID [M, N]
  bf16* k_dst;         // EPI_QKV: paged K pool; EPI_CROSSKV: cross K [batch, heads, frames_cap, 64]
  bf16* v_dst;
  int heads;
  int pages_per_slot;
  int frames_cap;
  int cross_slot;
  // words cleared after the wait: an accumulator whose reader has finished
  unsigned long long* zero;
  int zero_n;
  unsigned long long* acc_out;  // EPI_SLICES: [M, N]
  int* err;                     // device error word (a slice partial out of the fixed-point range)
  L2Ahead ahead;                // what the next kernel reads, prefetched into the L2 before the wait
};

// One 32-column slice partial of an EPI_SLICES row: the 8-product pieces of
// lanes 4t .. 4t+3 (columns 256c + 32t .. +31) added as (d0 + d1) + (d2 + d3);
// every lane of the group ends with the same value.
__device__ __forceinline__ float slice_partial(float d) {
  d += __shfl_xor_sync(0xffffffffu, d, 1);
  d += __shfl_xor_sync(0xffffffffu, d, 2);
  return d;
}

__device__ __forceinline__ float dot8(const uint4 w, const uint4 x) {
  float s = bf_lo(w.x) * bf_lo(x.x);
  s = fmaf(bf_hi(w.x), bf_hi(x.x), s);
  s = fmaf(bf_lo(w.y), bf_lo(x.y), s);
  s = fmaf(bf_hi(w.y), bf_hi(x.y), s);
  s = fmaf(bf_lo(w.z), bf_lo(x.z), s);
  s = fmaf(bf_hi(w.z), bf_hi(x.z), s);
  s = fmaf(bf_lo(w.w), bf_lo(x.w), s);
  s = fmaf(bf_hi(w.w), bf_hi(x.w), s);
  return s;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float gelu_erf(float x) { return x * 0.5f * (1.0f + erff(x * 0.70710678118654752440f)); }

// Epilogue of output (m, n) given v = accumulator + bias.
template <int EPI>
__device__ __forceinline__ void proj_epilogue_biased(const ProjArgs& a, int m, int n, float v) {
  if constexpr (EPI == EPI_RESID) {
    a.r_out[(size_t)m * a.N + n] = a.x_res[(size_t)m * a.N + n] + round_bf16(v);
  } else if constexpr (EPI == EPI_BF16) {
    a.out[(size_t)m * a.ldo + n] = __float2bfloat16_rn(v);
  } else if constexpr (EPI == EPI_GELU) {
    a.out[(size_t)m * a.ldo + n] = __float2bfloat16_rn(gelu_erf(round_bf16(v)));
  } else if constexpr (EPI == EPI_QKV) {
    const int D = a.heads * kHeadDim;
    if (n < D) {
      a.out[(size_t)m * a.ldo + n] = __float2bfloat16_rn(v);
    } else if (row_active(a.rm, a.st, m)) {
      const int c = n - D;
      const int which = c >= D;
      const int cc = which ? c - D : c;
      const int slot = row_slot(a.rm, m), pos = row_pos(a.rm, a.st, m);
      bf16* dst = which ? a.v_dst : a.k_dst;
      dst[paged_offset(a.st.page_table, a.pages_per_slot, a.heads, slot, cc / kHeadDim, pos) + (cc % kHeadDim)] =
          __float2bfloat16_rn(v);
    }
  } else {  // EPI_CROSSKV: row m is encoder frame m of slot cross_slot
    const int D = a.heads * kHeadDim;
    const int which = n >= D;
    const int c = which ? n - D : n;
    bf16* dst = which ? a.v_dst : a.k_dst;
    dst[(((size_t)a.cross_slot * a.heads + c / kHeadDim) * a.frames_cap + m) * kHeadDim + (c % kHeadDim)] =
        __float2bfloat16_rn(v);
  }
}

template <int EPI>
__device__ __forceinline__ void proj_epilogue(const ProjArgs& a, int m, int n, float acc) {
  proj_epilogue_biased<EPI>(a, m, n, acc + __bfloat162float(a.bias[n]));
}

// The 8 LayerNorm inputs at columns col .. col+7 (< K) of row m.
template <int IN>
__device__ __forceinline__ void ln_inputs8(const ProjArgs& a, int m, int col, float v[8]) {
  if constexpr (IN == IN_ACC) {
    const float* x = a.r + (size_t)m * a.K + col;
    const ulonglong2* sum = reinterpret_cast<const ulonglong2*>(a.acc + (size_t)m * a.K + col);
    const uint4 b = *reinterpret_cast<const uint4*>(a.acc_bias + col);
    const float4 x0 = *reinterpret_cast<const float4*>(x), x1 = *reinterpret_cast<const float4*>(x + 4);
    const ulonglong2 s0 = __ldcg(sum), s1 = __ldcg(sum + 1), s2 = __ldcg(sum + 2), s3 = __ldcg(sum + 3);
    // the out-projection is a bf16 Linear output (bias added, rounded once), then added to x
    v[0] = x0.x + round_bf16(acc_value(s0.x) + bf_lo(b.x));
    v[1] = x0.y + round_bf16(acc_value(s0.y) + bf_hi(b.x));
    v[2] = x0.z + round_bf16(acc_value(s1.x) + bf_lo(b.y));
    v[3] = x0.w + round_bf16(acc_value(s1.y) + bf_hi(b.y));
    v[4] = x1.x + round_bf16(acc_value(s2.x) + bf_lo(b.z));
    v[5] = x1.y + round_bf16(acc_value(s2.y) + bf_hi(b.z));
    v[6] = x1.z + round_bf16(acc_value(s3.x) + bf_lo(b.w));
    v[7] = x1.w + round_bf16(acc_value(s3.y) + bf_hi(b.w));
  } else {
    const float* src0 = IN == IN_EMBED ? a.tok_emb + (size_t)row_token(a.rm, a.st, m) * a.K : a.r + (size_t)m * a.K;
    float4 p0 = *reinterpret_cast<const float4*>(src0 + col);
    float4 p1 = *reinterpret_cast<const float4*>(src0 + col + 4);
    if constexpr (IN == IN_EMBED) {
      const float* src1 = a.pos_emb + (size_t)(row_pos(a.rm, a.st, m) + 2) * a.K;  // POSITION_OFFSET
      const float4 q0 = *reinterpret_cast<const float4*>(src1 + col);
      const float4 q1 = *reinterpret_cast<const float4*>(src1 + col + 4);
      p0.x += q0.x; p0.y += q0.y; p0.z += q0.z; p0.w += q0.w;
      p1.x += q1.x; p1.y += q1.y; p1.z += q1.z; p1.w += q1.w;
    }
    v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
    v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
  }
}

// LayerNorm statistics in one fixed order whatever the thread layout: the 8
// values of each column group g (columns 8g .. 8g+7) are summed in column
// order, lane l then adds the groups l, l + 32, l + 64, ... in that order, and
// the 32 lanes are added by warp_sum's butterfly; the variance takes the same
// order over (v - mean)^2.  Every LayerNorm of a step (projection prologues by
// a warp or a whole block, the attention prologue, the tensor-core pre-pass,
// the logits) uses it, so a row normalises to the same bits in a prefill chunk
// and in a decode step.
__device__ __forceinline__ float group_sum8(const float* v) {
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) s += v[j];
  return s;
}

__device__ __forceinline__ float group_sq8(const float* v, float mean) {
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float d = v[j] - mean;
    s = fmaf(d, d, s);
  }
  return s;
}

__device__ __forceinline__ float ln_apply(float v, float mean, float rstd, float g, float b) {
  return fmaf((v - mean) * rstd, g, b);
}

// Normalise rows [m0, m0+mc) into xs (bfloat16, KP columns per row, zero
// padded) and keep the float32 result in x_out.  One warp per row; each lane
// holds its 8*KCH columns (groups lane + 32c) in registers.
// sgamma / sbeta: the LayerNorm parameters already in shared memory (or null: read from a.gamma / a.beta).
template <int KCH, int IN>
__device__ __forceinline__ void stage_ln_rows(const ProjArgs& a, bf16* xs, int m0, int mc, int warp, int lane,
                                              int nwarps, bool own_rows = false, const float* sgamma = nullptr,
                                              const float* sbeta = nullptr) {
  const float* gam = sgamma ? sgamma : a.gamma;
  const float* bet = sbeta ? sbeta : a.beta;
  constexpr int KP = KCH * 256;
  const int K = a.K;
  for (int i = warp; i < mc; i += nwarps) {
    const int m = m0 + i;
    float v[KCH * 8];
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < KCH; ++c) {
      const int col = c * 256 + lane * 8;
      if (col < K) {
        ln_inputs8<IN>(a, m, col, v + c * 8);
        sum += group_sum8(v + c * 8);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[c * 8 + j] = 0.f;
      }
    }
    const float mean = warp_sum(sum) / (float)K;
    float sq = 0.f;
#pragma unroll
    for (int c = 0; c < KCH; ++c)
      if (c * 256 + lane * 8 < K) sq += group_sq8(v + c * 8, mean);
    const float rstd = rsqrtf(warp_sum(sq) / (float)K + kLnEps);
    // x_out is written once per row: by this CTA when it owns the rows it
    // stages, else by CTA m % gridDim.x (every CTA stages every row)
    const bool keep = a.x_out != nullptr && (own_rows || (m % gridDim.x) == blockIdx.x);
#pragma unroll
    for (int c = 0; c < KCH; ++c) {
      const int col = c * 256 + lane * 8;
      uint4 packed = make_uint4(0, 0, 0, 0);
      if (col < K) {
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = ln_apply(v[c * 8 + j], mean, rstd, gam[col + j], bet[col + j]);
        packed = make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
        if (keep) {
          float* dst = a.x_out + (size_t)m * K + col;
          *reinterpret_cast<float4*>(dst) = make_float4(y[0], y[1], y[2], y[3]);
          *reinterpret_cast<float4*>(dst + 4) = make_float4(y[4], y[5], y[6], y[7]);
        }
      }
      *reinterpret_cast<uint4*>(xs + (size_t)i * KP + col) = packed;
    }
  }
}

// Mean and 1/sqrt(var + eps) of one row whose column groups are spread over
// the NT threads of the block (thread t holds groups t + NT*c in v), in the
// fixed order above, returned to every thread.  red: shared memory for KCH*32
// floats; warps may still be reading it when the first returns, so a caller
// that calls again with the same `red` synchronises the block in between.
template <int KCH, int NT>
__device__ __forceinline__ float2 block_ln_stats(const float* v, int K, float* red) {
  constexpr int kG = (KCH * 32 + NT - 1) / NT;  // groups per thread
  const int t = threadIdx.x, lane = t & 31;
#pragma unroll
  for (int c = 0; c < kG; ++c) {
    const int g = t + NT * c;
    if (g < KCH * 32 && g * 8 < K) red[g] = group_sum8(v + c * 8);
  }
  __syncthreads();
  // every warp adds the group sums itself, in the same order: the same mean in
  // each, with no second barrier to broadcast it
  float mean;
  {
    float p = 0.f;
#pragma unroll
    for (int c = 0; c < KCH; ++c)
      if ((lane + 32 * c) * 8 < K) p += red[lane + 32 * c];
    mean = warp_sum(p) / (float)K;
  }
  __syncthreads();  // every warp has read the sums before they are overwritten
#pragma unroll
  for (int c = 0; c < kG; ++c) {
    const int g = t + NT * c;
    if (g < KCH * 32 && g * 8 < K) red[g] = group_sq8(v + c * 8, mean);
  }
  __syncthreads();
  float p = 0.f;
#pragma unroll
  for (int c = 0; c < KCH; ++c)
    if ((lane + 32 * c) * 8 < K) p += red[lane + 32 * c];
  p = warp_sum(p);
  return make_float2(mean, rsqrtf(p / (float)K + kLnEps));
}

// One LayerNorm'd row (IN_LN, IN_EMBED or IN_ACC) staged by all NT threads of
// the CTA (8 columns per thread and pass), for launches of a single row: the
// whole block shares the row's loads instead of one warp.  `keep`: this CTA
// writes the float32 row to x_out.
template <int KCH, int IN, int NT = 128>
__device__ __forceinline__ void stage_ln_row_block(const ProjArgs& a, bf16* xs, int m, const float* gam,
                                                   const float* bet, bool keep) {
  constexpr int kG = (KCH * 32 + NT - 1) / NT;  // 8-column groups per thread
  __shared__ float ln_red[KCH * 32 + 2];
  const int K = a.K, t = threadIdx.x;
  float v[kG * 8];
#pragma unroll
  for (int c = 0; c < kG; ++c) {
    const int col = (t + NT * c) * 8;
    if (col < K) {
      ln_inputs8<IN>(a, m, col, v + c * 8);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[c * 8 + j] = 0.f;
    }
  }
  const float2 st = block_ln_stats<KCH, NT>(v, K, ln_red);
  keep = keep && a.x_out != nullptr;
#pragma unroll
  for (int c = 0; c < kG; ++c) {
    const int col = (t + NT * c) * 8;
    if (col < KCH * 256) {
      uint4 packed = make_uint4(0, 0, 0, 0);
      if (col < K) {
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = ln_apply(v[c * 8 + j], st.x, st.y, gam[col + j], bet[col + j]);
        packed = make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
        if (keep) {
          float* dst = a.x_out + (size_t)m * K + col;
          *reinterpret_cast<float4*>(dst) = make_float4(y[0], y[1], y[2], y[3]);
          *reinterpret_cast<float4*>(dst + 4) = make_float4(y[4], y[5], y[6], y[7]);
        }
      }
      *reinterpret_cast<uint4*>(xs + col) = packed;
    }
  }
}

// Threads per CTA of proj_kernel: 8 warps for single-row launches (the row's
// staging is shared by twice as many output rows), else 4.
template <int MC>
__host__ __device__ constexpr int proj_threads() {
  return MC == 1 ? 256 : 128;
}

template <int KCH, int MC, int IN, int EPI>
__global__ void __launch_bounds__(proj_threads<MC>()) proj_kernel(const ProjArgs a) {
  constexpr int NT = proj_threads<MC>();
  constexpr int kWarps = NT / 32;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int KP = KCH * 256;
  constexpr bool kLn = ln_input<IN>();
  bf16* xs = reinterpret_cast<bf16*>(smem_raw);  // [MC][KP]
  float* sgamma = reinterpret_cast<float*>(smem_raw + (size_t)MC * KP * sizeof(bf16));  // [KP] (LayerNorm inputs)
  float* sbeta = sgamma + KP;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int K = a.K;
  const int stride = gridDim.x * kWarps;
  const int first = blockIdx.x * kWarps + warp;

  // The weights do not depend on earlier kernels: start streaming this warp's
  // first row before waiting for them.
  uint4 w[KCH];
#pragma unroll
  for (int c = 0; c < KCH; ++c) {
    const int col = c * 256 + lane * 8;
    w[c] = (first < a.N && col < K) ? ld_stream(a.W + (size_t)first * K + col) : make_uint4(0, 0, 0, 0);
  }
  // ... and so do the LayerNorm parameters and the bias of that row
  if constexpr (kLn) {
    for (int i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
      *reinterpret_cast<float4*>(sgamma + i) = *reinterpret_cast<const float4*>(a.gamma + i);
      *reinterpret_cast<float4*>(sbeta + i) = *reinterpret_cast<const float4*>(a.beta + i);
    }
  }
  const float bias_first = (EPI != EPI_SLICES && first < a.N) ? __bfloat162float(a.bias[first]) : 0.f;
  if (threadIdx.x == 0) l2_ahead(a.ahead, blockIdx.x, gridDim.x);
  pdl_launch_dependents();
  pdl_wait();
  if (a.zero) {  // the launch before this one has read the accumulator
    for (int i = blockIdx.x * NT + threadIdx.x; i < a.zero_n; i += gridDim.x * NT) a.zero[i] = 0ull;
  }
  // the residual input of this warp's first row, requested before the staging
  float xres_first = 0.f;
  if constexpr (EPI == EPI_RESID) {
    if (lane < min(MC, a.M) && first < a.N) xres_first = a.x_res[(size_t)lane * a.N + first];
  }
  if constexpr (kLn) __syncthreads();  // the LayerNorm parameters are in shared memory

  for (int m0 = 0; m0 < a.M; m0 += MC) {
    const int mc = min(MC, a.M - m0);
    if (m0 > 0) __syncthreads();
    if constexpr (kLn && MC == 1) {
      stage_ln_row_block<KCH, IN, NT>(a, xs, m0, sgamma, sbeta, (m0 % gridDim.x) == blockIdx.x);
    } else if constexpr (kLn) {
      stage_ln_rows<KCH, IN>(a, xs, m0, mc, warp, lane, 4, false, sgamma, sbeta);
    } else {
      if constexpr (IN == IN_BF16 && MC == 1) {
        // one bf16 row: every piece of this thread requested before the first is stored
        constexpr int kIt = (KP / 8 + NT - 1) / NT;
        uint4 got[kIt];
#pragma unroll
        for (int t = 0; t < kIt; ++t) {
          const int col = (threadIdx.x + NT * t) * 8;
          got[t] = col < K ? *reinterpret_cast<const uint4*>(static_cast<const bf16*>(a.xin) + (size_t)m0 * a.ldx + col)
                           : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int t = 0; t < kIt; ++t) {
          const int col = (threadIdx.x + NT * t) * 8;
          if (col < KP) *reinterpret_cast<uint4*>(xs + col) = got[t];
        }
      }
      for (int idx = threadIdx.x; !(IN == IN_BF16 && MC == 1) && idx < MC * (KP / 8); idx += blockDim.x) {
        const int i = idx / (KP / 8), col = (idx % (KP / 8)) * 8;
        uint4 packed = make_uint4(0, 0, 0, 0);
        if (i < mc && col < K) {
          if constexpr (IN == IN_BF16) {
            packed = *reinterpret_cast<const uint4*>(static_cast<const bf16*>(a.xin) + (size_t)(m0 + i) * a.ldx + col);
          } else {
            const float* s = static_cast<const float*>(a.xin) + (size_t)(m0 + i) * a.ldx + col;
            float4 p0 = *reinterpret_cast<const float4*>(s), p1 = *reinterpret_cast<const float4*>(s + 4);
            packed = make_uint4(pack_bf16(p0.x, p0.y), pack_bf16(p0.z, p0.w), pack_bf16(p1.x, p1.y), pack_bf16(p1.z, p1.w));
          }
        }
        *reinterpret_cast<uint4*>(xs + (size_t)i * KP + col) = packed;
      }
    }
    if constexpr (kLn) {
      // rows mc..MC-1 of the last chunk are not staged: zero them
      for (int idx = threadIdx.x; idx < (MC - mc) * (KP / 8); idx += blockDim.x) {
        const int i = mc + idx / (KP / 8), col = (idx % (KP / 8)) * 8;
        *reinterpret_cast<uint4*>(xs + (size_t)i * KP + col) = make_uint4(0, 0, 0, 0);
      }
    }
    __syncthreads();

    for (int n = first; n < a.N; n += stride) {
      if (n != first || m0 > 0) {
#pragma unroll
        for (int c = 0; c < KCH; ++c) {
          const int col = c * 256 + lane * 8;
          w[c] = col < K ? ld_stream(a.W + (size_t)n * K + col) : make_uint4(0, 0, 0, 0);
        }
      }
      if constexpr (EPI == EPI_SLICES) {
        // per 32-column slice: partial product, rounded to fixed point, summed as integers
        long long isum[MC];
        bool ok = true;
#pragma unroll
        for (int i = 0; i < MC; ++i) isum[i] = 0;
#pragma unroll
        for (int c = 0; c < KCH; ++c) {
#pragma unroll
          for (int i = 0; i < MC; ++i) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + (size_t)i * KP + c * 256 + lane * 8);
            const float p = slice_partial(dot8(w[c], xv));
            ok &= fabsf(p) < kAccLimit;
            isum[i] += __float2ll_rn(p * kAccScale);
          }
        }
#pragma unroll
        for (int i = 0; i < MC; ++i) {
          // the 4 lanes of a slice group hold the same sum: add one lane per group
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) isum[i] += __shfl_xor_sync(0xffffffffu, isum[i], o);
          if (lane == i && i < mc) a.acc_out[(size_t)(m0 + i) * a.N + n] = (unsigned long long)isum[i];
        }
        if (__any_sync(0xffffffffu, !ok) && lane == 0 && a.err) atomicExch(a.err, kErrAccRange);
        continue;
      }
      float acc[MC];
#pragma unroll
      for (int i = 0; i < MC; ++i) acc[i] = 0.f;
#pragma unroll
      for (int c = 0; c < KCH; ++c) {
#pragma unroll
        for (int i = 0; i < MC; ++i) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xs + (size_t)i * KP + c * 256 + lane * 8);
          acc[i] += dot8(w[c], xv);
        }
      }
#pragma unroll
      for (int i = 0; i < MC; ++i) {
        acc[i] = warp_sum(acc[i]);
        if (lane == i && i < mc) {
          const float v = acc[i] + (n == first ? bias_first : __bfloat162float(a.bias[n]));
          if constexpr (EPI == EPI_RESID) {
            const size_t o = (size_t)(m0 + i) * a.N + n;
            a.r_out[o] = (n == first && m0 == 0 ? xres_first : a.x_res[o]) + round_bf16(v);
          } else {
            proj_epilogue_biased<EPI>(a, m0 + i, n, v);
          }
        }
      }
    }
  }
}

}  // namespace s2r
