// Fused FFN of one decode row: cross_attn_norm, fc1 + GELU and fc2 in one launch.
//
// Replaces the reference's `layer.cross_attn_norm(x + cross)` and
// `fc2(gelu(fc1(x)))` (decoder.py:81-84, engine.py:313-314) for engines with a
// single slot, whose step would otherwise spend two launches and a round trip
// of the 4,096-wide hidden vector through memory on it.  CTA s owns the 32
// hidden units [32s, 32s + 32):
//   1. (before the PDL wait) its 32 rows of W1, its fc1 bias and its slice of
//      W2 (stored slice-major, w2s[s][n][0..31] = W2[n][32s .. 32s + 31]) are
//      bulk-copied into shared memory, with the LayerNorm parameters and the
//      cross out-projection bias;
//   2. the input row LayerNorm(x + bf16(acc_in + bias_in)) in the fixed order
//      every LayerNorm of the step uses (CTA 0 keeps the float32 row, the
//      residual of the FFN);
//   3. its 32 hidden units with the projection kernel's fc1 arithmetic
//      (16-byte pieces in order, warp butterfly, + bias, bf16, exact GELU, bf16);
//   4. for every output feature n, the slice's partial product with the
//      projection kernel's EPI_SLICES arithmetic, added to acc_out[n] as a
//      fixed-point sum (acc_add).
// The projection kernels' fc1 + fc2 (EPI_SLICES) produce the same bits: the
// prefill of a prefix and the decode of the same tokens agree exactly.
#pragma once

#include "common.cuh"
#include "mbarrier.cuh"
#include "proj.cuh"

namespace s2r {

constexpr int kFfnThreads = 256;
constexpr int kFfnSlice = kSliceCols;  // hidden units per CTA (32)
constexpr int kErrFfnStage = 9;        // a bulk copy of the fused FFN did not complete in time

struct FfnArgs {
  int D, FFN;
  int m;  // the row (slot) this launch serves
  // input row: LayerNorm(x_in + bf16(acc_in + bias_in)), kept in x_out by CTA 0
  const float* x_in;                 // [rows][D]
  const unsigned long long* acc_in;  // [rows][D]
  const bf16* bias_in;               // [D]
  const float *ln_g, *ln_b;          // [D]
  float* x_out;                      // [rows][D]
  const bf16* w1;                    // [FFN][D]
  const bf16* b1;                    // [FFN]
  const bf16* w2s;                   // [FFN/32][D][32]
  unsigned long long* acc_out;       // [rows][D]
  unsigned long long* zero;          // cleared after the wait (an accumulator already read)
  int zero_n;
  int* err;
  L2Ahead ahead;  // what the next kernel reads, prefetched into the L2 before the wait
};

// Dynamic shared memory: W1 rows [32][D], W2 slice [D][32] (bf16), LayerNorm
// weight and bias [D] (f32), input bias [D] and the normalised row [KP] (bf16).
__host__ __device__ constexpr size_t ffn_smem_bytes(int D) {
  return (size_t)kFfnSlice * D * 2 * 2 + (size_t)D * 4 * 2 + (size_t)D * 2 + (size_t)((D + 255) / 256 * 256) * 2;
}

template <int KCH>
__global__ void __launch_bounds__(kFfnThreads) ffn_row_kernel(const FfnArgs a) {
  extern __shared__ __align__(16) unsigned char ffn_smem[];
  constexpr int KP = KCH * 256;
  const int D = a.D, s = blockIdx.x;
  bf16* sw1 = reinterpret_cast<bf16*>(ffn_smem);                      // [32][D]
  bf16* sw2 = sw1 + (size_t)kFfnSlice * D;                            // [D][32]
  float* sg = reinterpret_cast<float*>(sw2 + (size_t)kFfnSlice * D);  // [D]
  float* sb = sg + D;                                                 // [D]
  bf16* sbi = reinterpret_cast<bf16*>(sb + D);                        // [D]
  bf16* sx = sbi + D;                                                 // [KP]
  __shared__ __align__(16) bf16 sh[kFfnSlice];  // the slice's hidden units
  __shared__ float ln_red[KCH * 32 + 2];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (tid == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const unsigned w_bytes = (unsigned)(kFfnSlice * D * 2);
    mbar_expect_tx(&bar, 2 * w_bytes + (unsigned)D * 10);
    bulk_load(sw1, a.w1 + (size_t)s * kFfnSlice * D, w_bytes, &bar);
    bulk_load(sw2, a.w2s + (size_t)s * D * kFfnSlice, w_bytes, &bar);
    bulk_load(sg, a.ln_g, (unsigned)D * 4, &bar);
    bulk_load(sb, a.ln_b, (unsigned)D * 4, &bar);
    bulk_load(sbi, a.bias_in, (unsigned)D * 2, &bar);
  }
  // fc1 bias of this warp's 4 hidden units (lane j < 4 holds unit 4 * warp + j)
  const float b1 = lane < 4 ? __bfloat162float(a.b1[s * kFfnSlice + warp * 4 + lane]) : 0.f;
  if (tid == 0) l2_ahead(a.ahead, blockIdx.x, gridDim.x);
  __syncthreads();  // the barrier is initialised
  pdl_launch_dependents();
  pdl_wait();
  if (a.zero) {
    for (int i = blockIdx.x * kFfnThreads + tid; i < a.zero_n; i += gridDim.x * kFfnThreads) a.zero[i] = 0ull;
  }

  // ---- the input row
  ProjArgs pa{};
  pa.K = D;
  pa.r = a.x_in;
  pa.acc = a.acc_in;
  pa.acc_bias = sbi;
  float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const int col = tid * 8;
  const bool staged = mbar_wait(&bar, 0);
  if (!staged && tid == 0) atomicExch(a.err, kErrFfnStage);
  if (col < D) ln_inputs8<IN_ACC>(pa, a.m, col, v);
  const float2 st = block_ln_stats<KCH, kFfnThreads>(v, D, ln_red);
  if (col < KP) {
    uint4 packed = make_uint4(0, 0, 0, 0);
    if (col < D) {
      float y[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = ln_apply(v[j], st.x, st.y, sg[col + j], sb[col + j]);
      packed = make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
      if (blockIdx.x == 0) {
        float* dst = a.x_out + (size_t)a.m * D + col;
        *reinterpret_cast<float4*>(dst) = make_float4(y[0], y[1], y[2], y[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(y[4], y[5], y[6], y[7]);
      }
    }
    *reinterpret_cast<uint4*>(sx + col) = packed;
  }
  __syncthreads();

  // ---- fc1 + GELU: 4 hidden units per warp, each in the projection kernel's order (16-byte
  // pieces in order, then the butterfly); the four units' chains interleaved, and lane u
  // applies unit u's bias and GELU
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < KCH; ++c) {
    const int cc = c * 256 + lane * 8;
    const uint4 xv = *reinterpret_cast<const uint4*>(sx + cc);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const bf16* wrow = sw1 + (size_t)(warp * 4 + u) * D;
      const uint4 w = cc < D ? *reinterpret_cast<const uint4*>(wrow + cc) : make_uint4(0, 0, 0, 0);
      acc[u] += dot8(w, xv);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);
  }
  if (lane < 4) {
    const float mine = lane == 0 ? acc[0] : lane == 1 ? acc[1] : lane == 2 ? acc[2] : acc[3];
    sh[warp * 4 + lane] = __float2bfloat16_rn(gelu_erf(round_bf16(mine + b1)));
  }
  __syncthreads();

  // ---- fc2 slice partials: 4 lanes (8 hidden units each) per output feature
  const int q = lane & 3, grp = tid >> 2;  // 64 groups
  const uint4 hx = *reinterpret_cast<const uint4*>(sh + q * 8);
  bool in_range = true;
  for (int n = grp; n < D; n += kFfnThreads / 4) {
    const uint4 w = *reinterpret_cast<const uint4*>(sw2 + (size_t)n * kFfnSlice + q * 8);
    const float p = slice_partial(dot8(w, hx));
    if (q == 0) in_range &= acc_add(a.acc_out + (size_t)a.m * D + n, p);
  }
  if (!in_range) atomicExch(a.err, kErrAccRange);
  if (!staged) mbar_wait(&bar, 0);  // no copy may still be landing when the CTA exits
}

}  // namespace s2r
