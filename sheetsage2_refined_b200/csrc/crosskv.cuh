// Cross K/V projection of one window for every layer in one persistent launch
// (tcgen05 + TMA, sm_100a).
//
// A window's `load` projects the encoder memory X [F, D] through the cross
// key and value weights of every layer (decoder.py:98-116, engine.py:196-214):
// K_l = X Wk_l^T + bk_l, V_l = X Wv_l^T + bv_l, each rounded to bf16 and
// written straight into the slot's cross K/V [heads, frames_cap, 64].  With
// the L layers' [Wk; Wv] stacked into one [L * 2D, D] matrix this is a single
// dense GEMM of F x (L * 2D) x D: 75 GFLOP for 1,500 frames at d1024 x 12
// layers.
//
// Tiles are 128 frames (the MMA's M, one tensor-memory lane per frame) by 256
// output features (the MMA's N), K in 64-wide stages.  One CTA per SM walks
// the tiles persistently (tile = blockIdx.x + i * gridDim.x, frame tiles
// fastest so that CTAs running at the same time share weight tiles in L2):
//
//   warp 0, one lane: TMA producer, a 4-stage ring of (frames 128x64,
//                     weights 256x64) bf16 tiles with the 128-byte swizzle;
//   warp 1, one lane: issues tcgen05.mma (4 per stage) into one of two
//                     256-column fp32 accumulators in tensor memory and
//                     commits each stage back to the producer and each
//                     finished tile to the epilogue;
//   warps 2-5:        epilogue: tcgen05.ld 32 features of one frame per
//                     thread, + bias, bf16, four 16-byte stores per thread
//                     (32 features of one head are 64 contiguous bytes), then
//                     hand the accumulator back.  The two accumulators let the
//                     epilogue of one tile run under the MMAs of the next.
//
// Every mbarrier wait is bounded; on a timeout the thread records
// kErrGemmWait, the CTA stops, waits (bounded) for the copies and MMAs it
// issued, frees its tensor memory and returns.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "mbarrier.cuh"

namespace s2r {

constexpr int kCkvThreads = 192;  // producer warp, MMA warp, 4 epilogue warps
constexpr int kCkvBlockM = 128;   // frames per tile
constexpr int kCkvBlockN = 256;   // output features per tile
constexpr int kCkvBlockK = 64;    // K per stage: one 128-byte swizzle row of bf16
constexpr int kCkvStages = 4;     // ring depth of the production instantiation
constexpr int kCkvMaxLayers = 32;  // layers per launch (more are split over launches)
constexpr uint32_t kCkvBytesA = kCkvBlockM * kCkvBlockK * 2;  // 16 KB
constexpr uint32_t kCkvBytesB = kCkvBlockN * kCkvBlockK * 2;  // 32 KB
__host__ __device__ constexpr size_t ckv_smem_bytes(int stages) {
  return (size_t)stages * (kCkvBytesA + kCkvBytesB) + 1024;  // + slack for 1024-byte alignment
}

struct CrossKvArgs {
  int frames;      // rows of X: the window's frames
  int D;           // width = K, heads * 64
  int heads;
  int layers;      // layers of this launch (<= kCkvMaxLayers)
  int frames_cap;  // frames per slot in the cross K/V buffers
  int slot;
  int* err;
  const bf16* bias[kCkvMaxLayers];  // [2D]: key bias, then value bias
  bf16* k_dst[kCkvMaxLayers];       // [slots, heads, frames_cap, 64]
  bf16* v_dst[kCkvMaxLayers];
};

__device__ __forceinline__ void umma_bf16_n256(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t accumulate) {
  // kind::f16, f32 accumulator, A and B bf16 and K-major, N = 256, M = 128
  constexpr uint32_t idesc =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kCkvBlockN >> 3) << 17) | ((uint32_t)(kCkvBlockM >> 4) << 24);
  umma_bf16(tmem_d, a_desc, b_desc, idesc, accumulate);
}

template <int STAGES>
__global__ void __launch_bounds__(kCkvThreads, 1)
    crosskv_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                   const __grid_constant__ CrossKvArgs a) {
  extern __shared__ __align__(1024) unsigned char ckv_smem[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(ckv_smem) + 1023) & ~uintptr_t(1023));
  unsigned char* sa = base;                                // [stages][128 frames][128 B]
  unsigned char* sb = base + STAGES * kCkvBytesA;      // [stages][256 features][128 B]
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], done;
  __shared__ uint32_t tmem_base;
  __shared__ int aborted;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int features = a.layers * 2 * a.D;
  const int m_tiles = (a.frames + kCkvBlockM - 1) / kCkvBlockM;
  const int n_tiles = (features + kCkvBlockN - 1) / kCkvBlockN;
  const int tiles = m_tiles * n_tiles;
  const int k_tiles = (a.D + kCkvBlockK - 1) / kCkvBlockK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(&done, 1);
    aborted = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(2 * kCkvBlockN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_launch_dependents();
  pdl_wait();  // the memory rows and the cross K/V buffers belong to the work before this launch

  if (warp == 0) {
    if (lane == 0) {
      // ---- producer
      int it = 0, issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % m_tiles) * kCkvBlockM, n0 = (tile / m_tiles) * kCkvBlockN;
        for (int kt = 0; kt < k_tiles; ++kt, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1)) {
            atomicExch(a.err, kErrGemmWait);
            aborted = 1;
            ok = false;
            break;
          }
          if (*(volatile int*)&aborted) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], kCkvBytesA + kCkvBytesB);
          tma_load_2d(sa + s * kCkvBytesA, &map_x, kt * kCkvBlockK, m0, &full[s]);
          tma_load_2d(sb + s * kCkvBytesB, &map_w, kt * kCkvBlockK, n0, &full[s]);
          issued = it + 1;
        }
      }
      if (!ok)  // wait (bounded) for the copies still in flight before the CTA may exit
        for (int i = max(0, issued - STAGES); i < issued; ++i) mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1, use = local >> 1;
        if (use > 0 && !mbar_wait(&acc_empty[acc], (use - 1) & 1)) {
          atomicExch(a.err, kErrGemmWait);
          aborted = 1;
          break;
        }
        tmem_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * kCkvBlockN);
        for (int kt = 0; kt < k_tiles; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1) || *(volatile int*)&aborted) {
            atomicExch(a.err, kErrGemmWait);
            aborted = 1;
            ok = false;
            break;
          }
          tmem_fence_after();
          const uint64_t da = umma_desc_sw128(sa + s * kCkvBytesA);
          const uint64_t db = umma_desc_sw128(sb + s * kCkvBytesB);
#pragma unroll
          for (int k = 0; k < kCkvBlockK / 16; ++k)  // K = 16 per MMA: +32 bytes, +2 in the address field
            umma_bf16_n256(d, da + 2 * k, db + 2 * k, (kt > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[acc]);
      }
      umma_commit(&done);  // arrives once every MMA this thread issued has completed
    }
  } else {
    // ---- epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. +31 = frames of the tile
    const int g = warp & 3;
    const int D2 = 2 * a.D;
    int local = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1, use = local >> 1;
      const int m0 = (tile % m_tiles) * kCkvBlockM, n0 = (tile / m_tiles) * kCkvBlockN;
      // one decision for the whole warp: the tensor-memory loads below are warp-wide
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], use & 1) && !*(volatile int*)&aborted)) {
        if (lane == 0) atomicExch(a.err, kErrGemmWait);
        aborted = 1;
        break;
      }
      tmem_fence_after();
      const int frame = m0 + g * 32 + lane;
      const uint32_t taddr = tmem + ((uint32_t)(g * 32) << 16) + (uint32_t)(acc * kCkvBlockN);
#pragma unroll 1
      for (int c = 0; c < kCkvBlockN; c += 32) {
        const int f0 = n0 + c;  // 32 features: one half of one head of one layer (D is a multiple of 64)
        if (f0 >= features) break;
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        tmem_wait_ld();
        const int l = f0 / D2, c2 = f0 - l * D2;
        const int which = c2 >= a.D, cc = c2 - which * a.D;
        const uint4* bsrc = reinterpret_cast<const uint4*>(a.bias[l] + c2);
        if (frame < a.frames) {
          bf16* dst = (which ? a.v_dst[l] : a.k_dst[l]) +
                      (((size_t)a.slot * a.heads + (cc >> 6)) * a.frames_cap + frame) * kHeadDim + (cc & 63);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 b = __ldg(bsrc + q);
            const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float v0 = __uint_as_float(r[q * 8 + 2 * j]) + bf_lo(bw[j]);
              const float v1 = __uint_as_float(r[q * 8 + 2 * j + 1]) + bf_hi(bw[j]);
              o[j] = pack_bf16(v0, v1);
            }
            reinterpret_cast<uint4*>(dst)[q] = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
      }
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&done, 0);  // every MMA has completed before the tensor memory is freed
  __syncthreads();
  tmem_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kCkvBlockN)
                 : "memory");
}

}  // namespace s2r
