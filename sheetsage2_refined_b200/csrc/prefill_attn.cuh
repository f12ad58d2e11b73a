// Causal prefill attention on tensor cores (tcgen05 + TMA, sm_100a).
//
// A window's prefix is prefilled in chunks of up to 128 consecutive positions
// of one slot (engine.py:199-205 runs the decoder over the whole prefix at
// once: decoder.py:118-151, scaled_dot_product_attention with is_causal).
// Every row of a chunk attends to the same keys, so one CTA takes all 128
// rows of one head and streams the keys through shared memory once:
//
//   S = Q K^T          tcgen05.mma M128 (rows) N64 (keys) K64, fp32 in tensor memory
//   online softmax     one thread per row, as the reference's flash prefill:
//                      s * 1/8 in fp32, running max m and sum l in fp32,
//                      p = bf16(exp(s - m)), l += sum of the fp32 values
//   O += P V           tcgen05.mma M128 (rows) N64 (dims) K64 (keys), P and V^T
//                      written into shared memory by the softmax threads;
//                      O = O * exp(m_old - m_new) + PV kept in registers
//   out = bf16(O / l)
//
// self (causal): row i (position pos0 + i) sees keys 0 .. pos0 + i of the
//   slot's paged pool, 64-token pages: one page per key tile;
// cross: every row sees the slot's first `frames` encoder frames.
//
// The key tiles of a (chunk, head) are split over a cluster of S CTAs (S <= 8);
// each keeps (m, l, O) per row, and after a cluster barrier CTA r combines
// the rows i = r (mod S) from all S partials through distributed shared memory:
// M = max m_s, out = sum_s O_s exp(m_s - M) / sum_s l_s exp(m_s - M).
//
// Warp roles (192 threads): warp 0 lane 0 loads Q once and the (K, V) tiles
// into a 4-stage ring (TMA); warp 1 lane 0 issues the MMAs; warps 2-5 (one
// thread per row: tensor-memory lane = row) run the softmax, write P and the
// transposed V tile (128-byte swizzle, the layout the MMA descriptors read),
// and accumulate O.  S and PV are double-buffered in tensor memory so that
// the MMAs of one tile run under the softmax of the next.
//
// Every mbarrier wait is bounded; on a timeout the CTA records kErrPrefillWait,
// stops, still takes part in every cluster barrier, waits (bounded) for its
// copies and MMAs, frees its tensor memory and returns.
#pragma once

#include <cooperative_groups.h>
#include <cuda.h>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "mbarrier.cuh"

namespace s2r {

constexpr int kPfThreads = 192;
constexpr int kPfRows = 128;         // query rows per CTA (the MMA's M)
constexpr int kPfKeys = 64;          // keys per tile (one page of the self-attention pool)
constexpr int kPfStages = 4;         // (K, V) tiles in flight
constexpr int kPfMaxSplits = 8;      // CTAs per (chunk, head)
constexpr int kErrPrefillWait = 10;  // a wait of the prefill attention timed out
constexpr uint32_t kPfTileBytes = kPfKeys * kHeadDim * 2;  // 8 KB: 64 rows of 128 bytes
constexpr uint32_t kPfQBytes = kPfRows * kHeadDim * 2;     // 16 KB

// Dynamic shared memory: Q, the (K, V) ring, P x2, V^T x2 (all 1024-byte aligned).
struct PfSmem {
  static constexpr size_t q = 0;
  static constexpr size_t ring = q + kPfQBytes;
  static constexpr size_t p = ring + (size_t)kPfStages * 2 * kPfTileBytes;
  static constexpr size_t vt = p + 2 * (size_t)kPfQBytes;
  static constexpr size_t total = vt + 2 * (size_t)kPfTileBytes + 1024;  // + alignment slack
};
// after the loop the ring holds this rank's partial (m, l, O) for the combine
constexpr int kPfOStride = kHeadDim + 4;  // floats per row of the partial O (padded against bank conflicts)
static_assert((size_t)kPfRows * (kPfOStride + 2) * 4 <= (size_t)kPfStages * 2 * kPfTileBytes, "partials fit the ring");

struct PrefillAttnArgs {
  int rows;   // rows of the chunk (<= 128): positions pos0 .. pos0 + rows - 1 of slot `slot`
  int pos0;
  int slot;
  int cross;  // 0: causal self-attention over the paged pool; 1: cross-attention over `frames`
  int H;
  int D;
  int pages_per_slot;
  int frames_cap;
  int tiles;  // key tiles of the chunk's longest row
  int per;    // key tiles per CTA of the cluster
  const int32_t* page_table;  // [batch, pages_per_slot]
  const int32_t* frames;      // [batch] real frames
  bf16* out;                  // [rows, D] (row stride D)
  int* err;
};

// Offset of the 16-byte piece `c` (0..7) of row `r` in a tile of 128-byte rows
// laid out with the 128-byte swizzle (tile base 1024-byte aligned).
__device__ __forceinline__ uint32_t sw128_off(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// Generic-proxy writes to shared memory made visible to the tensor core's reads.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int kUnused>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const __grid_constant__ PrefillAttnArgs a) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(1024) unsigned char pf_smem[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(pf_smem) + 1023) & ~uintptr_t(1023));
  unsigned char* sq = base + PfSmem::q;
  unsigned char* ring = base + PfSmem::ring;  // stage s: K at 2s, V at 2s + 1 (8 KB each)
  unsigned char* sp = base + PfSmem::p;       // P of tile parity b at b * 16 KB: [128 rows][64 keys]
  unsigned char* svt = base + PfSmem::vt;     // V^T of tile parity b at b * 8 KB: [64 dims][64 keys]
  __shared__ __align__(8) uint64_t q_full, full[kPfStages], empty[kPfStages], s_full[2], s_empty[2], p_full[2],
      pv_full[2], pv_empty[2], done;
  __shared__ uint32_t tmem_base;
  __shared__ int aborted;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = (int)gridDim.x, rank = (int)blockIdx.x, h = (int)blockIdx.y;
  const int t0 = min(a.tiles, rank * a.per), t1 = min(a.tiles, t0 + a.per);
  const int nt = t1 - t0;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);  // one arrival per softmax warp
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);
      mbar_init(&p_full[b], 4);
      mbar_init(&pv_full[b], 1);
      mbar_init(&pv_empty[b], 4);
    }
    mbar_init(&done, 1);
    aborted = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {  // S: columns [0, 128) (two 64-column buffers); PV: [128, 256)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_launch_dependents();
  pdl_wait();  // queries and this chunk's keys come from the kernels before

  auto fail = [&]() {
    atomicExch(a.err, kErrPrefillWait);
    aborted = 1;
  };
  auto key_row = [&](int t) -> int {  // first row of key tile t in the K/V tensor maps
    if (a.cross) return (a.slot * a.H + h) * a.frames_cap + t * kPfKeys;
    const int page = a.page_table[(size_t)a.slot * a.pages_per_slot + t];
    return (page * a.H + h) * kPfKeys;
  };

  if (warp == 0) {
    if (lane == 0 && nt > 0) {
      // ---- producer: Q once, then the (K, V) tiles of this CTA's range
      int issued = 0;
      mbar_expect_tx(&q_full, kPfQBytes);
      tma_load_2d(sq, &map_q, h * kHeadDim, 0, &q_full);
      for (int i = 0; i < nt; ++i) {
        const int s = i % kPfStages;
        if (i >= kPfStages && !mbar_wait(&empty[s], ((i / kPfStages) - 1) & 1)) {
          fail();
          break;
        }
        if (*(volatile int*)&aborted) break;
        const int row = key_row(t0 + i);
        mbar_expect_tx(&full[s], 2 * kPfTileBytes);
        tma_load_2d(ring + (2 * s) * kPfTileBytes, &map_k, 0, row, &full[s]);
        tma_load_2d(ring + (2 * s + 1) * kPfTileBytes, &map_v, 0, row, &full[s]);
        issued = i + 1;
      }
      // every copy has landed before the CTA may exit or reuse the ring (bounded)
      mbar_wait(&q_full, 0);
      for (int i = max(0, issued - kPfStages); i < issued; ++i) mbar_wait(&full[i % kPfStages], (i / kPfStages) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: S_t = Q K_t^T, then PV_{t-1} = P_{t-1} V_{t-1}
      const uint32_t idesc = umma_idesc_bf16(kPfKeys);  // M 128, N 64, bf16 in, fp32 out, both K-major
      bool ok = nt == 0 || mbar_wait(&q_full, 0);
      if (!ok) fail();
      auto issue_pv = [&](int u) -> bool {
        const int b = u & 1;
        if (!mbar_wait(&p_full[b], (u >> 1) & 1)) return false;
        if (u >= 2 && !mbar_wait(&pv_empty[b], ((u >> 1) - 1) & 1)) return false;
        if (*(volatile int*)&aborted) return false;
        tmem_fence_after();
        const uint64_t da = umma_desc_sw128(sp + b * kPfQBytes);
        const uint64_t db = umma_desc_sw128(svt + b * kPfTileBytes);
#pragma unroll
        for (int k = 0; k < kPfKeys / 16; ++k)
          umma_bf16(tmem + 128 + b * 64, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
        umma_commit(&pv_full[b]);
        return true;
      };
      for (int t = 0; t < nt && ok; ++t) {
        const int s = t % kPfStages, b = t & 1;
        if (!mbar_wait(&full[s], (t / kPfStages) & 1) || (t >= 2 && !mbar_wait(&s_empty[b], ((t >> 1) - 1) & 1)) ||
            *(volatile int*)&aborted) {
          fail();
          ok = false;
          break;
        }
        tmem_fence_after();
        const uint64_t da = umma_desc_sw128(sq);
        const uint64_t db = umma_desc_sw128(ring + (2 * s) * kPfTileBytes);
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) umma_bf16(tmem + b * 64, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
        umma_commit(&s_full[b]);
        if (t >= 1 && !issue_pv(t - 1)) {
          fail();
          ok = false;
        }
      }
      if (ok && nt > 0 && !issue_pv(nt - 1)) fail();
      umma_commit(&done);  // arrives once every MMA issued has completed
    }
  }

  // ---- softmax warps: thread = row i (tensor-memory lane)
  const bool sm_warp = warp >= 2;
  const int i = (warp & 3) * 32 + lane;
  const int limit = a.cross ? a.frames[a.slot] : a.pos0 + i + 1;  // keys [0, limit) visible to row i
  float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
  float o[kHeadDim];
#pragma unroll
  for (int d = 0; d < kHeadDim; ++d) o[d] = 0.f;
  if (sm_warp) {
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    auto consume_pv = [&](int u, float alpha) -> bool {  // O = O * alpha + PV_u
      const int b = u & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&pv_full[b], (u >> 1) & 1) && !*(volatile int*)&aborted)) return false;
      tmem_fence_after();
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + 128 + b * 64 + half * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) o[half * 32 + j] = fmaf(o[half * 32 + j], alpha, __uint_as_float(r[j]));
      }
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pv_empty[b]);
      return true;
    };
    bool ok = true;
    for (int t = 0; t < nt; ++t) {
      const int s = t % kPfStages, b = t & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (t >> 1) & 1) && !*(volatile int*)&aborted)) {
        ok = false;
        break;
      }
      tmem_fence_after();
      float sc[kPfKeys];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + b * 64 + half * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) sc[half * 32 + j] = __uint_as_float(r[j]);
      }
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[b]);
      // scale, mask, running max
      const int j0 = (t0 + t) * kPfKeys;
      float tmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < kPfKeys; ++j) {
        sc[j] = j0 + j < limit ? sc[j] * 0.125f : -INFINITY;  // head_dim ** -0.5 for head_dim 64
        tmax = fmaxf(tmax, sc[j]);
      }
      const float m_new = fmaxf(m, tmax);
      const float alpha = m_new == -INFINITY ? 1.f : __expf(m - m_new);
      float rowsum = 0.f;
      uint32_t pk[kPfKeys / 2];
#pragma unroll
      for (int j = 0; j < kPfKeys; j += 2) {
        const float p0 = sc[j] == -INFINITY ? 0.f : __expf(sc[j] - m_new);
        const float p1 = sc[j + 1] == -INFINITY ? 0.f : __expf(sc[j + 1] - m_new);
        rowsum += p0 + p1;
        pk[j / 2] = pack_bf16(p0, p1);
      }
      l = l * alpha + rowsum;
      m = m_new;
      // P row i into the swizzled tile (the PV MMA's A operand); tile t-2's PV, which read this
      // buffer, was consumed in the previous iteration
      unsigned char* prow = sp + b * kPfQBytes;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + sw128_off(i, c)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      // V_t transposed into V^T [dims][keys] (the PV MMA's B operand): 512 pieces of 8 keys
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (t / kPfStages) & 1))) {
        ok = false;
        break;
      }
      const unsigned char* vsrc = ring + (2 * s + 1) * kPfTileBytes;
      unsigned char* vdst = svt + b * kPfTileBytes;
      const int tid = threadIdx.x - 64;
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int item = tid + 128 * it, d = item & 63, kc = item >> 6;
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k0 = kc * 8 + 2 * e;
          const bf16 lo = *reinterpret_cast<const bf16*>(vsrc + sw128_off(k0, d >> 3) + (d & 7) * 2);
          const bf16 hi = *reinterpret_cast<const bf16*>(vsrc + sw128_off(k0 + 1, d >> 3) + (d & 7) * 2);
          w[e] = (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
        }
        *reinterpret_cast<uint4*>(vdst + sw128_off(d, kc)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_async_smem();  // the generic-proxy writes of P and V^T, visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[s]);  // K_t (read by S_t, complete) and V_t (copied) are free
        mbar_arrive(&p_full[b]);
      }
      if (t >= 1 && !consume_pv(t - 1, alpha_prev)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok && nt > 0 && !consume_pv(nt - 1, alpha_prev)) ok = false;
    if (!ok && lane == 0) fail();
  }

  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&done, 0);  // every MMA has completed
  __syncthreads();
  tmem_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");

  const bool good = !*(volatile int*)&aborted;
  if (S == 1) {
    if (sm_warp && good && i < a.rows) {
      const float inv = 1.f / l;
      bf16* dst = a.out + (size_t)i * a.D + h * kHeadDim;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = pack_bf16(o[c * 8 + 2 * e] * inv, o[c * 8 + 2 * e + 1] * inv);
        reinterpret_cast<uint4*>(dst)[c] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    return;
  }
  // ---- combine the S partials through distributed shared memory
  cg::cluster_group cluster = cg::this_cluster();
  float* po = reinterpret_cast<float*>(ring);  // [128][kPfOStride]
  float* pm = po + kPfRows * kPfOStride;       // [128]
  float* pl = pm + kPfRows;                    // [128]
  if (sm_warp) {
    pm[i] = good ? m : -INFINITY;
    pl[i] = good ? l : 0.f;
#pragma unroll
    for (int d = 0; d < kHeadDim; d += 4)
      *reinterpret_cast<float4*>(po + i * kPfOStride + d) = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
  }
  cluster_arrive();
  cluster_wait();  // every rank's partials are in its shared memory
  if (sm_warp && good) {
    const int tid = threadIdx.x - 64;
    const int mine = (a.rows - rank + S - 1) / S;  // rows i = rank + S k of this CTA
    for (int item = tid; item < mine * (kHeadDim / 4); item += 128) {
      const int row = rank + S * (item / (kHeadDim / 4)), d = (item % (kHeadDim / 4)) * 4;
      float M = -INFINITY;
      for (int r = 0; r < S; ++r) M = fmaxf(M, cluster.map_shared_rank(pm, r)[row]);
      float L = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < S; ++r) {
        const float mr = cluster.map_shared_rank(pm, r)[row];
        const float w = mr == -INFINITY ? 0.f : __expf(mr - M);
        L += cluster.map_shared_rank(pl, r)[row] * w;
        const float4 x = *reinterpret_cast<const float4*>(cluster.map_shared_rank(po, r) + row * kPfOStride + d);
        acc.x = fmaf(x.x, w, acc.x);
        acc.y = fmaf(x.y, w, acc.y);
        acc.z = fmaf(x.z, w, acc.z);
        acc.w = fmaf(x.w, w, acc.w);
      }
      const float inv = 1.f / L;
      bf16* dst = a.out + (size_t)row * a.D + h * kHeadDim + d;
      *reinterpret_cast<uint2*>(dst) =
          make_uint2(pack_bf16(acc.x * inv, acc.y * inv), pack_bf16(acc.z * inv, acc.w * inv));
    }
  }
  cluster_arrive();
  cluster_wait();  // peers keep their shared memory until every CTA has read it
}

}  // namespace s2r
