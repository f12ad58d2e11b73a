// Shared device helpers for the decode-step kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace s2r {

using bf16 = __nv_bfloat16;

constexpr int kHeadDim = 64;
constexpr int kPageTokens = 64;
constexpr float kLnEps = 1e-5f;  // torch.nn.LayerNorm default

// bfloat16 -> float of the low / high half of a packed pair.
__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Round to bfloat16 (nearest, ties to even) and widen back.
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// 16-byte streaming load that does not allocate in L1 (weights, K/V).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait until every kernel this one depends on has finished and
// its writes are visible.  Both are no-ops when the launch has no PDL edge.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Nanoseconds of the GPU's global timer (bounds on spin waits).
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Cluster barrier in two halves (release on arrive, acquire on wait), every
// thread of every CTA of the cluster taking part.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// Arrive without ordering memory (execution only).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// Byte ranges the next kernel of the stream reads that nothing writes during
// a decode step (weights; a window's cross keys and values).  Each CTA of the
// kernel before it asks the L2 for its share ahead of its own PDL wait, so
// the next kernel's loads hit the L2 even where it cannot start beside this
// one (its shared memory does not fit next to this kernel's).  Ranges start
// 16-byte aligned and their lengths are multiples of 16 (the host drops a
// range that is not); n = 0 marks an unused entry.
constexpr int kL2AheadRanges = 4;
constexpr uint32_t kL2AheadPiece = 32768;  // bytes per bulk prefetch instruction

struct L2Ahead {
  const void* p[kL2AheadRanges];
  uint32_t n[kL2AheadRanges];
};

// Ask the L2 for n bytes at p (16-byte aligned, n a multiple of 16); no data
// reaches the SM and nothing waits for it.
__device__ __forceinline__ void l2_prefetch_bytes(const void* p, uint64_t n) {
  const char* base = static_cast<const char*>(p);
  for (uint64_t o = 0; o < n; o += kL2AheadPiece) {
    const uint32_t len = (uint32_t)(n - o < kL2AheadPiece ? n - o : kL2AheadPiece);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + o), "r"(len) : "memory");
  }
}

// CTA `cta` of `ctas` prefetches its 16-byte-aligned share of every range.
__device__ __forceinline__ void l2_ahead(const L2Ahead& pf, unsigned cta, unsigned ctas) {
#pragma unroll
  for (int i = 0; i < kL2AheadRanges; ++i) {
    const uint64_t n = pf.n[i];
    if (n == 0) continue;
    const uint64_t per = (n / 16 + ctas - 1) / ctas * 16;
    const uint64_t s = (uint64_t)cta * per;
    if (s >= n) continue;
    const uint64_t e = s + per < n ? s + per : n;
    l2_prefetch_bytes(static_cast<const char*>(pf.p[i]) + s, e - s);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Fixed-point sums across CTAs.  A float partial v is added to a 64-bit
// accumulator as round(v * 2^32) with an integer atomic, so the total does
// not depend on the order in which CTAs arrive (deterministic, batch- and
// schedule-invariant) and is exact up to the one rounding per partial.
// Partials must stay below 2^26 in magnitude (|total| < 2^31 for up to 32
// of them); a larger or NaN partial is not added and reported by the caller.
constexpr int kErrAccRange = 7;             // device error word: a partial out of the fixed-point range
constexpr float kAccScale = 4294967296.0f;  // 2^32
constexpr float kAccLimit = 67108864.0f;    // 2^26

__device__ __forceinline__ bool acc_add(unsigned long long* p, float v) {
  if (!(fabsf(v) < kAccLimit)) return false;
  atomicAdd(p, (unsigned long long)__float2ll_rn(v * kAccScale));  // a reduction: no value returned
  return true;
}

// The float value of an accumulator: the nearest float to the integer, scaled back.
__device__ __forceinline__ float acc_value(unsigned long long u) {
  return __ll2float_rn((long long)u) * (1.0f / kAccScale);
}

// Which slot, position and input token a row of the current launch stands for.
// Decode: row r is slot r with the slot's own token and position.  Prefill:
// every row belongs to one slot, rows are consecutive positions from pos0 and
// the tokens come from a device array.
struct RowMap {
  int prefill;            // 0 decode, 1 prefill
  int slot;               // prefill slot
  int pos0;               // prefill first position
  const int32_t* tokens;  // prefill tokens [rows]
};

struct SlotState {
  int64_t* token;
  int64_t* position;
  uint8_t* finished;
  int64_t* ended;
  uint8_t* in_shift;
  int64_t* shift_run;
  int64_t* payload;
  int64_t* last_field;
  int64_t* incomplete;
  int64_t* g;
  int64_t* count;
  int64_t* target;
  double* stop;
  int64_t* out;         // [batch, max_tokens]
  int32_t* frames;      // real cross frames per slot
  int32_t* page_table;  // [batch, pages_per_slot]
};

__device__ __forceinline__ int row_slot(const RowMap& rm, int r) { return rm.prefill ? rm.slot : r; }
__device__ __forceinline__ int row_pos(const RowMap& rm, const SlotState& st, int r) {
  return rm.prefill ? rm.pos0 + r : (int)st.position[r];
}
__device__ __forceinline__ int row_token(const RowMap& rm, const SlotState& st, int r) {
  return rm.prefill ? rm.tokens[r] : (int)st.token[r];
}
__device__ __forceinline__ bool row_active(const RowMap& rm, const SlotState& st, int r) {
  return rm.prefill ? true : st.finished[r] == 0;
}

// Address of token t's 64-dim vector of head h in a paged K or V pool laid
// out [page][head][kPageTokens][kHeadDim].
__device__ __forceinline__ size_t paged_offset(const int32_t* page_table, int pages_per_slot, int heads, int slot,
                                               int h, int t) {
  int page = page_table[(size_t)slot * pages_per_slot + (t / kPageTokens)];
  return (((size_t)page * heads + h) * kPageTokens + (t % kPageTokens)) * kHeadDim;
}

}  // namespace s2r
