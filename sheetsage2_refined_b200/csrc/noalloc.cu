// Masked greedy argmax that allocates nothing: s2r_masked_argmax_noalloc.
//
// This is the selection step of the fused logits kernel (logits.cuh) on its
// own: out[r] = argmax over v of (allowed[r][v] ? logits[r][v] + bias[v] :
// -inf), the lowest index winning ties and index 0 for a row with nothing
// allowed, as torch.argmax over the reference's masked logits
// (engine.py:316-317,349-350).  Like the fused kernel it reduces across CTAs
// through per-row 64-bit keys and a ticket counter; here those live in a
// file-scope device array instead of memory the engine allocates, so a call
// makes no cudaMalloc / cudaFree and touches no allocator.
//
// Who needs it: callers that cannot call cudaMalloc while they decode, such
// as a host that hands all device memory to its own pool allocator up front
// and forbids stray allocations, or a serving loop that must not stall the
// device (cudaFree synchronises it, and cudaMalloc may).
//
// Limits and sharing: at most kNoAllocMaxRows rows per call.  The scratch
// array is process-wide (every GPU that loads the library holds its own copy
// until exit) and shared by every call: calls that overlap on the GPU (two
// streams, two threads) race on it and must be serialised by the caller.
// Each call clears the scratch before use.  The first call on a device looks
// up the array's device address (cudaGetSymbolAddress) and should come
// before any stream capture on that device.  That address belongs to the
// device's primary context and is kept for the life of the process: after a
// cudaDeviceReset of the device the entry point must not be called again.
//
// The selection keys (select.cuh) are the fused logits kernel's own, so both
// paths pick the same token, -inf and signed-zero cases included.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/s2r.h"
#include "common.cuh"
#include "select.cuh"

namespace {

constexpr int kNoAllocMaxRows = 1024;
constexpr int kNoAllocMaxDevices = 64;
constexpr int kNoAllocThreads = 256;

// [0, kNoAllocMaxRows): per-row argmax keys; [kNoAllocMaxRows]: CTA ticket.
static __device__ __align__(256) unsigned long long g_argmax_scratch[kNoAllocMaxRows + 1];

std::mutex g_setup_mutex;
unsigned long long* g_scratch_ptr[kNoAllocMaxDevices] = {};

__global__ void __launch_bounds__(kNoAllocThreads)
    masked_argmax_noalloc_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                 const uint8_t* __restrict__ allowed, int rows, int vocab,
                                 unsigned long long* scratch, int64_t* __restrict__ out) {
  __shared__ unsigned long long wbest[kNoAllocThreads / 32];
  __shared__ int is_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned int* ticket = reinterpret_cast<unsigned int*>(scratch + kNoAllocMaxRows);
  for (int r = 0; r < rows; ++r) {
    unsigned long long best = 0ull;
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < vocab; v += gridDim.x * blockDim.x) {
      const size_t i = (size_t)r * vocab + v;
      if (allowed[i]) {
        const unsigned long long k = s2r::argmax_key(logits[i] + (bias ? bias[v] : 0.f), v);
        best = k > best ? k : best;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) wbest[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long k = 0ull;
      for (int w = 0; w < kNoAllocThreads / 32; ++w) k = wbest[w] > k ? wbest[w] : k;
      if (k) atomicMax(scratch + r, k);
    }
    __syncthreads();
  }
  __threadfence();
  if (threadIdx.x == 0) is_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    // nothing allowed, or a best value of -inf: index 0, as torch.argmax
    out[r] = s2r::key_token(atomicExch(scratch + r, 0ull));
  }
  if (threadIdx.x == 0) *ticket = 0u;
}

}  // namespace

// Records `msg` as s2r_last_error() of this thread (defined with the engine).
__attribute__((visibility("hidden"))) int s2r_record_error(int code, const char* msg);

static int noalloc_fail(int code, const char* msg) { return s2r_record_error(code, msg); }

extern "C" int32_t s2r_masked_argmax_noalloc(const float* logits, const float* bias, const uint8_t* allowed,
                                             int32_t rows, int32_t vocab, int64_t* out, void* stream) {
  if (!logits || !allowed || !out) return noalloc_fail(S2R_EINVAL, "s2r_masked_argmax_noalloc: NULL pointer");
  if (rows < 1 || vocab < 1) return noalloc_fail(S2R_EINVAL, "s2r_masked_argmax_noalloc: rows and vocab must be >= 1");
  if (rows > kNoAllocMaxRows)
    return noalloc_fail(S2R_EINVAL, "s2r_masked_argmax_noalloc: more than 1024 rows (the static scratch holds 1024)");
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kNoAllocMaxDevices)
    return noalloc_fail(S2R_ECUDA, "s2r_masked_argmax_noalloc: no usable current device");
  unsigned long long* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[device]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_argmax_scratch) != cudaSuccess || !p)
        return noalloc_fail(S2R_ECUDA, "s2r_masked_argmax_noalloc: cudaGetSymbolAddress of the scratch failed");
      g_scratch_ptr[device] = static_cast<unsigned long long*>(p);
    }
    scratch = g_scratch_ptr[device];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, sizeof(unsigned long long) * (kNoAllocMaxRows + 1), s) != cudaSuccess)
    return noalloc_fail(S2R_ECUDA, "s2r_masked_argmax_noalloc: clearing the scratch failed");
  int blocks = (vocab + kNoAllocThreads - 1) / kNoAllocThreads;
  blocks = blocks < 1 ? 1 : (blocks > 296 ? 296 : blocks);
  masked_argmax_noalloc_kernel<<<blocks, kNoAllocThreads, 0, s>>>(logits, bias, allowed, rows, vocab, scratch, out);
  if (cudaGetLastError() != cudaSuccess) return noalloc_fail(S2R_ECUDA, "s2r_masked_argmax_noalloc: launch failed");
  return S2R_OK;
}
