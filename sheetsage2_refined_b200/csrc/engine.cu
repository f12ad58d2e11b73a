// Host side of the decode engine and the C ABI declared in include/s2r.h.
//
// The engine owns every device buffer of a BatchDecoder
// (sheetsage2_refined/engine.py:118-149): bfloat16 weight copies, the paged
// self K/V pool, per-slot cross K/V, activations of one step, the slot state
// and the output tokens.  A decode step is a fixed sequence of kernel
// launches (8 per layer + 1) that reads every per-slot quantity (token,
// position, real frames, grammar state) from device memory, so one CUDA graph
// captured once serves every step, whatever the slots' lengths; consecutive
// kernels are chained with programmatic dependent launch so that each one
// starts streaming its weights while the previous one finishes.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "../../include/s2r.h"
#include "attention.cuh"
#include "ffn.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "kernels.h"
#include "logits.cuh"
#include "proj.cuh"

using namespace s2r;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define CK(call)                                                                                  \
  do {                                                                                            \
    cudaError_t err_ = (call);                                                                    \
    if (err_ != cudaSuccess) return fail(S2R_ECUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(err_), __FILE__, __LINE__); \
  } while (0)

constexpr int kPrefillRows = kPfRows;  // positions per prefill chunk (128: one tensor-core attention tile)
// Prefill chunks of at most this many rows run on the engine's decode kernels (for engines
// below 16 slots: the CUDA-core kernels, one pass over the weights for up to 8 rows, and the
// same arithmetic as a decode step, so a short prefix gives bit-identical K/V to forcing it
// token by token); longer chunks run on tensor cores.
constexpr int kFusedPrefillMaxRows = 8;

int kch_for(int k) { return k <= 256 ? 1 : k <= 512 ? 2 : k <= 1024 ? 4 : k <= 2048 ? 8 : 16; }
int mc_for(int m) { return m >= 5 ? 8 : m >= 3 ? 4 : m; }

// Every kernel prefers the largest shared-memory carveout.  An SM changes its
// L1 / shared-memory split only while it is idle, so kernels with different
// splits do not share an SM: the next launch's CTAs (started early under PDL)
// wait for SMs to drain, and a cluster of the attention, which needs 8 SMs
// with room in one GPC, can wait for a second wave.  Set once per kernel and
// device.
void prefer_max_shared(const void* kernel) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  std::lock_guard<std::mutex> lock(mu);
  if (done.insert({dev, kernel}).second)
    cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
}

// Launch with optional programmatic dependent launch and cluster shape.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                      int cluster, Args&&... args) {
  prefer_max_shared(reinterpret_cast<const void*>(kernel));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster > 0) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = cluster;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Host replay of the class grammar (grammar.py:140-180), used for prefixes.
struct HostGrammarState {
  uint8_t in_shift = 1, finished = 0;
  int64_t shift_run = 0, payload = 0, last_field = -1, incomplete = 0, ended = 0, g = 0;
};

}  // namespace

struct LayerBufs {
  bf16 *wqkv, *bqkv, *wo, *bo, *wcq, *bcq, *wckv, *bckv, *wco, *bco, *w1, *b1, *w2, *b2;
  float *ln_self_g, *ln_self_b, *ln_cross_g, *ln_cross_b, *ln_final_g, *ln_final_b;
  bf16 *kpool, *vpool, *ck, *cv;
  bf16* w2s;             // fc2 weight slice-major [FFN/32][D][32] for the fused FFN of one-slot engines
};

struct s2r_ctx {
  s2r_config cfg{};
  int device = 0;
  int D = 0, H = 0, F = 0, FFN = 0, V = 0, L = 0, B = 0, T = 0, maxM = 0, pps = 0, n_pages = 0;
  int num_sms = 148;
  int smem_per_sm = 228 * 1024;  // shared memory of one SM (bytes)
  bool pdl = true, use_graph = true;
  bool fence_next = false;  // the next launch starts a decode step or prefill chunk: no programmatic overlap
  std::vector<void*> allocs;
  char* arena = nullptr;  // the current arena of small buffers and its fill
  size_t arena_used = 0;
  // weights
  float *tok_emb = nullptr, *pos_emb = nullptr, *emb_ln_g = nullptr, *emb_ln_b = nullptr;
  bf16* emb_bf16 = nullptr;
  std::vector<LayerBufs> layers;
  // activations of one step
  float *r = nullptr, *x = nullptr;
  bf16 *q = nullptr, *att = nullptr, *hid = nullptr;
  void* mem_stage = nullptr;
  int32_t* prefill_tokens = nullptr;
  unsigned long long* keys = nullptr;
  unsigned int* counter = nullptr;
  int* dev_error = nullptr;  // set by kernels on a broken invariant (0: none)
  float* bias = nullptr;
  bool has_bias = false;
  int64_t* dbg_forced = nullptr;
  float* dbg_logits = nullptr;
  int64_t* dbg_greedy = nullptr;
  SlotState st{};
  Grammar gr{};
  Rescore rs{};  // frame-head rescoring (device tables and state)
  int rs_time_hz = 100;
  int rs_meters = 0;  // entries of the device meter tables (sized by the first s2r_set_rescore)
  // host copies for prefix replay
  std::vector<int8_t> h_token_class;
  std::vector<int32_t> h_field;
  std::vector<double> h_time;
  // slots
  std::vector<int> loaded, bound;
  std::vector<std::vector<int>> slot_pages;
  std::vector<int> free_pages;
  std::vector<int32_t> h_page_table;
  // graph
  cudaGraphExec_t graph = nullptr;
  bool graph_dirty = true;
  cudaStream_t cap_stream = nullptr;
  // asynchronous polls and takes (pinned host copies, allocated on first use)
  uint8_t* h_fin = nullptr;      // [B] finished flags of the last asynchronous poll
  int* h_err = nullptr;          // the device error word read with them
  cudaEvent_t poll_ev = nullptr;  // the poll's copies have landed
  cudaStream_t poll_stream = nullptr;
  bool poll_pending = false;
  int64_t* h_out = nullptr;      // [B][T] tokens of asynchronous takes
  int64_t* h_pos_end = nullptr;  // [B][2] position and end reason of each
  std::vector<cudaEvent_t> take_ev;
  std::vector<uint8_t> take_pending;
  // tensor-core projections (tcgen05 GEMM): the step and prefill projections
  // when `tc` (16 or more slots), the cross K/V projection at load when `tc_cross`
  bool tc = false, tc_cross = false;
  // engines below 16 slots decode on the CUDA-core kernels but run prefill chunks of more
  // than kFusedPrefillMaxRows rows through the tensor-core layer (load_slot switches the
  // engine to it for those chunks: PrefillOnTensorCores)
  bool tc_prefill = false;
  int tc_nb = 64;                  // rows per MMA tile of the step and prefill projections
  // engines below 16 slots fuse each attention with its out-projection (fixed-point sums in
  // acc_self / acc_cross); the next launch adds bias and residual and normalises (IN_ACC)
  bool fuse_out = false;
  unsigned long long* acc_self = nullptr;   // [maxM][D]
  unsigned long long* acc_cross = nullptr;  // [maxM][D]
  unsigned long long* acc_ffn = nullptr;    // [maxM][D] fc2 sums (EPI_SLICES), read by the next LayerNorm
  float* x_b = nullptr;                     // [maxM][D] the cross attention's residual input
  float* x_c = nullptr;                     // [maxM][D] the FFN's residual input
  bool fuse_ffn = false;                    // one-slot engines: decode steps run the FFN as one kernel
  int attn_splits = 8;             // CTAs (one cluster) per (row, head) of the self-attention
  int attn_splits_cross = 8;       // ... and of the cross-attention
  int32_t *order_self = nullptr, *order_cross = nullptr;  // [B] decode rows, longest first (tensor-core engines)
  int32_t* h_order = nullptr;                             // pinned [2B] staging of both orders
  cudaEvent_t order_copied = nullptr;                     // the last upload of h_order has run
  std::vector<int32_t> h_frames;                          // real frames per slot
  bf16* xln = nullptr;             // [maxM][KP] LayerNorm'd rows, the X operand of LN'd projections
  bf16* mem_bf16 = nullptr;        // [F][D] float32 encoder memory rounded to bf16
  bf16* wckv_all = nullptr;        // [L][2D][D]: every layer's [Wck; Wcv] (layers[l].wckv points into it)
  // profiling: when set, an event is recorded after every launch of a step
  std::vector<std::pair<int, cudaEvent_t>>* prof = nullptr;
};

namespace {

// Buffers up to kArenaPiece bytes (activations, slot state, biases and
// LayerNorm weights) are packed into 32 MB arenas, so that everything a step
// touches besides the weight matrices and the K/V pools sits in a few large
// pages; larger buffers get their own allocation.
constexpr size_t kArenaPiece = 4u << 20;
constexpr size_t kArenaChunk = 32u << 20;

template <typename T>
int dalloc(s2r_ctx* c, T** p, size_t count) {
  const size_t bytes = std::max<size_t>(count, 1) * sizeof(T);
  if (bytes <= kArenaPiece) {
    size_t off = (c->arena_used + 255) & ~(size_t)255;
    if (!c->arena || off + bytes > kArenaChunk) {
      void* chunk = nullptr;
      cudaError_t e = cudaMalloc(&chunk, kArenaChunk);
      if (e != cudaSuccess) return fail(S2R_ENOMEM, "cudaMalloc(%zu bytes): %s", kArenaChunk, cudaGetErrorString(e));
      c->allocs.push_back(chunk);
      c->arena = static_cast<char*>(chunk);
      off = 0;
    }
    *p = reinterpret_cast<T*>(c->arena + off);
    c->arena_used = off + bytes;
    return S2R_OK;
  }
  void* ptr = nullptr;
  cudaError_t e = cudaMalloc(&ptr, bytes);
  if (e != cudaSuccess) return fail(S2R_ENOMEM, "cudaMalloc(%zu bytes): %s", bytes, cudaGetErrorString(e));
  c->allocs.push_back(ptr);
  *p = static_cast<T*>(ptr);
  return S2R_OK;
}

#define TRY(x)                  \
  do {                          \
    int rc_ = (x);              \
    if (rc_ != S2R_OK) return rc_; \
  } while (0)

enum KernelClass { K_QKV = 0, K_SELF_ATTN, K_SELF_OUT, K_CROSS_Q, K_CROSS_ATTN, K_CROSS_OUT, K_FC1, K_FC2, K_LOGITS, K_CLASSES };

int mark(s2r_ctx* c, int cls, cudaStream_t s) {
  if (!c->prof) return S2R_OK;
  cudaEvent_t e;
  CK(cudaEventCreate(&e));
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  CK(cudaStreamIsCapturing(s, &cap));
  if (cap == cudaStreamCaptureStatusActive)
    CK(cudaEventRecordWithFlags(e, s, cudaEventRecordExternal));  // an event node of the graph
  else
    CK(cudaEventRecord(e, s));
  c->prof->push_back({cls, e});
  return S2R_OK;
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

// out[s][n][j] = in[n][32s + j] for the [D, FFN] fc2 weight: each 32-column
// slice of every row made contiguous for the fused FFN kernel.
__global__ void slice_major_kernel(const bf16* __restrict__ in, bf16* __restrict__ out, int D, int FFN) {
  const size_t total = (size_t)D * FFN;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % kSliceCols);
    const size_t rest = i / kSliceCols;
    const int n = (int)(rest % D), sl = (int)(rest / D);
    out[i] = in[(size_t)n * FFN + sl * kSliceCols + j];
  }
}

// Copy float32 weights (host or device) into `dst` as bfloat16, through a
// float32 staging buffer.
int upload_bf16(s2r_ctx* c, bf16* dst, const float* src, size_t n, float* stage) {
  if (!src) return fail(S2R_EINVAL, "a weight pointer is NULL");
  CK(cudaMemcpy(stage, src, n * sizeof(float), cudaMemcpyDefault));
  f32_to_bf16_kernel<<<std::min<size_t>((n + 255) / 256, 4096), 256>>>(stage, dst, n);
  CK(cudaGetLastError());
  return S2R_OK;
}

int upload_f32(float* dst, const float* src, size_t n) {
  if (!src) return fail(S2R_EINVAL, "a weight pointer is NULL");
  CK(cudaMemcpy(dst, src, n * sizeof(float), cudaMemcpyDefault));
  return S2R_OK;
}

// Programmatic dependent launch for the next kernel, except for the first
// kernel of a decode step or prefill chunk (fence_next): that one starts after
// everything before it has completed, so the step's kernels may read data
// written before the step (cross K/V, earlier positions' K/V) ahead of their
// griddepcontrol.wait.
bool next_pdl(s2r_ctx* c) {
  const bool fenced = c->fence_next;
  c->fence_next = false;
  return c->pdl && !fenced;
}

ProjArgs proj_base(s2r_ctx* c) {
  ProjArgs a{};
  a.err = c->dev_error;
  a.st = c->st;
  a.heads = c->H;
  a.pages_per_slot = c->pps;
  a.frames_cap = c->F;
  return a;
}

// ---- tensor-core projections --------------------------------------------

constexpr int kTcMinBatch = 16;     // engines with this many slots run step projections on tensor cores
constexpr int kTcMinKPerSplit = 2;  // K tiles (of 64) per split-K slice, at least

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major bf16 matrix [rows][inner] with `row_bytes` between rows, read in
// boxes of 64 columns x box_rows rows with the 128-byte swizzle; reads outside
// the matrix return zeros.
int encode_rows(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(S2R_ECUDA, "the driver has no cuTensorMapEncodeTiled");
  if (reinterpret_cast<uintptr_t>(ptr) % 16 || row_bytes % 16 || rows == 0 || inner == 0)
    return fail(S2R_EINVAL, "tensor map: pointer or row stride not 16-byte aligned, or an empty matrix");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)kTcBlockK, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(S2R_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return S2R_OK;
}

// Split-K cluster size (1, 2, 4 or 8) for `tiles` output tiles of k_tiles K
// tiles each: up to two CTAs an SM (one an SM measured 2% slower on the
// 64-slot step; fewer, longer slices 2% slower again), at least
// kTcMinKPerSplit K tiles per slice.  The step and prefill projections pass the feature tiles only,
// so that the split, and with it a row's result, does not depend on how many
// rows share the launch.
void tc_split(int tiles, int k_tiles, int sms, int* splits, int* per) {
  int sp = 1;
  while (sp < kTcMaxSplits && tiles * sp * 2 <= 2 * sms && k_tiles / (sp * 2) >= kTcMinKPerSplit) sp *= 2;
  *per = (k_tiles + sp - 1) / sp;
  *splits = sp;
}

// One step or prefill projection on tensor cores: the LayerNorm that produces
// its bf16 rows (when the input is not bf16 already), then the GEMM with the
// projection's epilogue.  `lg` is the logits epilogue's state.
int launch_proj_tc(s2r_ctx* c, ProjArgs a, int in, int epi, cudaStream_t s, const LogitsArgs* lg = nullptr) {
  if (in != IN_LN && in != IN_EMBED && in != IN_BF16)
    return fail(S2R_ENOTSUP, "tensor-core projections take LayerNorm'd or bf16 rows (input mode %d)", in);
  // prefill chunks of more rows than a decode tile take several row tiles (128-row tiles for
  // 128-row chunks measured slower: one CTA an SM)
  const int nb = c->tc_nb;
  const void* x = a.xin;
  int ldx = a.ldx;
  if (in == IN_LN || in == IN_EMBED) {
    const int kch = kch_for(a.K);
    LnFn fn = ln_fn(in, kch);
    CK(launch_ex(fn, dim3(a.M), dim3(128), 0, s, next_pdl(c), 0, a, c->xln));
    x = c->xln;
    ldx = kch * 256;
  }
  const int n_tiles = (a.N + kTcBlockN - 1) / kTcBlockN, m_tiles = (a.M + nb - 1) / nb;
  const int k_tiles = (a.K + kTcBlockK - 1) / kTcBlockK;
  int splits = 1, per = k_tiles;
  tc_split(n_tiles, k_tiles, c->num_sms, &splits, &per);
  GemmFn fn = gemm_fn(nb, epi);
  if (!fn) return fail(S2R_ENOTSUP, "no tensor-core projection for epilogue %d with %d-row tiles", epi, nb);
  CUtensorMap map_w, map_x;
  TRY(encode_rows(&map_w, a.W, a.K, a.N, (uint64_t)a.K * sizeof(bf16), kTcBlockN));
  TRY(encode_rows(&map_x, x, a.K, a.M, (uint64_t)ldx * sizeof(bf16), nb));
  TcArgs t{};
  t.p = a;
  t.k_tiles_per_split = per;
  t.err = c->dev_error;
  if (lg) t.lg = *lg;
  const size_t smem = tc_smem_bytes(nb);
  CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CK(launch_ex(fn, dim3(splits, n_tiles, m_tiles), dim3(kTcThreads), smem, s, next_pdl(c), splits > 1 ? splits : 0, map_w,
               map_x, t));
  return S2R_OK;
}

int launch_proj(s2r_ctx* c, ProjArgs a, int in, int epi, cudaStream_t s) {
  if (c->tc && epi != EPI_CROSSKV) return launch_proj_tc(c, a, in, epi, s);
  const int kch = kch_for(a.K), mc = mc_for(std::min(a.M, 8));
  ProjFn fn = proj_fn(in, epi, kch, mc);
  if (!fn) return fail(S2R_ENOTSUP, "no projection kernel for in=%d epi=%d", in, epi);
  // staged rows, then the LayerNorm parameters for LayerNorm'd inputs
  const size_t smem = (size_t)(mc == 8 ? 8 : mc) * kch * 256 * sizeof(bf16) +
                      ((in == IN_LN || in == IN_EMBED || in == IN_ACC) ? 2 * (size_t)kch * 256 * sizeof(float) : 0);
  CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int threads = mc == 1 ? proj_threads<1>() : proj_threads<2>(), warps = threads / 32;
  const int blocks = (a.N + warps - 1) / warps;
  CK(launch_ex(fn, dim3(blocks), dim3(threads), smem, s, next_pdl(c), 0, a));
  return S2R_OK;
}

// Cross K/V of one window for every layer (decoder.py:98-116): one
// persistent tcgen05 launch per group of up to kCkvMaxLayers layers, over the
// stacked [Wck; Wcv] of the group.  x: the window's frames as bf16 rows [frames, D].
int launch_crosskv(s2r_ctx* c, const bf16* x, int frames, int slot, cudaStream_t s) {
  CrossKvFn fn = crosskv_fn();
  const size_t smem = ckv_smem_bytes(kCkvStages);
  CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const uint64_t D = c->D;
  CUtensorMap map_x;
  TRY(encode_rows(&map_x, x, D, (uint64_t)frames, D * sizeof(bf16), kCkvBlockM));
  for (int l0 = 0; l0 < c->L; l0 += kCkvMaxLayers) {
    const int nl = std::min(kCkvMaxLayers, c->L - l0);
    CUtensorMap map_w;
    TRY(encode_rows(&map_w, c->wckv_all + (size_t)l0 * 2 * D * D, D, (uint64_t)nl * 2 * D, D * sizeof(bf16),
                    kCkvBlockN));
    CrossKvArgs a{};
    a.frames = frames;
    a.D = c->D;
    a.heads = c->H;
    a.layers = nl;
    a.frames_cap = c->F;
    a.slot = slot;
    a.err = c->dev_error;
    for (int i = 0; i < nl; ++i) {
      a.bias[i] = c->layers[l0 + i].bckv;
      a.k_dst[i] = c->layers[l0 + i].ck;
      a.v_dst[i] = c->layers[l0 + i].cv;
    }
    const long long tiles =
        (long long)((frames + kCkvBlockM - 1) / kCkvBlockM) * ((nl * 2 * c->D + kCkvBlockN - 1) / kCkvBlockN);
    const int grid = (int)std::min<long long>(tiles, c->num_sms);
    CK(launch_ex(fn, dim3(grid), dim3(kCkvThreads), smem, s, next_pdl(c), 0, map_x, map_w, a));
  }
  return S2R_OK;
}

// Every (row, head) of an engine is split over the same number of CTAs
// (attn_splits, attn_splits_cross) whatever the rows of the launch, so a
// row's result never depends on how many rows share it (decode with any
// slots live and prefill chunks give bit-identical K/V and outputs).  Engines
// of fewer than 16 slots split 8 ways; tensor-core engines split so that the
// (row, head) pairs of a full batch cover the SMs about four times, and
// twice that for the cross-attention, whose rows are long (every encoder
// frame) and uneven.
constexpr int kAttnSplits = 8;
// Engines below 16 slots whose heads are few split the cross attention 16 ways (non-portable
// clusters of 16) when one row's 16 CTAs per head fit the SMs in one wave: the product decoder's
// 8 heads over 7,500 frames ran on only 64 CTAs with 8-way splits.  The choice depends on the
// heads only, not on the slots, so a slot's result does not depend on the engine's batch.
constexpr int kAttnWideSplits = 16;

int attn_splits_for(const s2r_ctx* c, int cover) {
  if (!c->tc) return kAttnSplits;
  int sp = 1;
  while (sp < kAttnSplits && c->B * c->H * sp * 2 <= cover * c->num_sms) sp *= 2;
  return sp;
}

// Decode rows longest first (self: by position, cross: by real frames), so
// that the attention CTAs of the longest rows start first and the short
// ones fill in behind them.  Uploaded before each run; the order does not
// change any row's result.
int upload_row_order(s2r_ctx* c, cudaStream_t s) {
  if (!c->order_self) return S2R_OK;
  CK(cudaEventSynchronize(c->order_copied));  // the previous upload has left the staging buffer
  int32_t* by_pos = c->h_order;
  int32_t* by_frames = c->h_order + c->B;
  for (int i = 0; i < c->B; ++i) by_pos[i] = by_frames[i] = i;
  std::stable_sort(by_pos, by_pos + c->B, [&](int a, int b) {
    return (c->loaded[a] ? c->bound[a] : -1) > (c->loaded[b] ? c->bound[b] : -1);
  });
  std::stable_sort(by_frames, by_frames + c->B, [&](int a, int b) {
    return (c->loaded[a] ? c->h_frames[a] : -1) > (c->loaded[b] ? c->h_frames[b] : -1);
  });
  CK(cudaMemcpyAsync(c->order_self, by_pos, c->B * sizeof(int32_t), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(c->order_cross, by_frames, c->B * sizeof(int32_t), cudaMemcpyHostToDevice, s));
  CK(cudaEventRecord(c->order_copied, s));
  return S2R_OK;
}

// How an attention launch of M rows gets its keys (kAttnPre*), how many rows
// it stages, whether it computes its own query rows, and its dynamic shared
// memory.  The same for every launch of an engine with the same M.
struct AttnPlan {
  int C = 1, chunk_cap = 0, pre = kAttnPreNone, stage_cap = 0;
  bool fuse_q = false;
  size_t smem = 0;
};

AttnPlan plan_attn(const s2r_ctx* c, int M, bool cross) {
  AttnPlan p;
  p.C = cross ? c->attn_splits_cross : c->attn_splits;
  p.chunk_cap = ((cross ? c->F : c->T) + p.C - 1) / p.C;
  p.pre = c->tc ? kAttnPreNone : kAttnPreRegs;
  // the cross attention of a fused engine can compute its own query rows
  // (8 per CTA, one per warp) when it stages and splits 8 ways
  const bool can_fuse_q = cross && c->fuse_out && (p.C == 8 || p.C == 16) && c->D % 256 == 0 && c->D <= 1024;
  if (!c->tc) {
    // Stage the CTAs' earlier keys and values in shared memory when the
    // launch fits on the SMs in one wave with room left for a CTA of the
    // other attention kernel beside each and for the projection kernels in
    // flight (kernels start ahead of their inputs under PDL).
    const int ctas = M * c->H * p.C;
    const int per_sm = std::max(1, (ctas + c->num_sms - 1) / c->num_sms);
    const size_t budget = ((size_t)c->smem_per_sm - kAttnOtherSmem) / (2 * per_sm);
    const size_t fixed =
        AttnSmem(p.chunk_cap, 0, c->D, can_fuse_q).total + (p.C > 8 ? kAttnStaticSmemWide : kAttnStaticSmem);
    if (budget > fixed) {
      const int cap = (int)std::min<size_t>(p.chunk_cap, (budget - fixed) / (2 * kHeadDim * 2));
      if (cap == p.chunk_cap || cap >= kAttnGroups * kAttnUnroll) {
        p.pre = kAttnPreStage;
        p.stage_cap = cap;
        p.fuse_q = can_fuse_q;
      }
    }
  }
  p.smem = AttnSmem(p.chunk_cap, p.stage_cap, c->D, p.fuse_q).total;
  return p;
}

// Switch the cross attention to kAttnWideSplits CTAs per (row, head) if the device can
// schedule a cluster of that size with the kernel's shared memory (else keep 8).
int widen_cross_splits(s2r_ctx* c) {
  const int keep = c->attn_splits_cross;
  c->attn_splits_cross = kAttnWideSplits;
  const AttnPlan p = plan_attn(c, c->B, true);
  void (*fn)(const AttnArgs) = p.pre == kAttnPreStage ? attn_kernel<kAttnPreStage, true, kAttnWideSplits>
                                                      : attn_kernel<kAttnPreRegs, true, kAttnWideSplits>;
  CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem));
  CK(cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kAttnWideSplits, c->H, 1);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = p.smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = kAttnWideSplits;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) != cudaSuccess || clusters < 1) {
    cudaGetLastError();  // not schedulable here: keep the portable split
    c->attn_splits_cross = keep;
  }
  return S2R_OK;
}

// What a kernel of a one-slot decode step reads that no kernel of the step
// writes, for the kernel before it to prefetch into the L2 (l2_ahead).  Only
// where the kernel cannot load it ahead of its own PDL wait: the fused FFN
// (its shared memory does not fit beside the cross attention's, so it starts
// late), the logits (the same for the product vocabulary's 33 MB) and the
// step's first QKV projection (the step boundary has no programmatic
// overlap).  The other kernels load their weights before their wait while
// the kernel before them runs; prefetching those as well was slower.
enum AheadOf { kAheadFfn, kAheadQkv, kAheadLogits };

void add_ahead(L2Ahead& pf, int& i, const void* p, size_t n) {
  n &= ~(size_t)15;
  if (!p || n == 0 || (reinterpret_cast<uintptr_t>(p) & 15) || n > 0xffffffffu || i >= kL2AheadRanges) return;
  pf.p[i] = p;
  pf.n[i] = (uint32_t)n;
  ++i;
}

L2Ahead l2_ahead_of(const s2r_ctx* c, int l, AheadOf next) {
  L2Ahead pf{};
  int i = 0;
  if (!c->fuse_ffn) return pf;
  const size_t D = c->D, w = D * D * sizeof(bf16);
  const LayerBufs& lb = c->layers[l];
  switch (next) {
    case kAheadFfn:
      add_ahead(pf, i, lb.w1, (size_t)c->FFN * D * sizeof(bf16));
      add_ahead(pf, i, lb.w2s, (size_t)c->FFN * D * sizeof(bf16));
      break;
    case kAheadQkv:
      add_ahead(pf, i, lb.wqkv, 3 * w);
      break;
    case kAheadLogits:
      add_ahead(pf, i, c->emb_bf16, (size_t)c->V * D * sizeof(bf16));
      break;
  }
  return pf;
}

int launch_attn(s2r_ctx* c, RowMap rm, int M, int layer, bool cross, cudaStream_t s, L2Ahead ahead = L2Ahead{}) {
  const AttnPlan plan = plan_attn(c, M, cross);
  AttnArgs a{};
  a.ahead = ahead;
  a.M = M;
  a.H = c->H;
  a.rm = rm;
  a.st = c->st;
  a.q = c->q;
  a.ldq = c->D;
  a.out = c->att;
  a.ldo = c->D;
  a.cross = cross;
  a.k = cross ? c->layers[layer].ck : c->layers[layer].kpool;
  a.v = cross ? c->layers[layer].cv : c->layers[layer].vpool;
  a.pages_per_slot = c->pps;
  a.frames_cap = c->F;
  const int C = plan.C;
  a.splits = C;
  a.err = c->dev_error;
  a.order = rm.prefill ? nullptr : (cross ? c->order_cross : c->order_self);
  if (c->fuse_out) {
    const LayerBufs& w = c->layers[layer];
    a.D = c->D;
    a.wo = cross ? w.wco : w.wo;
    a.acc_out = cross ? c->acc_cross : c->acc_self;
    if (cross && plan.fuse_q && c->fuse_ffn && !rm.prefill) {  // QKV has read acc_ffn; the fused FFN adds into it
      a.zero = c->acc_ffn;
      a.zero_n = M * c->D;
    }
    if (plan.fuse_q) {  // the cross attention's input: self_attn_norm(x + bf16(self out-projection))
      a.acc_in = c->acc_self;
      a.bias_in = w.bo;
      a.x_in = c->x;
      a.x_out = c->x_b;
      a.ln_g = w.ln_self_g;
      a.ln_b = w.ln_self_b;
      a.wq = w.wcq;
      a.bq = w.bcq;
      a.fuse_q = 1;
    }
  }
  a.chunk_cap = plan.chunk_cap;
  a.stage_cap = plan.stage_cap;
  const int pre = plan.pre;
  const size_t smem = plan.smem;
  // tensor-core engines read keys in the loops and keep their out-projection a GEMM; the
  // others load keys ahead of the wait and fuse the out-projection
  if ((pre == kAttnPreNone) == c->fuse_out) return fail(S2R_ENOTSUP, "no attention kernel for this engine");
  void (*fn)(const AttnArgs) = pre == kAttnPreNone ? attn_kernel<kAttnPreNone, false>
                               : C > 8 ? (pre == kAttnPreRegs ? attn_kernel<kAttnPreRegs, true, kAttnWideSplits>
                                                              : attn_kernel<kAttnPreStage, true, kAttnWideSplits>)
                               : pre == kAttnPreRegs ? attn_kernel<kAttnPreRegs, true>
                                                     : attn_kernel<kAttnPreStage, true>;
  CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  if (C > 8) CK(cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  CK(launch_ex(fn, dim3(C, c->H, M), dim3(kAttnThreads), smem, s, next_pdl(c), C, a));
  return S2R_OK;
}

// Attention of a prefill chunk on tensor cores (prefill_attn.cuh): the chunk's
// M rows (positions pos0 .. pos0 + M - 1 of one slot) of every head against
// the slot's keys, key tiles split over a cluster of up to 8 CTAs per head.
int launch_prefill_attn(s2r_ctx* c, RowMap rm, int M, int layer, bool cross, cudaStream_t s) {
  if (M > kPfRows) return fail(S2R_EINVAL, "a prefill chunk holds at most %d rows", kPfRows);
  const int n_max = cross ? c->h_frames[rm.slot] : rm.pos0 + M;
  const int tiles = (n_max + kPfKeys - 1) / kPfKeys;
  int splits = std::min(kPfMaxSplits, std::max(1, (tiles + 3) / 4));  // at least 4 key tiles a CTA
  const int per = (tiles + splits - 1) / splits;
  splits = (tiles + per - 1) / per;  // no CTA without keys
  const LayerBufs& w = c->layers[layer];
  CUtensorMap map_q, map_k, map_v;
  TRY(encode_rows(&map_q, c->q, c->D, (uint64_t)M, (uint64_t)c->D * sizeof(bf16), kPfRows));
  const uint64_t key_rows = cross ? (uint64_t)c->B * c->H * c->F : (uint64_t)c->n_pages * c->H * kPageTokens;
  TRY(encode_rows(&map_k, cross ? w.ck : w.kpool, kHeadDim, key_rows, kHeadDim * sizeof(bf16), kPfKeys));
  TRY(encode_rows(&map_v, cross ? w.cv : w.vpool, kHeadDim, key_rows, kHeadDim * sizeof(bf16), kPfKeys));
  PrefillAttnArgs a{};
  a.rows = M;
  a.pos0 = rm.pos0;
  a.slot = rm.slot;
  a.cross = cross;
  a.H = c->H;
  a.D = c->D;
  a.pages_per_slot = c->pps;
  a.frames_cap = c->F;
  a.tiles = tiles;
  a.per = per;
  a.page_table = c->st.page_table;
  a.frames = c->st.frames;
  a.out = c->att;
  a.err = c->dev_error;
  PrefillAttnFn fn = prefill_attn_fn();
  CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PfSmem::total));
  CK(launch_ex(fn, dim3(splits, c->H), dim3(kPfThreads), PfSmem::total, s, next_pdl(c), splits > 1 ? splits : 0, map_q,
               map_k, map_v, a));
  return S2R_OK;
}

// One decoder layer for M rows.  `last_kv_only`: only the K/V append (the
// prefill's last layer needs nothing else).
int enqueue_layer(s2r_ctx* c, RowMap rm, int M, int l, bool last_kv_only, cudaStream_t s) {
  const LayerBufs& w = c->layers[l];
  const int D = c->D;
  {  // 1. (embedding +) LayerNorm -> QKV, K/V append
    ProjArgs a = proj_base(c);
    a.rm = rm;
    a.M = M;
    a.K = D;
    a.N = 3 * D;
    int in = IN_LN;
    if (l == 0) {
      in = IN_EMBED;
      a.tok_emb = c->tok_emb;
      a.pos_emb = c->pos_emb;
      a.gamma = c->emb_ln_g;
      a.beta = c->emb_ln_b;
    } else if (c->fuse_out) {  // final_norm(x + bf16(fc2 sums + b2)) of the layer before
      in = IN_ACC;
      a.r = c->x_c;
      a.acc = c->acc_ffn;
      a.acc_bias = c->layers[l - 1].b2;
      a.gamma = c->layers[l - 1].ln_final_g;
      a.beta = c->layers[l - 1].ln_final_b;
    } else {
      a.r = c->r;
      a.gamma = c->layers[l - 1].ln_final_g;
      a.beta = c->layers[l - 1].ln_final_b;
    }
    a.x_out = c->x;
    a.W = w.wqkv;
    a.bias = w.bqkv;
    a.out = c->q;
    a.ldo = D;
    a.k_dst = w.kpool;
    a.v_dst = w.vpool;
    if (c->fuse_out) {  // the FFN before (or the last step's) has read acc_cross
      a.zero = c->acc_cross;
      a.zero_n = M * D;
    }
    TRY(launch_proj(c, a, in, EPI_QKV, s));
    TRY(mark(c, K_QKV, s));
  }
  if (last_kv_only) return S2R_OK;
  if (c->fuse_out) {
    // each attention fused with its out-projection (attention.cuh): fixed-point sums in
    // acc_self / acc_cross; the launch after it adds bias and residual and normalises (IN_ACC)
    const bool ahead = c->fuse_ffn && !rm.prefill;
    TRY(launch_attn(c, rm, M, l, false, s));  // 2-3. self-attention + out-projection
    TRY(mark(c, K_SELF_ATTN, s));
    if (!plan_attn(c, M, true).fuse_q) {  // 4. self_attn_norm -> cross q (else the cross attention does it)
      ProjArgs a = proj_base(c);
      a.rm = rm;
      a.M = M;
      a.K = D;
      a.N = D;
      a.r = c->x;
      a.acc = c->acc_self;
      a.acc_bias = w.bo;
      a.gamma = w.ln_self_g;
      a.beta = w.ln_self_b;
      a.x_out = c->x_b;
      a.W = w.wcq;
      a.bias = w.bcq;
      a.out = c->q;
      a.ldo = D;
      if (c->fuse_ffn && !rm.prefill) {  // the QKV projection has read acc_ffn; the fused FFN adds into it
        a.zero = c->acc_ffn;
        a.zero_n = M * D;
      }
      TRY(launch_proj(c, a, IN_ACC, EPI_BF16, s));
      TRY(mark(c, K_CROSS_Q, s));
    }
    TRY(launch_attn(c, rm, M, l, true, s, ahead ? l2_ahead_of(c, l, kAheadFfn) : L2Ahead{}));  // 5-6. cross-attention + out-projection
    TRY(mark(c, K_CROSS_ATTN, s));
    if (c->fuse_ffn && !rm.prefill) {  // 7-8. cross_attn_norm, fc1, GELU and fc2 in one launch
      FfnArgs f{};
      f.D = D;
      f.FFN = c->FFN;
      f.m = 0;
      f.x_in = c->x_b;
      f.acc_in = c->acc_cross;
      f.bias_in = w.bco;
      f.ln_g = w.ln_cross_g;
      f.ln_b = w.ln_cross_b;
      f.x_out = c->x_c;
      f.w1 = w.w1;
      f.b1 = w.b1;
      f.w2s = w.w2s;
      f.acc_out = c->acc_ffn;
      f.zero = c->acc_self;
      f.zero_n = M * D;
      f.err = c->dev_error;
      if (l + 1 == c->L) f.ahead = l2_ahead_of(c, l, kAheadLogits);
      const int kch = kch_for(D);
      void (*fn)(const FfnArgs) = kch == 1 ? ffn_row_kernel<1> : kch == 2 ? ffn_row_kernel<2> : ffn_row_kernel<4>;
      const size_t smem = ffn_smem_bytes(D);
      CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      CK(launch_ex(fn, dim3(c->FFN / kFfnSlice), dim3(kFfnThreads), smem, s, next_pdl(c), 0, f));
      TRY(mark(c, K_FC1, s));
      return S2R_OK;
    }
    {  // 7. cross_attn_norm -> fc1 + GELU; acc_self has been read
      ProjArgs a = proj_base(c);
      a.rm = rm;
      a.M = M;
      a.K = D;
      a.N = c->FFN;
      a.r = c->x_b;
      a.acc = c->acc_cross;
      a.acc_bias = w.bco;
      a.gamma = w.ln_cross_g;
      a.beta = w.ln_cross_b;
      a.x_out = c->x_c;
      a.W = w.w1;
      a.bias = w.b1;
      a.out = c->hid;
      a.ldo = c->FFN;
      a.zero = c->acc_self;
      a.zero_n = M * D;
      TRY(launch_proj(c, a, IN_ACC, EPI_GELU, s));
      TRY(mark(c, K_FC1, s));
    }
  } else {
  // 2. self-attention (prefill chunks of more than kFusedPrefillMaxRows rows: all rows of a head
  // in one tensor-core tile; shorter ones, like decode rows, one cluster per row and head)
  const bool pf_tile = rm.prefill && M > kFusedPrefillMaxRows;
  TRY(pf_tile ? launch_prefill_attn(c, rm, M, l, false, s) : launch_attn(c, rm, M, l, false, s));
  TRY(mark(c, K_SELF_ATTN, s));
  {                                         // 3. out-projection + residual
    ProjArgs a = proj_base(c);
    a.rm = rm;
    a.M = M;
    a.K = D;
    a.N = D;
    a.xin = c->att;
    a.ldx = D;
    a.W = w.wo;
    a.bias = w.bo;
    a.r_out = c->r;
    a.x_res = c->x;
    TRY(launch_proj(c, a, IN_BF16, EPI_RESID, s));
    TRY(mark(c, K_SELF_OUT, s));
  }
  {  // 4. self_attn_norm -> cross q
    ProjArgs a = proj_base(c);
    a.rm = rm;
    a.M = M;
    a.K = D;
    a.N = D;
    a.r = c->r;
    a.gamma = w.ln_self_g;
    a.beta = w.ln_self_b;
    a.x_out = c->x;
    a.W = w.wcq;
    a.bias = w.bcq;
    a.out = c->q;
    a.ldo = D;
    TRY(launch_proj(c, a, IN_LN, EPI_BF16, s));
    TRY(mark(c, K_CROSS_Q, s));
  }
  TRY(pf_tile ? launch_prefill_attn(c, rm, M, l, true, s) : launch_attn(c, rm, M, l, true, s));  // 5. cross-attention
  TRY(mark(c, K_CROSS_ATTN, s));
  {                                        // 6. cross out-projection + residual
    ProjArgs a = proj_base(c);
    a.rm = rm;
    a.M = M;
    a.K = D;
    a.N = D;
    a.xin = c->att;
    a.ldx = D;
    a.W = w.wco;
    a.bias = w.bco;
    a.r_out = c->r;
    a.x_res = c->x;
    TRY(launch_proj(c, a, IN_BF16, EPI_RESID, s));
    TRY(mark(c, K_CROSS_OUT, s));
  }
  {  // 7. cross_attn_norm -> fc1 + GELU
    ProjArgs a = proj_base(c);
    a.rm = rm;
    a.M = M;
    a.K = D;
    a.N = c->FFN;
    a.r = c->r;
    a.gamma = w.ln_cross_g;
    a.beta = w.ln_cross_b;
    a.x_out = c->x;
    a.W = w.w1;
    a.bias = w.b1;
    a.out = c->hid;
    a.ldo = c->FFN;
    TRY(launch_proj(c, a, IN_LN, EPI_GELU, s));
    TRY(mark(c, K_FC1, s));
  }
  }
  {  // 8. fc2 (+ residual); acc_cross has been read
    ProjArgs a = proj_base(c);
    a.rm = rm;
    a.M = M;
    a.K = c->FFN;
    a.N = D;
    a.xin = c->hid;
    a.ldx = c->FFN;
    a.W = w.w2;
    a.bias = w.b2;
    if (c->fuse_out) {  // fixed-point sums; the next LayerNorm adds bias and residual (IN_ACC)
      a.acc_out = c->acc_ffn;
      a.zero = c->acc_cross;
      a.zero_n = M * D;
      TRY(launch_proj(c, a, IN_BF16, EPI_SLICES, s));
    } else {
      a.r_out = c->r;
      a.x_res = c->x;
      TRY(launch_proj(c, a, IN_BF16, EPI_RESID, s));
    }
    TRY(mark(c, K_FC2, s));
  }
  return S2R_OK;
}

// For the lifetime of this object, an engine whose decode runs on the CUDA-core
// kernels (fused attention and out-projection, fixed-point sums) enqueues layers
// as a tensor-core engine does: LayerNorm pre-pass and tcgen05 GEMMs for every
// projection, attention rows without the fused out-projection, float32
// residual rows.  Used for prefill chunks of many rows, whose projections are
// dense GEMMs; the fixed-point accumulators of the decode path are not touched,
// and no buffer the decode path keeps across steps is written.
struct PrefillOnTensorCores {
  s2r_ctx* c;
  bool on, tc, fuse_out, fuse_ffn;
  PrefillOnTensorCores(s2r_ctx* ctx, bool enable)
      : c(ctx), on(enable), tc(ctx->tc), fuse_out(ctx->fuse_out), fuse_ffn(ctx->fuse_ffn) {
    if (!on) return;
    c->tc = true;
    c->fuse_out = false;
    c->fuse_ffn = false;
  }
  ~PrefillOnTensorCores() {
    if (!on) return;
    c->tc = tc;
    c->fuse_out = fuse_out;
    c->fuse_ffn = fuse_ffn;
  }
};

int enqueue_step(s2r_ctx* c, cudaStream_t s, const int64_t* forced, float* logits, int64_t* greedy) {
  RowMap rm{0, 0, 0, nullptr};
  c->fence_next = true;
  for (int l = 0; l < c->L; ++l) TRY(enqueue_layer(c, rm, c->B, l, false, s));
  LogitsArgs a{};
  a.M = c->B;
  a.V = c->V;
  a.D = c->D;
  a.max_tokens = c->T;
  a.st = c->st;
  a.gr = c->gr;
  a.r = c->r;
  if (c->fuse_out) {  // final_norm(x + bf16(fc2 sums + b2))
    a.r = c->x_c;
    a.acc = c->acc_ffn;
    a.acc_bias = c->layers[c->L - 1].b2;
  }
  a.gamma = c->layers[c->L - 1].ln_final_g;
  a.beta = c->layers[c->L - 1].ln_final_b;
  a.emb = c->emb_bf16;
  a.bias = c->has_bias ? c->bias : nullptr;
  a.keys = c->keys;
  a.counter = c->counter;
  a.forced = forced;
  a.logits_out = logits;
  a.greedy_out = greedy;
  a.rs = c->rs;
  a.ahead = l2_ahead_of(c, 0, kAheadQkv);  // the next step's first kernel
  if (c->tc) {
    ProjArgs p = proj_base(c);
    p.rm = rm;
    p.M = c->B;
    p.K = c->D;
    p.N = c->V;
    p.r = c->r;
    p.gamma = a.gamma;
    p.beta = a.beta;
    p.x_out = nullptr;
    p.W = c->emb_bf16;
    TRY(launch_proj_tc(c, p, IN_LN, EPI_LOGITS, s, &a));
    TRY(mark(c, K_LOGITS, s));
    return S2R_OK;
  }
  const int kch = kch_for(c->D), mc = mc_for(std::min(c->B, 8));
  LogitsFn fn = logits_fn(kch, mc);
  const size_t smem = (size_t)mc * kch * 256 * sizeof(bf16);
  CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int blocks = std::max(1, std::min((c->V + 7) / 8, 2 * c->num_sms));
  CK(launch_ex(fn, dim3(blocks), dim3(kLogitsThreads), smem, s, next_pdl(c), 0, a));
  TRY(mark(c, K_LOGITS, s));
  return S2R_OK;
}

int ensure_graph(s2r_ctx* c) {
  if (!c->graph_dirty && c->graph) return S2R_OK;
  if (c->graph) {
    cudaGraphExecDestroy(c->graph);
    c->graph = nullptr;
  }
  CK(cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_step(c, c->cap_stream, nullptr, nullptr, nullptr);
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(c->cap_stream, &graph);
  if (rc != S2R_OK) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return fail(S2R_ECUDA, "graph capture: %s", cudaGetErrorString(e));
  e = cudaGraphInstantiate(&c->graph, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return fail(S2R_ECUDA, "graph instantiate: %s", cudaGetErrorString(e));
  c->graph_dirty = false;
  return S2R_OK;
}

void release_pages(s2r_ctx* c, int slot) {
  for (int p : c->slot_pages[slot]) c->free_pages.push_back(p);
  c->slot_pages[slot].clear();
}

// Give `slot` pages for positions 0..last; returns S2R_ENOMEM if the pool is empty.
int grow_pages(s2r_ctx* c, int slot, int last, bool* changed) {
  const int need = last / kPageTokens + 1;
  while ((int)c->slot_pages[slot].size() < need) {
    if (c->free_pages.empty()) return fail(S2R_ENOMEM, "K/V page pool exhausted (%d pages)", c->n_pages);
    const int p = c->free_pages.back();
    c->free_pages.pop_back();
    c->h_page_table[(size_t)slot * c->pps + c->slot_pages[slot].size()] = p;
    c->slot_pages[slot].push_back(p);
    *changed = true;
  }
  return S2R_OK;
}

int upload_page_row(s2r_ctx* c, int slot, cudaStream_t s) {
  CK(cudaMemcpyAsync(c->st.page_table + (size_t)slot * c->pps, c->h_page_table.data() + (size_t)slot * c->pps,
                     c->pps * sizeof(int32_t), cudaMemcpyHostToDevice, s));
  return S2R_OK;
}

void replay_class(const s2r_ctx* c, HostGrammarState& st, int64_t tok) {
  const int kind = c->h_token_class[tok];
  const bool is_shift = kind == kShiftT, is_field = kind != kShiftT && kind != kEosT;
  const bool new_event = is_shift && !st.in_shift && st.payload > 0;
  int64_t payload = new_event ? 0 : st.payload;
  if (is_field) payload += 1;
  int64_t last = new_event ? -1 : st.last_field;
  if (is_field) last = c->h_field[kind];
  int64_t inc = new_event ? kNone : st.incomplete;
  if (is_field) inc = kind == kMeterT ? kAfterMeter : kind == kPitchT ? kAfterPitch : kind == kBassT ? kAfterBass : kNone;
  const uint8_t in_shift = is_shift ? 1 : (is_field ? 0 : st.in_shift);
  const int64_t run = is_shift ? st.shift_run + 1 : (is_field ? 0 : st.shift_run);
  const bool eos = kind == kEosT;
  const bool stopped = kind == kTimeT && c->h_time[tok] >= INFINITY;  // prefixes replay with stop = +inf
  st.payload = payload;
  st.last_field = last;
  st.incomplete = inc;
  st.in_shift = in_shift;
  st.shift_run = run;
  if (eos || stopped) {
    st.ended = eos ? 1 : 2;
    st.finished = 1;
  }
}

// Tensor-core projection buffers.  The step and prefill projections and the
// logits run on tensor cores when the engine has kTcMinBatch or more slots
// (fewer rows are faster on the CUDA-core kernels, which stream the weights
// once at full width); the cross K/V projection at load always does.
// S2R_FLAG_NO_TENSOR_CORE keeps every projection on the CUDA-core kernels.
int setup_tensor_core(s2r_ctx* c) {
  const bool allowed = !(c->cfg.flags & S2R_FLAG_NO_TENSOR_CORE);
  if (allowed && !tensor_map_encoder()) return fail(S2R_ECUDA, "the driver has no cuTensorMapEncodeTiled");
  c->tc_cross = allowed;
  c->tc = allowed && c->B >= kTcMinBatch && c->D >= kTcBlockN;
  c->tc_prefill = allowed && !c->tc && c->D >= kTcBlockN;
  c->tc_nb = c->B <= 64 ? 64 : c->B <= 128 ? 128 : 256;  // prefill chunks of more rows take several row tiles
  if (!allowed) return S2R_OK;
  if (c->tc || c->tc_prefill) {
    TRY(dalloc(c, &c->xln, (size_t)c->maxM * kch_for(c->D) * 256));
    CK(cudaMemset(c->xln, 0, (size_t)c->maxM * kch_for(c->D) * 256 * sizeof(bf16)));
  }
  TRY(dalloc(c, &c->mem_bf16, (size_t)c->F * c->D));
  return S2R_OK;
}

// Read (and clear) the device error word after the stream's work has finished.
int check_device_error(s2r_ctx* c, cudaStream_t s) {
  int err = 0;
  CK(cudaMemcpyAsync(&err, c->dev_error, sizeof(int), cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if (err == 0) return S2R_OK;
  CK(cudaMemsetAsync(c->dev_error, 0, sizeof(int), s));
  CK(cudaMemsetAsync(c->counter, 0, sizeof(unsigned), s));
  CK(cudaMemsetAsync(c->keys, 0, (size_t)c->B * kKeyStride * sizeof(unsigned long long), s));
  if (c->acc_self) CK(cudaMemsetAsync(c->acc_self, 0, (size_t)c->maxM * c->D * sizeof(unsigned long long), s));
  if (c->acc_cross) CK(cudaMemsetAsync(c->acc_cross, 0, (size_t)c->maxM * c->D * sizeof(unsigned long long), s));
  if (c->acc_ffn) CK(cudaMemsetAsync(c->acc_ffn, 0, (size_t)c->maxM * c->D * sizeof(unsigned long long), s));
  return fail(S2R_EDEVICE, "a kernel reported error %d (%s); its work was skipped", err,
              err == kErrAttnCluster ? "attention launched without its cluster shape"
              : err == kErrAttnChunk ? "attention keys exceed the score buffer"
              : err == kErrAttnStage ? "a bulk copy of the attention kernel did not complete in time"
              : err == kErrAttnExchange ? "a value sent between attention CTAs did not arrive in time"
              : err == kErrGemmWait  ? "a wait of the tensor-core projection timed out"
              : err == kErrPrefillWait ? "a wait of the prefill attention timed out"
              : err == kErrFfnStage  ? "a bulk copy of the fused FFN did not complete in time"
              : err == kErrAccRange  ? "an out-projection partial was too large (or NaN) for the fixed-point sum"
                                     : "unknown code");
}

template <typename T>
int put(T* dev, int slot, T value, cudaStream_t s) {
  CK(cudaMemcpyAsync(dev + slot, &value, sizeof(T), cudaMemcpyHostToDevice, s));
  return S2R_OK;
}

}  // namespace

__attribute__((visibility("hidden"))) int s2r_record_error(int code, const char* msg) {
  return fail(code, "%s", msg);
}

extern "C" {

int32_t s2r_abi_version(void) { return S2R_ABI_VERSION; }

const char* s2r_last_error(void) { return g_last_error.c_str(); }

int32_t s2r_create(const s2r_config* cfg, const s2r_weights* w, const s2r_grammar* g, int32_t device, s2r_ctx** out) {
  if (!cfg || !w || !g || !out) return fail(S2R_EINVAL, "s2r_create: NULL argument");
  *out = nullptr;
  const s2r_config k = *cfg;
  if (k.width <= 0 || k.heads <= 0 || k.width != k.heads * kHeadDim)
    return fail(S2R_ENOTSUP, "width must be heads * 64 (width %d, heads %d)", k.width, k.heads);
  if (k.width % 64 || k.width > 4096 || k.ffn_width <= 0 || k.ffn_width % 64 || k.ffn_width > 4096)
    return fail(S2R_ENOTSUP, "width and ffn_width must be multiples of 64 up to 4096");
  if (k.layers <= 0 || k.vocab_size <= 4 || k.max_tokens < 2 || k.batch <= 0 || k.frames <= 0)
    return fail(S2R_EINVAL, "invalid sizes (layers %d vocab %d max_tokens %d batch %d frames %d)", k.layers,
                k.vocab_size, k.max_tokens, k.batch, k.frames);
  if (g->kind != S2R_GRAMMAR_CLASS && g->kind != S2R_GRAMMAR_TABLE) return fail(S2R_EINVAL, "unknown grammar kind");
  if (g->kind == S2R_GRAMMAR_CLASS && (!g->token_class || !g->field_of_class || !g->time_seconds))
    return fail(S2R_EINVAL, "class grammar needs token_class, field_of_class and time_seconds");
  if (g->kind == S2R_GRAMMAR_TABLE && (!g->table || g->states <= 0))
    return fail(S2R_EINVAL, "table grammar needs a table and states > 0");
  if (!w->layers) return fail(S2R_EINVAL, "weights.layers is NULL");
  if ((uint32_t)k.flags & ~(S2R_FLAG_NO_PDL | S2R_FLAG_NO_GRAPH | S2R_FLAG_NO_TENSOR_CORE))
    return fail(S2R_EINVAL, "unknown flag bits 0x%x", (unsigned)k.flags);

  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(S2R_EINVAL, "device %d out of range (%d devices)", device, ndev);
  CK(cudaSetDevice(device));

  s2r_ctx* c = new s2r_ctx();
  c->cfg = k;
  c->device = device;
  c->D = k.width;
  c->H = k.heads;
  c->F = k.frames;
  c->FFN = k.ffn_width;
  c->V = k.vocab_size;
  c->L = k.layers;
  c->B = k.batch;
  c->T = k.max_tokens;
  c->maxM = std::max(k.batch, kPrefillRows);
  c->pps = (k.max_tokens + kPageTokens - 1) / kPageTokens;
  c->n_pages = k.kv_pages > 0 ? k.kv_pages : k.batch * c->pps;
  c->pdl = !(k.flags & S2R_FLAG_NO_PDL);
  c->use_graph = !(k.flags & S2R_FLAG_NO_GRAPH);
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&c->smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device);
  auto cleanup = [&](int rc) {
    s2r_destroy(c);
    return rc;
  };
#define TRYC(x)                    \
  do {                             \
    int rc_ = (x);                 \
    if (rc_ != S2R_OK) return cleanup(rc_); \
  } while (0)
#define CKC(call)                                                                                    \
  do {                                                                                               \
    cudaError_t err_ = (call);                                                                       \
    if (err_ != cudaSuccess)                                                                         \
      return cleanup(fail(S2R_ECUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(err_), __FILE__, __LINE__)); \
  } while (0)

  const size_t D = c->D, V = c->V, FFN = c->FFN, T = c->T;
  // weights
  TRYC(dalloc(c, &c->tok_emb, V * D));
  TRYC(dalloc(c, &c->pos_emb, (T + 2) * D));
  TRYC(dalloc(c, &c->emb_ln_g, D));
  TRYC(dalloc(c, &c->emb_ln_b, D));
  TRYC(dalloc(c, &c->emb_bf16, V * D));
  float* stage = nullptr;
  TRYC(dalloc(c, &stage, std::max(V * D, std::max(3 * D * D, FFN * D))));
  TRYC(upload_f32(c->tok_emb, w->token_embedding, V * D));
  TRYC(upload_f32(c->pos_emb, w->position_embedding, (T + 2) * D));
  TRYC(upload_f32(c->emb_ln_g, w->embedding_norm_w, D));
  TRYC(upload_f32(c->emb_ln_b, w->embedding_norm_b, D));
  TRYC(upload_bf16(c, c->emb_bf16, w->token_embedding, V * D, stage));
  c->layers.resize(c->L);
  // the cross key/value weights of every layer, stacked [L * 2D, D], so that one
  // launch projects a window for all layers
  TRYC(dalloc(c, &c->wckv_all, (size_t)c->L * 2 * D * D));
  const size_t pool = (size_t)c->n_pages * c->H * kPageTokens * kHeadDim;
  const size_t cross = (size_t)c->B * c->H * c->F * kHeadDim;
  for (int l = 0; l < c->L; ++l) {
    const s2r_layer_weights& lw = w->layers[l];
    LayerBufs& b = c->layers[l];
    TRYC(dalloc(c, &b.wqkv, 3 * D * D));
    TRYC(dalloc(c, &b.bqkv, 3 * D));
    TRYC(dalloc(c, &b.wo, D * D));
    TRYC(dalloc(c, &b.bo, D));
    TRYC(dalloc(c, &b.wcq, D * D));
    TRYC(dalloc(c, &b.bcq, D));
    b.wckv = c->wckv_all + (size_t)l * 2 * D * D;
    TRYC(dalloc(c, &b.bckv, 2 * D));
    TRYC(dalloc(c, &b.wco, D * D));
    TRYC(dalloc(c, &b.bco, D));
    TRYC(dalloc(c, &b.w1, FFN * D));
    TRYC(dalloc(c, &b.b1, FFN));
    TRYC(dalloc(c, &b.w2, D * FFN));
    TRYC(dalloc(c, &b.b2, D));
    TRYC(dalloc(c, &b.ln_self_g, D));
    TRYC(dalloc(c, &b.ln_self_b, D));
    TRYC(dalloc(c, &b.ln_cross_g, D));
    TRYC(dalloc(c, &b.ln_cross_b, D));
    TRYC(dalloc(c, &b.ln_final_g, D));
    TRYC(dalloc(c, &b.ln_final_b, D));
    TRYC(dalloc(c, &b.kpool, pool));
    TRYC(dalloc(c, &b.vpool, pool));
    TRYC(dalloc(c, &b.ck, cross));
    TRYC(dalloc(c, &b.cv, cross));
    TRYC(upload_bf16(c, b.wqkv, lw.self_q_w, D * D, stage));
    TRYC(upload_bf16(c, b.wqkv + D * D, lw.self_k_w, D * D, stage));
    TRYC(upload_bf16(c, b.wqkv + 2 * D * D, lw.self_v_w, D * D, stage));
    TRYC(upload_bf16(c, b.bqkv, lw.self_q_b, D, stage));
    TRYC(upload_bf16(c, b.bqkv + D, lw.self_k_b, D, stage));
    TRYC(upload_bf16(c, b.bqkv + 2 * D, lw.self_v_b, D, stage));
    TRYC(upload_bf16(c, b.wo, lw.self_out_w, D * D, stage));
    TRYC(upload_bf16(c, b.bo, lw.self_out_b, D, stage));
    TRYC(upload_bf16(c, b.wcq, lw.cross_q_w, D * D, stage));
    TRYC(upload_bf16(c, b.bcq, lw.cross_q_b, D, stage));
    TRYC(upload_bf16(c, b.wckv, lw.cross_k_w, D * D, stage));
    TRYC(upload_bf16(c, b.wckv + D * D, lw.cross_v_w, D * D, stage));
    TRYC(upload_bf16(c, b.bckv, lw.cross_k_b, D, stage));
    TRYC(upload_bf16(c, b.bckv + D, lw.cross_v_b, D, stage));
    TRYC(upload_bf16(c, b.wco, lw.cross_out_w, D * D, stage));
    TRYC(upload_bf16(c, b.bco, lw.cross_out_b, D, stage));
    TRYC(upload_bf16(c, b.w1, lw.fc1_w, FFN * D, stage));
    TRYC(upload_bf16(c, b.b1, lw.fc1_b, FFN, stage));
    TRYC(upload_bf16(c, b.w2, lw.fc2_w, D * FFN, stage));
    TRYC(upload_bf16(c, b.b2, lw.fc2_b, D, stage));
    TRYC(upload_f32(b.ln_self_g, lw.self_norm_w, D));
    TRYC(upload_f32(b.ln_self_b, lw.self_norm_b, D));
    TRYC(upload_f32(b.ln_cross_g, lw.cross_norm_w, D));
    TRYC(upload_f32(b.ln_cross_b, lw.cross_norm_b, D));
    TRYC(upload_f32(b.ln_final_g, lw.final_norm_w, D));
    TRYC(upload_f32(b.ln_final_b, lw.final_norm_b, D));
    CKC(cudaMemset(b.kpool, 0, pool * sizeof(bf16)));
    CKC(cudaMemset(b.vpool, 0, pool * sizeof(bf16)));
    CKC(cudaMemset(b.ck, 0, cross * sizeof(bf16)));
    CKC(cudaMemset(b.cv, 0, cross * sizeof(bf16)));
  }
  // activations
  const size_t M = c->maxM;
  TRYC(dalloc(c, &c->r, M * D));
  TRYC(dalloc(c, &c->x, M * D));
  TRYC(dalloc(c, &c->q, M * D));
  TRYC(dalloc(c, &c->att, M * D));
  TRYC(dalloc(c, &c->hid, M * FFN));
  float* mem_stage = nullptr;
  TRYC(dalloc(c, &mem_stage, (size_t)c->F * D));
  c->mem_stage = mem_stage;
  TRYC(dalloc(c, &c->prefill_tokens, kPrefillRows));
  TRYC(setup_tensor_core(c));
  c->fuse_out = !c->tc;
  c->fuse_ffn = c->fuse_out && c->B == 1 && c->D <= 1024 && c->FFN % kFfnSlice == 0 &&
                ffn_smem_bytes(c->D) + 4096 <= (size_t)227 * 1024;
  if (c->fuse_ffn) {
    for (int l = 0; l < c->L; ++l) {
      LayerBufs& b = c->layers[l];
      TRYC(dalloc(c, &b.w2s, FFN * D));
      slice_major_kernel<<<1024, 256>>>(b.w2, b.w2s, (int)D, (int)FFN);
      CKC(cudaGetLastError());
    }
  }
  if (c->fuse_out) {
    TRYC(dalloc(c, &c->acc_self, (size_t)c->maxM * D));
    TRYC(dalloc(c, &c->acc_cross, (size_t)c->maxM * D));
    TRYC(dalloc(c, &c->x_b, (size_t)c->maxM * D));
    TRYC(dalloc(c, &c->x_c, (size_t)c->maxM * D));
    TRYC(dalloc(c, &c->acc_ffn, (size_t)c->maxM * D));
    CKC(cudaMemset(c->x_c, 0, (size_t)c->maxM * D * sizeof(float)));
    CKC(cudaMemset(c->acc_ffn, 0, (size_t)c->maxM * D * sizeof(unsigned long long)));
    CKC(cudaMemset(c->acc_self, 0, (size_t)c->maxM * D * sizeof(unsigned long long)));
    CKC(cudaMemset(c->acc_cross, 0, (size_t)c->maxM * D * sizeof(unsigned long long)));
    CKC(cudaMemset(c->x_b, 0, (size_t)c->maxM * D * sizeof(float)));
  }
  c->attn_splits = attn_splits_for(c, 4);
  c->attn_splits_cross = attn_splits_for(c, 8);
  if (!c->tc && c->H * kAttnWideSplits <= c->num_sms) TRYC(widen_cross_splits(c));
  c->h_frames.assign(c->B, 0);
  if (c->tc) {
    TRYC(dalloc(c, &c->order_self, c->B));
    TRYC(dalloc(c, &c->order_cross, c->B));
    CKC(cudaMallocHost(&c->h_order, 2 * (size_t)c->B * sizeof(int32_t)));
    CKC(cudaEventCreateWithFlags(&c->order_copied, cudaEventDisableTiming));
    std::vector<int32_t> ident(c->B);
    for (int i = 0; i < c->B; ++i) ident[i] = i;
    CKC(cudaMemcpy(c->order_self, ident.data(), c->B * sizeof(int32_t), cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(c->order_cross, ident.data(), c->B * sizeof(int32_t), cudaMemcpyHostToDevice));
  }
  TRYC(dalloc(c, &c->keys, (size_t)c->B * kKeyStride));
  TRYC(dalloc(c, &c->counter, 1));
  TRYC(dalloc(c, &c->dev_error, 1));
  CKC(cudaMemset(c->dev_error, 0, sizeof(int)));
  TRYC(dalloc(c, &c->bias, V));
  TRYC(dalloc(c, &c->dbg_forced, c->B));
  TRYC(dalloc(c, &c->dbg_logits, (size_t)c->B * V));
  TRYC(dalloc(c, &c->dbg_greedy, c->B));
  CKC(cudaMemset(c->keys, 0, (size_t)c->B * kKeyStride * sizeof(unsigned long long)));
  CKC(cudaMemset(c->counter, 0, sizeof(unsigned int)));
  CKC(cudaMemset(c->bias, 0, V * sizeof(float)));
  CKC(cudaMemset(c->r, 0, M * D * sizeof(float)));
  CKC(cudaMemset(c->x, 0, M * D * sizeof(float)));
  // slot state (engine.py:138-146, grammar.py:99-112): every slot starts finished
  SlotState& st = c->st;
  const size_t B = c->B;
  TRYC(dalloc(c, &st.token, B));
  TRYC(dalloc(c, &st.position, B));
  TRYC(dalloc(c, &st.finished, B));
  TRYC(dalloc(c, &st.ended, B));
  TRYC(dalloc(c, &st.in_shift, B));
  TRYC(dalloc(c, &st.shift_run, B));
  TRYC(dalloc(c, &st.payload, B));
  TRYC(dalloc(c, &st.last_field, B));
  TRYC(dalloc(c, &st.incomplete, B));
  TRYC(dalloc(c, &st.g, B));
  TRYC(dalloc(c, &st.count, B));
  TRYC(dalloc(c, &st.target, B));
  TRYC(dalloc(c, &st.stop, B));
  TRYC(dalloc(c, &st.out, B * T));
  TRYC(dalloc(c, &st.frames, B));
  TRYC(dalloc(c, &st.page_table, B * c->pps));
  {
    std::vector<int64_t> eos(B, 2), zeros(B, 0), minus(B, -1), none(B, INT64_MAX);
    std::vector<uint8_t> ones(B, 1);
    std::vector<double> inf(B, INFINITY);
    std::vector<int32_t> frames(B, c->F);
    CKC(cudaMemcpy(st.token, eos.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.position, zeros.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.finished, ones.data(), B, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.ended, zeros.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.in_shift, ones.data(), B, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.shift_run, zeros.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.payload, zeros.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.last_field, minus.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.incomplete, zeros.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.g, zeros.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.count, zeros.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.target, none.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(st.stop, inf.data(), B * 8, cudaMemcpyHostToDevice));
    CKC(cudaMemset(st.out, 0, B * T * 8));
    CKC(cudaMemcpy(st.frames, frames.data(), B * 4, cudaMemcpyHostToDevice));
  }
  c->h_page_table.assign(B * c->pps, 0);
  CKC(cudaMemset(st.page_table, 0, B * c->pps * sizeof(int32_t)));
  for (int p = c->n_pages - 1; p >= 0; --p) c->free_pages.push_back(p);
  c->slot_pages.assign(B, {});
  c->loaded.assign(B, 0);
  c->bound.assign(B, 0);
  // grammar
  Grammar& gr = c->gr;
  gr.kind = g->kind;
  if (g->kind == S2R_GRAMMAR_CLASS) {
    c->h_token_class.resize(V);
    c->h_field.resize(13);
    c->h_time.resize(V);
    CKC(cudaMemcpy(c->h_token_class.data(), g->token_class, V, cudaMemcpyDefault));
    CKC(cudaMemcpy(c->h_field.data(), g->field_of_class, 13 * 4, cudaMemcpyDefault));
    CKC(cudaMemcpy(c->h_time.data(), g->time_seconds, V * 8, cudaMemcpyDefault));
    for (size_t v = 0; v < V; ++v)
      if (c->h_token_class[v] < 0 || c->h_token_class[v] > 12) {
        return cleanup(fail(S2R_EINVAL, "token_class[%zu] = %d is not a class 0..12", v, c->h_token_class[v]));
      }
    int8_t* tc = nullptr;
    int32_t* fc = nullptr;
    double* ts = nullptr;
    TRYC(dalloc(c, &tc, V));
    TRYC(dalloc(c, &fc, 13));
    TRYC(dalloc(c, &ts, V));
    CKC(cudaMemcpy(tc, c->h_token_class.data(), V, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(fc, c->h_field.data(), 13 * 4, cudaMemcpyHostToDevice));
    CKC(cudaMemcpy(ts, c->h_time.data(), V * 8, cudaMemcpyHostToDevice));
    gr.token_class = tc;
    gr.field_of_class = fc;
    gr.time_seconds = ts;
  } else {
    uint8_t* tb = nullptr;
    TRYC(dalloc(c, &tb, (size_t)g->states * V));
    CKC(cudaMemcpy(tb, g->table, (size_t)g->states * V, cudaMemcpyDefault));
    gr.table = tb;
    gr.states = g->states;
    gr.multiplier = g->multiplier;
  }
  CKC(cudaStreamCreateWithFlags(&c->cap_stream, cudaStreamNonBlocking));
  CKC(cudaDeviceSynchronize());
  *out = c;
  return S2R_OK;
#undef TRYC
#undef CKC
}

int32_t s2r_destroy(s2r_ctx* c) {
  if (!c) return S2R_OK;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  if (c->graph) cudaGraphExecDestroy(c->graph);
  if (c->cap_stream) cudaStreamDestroy(c->cap_stream);
  if (c->order_copied) cudaEventDestroy(c->order_copied);
  if (c->h_order) cudaFreeHost(c->h_order);
  if (c->poll_ev) cudaEventDestroy(c->poll_ev);
  for (cudaEvent_t e : c->take_ev) cudaEventDestroy(e);
  if (c->h_fin) cudaFreeHost(c->h_fin);
  if (c->h_err) cudaFreeHost(c->h_err);
  if (c->h_out) cudaFreeHost(c->h_out);
  if (c->h_pos_end) cudaFreeHost(c->h_pos_end);
  for (void* p : c->allocs) cudaFree(p);
  delete c;
  return S2R_OK;
}

int32_t s2r_set_logit_bias(s2r_ctx* c, const float* bias) {
  if (!c) return fail(S2R_EINVAL, "NULL engine");
  CK(cudaSetDevice(c->device));
  CK(cudaDeviceSynchronize());
  if (bias) {
    CK(cudaMemcpy(c->bias, bias, (size_t)c->V * sizeof(float), cudaMemcpyDefault));
  } else {
    CK(cudaMemset(c->bias, 0, (size_t)c->V * sizeof(float)));
  }
  if (c->has_bias != (bias != nullptr)) c->graph_dirty = true;
  c->has_bias = bias != nullptr;
  return S2R_OK;
}

int32_t s2r_set_rescore(s2r_ctx* c, const s2r_rescore* in) {
  if (!c) return fail(S2R_EINVAL, "NULL engine");
  CK(cudaSetDevice(c->device));
  CK(cudaDeviceSynchronize());
  bool on = false;
  if (in)
    for (int t = 0; t < S2R_FRAME_TERMS; ++t) on = on || in->weight[t] != 0.f;
  c->graph_dirty = true;
  if (!on) {
    c->rs.on = 0;
    return S2R_OK;
  }
  if (c->gr.kind != S2R_GRAMMAR_CLASS) return fail(S2R_ENOTSUP, "frame-head rescoring needs the class grammar");
  const int32_t* spans[5] = {in->bass_span, in->detail_span, in->key_span, in->eighth_span, in->meter_span};
  for (const int32_t* sp : spans)
    if (sp[0] < 0 || sp[1] <= sp[0] || sp[1] > c->V) return fail(S2R_EINVAL, "rescoring span [%d, %d) outside the vocabulary", sp[0], sp[1]);
  if (in->bass_span[1] - in->bass_span[0] != 12 || in->key_span[1] - in->key_span[0] != 24)
    return fail(S2R_EINVAL, "rescoring: the bass span must hold 12 tokens and the key span 24");
  if (!in->meter_beats || !in->meter_unit || in->time_hz <= 0) return fail(S2R_EINVAL, "rescoring: meter tables and time_hz needed");
  const int n_meters = in->meter_span[1] - in->meter_span[0];
  for (int i = 0; i < n_meters; ++i)
    if (in->meter_beats[i] < 0 || in->meter_beats[i] > 15) return fail(S2R_EINVAL, "meter_beats[%d] = %d not in [0, 15]", i, in->meter_beats[i]);
  Rescore& r = c->rs;
  const int no_chord = in->detail_span[1] - in->detail_span[0];
  if (r.frame_now && no_chord != r.d1 - r.d0) return fail(S2R_EINVAL, "rescoring: the detail span width cannot change");
  if (r.frame_now && n_meters > c->rs_meters)
    return fail(S2R_EINVAL, "rescoring: the meter span grew from %d to %d tokens", c->rs_meters, n_meters);
  if (!r.frame_now) {  // first call: tables and state
    for (int t = 0; t < FT_COUNT; ++t) {
      float* tab = nullptr;
      const size_t n = (size_t)c->B * c->F * frame_term_width(t, no_chord);
      TRY(dalloc(c, &tab, n));
      CK(cudaMemset(tab, 0, n * sizeof(float)));
      r.table[t] = tab;
    }
    int32_t *beats = nullptr, *unit = nullptr;
    TRY(dalloc(c, &beats, n_meters));
    TRY(dalloc(c, &unit, n_meters));
    r.meter_beats = beats;
    r.meter_unit = unit;
    c->rs_meters = n_meters;
    TRY(dalloc(c, &r.frame_now, c->B));
    TRY(dalloc(c, &r.key_seen, c->B));
    TRY(dalloc(c, &r.active_meter, c->B));
    TRY(dalloc(c, &r.meter_changed, c->B));
    CK(cudaMemset(r.frame_now, 0, c->B * sizeof(int32_t)));
    CK(cudaMemset(r.key_seen, 0, c->B));
    CK(cudaMemset(r.active_meter, 0xff, c->B * sizeof(int32_t)));  // -1: no meter stated
    CK(cudaMemset(r.meter_changed, 0, c->B));
  }
  CK(cudaMemcpy(const_cast<int32_t*>(r.meter_beats), in->meter_beats, n_meters * sizeof(int32_t), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(const_cast<int32_t*>(r.meter_unit), in->meter_unit, n_meters * sizeof(int32_t), cudaMemcpyHostToDevice));
  for (int t = 0; t < FT_COUNT; ++t) r.w[t] = in->weight[t];
  r.b0 = in->bass_span[0], r.b1 = in->bass_span[1];
  r.d0 = in->detail_span[0], r.d1 = in->detail_span[1];
  r.k0 = in->key_span[0], r.k1 = in->key_span[1];
  r.e0 = in->eighth_span[0], r.e1 = in->eighth_span[1];
  r.m0 = in->meter_span[0], r.m1 = in->meter_span[1];
  r.frames = c->F;
  c->rs_time_hz = in->time_hz;
  r.on = 1;
  return S2R_OK;
}

int32_t s2r_load_frame_tables(s2r_ctx* c, int32_t slot, const float* const* tables, const int32_t* rows, void* stream) {
  if (!c) return fail(S2R_EINVAL, "NULL engine");
  if (!c->rs.on) return fail(S2R_ESTATE, "frame-head rescoring is not enabled (s2r_set_rescore)");
  if (slot < 0 || slot >= c->B) return fail(S2R_EINVAL, "slot %d out of range [0, %d)", slot, c->B);
  CK(cudaSetDevice(c->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int no_chord = c->rs.d1 - c->rs.d0;
  for (int t = 0; t < FT_COUNT; ++t) {
    const size_t width = frame_term_width(t, no_chord);
    float* dst = const_cast<float*>(c->rs.table[t]) + (size_t)slot * c->F * width;
    CK(cudaMemsetAsync(dst, 0, (size_t)c->F * width * sizeof(float), s));
    const int n = (tables && rows && tables[t]) ? std::min<int>(std::max(rows[t], 0), c->F) : 0;
    if (n > 0) CK(cudaMemcpyAsync(dst, tables[t], (size_t)n * width * sizeof(float), cudaMemcpyDefault, s));
  }
  return S2R_OK;
}

int32_t s2r_load_slot(s2r_ctx* c, int32_t slot, const void* memory, int32_t memory_dtype, int32_t memory_frames,
                      int32_t frames, const int64_t* prefix, int32_t n_prefix, double stop_seconds, int64_t target,
                      void* stream) {
  if (!c) return fail(S2R_EINVAL, "NULL engine");
  if (slot < 0 || slot >= c->B) return fail(S2R_EINVAL, "slot %d out of range [0, %d)", slot, c->B);
  if (!memory || (memory_dtype != S2R_F32 && memory_dtype != S2R_BF16)) return fail(S2R_EINVAL, "bad memory argument");
  if (frames < 1 || frames > memory_frames || frames > c->F)
    return fail(S2R_EINVAL, "frames %d must be in [1, min(memory_frames %d, engine frames %d)]", frames, memory_frames, c->F);
  if (!prefix || n_prefix < 1) return fail(S2R_EINVAL, "empty prefix");
  if (n_prefix > c->T - 1)
    return fail(S2R_EINVAL, "prefix of %d tokens does not fit the context of %d", n_prefix, c->T);
  int out_index = -1;
  for (int i = 0; i < n_prefix; ++i) {
    if (prefix[i] < 0 || prefix[i] >= c->V) return fail(S2R_EINVAL, "prefix token %lld outside the vocabulary", (long long)prefix[i]);
    if (out_index < 0 && prefix[i] == 3) out_index = i;
  }
  if (out_index < 0) return fail(S2R_EINVAL, "prefix has no <out> token (3)");
  CK(cudaSetDevice(c->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int D = c->D;

  // grammar state after the prefix (grammar.py:182-197)
  HostGrammarState gs;
  for (int i = out_index + 1; i < n_prefix; ++i) {
    if (c->gr.kind == S2R_GRAMMAR_TABLE)
      gs.g = (c->gr.multiplier * gs.g + prefix[i]) % c->gr.states;
    else
      replay_class(c, gs, prefix[i]);
  }
  // pages for positions 0 .. n-1
  release_pages(c, slot);
  std::fill(c->h_page_table.begin() + (size_t)slot * c->pps, c->h_page_table.begin() + (size_t)(slot + 1) * c->pps, 0);
  bool changed = false;
  TRY(grow_pages(c, slot, n_prefix - 1, &changed));
  TRY(upload_page_row(c, slot, s));

  SlotState& st = c->st;
  TRY(put<int32_t>(st.frames, slot, frames, s));
  c->h_frames[slot] = frames;
  TRY(put<double>(st.stop, slot, stop_seconds, s));
  TRY(put<int64_t>(st.target, slot, target, s));
  TRY(put<int64_t>(st.g, slot, gs.g, s));
  TRY(put<int64_t>(st.count, slot, 0, s));
  TRY(put<uint8_t>(st.in_shift, slot, gs.in_shift, s));
  TRY(put<int64_t>(st.shift_run, slot, gs.shift_run, s));
  TRY(put<int64_t>(st.payload, slot, gs.payload, s));
  TRY(put<int64_t>(st.last_field, slot, gs.last_field, s));
  TRY(put<int64_t>(st.incomplete, slot, gs.incomplete, s));
  TRY(put<int64_t>(st.ended, slot, gs.ended, s));
  TRY(put<uint8_t>(st.finished, slot, gs.finished, s));
  TRY(put<int64_t>(st.token, slot, prefix[n_prefix - 1], s));
  TRY(put<int64_t>(st.position, slot, (int64_t)n_prefix - 1, s));
  CK(cudaMemcpyAsync(st.out + (size_t)slot * c->T, prefix, n_prefix * sizeof(int64_t), cudaMemcpyDefault, s));

  if (c->rs.on) {  // rescoring state after the prefix (engine.py:225-232)
    const Rescore& r = c->rs;
    int32_t frame_now = 0, active = -1;
    uint8_t key_seen = 0;
    for (int i = 0; i < n_prefix; ++i) {
      const int64_t t = prefix[i];
      const double sec = c->h_time[(size_t)t];
      if (sec > -INFINITY) {
        const long long f = (long long)(sec * c->rs_time_hz) * 25 / c->rs_time_hz;
        frame_now = (int32_t)std::min<long long>(f, c->F - 1);
      }
      if (t >= r.k0 && t < r.k1) key_seen = 1;
      if (t >= r.m0 && t < r.m1) active = (int32_t)(t - r.m0);
    }
    TRY(put<int32_t>(r.frame_now, slot, frame_now, s));
    TRY(put<uint8_t>(r.key_seen, slot, key_seen, s));
    TRY(put<int32_t>(r.active_meter, slot, active, s));
    TRY(put<uint8_t>(r.meter_changed, slot, (uint8_t)0, s));
  }
  // cross K/V of the window (decoder.py:98-116), written straight into the slot
  const size_t elem = memory_dtype == S2R_F32 ? 4 : 2;
  CK(cudaMemcpyAsync(c->mem_stage, memory, (size_t)frames * D * elem, cudaMemcpyDefault, s));
  if (c->tc_cross) {
    const bf16* x = static_cast<const bf16*>(c->mem_stage);
    if (memory_dtype == S2R_F32) {
      const size_t n = (size_t)frames * D;
      f32_to_bf16_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 4 * (size_t)c->num_sms), 256, 0, s>>>(
          static_cast<const float*>(c->mem_stage), c->mem_bf16, n);
      CK(cudaGetLastError());
      x = c->mem_bf16;
    }
    TRY(launch_crosskv(c, x, frames, slot, s));
  }
  for (int l = 0; l < c->L && !c->tc_cross; ++l) {
    ProjArgs a = proj_base(c);
    a.M = frames;
    a.K = D;
    a.N = 2 * D;
    a.xin = c->mem_stage;
    a.ldx = D;
    a.W = c->layers[l].wckv;
    a.bias = c->layers[l].bckv;
    a.k_dst = c->layers[l].ck;
    a.v_dst = c->layers[l].cv;
    a.cross_slot = slot;
    TRY(launch_proj(c, a, memory_dtype == S2R_F32 ? IN_F32 : IN_BF16, EPI_CROSSKV, s));
  }
  // prefix prefill: K/V of prefix[0 .. n-2] at positions 0 .. n-2 (engine.py:199-205)
  std::vector<int32_t> toks(kPrefillRows);
  for (int p0 = 0; p0 < n_prefix - 1; p0 += kPrefillRows) {
    const int rows = std::min(kPrefillRows, n_prefix - 1 - p0);
    for (int i = 0; i < rows; ++i) toks[i] = (int32_t)prefix[p0 + i];
    int32_t* dst = c->prefill_tokens;
    CK(cudaMemcpyAsync(dst, toks.data(), rows * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    RowMap rm{1, slot, p0, dst};
    c->fence_next = true;
    PrefillOnTensorCores mode(c, c->tc_prefill && rows > kFusedPrefillMaxRows);
    for (int l = 0; l < c->L; ++l) TRY(enqueue_layer(c, rm, rows, l, l == c->L - 1, s));
  }
  CK(cudaGetLastError());
  c->loaded[slot] = 1;
  c->bound[slot] = n_prefix - 1;
  return S2R_OK;
}

int32_t s2r_step(s2r_ctx* c, int32_t n_steps, void* stream) {
  if (!c) return fail(S2R_EINVAL, "NULL engine");
  if (n_steps <= 0) return S2R_OK;
  CK(cudaSetDevice(c->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int slot = 0; slot < c->B; ++slot) {
    if (!c->loaded[slot]) continue;
    c->bound[slot] = std::min(c->bound[slot] + n_steps, c->T - 1);
    bool changed = false;
    TRY(grow_pages(c, slot, c->bound[slot], &changed));
    if (changed) TRY(upload_page_row(c, slot, s));
  }
  TRY(upload_row_order(c, s));
  if (c->use_graph) {
    TRY(ensure_graph(c));
    for (int i = 0; i < n_steps; ++i) CK(cudaGraphLaunch(c->graph, s));
  } else {
    for (int i = 0; i < n_steps; ++i) TRY(enqueue_step(c, s, nullptr, nullptr, nullptr));
  }
  CK(cudaGetLastError());
  return S2R_OK;
}

int32_t s2r_step_debug(s2r_ctx* c, const int64_t* forced, float* logits, int64_t* greedy, void* stream) {
  if (!c) return fail(S2R_EINVAL, "NULL engine");
  CK(cudaSetDevice(c->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (forced) {
    for (int i = 0; i < c->B; ++i)
      if (forced[i] >= c->V) return fail(S2R_EINVAL, "forced token %lld outside the vocabulary", (long long)forced[i]);
    CK(cudaMemcpyAsync(c->dbg_forced, forced, c->B * sizeof(int64_t), cudaMemcpyHostToDevice, s));
  }
  for (int slot = 0; slot < c->B; ++slot) {
    if (!c->loaded[slot]) continue;
    c->bound[slot] = std::min(c->bound[slot] + 1, c->T - 1);
    bool changed = false;
    TRY(grow_pages(c, slot, c->bound[slot], &changed));
    if (changed) TRY(upload_page_row(c, slot, s));
  }
  TRY(enqueue_step(c, s, forced ? c->dbg_forced : nullptr, logits ? c->dbg_logits : nullptr,
                   greedy ? c->dbg_greedy : nullptr));
  if (logits)
    CK(cudaMemcpyAsync(logits, c->dbg_logits, (size_t)c->B * c->V * sizeof(float), cudaMemcpyDeviceToHost, s));
  if (greedy) CK(cudaMemcpyAsync(greedy, c->dbg_greedy, c->B * sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  return check_device_error(c, s);
}

int32_t s2r_poll_finished(s2r_ctx* c, uint8_t* finished, void* stream) {
  if (!c || !finished) return fail(S2R_EINVAL, "NULL argument");
  CK(cudaSetDevice(c->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaMemcpyAsync(finished, c->st.finished, c->B, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  return check_device_error(c, s);
}

int32_t s2r_take(s2r_ctx* c, int32_t slot, int64_t* tokens, int32_t capacity, int32_t* length, int32_t* ended,
                 void* stream) {
  if (!c || !length || !ended) return fail(S2R_EINVAL, "NULL argument");
  if (slot < 0 || slot >= c->B) return fail(S2R_EINVAL, "slot %d out of range [0, %d)", slot, c->B);
  if (!c->loaded[slot]) return fail(S2R_ESTATE, "slot %d is not loaded", slot);
  CK(cudaSetDevice(c->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t pos = 0, end = 0;
  CK(cudaMemcpyAsync(&pos, c->st.position + slot, 8, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(&end, c->st.ended + slot, 8, cudaMemcpyDeviceToHost, s));
  TRY(check_device_error(c, s));
  const int n = (int)pos + 1;
  std::vector<int64_t> buf(n);
  CK(cudaMemcpyAsync(buf.data(), c->st.out + (size_t)slot * c->T, n * sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if (buf.back() != 2) buf.push_back(2);  // always ends in <eos> (engine.py:259-260)
  *length = (int32_t)buf.size();
  if (!tokens || capacity < (int32_t)buf.size()) return fail(S2R_EINVAL, "capacity %d < %zu tokens", capacity, buf.size());
  std::memcpy(tokens, buf.data(), buf.size() * sizeof(int64_t));
  *ended = (int32_t)end;
  c->loaded[slot] = 0;
  release_pages(c, slot);
  return S2R_OK;
}

// Pinned host buffers and events of the asynchronous polls and takes.
static int setup_async(s2r_ctx* c) {
  if (c->h_fin) return S2R_OK;
  CK(cudaMallocHost(&c->h_fin, c->B));
  CK(cudaMallocHost(&c->h_err, sizeof(int)));
  CK(cudaMallocHost(&c->h_out, (size_t)c->B * c->T * sizeof(int64_t)));
  CK(cudaMallocHost(&c->h_pos_end, (size_t)c->B * 2 * sizeof(int64_t)));
  CK(cudaEventCreateWithFlags(&c->poll_ev, cudaEventDisableTiming));
  c->take_ev.assign(c->B, nullptr);
  for (int b = 0; b < c->B; ++b) CK(cudaEventCreateWithFlags(&c->take_ev[b], cudaEventDisableTiming));
  c->take_pending.assign(c->B, 0);
  return S2R_OK;
}

int32_t s2r_poll_finished_async(s2r_ctx* c, void* stream) {
  if (!c) return fail(S2R_EINVAL, "NULL engine");
  CK(cudaSetDevice(c->device));
  TRY(setup_async(c));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaMemcpyAsync(c->h_fin, c->st.finished, c->B, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(c->h_err, c->dev_error, sizeof(int), cudaMemcpyDeviceToHost, s));
  CK(cudaEventRecord(c->poll_ev, s));
  c->poll_stream = s;
  c->poll_pending = true;
  return S2R_OK;
}

int32_t s2r_poll_finished_ready(s2r_ctx* c, uint8_t* finished, int32_t wait, int32_t* ready) {
  if (!c || !finished || !ready) return fail(S2R_EINVAL, "NULL argument");
  if (!c->poll_pending) return fail(S2R_ESTATE, "no asynchronous poll was requested (s2r_poll_finished_async)");
  CK(cudaSetDevice(c->device));
  *ready = 0;
  cudaError_t q = wait ? cudaEventSynchronize(c->poll_ev) : cudaEventQuery(c->poll_ev);
  if (q == cudaErrorNotReady) {
    (void)cudaGetLastError();  // not an error: the copy is still queued
    return S2R_OK;
  }
  CK(q);
  c->poll_pending = false;
  std::memcpy(finished, c->h_fin, c->B);
  *ready = 1;
  if (*c->h_err != 0) return check_device_error(c, c->poll_stream);
  return S2R_OK;
}

int32_t s2r_take_async(s2r_ctx* c, int32_t slot, void* stream) {
  if (!c) return fail(S2R_EINVAL, "NULL engine");
  if (slot < 0 || slot >= c->B) return fail(S2R_EINVAL, "slot %d out of range [0, %d)", slot, c->B);
  if (!c->loaded[slot]) return fail(S2R_ESTATE, "slot %d is not loaded", slot);
  CK(cudaSetDevice(c->device));
  TRY(setup_async(c));
  if (c->take_pending[slot]) return fail(S2R_ESTATE, "slot %d has an asynchronous take whose tokens were not read", slot);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t* dst = c->h_out + (size_t)slot * c->T;
  CK(cudaMemcpyAsync(dst, c->st.out + (size_t)slot * c->T, (size_t)c->T * sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(c->h_pos_end + 2 * slot, c->st.position + slot, 8, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(c->h_pos_end + 2 * slot + 1, c->st.ended + slot, 8, cudaMemcpyDeviceToHost, s));
  CK(cudaEventRecord(c->take_ev[slot], s));
  // the slot is free for the work queued after the copies (a load on the same stream)
  c->take_pending[slot] = 1;
  c->loaded[slot] = 0;
  release_pages(c, slot);
  return S2R_OK;
}

int32_t s2r_take_ready(s2r_ctx* c, int32_t slot, int64_t* tokens, int32_t capacity, int32_t* length, int32_t* ended,
                       int32_t wait, int32_t* ready) {
  if (!c || !length || !ended || !ready) return fail(S2R_EINVAL, "NULL argument");
  if (slot < 0 || slot >= c->B) return fail(S2R_EINVAL, "slot %d out of range [0, %d)", slot, c->B);
  if (c->take_pending.empty() || !c->take_pending[slot])
    return fail(S2R_ESTATE, "slot %d has no asynchronous take (s2r_take_async)", slot);
  CK(cudaSetDevice(c->device));
  *ready = 0;
  cudaError_t q = wait ? cudaEventSynchronize(c->take_ev[slot]) : cudaEventQuery(c->take_ev[slot]);
  if (q == cudaErrorNotReady) {
    (void)cudaGetLastError();
    return S2R_OK;
  }
  CK(q);
  const int64_t* row = c->h_out + (size_t)slot * c->T;
  const int n = (int)c->h_pos_end[2 * slot] + 1;
  const int total = n + (row[n - 1] != 2 ? 1 : 0);  // always ends in <eos> (engine.py:259-260)
  *length = total;
  *ready = 1;
  if (!tokens || capacity < total) return fail(S2R_EINVAL, "capacity %d < %d tokens", capacity, total);
  std::memcpy(tokens, row, (size_t)n * sizeof(int64_t));
  if (total > n) tokens[n] = 2;
  *ended = (int32_t)c->h_pos_end[2 * slot + 1];
  c->take_pending[slot] = 0;
  return S2R_OK;
}

int32_t s2r_get_buffer(s2r_ctx* c, const char* name, void** ptr, int64_t* numel, int32_t* dtype) {
  if (!c || !name || !ptr || !numel || !dtype) return fail(S2R_EINVAL, "NULL argument");
  const SlotState& st = c->st;
  const int64_t B = c->B;
  struct Entry {
    const char* name;
    void* p;
    int64_t n;
    int32_t t;
  } table[] = {
      {"token", st.token, B, 2},          {"position", st.position, B, 2},   {"finished", st.finished, B, 3},
      {"ended", st.ended, B, 2},          {"in_shift", st.in_shift, B, 3},   {"shift_run", st.shift_run, B, 2},
      {"payload", st.payload, B, 2},      {"last_field", st.last_field, B, 2}, {"incomplete", st.incomplete, B, 2},
      {"g", st.g, B, 2},                  {"count", st.count, B, 2},         {"target", st.target, B, 2},
      {"stop", st.stop, B, 4},            {"out", st.out, B * c->T, 2},      {"frames", st.frames, B, 5},
      {"cross_k", c->layers[0].ck, B * c->H * c->F * kHeadDim, 1},
      {"cross_v", c->layers[0].cv, B * c->H * c->F * kHeadDim, 1},
  };
  // "cross_k.<layer>" / "cross_v.<layer>": any layer's cross K/V
  for (const char* which : {"cross_k.", "cross_v."}) {
    const size_t n = std::strlen(which);
    if (std::strncmp(name, which, n) == 0) {
      char* end = nullptr;
      const long l = std::strtol(name + n, &end, 10);
      if (end == name + n || *end != '\0' || l < 0 || l >= c->L) return fail(S2R_EINVAL, "no buffer named '%s'", name);
      *ptr = which[6] == 'k' ? c->layers[l].ck : c->layers[l].cv;
      *numel = B * c->H * c->F * kHeadDim;
      *dtype = 1;
      return S2R_OK;
    }
  }
  for (const Entry& e : table)
    if (std::strcmp(e.name, name) == 0 && e.p != nullptr) {
      *ptr = e.p;
      *numel = e.n;
      *dtype = e.t;
      return S2R_OK;
    }
  return fail(S2R_EINVAL, "no buffer named '%s'", name);
}

int32_t s2r_profile_step(s2r_ctx* c, float* ms, double* bytes, int32_t* launches, void* stream) {
  if (!c || !ms || !bytes || !launches) return fail(S2R_EINVAL, "NULL argument");
  CK(cudaSetDevice(c->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // algorithmic bytes need the live lengths: read positions, frames and flags
  std::vector<int64_t> pos(c->B);
  std::vector<int32_t> frames(c->B);
  std::vector<uint8_t> fin(c->B);
  CK(cudaMemcpyAsync(pos.data(), c->st.position, c->B * 8, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(frames.data(), c->st.frames, c->B * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(fin.data(), c->st.finished, c->B, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  const double D = c->D, FFN = c->FFN, V = c->V, M = c->B, H = c->H;
  double self_kv = 0, cross_kv = 0;
  int active = 0;
  for (int b = 0; b < c->B; ++b)
    if (!fin[b]) {
      ++active;
      self_kv += (double)(pos[b] + 1) * H * kHeadDim * 2 * 2;
      cross_kv += (double)frames[b] * H * kHeadDim * 2 * 2;
    }
  double per[K_CLASSES] = {
      3 * D * D * 2 + 3 * D * 2 + M * D * 8 + M * 3 * D * 2,  // qkv: W, b, r in, x out, q/k/v out
      self_kv + active * D * 4,                               // self attention: K, V, q in, out
      D * D * 2 + D * 2 + M * D * (2 + 4 + 4),                // self out-proj: W, b, a in, x in, r out
      D * D * 2 + D * 2 + M * D * (4 + 4 + 2),                // cross q
      cross_kv + active * D * 4,                              // cross attention
      D * D * 2 + D * 2 + M * D * (2 + 4 + 4),                // cross out-proj
      FFN * D * 2 + FFN * 2 + M * D * 8 + M * FFN * 2,        // fc1
      D * FFN * 2 + D * 2 + M * FFN * 2 + M * D * 8,          // fc2
      V * D * 2 + M * D * 4 + V,                              // logits: E, r in, grammar column
  };
  if (c->fuse_out) {  // the out-projections run inside the attention launches
    per[K_SELF_ATTN] += per[K_SELF_OUT];
    per[K_CROSS_ATTN] += per[K_CROSS_OUT];
    per[K_SELF_OUT] = per[K_CROSS_OUT] = 0.0;
    if (plan_attn(c, c->B, true).fuse_q) {  // and so does the cross q projection
      per[K_CROSS_ATTN] += per[K_CROSS_Q];
      per[K_CROSS_Q] = 0.0;
    }
    if (c->fuse_ffn) {  // fc1 and fc2 in one launch
      per[K_FC1] += per[K_FC2];
      per[K_FC2] = 0.0;
    }
  }
  for (int b = 0; b < c->B; ++b) {
    if (!c->loaded[b]) continue;
    c->bound[b] = std::min(c->bound[b] + 1, c->T - 1);
    bool changed = false;
    TRY(grow_pages(c, b, c->bound[b], &changed));
    if (changed) TRY(upload_page_row(c, b, s));
  }
  // The step is captured into a graph with an event node after every kernel
  // (no programmatic overlap, so each interval holds one kernel and no host
  // launch time) and replayed once.
  std::vector<std::pair<int, cudaEvent_t>> ev;
  cudaEvent_t start;
  CK(cudaEventCreate(&start));
  const bool pdl = c->pdl;
  c->pdl = false;
  c->prof = &ev;
  if (!c->use_graph) {  // plain launches: the events also hold the host's launch time
    CK(cudaEventRecord(start, s));
    int rc0 = enqueue_step(c, s, nullptr, nullptr, nullptr);
    c->prof = nullptr;
    c->pdl = pdl;
    if (rc0 != S2R_OK) return rc0;
    CK(cudaStreamSynchronize(s));
  } else {
  CK(cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal));
  cudaError_t e0 = cudaEventRecordWithFlags(start, c->cap_stream, cudaEventRecordExternal);
  int rc = e0 == cudaSuccess ? enqueue_step(c, c->cap_stream, nullptr, nullptr, nullptr) : S2R_ECUDA;
  cudaGraph_t graph = nullptr;
  cudaError_t e1 = cudaStreamEndCapture(c->cap_stream, &graph);
  c->prof = nullptr;
  c->pdl = pdl;
  if (rc != S2R_OK || e0 != cudaSuccess || e1 != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    return rc != S2R_OK ? rc : fail(S2R_ECUDA, "profile capture failed");
  }
  cudaGraphExec_t exec = nullptr;
  cudaError_t e2 = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e2 != cudaSuccess) return fail(S2R_ECUDA, "profile graph: %s", cudaGetErrorString(e2));
  CK(cudaGraphLaunch(exec, s));
  CK(cudaStreamSynchronize(s));
  cudaGraphExecDestroy(exec);
  }
  for (int k = 0; k < K_CLASSES; ++k) {
    ms[k] = 0.f;
    bytes[k] = per[k];
    launches[k] = 0;
  }
  cudaEvent_t prev = start;
  for (auto& [cls, e] : ev) {
    float t = 0.f;
    CK(cudaEventElapsedTime(&t, prev, e));
    ms[cls] += t;
    launches[cls] += 1;
    prev = e;
  }
  cudaEventDestroy(start);
  for (auto& pe : ev) cudaEventDestroy(pe.second);
  return S2R_OK;
}

int32_t s2r_step_launches(s2r_ctx* c) {
  if (!c) return 0;
  // tensor-core engines add a LayerNorm launch before each LayerNorm'd projection and the logits
  if (c->tc) return 11 * c->L + 2;
  // attention fused with its out-projection; the cross q launch folds into
  // the cross attention when that computes its own query rows
  // and one-slot engines run the FFN as one launch
  return ((plan_attn(c, c->B, true).fuse_q ? 5 : 6) - (c->fuse_ffn ? 1 : 0)) * c->L + 1;
}

int32_t s2r_free_pages(s2r_ctx* c) { return c ? (int32_t)c->free_pages.size() : 0; }

}  // extern "C"
