// Kernel selectors: each returns the instantiation of a kernel template for
// run-time shape parameters.  They live in separate translation units
// (kernels_*.cu) so that the template instantiations compile in parallel;
// kernels_select.cu dispatches to them.
#pragma once

#include <cuda.h>

#include "crosskv.cuh"
#include "gemm_tc.cuh"
#include "logits.cuh"
#include "prefill_attn.cuh"
#include "proj.cuh"

namespace s2r {

typedef void (*ProjFn)(const ProjArgs);
typedef void (*LogitsFn)(const LogitsArgs);
typedef void (*GemmFn)(CUtensorMap, CUtensorMap, TcArgs);
typedef void (*LnFn)(const ProjArgs, bf16*);
typedef void (*CrossKvFn)(CUtensorMap, CUtensorMap, CrossKvArgs);
typedef void (*PrefillAttnFn)(CUtensorMap, CUtensorMap, CUtensorMap, PrefillAttnArgs);

// CUDA-core projection for in (InMode) x epi (EpiMode), K in kch 256-column
// chunks, mc rows per pass; nullptr for a combination the engine never runs.
ProjFn proj_fn(int in, int epi, int kch, int mc);
// CUDA-core fused logits / grammar / argmax / commit.
LogitsFn logits_fn(int kch, int mc);
// Tensor-core GEMM with nb-row tiles and epilogue epi (EpiMode or EPI_LOGITS).
GemmFn gemm_fn(int nb, int epi);
// LayerNorm rows into the tensor-core GEMM's bf16 operand (in: IN_LN or IN_EMBED).
LnFn ln_fn(int in, int kch);
// Cross K/V projection of a window for a group of layers (persistent tcgen05 GEMM).
CrossKvFn crosskv_fn();
// Attention of a prefill chunk (tcgen05, online softmax, cluster split over the keys).
PrefillAttnFn prefill_attn_fn();

// ---- template pickers shared by the kernels_*.cu translation units

template <int IN, int EPI, int KCH>
ProjFn pick_mc(int mc) {
  switch (mc) {
    case 1: return proj_kernel<KCH, 1, IN, EPI>;
    case 2: return proj_kernel<KCH, 2, IN, EPI>;
    case 4: return proj_kernel<KCH, 4, IN, EPI>;
    default: return proj_kernel<KCH, 8, IN, EPI>;
  }
}

template <int IN, int EPI>
ProjFn pick_proj(int kch, int mc) {
  switch (kch) {
    case 1: return pick_mc<IN, EPI, 1>(mc);
    case 2: return pick_mc<IN, EPI, 2>(mc);
    case 4: return pick_mc<IN, EPI, 4>(mc);
    case 8: return pick_mc<IN, EPI, 8>(mc);
    default: return pick_mc<IN, EPI, 16>(mc);
  }
}

template <int KCH>
LogitsFn pick_logits_mc(int mc) {
  switch (mc) {
    case 1: return logits_kernel<KCH, 1>;
    case 2: return logits_kernel<KCH, 2>;
    case 4: return logits_kernel<KCH, 4>;
    default: return logits_kernel<KCH, 8>;
  }
}

// Per-translation-unit parts of the selectors above.
ProjFn proj_fn_ln(int in, int epi, int kch, int mc);    // kernels_proj_ln.cu: LayerNorm'd inputs
ProjFn proj_fn_rows(int in, int epi, int kch, int mc);  // kernels_proj_rows.cu: bf16 / f32 rows

}  // namespace s2r
