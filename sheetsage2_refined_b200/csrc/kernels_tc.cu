// Instantiations of the tensor-core GEMM, its LayerNorm pre-pass, the
// all-layer cross K/V projection and the prefill attention.
#include "kernels.h"

namespace s2r {

template <int NB>
GemmFn pick_gemm(int epi) {
  switch (epi) {
    case EPI_QKV: return gemm_tc_kernel<NB, EPI_QKV>;
    case EPI_RESID: return gemm_tc_kernel<NB, EPI_RESID>;
    case EPI_BF16: return gemm_tc_kernel<NB, EPI_BF16>;
    case EPI_GELU: return gemm_tc_kernel<NB, EPI_GELU>;
    case EPI_LOGITS: return gemm_tc_kernel<NB, EPI_LOGITS>;
    default: return nullptr;
  }
}

GemmFn gemm_fn(int nb, int epi) {
  switch (nb) {
    case 64: return pick_gemm<64>(epi);
    case 128: return pick_gemm<128>(epi);
    case 256: return pick_gemm<256>(epi);
    default: return nullptr;
  }
}


template <int IN>
LnFn pick_ln(int kch) {
  switch (kch) {
    case 1: return ln_rows_kernel<1, IN>;
    case 2: return ln_rows_kernel<2, IN>;
    case 4: return ln_rows_kernel<4, IN>;
    case 8: return ln_rows_kernel<8, IN>;
    default: return ln_rows_kernel<16, IN>;
  }
}

CrossKvFn crosskv_fn() { return crosskv_kernel<kCkvStages>; }

PrefillAttnFn prefill_attn_fn() { return prefill_attn_kernel<0>; }

LnFn ln_fn(int in, int kch) { return in == IN_EMBED ? pick_ln<IN_EMBED>(kch) : pick_ln<IN_LN>(kch); }

}  // namespace s2r
