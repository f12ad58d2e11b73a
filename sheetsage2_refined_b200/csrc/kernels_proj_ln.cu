// CUDA-core projections of LayerNorm'd rows (QKV, cross q, fc1), from residual sums or out-projection sums.
#include "kernels.h"

namespace s2r {

ProjFn proj_fn_ln(int in, int epi, int kch, int mc) {
  if (in == IN_EMBED && epi == EPI_QKV) return pick_proj<IN_EMBED, EPI_QKV>(kch, mc);
  if (in == IN_LN && epi == EPI_QKV) return pick_proj<IN_LN, EPI_QKV>(kch, mc);
  if (in == IN_LN && epi == EPI_BF16) return pick_proj<IN_LN, EPI_BF16>(kch, mc);
  if (in == IN_LN && epi == EPI_GELU) return pick_proj<IN_LN, EPI_GELU>(kch, mc);
  if (in == IN_ACC && epi == EPI_QKV) return pick_proj<IN_ACC, EPI_QKV>(kch, mc);  // QKV after an FFN
  if (in == IN_ACC && epi == EPI_BF16) return pick_proj<IN_ACC, EPI_BF16>(kch, mc);  // cross q after an attention
  if (in == IN_ACC && epi == EPI_GELU) return pick_proj<IN_ACC, EPI_GELU>(kch, mc);  // fc1 after an attention
  return nullptr;
}

}  // namespace s2r
