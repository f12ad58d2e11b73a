// CUDA-core projections of bf16 / f32 rows (out-projections, fc2, cross K/V) and the logits.
#include "kernels.h"

namespace s2r {

ProjFn proj_fn_rows(int in, int epi, int kch, int mc) {
  if (in == IN_BF16 && epi == EPI_RESID) return pick_proj<IN_BF16, EPI_RESID>(kch, mc);
  if (in == IN_BF16 && epi == EPI_SLICES) return pick_proj<IN_BF16, EPI_SLICES>(kch, mc);  // fc2 into fixed-point sums
  if (in == IN_BF16 && epi == EPI_CROSSKV) return pick_proj<IN_BF16, EPI_CROSSKV>(kch, mc);
  if (in == IN_F32 && epi == EPI_CROSSKV) return pick_proj<IN_F32, EPI_CROSSKV>(kch, mc);
  return nullptr;
}

LogitsFn logits_fn(int kch, int mc) {
  switch (kch) {
    case 1: return pick_logits_mc<1>(mc);
    case 2: return pick_logits_mc<2>(mc);
    case 4: return pick_logits_mc<4>(mc);
    case 8: return pick_logits_mc<8>(mc);
    default: return pick_logits_mc<16>(mc);
  }
}

}  // namespace s2r
