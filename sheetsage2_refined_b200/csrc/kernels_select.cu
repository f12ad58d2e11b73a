// Run-time selectors over the kernel instantiations of the kernels_*.cu units.
#include "kernels.h"

namespace s2r {

ProjFn proj_fn(int in, int epi, int kch, int mc) {
  if (ProjFn f = proj_fn_ln(in, epi, kch, mc)) return f;
  return proj_fn_rows(in, epi, kch, mc);
}

StepFn step_fn(int kch, int mr) {
  switch (kch) {
    case 1: return step_fn_kch1(mr);
    case 2: return step_fn_kch2(mr);
    default: return step_fn_kch4(mr);
  }
}

}  // namespace s2r
