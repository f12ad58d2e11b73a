// Run-time selectors over the kernel instantiations of the kernels_*.cu units.
#include "kernels.h"

namespace s2r {

ProjFn proj_fn(int in, int epi, int kch, int mc) {
  if (ProjFn f = proj_fn_ln(in, epi, kch, mc)) return f;
  return proj_fn_rows(in, epi, kch, mc);
}

}  // namespace s2r
