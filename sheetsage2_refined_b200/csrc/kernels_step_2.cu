// The persistent one-kernel decode step for K in 2 256-column chunk(s).
#include "kernels.h"

namespace s2r {

StepFn step_fn_kch2(int mr) { return pick_step_mr<2>(mr); }

}  // namespace s2r
