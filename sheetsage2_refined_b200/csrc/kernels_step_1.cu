// The persistent one-kernel decode step for K in 1 256-column chunk(s).
#include "kernels.h"

namespace s2r {

StepFn step_fn_kch1(int mr) { return pick_step_mr<1>(mr); }

}  // namespace s2r
