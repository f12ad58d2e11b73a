// The persistent one-kernel decode step for K in 4 256-column chunk(s).
#include "kernels.h"

namespace s2r {

StepFn step_fn_kch4(int mr) { return pick_step_mr<4>(mr); }

}  // namespace s2r
