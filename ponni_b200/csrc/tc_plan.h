// Host planner of the tensor-core dense-chain kernel (tc_plan.cu).
#pragma once
#include <string>
#include <vector>

#include "model.h"
#include "tc_program.h"

namespace ponni_b200 {

// Build the TcProgram and the staged parameter image for `m`; false (with
// the reason in `why`) when the model is not a dense chain the kernel supports.
// `rec` (optional) receives the image location of every trainable parameter.
bool tc_plan(const ponni_b200_model* m, TcProgram& p, std::vector<unsigned char>& image, std::string& why,
             ParamMap* rec = nullptr);

}  // namespace ponni_b200
