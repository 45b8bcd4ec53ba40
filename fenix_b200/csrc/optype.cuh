// optype.cuh — operand element types of the tensor-core paths (values are fx_precision's).
#pragma once

namespace fxk {
enum OpType : int { kOpBF16 = 0, kOpE4M3 = 1, kOpF16 = 2 };
}  // namespace fxk
