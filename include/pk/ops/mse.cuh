// MSELoss: dy = 2(y-t)/(B m), loss += sum (y-t)^2 / (B m) (pkt include/ops/mse.cuh:13-68).
#pragma once
#include "../op_traits.cuh"
namespace pk {
struct MSELossArgs {
  const float* y;
  const float* target;
  float* dy;
  float* loss;
  int batch;
  int m;
};
static_assert(sizeof(MSELossArgs) == 40, "pkt MSELossArgs layout");
template <> struct OpTraits<OpCode::MSELoss> { using Args = MSELossArgs; };
using LossReduceArgs = pkt_loss_reduce_args;  // deterministic sum of tile partials (new)
template <> struct OpTraits<OpCode::LossReduce> { using Args = LossReduceArgs; };
}  // namespace pk
