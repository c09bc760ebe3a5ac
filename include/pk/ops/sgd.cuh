// SGDUpdate: W -= lr * dW (pkt include/ops/sgd.cuh:12-52), spread over every
// compute thread of the CTA, 128-bit vectorised.
#pragma once
#include "../op_traits.cuh"
namespace pk {
struct SGDUpdateArgs {
  float* W;
  const float* dW;
  float lr;
  int size;
};
static_assert(sizeof(SGDUpdateArgs) == 24, "pkt SGDUpdateArgs layout");
template <> struct OpTraits<OpCode::SGDUpdate> { using Args = SGDUpdateArgs; };
using SGDMixedArgs = pkt_sgd_mixed_args;  // fp32 master - lr*g, bf16 copy (new)
template <> struct OpTraits<OpCode::SGDMixed> { using Args = SGDMixedArgs; };
using BiasSGDArgs = pkt_bias_sgd_args;  // bias -= lr * sum of column partials (new)
template <> struct OpTraits<OpCode::BiasSGD> { using Args = BiasSGDArgs; };
}  // namespace pk
