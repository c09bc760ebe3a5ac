// LinearBackward: dW = dy^T x over a tile, overwriting (pkt include/ops/linear_bwd.cuh:16-27),
// any batch (pkt's limit batch <= 64 does not apply), fp32.
#pragma once
#include "../op_traits.cuh"
namespace pk {
struct LinearBackwardArgs {
  const float* dy;
  const float* x;
  float* dW;
  int batch, m, n, tile_m_start, tile_m_count, tile_n_start, tile_n_count;
};
static_assert(sizeof(LinearBackwardArgs) == 56, "pkt LinearBackwardArgs layout");
template <> struct OpTraits<OpCode::LinearBackward> { using Args = LinearBackwardArgs; };
}  // namespace pk
