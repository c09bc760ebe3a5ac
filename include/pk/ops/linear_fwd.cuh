// LinearForward: y = x W^T over a tile (pkt include/ops/linear_fwd.cuh:18-29),
// any tile shape (pkt's limits tile_m == 2, n <= 1024 do not apply), fp32.
// Large GEMMs belong on OpCode::Gemm (tcgen05 tiles, see gemm.cuh).
#pragma once
#include "../op_traits.cuh"
namespace pk {
struct LinearForwardArgs {
  const float* W;
  const float* x;
  float* y;
  int batch, m, n, tile_m_start, tile_m_count, tile_n_start, tile_n_count;
};
static_assert(sizeof(LinearForwardArgs) == 56, "pkt LinearForwardArgs layout");
template <> struct OpTraits<OpCode::LinearForward> { using Args = LinearForwardArgs; };
}  // namespace pk
