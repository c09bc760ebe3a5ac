// Axpy: y = a*x + y (pkt include/ops/axpy.cuh:9-54). 128-bit vectorised, one
// fused multiply-add per element (bit-identical to pkt's kernel).
#pragma once
#include "../op_traits.cuh"
namespace pk {
struct AxpyArgs {
  const float* x;
  float* y;
  float a;
  int n;
};
static_assert(sizeof(AxpyArgs) == 24, "pkt AxpyArgs layout");
template <> struct OpTraits<OpCode::Axpy> { using Args = AxpyArgs; };
}  // namespace pk
