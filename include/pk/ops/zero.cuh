// ZeroMemory (pkt include/ops/zero.cuh:10-48).
#pragma once
#include "../op_traits.cuh"
namespace pk {
struct ZeroMemoryArgs {
  float* ptr;
  int size;
};
static_assert(sizeof(ZeroMemoryArgs) == 16, "pkt ZeroMemoryArgs layout");
template <> struct OpTraits<OpCode::ZeroMemory> { using Args = ZeroMemoryArgs; };
}  // namespace pk
