// Gemm (pkt's reserved OpCode::Gemm = 3, a commented-out stub in pkt's
// dispatch.cuh): one tcgen05 tile of a GEMM registered with
// pk::Runtime::register_gemm (TMA tensor maps built on the host).
#pragma once
#include "../op_traits.cuh"
namespace pk {
using GemmTileArgs = pkt_gemm_tile_args;
using GemmDesc = pkt_gemm_desc;
template <> struct OpTraits<OpCode::Gemm> { using Args = GemmTileArgs; };
}  // namespace pk
