// pk::OpTraits<OpCode> (pkt include/op_traits.cuh:8-15): the plugin point. A
// specialisation names its Args (the 64-byte task payload) and, for an op a
// program adds, the three device phases pkt dispatches (pkt
// include/dispatch.cuh:31-179):
//   load(args, br, slot, lane, reuse_hits, refill_count)      one warp
//   compute(args, br, slot, lane, compute_warp_idx, num_compute_warps)
//   store(args, br, slot, lane)                               one warp
// pk::launch_with_ops<Codes...> (pk/kernel.cuh) compiles the persistent
// megakernel with those ops dispatched besides the built-in ones. The built-in
// ops' specialisations (pk/ops/*.cuh) carry only Args: their device code is the
// tcgen05 / element-wise machinery inside libpkt_b200.
#pragma once

#include "task.cuh"

namespace pk {
template <OpCode Code>
struct OpTraits;
}  // namespace pk
