// Running a program's own ops in the persistent megakernel: pkt's plugin point
// (template <OpCode> struct OpTraits with load / compute / store, pkt
// include/op_traits.cuh:8-15, dispatched per phase by include/dispatch.cuh:31-179).
//
//   namespace pk {
//   constexpr OpCode kScale = OpCode(100);
//   template <> struct OpTraits<kScale> {
//     struct Args { const float* x; float* y; float a; int n; };
//     __device__ static void load(const Args&, BlockRuntime&, int slot, int lane,
//                                 unsigned long long* reuse, unsigned long long* refill);
//     __device__ static void compute(const Args&, BlockRuntime&, int slot, int lane,
//                                    int compute_warp_idx, int num_compute_warps);
//     __device__ static void store(const Args&, BlockRuntime&, int slot, int lane);
//   };
//   }
//   ...
//   pk::Runtime rt; rt.initialize(n); rt.submit_tasks(tasks);
//   pk::launch_with_ops<pk::kScale>(rt);   // instead of rt.launch(); built-in ops still run
//   rt.synchronize();
//
// This header holds the whole megakernel (pk/detail/megakernel.cuh): the
// including translation unit (nvcc, -gencode arch=compute_100a,code=sm_100a)
// compiles an instantiation of it that dispatches the listed opcodes to their
// OpTraits besides the built-in ones, and launches it with the runtime's task
// list, tokens and counters (pkt_runtime_prepare_launch). An op's three phases
// run in order on the compute warps of one CTA (load and store by the first
// warp, compute by all four), with pkt's BlockRuntime: br.slot(slot).task is the
// task, pages 0 and 1 of slot `slot` are 4 KB of shared memory each. Tokens,
// epochs and the bounded dependency waits are the runtime's, as for every task.
#pragma once

#include <cuda_runtime.h>

#include "block_runtime.cuh"
#include "detail/megakernel.cuh"
#include "op_traits.cuh"
#include "runtime.hpp"
#include "task.cuh"

namespace pk {

// The opcodes a megakernel instantiation dispatches to pk::OpTraits.
template <OpCode... Codes>
struct OpSet {
  static_assert(sizeof...(Codes) > 0, "list at least one opcode");

  __device__ static bool handles(std::uint16_t op) { return ((op == std::uint16_t(Codes)) || ...); }

  __device__ static void load(std::uint16_t op, const Task& t, BlockRuntime& br, int slot, int lane,
                              unsigned long long* reuse, unsigned long long* refill) {
    ((op == std::uint16_t(Codes)
          ? (OpTraits<Codes>::load(decode_args<typename OpTraits<Codes>::Args>(t), br, slot, lane, reuse, refill),
             0)
          : 0),
     ...);
  }

  __device__ static void compute(std::uint16_t op, const Task& t, BlockRuntime& br, int slot, int lane, int cwarp,
                                 int ncwarps) {
    ((op == std::uint16_t(Codes)
          ? (OpTraits<Codes>::compute(decode_args<typename OpTraits<Codes>::Args>(t), br, slot, lane, cwarp,
                                      ncwarps),
             0)
          : 0),
     ...);
  }

  __device__ static void store(std::uint16_t op, const Task& t, BlockRuntime& br, int slot, int lane) {
    ((op == std::uint16_t(Codes)
          ? (OpTraits<Codes>::store(decode_args<typename OpTraits<Codes>::Args>(t), br, slot, lane), 0)
          : 0),
     ...);
  }
};

// pkt_runtime_launch for a megakernel that also runs the listed ops. Returns the
// C-ABI status (0 = ok); a failure is also kept in the Runtime's last_error().
template <OpCode... Codes>
inline int launch_with_ops(pkt_runtime* rt, int num_blocks = 0, cudaStream_t stream = nullptr) {
  pkb::KParams kp{};
  int blocks = 0, pair = 1;
  int rc = pkt_runtime_prepare_launch(rt, num_blocks, stream, &kp, int(sizeof(kp)), &blocks, &pair);
  if (rc) return rc;
  const cudaError_t e = pkb::launch_megakernel_ops<OpSet<Codes...>>(kp, blocks, stream, pair);
  return e == cudaSuccess ? PKT_OK : PKT_ERR_CUDA;
}

template <OpCode... Codes>
inline int launch_with_ops(Runtime& rt, int num_blocks = 0, cudaStream_t stream = nullptr) {
  return launch_with_ops<Codes...>(rt.handle(), num_blocks, stream);
}

}  // namespace pk
