// pk::SlotPhase / PipelineSlot (pkt include/pipeline.cuh:14-57). On B200 the slot
// handoff is mbarrier phase bits; the enum values and the 128-byte slot
// alignment are kept for code that inspects them.
#pragma once

#include "task.cuh"

namespace pk {

enum class SlotPhase : int { Empty = 0, Loading, Loaded, Computing, Computed, Storing, Done };

struct alignas(128) PipelineSlot {
  Task task;
  int phase;
  int task_seq;
  int compute_warps_done;

  __host__ __device__ inline void reset() {
    phase = int(SlotPhase::Empty);
    task_seq = -1;
    compute_warps_done = 0;
  }
};

// Next index of the slot ring (pkt include/pipeline.cuh:50-57), host and device.
__host__ __device__ inline int ring_advance(int index) {
  if constexpr ((Config::kPipelineStages & (Config::kPipelineStages - 1)) == 0)
    return (index + 1) & (Config::kPipelineStages - 1);
  else
    return (index + 1) % Config::kPipelineStages;
}

#ifdef __CUDACC__
// Waits until *phase holds `target` (pkt include/pipeline.cuh:40-47: acquire
// loads with a doubling nanosleep backoff up to 1 us). Unlike pkt's it gives up
// after `budget_ns` (default 2 s) and returns false instead of spinning forever.
__device__ inline bool wait_for_phase(const int* phase, SlotPhase target,
                                      unsigned long long budget_ns = 2000000000ull) {
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  unsigned backoff = 10;
  while (true) {
    int v;
    asm volatile("ld.acquire.cta.b32 %0, [%1];" : "=r"(v) : "l"(phase) : "memory");
    if (v == int(target)) return true;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > budget_ns) return false;
    __nanosleep(backoff);
    backoff = backoff < 500 ? backoff * 2 : 1000;
  }
}
#endif

}  // namespace pk
