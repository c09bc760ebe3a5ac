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
};

inline int ring_advance(int index) {
  if constexpr ((Config::kPipelineStages & (Config::kPipelineStages - 1)) == 0)
    return (index + 1) & (Config::kPipelineStages - 1);
  else
    return (index + 1) % Config::kPipelineStages;
}

}  // namespace pk
