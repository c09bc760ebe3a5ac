// Slot ring constants and warp roles (cases of pkt's tests/test_pipeline.cu:10-78, host part).
#include "check.hpp"
#include "pk/config.cuh"
#include "pk/pipeline.cuh"

using namespace pk;

static bool slot_alignment() {
  CHECK(alignof(PipelineSlot) == 128, "PipelineSlot 128-byte aligned");
  return true;
}

static bool slot_phase_values() {
  CHECK(int(SlotPhase::Empty) == 0 && int(SlotPhase::Loading) == 1 && int(SlotPhase::Loaded) == 2 &&
            int(SlotPhase::Computing) == 3 && int(SlotPhase::Computed) == 4 &&
            int(SlotPhase::Storing) == 5 && int(SlotPhase::Done) == 6,
        "SlotPhase 0..6");
  return true;
}

static bool ring_wraps() {
  int idx = 0;
  for (int i = 0; i < Config::kPipelineStages * 3; ++i) {
    idx = ring_advance(idx);
    CHECK(idx == (i + 1) % Config::kPipelineStages, "ring_advance");
  }
  return true;
}

static bool config_consistency() {
  CHECK(Config::kTotalWarps == 3 + Config::kNumComputeWarps, "total warps");
  CHECK(Config::kThreadsPerBlock == Config::kTotalWarps * Config::kWarpSize, "threads per block");
  WarpRoles r;
  CHECK(r.controller == 0 && r.loader == 1 && r.storer == 2 && r.first_compute == 3 && r.num_compute == 4,
        "default warp roles");
  CHECK(is_compute(3, r) && is_compute(6, r) && !is_compute(7, r) && compute_warp_index(5, r) == 2,
        "role helpers");
  return true;
}

int main() {
  Case cs[] = {{"slot_alignment", slot_alignment},
               {"slot_phase_values", slot_phase_values},
               {"ring_wraps", ring_wraps},
               {"config_consistency", config_consistency}};
  return run_cases(cs, 4);
}
