// pk::PerfBlock: per-CTA counters of the last launch (pkt include/perf_counters.cuh:8-53
// names the fields; this build reports the ones its roles measure, one row of
// PKT_PERF_WORDS words per CTA).
#pragma once
namespace pk {
struct PerfBlock {
  unsigned long long tasks_issued{0};
  unsigned long long gemm_tiles{0};
  unsigned long long ctrl_wait_cycles{0};      // dependency waits
  unsigned long long ctrl_slot_wait_cycles{0};
  unsigned long long load_wait_slot_cycles{0};  // loader waiting for free stages
  unsigned long long mma_full_wait_cycles{0};
  unsigned long long mma_tmem_wait_cycles{0};
  unsigned long long compute_wait_loaded_cycles{0};  // epilogue waiting for accumulators
  unsigned long long compute_work_cycles{0};         // GEMM epilogues
  unsigned long long simt_work_cycles{0};            // element-wise ops
  unsigned long long total_cycles{0};
  unsigned long long mma_slot_wait_cycles{0};
  unsigned long long mma_issue_cycles{0};
  unsigned long long kblocks{0};
  unsigned long long mma_gap_cycles{0};       // between one tile's last MMA and the next tile's first
  unsigned long long mma_lifetime_cycles{0};
};
static_assert(sizeof(PerfBlock) == 16 * 8, "one PerfBlock per PKT_PERF_WORDS row");
}  // namespace pk
