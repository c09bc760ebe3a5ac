// pk::ProfileCounters (pkt include/profile_ranges.cuh:7-23). Runtime::fetch_profile
// fills it from the per-CTA role counters (summed over CTAs, in cycles).
#pragma once
namespace pk {
enum class ProfileRange : int {
  ControllerDepsWait = 0,
  ControllerQueuePop = 1,
  LoaderSlotWait = 2,
  LoaderLoad = 3,
  ComputeSlotWait = 4,
  ComputeMath = 5,
  StorerSlotWait = 6,
  StorerThreadfence = 7,
  StorerDepsMarkReady = 8,
  Count = 9,
};
struct ProfileCounters {
  unsigned long long cycles[static_cast<int>(ProfileRange::Count)];
};
}  // namespace pk
