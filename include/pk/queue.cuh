// pk::GlobalQueue (pkt include/queue.cuh:12-16). The device-resident queue and
// its cursor are owned by the runtime inside libpkt_b200; this is the host view.
#pragma once

#include "task.cuh"

namespace pk {
struct GlobalQueue {
  Task* tasks{nullptr};
  int total{0};
  int* next_index{nullptr};
};
}  // namespace pk
