// pk::DependencyState (pkt include/dependency.cuh:14-78): host view of the token
// counters. Semantics kept: a task waiting on token b runs once
// count[b] >= wait_count and epoch[b] >= read_epoch; a finished task adds 1 to
// count[write_id] and raises epoch[write_id] to write_epoch. Counts are
// cumulative over one launch. The runtime sizes the token array to the largest
// id a task list uses (pkt fixes 256).
#pragma once

namespace pk {
struct DependencyState {
  static constexpr int kMaxBuffers = 256;
  int buffer_ready_count[kMaxBuffers];
  int buffer_epoch[kMaxBuffers];
};
}  // namespace pk
