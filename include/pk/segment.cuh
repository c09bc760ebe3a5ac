// pk::SegmentDesc (pkt include/segment.cuh:7-10): [begin, end) task ranges.
#pragma once

namespace pk {
struct SegmentDesc {
  int begin;
  int end;
};
}  // namespace pk
