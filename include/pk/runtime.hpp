// pk::Runtime — pkt's host runtime class (pkt include/runtime.hpp:22-450), same
// method names and argument meaning, implemented over the C-ABI of
// libpkt_b200.so (include/pkt_b200.h). A pkt program that includes
// "pk/runtime.hpp" and "pk/ops/*.cuh" instead of pkt's headers and links
// -lpkt_b200 builds and runs unchanged.
//
// Differences from pkt, all additive:
//   * every CUDA / device failure is kept: last_error() returns the C-ABI status
//     of the last failing call (0 = ok) and last_error_string() its message;
//     pkt checked no CUDA call;
//   * synchronize() also reads the device status word: a dependency wait that
//     ran out of time, an unknown opcode or a rejected task is reported instead
//     of hanging or being silently skipped;
//   * register_gemm() / set_cta_pair() expose the tcgen05 GEMM tiles behind
//     pkt's reserved OpCode::Gemm.
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "../pkt_b200.h"
#include "dependency.cuh"
#include "ops/gemm.cuh"
#include "perf_counters.cuh"
#include "profile_ranges.cuh"
#include "queue.cuh"
#include "segment.cuh"
#include "task.cuh"

namespace pk {

class Runtime {
 public:
  Runtime() {
    int dev = 0;
    cudaGetDevice(&dev);
    record(pkt_runtime_create(dev, &rt_));
  }
  ~Runtime() {
    if (rt_) pkt_runtime_destroy(rt_);
  }
  Runtime(const Runtime&) = delete;
  Runtime& operator=(const Runtime&) = delete;

  void initialize(int max_tasks) { record(pkt_runtime_initialize(rt_, max_tasks)); }

  void submit_tasks(const std::vector<Task>& tasks) {
    record(pkt_runtime_submit(rt_, reinterpret_cast<const pkt_task*>(tasks.data()),
                              static_cast<int>(tasks.size())));
  }

  void set_segments(const std::vector<SegmentDesc>& segments) {
    std::vector<int> flat;
    flat.reserve(segments.size() * 2);
    for (const auto& s : segments) {
      flat.push_back(s.begin);
      flat.push_back(s.end);
    }
    record(pkt_runtime_set_segments(rt_, flat.data(), static_cast<int>(segments.size())));
  }

  void set_segment_window_size(int window_size) {
    record(pkt_runtime_set_segment_window_size(rt_, window_size));
  }

  void launch(int num_blocks, cudaStream_t stream = nullptr) {
    record(pkt_runtime_launch(rt_, num_blocks, stream));
  }

  void synchronize() { record(pkt_runtime_synchronize(rt_)); }

  // Sums the per-CTA role counters of the last launch into pkt's ranges; needs
  // set_perf_enabled(true) before the launch.
  bool fetch_profile(ProfileCounters* out) {
    std::vector<PerfBlock> blocks;
    if (!out || !fetch_perf_blocks(blocks)) return false;
    *out = ProfileCounters{};
    for (const auto& b : blocks) {
      out->cycles[int(ProfileRange::ControllerDepsWait)] += b.ctrl_wait_cycles;
      out->cycles[int(ProfileRange::LoaderSlotWait)] += b.load_wait_slot_cycles;
      out->cycles[int(ProfileRange::ComputeSlotWait)] += b.compute_wait_loaded_cycles;
      out->cycles[int(ProfileRange::ComputeMath)] += b.compute_work_cycles + b.simt_work_cycles;
      out->cycles[int(ProfileRange::StorerSlotWait)] += b.mma_full_wait_cycles;
    }
    return true;
  }

  bool fetch_task_counter(unsigned long long* out) {
    return out && record(pkt_runtime_fetch_task_counter(rt_, out)) == PKT_OK;
  }
  void set_task_accounting_enabled(bool enabled) {
    record(pkt_runtime_set_task_accounting(rt_, enabled ? 1 : 0));
  }
  void set_perf_enabled(bool enabled) {
    perf_ = enabled;
    record(pkt_runtime_set_perf(rt_, enabled ? 1 : 0));
  }
  int last_launch_blocks() const { return pkt_runtime_last_launch_blocks(rt_); }

  bool fetch_perf_blocks(std::vector<PerfBlock>& out) {
    if (!perf_) return false;
    const int nb = last_launch_blocks();
    if (nb <= 0) return false;
    out.resize(static_cast<size_t>(nb));
    int got = 0;
    if (record(pkt_runtime_fetch_perf(rt_, reinterpret_cast<unsigned long long*>(out.data()), nb,
                                      &got)) != PKT_OK)
      return false;
    out.resize(static_cast<size_t>(got));
    return true;
  }

  // Segment gating is not a separate scheduler here: segments are kept as hints.
  bool fetch_segment_state(std::vector<int>& completed, int* seg_lo, int* seg_hi, int* window) {
    (void)completed;
    (void)seg_lo;
    (void)seg_hi;
    (void)window;
    return false;
  }

  static int get_num_sms() {
    int device = 0;
    cudaGetDevice(&device);
    return pkt_num_sms(device);
  }

  // ---- additions
  int register_gemm(const GemmDesc& desc) {
    int id = -1;
    record(pkt_runtime_register_gemms(rt_, &desc, 1, &id));
    return id;
  }
  void set_cta_pair(int pair) { record(pkt_runtime_set_cta_pair(rt_, pair)); }
  void set_timeout_ns(unsigned long long ns) { record(pkt_runtime_set_timeout_ns(rt_, ns)); }
  int status(int* code, int* task_index, int* detail) {
    return record(pkt_runtime_status(rt_, code, task_index, detail));
  }
  int last_error() const { return last_error_; }
  const std::string& last_error_string() const { return last_error_string_; }
  pkt_runtime* handle() { return rt_; }

 private:
  int record(int rc) {
    if (rc != PKT_OK) {
      last_error_ = rc;
      last_error_string_ = pkt_last_error();
    }
    return rc;
  }
  pkt_runtime* rt_ = nullptr;
  bool perf_ = false;
  int last_error_ = PKT_OK;
  std::string last_error_string_;
};

}  // namespace pk
