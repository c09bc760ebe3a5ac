// Host-side runtime object behind pkt_runtime (C-ABI) and the MLP engine.
#pragma once

#include <cuda_runtime.h>

#include <vector>

#include "../../include/pk/detail/internal.h"

namespace pkb {

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
int gemm_tiles(const pkt_gemm_desc& d, int* tm, int* tn);
int build_dev_gemm(const pkt_gemm_desc& d, DevGemm* g);
bool make_store_map(CUtensorMap* map, const void* base, int dtype, long long cols, long long rows,
                    long long ld);

struct Runtime {
  int device = -1;
  int num_sms = 0;
  pkt_task* d_tasks = nullptr;
  int max_tasks = 0;
  int num_tasks = 0;
  int* d_state = nullptr;
  int token_cap = 0;
  int num_tokens = 256;
  DevGemm* d_gemms = nullptr;
  int num_gemms = 0;
  int gemm_cap = 0;
  std::vector<DevGemm> host_gemms;
  unsigned long long* d_counter = nullptr;
  bool accounting = false;
  bool perf_enabled = false;
  unsigned long long* d_perf = nullptr;
  int perf_cap = 0;
  unsigned long long* d_clock = nullptr;  // [3]: SM cycles, ns, launches (KParams::clock_acc)
  bool trace_enabled = false;
  unsigned long long* d_trace = nullptr;  // [trace_cap][kTraceWords]
  int trace_cap = 0;
  int trace_tasks = 0;  // tasks of the last traced launch
  int last_blocks = 0;
  unsigned long long timeout_ns = 2000000000ull;
  std::vector<int> segments;
  int segment_window = 4;
  int cta_pair = 1;

  ~Runtime();
  static int create(int dev, Runtime** out);
  void release();
  int initialize(int max_tasks);
  int ensure_tokens(int need);
  static int scan_tokens(const pkt_task* tasks, int n);
  int submit_async(const pkt_task* tasks, int n, cudaStream_t stream, bool sync_copy);
  int reset_state(cudaStream_t stream, bool sync);
  int launch(int blocks, cudaStream_t stream);
  // Everything launch does but the launch: the grid (clamped), the cleared
  // counters and the kernel parameters of the submitted list.
  int prepare(int blocks, cudaStream_t stream, KParams* out, int* out_blocks);
  int status(int* code, int* task, int* detail);
  int register_gemms(const pkt_gemm_desc* descs, int n, int* first);
  // Clamps a persistent grid to the CTAs that fit on the device at once (and to
  // whole clusters of `pair`); 0 or a negative count asks for the largest grid.
  int clamp_blocks(int blocks, int pair, int* out);
  int clock_stats(unsigned long long* out3, bool reset);
  // Trace buffer for a launch of n tasks (cleared on `stream`); null when tracing is off.
  int trace_for(int n, cudaStream_t stream, unsigned long long** out);
  int fetch_trace(unsigned long long* out, int max_tasks, int* n);
};

}  // namespace pkb
