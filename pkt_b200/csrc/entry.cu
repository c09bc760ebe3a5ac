// Stand-alone entry points built on the runtime: pkt_axpy (the
// examples/axpy_example.cu workload: y = a*x + y as a list of Axpy tasks).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/pk/detail/internal.h"
#include "runtime_impl.h"

namespace pkb {
namespace {
std::mutex g_mu;
Runtime* g_axpy_rt[64] = {};
std::vector<pkt_task> g_axpy_tasks[64];
}  // namespace
}  // namespace pkb

extern "C" int pkt_axpy(const float* x, float* y, float a, long long n, void* stream) {
  using namespace pkb;
  if (n < 0 || (n > 0 && (!x || !y))) return fail(PKT_ERR_ARGS, "bad axpy arguments");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(PKT_ERR_ARGS, "device id out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_axpy_rt[dev]) {
    int rc = Runtime::create(dev, &g_axpy_rt[dev]);
    if (rc) return rc;
  }
  Runtime* rt = g_axpy_rt[dev];
  // 128K floats per task: 1.5 MB of traffic, so the per-task handoff is a few
  // per cent of its time, and still several tasks per SM for balance at the
  // sizes where bandwidth matters; small arrays are split finer so every SM
  // gets work.
  long long chunk = 131072;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  while (chunk > 4096 && (n + chunk - 1) / chunk < 4LL * sms) chunk /= 2;
  const int ntask = int((n + chunk - 1) / chunk);
  std::vector<pkt_task>& tl = g_axpy_tasks[dev];
  tl.assign(ntask, pkt_task{});
  for (int i = 0; i < ntask; ++i) {
    AxpyArgs args{x + i * chunk, y + i * chunk, a, int(std::min(chunk, n - i * chunk))};
    tl[i].header.opcode = PKT_OP_AXPY;
    tl[i].header.arg_bytes = sizeof(args);
    std::memcpy(tl[i].args, &args, sizeof(args));
  }
  int rc = rt->initialize(std::max(ntask, rt->max_tasks));
  if (rc) return rc;
  rc = rt->submit_async(tl.data(), ntask, static_cast<cudaStream_t>(stream), false);
  if (rc) return rc;
  return rt->launch(0, static_cast<cudaStream_t>(stream));
}
