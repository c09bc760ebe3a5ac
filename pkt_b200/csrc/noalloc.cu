// pkt_axpy_noalloc: the axpy entry point for callers that must not allocate.
//
// pkt_axpy (entry.cu) keeps its task list and the megakernel's token / status
// words in device memory that its runtime obtains with cudaMalloc. Some callers
// cannot allow that: code running while a caching allocator owns the device
// memory budget, code that must not synchronise the device (cudaMalloc / cudaFree
// may), or a host program that pre-plans all memory up front. This variant keeps
// that scratch in one fixed array in the library's own device memory instead:
// it calls no cudaMalloc, cudaFree or allocating library routine.
//
// Limits and sharing:
//   * at most kNoAllocMaxTasks tasks of kNoAllocChunk floats each, i.e.
//     n <= 2048 * 32768 = 67,108,864 elements; larger n is rejected with
//     PKT_ERR_ARGS before anything is launched;
//   * every GPU that loads the library holds the ~192 KB array until the process
//     exits;
//   * all calls on a device share the one array: calls that overlap on the GPU
//     (different streams, or different host threads without ordering) race on
//     it. Calls on one stream are ordered and safe;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress with that device current); make that first call
//     before any stream capture;
//   * every wait inside the launch has a fixed budget of 2 s; what went wrong
//     on the device (a timeout, a rejected task) stays in the array's status
//     words until the next call, and pkt_axpy_noalloc_status reads it.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "../../include/pk/detail/internal.h"
#include "runtime_impl.h"

namespace pkb {
namespace {

constexpr int kNoAllocMaxTasks = 2048;
constexpr long long kNoAllocChunk = 32768;  // floats per task, as pkt_axpy
constexpr int kNoAllocTokens = 1;           // axpy tasks declare no dependencies

struct NoAllocScratch {
  pkt_task tasks[kNoAllocMaxTasks];
  int state[kStateHeader + 2 * kNoAllocTokens];  // cursor, status words, token counters
};

// The scratch itself. In host code this name is only a stand-in for the
// symbol; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[sizeof(NoAllocScratch)];

std::mutex g_mu;
NoAllocScratch* g_scratch_dev[64] = {};
int g_num_sms[64] = {};

// Writes the axpy task list and zeroes the cursor / status / token words, so a
// call never sees the previous call's contents.
__global__ void build_axpy_tasks(NoAllocScratch* s, const float* x, float* y, float a,
                                 long long n, int ntask) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < ntask) {
    pkt_task t;
    memset(&t, 0, sizeof(t));
    t.header.opcode = PKT_OP_AXPY;
    AxpyArgs args{x + i * kNoAllocChunk, y + i * kNoAllocChunk, a,
                  int(n - i * kNoAllocChunk < kNoAllocChunk ? n - i * kNoAllocChunk : kNoAllocChunk)};
    t.header.arg_bytes = sizeof(args);
    memcpy(t.args, &args, sizeof(args));
    s->tasks[i] = t;
  }
  if (i < kStateHeader + 2 * kNoAllocTokens) s->state[i] = 0;
}

}  // namespace
}  // namespace pkb

namespace pkb {
namespace {
// Looks up (once per device, with that device current) the scratch array's
// device address.
int noalloc_scratch(NoAllocScratch** s, int* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(PKT_ERR_ARGS, "device id out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_dev[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    e = cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    g_scratch_dev[dev] = static_cast<NoAllocScratch*>(ptr);
  }
  *s = g_scratch_dev[dev];
  if (sms) *sms = g_num_sms[dev];
  return PKT_OK;
}
}  // namespace
}  // namespace pkb

extern "C" int pkt_axpy_noalloc_status(int* code, int* task_index, int* detail) {
  using namespace pkb;
  NoAllocScratch* s = nullptr;
  int rc = noalloc_scratch(&s, nullptr);
  if (rc) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int h[4] = {0, 0, 0, 0};
  e = cudaMemcpy(h, s->state, sizeof(h), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read no-alloc status words");
  if (code) *code = h[1];
  if (task_index) *task_index = h[2];
  if (detail) *detail = h[3];
  return PKT_OK;
}

extern "C" int pkt_axpy_noalloc(const float* x, float* y, float a, long long n, void* stream) {
  using namespace pkb;
  if (n < 0 || (n > 0 && (!x || !y))) return fail(PKT_ERR_ARGS, "bad axpy arguments");
  if (n > kNoAllocMaxTasks * kNoAllocChunk)
    return fail(PKT_ERR_ARGS,
                "pkt_axpy_noalloc: n=%lld exceeds the fixed scratch limit of %lld elements "
                "(%d tasks of %lld); use pkt_axpy for larger arrays",
                n, (long long)kNoAllocMaxTasks * kNoAllocChunk, kNoAllocMaxTasks, kNoAllocChunk);
  NoAllocScratch* s = nullptr;
  int sms = 0;
  int rc = noalloc_scratch(&s, &sms);  // once per device: the array's device address
  if (rc) return rc;
  if (n == 0) return PKT_OK;
  int resident = 0;
  cudaError_t e = max_resident_blocks(1, &resident);
  if (e != cudaSuccess) return cuda_fail(e, "occupancy of the persistent kernel");
  if (sms > resident) sms = resident;
  const int ntask = int((n + kNoAllocChunk - 1) / kNoAllocChunk);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // one thread per task, and at least as many threads as status / token words to clear
  const int threads = 128;
  const int work = ntask > kStateHeader + 2 * kNoAllocTokens ? ntask : kStateHeader + 2 * kNoAllocTokens;
  const int blocks = (work + threads - 1) / threads;
  build_axpy_tasks<<<blocks, threads, 0, st>>>(s, x, y, a, n, ntask);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch no-alloc task builder");
  KParams p{};
  p.tasks = s->tasks;
  p.num_tasks = ntask;
  p.num_tokens = kNoAllocTokens;
  p.state = s->state;
  p.gemms = nullptr;
  p.num_gemms = 0;
  p.chunk = 1;
  p.task_counter = nullptr;
  p.perf = nullptr;
  p.timeout_ns = 2000000000ull;
  e = launch_megakernel(p, sms, st, 1);
  if (e != cudaSuccess) return cuda_fail(e, "launch megakernel");
  return PKT_OK;
}
