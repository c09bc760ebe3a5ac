// Host runtime behind the C-ABI: owns the device task array, the token /
// status state, the registered GEMM table (with TMA tensor maps) and launches
// the persistent megakernel. Restates pkt's pk::Runtime (include/runtime.hpp:22-450)
// with every CUDA call checked and an error string instead of silent failure.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/pk/detail/internal.h"
#include "runtime_impl.h"

namespace pkb {

static thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PKT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ---------------------------------------------------------------- tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2D tiled map over a row-major [rows][ld] matrix whose logical width is `cols`;
// box = {box_x elements, box_y rows}, 128-byte swizzle, zero fill out of bounds.
static int make_map(CUtensorMap* map, const void* base, int dtype, long long cols, long long rows,
                    long long ld, int box_x, int box_y, bool atom32 = false) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(PKT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const int es = dtype == PKT_DTYPE_BF16 ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(PKT_ERR_ARGS, "TMA base address must be 16-byte aligned");
  if ((ld * es) % 16 != 0) return fail(PKT_ERR_ARGS, "row stride (ld=%lld) must be a multiple of 16 bytes", ld);
  if (box_x * es != 128) return fail(PKT_ERR_ARGS, "box inner extent must be 128 bytes");
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld * es)};
  cuuint32_t box[2] = {cuuint32_t(box_x), cuuint32_t(box_y)};
  cuuint32_t estr[2] = {1, 1};
  // TF32 operands: fp32 in memory, converted to TF32 by round-to-nearest as the TMA
  // unit loads them (plain truncation by the tensor core would bias every product).
  const CUtensorMapDataType tf32_type = CU_TENSOR_MAP_DATA_TYPE_TFLOAT32;
  CUresult r = enc(map, dtype == PKT_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : tf32_type,
                   2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PKT_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return PKT_OK;
}

// Tensor map for the epilogue's TMA tile stores: one box = 32 columns x 32 rows
// (the chunk one compute warp holds), swizzled (64-byte rows for bf16, 128-byte
// rows for fp32) so the warp's row-per-lane shared-memory writes are free of
// bank conflicts. Returns false (and the epilogue keeps its plain stores) where
// TMA cannot address the matrix.
bool make_store_map(CUtensorMap* map, const void* base, int dtype, long long cols,
                           long long rows, long long ld) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc || base == nullptr) return false;
  const int es = dtype == PKT_DTYPE_BF16 ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * es) % 16 != 0) return false;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld * es)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype == PKT_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                   2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   es == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Tensor map for L2 prefetches of the rows a tile's epilogue reads: one box =
// `box_cols` columns x 128 rows, no swizzle (a prefetch never lands in shared
// memory). False where TMA cannot address the matrix (the epilogue then just
// reads without the prefetch).
static bool make_prefetch_map(CUtensorMap* map, const void* base, int dtype, long long cols,
                              long long rows, long long ld, int box_cols) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc || base == nullptr || box_cols <= 0 || box_cols > 256) return false;
  const int es = dtype == PKT_DTYPE_BF16 ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * es) % 16 != 0 || (box_cols * es) % 16 != 0)
    return false;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld * es)};
  cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(kBM)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int gemm_tiles(const pkt_gemm_desc& d, int* tm, int* tn) {
  if (d.M <= 0 || d.N <= 0 || d.K <= 0 || d.bn < 16 || d.bn > kMaxBN || d.bn % 16 != 0)
    return fail(PKT_ERR_ARGS, "GEMM shape M=%d N=%d K=%d bn=%d invalid", d.M, d.N, d.K, d.bn);
  const int pair = d.cta_pair == 2 ? 2 : 1;
  *tm = (d.M + kBM * pair - 1) / (kBM * pair);
  *tn = (d.N + d.bn - 1) / d.bn;
  return PKT_OK;
}

int build_dev_gemm(const pkt_gemm_desc& d, DevGemm* g) {
  std::memset(g, 0, sizeof(*g));
  g->d = d;
  int rc = gemm_tiles(d, &g->tiles_m, &g->tiles_n);
  if (rc) return rc;
  if (d.in_dtype != PKT_DTYPE_BF16 && d.in_dtype != PKT_DTYPE_TF32)
    return fail(PKT_ERR_ARGS, "GEMM in_dtype must be bf16 or tf32");
  if (d.epilogue != PKT_EPI_WGRAD_SGD && d.epilogue != PKT_EPI_WGRAD_PEER && d.out_dtype != PKT_DTYPE_BF16 &&
      d.out_dtype != PKT_DTYPE_F32)
    return fail(PKT_ERR_ARGS, "GEMM out_dtype must be bf16 or f32");
  const bool bf = d.in_dtype == PKT_DTYPE_BF16;
  const int es = bf ? 2 : 4;
  g->pair = d.cta_pair == 2 ? 2 : 1;
  g->b_rows = d.bn / g->pair;
  if (g->pair == 2 && (d.bn % 32 != 0))
    return fail(PKT_ERR_ARGS, "CTA-pair tiles need bn multiple of 32 (got %d)", d.bn);
  // K depth per stage: one 128-byte chunk per CTA-stage in single mode, two in pair
  // mode (8 MMAs per barrier round trip)
  g->kchunks = g->pair;
  g->bk = (bf ? 64 : 32) * g->kchunks;
  g->box_mn = 128 / es;
  g->num_kb = (d.K + g->bk - 1) / g->bk;
  g->mma_per_kb = 4 * g->kchunks;  // bf16: K=16 per MMA, tf32: K=8 per MMA
  const int kinstr = bf ? 16 : 8;
  // A operand: 128 rows of the tile.
  if (d.a_major == PKT_MAJOR_K) {
    rc = make_map(&g->map_a, d.a, d.in_dtype, d.K, d.M, d.lda, 128 / es, kBM);
    g->a_boxes = 1;
    g->a_box_bytes = kBM * 128;
    g->a_lbo = 16;
    g->a_sbo = 1024;
    g->a_layout = 2;
    g->a_kstep = kinstr * es;
    g->a_kgroup = g->a_box_bytes;  // next 128-byte K chunk = next box
    g->a_boxes = g->kchunks;
  } else {
    // MN-major: boxes of 128 bytes along M x bk rows of K. TF32 needs the
    // 32-byte-atom swizzle (4-row pattern, 512-byte K groups).
    rc = make_map(&g->map_a, d.a, d.in_dtype, d.M, d.K, d.lda, g->box_mn, g->bk, !bf);
    g->a_boxes = kBM / g->box_mn;
    g->a_box_bytes = g->bk * 128;
    g->a_lbo = g->a_box_bytes;
    g->a_sbo = bf ? 1024 : 512;
    g->a_layout = bf ? 2 : 1;
    g->a_kstep = kinstr * 128;
    g->a_kgroup = 4 * g->a_kstep;
  }
  if (rc) return rc;
  if (d.b_major == PKT_MAJOR_K) {
    rc = make_map(&g->map_b, d.b, d.in_dtype, d.K, d.N, d.ldb, 128 / es, g->b_rows);
    g->b_boxes = 1;
    g->b_box_bytes = g->b_rows * 128;
    g->b_lbo = 16;
    g->b_sbo = 1024;
    g->b_layout = 2;
    g->b_kstep = kinstr * es;
    g->b_kgroup = g->b_box_bytes;
    g->b_boxes = g->kchunks;
  } else {
    if (g->b_rows % g->box_mn != 0)
      return fail(PKT_ERR_ARGS, "MN-major B operand needs bn multiple of %d", g->box_mn * g->pair);
    rc = make_map(&g->map_b, d.b, d.in_dtype, d.N, d.K, d.ldb, g->box_mn, g->bk, !bf);
    g->b_boxes = g->b_rows / g->box_mn;
    g->b_box_bytes = g->bk * 128;
    g->b_lbo = g->b_box_bytes;
    g->b_sbo = bf ? 1024 : 512;
    g->b_layout = bf ? 2 : 1;
    g->b_kstep = kinstr * 128;
    g->b_kgroup = 4 * g->b_kstep;
  }
  if (rc) return rc;
  // bytes landing on the (leader's) full barrier per stage: both CTAs' loads in pair mode
  g->stage_tx = g->pair * (g->a_boxes * g->a_box_bytes + g->b_boxes * g->b_box_bytes);
  const uint32_t fmt = bf ? 1u : 2u;
  g->idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(d.a_major) << 15) |
             (uint32_t(d.b_major) << 16) | (uint32_t(d.bn >> 3) << 17) |
             (uint32_t((kBM * g->pair) >> 4) << 24);
  // epilogue operand checks
  if (!d.out && d.epilogue != PKT_EPI_WGRAD_SGD && d.epilogue != PKT_EPI_WGRAD_PEER) return fail(PKT_ERR_ARGS, "GEMM output pointer missing");
  if ((d.epilogue == PKT_EPI_MSE || d.epilogue == PKT_EPI_DGRAD_RELU) && !d.aux)
    return fail(PKT_ERR_ARGS, "MSE / DGRAD epilogue needs aux");
  if ((d.epilogue == PKT_EPI_WGRAD_SGD || d.epilogue == PKT_EPI_WGRAD_PEER) && (!d.w_in || !d.w_out))
    return fail(PKT_ERR_ARGS, "WGRAD_SGD / WGRAD_PEER epilogues need w_in / w_out");
  if (d.epilogue < 0 || d.epilogue > PKT_EPI_WGRAD_PEER) return fail(PKT_ERR_ARGS, "bad epilogue");
  // TMA tile stores need whole 32-column chunks inside a tile (a box must not
  // spill into the neighbouring tile's columns).
  if (d.bn % 32 == 0) {
    if (d.epilogue == PKT_EPI_WGRAD_SGD || d.epilogue == PKT_EPI_WGRAD_PEER) {
      g->tma_w = make_store_map(&g->map_w, d.w_out, PKT_DTYPE_F32, d.N, d.M, d.ldw) &&
                 (d.w_shadow == nullptr ||
                  make_store_map(&g->map_shadow, d.w_shadow, PKT_DTYPE_BF16, d.N, d.M, d.ldw));
    } else {
      g->tma_out = make_store_map(&g->map_out, d.out, d.out_dtype, d.N, d.M, d.ldo);
    }
  }
  if (d.epilogue == PKT_EPI_MSE || d.epilogue == PKT_EPI_DGRAD_RELU)
    g->pf_ok = make_prefetch_map(&g->map_pf, d.aux, d.in_dtype == PKT_DTYPE_BF16 ? PKT_DTYPE_BF16 : PKT_DTYPE_F32,
                                 d.N, d.M, d.ldaux, d.bn);
  else if (d.epilogue == PKT_EPI_WGRAD_SGD)
    g->pf_ok = make_prefetch_map(&g->map_pf, d.w_in, PKT_DTYPE_F32, d.N, d.M, d.ldw, d.bn);
  return PKT_OK;
}

// ---------------------------------------------------------------- runtime object
Runtime::~Runtime() { release(); }

void Runtime::release() {
  if (device >= 0) cudaSetDevice(device);
  cudaFree(d_tasks);
  cudaFree(d_state);
  cudaFree(d_gemms);
  cudaFree(d_counter);
  cudaFree(d_perf);
  cudaFree(d_clock);
  d_clock = nullptr;
  cudaFree(d_trace);
  d_trace = nullptr;
  trace_cap = 0;
  d_tasks = nullptr;
  d_state = nullptr;
  d_gemms = nullptr;
  d_counter = nullptr;
  d_perf = nullptr;
}

int Runtime::ensure_tokens(int need) {
  if (need <= token_cap) return PKT_OK;
  int cap = std::max(256, token_cap);
  while (cap < need) cap *= 2;
  int* ns = nullptr;
  cudaError_t e = cudaMalloc(&ns, sizeof(int) * state_ints(cap));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(token state)");
  cudaMemset(ns, 0, sizeof(int) * state_ints(cap));
  cudaFree(d_state);
  d_state = ns;
  token_cap = cap;
  return PKT_OK;
}

int Runtime::initialize(int max_tasks_) {
  if (max_tasks_ < 0) return fail(PKT_ERR_ARGS, "max_tasks must be >= 0");
  cudaSetDevice(device);
  if (max_tasks_ > max_tasks) {
    cudaFree(d_tasks);
    d_tasks = nullptr;
    cudaError_t e = cudaMalloc(&d_tasks, sizeof(pkt_task) * std::max(1, max_tasks_));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(tasks)");
    max_tasks = max_tasks_;
  }
  int rc = ensure_tokens(256);
  if (rc) return rc;
  if (!d_counter) {
    cudaError_t e = cudaMalloc(&d_counter, sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(counter)");
  }
  if (!d_clock) {
    cudaError_t e = cudaMalloc(&d_clock, 3 * sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(clock words)");
    e = cudaMemset(d_clock, 0, 3 * sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_fail(e, "clear clock words");
  }
  return PKT_OK;
}

int Runtime::clamp_blocks(int blocks, int pair, int* out) {
  cudaSetDevice(device);
  int resident = 0;
  cudaError_t e = max_resident_blocks(pair, &resident);
  if (e != cudaSuccess) return cuda_fail(e, "occupancy of the persistent kernel");
  if (blocks <= 0 || blocks > resident) blocks = resident;
  if (pair == 2 && (blocks & 1)) blocks = blocks + 1 <= resident ? blocks + 1 : blocks - 1;
  if (blocks <= 0) return fail(PKT_ERR_UNSUPPORTED, "no CTA of the persistent kernel fits on device %d", device);
  *out = blocks;
  return PKT_OK;
}

int Runtime::trace_for(int n, cudaStream_t stream, unsigned long long** out) {
  *out = nullptr;
  if (!trace_enabled) return PKT_OK;
  if (n > trace_cap) {
    cudaFree(d_trace);
    d_trace = nullptr;
    trace_cap = 0;
    cudaError_t e = cudaMalloc(&d_trace, sizeof(unsigned long long) * kTraceWords * std::max(1, n));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(trace)");
    trace_cap = std::max(1, n);
  }
  cudaError_t e = cudaMemsetAsync(d_trace, 0, sizeof(unsigned long long) * kTraceWords * std::max(1, n), stream);
  if (e != cudaSuccess) return cuda_fail(e, "clear trace");
  trace_tasks = n;
  *out = d_trace;
  return PKT_OK;
}

int Runtime::fetch_trace(unsigned long long* out, int max_tasks, int* n) {
  cudaSetDevice(device);
  if (!d_trace) return fail(PKT_ERR_ARGS, "no traced launch (enable tracing first)");
  const int k = std::min(max_tasks, trace_tasks);
  cudaError_t e = cudaMemcpy(out, d_trace, sizeof(unsigned long long) * kTraceWords * k, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read trace");
  *n = k;
  return PKT_OK;
}

int Runtime::clock_stats(unsigned long long* out3, bool reset) {
  cudaSetDevice(device);
  if (!d_clock) return fail(PKT_ERR_ARGS, "runtime not initialized");
  if (out3) {
    cudaError_t e = cudaMemcpy(out3, d_clock, 3 * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "read clock words");
  }
  if (reset) {
    cudaError_t e = cudaMemset(d_clock, 0, 3 * sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_fail(e, "clear clock words");
  }
  return PKT_OK;
}

int Runtime::scan_tokens(const pkt_task* tasks, int n) {
  int mx = 0;
  for (int i = 0; i < n; ++i) {
    const pkt_task_header& h = tasks[i].header;
    mx = std::max({mx, int(h.buffer_read_id), int(h.buffer_write_id), int(h.ext_ids & 0xffffu),
                   int(h.ext_ids >> 16)});
  }
  return mx + 1;
}

int Runtime::submit_async(const pkt_task* tasks, int n, cudaStream_t stream, bool sync_copy) {
  if (n < 0 || (n > 0 && !tasks)) return fail(PKT_ERR_ARGS, "bad task list");
  if (n > max_tasks) return fail(PKT_ERR_ARGS, "%d tasks exceed capacity %d", n, max_tasks);
  cudaSetDevice(device);
  int rc = ensure_tokens(scan_tokens(tasks, n));
  if (rc) return rc;
  num_tokens = token_cap;
  if (n > 0) {
    cudaError_t e = sync_copy ? cudaMemcpy(d_tasks, tasks, sizeof(pkt_task) * n, cudaMemcpyHostToDevice)
                              : cudaMemcpyAsync(d_tasks, tasks, sizeof(pkt_task) * n,
                                                cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return cuda_fail(e, "copy tasks");
  }
  num_tasks = n;
  return reset_state(stream, sync_copy);
}

int Runtime::reset_state(cudaStream_t stream, bool sync) {
  cudaError_t e = sync ? cudaMemset(d_state, 0, sizeof(int) * state_ints(num_tokens))
                       : cudaMemsetAsync(d_state, 0, sizeof(int) * state_ints(num_tokens), stream);
  if (e != cudaSuccess) return cuda_fail(e, "reset token state");
  if (accounting) {
    e = sync ? cudaMemset(d_counter, 0, sizeof(unsigned long long))
             : cudaMemsetAsync(d_counter, 0, sizeof(unsigned long long), stream);
    if (e != cudaSuccess) return cuda_fail(e, "reset task counter");
  }
  return PKT_OK;
}

int Runtime::launch(int blocks, cudaStream_t stream) {
  KParams p{};
  int rc = prepare(blocks, stream, &p, &blocks);
  if (rc) return rc;
  cudaError_t e = launch_megakernel(p, blocks, stream, cta_pair);
  if (e != cudaSuccess) return cuda_fail(e, "launch megakernel");
  return PKT_OK;
}

int Runtime::prepare(int blocks, cudaStream_t stream, KParams* out, int* out_blocks) {
  cudaSetDevice(device);
  if (!d_state) return fail(PKT_ERR_ARGS, "runtime not initialized");
  // pkt launches whatever grid it is given (include/runtime.hpp:175-228); a
  // persistent grid larger than what fits at once is clamped here, and an odd
  // count in pair mode is rounded to whole clusters.
  if (blocks <= 0) blocks = num_sms;
  int rc = clamp_blocks(blocks, cta_pair, &blocks);
  if (rc) return rc;
  if (perf_enabled && blocks + 1 > perf_cap) {
    cudaFree(d_perf);
    cudaError_t e = cudaMalloc(&d_perf, sizeof(unsigned long long) * PKT_PERF_WORDS * (blocks + 1));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(perf)");
    perf_cap = blocks + 1;
  }
  if (perf_enabled) cudaMemsetAsync(d_perf, 0, sizeof(unsigned long long) * PKT_PERF_WORDS * perf_cap, stream);
  KParams p{};
  p.tasks = d_tasks;
  p.num_tasks = num_tasks;
  p.num_tokens = num_tokens;
  p.state = d_state;
  p.gemms = d_gemms;
  p.num_gemms = num_gemms;
  p.chunk = 1;
  p.task_counter = accounting ? d_counter : nullptr;
  p.perf = perf_enabled ? d_perf : nullptr;
  p.timeout_ns = timeout_ns;
  p.clock_acc = d_clock;
  rc = trace_for(num_tasks, stream, &p.trace);
  if (rc) return rc;
  last_blocks = blocks;
  *out = p;
  *out_blocks = blocks;
  return PKT_OK;
}

int Runtime::status(int* code, int* task, int* detail) {
  cudaSetDevice(device);
  int h[4] = {0, 0, 0, 0};
  cudaError_t e = cudaMemcpy(h, d_state, sizeof(h), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  if (code) *code = h[1];
  if (task) *task = h[2];
  if (detail) *detail = h[3];
  return PKT_OK;
}

int Runtime::register_gemms(const pkt_gemm_desc* descs, int n, int* first) {
  cudaSetDevice(device);
  std::vector<DevGemm> add(n);
  for (int i = 0; i < n; ++i) {
    int rc = build_dev_gemm(descs[i], &add[i]);
    if (rc) return rc;
  }
  if (num_gemms + n > gemm_cap) {
    int cap = std::max(16, gemm_cap);
    while (cap < num_gemms + n) cap *= 2;
    DevGemm* ng = nullptr;
    cudaError_t e = cudaMalloc(&ng, sizeof(DevGemm) * cap);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(gemm table)");
    if (num_gemms) cudaMemcpy(ng, d_gemms, sizeof(DevGemm) * num_gemms, cudaMemcpyDeviceToDevice);
    cudaFree(d_gemms);
    d_gemms = ng;
    gemm_cap = cap;
  }
  cudaError_t e = cudaMemcpy(d_gemms + num_gemms, add.data(), sizeof(DevGemm) * n, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "copy gemm table");
  host_gemms.insert(host_gemms.end(), add.begin(), add.end());
  if (first) *first = num_gemms;
  num_gemms += n;
  return PKT_OK;
}

int Runtime::create(int dev, Runtime** out) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (dev < 0 || dev >= count) return fail(PKT_ERR_ARGS, "device %d out of range (%d devices)", dev, count);
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (prop.major != 10) return fail(PKT_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", dev, prop.major, prop.minor);
  Runtime* r = new Runtime();
  r->device = dev;
  r->num_sms = prop.multiProcessorCount;
  int rc = r->initialize(0);
  if (rc) {
    delete r;
    return rc;
  }
  *out = r;
  return PKT_OK;
}

}  // namespace pkb

// ======================================================================= C-ABI
using pkb::Runtime;
struct pkt_runtime {
  Runtime* rt;
};

extern "C" {

const char* pkt_last_error(void) { return pkb::g_last_error.c_str(); }

int pkt_num_sms(int device) {
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return pkb::cuda_fail(e, "cudaGetDeviceProperties");
  return prop.multiProcessorCount;
}

int pkt_runtime_create(int device, pkt_runtime** out) {
  if (!out) return pkb::fail(PKT_ERR_ARGS, "null out");
  Runtime* r = nullptr;
  int rc = Runtime::create(device, &r);
  if (rc) return rc;
  *out = new pkt_runtime{r};
  return PKT_OK;
}

int pkt_runtime_destroy(pkt_runtime* rt) {
  if (!rt) return PKT_OK;
  delete rt->rt;
  delete rt;
  return PKT_OK;
}

int pkt_runtime_initialize(pkt_runtime* rt, int max_tasks) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  return rt->rt->initialize(max_tasks);
}

int pkt_runtime_submit(pkt_runtime* rt, const pkt_task* tasks, int n) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  return rt->rt->submit_async(tasks, n, nullptr, true);
}

int pkt_runtime_submit_async(pkt_runtime* rt, const pkt_task* tasks, int n, void* stream) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  return rt->rt->submit_async(tasks, n, static_cast<cudaStream_t>(stream), false);
}

int pkt_runtime_set_segments(pkt_runtime* rt, const int* pairs, int n) {
  if (!rt || n < 0 || (n > 0 && !pairs)) return pkb::fail(PKT_ERR_ARGS, "bad segments");
  rt->rt->segments.assign(pairs, pairs + 2 * n);
  return PKT_OK;
}

int pkt_runtime_set_segment_window_size(pkt_runtime* rt, int window) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  rt->rt->segment_window = window;
  return PKT_OK;
}

int pkt_runtime_launch(pkt_runtime* rt, int num_blocks, void* stream) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  return rt->rt->launch(num_blocks, static_cast<cudaStream_t>(stream));
}

int pkt_runtime_synchronize(pkt_runtime* rt) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  cudaSetDevice(rt->rt->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return pkb::cuda_fail(e, "cudaDeviceSynchronize");
  int code = 0, task = 0, detail = 0;
  int rc = rt->rt->status(&code, &task, &detail);
  if (rc) return rc;
  if (code == PKT_DEV_TIMEOUT_DEPS || code == PKT_DEV_TIMEOUT_PIPE)
    return pkb::fail(PKT_ERR_TIMEOUT, "device wait timed out (code %d, task %d, detail %d)", code, task, detail);
  if (code == PKT_DEV_BAD_OPCODE)
    return pkb::fail(PKT_ERR_OPCODE, "unknown opcode %d at task %d", detail, task);
  if (code != 0) return pkb::fail(PKT_ERR_ARGS, "device rejected task %d (code %d, detail %d)", task, code, detail);
  return PKT_OK;
}

int pkt_runtime_status(pkt_runtime* rt, int* code, int* task_index, int* detail) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  return rt->rt->status(code, task_index, detail);
}

int pkt_runtime_register_gemms(pkt_runtime* rt, const pkt_gemm_desc* descs, int n, int* first_id) {
  if (!rt || n <= 0 || !descs) return pkb::fail(PKT_ERR_ARGS, "bad gemm registration");
  return rt->rt->register_gemms(descs, n, first_id);
}

int pkt_runtime_clear_gemms(pkt_runtime* rt) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  rt->rt->num_gemms = 0;
  rt->rt->host_gemms.clear();
  return PKT_OK;
}

int pkt_gemm_tiles(const pkt_gemm_desc* d, int* tiles_m, int* tiles_n) {
  if (!d || !tiles_m || !tiles_n) return pkb::fail(PKT_ERR_ARGS, "null argument");
  return pkb::gemm_tiles(*d, tiles_m, tiles_n);
}

int pkt_runtime_set_timeout_ns(pkt_runtime* rt, unsigned long long ns) {
  if (!rt || ns == 0) return pkb::fail(PKT_ERR_ARGS, "bad timeout");
  rt->rt->timeout_ns = ns;
  return PKT_OK;
}

int pkt_runtime_set_cta_pair(pkt_runtime* rt, int pair) {
  if (!rt || (pair != 1 && pair != 2)) return pkb::fail(PKT_ERR_ARGS, "cta pair must be 1 or 2");
  rt->rt->cta_pair = pair;
  return PKT_OK;
}

int pkt_runtime_set_task_accounting(pkt_runtime* rt, int enabled) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  rt->rt->accounting = enabled != 0;
  return PKT_OK;
}

int pkt_runtime_fetch_task_counter(pkt_runtime* rt, unsigned long long* out) {
  if (!rt || !out) return pkb::fail(PKT_ERR_ARGS, "null argument");
  if (!rt->rt->accounting) return pkb::fail(PKT_ERR_ARGS, "task accounting is off");
  cudaSetDevice(rt->rt->device);
  cudaError_t e = cudaMemcpy(out, rt->rt->d_counter, sizeof(*out), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return pkb::cuda_fail(e, "read task counter");
  return PKT_OK;
}

int pkt_runtime_set_perf(pkt_runtime* rt, int enabled) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  rt->rt->perf_enabled = enabled != 0;
  return PKT_OK;
}

int pkt_runtime_fetch_perf(pkt_runtime* rt, unsigned long long* out, int max_blocks, int* blocks) {
  if (!rt || !out || !blocks) return pkb::fail(PKT_ERR_ARGS, "null argument");
  if (!rt->rt->perf_enabled || !rt->rt->d_perf) return pkb::fail(PKT_ERR_ARGS, "perf counters are off");
  const int nb = std::min(max_blocks, rt->rt->last_blocks);
  cudaSetDevice(rt->rt->device);
  cudaError_t e = cudaMemcpy(out, rt->rt->d_perf, sizeof(unsigned long long) * PKT_PERF_WORDS * nb,
                             cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return pkb::cuda_fail(e, "read perf");
  *blocks = nb;
  return PKT_OK;
}

int pkt_runtime_last_launch_blocks(pkt_runtime* rt) { return rt ? rt->rt->last_blocks : 0; }

int pkt_runtime_set_trace(pkt_runtime* rt, int enabled) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  rt->rt->trace_enabled = enabled != 0;
  return PKT_OK;
}

int pkt_runtime_fetch_trace(pkt_runtime* rt, unsigned long long* out, int max_tasks, int* n) {
  if (!rt || !out || !n) return pkb::fail(PKT_ERR_ARGS, "null argument");
  return rt->rt->fetch_trace(out, max_tasks, n);
}

int pkt_runtime_prepare_launch(pkt_runtime* rt, int num_blocks, void* stream, void* kparams, int kparams_bytes,
                               int* blocks, int* pair) {
  if (!rt || !kparams || !blocks || !pair) return pkb::fail(PKT_ERR_ARGS, "null argument");
  if (kparams_bytes != int(sizeof(pkb::KParams)))
    return pkb::fail(PKT_ERR_ARGS, "kernel parameter block is %d bytes here, %d in the caller's headers",
                     int(sizeof(pkb::KParams)), kparams_bytes);
  int rc = rt->rt->prepare(num_blocks, static_cast<cudaStream_t>(stream), static_cast<pkb::KParams*>(kparams), blocks);
  if (rc) return rc;
  *pair = rt->rt->cta_pair;
  return PKT_OK;
}

int pkt_runtime_clock_stats(pkt_runtime* rt, unsigned long long* out3, int reset) {
  if (!rt) return pkb::fail(PKT_ERR_ARGS, "null runtime");
  return rt->rt->clock_stats(out3, reset != 0);
}

}  // extern "C"
