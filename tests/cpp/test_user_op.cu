// A program's own op in the persistent megakernel through pkt's plugin point
// (pk::OpTraits<Code> with load / compute / store, launched by
// pk::launch_with_ops): the op stages its input in a shared-memory page in the
// load phase, computes into a second page with all four compute warps, stores in
// the store phase, and depends on a built-in Axpy task through a token.
// Results are compared with the host bit for bit.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "check.hpp"
#include "pk/kernel.cuh"
#include "pk/ops/axpy.cuh"

namespace pk {

constexpr OpCode kScaleShift = OpCode(100);

struct ScaleShiftArgs {
  const float* x;
  float* y;
  float a, b;
  int n;  // <= 1024: one 4 KB page
};

// y = a * x + b, staged through pages 0 (x) and 1 (y) of the task's slot.
template <>
struct OpTraits<kScaleShift> {
  using Args = ScaleShiftArgs;

  __device__ static void load(const Args& args, BlockRuntime& br, int slot, int lane,
                              unsigned long long* reuse, unsigned long long* refill) {
    (void)reuse;
    (void)refill;
    const PageHandle xp = br.page_handle(slot, 0);
    const unsigned long long tag = make_page_tag(args.x, args.n, 0, 0);
    if (br.page_is_ready_with_tag(xp, tag)) return;  // staged by the previous task
    br.page_wait_begin_overwrite(xp);
    float* sx = br.page_ptr<float>(xp);
    for (int i = lane; i < args.n; i += Config::kWarpSize) sx[i] = args.x[i];
    __syncwarp();
    if (lane == 0) br.page_publish(xp, tag);
    __syncwarp();
  }

  __device__ static void compute(const Args& args, BlockRuntime& br, int slot, int lane, int cwarp, int ncwarps) {
    const float* sx = br.page_ptr<float>(br.page_handle(slot, 0));
    float* sy = br.page_ptr<float>(br.page_handle(slot, 1));
    for (int i = cwarp * Config::kWarpSize + lane; i < args.n; i += ncwarps * Config::kWarpSize)
      sy[i] = fmaf(args.a, sx[i], args.b);
  }

  __device__ static void store(const Args& args, BlockRuntime& br, int slot, int lane) {
    const float* sy = br.page_ptr<float>(br.page_handle(slot, 1));
    for (int i = lane; i < args.n; i += Config::kWarpSize) args.y[i] = sy[i];
  }
};

}  // namespace pk

using namespace pk;

static float *dx, *dy, *dz;
static const int kChunk = 1000, kChunks = 300, kN = kChunk * kChunks;
static std::vector<float> hx(kN), hy(kN);

static bool setup() {
  int ndev = 0;
  CHECK(cudaGetDeviceCount(&ndev) == cudaSuccess && ndev > 0, "no CUDA device");
  std::mt19937 rng(7);
  std::uniform_real_distribution<float> u(-1.f, 1.f);
  for (int i = 0; i < kN; ++i) {
    hx[i] = u(rng);
    hy[i] = u(rng);
  }
  CHECK(cudaMalloc(&dx, kN * 4) == cudaSuccess && cudaMalloc(&dy, kN * 4) == cudaSuccess &&
            cudaMalloc(&dz, kN * 4) == cudaSuccess, "cudaMalloc");
  cudaMemcpy(dx, hx.data(), kN * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dy, hy.data(), kN * 4, cudaMemcpyHostToDevice);
  cudaMemset(dz, 0, kN * 4);
  return true;
}

// chunk c: built-in Axpy y_c = 2 x_c + y_c (publishes token 1 + c), then the
// program's op z_c = 0.5 y_c - 1 (waits for that token), twice over the same y_c
// (the second finds it staged: same tag)
static bool user_op_after_builtin_op() {
  std::vector<Task> tasks;
  const float a = 2.0f, s = 0.5f, t = -1.0f;
  for (int c = 0; c < kChunks; ++c) {
    Task ax{};
    encode_args(ax, OpCode::Axpy, AxpyArgs{dx + c * kChunk, dy + c * kChunk, a, kChunk});
    ax.header.buffer_write_id = uint16_t(1 + c);
    tasks.push_back(ax);
  }
  for (int c = 0; c < kChunks; ++c)
    for (int rep = 0; rep < 2; ++rep) {
      Task op{};
      encode_args(op, kScaleShift, ScaleShiftArgs{dy + c * kChunk, dz + c * kChunk, s, t, kChunk});
      op.header.buffer_read_id = uint16_t(1 + c);
      op.header.wait_count = 1;
      tasks.push_back(op);
    }
  Runtime rt;
  rt.initialize(int(tasks.size()));
  rt.submit_tasks(tasks);
  CHECK(launch_with_ops<kScaleShift>(rt) == 0, "launch_with_ops");
  rt.synchronize();
  CHECK(rt.last_error() == 0, rt.last_error_string().c_str());
  std::vector<float> gz(kN), gy(kN);
  cudaMemcpy(gz.data(), dz, kN * 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(gy.data(), dy, kN * 4, cudaMemcpyDeviceToHost);
  int bad = 0;
  for (int i = 0; i < kN; ++i) {
    const float y1 = std::fma(a, hx[i], hy[i]);
    const float z = std::fma(s, y1, t);
    if (gy[i] != y1 || gz[i] != z) ++bad;
  }
  CHECK(bad == 0, "results differ from the host");
  return true;
}

// an opcode the instantiation does not list is still rejected
static bool unlisted_opcode_rejected() {
  Runtime rt;
  std::vector<Task> one(1);
  encode_args(one[0], OpCode(101), ScaleShiftArgs{dy, dz, 0.5f, -1.0f, 4});
  rt.initialize(1);
  rt.submit_tasks(one);
  CHECK(launch_with_ops<kScaleShift>(rt) == 0, "launch_with_ops");
  rt.synchronize();
  CHECK(rt.last_error() == PKT_ERR_OPCODE, "unknown opcode not reported");
  return true;
}

int main() {
  const Case cases[] = {{"setup", setup},
                        {"user_op_after_builtin_op", user_op_after_builtin_op},
                        {"unlisted_opcode_rejected", unlisted_opcode_rejected}};
  return run_cases(cases, 3);
}
