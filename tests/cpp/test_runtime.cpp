// pk::Runtime on the GPU: the integration cases of pkt's tests/test_runtime.cu,
// tests/test_axpy.cu and tests/test_paging.cu, restated against the drop-in
// headers. Axpy results must equal fmaf(a, x, y) bit for bit.
#include <cuda_runtime.h>

#include <cmath>
#include <random>
#include <vector>

#include "check.hpp"
#include "pk/ops/axpy.cuh"
#include "pk/ops/linear_fwd.cuh"
#include "pk/runtime.hpp"

using namespace pk;

static bool have_gpu() {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
}

// Runs `ntasks` Axpy tasks of n elements each and compares with fmaf on the host.
static bool run_axpy(int ntasks, int n, float a, int blocks, unsigned seed) {
  const size_t total = size_t(ntasks) * n;
  std::vector<float> hx(total), hy(total), ref(total);
  std::mt19937 rng(seed);
  std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
  for (size_t i = 0; i < total; ++i) {
    hx[i] = dist(rng);
    hy[i] = dist(rng);
    ref[i] = std::fmaf(a, hx[i], hy[i]);
  }
  float *dx = nullptr, *dy = nullptr;
  CHECK(cudaMalloc(&dx, total * 4) == cudaSuccess && cudaMalloc(&dy, total * 4) == cudaSuccess, "malloc");
  cudaMemcpy(dx, hx.data(), total * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dy, hy.data(), total * 4, cudaMemcpyHostToDevice);
  Runtime rt;
  rt.initialize(ntasks);
  std::vector<Task> tasks(ntasks);
  for (int i = 0; i < ntasks; ++i)
    encode_args(tasks[i], OpCode::Axpy, AxpyArgs{dx + size_t(i) * n, dy + size_t(i) * n, a, n});
  rt.set_task_accounting_enabled(true);
  rt.submit_tasks(tasks);
  rt.launch(blocks);
  rt.synchronize();
  unsigned long long issued = 0;
  const bool counted = rt.fetch_task_counter(&issued);
  cudaMemcpy(hy.data(), dy, total * 4, cudaMemcpyDeviceToHost);
  cudaFree(dx);
  cudaFree(dy);
  CHECK(rt.last_error() == PKT_OK, rt.last_error_string().c_str());
  CHECK(counted && issued == static_cast<unsigned long long>(ntasks), "every task issued once");
  for (size_t i = 0; i < total; ++i) CHECK(hy[i] == ref[i], "axpy bit-exact");
  return true;
}

static bool gpu_present() {
  CHECK(have_gpu(), "a CUDA device is required");
  return true;
}
static bool axpy_sizes() {
  for (int n : {32, 128, 512, 1024, 2048}) CHECK(run_axpy(1, n, 2.5f, 1, 42), "size");
  return true;
}
static bool axpy_alpha_zero_and_negative() {
  return run_axpy(100, 1024, 0.0f, 0, 123) && run_axpy(100, 1024, -1.5f, 0, 0);
}
static bool axpy_1000_tiny_tasks() { return run_axpy(1000, 32, 2.0f, 0, 999); }
static bool block_counts() {
  for (int b : {1, 2, 4, 8, 16}) CHECK(run_axpy(100, 333, 0.5f, b, 777), "block count");
  return true;
}
static bool tasks_5000() { return run_axpy(5000, 64, 1.25f, 0, 4); }

static bool empty_list() {
  Runtime rt;
  rt.initialize(10);
  rt.submit_tasks({});
  rt.launch(1);
  rt.synchronize();
  CHECK(rt.last_error() == PKT_OK, rt.last_error_string().c_str());
  return true;
}

static bool num_sms() {
  const int n = Runtime::get_num_sms();
  CHECK(n > 0 && n < 1000, "plausible SM count");
  return true;
}

static bool resubmission() {
  const int n = 256;
  std::vector<float> ones(n, 1.0f), zeros(n, 0.0f), out(n);
  float *dx, *dy;
  cudaMalloc(&dx, n * 4);
  cudaMalloc(&dy, n * 4);
  cudaMemcpy(dx, ones.data(), n * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dy, zeros.data(), n * 4, cudaMemcpyHostToDevice);
  Runtime rt;
  rt.initialize(1);
  std::vector<Task> t(1);
  encode_args(t[0], OpCode::Axpy, AxpyArgs{dx, dy, 1.0f, n});
  for (int r = 0; r < 3; ++r) {
    rt.submit_tasks(t);
    rt.launch(1);
    rt.synchronize();
  }
  cudaMemcpy(out.data(), dy, n * 4, cudaMemcpyDeviceToHost);
  cudaFree(dx);
  cudaFree(dy);
  for (float v : out) CHECK(v == 3.0f, "three submissions give 3");
  return true;
}

static bool linear_forward_identity() {
  const int m = 8, n = 8, batch = 2;
  std::vector<float> W(m * n, 0.0f), x(batch * n), y(batch * m, 0.0f);
  for (int i = 0; i < m; ++i) W[i * n + i] = 1.0f;
  for (int b = 0; b < batch; ++b)
    for (int j = 0; j < n; ++j) x[b * n + j] = float(j + 1);
  float *dW, *dx, *dy;
  cudaMalloc(&dW, W.size() * 4);
  cudaMalloc(&dx, x.size() * 4);
  cudaMalloc(&dy, y.size() * 4);
  cudaMemcpy(dW, W.data(), W.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dx, x.data(), x.size() * 4, cudaMemcpyHostToDevice);
  cudaMemset(dy, 0, y.size() * 4);
  Runtime rt;
  rt.initialize(1);
  std::vector<Task> t(1);
  encode_args(t[0], OpCode::LinearForward, LinearForwardArgs{dW, dx, dy, batch, m, n, 0, batch, 0, m});
  rt.submit_tasks(t);
  rt.launch(1);
  rt.synchronize();
  cudaMemcpy(y.data(), dy, y.size() * 4, cudaMemcpyDeviceToHost);
  cudaFree(dW);
  cudaFree(dx);
  cudaFree(dy);
  for (int b = 0; b < batch; ++b)
    for (int i = 0; i < m; ++i) CHECK(std::fabs(y[b * m + i] - x[b * n + i]) < 1e-5f, "y = x");
  return true;
}

static bool bad_dependency_reports_timeout() {
  float* d;
  cudaMalloc(&d, 64 * 4);
  Runtime rt;
  rt.initialize(1);
  rt.set_timeout_ns(50000000ull);
  std::vector<Task> t(1);
  encode_args(t[0], OpCode::Axpy, AxpyArgs{d, d, 1.0f, 64});
  t[0].header.buffer_read_id = 9;
  t[0].header.wait_count = 1;
  rt.submit_tasks(t);
  rt.launch(1);
  rt.synchronize();
  cudaFree(d);
  CHECK(rt.last_error() == PKT_ERR_TIMEOUT, "synchronize reports the timeout");
  int code = 0, task = -1, detail = 0;
  rt.status(&code, &task, &detail);
  CHECK(code == PKT_DEV_TIMEOUT_DEPS && task == 0 && detail == 9, "status word names task and token");
  return true;
}

int main() {
  Case cs[] = {{"gpu_present", gpu_present},
               {"empty_list", empty_list},
               {"num_sms", num_sms},
               {"axpy_sizes", axpy_sizes},
               {"axpy_alpha_zero_and_negative", axpy_alpha_zero_and_negative},
               {"axpy_1000_tiny_tasks", axpy_1000_tiny_tasks},
               {"block_counts", block_counts},
               {"tasks_5000", tasks_5000},
               {"resubmission", resubmission},
               {"linear_forward_identity", linear_forward_identity},
               {"bad_dependency_reports_timeout", bad_dependency_reports_timeout}};
  return run_cases(cs, sizeof(cs) / sizeof(cs[0]));
}
