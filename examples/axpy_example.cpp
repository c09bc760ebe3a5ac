// The axpy demo of pkt (examples/axpy_example.cu) on the B200 runtime: 1000 Axpy
// tasks of 1024 floats, one persistent launch on every SM, checked against the
// host and reported in GB/s (12 bytes per element: read x, read y, write y).
//   axpy_example [--tasks N] [--per-task N] [--alpha A]
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <random>
#include <vector>

#include "pk/ops/axpy.cuh"
#include "pk/runtime.hpp"

int main(int argc, char** argv) {
  int num_tasks = 1000, per_task = 1024;
  float alpha = 2.5f;
  for (int i = 1; i + 1 < argc; i += 2) {
    if (!std::strcmp(argv[i], "--tasks")) num_tasks = std::atoi(argv[i + 1]);
    else if (!std::strcmp(argv[i], "--per-task")) per_task = std::atoi(argv[i + 1]);
    else if (!std::strcmp(argv[i], "--alpha")) alpha = std::strtof(argv[i + 1], nullptr);
  }
  const size_t n = size_t(num_tasks) * per_task;
  std::cout << "Megakernel AXPY Example (B200)\n";
  std::cout << "Tasks: " << num_tasks << "\nElements per task: " << per_task << "\n\n";
  std::vector<float> hx(n), hy(n), ref(n);
  std::mt19937 rng(42);
  std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
  for (size_t i = 0; i < n; ++i) {
    hx[i] = dist(rng);
    hy[i] = dist(rng);
    ref[i] = std::fmaf(alpha, hx[i], hy[i]);
  }
  float *dx = nullptr, *dy = nullptr;
  if (cudaMalloc(&dx, n * 4) != cudaSuccess || cudaMalloc(&dy, n * 4) != cudaSuccess) {
    std::cerr << "cudaMalloc failed\n";
    return 2;
  }
  cudaMemcpy(dx, hx.data(), n * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dy, hy.data(), n * 4, cudaMemcpyHostToDevice);
  pk::Runtime runtime;
  runtime.initialize(num_tasks);
  std::vector<pk::Task> tasks(num_tasks);
  for (int i = 0; i < num_tasks; ++i)
    pk::encode_args(tasks[i], pk::OpCode::Axpy,
                    pk::AxpyArgs{dx + size_t(i) * per_task, dy + size_t(i) * per_task, alpha, per_task});
  runtime.submit_tasks(tasks);
  const int sms = pk::Runtime::get_num_sms();
  std::cout << "Launching on " << sms << " SMs\n";
  cudaEvent_t start, stop;
  cudaEventCreate(&start);
  cudaEventCreate(&stop);
  cudaEventRecord(start);
  runtime.launch(sms);
  cudaEventRecord(stop);
  runtime.synchronize();
  if (runtime.last_error() != PKT_OK) {
    std::cerr << "runtime error: " << runtime.last_error_string() << "\n";
    return 1;
  }
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, start, stop);
  cudaMemcpy(hy.data(), dy, n * 4, cudaMemcpyDeviceToHost);
  float max_error = 0.0f;
  for (size_t i = 0; i < n; ++i) max_error = std::max(max_error, std::fabs(hy[i] - ref[i]));
  std::cout << "\nResults:\n--------\n";
  std::cout << "Time: " << ms << " ms\n";
  std::cout << "Throughput: " << (n * 12.0 / ms / 1e6) << " GB/s\n";
  std::cout << "Max error: " << max_error << "\n";
  std::cout << "Status: " << (max_error == 0.0f ? "PASSED" : "FAILED") << "\n";
  cudaFree(dx);
  cudaFree(dy);
  return max_error == 0.0f ? 0 : 1;
}
