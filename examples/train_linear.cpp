// pkt's train_linear demo (examples/train_linear.cu) on the B200 build.
//
// --engine tasks (default): pkt's own task DAG for y = x W^T — per step: zero
//   loss, LinearForward tiles, MSELoss, zero dW, LinearBackward tiles,
//   SGDUpdate — built with pk::encode_args and pkt's token / epoch bookkeeping
//   and run in ONE persistent launch by pk::Runtime (the drop-in path). Each
//   step's loss goes to its own slot so the whole curve comes back.
// --engine mlp: the same problem (or --layers a,b,c for an MLP, --bias) on the
//   tcgen05 MLP engine (pkt_mlp_*), TF32 or bf16.
// Output lines follow pkt's ("CPU final loss:", "Time:", "Time per step:",
// "Final loss (host recompute):") so scripts that parse pkt's output work.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <fstream>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "pk/ops/linear_bwd.cuh"
#include "pk/ops/linear_fwd.cuh"
#include "pk/ops/mse.cuh"
#include "pk/ops/sgd.cuh"
#include "pk/ops/zero.cuh"
#include "pk/runtime.hpp"

namespace {

// pkt's generator (mt19937(42); W ~ N(0, 2/(m+n)); x ~ N(0,1); target = W x + N(0, 0.01^2)).
void make_data(int m, int n, int batch, std::vector<float>& W, std::vector<float>& x,
               std::vector<float>& t) {
  std::mt19937 rng(42);
  std::normal_distribution<float> wd(0.0f, std::sqrt(2.0f / float(m + n))), xd(0.0f, 1.0f),
      nd(0.0f, 0.01f);
  W.resize(size_t(m) * n);
  x.resize(size_t(batch) * n);
  t.resize(size_t(batch) * m);
  for (auto& v : W) v = wd(rng);
  for (auto& v : x) v = xd(rng);
  for (int b = 0; b < batch; ++b)
    for (int i = 0; i < m; ++i) {
      float acc = 0.f;
      for (int j = 0; j < n; ++j) acc += W[size_t(i) * n + j] * x[size_t(b) * n + j];
      t[size_t(b) * m + i] = acc + nd(rng);
    }
}

float host_loss(const std::vector<float>& W, const std::vector<float>& x, const std::vector<float>& t,
                int batch, int m, int n) {
  double acc = 0.0;
  for (int b = 0; b < batch; ++b)
    for (int i = 0; i < m; ++i) {
      float y = 0.f;
      for (int j = 0; j < n; ++j) y += W[size_t(i) * n + j] * x[size_t(b) * n + j];
      const double d = double(y) - t[size_t(b) * m + i];
      acc += d * d;
    }
  return float(acc / (double(batch) * m));
}

// pkt's host training loop, float accumulation in pkt's loop order.
float cpu_train(std::vector<float> W, const std::vector<float>& x, const std::vector<float>& t,
                int batch, int m, int n, int steps, float lr) {
  std::vector<float> y(size_t(batch) * m), dy(size_t(batch) * m);
  float loss = 0.f;
  for (int s = 0; s < steps; ++s) {
    for (int b = 0; b < batch; ++b)
      for (int i = 0; i < m; ++i) {
        float acc = 0.f;
        for (int j = 0; j < n; ++j) acc += W[size_t(i) * n + j] * x[size_t(b) * n + j];
        y[size_t(b) * m + i] = acc;
      }
    loss = 0.f;
    const float scale = 2.0f / float(batch * m);
    for (int i = 0; i < batch * m; ++i) {
      const float d = y[i] - t[i];
      dy[i] = scale * d;
      loss += d * d;
    }
    loss /= float(batch * m);
    for (int i = 0; i < m; ++i)
      for (int j = 0; j < n; ++j) {
        float g = 0.f;
        for (int b = 0; b < batch; ++b) g += dy[size_t(b) * m + i] * x[size_t(b) * n + j];
        W[size_t(i) * n + j] -= lr * g;
      }
  }
  return loss;
}

struct Opts {
  int m = 1024, n = 1024, batch = 64, steps = 20, fwd_tm = 2, fwd_tn = 128, bwd_tm = 64, bwd_tn = 128;
  int blocks = -1, repeats = 1, seg_window = 0;
  float lr = 1e-3f;
  bool skip_cpu = false, check_loss = false, check_tasks = false, bias = false;
  bool perf = false, print_profile = false;
  std::string engine = "tasks", dtype = "tf32", layers, perf_json;
};

// Per-role summary of the per-CTA counters of one launch (pkt's --perf report,
// examples/train_linear.cu:724-895), in ms per step averaged over CTAs (cycles
// converted with the launch's measured SM clock), and --perf-json.
int report_perf(const std::vector<pk::PerfBlock>& blocks, double sm_mhz, float step_ms, int steps,
                const Opts& o) {
  if (blocks.empty()) {
    std::cerr << "Failed to fetch perf counters.\n";
    return 3;
  }
  pk::PerfBlock tot{};
  unsigned long long tmin = ~0ull, tmax = 0;
  for (const pk::PerfBlock& b : blocks) {
    const unsigned long long* src = reinterpret_cast<const unsigned long long*>(&b);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(&tot);
    for (size_t i = 0; i < sizeof(pk::PerfBlock) / 8; ++i) dst[i] += src[i];
    tmin = std::min(tmin, b.tasks_issued);
    tmax = std::max(tmax, b.tasks_issued);
  }
  const double nb = double(blocks.size());
  auto ms = [&](unsigned long long cyc) { return double(cyc) / nb / (sm_mhz * 1e3) / steps; };
  struct Row {
    const char* name;
    unsigned long long cyc;
  };
  const Row rows[] = {{"controller.deps_wait", tot.ctrl_wait_cycles},
                      {"controller.slot_wait", tot.ctrl_slot_wait_cycles},
                      {"loader.stage_wait", tot.load_wait_slot_cycles},
                      {"mma.stage_wait", tot.mma_full_wait_cycles},
                      {"mma.accumulator_wait", tot.mma_tmem_wait_cycles},
                      {"mma.issue", tot.mma_issue_cycles},
                      {"compute.accumulator_wait", tot.compute_wait_loaded_cycles},
                      {"compute.gemm_epilogue", tot.compute_work_cycles},
                      {"compute.elementwise", tot.simt_work_cycles},
                      {"total", tot.total_cycles}};
  std::cout << "\nPer-role counters (averaged per CTA, per step; SM clock " << sm_mhz << " MHz):\n";
  std::cout << "  blocks: " << blocks.size() << "  steps: " << steps << "  step_ms: " << step_ms << "\n";
  std::cout << "  tasks per CTA: min " << tmin << " max " << tmax << "  GEMM tiles: " << tot.gemm_tiles << "\n";
  for (const Row& r : rows) {
    const double v = ms(r.cyc);
    std::cout << "  " << r.name << ": " << v << " ms (" << (step_ms > 0 ? 100.0 * v / step_ms : 0.0) << "%)\n";
  }
  if (!o.perf_json.empty()) {
    std::ofstream out(o.perf_json);
    if (!out) {
      std::cerr << "Failed to open --perf-json path: " << o.perf_json << "\n";
      return 3;
    }
    out << "{\n  \"blocks\": " << blocks.size() << ",\n  \"step_ms\": " << step_ms
        << ",\n  \"sm_mhz\": " << sm_mhz << ",\n  \"tasks_completed_min\": " << tmin
        << ",\n  \"tasks_completed_max\": " << tmax << ",\n  \"ratios\": {\n"
        << "    \"ctrl_wait_frac\": " << (tot.total_cycles ? double(tot.ctrl_wait_cycles) / tot.total_cycles : 0.0)
        << ",\n    \"mma_issue_frac\": " << (tot.total_cycles ? double(tot.mma_issue_cycles) / tot.total_cycles : 0.0)
        << ",\n    \"compute_work_frac\": "
        << (tot.total_cycles ? double(tot.compute_work_cycles + tot.simt_work_cycles) / tot.total_cycles : 0.0)
        << "\n  },\n  \"totals\": {\n";
    static const char* names[] = {"tasks_issued", "gemm_tiles", "ctrl_wait_cycles", "ctrl_slot_wait_cycles",
                                  "load_wait_slot_cycles", "mma_full_wait_cycles", "mma_tmem_wait_cycles",
                                  "compute_wait_loaded_cycles", "compute_work_cycles", "simt_work_cycles",
                                  "total_cycles", "mma_slot_wait_cycles", "mma_issue_cycles", "kblocks",
                                  "mma_gap_cycles", "mma_lifetime_cycles"};
    const unsigned long long* v = reinterpret_cast<const unsigned long long*>(&tot);
    for (int i = 0; i < 16; ++i) out << "    \"" << names[i] << "\": " << v[i] << (i < 15 ? ",\n" : "\n");
    out << "  }\n}\n";
  }
  return 0;
}

double clock_mhz(const unsigned long long c[3]) { return c[1] ? double(c[0]) * 1e3 / double(c[1]) : 0.0; }

bool parse(int argc, char** argv, Opts& o) {
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto val = [&]() -> const char* { return i + 1 < argc ? argv[++i] : ""; };
    if (a == "--m") o.m = std::atoi(val());
    else if (a == "--n") o.n = std::atoi(val());
    else if (a == "--batch") o.batch = std::atoi(val());
    else if (a == "--steps") o.steps = std::atoi(val());
    else if (a == "--lr") o.lr = std::strtof(val(), nullptr);
    else if (a == "--fwd-tile-m") o.fwd_tm = std::atoi(val());
    else if (a == "--fwd-tile-n") o.fwd_tn = std::atoi(val());
    else if (a == "--bwd-tile-m") o.bwd_tm = std::atoi(val());
    else if (a == "--bwd-tile-n") o.bwd_tn = std::atoi(val());
    else if (a == "--blocks") o.blocks = std::atoi(val());
    else if (a == "--skip-cpu") o.skip_cpu = true;
    else if (a == "--check-loss") o.check_loss = true;
    else if (a == "--check-tasks") o.check_tasks = true;
    else if (a == "--bias") o.bias = true;
    else if (a == "--engine") o.engine = val();
    else if (a == "--dtype") o.dtype = val();
    else if (a == "--layers") o.layers = val();
    else if (a == "--repeats") o.repeats = std::atoi(val());
    else if (a == "--seg-window") o.seg_window = std::atoi(val());
    else if (a == "--perf") o.perf = true;
    else if (a == "--perf-json") { o.perf = true; o.perf_json = val(); }
    else if (a == "--print-profile") { o.perf = true; o.print_profile = true; }
    else {
      std::cerr << "Unknown arg " << a << "\n";
      return false;
    }
  }
  return o.m > 0 && o.n > 0 && o.batch > 0 && o.steps > 0 && o.repeats > 0 && o.fwd_tm > 0 && o.fwd_tn > 0 &&
         o.bwd_tm > 0 && o.bwd_tn > 0 && (o.engine == "tasks" || o.engine == "mlp");
}

}  // namespace

namespace {

// pkt's single-Linear DAG (tokens: 1 loss-start, 2 grad-ready, 3 dW, 4 W).
int run_tasks(const Opts& o, std::vector<float>& W, const std::vector<float>& x,
              const std::vector<float>& t, std::vector<float>& losses, float& ms) {
  const int m = o.m, n = o.n, batch = o.batch;
  float *dW, *dx, *dy, *dt, *ddy, *ddW, *dloss;
  cudaMalloc(&dW, W.size() * 4);
  cudaMalloc(&dx, x.size() * 4);
  cudaMalloc(&dy, size_t(batch) * m * 4);
  cudaMalloc(&dt, t.size() * 4);
  cudaMalloc(&ddy, size_t(batch) * m * 4);
  cudaMalloc(&ddW, W.size() * 4);
  cudaMalloc(&dloss, size_t(o.steps) * 4);
  cudaMemcpy(dW, W.data(), W.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dx, x.data(), x.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dt, t.data(), t.size() * 4, cudaMemcpyHostToDevice);
  std::vector<pk::Task> tasks;
  auto add = [&](pk::Task tk, uint16_t rid, uint16_t wid, uint32_t wc, uint32_t re, uint32_t we) {
    tk.header.buffer_read_id = rid;
    tk.header.buffer_write_id = wid;
    tk.header.wait_count = wc;
    tk.header.read_epoch = re;
    tk.header.write_epoch = we;
    tasks.push_back(tk);
  };
  uint32_t r_loss = 0, r_grad = 0, r_dw = 0, r_w = 0, e_grad = 0, e_dw = 0, e_w = 0;
  for (int s = 0; s < o.steps; ++s) {
    const uint32_t ep = s + 1;
    pk::Task tk{};
    pk::encode_args(tk, pk::OpCode::ZeroMemory, pk::ZeroMemoryArgs{dloss + s, 1});
    add(tk, 0, 1, 0, 0, ep);
    ++r_loss;
    for (int ms0 = 0; ms0 < batch; ms0 += o.fwd_tm)
      for (int ns = 0; ns < m; ns += o.fwd_tn) {
        pk::encode_args(tk, pk::OpCode::LinearForward,
                        pk::LinearForwardArgs{dW, dx, dy, batch, m, n, ms0, std::min(o.fwd_tm, batch - ms0), ns,
                                              std::min(o.fwd_tn, m - ns)});
        add(tk, 4, 1, r_w, e_w, ep);
        ++r_loss;
      }
    pk::encode_args(tk, pk::OpCode::MSELoss, pk::MSELossArgs{dy, dt, ddy, dloss + s, batch, m});
    add(tk, 1, 2, r_loss, ep, ++e_grad);
    ++r_grad;
    pk::encode_args(tk, pk::OpCode::ZeroMemory, pk::ZeroMemoryArgs{ddW, m * n});
    add(tk, 0, 2, 0, 0, ++e_grad);
    ++r_grad;
    for (int ms0 = 0; ms0 < m; ms0 += o.bwd_tm)
      for (int ns = 0; ns < n; ns += o.bwd_tn) {
        pk::encode_args(tk, pk::OpCode::LinearBackward,
                        pk::LinearBackwardArgs{ddy, dx, ddW, batch, m, n, ms0, std::min(o.bwd_tm, m - ms0), ns,
                                               std::min(o.bwd_tn, n - ns)});
        add(tk, 2, 3, r_grad, e_grad, ++e_dw);
        ++r_dw;
      }
    pk::encode_args(tk, pk::OpCode::SGDUpdate, pk::SGDUpdateArgs{dW, ddW, o.lr, m * n});
    add(tk, 3, 4, r_dw, e_dw, ++e_w);
    ++r_w;
  }
  std::cout << "Tasks: " << tasks.size() << " (" << tasks.size() / o.steps << " per step), 1 launch\n";
  pk::Runtime rt;
  rt.initialize(int(tasks.size()));
  rt.set_task_accounting_enabled(o.check_tasks);
  rt.set_perf_enabled(o.perf);
  if (o.seg_window > 0) rt.set_segment_window_size(o.seg_window);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  // --repeats: the whole task list again from the same starting weights; the
  // fastest launch is reported (pkt reports per repeat)
  const std::vector<float> W0 = W;
  ms = 0.f;
  int rc = PKT_OK;
  for (int rep = 0; rep < o.repeats && rc == PKT_OK; ++rep) {
    if (rep) cudaMemcpy(dW, W0.data(), W0.size() * 4, cudaMemcpyHostToDevice);
    rt.submit_tasks(tasks);
    pkt_runtime_clock_stats(rt.handle(), nullptr, 1);
    cudaEventRecord(a);
    rt.launch(o.blocks > 0 ? o.blocks : pk::Runtime::get_num_sms());
    cudaEventRecord(b);
    rt.synchronize();
    float t = 0.f;
    cudaEventElapsedTime(&t, a, b);
    ms = rep == 0 ? t : std::min(ms, t);
    rc = rt.last_error();
  }
  if (!rc && o.perf) {
    unsigned long long clk[3] = {0, 0, 0};
    pkt_runtime_clock_stats(rt.handle(), clk, 0);
    std::vector<pk::PerfBlock> blocks;
    rt.fetch_perf_blocks(blocks);
    rc = report_perf(blocks, clock_mhz(clk), ms / o.steps, o.steps, o);
  }
  if (rc != PKT_OK) std::cerr << "runtime error: " << rt.last_error_string() << "\n";
  if (!rc && o.check_tasks) {
    unsigned long long issued = 0;
    if (!rt.fetch_task_counter(&issued) || issued != tasks.size()) {
      std::cerr << "task accounting mismatch: issued=" << issued << " expected=" << tasks.size() << "\n";
      rc = 3;
    }
  }
  losses.resize(o.steps);
  cudaMemcpy(losses.data(), dloss, losses.size() * 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(W.data(), dW, W.size() * 4, cudaMemcpyDeviceToHost);
  for (float* p : {dW, dx, dy, dt, ddy, ddW, dloss}) cudaFree(p);
  return rc;
}

// The same problem (or an MLP) through the tcgen05 MLP engine.
int run_mlp(const Opts& o, std::vector<float>& W, const std::vector<float>& x,
            const std::vector<float>& t, std::vector<float>& losses, float& ms) {
  std::vector<int> dims;
  if (o.layers.empty()) {
    dims = {o.n, o.m};
  } else {
    std::stringstream ss(o.layers);
    std::string tok;
    while (std::getline(ss, tok, ',')) dims.push_back(std::atoi(tok.c_str()));
    if (dims.front() != o.n || dims.back() != o.m) {
      std::cerr << "--layers must start with n and end with m\n";
      return 2;
    }
  }
  const int L = int(dims.size()) - 1;
  const bool bf = o.dtype == "bf16";
  pkt_mlp_config cfg{L, dims.data(), o.batch, bf ? PKT_DTYPE_BF16 : PKT_DTYPE_TF32, o.bias ? 1 : 0, 0, o.lr,
                     0, 0, 0};
  int dev = 0;
  cudaGetDevice(&dev);
  pkt_mlp* h = nullptr;
  if (pkt_mlp_create(dev, &cfg, &h) != PKT_OK) {
    std::cerr << "pkt_mlp_create: " << pkt_last_error() << "\n";
    return 1;
  }
  // parameters: the demo's W for a single layer, else a seeded Kaiming-uniform init
  std::vector<float> Wall;
  if (L == 1) {
    Wall = W;
  } else {
    std::mt19937 rng(7);
    for (int l = 0; l < L; ++l) {
      std::uniform_real_distribution<float> u(-std::sqrt(6.0f / dims[l]), std::sqrt(6.0f / dims[l]));
      for (long long i = 0; i < (long long)dims[l] * dims[l + 1]; ++i) Wall.push_back(u(rng));
    }
  }
  pkt_mlp_set_params(h, Wall.data(), nullptr);
  auto to_bf16 = [](const std::vector<float>& v) {
    std::vector<uint16_t> r(v.size());
    for (size_t i = 0; i < v.size(); ++i) {
      uint32_t u;
      std::memcpy(&u, &v[i], 4);
      r[i] = uint16_t((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
    }
    return r;
  };
  std::vector<uint16_t> xb, tb;
  if (bf) {
    xb = to_bf16(x);
    tb = to_bf16(t);
  }
  pkt_mlp_load_batch(h, bf ? (const void*)xb.data() : x.data(), bf ? (const void*)tb.data() : t.data(), 0,
                     nullptr);
  cudaDeviceSynchronize();
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  if (o.perf) pkt_mlp_set_perf(h, 1);
  pkt_mlp_clock_stats(h, nullptr, 1);
  cudaEventRecord(a);
  int rc = pkt_mlp_train(h, o.steps, nullptr);
  cudaEventRecord(b);
  cudaEventSynchronize(b);
  cudaEventElapsedTime(&ms, a, b);
  if (!rc && o.perf) {
    // the counters cover the last launch: one step, or the last group of steps
    // the engine ran in one launch
    unsigned long long clk[3] = {0, 0, 0};
    pkt_mlp_clock_stats(h, clk, 0);
    std::vector<pk::PerfBlock> blocks(1024);
    int got = 0;
    pkt_mlp_fetch_perf(h, reinterpret_cast<unsigned long long*>(blocks.data()), int(blocks.size()), &got);
    blocks.resize(size_t(got));
    const int per_launch = clk[2] ? int(o.steps / clk[2]) : 1;
    rc = report_perf(blocks, clock_mhz(clk), ms / o.steps, per_launch > 0 ? per_launch : 1, o);
  }
  losses.resize(o.steps);
  int got = 0;
  if (!rc) rc = pkt_mlp_losses(h, losses.data(), o.steps, &got);
  if (!rc && L == 1) rc = pkt_mlp_get_params(h, W.data(), nullptr);
  if (rc) std::cerr << "engine error: " << pkt_last_error() << "\n";
  pkt_mlp_destroy(h);
  return rc;
}

}  // namespace

int main(int argc, char** argv) {
  Opts o;
  if (!parse(argc, argv, o)) {
    std::cerr << "usage: train_linear [--m M] [--n N] [--batch B] [--steps S] [--lr LR] "
                 "[--fwd-tile-m/n T] [--bwd-tile-m/n T] [--blocks K] [--skip-cpu] [--check-loss] "
                 "[--check-tasks] [--engine tasks|mlp] [--dtype tf32|bf16] [--bias] [--layers n,...,m] "
                 "[--repeats R] [--perf] [--perf-json PATH] [--print-profile] [--seg-window W]\n";
    return 2;
  }
  std::cout << "Megakernel Training Demo (B200)\n========================\n";
  std::cout << "Model: y = Wx, W:[" << o.m << "," << o.n << "]\nBatch: " << o.batch << "\nSteps: " << o.steps
            << ", LR: " << o.lr << "\nEngine: " << o.engine << "\n";
  std::vector<float> W, x, t;
  make_data(o.m, o.n, o.batch, W, x, t);
  std::cout << "Initial host loss: " << host_loss(W, x, t, o.batch, o.m, o.n) << "\n";
  float cpu_final = -1.f;
  if (!o.skip_cpu && (long long)o.batch * o.m * o.n <= 100000000LL) {
    cpu_final = cpu_train(W, x, t, o.batch, o.m, o.n, o.steps, o.lr);
    std::cout << "CPU final loss: " << cpu_final << "\n";
  } else {
    std::cout << "CPU baseline skipped\n";
  }
  std::vector<float> losses;
  float ms = 0.f;
  const int rc = o.engine == "tasks" ? run_tasks(o, W, x, t, losses, ms) : run_mlp(o, W, x, t, losses, ms);
  if (rc) return rc;
  std::cout << "Time: " << ms << " ms\n";
  std::cout << "Time per step: " << ms / o.steps << " ms\n";
  std::cout << "Device first step loss: " << losses.front() << "\n";
  std::cout << "Device final loss: " << losses.back() << "\n";
  if (o.engine == "tasks" || o.layers.empty()) {
    const float final_host = host_loss(W, x, t, o.batch, o.m, o.n);
    std::cout << "Final loss (host recompute): " << final_host << "\n";
    if (o.check_loss) {
      // pkt's tolerance (examples/train_linear.cu:994-1001): abs 5e-5 or rel 5e-2
      const float ref = cpu_final >= 0.f ? cpu_final : final_host;
      const float diff = std::fabs(losses.back() - ref);
      if (diff > 5e-5f && diff > 5e-2f * std::fabs(ref)) {
        std::cerr << "check-loss failed: device " << losses.back() << " vs " << ref << "\n";
        return 4;
      }
      std::cout << "check-loss passed\n";
    }
  }
  std::cout << "Summary: steps=" << o.steps << " ms/step=" << ms / o.steps << "\n";
  return 0;
}
