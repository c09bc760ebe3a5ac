// pk::Config / WarpRoles with pkt's names and values (pkt include/config.cuh:8-127).
// The B200 megakernel keeps pkt's warp numbering: warp 0 controller, warp 1
// loader (TMA producer), warp 2 MMA issuer (pkt's "storer" slot), warps 3-6
// compute (TMEM epilogues and element-wise ops, which also store).
#pragma once

#include <cstdint>

#ifndef __CUDACC__
#ifndef __device__
#define __device__
#endif
#ifndef __host__
#define __host__
#endif
#endif

namespace pk {

struct Config {
  static constexpr int kWarpSize = 32;
  static constexpr int kPipelineStages = 4;  // task-slot ring depth
  static constexpr int kArgBytes = 64;
  static constexpr int kControllerWarp = 0;
  static constexpr int kLoaderWarp = 1;
  static constexpr int kStorerWarp = 2;  // the tcgen05 MMA issuer on B200
  static constexpr int kFirstComputeWarp = 3;
  static constexpr int kNumComputeWarps = 4;
  static constexpr int kTotalWarps = kFirstComputeWarp + kNumComputeWarps;
  static constexpr int kThreadsPerBlock = kTotalWarps * kWarpSize;
  static constexpr int kChunkSize = 32;  // accepted for compatibility; the B200 queue hands out 1 task
  static constexpr int kPagesPerSlot = 2;
  static constexpr int kMaxLogicalPages = kPipelineStages * kPagesPerSlot;
  static constexpr int kPageWords = 1024;
  static constexpr int kPageBytes = kPageWords * sizeof(int);
  static constexpr int kGemmKChunk = 16;  // K of one bf16 tcgen05.mma
  static constexpr int kLinearFwdThreadNFrag = 4;
  static constexpr int kLinearBwdThreadNFrag = 4;
  static constexpr bool kUseTensorCores = true;  // GEMM tiles always run on tcgen05
};

struct WarpRoles {
  int controller{Config::kControllerWarp};
  int loader{Config::kLoaderWarp};
  int storer{Config::kStorerWarp};
  int first_compute{Config::kFirstComputeWarp};
  int num_compute{Config::kNumComputeWarps};
};

#ifdef __CUDACC__
__device__ inline int lane_id() { return threadIdx.x & (Config::kWarpSize - 1); }
__device__ inline int warp_id() { return threadIdx.x / Config::kWarpSize; }
#endif
__host__ __device__ inline bool is_controller(int wid, const WarpRoles& r) { return wid == r.controller; }
__host__ __device__ inline bool is_loader(int wid, const WarpRoles& r) { return wid == r.loader; }
__host__ __device__ inline bool is_storer(int wid, const WarpRoles& r) { return wid == r.storer; }
__host__ __device__ inline bool is_compute(int wid, const WarpRoles& r) {
  return wid >= r.first_compute && wid < r.first_compute + r.num_compute;
}
__host__ __device__ inline int compute_warp_index(int wid, const WarpRoles& r) { return wid - r.first_compute; }

}  // namespace pk
