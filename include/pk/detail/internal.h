// Definitions shared by the host runtime and the device megakernel.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "../../pkt_b200.h"

namespace pkb {

// pkt's argument structs (include/ops/*.cuh), byte-identical.
struct ZeroMemoryArgs {  // include/ops/zero.cuh:10-13
  float* ptr;
  int size;
};
struct AxpyArgs {  // include/ops/axpy.cuh:9-15
  const float* x;
  float* y;
  float a;
  int n;
};
struct LinearForwardArgs {  // include/ops/linear_fwd.cuh:18-29
  const float* W;
  const float* x;
  float* y;
  int batch, m, n, tile_m_start, tile_m_count, tile_n_start, tile_n_count;
};
struct LinearBackwardArgs {  // include/ops/linear_bwd.cuh:16-27
  const float* dy;
  const float* x;
  float* dW;
  int batch, m, n, tile_m_start, tile_m_count, tile_n_start, tile_n_count;
};
struct MSELossArgs {  // include/ops/mse.cuh:13-20
  const float* y;
  const float* target;
  float* dy;
  float* loss;
  int batch, m;
};
struct SGDUpdateArgs {  // include/ops/sgd.cuh:12-17
  float* W;
  const float* dW;
  float lr;
  int size;
};
static_assert(sizeof(ZeroMemoryArgs) == 16, "pkt ZeroMemoryArgs layout");
static_assert(sizeof(AxpyArgs) == 24, "pkt AxpyArgs layout");
static_assert(sizeof(LinearForwardArgs) == 56, "pkt LinearForwardArgs layout");
static_assert(sizeof(LinearBackwardArgs) == 56, "pkt LinearBackwardArgs layout");
static_assert(sizeof(MSELossArgs) == 40, "pkt MSELossArgs layout");
static_assert(sizeof(SGDUpdateArgs) == 24, "pkt SGDUpdateArgs layout");
static_assert(sizeof(pkt_task) == 96, "pkt Task is 96 bytes");
static_assert(sizeof(pkt_task_header) == 32, "pkt TaskHeader is 32 bytes");
static_assert(sizeof(pkt_bias_sgd_args) <= 64 && sizeof(pkt_sgd_mixed_args) <= 64 &&
                  sizeof(pkt_loss_reduce_args) <= 64 && sizeof(pkt_gemm_tile_args) <= 64,
              "args fit the 64-byte payload");

// CTA shape of the megakernel (pkt's warp numbering, include/config.cuh:17-27):
//   warp 0 controller  : dequeues tasks, waits on dependency tokens, fills the slot ring
//   warp 1 loader      : TMA tile loads into the shared-memory stage ring
//   warp 2 MMA issuer  : tcgen05.mma into the TMEM accumulators (pkt's "storer" index)
//   warps 3-6 compute  : TMEM epilogues, SIMT ops, stores and token publication
constexpr int kThreads = 224;
constexpr int kCtrlWarp = 0;
constexpr int kLoadWarp = 1;
constexpr int kMmaWarp = 2;
constexpr int kEpiWarp0 = 3;
constexpr int kEpiThreads = 128;
constexpr int kStages = 4;       // single-CTA mode: 48 KB stages
constexpr int kStagesPair = 3;   // pair mode: 64 KB stages (A 128x128 + half of B, K depth 128 bf16)
constexpr int kSlots = 4;
constexpr int kBM = 128;
constexpr int kMaxBN = 256;
constexpr int kATileBytes = kBM * 128;
constexpr int kBTileBytes = kMaxBN * 128;
constexpr int kStageBytes = kATileBytes + kBTileBytes;
constexpr int kEpiStageBytes = 6144;  // per compute warp: one 32x32 chunk, fp32 (4 KB) + bf16 (2 KB)
constexpr int kTmemCols = 512;  // two 256-column fp32 accumulators
constexpr uint16_t kOpStop = 0xFFFF;

// Device copy of one registered GEMM.
struct alignas(128) DevGemm {
  CUtensorMap map_a;
  CUtensorMap map_b;
  pkt_gemm_desc d;
  uint32_t idesc;
  int tiles_m, tiles_n, num_kb, bk;
  int a_boxes, b_boxes;    // TMA boxes per stage
  int box_mn;              // elements per 128-byte row (MN-major box width)
  uint32_t stage_tx;       // bytes landed per stage
  uint32_t a_lbo, b_lbo;   // descriptor leading-byte offsets
  uint32_t a_kstep, b_kstep;  // descriptor start advance per MMA within a 4-MMA K group (bytes)
  uint32_t a_kgroup, b_kgroup;  // descriptor start advance per 4-MMA K group (bytes)
  int kchunks;                // 128-byte K chunks per stage (1 single-CTA, 2 pair)
  uint32_t a_box_bytes, b_box_bytes;
  int pair;                     // 1: single CTA tiles (128 rows), 2: CTA-pair tiles (256 rows)
  int b_rows;                   // rows of B (N direction) each CTA loads: bn / pair
  uint32_t a_sbo, b_sbo;        // descriptor stride-byte offsets
  uint32_t a_layout, b_layout;  // descriptor swizzle mode: 2 = 128B, 1 = 128B with 32B atoms
  int mma_per_kb;
  int tma_out;     // 1: the epilogue writes `out` with TMA tile stores through map_out
  int tma_w;       // 1: WGRAD_SGD writes w_out / w_shadow through map_w / map_shadow
  int dp_tile_base;  // WGRAD_PEER: index of tile (0, 0) among all weight tiles of a step
  int dp_layer;      // WGRAD_PEER: layer of the weights (counter of the next step's copies)
  CUtensorMap map_out;     // out: boxes of 32 columns x 32 rows (one compute warp's chunk)
  CUtensorMap map_w;       // w_out (fp32)
  CUtensorMap map_shadow;  // w_shadow (bf16)
  CUtensorMap map_pf;      // the matrix the epilogue reads rows of (aux or w_in): L2 prefetch boxes
  int pf_ok;               // 1: map_pf is valid (the loader prefetches each tile's box)
  int pad_pf;
};

// Per-CTA perf words (pkt_runtime_fetch_perf), cycles unless noted.
enum PerfWord {
  kPerfTasks = 0,         // tasks executed (count)
  kPerfGemmTiles = 1,     // GEMM tiles executed (count)
  kPerfCtrlDepWait = 2,
  kPerfCtrlSlotWait = 3,
  kPerfLoadStageWait = 4,
  kPerfMmaFullWait = 5,
  kPerfMmaTmemWait = 6,
  kPerfEpiTmemWait = 7,
  kPerfEpiGemm = 8,
  kPerfEpiSimt = 9,
  kPerfTotal = 10,
  kPerfMmaSlotWait = 11,   // MMA issuer waiting for the next task
  kPerfMmaIssue = 12,      // MMA issuer between stage-full and commit
  kPerfKBlocks = 13,       // k-blocks issued (count)
};

// Fused data parallel: every rank's exchange region (one cudaMalloc, same
// layout everywhere; peers' regions are CUDA IPC mappings) and the offsets of
// its parts. Counters only grow (never reset between steps): targets are
// multiples of the step index the launch carries.
struct DpPeers {
  int world, rank, pair;
  int num_layers;
  long long slot_bytes;       // one partial tile slot: pair*128 rows x 256 floats
  long long recv_off;         // partial slots [owned tile][source rank]
  long long arrive_off;       // int per owned tile: other ranks' partial slots written (x pair)
  long long wready_off;       // int per layer: owner broadcasts received (x pair)
  long long bias_recv_off;    // fp32 [2 step parities][world][bias_total]
  long long barrive_off;      // int per layer: bias vectors received (x pair)
  int bias_total;             // floats in one rank's bias gradient vector
  int pad_;
  uint8_t* base[PKT_DP_MAX_RANKS];
  // per rank: its partial slots as one fp32 matrix [slots * pair*128 rows][256],
  // boxes of 32 x 32 (TMA tile stores from a compute warp's staging buffer)
  CUtensorMap recv_map[PKT_DP_MAX_RANKS];
};

struct KParams {
  const pkt_task* tasks;
  int num_tasks;
  int num_tokens;
  int* state;  // [0] cursor, [1..3] status code/task/detail, [4..] token counts, then epochs
  const DevGemm* gemms;
  int num_gemms;
  int chunk;
  unsigned long long* task_counter;
  unsigned long long* perf;  // [gridDim.x][PKT_PERF_WORDS] or null
  unsigned long long timeout_ns;
  const DpPeers* dp;  // fused data parallel (null otherwise)
  int dp_step;        // fused data-parallel steps completed before this launch
  // >0: a controller dequeues its next task only while fewer than this many of
  // the tasks it published wait for its compute warps (0: the slot ring alone)
  int lookahead;
  // optional [3]: += SM cycles, += nanoseconds of CTA 0's lifetime, += 1 per launch
  unsigned long long* clock_acc;
  // optional [num_tasks][kTraceWords]: per task, %globaltimer stamps of its stages
  unsigned long long* trace;
};

// Words of one task's trace record (pkt_mlp_fetch_trace / pkt_runtime_fetch_trace).
enum TraceWord {
  kTrCta = 0,       // bits 0-15 CTA, 16-31 opcode; GEMM tiles: 32-47 GEMM id, 48-55 tile_m, 56-63 tile_n (low 8 bits)
  kTrDequeue = 1,   // controller took it from the queue
  kTrReady = 2,     // its dependencies were satisfied (published to the slot ring)
  kTrLoad = 3,      // loader issued its first TMA load (GEMM tiles)
  kTrMma0 = 4,      // MMA issuer issued its first MMA (first stage had landed)
  kTrMma1 = 5,      // MMA issuer committed its last MMA
  kTrExec = 6,      // compute warps started it (GEMM: the accumulator was complete)
  kTrDone = 7,      // compute warps finished it (before its token was published)
};
constexpr int kTraceWords = 8;

constexpr int kStateHeader = 8;  // ints before the token counters
inline int state_ints(int num_tokens) { return kStateHeader + 2 * num_tokens; }

// Launches the megakernel (megakernel.cu); pair = 2 launches clusters of two CTAs.
// `blocks` must not exceed max_resident_blocks(pair): every CTA of the persistent
// grid is resident at once.
cudaError_t launch_megakernel(const KParams& p, int blocks, cudaStream_t stream, int pair = 1);
// CTAs of the megakernel variant that fit on the current device at the same time.
cudaError_t max_resident_blocks(int pair, int* blocks);

}  // namespace pkb
