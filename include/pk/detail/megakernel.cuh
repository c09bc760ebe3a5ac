// The persistent sm_100a megakernel: one CTA per SM pulls pkt tasks from a
// device-resident queue and runs them through a warp-specialised pipeline.
//
// Replaces pkt's persistent_kernel (include/kernel.cuh:1351-1517) and its role
// loops (controller :683-953, loader :956-1067, compute :1069-1205, storer
// :1207-1341). What changed, B200-first:
//   * intra-CTA handoff is mbarrier phase bits (slot ring + stage ring + TMEM
//     accumulator ring), not polled smem atomics with nanosleep backoff
//     (include/pipeline.cuh:40-47);
//   * GEMM tiles (pkt's reserved OpCode::Gemm) run on tcgen05: TMA bulk-tensor
//     loads (128B swizzle, no multicast) -> one elected thread issues
//     tcgen05.mma into a double-buffered TMEM accumulator -> four warps read
//     TMEM and apply the fused epilogue (bias+ReLU, MSE+dY, ReLU-masked dgrad,
//     weight-gradient + SGD);
//   * cross-CTA dependencies keep pkt's token semantics (cumulative count +
//     max epoch, include/dependency.cuh:29-77) with ld.acquire / red.release,
//     plus an optional second token per task (pkt's reserved header words);
//   * every wait is bounded by a %globaltimer budget; on expiry the device
//     writes a status word (code, task, detail) and every CTA drains, so a
//     malformed DAG returns an error instead of hanging the GPU (pkt spins
//     forever, include/kernel.cuh:873-881).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../block_runtime.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace pkb {

// Ops run by the megakernel besides its built-in opcodes: none in libpkt_b200's
// own instantiation; pk::OpSet<...> (pk/kernel.cuh) for a program's own
// pk::OpTraits specialisations.
struct NoUserOps {
  __device__ static bool handles(uint16_t) { return false; }
  __device__ static void load(uint16_t, const pk::Task&, pk::BlockRuntime&, int, int, unsigned long long*,
                              unsigned long long*) {}
  __device__ static void compute(uint16_t, const pk::Task&, pk::BlockRuntime&, int, int, int, int) {}
  __device__ static void store(uint16_t, const pk::Task&, pk::BlockRuntime&, int, int) {}
};

namespace {

// P = 1: one CTA per tile, 4 stages of 48 KB (A 128x64 + B up to 256x64 bf16).
// P = 2: CTA pairs, 6 stages of 32 KB (A 128x64 + this CTA's half of B).
template <int P>
struct SmemT {
  static constexpr int NST = P == 2 ? kStagesPair : kStages;
  static constexpr int A_BYTES = P * kATileBytes;  // pair: two 128-byte K chunks of A
  static constexpr int SB = P == 2 ? A_BYTES + kBTileBytes : kStageBytes;
  uint8_t stages[NST][SB];  // 1024-byte aligned (kernel aligns the base)
  // per compute warp (TMEM lane quadrant): staging of one 32x32 output chunk for
  // the TMA tile stores; every buffer starts on a 1024-byte boundary (swizzle)
  uint8_t epi_stage[4][kEpiStageBytes];
  pkt_task slots[kSlots];
  uint64_t full[NST];
  uint64_t empty[NST];
  uint64_t slot_full[kSlots];
  uint64_t slot_empty[kSlots];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_drain;
  uint64_t pair_done[kSlots];  // leader: the other CTA of the pair finished task seq
  uint32_t tmem_base;
  int dp_ok;  // PKT_OP_DP_REDUCE: every rank's partial of the current tile arrived
  int taken;  // tasks the compute warps have taken from the slot ring (leader CTA)
  pk::PipelineSlot user_slot;                  // the task a pk::OpTraits op sees as br.slot(0)
  pk::PageMeta page_meta[pk::Config::kPagesPerSlot];  // leases / tags of its pages (in epi_stage)
  float red[8][4][32];  // per 32-column chunk, per TMEM lane quadrant: column partial sums
  float lossred[4];
  float simt_red[4];
  double simt_redd[4];
};

template <int P>
constexpr int smem_bytes() { return int(sizeof(SmemT<P>)) + 1024; }
static_assert(smem_bytes<1>() <= 227 * 1024 && smem_bytes<2>() <= 227 * 1024,
              "shared memory layout exceeds the 227 KB a CTA can use");

__device__ __forceinline__ int* tok_count(const KParams& p) { return p.state + kStateHeader; }
__device__ __forceinline__ int* tok_epoch(const KParams& p) {
  return p.state + kStateHeader + p.num_tokens;
}
__device__ __forceinline__ volatile int* status_word(const KParams& p) {
  return reinterpret_cast<volatile int*>(p.state + 1);
}

__device__ void set_error(const KParams& p, int code, int task, int detail) {
  if (atomicCAS(p.state + 1, 0, code) == 0) {
    p.state[2] = task;
    p.state[3] = detail;
    __threadfence();
  }
}

// Bounded mbarrier wait. Returns false when the budget ran out or another
// CTA reported an error while this one was waiting. `idle` waits (a consumer
// waiting for the controller's next task, which may itself be waiting on a
// dependency with the same budget) get four budgets plus one second, so the
// controller's dependency timeout is the one reported.
// Cycle stamp for the optional per-role counters; zero (and free) when they are off.
__device__ __forceinline__ long long stamp(bool on) { return on ? clock64() : 0; }

template <bool CL = false>
__device__ __forceinline__ bool try_wait_scoped(uint64_t* bar, uint32_t parity) {
  return CL ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
}

// CL: the barrier receives arrivals from the other CTA of a pair (cluster-scope acquire).
template <bool CL = false>
__device__ __forceinline__ bool wait_bar(const KParams& p, uint64_t* bar, uint32_t parity,
                                         int where, bool idle = false) {
  if (try_wait_scoped<CL>(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t budget = idle ? 4 * p.timeout_ns + 1000000000ull : p.timeout_ns;
  uint32_t it = 0;
  while (!try_wait_scoped<CL>(bar, parity)) {
    if ((++it & 63u) == 0) {
      if (*status_word(p) != 0) return false;
      if (globaltimer_ns() - t0 > budget) {
        set_error(p, PKT_DEV_TIMEOUT_PIPE, -1, where);
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ bool opcode_known(uint16_t op) {
  return op == PKT_OP_INVALID || op == PKT_OP_ZERO_MEMORY || op == PKT_OP_AXPY ||
         op == PKT_OP_GEMM || op == PKT_OP_LINEAR_FORWARD || op == PKT_OP_MSE_LOSS ||
         op == PKT_OP_LINEAR_BACKWARD || op == PKT_OP_SGD_UPDATE || op == PKT_OP_BIAS_SGD ||
         op == PKT_OP_LOSS_REDUCE || op == PKT_OP_SGD_MIXED || op == PKT_OP_DP_WAIT ||
         op == PKT_OP_DP_BIAS_SEND || op == PKT_OP_DP_BIAS_APPLY || op == PKT_OP_DP_REDUCE;
}

__device__ __forceinline__ void copy_task(pkt_task* dst, const pkt_task* src) {
  const int4* s = reinterpret_cast<const int4*>(src);
  int4* d = reinterpret_cast<int4*>(dst);
#pragma unroll
  for (int i = 0; i < 6; ++i) d[i] = s[i];
}

// Releases a slot of the ring: the ring lives in the leader CTA; the other CTA of a
// pair arrives on the leader's slot_empty remotely.
template <int P>
__device__ __forceinline__ void release_slot(SmemT<P>& s, int slot, uint32_t rank) {
  if (P == 1 || rank == 0)
    mbar_arrive(&s.slot_empty[slot]);
  else
    mbar_arrive_remote(mapa_shared(smem_u32(&s.slot_empty[slot]), 0));
}

// Publishes a task into slot `slot` of this CTA and, for pairs, of the other CTA.
template <int P>
__device__ __forceinline__ void publish_slot(SmemT<P>& s, int slot, const pkt_task& task) {
  copy_task(&s.slots[slot], &task);
  if (P == 2) {
    const uint32_t dst = mapa_shared(smem_u32(&s.slots[slot]), 1);
    const int4* src = reinterpret_cast<const int4*>(&task);
#pragma unroll
    for (int i = 0; i < 6; ++i) st_cluster_v4(dst + 16 * i, src[i]);
    mbar_arrive_remote(mapa_shared(smem_u32(&s.slot_full[slot]), 1));
  }
  mbar_arrive(&s.slot_full[slot]);
}

// ============================================================ controller
// Pause between two polls of a dependency token (ns; 0 = spin).
#ifndef PKT_POLL_SLEEP_NS
#define PKT_POLL_SLEEP_NS 32
#endif
constexpr unsigned kPollSleepNs = PKT_POLL_SLEEP_NS;

template <int P, class Ops>
__device__ void controller_loop(const KParams& p, SmemT<P>& s, unsigned long long* perf) {
  int seq = 0;
  unsigned long long dep_cycles = 0, slot_cycles = 0, ntasks = 0;
  int cursor_local = 0, cursor_end = 0;
  while (true) {
    if (*status_word(p) != 0) break;
    if (p.lookahead > 0) {
      // A task this CTA holds is a task no idle CTA can take: dequeue the next one
      // only when the pipeline is about to need it.
      const long long c1 = clock64();
      const uint64_t t0 = globaltimer_ns();
      uint32_t it = 0;
      bool ok = true;
      while (seq - *reinterpret_cast<volatile int*>(&s.taken) >= p.lookahead) {
        if ((++it & 63u) == 0) {
          if (*status_word(p) != 0 || globaltimer_ns() - t0 > p.timeout_ns) {
            ok = false;
            break;
          }
        }
      }
      slot_cycles += clock64() - c1;
      if (!ok) {
        if (*status_word(p) == 0) set_error(p, PKT_DEV_TIMEOUT_DEPS, -1, -4);
        break;
      }
    }
    if (cursor_local >= cursor_end) {
      const int start = atomicAdd(p.state, p.chunk);
      cursor_local = start;
      cursor_end = min(start + p.chunk, p.num_tasks);
      if (cursor_local >= cursor_end) break;
    }
    const int t = cursor_local++;
    unsigned long long* tr = p.trace ? p.trace + (size_t)t * kTraceWords : nullptr;
    if (tr) tr[kTrDequeue] = globaltimer_ns();
    pkt_task task;
    copy_task(&task, p.tasks + t);
    if (tr) {
      const pkt_gemm_tile_args* ga = reinterpret_cast<const pkt_gemm_tile_args*>(task.args);
      const bool gemm = task.header.opcode == PKT_OP_GEMM;
      tr[kTrCta] = (unsigned long long)blockIdx.x | ((unsigned long long)task.header.opcode << 16) |
                   (gemm ? ((unsigned long long)(ga->gemm & 0xffffu) << 32) |
                               ((unsigned long long)(ga->tile_m & 0xffu) << 48) |
                               ((unsigned long long)(ga->tile_n & 0xffu) << 56)
                         : 0ull);
    }
    const pkt_task_header& h = task.header;
    if (!opcode_known(h.opcode) && !Ops::handles(h.opcode)) {
      set_error(p, PKT_DEV_BAD_OPCODE, t, h.opcode);
      break;
    }
    const int r1 = h.buffer_read_id, r2 = int(h.ext_ids & 0xffffu);
    const int w1 = h.buffer_write_id, w2 = int(h.ext_ids >> 16);
    if (r1 >= p.num_tokens || r2 >= p.num_tokens || w1 >= p.num_tokens || w2 >= p.num_tokens) {
      set_error(p, PKT_DEV_BAD_ARGS, t, -1);
      break;
    }
    if (h.opcode == PKT_OP_GEMM) {
      const pkt_gemm_tile_args* a = reinterpret_cast<const pkt_gemm_tile_args*>(task.args);
      if (int(a->gemm) >= p.num_gemms || int(a->tile_m) >= p.gemms[a->gemm].tiles_m ||
          int(a->tile_n) >= p.gemms[a->gemm].tiles_n || p.gemms[a->gemm].pair != P) {
        set_error(p, PKT_DEV_BAD_ARGS, t, -2);
        break;
      }
    }
    // ---- dependency wait (pkt semantics: count >= wait_count && epoch >= read_epoch)
    if (r1 != 0 || r2 != 0) {
      const long long c0 = clock64();
      const uint64_t t0 = globaltimer_ns();
      uint32_t it = 0;
      bool ok = true;
      while (true) {
        bool ready = true;
        if (r1 != 0) {  // (epochs start at 0: a zero read_epoch needs no second load)
          ready = ld_acquire_gpu(tok_count(p) + r1) >= int(h.wait_count) &&
                  (h.read_epoch == 0 || ld_acquire_gpu(tok_epoch(p) + r1) >= int(h.read_epoch));
        }
        if (ready && r2 != 0) ready = ld_acquire_gpu(tok_count(p) + r2) >= int(h.ext_wait_count);
        if (ready) break;
        if ((++it & 15u) == 0) {
          if (*status_word(p) != 0) {
            ok = false;
            break;
          }
          if (globaltimer_ns() - t0 > p.timeout_ns) {
            set_error(p, PKT_DEV_TIMEOUT_DEPS, t, r1 != 0 ? r1 : r2);
            ok = false;
            break;
          }
        }
        if (kPollSleepNs > 0) __nanosleep(kPollSleepNs);
      }
      dep_cycles += clock64() - c0;
      if (!ok) break;
    }
    // ---- publish into the slot ring
    const int slot = seq % kSlots;
    const long long c1 = clock64();
    if (!wait_bar<(P == 2)>(p, &s.slot_empty[slot], ((seq / kSlots) & 1) ^ 1, 1)) break;
    slot_cycles += clock64() - c1;
    task.header.user_tag = uint32_t(t);
    if (tr) tr[kTrReady] = globaltimer_ns();
    if (p.task_counter) atomicAdd(p.task_counter, 1ull);
    publish_slot<P>(s, slot, task);
    ++seq;
    ++ntasks;
  }
  // ---- stop marker: consumers leave their loops when they reach it
  const int slot = seq % kSlots;
  if (wait_bar<(P == 2)>(p, &s.slot_empty[slot], ((seq / kSlots) & 1) ^ 1, 2)) {
    pkt_task stop{};
    stop.header.opcode = kOpStop;
    publish_slot<P>(s, slot, stop);
  }
  if (perf) {
    perf[kPerfTasks] = ntasks;
    perf[kPerfCtrlDepWait] = dep_cycles;
    perf[kPerfCtrlSlotWait] = slot_cycles;
  }
}

// ============================================================ loader (TMA producer)
// The epilogue of a tile reads rows of a second matrix with plain loads (dgrad:
// the activations for the ReLU mask; MSE: the targets; fused SGD: the fp32
// master weights). Those rows are usually not in L2 (the activations were
// written a whole forward pass earlier), so the loader asks for them at the tile
// start: one TMA L2 prefetch of this CTA's 128-row box, landing while the
// mainloop runs.
__device__ __forceinline__ void prefetch_epilogue_rows(const DevGemm& g, int rblock, int tile_n) {
  if (g.pf_ok) tma_prefetch_2d(&g.map_pf, tile_n * g.d.bn, rblock * kBM);
}

template <int P>
__device__ void loader_loop(const KParams& p, SmemT<P>& s, uint32_t rank, unsigned long long* perf) {
  constexpr int NST = SmemT<P>::NST;
  int seq = 0;
  uint32_t stage = 0, phase = 0, issued = 0;
  unsigned long long wait_cycles = 0;
  while (true) {
    const int slot = seq % kSlots;
    if (!wait_bar<(P == 2)>(p, &s.slot_full[slot], (seq / kSlots) & 1, 3, true)) break;
    const uint16_t op = s.slots[slot].header.opcode;
    const uint32_t tix = s.slots[slot].header.user_tag;
    pkt_gemm_tile_args ga = *reinterpret_cast<const pkt_gemm_tile_args*>(s.slots[slot].args);
    release_slot<P>(s, slot, rank);
    ++seq;
    if (op == kOpStop) break;
    if (op != PKT_OP_GEMM) continue;
    if (p.trace && rank == 0) p.trace[(size_t)tix * kTraceWords + kTrLoad] = globaltimer_ns();
    const DevGemm& g = p.gemms[ga.gemm];
    // Data of this tile was produced by other CTAs through generic stores and is
    // read here through the async proxy.
    fence_proxy_async_global();
    // pair mode: this CTA loads rows [rank*128, +128) of the 256-row A tile and
    // rows [rank*bn/2, +bn/2) of B; both CTAs' bytes count on the leader's barrier
    const int m0 = int(ga.tile_m) * kBM * P + int(rank) * kBM;
    const int n0 = int(ga.tile_n) * g.d.bn + int(rank) * g.b_rows;
    prefetch_epilogue_rows(g, int(ga.tile_m) * P + int(rank), int(ga.tile_n));
    // per-tile constants in registers (the asm "memory" clobbers would force reloads)
    const int num_kb = g.num_kb, bk = g.bk, box_mn = g.box_mn;
    const bool a_kmaj = g.d.a_major == PKT_MAJOR_K, b_kmaj = g.d.b_major == PKT_MAJOR_K;
    const int a_boxes = g.a_boxes, b_boxes = g.b_boxes;
    const int kbox = 128 / (g.d.in_dtype == PKT_DTYPE_BF16 ? 2 : 4);  // K elements per K-major box
    const uint32_t a_box_bytes = g.a_box_bytes, b_box_bytes = g.b_box_bytes, stage_tx = g.stage_tx;
    const void* map_a = &g.map_a;
    const void* map_b = &g.map_b;
    bool ok = true;
    const bool prof = perf != nullptr;
    for (int kb = 0; kb < num_kb; ++kb) {
      const long long c0 = stamp(prof);
      if (!wait_bar(p, &s.empty[stage], phase ^ 1, 4)) {
        ok = false;
        break;
      }
      wait_cycles += stamp(prof) - c0;
      if (rank == 0) mbar_arrive_expect_tx(&s.full[stage], stage_tx);
      uint8_t* sa = s.stages[stage];
      uint8_t* sb = s.stages[stage] + SmemT<P>::A_BYTES;
      const int k0 = kb * bk;
      // K-major: one box per 128-byte K chunk; MN-major: one box per 128-byte MN chunk
      if (P == 1) {
        for (int i = 0; i < a_boxes; ++i)
          tma_load_2d(sa + i * a_box_bytes, map_a, &s.full[stage], a_kmaj ? k0 + i * kbox : m0 + i * box_mn,
                      a_kmaj ? m0 : k0);
        for (int i = 0; i < b_boxes; ++i)
          tma_load_2d(sb + i * b_box_bytes, map_b, &s.full[stage], b_kmaj ? k0 + i * kbox : n0 + i * box_mn,
                      b_kmaj ? n0 : k0);
      } else {
        const uint32_t fb = mapa_shared(smem_u32(&s.full[stage]), 0);  // leader's barrier
        for (int i = 0; i < a_boxes; ++i)
          tma_load_2d_pair(sa + i * a_box_bytes, map_a, fb, a_kmaj ? k0 + i * kbox : m0 + i * box_mn,
                           a_kmaj ? m0 : k0);
        for (int i = 0; i < b_boxes; ++i)
          tma_load_2d_pair(sb + i * b_box_bytes, map_b, fb, b_kmaj ? k0 + i * kbox : n0 + i * box_mn,
                           b_kmaj ? n0 : k0);
      }
      ++issued;
      if (++stage == NST) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (!ok) break;
  }
  // Drain: wait (bounded) until every issued stage landed, so no bulk copy can
  // write into shared memory after the CTA exits. In pair mode the leader's
  // barriers count both CTAs' bytes; the other CTA is held by the final cluster
  // barrier until the leader has drained.
  const uint32_t n = rank != 0 ? 0 : (issued < uint32_t(NST) ? issued : uint32_t(NST));
  for (uint32_t i = 0; i < n; ++i) {
    const uint32_t idx = (stage + NST - 1 - i) % NST;
    const uint32_t fill = issued - 1 - i;  // fill number of that stage
    const uint32_t par = (fill / NST) & 1;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(&s.full[idx], par)) {
      if (globaltimer_ns() - t0 > p.timeout_ns) break;
    }
  }
  if (perf) perf[kPerfLoadStageWait] = wait_cycles;
}

// ============================================================ MMA issuer
// One stage's MMAs (4 per 128-byte K chunk: bf16 K=16, tf32 K=8) and the commit
// that frees the stage once they have read it. The operand type is a template
// argument so the issue stream holds no per-MMA branch; only the first MMA of a
// tile (acc_first == 0) overwrites the accumulator.
template <int P, bool TF32>
__device__ __forceinline__ void issue_kblock(uint64_t* empty_bar, uint32_t d_tmem, uint64_t a_hi,
                                             uint64_t b_hi, uint32_t sa, uint32_t sb, uint32_t idesc,
                                             uint32_t a_kstep, uint32_t b_kstep, uint32_t a_kgroup,
                                             uint32_t b_kgroup, uint32_t acc_first) {
#pragma unroll
  for (int k = 0; k < 4 * P; ++k) {
    const uint32_t ao = (k >> 2) * a_kgroup + (k & 3) * a_kstep;
    const uint32_t bo = (k >> 2) * b_kgroup + (k & 3) * b_kstep;
    const uint64_t ad = a_hi | uint64_t((sa + ao) >> 4);
    const uint64_t bd = b_hi | uint64_t((sb + bo) >> 4);
    const uint32_t accum = k == 0 ? acc_first : 1u;
    if (P == 2) {
      if (TF32)
        mma_tf32_pair(d_tmem, ad, bd, idesc, accum);
      else
        mma_bf16_pair(d_tmem, ad, bd, idesc, accum);
    } else {
      if (TF32)
        mma_tf32(d_tmem, ad, bd, idesc, accum);
      else
        mma_bf16(d_tmem, ad, bd, idesc, accum);
    }
  }
  // stage reusable (in both CTAs of a pair) once these MMAs have read it
  if (P == 2)
    mma_commit_pair_both(empty_bar);
  else
    mma_commit(empty_bar);
}

template <int P>
__device__ void mma_loop(const KParams& p, SmemT<P>& s, uint32_t tmem_base,
                         unsigned long long* perf) {
  constexpr int NST = SmemT<P>::NST;
  int seq = 0;
  uint32_t stage = 0, phase = 0, gemm_count = 0;
  unsigned long long full_wait = 0, tmem_wait = 0, tiles = 0, slot_wait = 0, issue = 0, kblocks = 0;
  unsigned long long gap = 0;
  long long tile_end = 0;
  const long long life0 = stamp(perf != nullptr);
  bool any_mma = false;
  // The whole warp runs the loop (converged); one elected lane issues each
  // tcgen05.mma / commit, as the instructions are single-thread.
  const bool elected = (threadIdx.x & 31) == 0;
  while (true) {
    const int slot = seq % kSlots;
    const long long cs = clock64();
    if (!wait_bar<(P == 2)>(p, &s.slot_full[slot], (seq / kSlots) & 1, 5, true)) break;
    slot_wait += clock64() - cs;
    const uint16_t op = s.slots[slot].header.opcode;
    const uint32_t tix = s.slots[slot].header.user_tag;
    pkt_gemm_tile_args ga = *reinterpret_cast<const pkt_gemm_tile_args*>(s.slots[slot].args);
    if (elected) mbar_arrive(&s.slot_empty[slot]);  // the MMA issuer only runs in the leader CTA
    __syncwarp();
    ++seq;
    if (op == kOpStop) break;
    if (op != PKT_OP_GEMM) continue;
    const DevGemm& g = p.gemms[ga.gemm];
    // Everything the issue loop needs goes to registers once per tile: the
    // "memory" clobber of each tcgen05.mma would otherwise make the compiler
    // reload these fields from global memory between MMAs and starve the pipe.
    const int num_kb = g.num_kb;
    const uint32_t idesc = g.idesc;
    const uint32_t a_kstep = g.a_kstep, b_kstep = g.b_kstep;
    const uint32_t a_kgroup = g.a_kgroup, b_kgroup = g.b_kgroup;
    const uint64_t a_hi = smem_desc(0, g.a_lbo, g.a_sbo, g.a_layout);
    const uint64_t b_hi = smem_desc(0, g.b_lbo, g.b_sbo, g.b_layout);
    const bool tf32 = g.d.in_dtype == PKT_DTYPE_TF32;
    const uint32_t acc = gemm_count & 1, use = gemm_count >> 1;
    const long long c0 = clock64();
    if (!wait_bar<(P == 2)>(p, &s.tmem_empty[acc], (use & 1) ^ 1, 6)) break;
    tmem_wait += clock64() - c0;
    tc_fence_after();
    const uint32_t d_tmem = tmem_base + acc * 256;
    bool ok = true;
    const bool prof = perf != nullptr;
    if (prof && tile_end != 0) gap += clock64() - tile_end;
    for (int kb = 0; kb < num_kb; ++kb) {
      const long long c1 = stamp(prof);
      if (!wait_bar(p, &s.full[stage], phase, 7)) {
        ok = false;
        break;
      }
      const long long c2 = stamp(prof);
      full_wait += c2 - c1;
      if (kb == 0 && p.trace && elected) p.trace[(size_t)tix * kTraceWords + kTrMma0] = globaltimer_ns();
      tc_fence_after();
      const uint32_t sa = smem_u32(s.stages[stage]);
      const uint32_t sb = sa + SmemT<P>::A_BYTES;
      if (elected) {
        if (tf32)
          issue_kblock<P, true>(&s.empty[stage], d_tmem, a_hi, b_hi, sa, sb, idesc, a_kstep, b_kstep,
                                a_kgroup, b_kgroup, kb > 0 ? 1u : 0u);
        else
          issue_kblock<P, false>(&s.empty[stage], d_tmem, a_hi, b_hi, sa, sb, idesc, a_kstep, b_kstep,
                                 a_kgroup, b_kgroup, kb > 0 ? 1u : 0u);
      }
      __syncwarp();
      any_mma = true;
      issue += stamp(prof) - c2;
      ++kblocks;
      if (++stage == NST) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (!ok) break;
    if (elected) {
      if (P == 2)
        mma_commit_pair_both(&s.tmem_full[acc]);  // accumulator complete in both CTAs
      else
        mma_commit(&s.tmem_full[acc]);
      if (p.trace) p.trace[(size_t)tix * kTraceWords + kTrMma1] = globaltimer_ns();
    }
    __syncwarp();
    ++gemm_count;
    ++tiles;
    tile_end = stamp(perf != nullptr);
  }
  if (any_mma) {
    // Every MMA this thread issued has finished before TMEM is released.
    if (elected) {
      if (P == 2)
        mma_commit_pair_local(&s.mma_drain);
      else
        mma_commit(&s.mma_drain);
    }
    __syncwarp();
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(&s.mma_drain, 0)) {
      if (globaltimer_ns() - t0 > p.timeout_ns) break;
    }
  }
  if (perf && elected) {
    perf[kPerfGemmTiles] = tiles;
    perf[kPerfMmaFullWait] = full_wait;
    perf[kPerfMmaTmemWait] = tmem_wait;
    perf[kPerfMmaSlotWait] = slot_wait;
    perf[kPerfMmaIssue] = issue;
    perf[kPerfKBlocks] = kblocks;
    perf[14] = gap;                      // from one tile's last commit to the next tile's k loop
    perf[15] = clock64() - life0;        // MMA issuer lifetime
  }
}

// ============================================================ epilogue helpers
struct EpiCtx {
  int et;    // 0..127 thread index among the compute warps of this CTA
  int lane;
  int q;     // TMEM lane quadrant of this warp (warp id % 4)
  uint32_t rank;  // CTA rank in its pair (0 when single)
  int tid;   // thread index across the pair's compute warps
  int nthr;  // compute threads across the pair (128 or 256)
};

__device__ __forceinline__ void epi_sync() { named_barrier_sync(1, kEpiThreads); }

// Transpose-reduce: on entry each lane holds 32 column values of its row; on
// exit lane l holds the sum over the warp's 32 rows of column l.
__device__ __forceinline__ float warp_column_sums(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int j = 0; j < off; ++j) {
      const float send = upper ? v[j] : v[j + off];
      const float keep = upper ? v[j + off] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

__device__ __forceinline__ float load_elem(const void* base, int dtype, long long idx) {
  if (dtype == PKT_DTYPE_BF16) {
    const uint16_t h = reinterpret_cast<const uint16_t*>(base)[idx];
    return __uint_as_float(uint32_t(h) << 16);
  }
  return reinterpret_cast<const float*>(base)[idx];
}

// Loads 32 consecutive elements (bf16 or fp32 storage) of one row into v.
__device__ __forceinline__ void load_row32(const void* base, int dtype, long long idx, int nvalid,
                                           bool vec, float (&v)[32]) {
  if (vec && nvalid == 32) {
    if (dtype == PKT_DTYPE_BF16) {
      const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + idx);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 w = p[i];
        v[8 * i + 0] = bf16_lo(w.x);
        v[8 * i + 1] = bf16_hi(w.x);
        v[8 * i + 2] = bf16_lo(w.y);
        v[8 * i + 3] = bf16_hi(w.y);
        v[8 * i + 4] = bf16_lo(w.z);
        v[8 * i + 5] = bf16_hi(w.z);
        v[8 * i + 6] = bf16_lo(w.w);
        v[8 * i + 7] = bf16_hi(w.w);
      }
    } else {
      const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 w = p[i];
        v[4 * i + 0] = w.x;
        v[4 * i + 1] = w.y;
        v[4 * i + 2] = w.z;
        v[4 * i + 3] = w.w;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (j < nvalid) ? load_elem(base, dtype, idx + j) : 0.f;
  }
}

// Rounds v to the storage type in place (so later reductions see stored values)
// and stores the valid part.
__device__ __forceinline__ void store_row32(void* base, int dtype, long long idx, int nvalid,
                                            bool vec, float (&v)[32]) {
  if (dtype == PKT_DTYPE_BF16) {
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
      v[2 * i] = bf16_lo(pk[i]);
      v[2 * i + 1] = bf16_hi(pk[i]);
    }
    uint16_t* b = reinterpret_cast<uint16_t*>(base) + idx;
    if (vec && nvalid == 32) {
      uint4* p = reinterpret_cast<uint4*>(b);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        p[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) b[j] = uint16_t((j & 1) ? (pk[j >> 1] >> 16) : (pk[j >> 1] & 0xffffu));
    }
  } else {
    float* f = reinterpret_cast<float*>(base) + idx;
    if (vec && nvalid == 32) {
      float4* p = reinterpret_cast<float4*>(f);
#pragma unroll
      for (int i = 0; i < 8; ++i) p[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) f[j] = v[j];
    }
  }
}

// Writes one row of a 32x32 chunk (this lane's row) into a TMA store staging
// buffer, in the swizzled layout of the store's tensor map: bf16 rows are 64
// bytes with their 16-byte units permuted by (row / 2) % 4 (64-byte swizzle),
// fp32 rows 128 bytes permuted by row % 8 (128-byte swizzle). bf16 values are
// rounded in place, as store_row32 does.
__device__ __forceinline__ void stage_row32(uint8_t* buf, int dtype, int lane, float (&v)[32]) {
  if (dtype == PKT_DTYPE_BF16) {
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
      v[2 * i] = bf16_lo(pk[i]);
      v[2 * i + 1] = bf16_hi(pk[i]);
    }
    uint8_t* row = buf + lane * 64;
    const int x = (lane >> 1) & 3;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<uint4*>(row + ((c ^ x) << 4)) =
          make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
  } else {
    uint8_t* row = buf + lane * 128;
    const int x = lane & 7;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(row + ((c ^ x) << 4)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  }
}

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// ============================================================ GEMM epilogue
// Waits (one thread) until *ctr >= target, reading at system scope: the
// counter is advanced by other GPUs through peer memory. The budget is the
// idle one: a peer may still be finishing its previous step.
__device__ bool dp_wait_geq(const KParams& p, const int* ctr, int target, int where) {
  if (ld_acquire_sys(ctr) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t budget = 4 * p.timeout_ns + 1000000000ull;
  uint32_t it = 0;
  while (ld_acquire_sys(ctr) < target) {
    __nanosleep(64);
    if ((++it & 15u) == 0) {
      if (*status_word(p) != 0) return false;
      if (globaltimer_ns() - t0 > budget) {
        set_error(p, PKT_DEV_TIMEOUT_DEPS, -1, where);
        return false;
      }
    }
  }
  return true;
}

template <int P>
__device__ void epilogue_gemm(const KParams& p, SmemT<P>& s, const EpiCtx& c, const DevGemm& g,
                              int tile_m, int tile_n, uint32_t tmem_base, uint32_t acc,
                              uint32_t use, unsigned long long& tmem_wait, uint32_t tix) {
  const pkt_gemm_desc& d = g.d;

  // Every descriptor field the chunk loop uses goes to registers first: the
  // "memory" clobber of each tcgen05.ld would otherwise make the compiler
  // reload them from global memory inside the loop.
  const int M = d.M, N = d.N, bn = d.bn, epi = d.epilogue;
  const int out_dtype = d.out_dtype, in_dtype = d.in_dtype;
  void* const out = d.out;
  const long long ldo = d.ldo, ldaux = d.ldaux, ldy = d.ldy, ldw = d.ldw;
  const float* const bias = d.bias;
  const bool relu = d.relu != 0;
  const void* const aux = d.aux;
  float* const y_out = static_cast<float*>(d.y_out);
  const float scale = d.scale, lr = d.lr;
  const float* const w_in = d.w_in;
  float* const w_out = d.w_out;
  void* const w_shadow = d.w_shadow;
  const int rblock = tile_m * P + int(c.rank);  // 128-row block of this CTA's rows
  const int row = rblock * kBM + c.q * 32 + c.lane;
  const bool row_ok = row < M;
  const int n0 = tile_n * bn;
  const int nchunks = (bn + 31) / 32;
  const bool want_colsum = (epi == PKT_EPI_MSE || epi == PKT_EPI_DGRAD_RELU) && d.colsum != nullptr;
  const int out_es = out_dtype == PKT_DTYPE_BF16 ? 2 : 4;
  const int in_es = in_dtype == PKT_DTYPE_BF16 ? 2 : 4;
  const bool add_bias = (epi == PKT_EPI_BIAS_ACT || epi == PKT_EPI_MSE) && bias != nullptr;
  float loss = 0.f;
  // TMA tile stores: each warp stages its 32 rows x 32 columns and one lane
  // stores the box; rows past M / columns past N are clipped by the TMA unit.
  const bool tma_out = g.tma_out != 0, tma_w = g.tma_w != 0;
  uint8_t* const stg = s.epi_stage[c.q];
  const int row0 = rblock * kBM + c.q * 32;
  // WGRAD_PEER (fused data parallel): tile t belongs to rank t % world. Every
  // rank, the owner included, writes its fp32 partial rows into its own slot of
  // the tile in the owner's exchange region and counts one arrival there; the
  // owner's PKT_OP_DP_REDUCE task, listed later, sums the slots. No epilogue waits
  // on another rank. Slot rows are 256 floats.
  const DpPeers* dp = epi == PKT_EPI_WGRAD_PEER ? p.dp : nullptr;
  if (epi == PKT_EPI_WGRAD_PEER && dp == nullptr) set_error(p, PKT_DEV_BAD_ARGS, -1, -3);
  const int dp_t = g.dp_tile_base + tile_m * g.tiles_n + tile_n;
  const int dp_tl = dp != nullptr ? dp_t / dp->world : 0;
  int peer_slot_row0 = 0;      // the warp's first row in the owner's slot matrix
  int* peer_arrive = nullptr;  // the owner's arrival counter of this tile
  if (dp != nullptr) {
    uint8_t* ob = dp->base[dp_t % dp->world];
    peer_slot_row0 = int(((long long)dp_tl * dp->world + dp->rank) * dp->pair * kBM) + int(c.rank) * kBM + c.q * 32;
    peer_arrive = reinterpret_cast<int*>(ob + dp->arrive_off) + dp_tl;
  }
  // bf16 output chunks are 2 KB: three of them rotate through the warp's 6 KB
  // staging area, so a chunk is staged while the two before it are still being
  // stored; fp32 chunks (4 KB) use the area one at a time.
  const bool rotate = out_dtype == PKT_DTYPE_BF16;
  int stage_ix = 0;
  auto emit_out = [&](float (&vv)[32], int col0, int nvalid) {
    if (tma_out) {
      uint8_t* buf = stg;
      if (rotate) {
        buf = stg + stage_ix * 2048;
        stage_ix = stage_ix == 2 ? 0 : stage_ix + 1;
        if (c.lane == 0) bulk_wait_read<2>();  // the store 3 chunks back has read `buf`
      } else if (c.lane == 0) {
        bulk_wait_read_all();  // the previous chunk's store has read the buffer
      }
      __syncwarp();
      stage_row32(buf, out_dtype, c.lane, vv);
      fence_proxy_async_smem();
      __syncwarp();
      if (c.lane == 0) {
        // a group per chunk (possibly empty) keeps the group count = chunk count
        if (row0 < M && col0 < N) tma_store_2d(&g.map_out, buf, col0, row0);
        bulk_commit();
      }
    } else {
      const long long o = (long long)row * ldo + col0;
      const bool vec = aligned16(reinterpret_cast<const uint8_t*>(out) + o * out_es);
      if (nvalid > 0) store_row32(out, out_dtype, o, nvalid, vec, vv);
    }
  };

  // The aux row segment (targets for MSE, activations for the ReLU mask) of
  // chunk ch+1 is loaded into registers while chunk ch is processed: one chunk's
  // worth of loads is always in flight (whole, aligned segments only; the rest
  // take the plain per-chunk path).
  const bool aux_rows = (epi == PKT_EPI_MSE || epi == PKT_EPI_DGRAD_RELU) && aux != nullptr;
  uint4 auxq[4];
  auto aux_issue = [&](int ch2) -> bool {
    const int col = n0 + ch2 * 32;
    // bf16 rows only (16 registers); fp32 aux rows take the per-chunk path
    if (!aux_rows || in_es != 2 || !row_ok || min(N - col, bn - ch2 * 32) < 32) return false;
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(aux) +
                                                      ((long long)row * ldaux + col) * in_es);
    if (!aligned16(src)) return false;
#pragma unroll
    for (int i = 0; i < 4; ++i) auxq[i] = src[i];
    return true;
  };
  // Chunk ch's aux values: from the registers loaded one chunk ahead, else loaded now.
  auto aux_take = [&](bool ready, long long oa, int nvalid, float (&a)[32]) {
    if (ready) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[8 * i + 0] = bf16_lo(auxq[i].x);
        a[8 * i + 1] = bf16_hi(auxq[i].x);
        a[8 * i + 2] = bf16_lo(auxq[i].y);
        a[8 * i + 3] = bf16_hi(auxq[i].y);
        a[8 * i + 4] = bf16_lo(auxq[i].z);
        a[8 * i + 5] = bf16_hi(auxq[i].z);
        a[8 * i + 6] = bf16_lo(auxq[i].w);
        a[8 * i + 7] = bf16_hi(auxq[i].w);
      }
    } else if (nvalid > 0) {
      const bool avec = aligned16(reinterpret_cast<const uint8_t*>(aux) + oa * in_es);
      load_row32(aux, in_dtype, oa, nvalid, avec, a);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) a[j] = 0.f;
    }
  };
  // bias of a chunk's 32 columns: one coalesced load per warp, broadcast by
  // shuffles; chunk ch+1's is loaded while chunk ch is processed
  auto bias_issue = [&](int ch2) -> float {
    const int col = n0 + ch2 * 32 + c.lane;
    return (add_bias && col < N) ? __ldg(bias + col) : 0.f;
  };
  // The first chunk's loads (aux rows, bias) go out before the accumulator
  // wait, so their latency overlaps the end of the mainloop.
  bool auxq_ready = aux_issue(0);
  float bl_next = bias_issue(0);

  const long long c0 = clock64();
  wait_bar(p, &s.tmem_full[acc], use & 1, 8);
  tmem_wait += clock64() - c0;
  if (p.trace && c.et == 0 && c.rank == 0) p.trace[(size_t)tix * kTraceWords + kTrExec] = globaltimer_ns();
  __syncwarp();  // tcgen05.ld is warp-collective
  tc_fence_after();

  // TMEM reads are double-buffered: chunk ch+1 is in flight while chunk ch is
  // processed and stored.
  const uint32_t tbase = tmem_base + (uint32_t(c.q * 32) << 16) + acc * 256;
  uint32_t r[32];
  tmem_ld32(tbase, r);
  tmem_ld_wait_regs(r);
  for (int ch = 0; ch < nchunks; ++ch) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    const bool more = ch + 1 < nchunks;
    if (more) tmem_ld32(tbase + (ch + 1) * 32, r);
    const int col0 = n0 + ch * 32;
    int nvalid = min(N - col0, bn - ch * 32);  // inside the matrix and inside this tile
    nvalid = nvalid < 0 ? 0 : (nvalid > 32 ? 32 : nvalid);
    if (!row_ok) nvalid = 0;

    const float bl = bl_next;
    if (more) bl_next = bias_issue(ch + 1);

    if (epi == PKT_EPI_STORE || epi == PKT_EPI_WGRAD_STORE) {
      emit_out(v, col0, nvalid);
    } else if (epi == PKT_EPI_BIAS_ACT) {
      if (add_bias) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += __shfl_sync(0xffffffffu, bl, j);
      }
      if (relu) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
      }
      emit_out(v, col0, nvalid);
    } else if (epi == PKT_EPI_MSE) {
      float t[32];
      aux_take(auxq_ready, (long long)row * ldaux + col0, nvalid, t);
      auxq_ready = more ? aux_issue(ch + 1) : false;
      if (add_bias) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += __shfl_sync(0xffffffffu, bl, j);
      }
      if (relu) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
      }
      if (y_out != nullptr && nvalid > 0) {
        float y[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) y[j] = v[j];
        const long long oy = (long long)row * ldy + col0;
        store_row32(y_out, PKT_DTYPE_F32, oy, nvalid, aligned16(y_out + oy), y);
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float diff = v[j] - t[j];
        const bool ok = j < nvalid;
        loss += ok ? diff * diff : 0.f;
        float gr = scale * diff;
        if (relu && v[j] <= 0.f) gr = 0.f;
        v[j] = ok ? gr : 0.f;
      }
      emit_out(v, col0, nvalid);
    } else if (epi == PKT_EPI_DGRAD_RELU) {
      float h[32];
      aux_take(auxq_ready, (long long)row * ldaux + col0, nvalid, h);
      auxq_ready = more ? aux_issue(ch + 1) : false;
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = (j < nvalid && h[j] > 0.f) ? v[j] : 0.f;
      emit_out(v, col0, nvalid);
    } else if (epi == PKT_EPI_WGRAD_PEER) {
      // the warp's 32 x 32 fp32 chunk goes to the owner as one TMA tile store
      if (dp != nullptr) {
        if (c.lane == 0) bulk_wait_read_all();
        __syncwarp();
        stage_row32(stg, PKT_DTYPE_F32, c.lane, v);
        fence_proxy_async_smem();
        __syncwarp();
        if (c.lane == 0) {
          tma_store_2d(&dp->recv_map[dp_t % dp->world], stg, ch * 32, peer_slot_row0);
          bulk_commit();
        }
      }
    } else if (epi == PKT_EPI_WGRAD_SGD) {
      float w[32];
      const long long ow = (long long)row * ldw + col0;
      const bool wvec = aligned16(w_in + ow) && aligned16(w_out + ow);
      if (tma_w) {
        if (nvalid > 0) {
          load_row32(w_in, PKT_DTYPE_F32, ow, nvalid, wvec, w);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) w[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = fmaf(-lr, v[j], w[j]);
        if (c.lane == 0) bulk_wait_read_all();
        __syncwarp();
        stage_row32(stg, PKT_DTYPE_F32, c.lane, w);
        if (w_shadow) stage_row32(stg + 4096, PKT_DTYPE_BF16, c.lane, w);
        fence_proxy_async_smem();
        __syncwarp();
        if (c.lane == 0 && row0 < M && col0 < N) {
          tma_store_2d(&g.map_w, stg, col0, row0);
          if (w_shadow) tma_store_2d(&g.map_shadow, stg + 4096, col0, row0);
          bulk_commit();
        }
      } else if (nvalid > 0) {
        load_row32(w_in, PKT_DTYPE_F32, ow, nvalid, wvec, w);
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = fmaf(-lr, v[j], w[j]);
        float w2[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) w2[j] = w[j];
        store_row32(w_out, PKT_DTYPE_F32, ow, nvalid, wvec, w);
        if (w_shadow) {
          const bool svec = aligned16(reinterpret_cast<const uint16_t*>(w_shadow) + ow);
          store_row32(w_shadow, PKT_DTYPE_BF16, ow, nvalid, svec, w2);
        }
      }
    }

    if (want_colsum) {
      // v holds the stored (rounded) values, zero outside the valid region.
      const float cs = warp_column_sums(v, c.lane);
      s.red[ch][c.q][c.lane] = cs;
    }
    if (more) tmem_ld_wait_regs(r);
  }
  // Accumulator fully read: hand it back to the MMA warp.
  tc_fence_before();
  __syncwarp();
  if (c.lane == 0) {
    if (P == 1 || c.rank == 0)
      mbar_arrive(&s.tmem_empty[acc]);
    else
      mbar_arrive_remote(mapa_shared(smem_u32(&s.tmem_empty[acc]), 0));
  }

  if (epi == PKT_EPI_MSE && d.loss_partials != nullptr) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) loss += __shfl_xor_sync(0xffffffffu, loss, off);
    if (c.lane == 0) s.lossred[c.q] = loss;
  }
  if (want_colsum || (epi == PKT_EPI_MSE && d.loss_partials != nullptr)) {
    epi_sync();
    if (want_colsum) {
      for (int i = c.et; i < nchunks * 32; i += kEpiThreads) {
        const int ch = i >> 5, j = i & 31;
        const int col = n0 + ch * 32 + j;
        if (col < d.N && ch * 32 + j < d.bn) {
          const float tot = ((s.red[ch][0][j] + s.red[ch][1][j]) + s.red[ch][2][j]) + s.red[ch][3][j];
          d.colsum[(long long)rblock * d.ldcol + col] = tot;
        }
      }
    }
    if (epi == PKT_EPI_MSE && d.loss_partials != nullptr && c.et == 0) {
      d.loss_partials[rblock * g.tiles_n + tile_n] =
          ((s.lossred[0] + s.lossred[1]) + s.lossred[2]) + s.lossred[3];
    }
  }
  // The tile's TMA stores have landed in global memory before the caller
  // publishes the tile's completion.
  if ((tma_out || tma_w || dp != nullptr) && c.lane == 0) bulk_wait_all();
  __syncwarp();
  if (dp != nullptr) {
    // every thread's rows (TMA stores included) visible system-wide, then one
    // arrive per CTA on the owner's counter of this tile
    fence_proxy_async_global();
    __threadfence_system();
    epi_sync();
    if (c.et == 0) red_release_sys_add(peer_arrive, 1);
  }
}

// ============================================================ SIMT ops
// Element-wise ops stride over every compute thread of the CTA (or CTA pair):
// `et` is the thread's index, `nthr` the thread count.
__device__ void op_axpy(const AxpyArgs& a, int et, int nthr) {
  const long long n = a.n;
  if (aligned16(a.x) && aligned16(a.y)) {
    const long long n4 = n >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    float4* y4 = reinterpret_cast<float4*>(a.y);
    long long i = et;
    // 16 float4 of x and of y in flight per thread (64 KB per 128 threads): the
    // latency of HBM needs that many bytes outstanding per SM to reach its bandwidth
    constexpr int U = 16;
    // Thread 0 of the task's threads asks the TMA unit to bring the window two
    // iterations ahead into L2 (each iteration of all threads covers one
    // contiguous window of U * nthr float4): HBM then sees the bulk engine's
    // parallelism, and the threads' loads mostly hit L2.
    const long long win = (long long)U * nthr;
    auto prefetch = [&](long long w0) {
      if (w0 >= n4) return;
      const uint32_t bytes = uint32_t(min(win, n4 - w0) * 16);
      prefetch_l2_bulk(x4 + w0, bytes);
      prefetch_l2_bulk(y4 + w0, bytes);
    };
    if (et == 0) {
      prefetch(0);
      prefetch(win);
    }
    for (; i + (U - 1) * nthr < n4; i += U * nthr) {
      if (et == 0) prefetch(i + 2 * win);
      float4 xv[U], yv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        xv[u] = __ldcs(x4 + i + u * nthr);
        yv[u] = __ldcs(y4 + i + u * nthr);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        yv[u].x = fmaf(a.a, xv[u].x, yv[u].x);
        yv[u].y = fmaf(a.a, xv[u].y, yv[u].y);
        yv[u].z = fmaf(a.a, xv[u].z, yv[u].z);
        yv[u].w = fmaf(a.a, xv[u].w, yv[u].w);
        __stcs(y4 + i + u * nthr, yv[u]);
      }
    }
    for (; i < n4; i += nthr) {
      const float4 xv = x4[i];
      float4 yv = y4[i];
      yv.x = fmaf(a.a, xv.x, yv.x);
      yv.y = fmaf(a.a, xv.y, yv.y);
      yv.z = fmaf(a.a, xv.z, yv.z);
      yv.w = fmaf(a.a, xv.w, yv.w);
      y4[i] = yv;
    }
    for (long long k = n4 * 4 + et; k < n; k += nthr) a.y[k] = fmaf(a.a, a.x[k], a.y[k]);
  } else {
    for (long long k = et; k < n; k += nthr) a.y[k] = fmaf(a.a, a.x[k], a.y[k]);
  }
}

__device__ void op_zero(const ZeroMemoryArgs& a, int et, int nthr) {
  const long long n = a.size;
  if (aligned16(a.ptr)) {
    const long long n4 = n >> 2;
    float4* p4 = reinterpret_cast<float4*>(a.ptr);
    for (long long i = et; i < n4; i += nthr) p4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (long long k = n4 * 4 + et; k < n; k += nthr) a.ptr[k] = 0.f;
  } else {
    for (long long k = et; k < n; k += nthr) a.ptr[k] = 0.f;
  }
}

// w_out = w - lr*g (single-rounding fma, as nvcc compiles pkt's `W[i] -= lr*dW[i]`,
// include/ops/sgd.cuh:41-43), optionally also writing the bf16 copy of w_out.
__device__ void op_sgd(const float* W, const float* dW, float* Wo, float lr, long long n,
                       uint16_t* shadow, int et, int nthr) {
  const bool vec = aligned16(W) && aligned16(dW) && aligned16(Wo) &&
                   (shadow == nullptr || (reinterpret_cast<uintptr_t>(shadow) & 7u) == 0);
  long long head = 0;
  if (vec) {
    const long long n4 = n >> 2;
    const float4* w4 = reinterpret_cast<const float4*>(W);
    const float4* g4 = reinterpret_cast<const float4*>(dW);
    float4* o4 = reinterpret_cast<float4*>(Wo);
    long long i = et;
    // 12 float4 of w and of g in flight per thread (48 KB per 128 threads)
    constexpr int U = 12;
    // thread 0 brings the window two iterations ahead into L2 (as op_axpy)
    const long long win = (long long)U * nthr;
    auto prefetch = [&](long long w0) {
      if (w0 >= n4) return;
      const uint32_t bytes = uint32_t(min(win, n4 - w0) * 16);
      prefetch_l2_bulk(w4 + w0, bytes);
      prefetch_l2_bulk(g4 + w0, bytes);
    };
    if (et == 0) {
      prefetch(0);
      prefetch(win);
    }
    for (; i + (U - 1) * nthr < n4; i += U * nthr) {
      if (et == 0) prefetch(i + 2 * win);
      float4 w[U], g[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        w[u] = __ldcs(w4 + i + u * nthr);
        g[u] = __ldcs(g4 + i + u * nthr);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        w[u].x = fmaf(-lr, g[u].x, w[u].x);
        w[u].y = fmaf(-lr, g[u].y, w[u].y);
        w[u].z = fmaf(-lr, g[u].z, w[u].z);
        w[u].w = fmaf(-lr, g[u].w, w[u].w);
        o4[i + u * nthr] = w[u];
        if (shadow)
          reinterpret_cast<uint2*>(shadow)[i + u * nthr] =
              make_uint2(pack_bf16x2(w[u].x, w[u].y), pack_bf16x2(w[u].z, w[u].w));
      }
    }
    for (; i < n4; i += nthr) {
      float4 w = w4[i];
      const float4 g = g4[i];
      w.x = fmaf(-lr, g.x, w.x);
      w.y = fmaf(-lr, g.y, w.y);
      w.z = fmaf(-lr, g.z, w.z);
      w.w = fmaf(-lr, g.w, w.w);
      o4[i] = w;
      if (shadow)
        reinterpret_cast<uint2*>(shadow)[i] = make_uint2(pack_bf16x2(w.x, w.y), pack_bf16x2(w.z, w.w));
    }
    head = n4 * 4;
  }
  for (long long k = head + et; k < n; k += nthr) {
    const float w = fmaf(-lr, dW[k], W[k]);
    Wo[k] = w;
    if (shadow) shadow[k] = f32_to_bf16_rn(w);
  }
}

// Deterministic sum over the 128 compute threads (fixed order), result on et == 0.
template <int P>
__device__ float epi_block_sum(SmemT<P>& s, const EpiCtx& c, float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if (c.lane == 0) s.simt_red[c.et >> 5] = v;
  epi_sync();
  float tot = ((s.simt_red[0] + s.simt_red[1]) + s.simt_red[2]) + s.simt_red[3];
  epi_sync();
  return tot;
}

template <int P>
__device__ void op_mse(SmemT<P>& s, const EpiCtx& c, const MSELossArgs& a) {
  const long long elems = (long long)a.batch * a.m;
  const float scale = 2.0f / float(a.batch * a.m);
  float part = 0.f;
  for (long long i = c.et; i < elems; i += kEpiThreads) {
    const float diff = a.y[i] - a.target[i];
    a.dy[i] = scale * diff;
    part = fmaf(diff, diff, part);
  }
  const float tot = epi_block_sum(s, c, part);
  if (c.et == 0) atomicAdd(a.loss, tot / float(elems));
}

// pkt's LinearForward task (include/ops/linear_fwd.cuh:18-29):
// y[b, j] = sum_k x[b, k] W[j, k] over its rows x columns tile, fp32 throughout
// (pkt rounds x to fp16 first; this keeps fp32). The tile's x rows are staged in
// shared memory (the epilogue staging area, free during element-wise tasks);
// each warp then owns output columns: its lanes stride K, reading W[j, :]
// coalesced once for all the tile's rows (four accumulators at a time), and a
// shuffle reduction gives the sums. Rows that do not fit the staging area are
// read from global memory instead.
template <int P>
__device__ void op_linear_forward(SmemT<P>& s, const EpiCtx& c, const LinearForwardArgs& a) {
  const int r0 = a.tile_m_start, c0 = a.tile_n_start, n = a.n;
  const int rows = max(0, min(a.tile_m_count, a.batch - r0));
  const int cols = max(0, min(a.tile_n_count, a.m - c0));
  float* xs = reinterpret_cast<float*>(&s.epi_stage[0][0]);
  const bool staged = (long long)rows * n <= (long long)sizeof(s.epi_stage) / 4;
  if (staged) {
    for (long long i = c.et; i < (long long)rows * n; i += kEpiThreads) xs[i] = a.x[(long long)r0 * n + i];
    epi_sync();
  }
  const float* xr = staged ? xs : a.x + (long long)r0 * n;
  const int warp = c.tid >> 5, nwarps = c.nthr >> 5;
  for (int j = warp; j < cols; j += nwarps) {
    const float* w = a.W + (long long)(c0 + j) * n;
    for (int rb = 0; rb < rows; rb += 4) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const int nr = min(4, rows - rb);
      for (int k = c.lane; k < n; k += 32) {
        const float wk = w[k];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (q < nr) acc[q] = fmaf(xr[(long long)(rb + q) * n + k], wk, acc[q]);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], off);
      }
      if (c.lane < nr) {
        float v = acc[0];
#pragma unroll
        for (int q = 1; q < 4; ++q) v = c.lane == q ? acc[q] : v;
        a.y[(long long)(r0 + rb + c.lane) * a.m + c0 + j] = v;
      }
    }
  }
  if (staged) epi_sync();  // the staging area is free again for the next task
}

__device__ void op_linear_backward(const LinearBackwardArgs& a, int et, int nthr) {
  // dW[r, c] = sum_b dy[b, r] x[b, c], overwriting the tile (include/ops/linear_bwd.cuh:94-157).
  const int rows = a.tile_m_count, cols = a.tile_n_count;
  const long long total = (long long)rows * cols;
  for (long long o = et; o < total; o += nthr) {
    const int r = a.tile_m_start + int(o / cols);
    const int cc = a.tile_n_start + int(o % cols);
    if (r >= a.m || cc >= a.n) continue;
    float acc = 0.f;
    for (int b = 0; b < a.batch; ++b) acc = fmaf(a.dy[(long long)b * a.m + r], a.x[(long long)b * a.n + cc], acc);
    a.dW[(long long)r * a.n + cc] = acc;
  }
}

// Column sums of `num` partial rows (row stride ld floats), summed from row 0
// up -- the order every path of the engine uses, so their results are
// bit-identical. Eight rows' loads are in flight before any is added.
__device__ __forceinline__ float column_sum_in_order(const float* partials, int num, long long ld, int col) {
  float sum = 0.f;
  int r = 0;
  for (; r + 8 <= num; r += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldcg(partials + (long long)(r + j) * ld + col);
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += v[j];
  }
  for (; r < num; ++r) sum += __ldcg(partials + (long long)r * ld + col);
  return sum;
}

// The same for four adjacent columns (col and ld multiples of 4, partials 16-byte aligned).
__device__ __forceinline__ float4 column_sum4_in_order(const float* partials, int num, long long ld, int col) {
  float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
  int r = 0;
  for (; r + 8 <= num; r += 8) {
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldcg(reinterpret_cast<const float4*>(partials + (long long)(r + j) * ld + col));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sum.x += v[j].x;
      sum.y += v[j].y;
      sum.z += v[j].z;
      sum.w += v[j].w;
    }
  }
  for (; r < num; ++r) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(partials + (long long)r * ld + col));
    sum.x += v.x;
    sum.y += v.y;
    sum.z += v.z;
    sum.w += v.w;
  }
  return sum;
}

// Calls f(col, sum) for every column of [c0, c1), the columns spread over the
// task's threads four at a time where the layout allows.
template <class F>
__device__ __forceinline__ void for_column_sums(const float* partials, int num, long long ld, int c0, int c1,
                                                int et, int nthr, F&& f) {
  if (aligned16(partials) && (ld & 3) == 0 && (c0 & 3) == 0) {
    for (int col = c0 + 4 * et; col < c1; col += 4 * nthr) {
      if (col + 4 <= c1) {
        const float4 v = column_sum4_in_order(partials, num, ld, col);
        f(col, v.x);
        f(col + 1, v.y);
        f(col + 2, v.z);
        f(col + 3, v.w);
      } else {
        for (int k = col; k < c1; ++k) f(k, column_sum_in_order(partials, num, ld, k));
      }
    }
  } else {
    for (int col = c0 + et; col < c1; col += nthr) f(col, column_sum_in_order(partials, num, ld, col));
  }
}

__device__ void op_bias_sgd(const pkt_bias_sgd_args& a, int et, int nthr) {
  for_column_sums(a.partials, a.num_partials, a.ld, a.col_begin, a.col_end, et, nthr, [&](int col, float sum) {
    if (a.grad_out) a.grad_out[col] = sum;
    if (a.bias) a.bias[col] = fmaf(-a.lr, sum, a.bias[col]);
  });
}

// ============================================================ fused data parallel
// Next step's weights of one layer: every owner's broadcast of every tile of
// the layer (one arrive per CTA of the owner's pair) has landed here.
__device__ void op_dp_wait(const KParams& p, const EpiCtx& c, const pkt_dp_wait_args& a) {
  const DpPeers* dp = p.dp;
  if (c.et == 0 && dp != nullptr) {
    const int* ctr = reinterpret_cast<const int*>(dp->base[dp->rank] + dp->wready_off) + a.layer;
    dp_wait_geq(p, ctr, p.dp_step * a.tiles * dp->pair, 1000 + a.layer);
  }
  epi_sync();
}

// An owned weight tile of the step (fused data parallel): once every rank's
// partial of the tile has arrived in this rank's slots (its arrival counter,
// one count per rank and CTA of a pair), the partials are summed in rank order,
// SGD updates the fp32 master (this rank owns it) and the new bf16 values go to
// every rank's copy of the next step's weights, own included; then every rank's
// "layer weights arrived" counter gets one count per CTA. A wait that runs out
// (the status word is set) leaves the master and every copy as they were and
// counts nothing, so the step fails without corrupting the weights.
template <int P>
__device__ void op_dp_reduce(const KParams& p, SmemT<P>& s, const EpiCtx& c, const pkt_gemm_tile_args& a,
                             unsigned long long* tr) {
  const DpPeers* dp = p.dp;
  if (dp == nullptr || int(a.gemm) >= p.num_gemms) return;
  const DevGemm& g = p.gemms[a.gemm];
  const pkt_gemm_desc& d = g.d;
  const int t = g.dp_tile_base + int(a.tile_m) * g.tiles_n + int(a.tile_n);
  const int tl = t / dp->world;
  uint8_t* own = dp->base[dp->rank];
  if (c.et == 0)
    s.dp_ok = int(dp_wait_geq(p, reinterpret_cast<const int*>(own + dp->arrive_off) + tl,
                              (p.dp_step + 1) * dp->world * dp->pair, 4000 + g.dp_layer));
  epi_sync();
  const bool ok = s.dp_ok != 0;
  epi_sync();  // every thread has read the flag before the next task may rewrite it
  if (tr) tr[kTrLoad] = globaltimer_ns();  // (SIMT tasks have no loads: the wait's end)
  if (!ok) return;
  const int rows_tile = dp->pair * kBM;
  const int row0 = int(a.tile_m) * rows_tile, n0 = int(a.tile_n) * d.bn;
  const int rows = min(rows_tile, d.M - row0), cols = min(d.bn, d.N - n0);
  const float* slots = reinterpret_cast<const float*>(own + dp->recv_off + (long long)tl * dp->world * dp->slot_bytes);
  const long long slot_floats = dp->slot_bytes / 4;
  const long long shadow_off = reinterpret_cast<const uint8_t*>(d.w_shadow) - own;
  const float lr = d.lr;
  const long long ldw = d.ldw;
  const int cg = (cols + 3) / 4;  // groups of 4 columns per row
  const int total = rows * cg;
  const bool vec = (cols & 3) == 0 && (ldw & 3) == 0 && (n0 & 3) == 0 &&
                   ((reinterpret_cast<uintptr_t>(d.w_in) | reinterpret_cast<uintptr_t>(d.w_out)) & 15) == 0 &&
                   (shadow_off & 7) == 0;
  if (vec) {
    // U groups of 4 columns per thread and pass, every load of a pass issued
    // before any of them is used: the slots and the master are read with U x
    // (world + 1) 16-byte loads in flight per thread instead of one dependent
    // chain, which is what bounds this pass (it moves ~20 bytes per element).
    constexpr int U = 8;
    for (int e0 = c.tid; e0 < total; e0 += U * c.nthr) {
      float4 gs[U], wv[U];
      int soff[U];
      long long idx[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int e = min(e0 + u * c.nthr, total - 1);  // tail: repeats a valid group, stored once
        const int r = e / cg, c4 = (e - r * cg) * 4;
        soff[u] = r * 256 + c4;
        idx[u] = (long long)(row0 + r) * ldw + n0 + c4;
        gs[u] = __ldcg(reinterpret_cast<const float4*>(slots + soff[u]));
        wv[u] = *reinterpret_cast<const float4*>(d.w_in + idx[u]);
      }
      for (int src = 1; src < dp->world; ++src) {
        float4 q[U];
#pragma unroll
        for (int u = 0; u < U; ++u) q[u] = __ldcg(reinterpret_cast<const float4*>(slots + src * slot_floats + soff[u]));
#pragma unroll
        for (int u = 0; u < U; ++u) {
          gs[u].x += q[u].x;
          gs[u].y += q[u].y;
          gs[u].z += q[u].z;
          gs[u].w += q[u].w;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (e0 + u * c.nthr >= total) break;
        float4 w;
        w.x = fmaf(-lr, gs[u].x, wv[u].x);
        w.y = fmaf(-lr, gs[u].y, wv[u].y);
        w.z = fmaf(-lr, gs[u].z, wv[u].z);
        w.w = fmaf(-lr, gs[u].w, wv[u].w);
        *reinterpret_cast<float4*>(d.w_out + idx[u]) = w;
        const uint2 pk = make_uint2(pack_bf16x2(w.x, w.y), pack_bf16x2(w.z, w.w));
        for (int r2 = 0; r2 < dp->world; ++r2)
          *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(dp->base[r2] + shadow_off) + idx[u]) = pk;
      }
    }
  } else {
    for (int e = c.tid; e < total; e += c.nthr) {
      const int r = e / cg, c4 = (e % cg) * 4;
      const int nv = min(4, cols - c4);
      float gs[4] = {0.f, 0.f, 0.f, 0.f};
      for (int src = 0; src < dp->world; ++src) {
        const float* sp = slots + src * slot_floats + (long long)r * 256 + c4;
        for (int k = 0; k < nv; ++k) gs[k] = src == 0 ? __ldcg(sp + k) : gs[k] + __ldcg(sp + k);
      }
      const long long idx = (long long)(row0 + r) * ldw + n0 + c4;
      for (int k = 0; k < nv; ++k) {
        const float w = fmaf(-lr, gs[k], d.w_in[idx + k]);
        d.w_out[idx + k] = w;
        const uint16_t h = f32_to_bf16_rn(w);
        for (int r2 = 0; r2 < dp->world; ++r2)
          reinterpret_cast<uint16_t*>(dp->base[r2] + shadow_off)[idx + k] = h;
      }
    }
  }
  __threadfence_system();
  epi_sync();
  if (c.et == 0)
    for (int r2 = 0; r2 < dp->world; ++r2)
      red_release_sys_add(reinterpret_cast<int*>(dp->base[r2] + dp->wready_off) + g.dp_layer, 1);
}

// This rank's bias gradient of one layer (column partials summed in row-block
// order) into every rank's receive vector for this step's parity.
__device__ void op_dp_bias_send(const KParams& p, const EpiCtx& c, const pkt_dp_bias_args& a) {
  const DpPeers* dp = p.dp;
  if (dp == nullptr) return;
  const int par = p.dp_step & 1;
  const long long off = ((long long)(par * dp->world + dp->rank)) * dp->bias_total + a.bias_off;
  for_column_sums(a.partials, a.num_partials, a.ld, 0, a.n, c.tid, c.nthr, [&](int col, float sum) {
    for (int r2 = 0; r2 < dp->world; ++r2)
      reinterpret_cast<float*>(dp->base[r2] + dp->bias_recv_off)[off + col] = sum;
  });
  __threadfence_system();
  epi_sync();
  if (c.et == 0)
    for (int r2 = 0; r2 < dp->world; ++r2)
      red_release_sys_add(reinterpret_cast<int*>(dp->base[r2] + dp->barrive_off) + a.layer, 1);
}

// Every rank sums the ranks' bias gradients in rank order and applies the same
// update, so the replicated biases stay bit-identical.
__device__ void op_dp_bias_apply(const KParams& p, const EpiCtx& c, const pkt_dp_bias_args& a) {
  const DpPeers* dp = p.dp;
  if (dp == nullptr) return;
  uint8_t* own = dp->base[dp->rank];
  if (c.et == 0) {
    const int* ctr = reinterpret_cast<const int*>(own + dp->barrive_off) + a.layer;
    dp_wait_geq(p, ctr, (p.dp_step + 1) * dp->world * dp->pair, 3000 + a.layer);
  }
  epi_sync();
  const int par = p.dp_step & 1;
  const float* recv = reinterpret_cast<const float*>(own + dp->bias_recv_off) +
                      (long long)par * dp->world * dp->bias_total + a.bias_off;
  for (int col = c.tid; col < a.n; col += c.nthr) {
    float sum = 0.f;
    for (int src = 0; src < dp->world; ++src) sum += __ldcg(recv + (long long)src * dp->bias_total + col);
    a.bias[col] = fmaf(-a.lr, sum, a.bias[col]);
  }
}

template <int P>
__device__ void op_loss_reduce(SmemT<P>& s, const EpiCtx& c, const pkt_loss_reduce_args& a) {
  double part = 0.0;
  for (int i = c.et; i < a.count; i += kEpiThreads) part += double(a.partials[i]);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
  if (c.lane == 0) s.simt_redd[c.et >> 5] = part;
  epi_sync();
  if (c.et == 0) {
    const double tot = ((s.simt_redd[0] + s.simt_redd[1]) + s.simt_redd[2]) + s.simt_redd[3];
    float* dst = a.loss;
    if (a.step) dst += (*a.step)++;
    *dst = float(tot * double(a.scale));
  }
  epi_sync();
}

// ============================================================ pk::OpTraits ops
// A program's own ops (pk::OpSet, pk/kernel.cuh) run with pkt's three phases
// (pkt include/dispatch.cuh:31-179): load by one warp, compute by the four compute
// warps (compute_warp_idx 0-3), store by one warp, in that order, all on the
// compute warps of this CTA (of the leader CTA in pair mode: pkt runs a task on
// one CTA). The op sees its task as br.slot(0) and pages 0 and 1 of slot 0,
// which live in the epilogue staging area: a tag (pkt's page reuse) survives
// from one such op to the next and is cleared by any GEMM tile in between.
template <int P, class Ops>
__device__ void run_user_op(SmemT<P>& s, const EpiCtx& c, const pkt_task& task) {
  if (c.rank != 0) return;
  const uint16_t op = task.header.opcode;
  if (c.et == 0) copy_task(reinterpret_cast<pkt_task*>(&s.user_slot.task), &task);
  epi_sync();
  pk::BlockRuntime br;
  br.slots = &s.user_slot;
  br.num_slots = 1;
  br.pages = reinterpret_cast<pk::Page*>(&s.epi_stage[0][0]);
  br.num_pages = pk::Config::kPagesPerSlot;
  br.page_meta = s.page_meta;
  const pk::Task& t = s.user_slot.task;
  const int cw = c.et >> 5;
  if (cw == 0) Ops::load(op, t, br, 0, c.lane, nullptr, nullptr);
  epi_sync();
  Ops::compute(op, t, br, 0, c.lane, cw, kEpiThreads / 32);
  epi_sync();
  if (cw == 0) Ops::store(op, t, br, 0, c.lane);
}

// ============================================================ compute warps
template <int P, class Ops>
__device__ void compute_loop(const KParams& p, SmemT<P>& s, uint32_t tmem_base, const EpiCtx& c,
                             unsigned long long* perf) {
  int seq = 0;
  uint32_t gemm_count = 0;
  unsigned long long tmem_wait = 0, gemm_cycles = 0, simt_cycles = 0;
  while (true) {
    const int slot = seq % kSlots;
    if (!wait_bar<(P == 2)>(p, &s.slot_full[slot], (seq / kSlots) & 1, 9, true)) break;
    pkt_task task;
    copy_task(&task, &s.slots[slot]);
    epi_sync();  // every compute thread has its copy
    if (c.et == 0) release_slot<P>(s, slot, c.rank);
    ++seq;
    if (c.et == 0 && c.rank == 0) *reinterpret_cast<volatile int*>(&s.taken) = seq;
    const uint16_t op = task.header.opcode;
    if (op == kOpStop) break;
    const long long c0 = clock64();
    unsigned long long* tr = (p.trace && c.et == 0 && c.rank == 0)
                                 ? p.trace + (size_t)task.header.user_tag * kTraceWords : nullptr;
    if (tr && op != PKT_OP_GEMM) tr[kTrExec] = globaltimer_ns();
    if (Ops::handles(op)) {
      run_user_op<P, Ops>(s, c, task);
    } else switch (op) {
      case PKT_OP_GEMM: {
        const pkt_gemm_tile_args& ga = *reinterpret_cast<const pkt_gemm_tile_args*>(task.args);
        const uint32_t acc = gemm_count & 1, use = gemm_count >> 1;
        epilogue_gemm<P>(p, s, c, p.gemms[ga.gemm], int(ga.tile_m), int(ga.tile_n), tmem_base, acc,
                         use, tmem_wait, task.header.user_tag);
        ++gemm_count;
        break;
      }
      case PKT_OP_AXPY:
        op_axpy(*reinterpret_cast<const AxpyArgs*>(task.args), c.tid, c.nthr);
        break;
      case PKT_OP_ZERO_MEMORY:
        op_zero(*reinterpret_cast<const ZeroMemoryArgs*>(task.args), c.tid, c.nthr);
        break;
      case PKT_OP_SGD_UPDATE: {
        const SGDUpdateArgs& a = *reinterpret_cast<const SGDUpdateArgs*>(task.args);
        op_sgd(a.W, a.dW, a.W, a.lr, a.size, nullptr, c.tid, c.nthr);
        break;
      }
      case PKT_OP_SGD_MIXED: {
        const pkt_sgd_mixed_args& a = *reinterpret_cast<const pkt_sgd_mixed_args*>(task.args);
        op_sgd(a.w, a.g, a.w_out ? a.w_out : const_cast<float*>(a.w), a.lr, a.n, a.w_bf16, c.tid,
               c.nthr);
        break;
      }
      case PKT_OP_MSE_LOSS:
        if (c.rank == 0) op_mse<P>(s, c, *reinterpret_cast<const MSELossArgs*>(task.args));
        break;
      case PKT_OP_LINEAR_FORWARD:
        op_linear_forward<P>(s, c, *reinterpret_cast<const LinearForwardArgs*>(task.args));
        break;
      case PKT_OP_LINEAR_BACKWARD:
        op_linear_backward(*reinterpret_cast<const LinearBackwardArgs*>(task.args), c.tid, c.nthr);
        break;
      case PKT_OP_BIAS_SGD:
        op_bias_sgd(*reinterpret_cast<const pkt_bias_sgd_args*>(task.args), c.tid, c.nthr);
        break;
      case PKT_OP_DP_WAIT:
        op_dp_wait(p, c, *reinterpret_cast<const pkt_dp_wait_args*>(task.args));
        break;
      case PKT_OP_DP_BIAS_SEND:
        op_dp_bias_send(p, c, *reinterpret_cast<const pkt_dp_bias_args*>(task.args));
        break;
      case PKT_OP_DP_REDUCE:
        op_dp_reduce<P>(p, s, c, *reinterpret_cast<const pkt_gemm_tile_args*>(task.args), tr);
        break;
      case PKT_OP_DP_BIAS_APPLY:
        op_dp_bias_apply(p, c, *reinterpret_cast<const pkt_dp_bias_args*>(task.args));
        break;
      case PKT_OP_LOSS_REDUCE:
        if (c.rank == 0) op_loss_reduce<P>(s, c, *reinterpret_cast<const pkt_loss_reduce_args*>(task.args));
        break;
      default:  // PKT_OP_INVALID: no work, tokens are still published
        break;
    }
    if (op == PKT_OP_GEMM) {
      gemm_cycles += clock64() - c0;
      // the epilogue staging doubles as the pages of pk::OpTraits ops: their
      // contents (and tags) are gone
      if (c.et < pk::Config::kPagesPerSlot) s.page_meta[c.et].reset();
    } else {
      simt_cycles += clock64() - c0;
    }
    if (tr) tr[kTrDone] = globaltimer_ns();
    // ---- publish completion. Every thread's stores are ordered before the
    // barrier; thread 0's release of the token is cumulative over what the
    // barrier ordered before it, so it needs no separate fence. The proxy fence
    // orders this thread's async-proxy (TMA store) writes, complete by now, with
    // the generic release. In a pair the other CTA fences its half at gpu scope
    // before it signals the leader.
    fence_proxy_async_global();
    epi_sync();
    if (P == 2 && c.et == 0 && c.rank != 0) __threadfence();
    if (P == 2 && c.et == 0) {
      // pair: the leader publishes once the other CTA's half is stored too
      const int ps = (seq - 1) % kSlots;
      if (c.rank != 0) {
        mbar_arrive_remote(mapa_shared(smem_u32(&s.pair_done[ps]), 0));
      } else {
        wait_bar<true>(p, &s.pair_done[ps], ((seq - 1) / kSlots) & 1, 10);
      }
    }
    if (c.et == 0 && c.rank == 0) {
      const pkt_task_header& h = task.header;
      if (h.buffer_write_id != 0) {
        atomicMax(tok_epoch(p) + h.buffer_write_id, int(h.write_epoch));
        red_release_gpu_add(tok_count(p) + h.buffer_write_id, 1);
      }
      const int w2 = int(h.ext_ids >> 16);
      if (w2 != 0) red_release_gpu_add(tok_count(p) + w2, 1);
    }
  }
  if (perf && c.et == 0) {
    perf[kPerfEpiTmemWait] = tmem_wait;
    perf[kPerfEpiGemm] = gemm_cycles;
    perf[kPerfEpiSimt] = simt_cycles;
  }
}

// P = 1: every CTA works alone. P = 2: launched in clusters of two; the pair
// shares one task ring (rank 0's controller feeds both CTAs), rank 0 issues the
// cta_group::2 MMAs for 256-row tiles, both CTAs load their operand halves and
// run the epilogue for their 128 rows.
template <int P, class Ops>
__global__ void __launch_bounds__(kThreads, 1) pk_megakernel(const __grid_constant__ KParams p) {
  extern __shared__ uint8_t smem_raw[];
  SmemT<P>& s = *reinterpret_cast<SmemT<P>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int NST = SmemT<P>::NST;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = P == 2 ? cluster_ctarank() : 0;
  unsigned long long* perf = p.perf ? p.perf + (size_t)blockIdx.x * PKT_PERF_WORDS : nullptr;
  const long long t_start = clock64();
  const uint64_t g_start = (p.clock_acc && blockIdx.x == 0 && threadIdx.x == 0) ? globaltimer_ns() : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&s.slot_full[i], 1);
      // leader: loader, MMA issuer, compute warps (+ the other CTA's loader and compute warps)
      mbar_init(&s.slot_empty[i], P == 2 ? 5 : 3);
      mbar_init(&s.pair_done[i], 1);
    }
    for (int i = 0; i < pk::Config::kPagesPerSlot; ++i) s.page_meta[i].reset();
    s.taken = 0;
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], 4 * P);  // one arrive per compute warp (of both CTAs)
    }
    mbar_init(&s.mma_drain, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    if (P == 2) {
      tmem_alloc_pair(&s.tmem_base, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&s.tmem_base, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (P == 2) cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;

  if (warp == kCtrlWarp) {
    if (lane == 0 && rank == 0) controller_loop<P, Ops>(p, s, perf);
    __syncwarp();
  } else if (warp == kLoadWarp) {
    if (lane == 0) loader_loop<P>(p, s, rank, perf);
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (rank == 0) mma_loop<P>(p, s, tmem_base, perf);
    __syncwarp();
  } else {
    const int et = int(threadIdx.x) - kEpiWarp0 * 32;
    EpiCtx c{et, lane, warp & 3, rank, int(rank) * kEpiThreads + et, kEpiThreads * P};
    compute_loop<P, Ops>(p, s, tmem_base, c, perf);
  }

  tc_fence_before();
  __syncthreads();
  if (P == 2) cluster_sync();  // neither CTA releases TMEM / exits while the other still works
  if (warp == kMmaWarp) {
    tc_fence_after();
    if (P == 2)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
  if (perf && threadIdx.x == 0) perf[kPerfTotal] = clock64() - t_start;
  if (p.clock_acc && blockIdx.x == 0 && threadIdx.x == 0) {
    // SM cycles and nanoseconds of CTA 0's lifetime (about the launch's):
    // their ratio over many launches is the effective SM clock of a timed region
    atomicAdd(p.clock_acc, static_cast<unsigned long long>(clock64() - t_start));
    atomicAdd(p.clock_acc + 1, static_cast<unsigned long long>(globaltimer_ns() - g_start));
    atomicAdd(p.clock_acc + 2, 1ull);
  }
}

template <int P>
cudaLaunchConfig_t make_config(int blocks, cudaStream_t stream, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes<P>();
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = P;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace

// Per device and per kernel instantiation: the shared-memory attribute is set
// once, and the number of CTAs that can be resident at the same time (clusters x
// P) is looked up once. Concurrent first launches from several host threads are
// serialised here.
template <int P, class Ops = NoUserOps>
cudaError_t prepare_variant(int dev, int* resident) {
  static std::mutex mu;
  static int cached[64] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (cached[dev] == 0) {
    cudaError_t e = cudaFuncSetAttribute(pk_megakernel<P, Ops>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_bytes<P>());
    if (e != cudaSuccess) return e;
    int n = 0;
    if (P == 1) {
      int per_sm = 0, sms = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pk_megakernel<1, Ops>, kThreads, smem_bytes<1>());
      if (e != cudaSuccess) return e;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return e;
      n = per_sm * sms;
    } else {
      cudaLaunchAttribute attr[1];
      cudaLaunchConfig_t cfg = make_config<P>(P, nullptr, attr);
      int clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&clusters, pk_megakernel<P, Ops>, &cfg);
      if (e != cudaSuccess) return e;
      n = clusters * P;
    }
    if (n <= 0) return cudaErrorInvalidConfiguration;
    cached[dev] = n;
  }
  *resident = cached[dev];
  return cudaSuccess;
}

template <int P, class Ops = NoUserOps>
cudaError_t launch_variant(const KParams& p, int blocks, cudaStream_t stream) {
  int dev = 0, resident = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = prepare_variant<P, Ops>(dev, &resident);
  if (e != cudaSuccess) return e;
  if (blocks > resident) return cudaErrorInvalidConfiguration;  // callers clamp first
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_config<P>(blocks, stream, attr);
  return cudaLaunchKernelEx(&cfg, pk_megakernel<P, Ops>, p);
}

// Launches the megakernel instantiated with a program's own ops (pk::OpSet).
template <class Ops>
cudaError_t launch_megakernel_ops(const KParams& p, int blocks, cudaStream_t stream, int pair) {
  if (pair == 2) return launch_variant<2, Ops>(p, blocks, stream);
  return launch_variant<1, Ops>(p, blocks, stream);
}

}  // namespace pkb
