// pk::BlockRuntime and its shared-memory pages: what a pk::OpTraits op's load /
// compute / store functions receive (pkt include/block_runtime.cuh:14-179, same
// names and member functions). In this build the megakernel runs such an op's
// three phases one after another on its compute warps (pk/kernel.cuh), so a
// page's lease is never contended; the lease and tag protocol is kept so ops
// written for pkt (tag-checked reuse of a staged tile, pkt
// include/ops/linear_fwd.cuh:194-247) work unchanged.
#pragma once

#include <cstddef>
#include <cstdint>

#include "config.cuh"
#include "dependency.cuh"
#include "pipeline.cuh"
#include "queue.cuh"

namespace pk {

struct Page {
  alignas(16) std::byte data[Config::kPageBytes];

  template <typename T>
  __device__ inline T* as() {
    static_assert(alignof(T) <= 16, "T alignment too large for Page");
    return reinterpret_cast<T*>(data);
  }
  template <typename T>
  __device__ inline const T* as() const {
    static_assert(alignof(T) <= 16, "T alignment too large for Page");
    return reinterpret_cast<const T*>(data);
  }
};

enum class PageLease : int { Free = 0, Loader = 1, Ready = 2, Storer = 3 };

struct PageHandle {
  int slot_idx{0};
  int page_idx{0};
};

// Lease state and content tag of one page (shared memory; block-scope atomics).
struct PageMeta {
  int lease;
  int pad;
  unsigned long long tag;

  __device__ inline void reset() {
    lease = int(PageLease::Free);
    tag = 0ull;
  }
};

// A 64-bit content tag from a pointer and three ints: each value folded in with
// the splitmix64 finaliser (Steele, Lea, Flood 2014); never 0, which marks an
// untagged page.
__host__ __device__ inline unsigned long long page_tag_mix(unsigned long long h, unsigned long long v) {
  unsigned long long z = h + 0x9e3779b97f4a7c15ull + v;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__host__ __device__ inline unsigned long long make_page_tag(const void* ptr, int a, int b, int c) {
  unsigned long long h = page_tag_mix(0, static_cast<unsigned long long>(reinterpret_cast<std::uintptr_t>(ptr)));
  h = page_tag_mix(h, static_cast<unsigned int>(a));
  h = page_tag_mix(h, static_cast<unsigned int>(b));
  h = page_tag_mix(h, static_cast<unsigned int>(c));
  return h ? h : 1ull;
}

struct BlockRuntime {
  PipelineSlot* slots{nullptr};
  int num_slots{1};
  WarpRoles roles{};
  GlobalQueue queue{};
  Page* pages{nullptr};
  int num_pages{0};
  PageMeta* page_meta{nullptr};
  volatile int* done{nullptr};
  DependencyState* deps{nullptr};
  int tasks_processed{0};

  __device__ inline PipelineSlot& slot(int index) { return slots[index]; }
  __device__ inline const PipelineSlot& slot(int index) const { return slots[index]; }
  __device__ inline int next_slot(int current) const { return ring_advance(current); }

  __device__ inline PageHandle page_handle(int slot_idx, int page_idx) const {
    return PageHandle{slot_idx, page_idx};
  }
  __device__ inline int physical_page_index(PageHandle h) const {
    return h.slot_idx * Config::kPagesPerSlot + h.page_idx;
  }
  __device__ inline Page& page(PageHandle h) { return pages[physical_page_index(h)]; }
  __device__ inline const Page& page(PageHandle h) const { return pages[physical_page_index(h)]; }
  template <typename T>
  __device__ inline T* page_ptr(PageHandle h) {
    return page(h).template as<T>();
  }
  template <typename T>
  __device__ inline const T* page_ptr(PageHandle h) const {
    return page(h).template as<T>();
  }
  __device__ inline PageMeta& meta(PageHandle h) { return page_meta[physical_page_index(h)]; }
  __device__ inline const PageMeta& meta(PageHandle h) const { return page_meta[physical_page_index(h)]; }

#ifdef __CUDACC__
  __device__ inline bool page_try_acquire(PageHandle h) {
    return atomicCAS(&meta(h).lease, int(PageLease::Free), int(PageLease::Loader)) == int(PageLease::Free);
  }
  // The phases of an op run in order on the same warps, so an acquire that
  // cannot succeed at once never will: it takes the page instead of spinning.
  __device__ inline void page_wait_acquire(PageHandle h) {
    if (!page_try_acquire(h)) atomicExch(&meta(h).lease, int(PageLease::Loader));
  }
  __device__ inline bool page_is_ready(PageHandle h) const {
    return *reinterpret_cast<const volatile int*>(&meta(h).lease) == int(PageLease::Ready);
  }
  __device__ inline unsigned long long page_tag(PageHandle h) const {
    return *reinterpret_cast<const volatile unsigned long long*>(&meta(h).tag);
  }
  __device__ inline bool page_is_ready_with_tag(PageHandle h, unsigned long long tag) const {
    return page_is_ready(h) && page_tag(h) == tag;
  }
  __device__ inline bool page_try_begin_overwrite(PageHandle h) {
    if (atomicCAS(&meta(h).lease, int(PageLease::Free), int(PageLease::Loader)) == int(PageLease::Free)) return true;
    return atomicCAS(&meta(h).lease, int(PageLease::Ready), int(PageLease::Loader)) == int(PageLease::Ready);
  }
  __device__ inline void page_wait_begin_overwrite(PageHandle h) {
    if (!page_try_begin_overwrite(h)) atomicExch(&meta(h).lease, int(PageLease::Loader));
  }
  __device__ inline void page_publish(PageHandle h, unsigned long long tag) {
    *reinterpret_cast<volatile unsigned long long*>(&meta(h).tag) = tag;
    __threadfence_block();
    atomicExch(&meta(h).lease, int(PageLease::Ready));
  }
  __device__ inline void page_publish_no_tag_change(PageHandle h) {
    __threadfence_block();
    atomicExch(&meta(h).lease, int(PageLease::Ready));
  }
  __device__ inline void page_release(PageHandle h) {
    __threadfence_block();
    atomicExch(&meta(h).lease, int(PageLease::Free));
  }
#endif
};

}  // namespace pk
