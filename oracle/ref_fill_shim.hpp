// ref_fill_shim.hpp -- host stand-ins for the TT dataflow API used by the reference's
// moreh_paged_fill_cache_varlen reader and writer kernels (patch 0002), so the two kernels
// compile and run on the CPU as the parity pin of the paged-fill restatement (test
// infrastructure only).
//
// * DRAM buffers and L1 live in mappings below 4 GiB, so the kernels' 32-bit buffer and L1
//   addresses are valid host pointers; a "NoC address" is a host address.
// * A tensor accessor addresses page `id` at base + id * page_size (interleaving across banks does
//   not change which bytes a page holds).
// * Circular buffers are linear regions large enough for everything one kernel pushes: the reader
//   runs to completion, then the writer consumes what it pushed (same order as on the device).
// * Named compile-time arguments are looked up at run time; the kernel sources are compiled with
//   `constexpr` defined away, so they read those values like any other constant.
#pragma once

#include <sys/mman.h>

#include <cstddef>
#include <cstdint>
#include <cstring>

#define tt_l1_ptr
#ifndef FORCE_INLINE
#define FORCE_INLINE inline __attribute__((always_inline))
#endif

namespace fillshim {

struct Named {
  const char *name;
  uint32_t value;
};

struct Cb {
  uint8_t *base = nullptr;
  uint32_t page = 0;
  uint64_t wr = 0, rd = 0;  // pages pushed / popped
};

struct State {
  const Named *named = nullptr;
  uint32_t n_named = 0;
  const uint32_t *args = nullptr;
  Cb cb[8];
  uint32_t tile_bytes = 0;
  uint64_t missing_named = 0;
};

inline State &st() {
  static State s;
  return s;
}

inline uint8_t *low_alloc(size_t bytes) {
  void *p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_32BIT, -1, 0);
  return p == MAP_FAILED ? nullptr : static_cast<uint8_t *>(p);
}
inline void low_free(void *p, size_t bytes) {
  if (p) munmap(p, bytes);
}
inline uint32_t addr32(const void *p) { return static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p)); }

}  // namespace fillshim

inline uint32_t rt_named_arg(const char *name) {
  auto &s = fillshim::st();
  for (uint32_t i = 0; i < s.n_named; ++i)
    if (std::strcmp(s.named[i].name, name) == 0) return s.named[i].value;
  ++s.missing_named;
  return 0;
}
#define get_named_compile_time_arg_val(name) rt_named_arg(name)

template <uint32_t N>
struct TensorAccessorArgs {
  static constexpr uint32_t next_compile_time_args_offset() { return N + 1; }
};

struct TensorAccessor {
  uint64_t base;
  uint32_t page_size;
  template <class A>
  TensorAccessor(const A &, uint32_t address, uint32_t page) : base(address), page_size(page) {}
  uint64_t get_noc_addr(uint32_t id, uint32_t offset = 0) const {
    return base + static_cast<uint64_t>(id) * page_size + offset;
  }
};

template <class T>
inline T get_arg_val(uint32_t idx) {
  return static_cast<T>(fillshim::st().args[idx]);
}

inline uint32_t get_tile_size(uint32_t) { return fillshim::st().tile_bytes; }

inline void noc_async_read(uint64_t src, uint32_t dst_l1, uint32_t size) {
  std::memcpy(reinterpret_cast<void *>(static_cast<uintptr_t>(dst_l1)), reinterpret_cast<const void *>(src), size);
}
inline void noc_async_read_tile(uint32_t id, const TensorAccessor &a, uint32_t dst_l1) {
  noc_async_read(a.get_noc_addr(id), dst_l1, a.page_size);
}
inline void noc_async_write_tile(uint32_t id, const TensorAccessor &a, uint32_t src_l1) {
  std::memcpy(reinterpret_cast<void *>(a.get_noc_addr(id)), reinterpret_cast<const void *>(static_cast<uintptr_t>(src_l1)),
              a.page_size);
}
inline void noc_async_read_barrier() {}
inline void noc_async_write_barrier() {}

inline void cb_reserve_back(uint32_t, uint32_t) {}
inline void cb_wait_front(uint32_t, uint32_t) {}
inline uint32_t get_write_ptr(uint32_t cb) {
  auto &c = fillshim::st().cb[cb];
  return fillshim::addr32(c.base + c.wr * c.page);
}
inline uint32_t get_read_ptr(uint32_t cb) {
  auto &c = fillshim::st().cb[cb];
  return fillshim::addr32(c.base + c.rd * c.page);
}
inline void cb_push_back(uint32_t cb, uint32_t n) { fillshim::st().cb[cb].wr += n; }
inline void cb_pop_front(uint32_t cb, uint32_t n) { fillshim::st().cb[cb].rd += n; }
