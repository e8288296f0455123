// ref_shim.hpp -- host stand-ins for the TT device dataflow API the reference's directory
// helpers call, so those helpers compile and run on the CPU (test infrastructure only).
//
// The reference's server directory code (dram_worker_kernel.cpp inside patch 0003) addresses
// DRAM through InterleavedAddrGen / noc_async_read / noc_async_write and L1 through 32-bit
// addresses cast to pointers. Here DRAM pages are plain host memory (a "NoC address" is a host
// pointer) and L1 is a region mapped below 4 GiB so that a 32-bit L1 address is a valid pointer.
#pragma once

#include <sys/mman.h>

#include <cstddef>
#include <cstdint>
#include <cstring>

#ifndef FORCE_INLINE
#define FORCE_INLINE inline __attribute__((always_inline))
#endif
#define tt_l1_ptr

// Reference ASSERTs become counted checks so a test can require that none fired.
extern "C" unsigned long long g_ref_assert_failures;
#define ASSERT(cond)                 \
  do {                               \
    if (!(cond)) ++g_ref_assert_failures; \
  } while (0)

template <bool DRAM>
struct InterleavedAddrGen {
  uint64_t bank_base_address;  // host address of page 0
  uint32_t page_size;
  uint64_t get_noc_addr(uint32_t id, uint32_t offset = 0) const {
    return bank_base_address + static_cast<uint64_t>(id) * page_size + offset;
  }
};

inline void noc_async_read(uint64_t src_noc_addr, uint32_t dst_l1_addr, uint32_t size) {
  std::memcpy(reinterpret_cast<void *>(static_cast<uintptr_t>(dst_l1_addr)),
              reinterpret_cast<const void *>(src_noc_addr), size);
}
inline void noc_async_write(uint32_t src_l1_addr, uint64_t dst_noc_addr, uint32_t size) {
  std::memcpy(reinterpret_cast<void *>(dst_noc_addr),
              reinterpret_cast<const void *>(static_cast<uintptr_t>(src_l1_addr)), size);
}
inline void noc_async_read_barrier() {}
inline void noc_async_write_barrier() {}
inline uint64_t get_timestamp() { return 0; }

// L1 stand-in: a low mapping whose addresses fit 32 bits.
inline uint8_t *ref_l1_alloc(size_t bytes) {
  void *p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_32BIT, -1, 0);
  if (p == MAP_FAILED) return nullptr;
  return static_cast<uint8_t *>(p);
}
inline uint32_t l1_addr(const void *p) { return static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p)); }
