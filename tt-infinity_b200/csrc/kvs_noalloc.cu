// kvs_noalloc.cu -- kvs_gather_chunk_noalloc: the chunk gather for callers that must not allocate.
//
// kvs_gather_chunk stages each call's metadata (member pointers, block sizes, region bases, block
// ids, header words) in a buffer it takes from the stream-ordered allocator. Some callers cannot
// allow that: a serving engine that has handed nearly all of HBM to its paged KV pool has no
// headroom for another allocation (and must not have its memory accounting disturbed), and a
// latency-critical restore path cannot afford cudaMalloc / cudaFree, which may synchronise the
// device. This entry point keeps the same metadata in one fixed device array that lives in this
// file instead, so it never calls cudaMalloc, cudaMallocAsync, cudaFree or any allocating library
// routine. Every GPU that loads the library holds that array (kNoAllocScratchBytes) until exit.
//
// The metadata reaches the array without any host-to-device memory copy: it travels by value in
// the parameters of small staging kernels (up to kParamChunkBytes per launch), which write it into
// the array in stream order ahead of the copy kernel. Kernel parameters are captured when the
// launch is queued, so the host-side image is free for the next call as soon as this call returns,
// and the calling thread never waits for earlier work on the stream.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "kvs.h"
#include "kvs_chunk_meta.hpp"
#include "kvs_kernels.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = KVS_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// Shared by every call on a device; each call overwrites the part it uses before its kernel reads
// it. Nothing in it needs to start at zero.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// One staging launch carries this many metadata bytes in its parameters (kernel parameters may
// take up to 32764 bytes).
constexpr uint32_t kParamChunkBytes = 30u << 10;
struct alignas(16) StageChunk {
  uint32_t offset;  // destination offset inside the scratch array (16-byte aligned)
  uint32_t bytes;   // multiple of 16
  uint32_t pad[2];
  uint8_t data[kParamChunkBytes];
};
static_assert(sizeof(StageChunk) <= 32764, "staging parameters exceed the kernel parameter limit");

__global__ void stage_meta_kernel(const __grid_constant__ StageChunk c) {
  const uint4 *src = reinterpret_cast<const uint4 *>(c.data);
  uint4 *dst = reinterpret_cast<uint4 *>(g_noalloc_scratch + c.offset);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < c.bytes / 16; i += gridDim.x * blockDim.x)
    dst[i] = src[i];
}

std::mutex g_setup_mu;
void *g_scratch_addr[kMaxDevices] = {};  // device address of g_noalloc_scratch, per device

// Host-side buffers of one call (static, so a call allocates nothing on the host either); a call
// holds g_image_mu while it packs them and queues its launches, which capture their parameters.
std::mutex g_image_mu;
uint8_t g_host_image[kNoAllocScratchBytes];  // one call's metadata, packed on the host
StageChunk g_chunk;                          // parameters of one staging launch

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  kvs::set_last_error(buf);  // reported by kvs_last_error()
  return code;
}

// Device address of the scratch array on `device` (the current device). The first call on a
// device looks it up once; `g_noalloc_scratch` itself is only a host-side stand-in.
int scratch_address(int device, uint8_t **out) {
  if (device < 0 || device >= kMaxDevices) return fail(KVS_E_INVAL, "device %d out of range", device);
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_addr[device]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(KVS_E_CUDA, "kvs_gather_chunk_noalloc: scratch set-up on device %d failed: %s", device,
                  cudaGetErrorString(e));
    g_scratch_addr[device] = p;
  }
  *out = static_cast<uint8_t *>(g_scratch_addr[device]);
  return KVS_OK;
}

// Writes image[0, bytes) into the scratch array in stream order, kParamChunkBytes per launch.
cudaError_t stage_image(const uint8_t *image, size_t bytes, cudaStream_t stream) {
  for (size_t off = 0; off < bytes; off += kParamChunkBytes) {
    const uint32_t n = (uint32_t)(bytes - off < kParamChunkBytes ? bytes - off : kParamChunkBytes);
    g_chunk.offset = (uint32_t)off;
    g_chunk.bytes = n;
    std::memcpy(g_chunk.data, image + off, n);
    const uint32_t words = n / 16;
    const uint32_t grid = words / 256 + 1 < 8 ? words / 256 + 1 : 8;
    stage_meta_kernel<<<grid, 256, 0, stream>>>(g_chunk);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

extern "C" int kvs_gather_chunk_noalloc(const uint64_t *member_ptrs, uint32_t n_ranks, uint32_t n_members,
                                        const uint64_t *member_block_bytes, const uint64_t *member_extent,
                                        const uint32_t *block_ids, uint32_t n_blocks, const uint64_t *region_bases,
                                        const uint32_t *header_words, uint32_t n_header_words, void *blob,
                                        uint64_t blob_bytes, void *stream) {
  const char *op = "kvcache gather (no-alloc)";
  const size_t need = kvs::chunk_meta_bytes(n_ranks, n_members, n_blocks, n_header_words);
  if (need > kNoAllocScratchBytes)
    return fail(KVS_E_INVAL,
                "%s: %u ranks x %u members, %u blocks and %u header words need %zu bytes of metadata, more than "
                "the %zu-byte scratch; use kvs_gather_chunk",
                op, n_ranks, n_members, n_blocks, n_header_words, need, kNoAllocScratchBytes);
  const kvs::ChunkArgs a{member_ptrs, n_ranks,      n_members,    member_block_bytes, member_extent, block_ids,
                         n_blocks,    region_bases, header_words, n_header_words,     blob,          blob_bytes,
                         1};
  kvs::ChunkMeta m{};
  int rc = kvs::check_chunk_args(a, op, &m);
  if (rc != KVS_OK) return rc;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != m.device) cudaSetDevice(m.device);
  do {
    uint8_t *scratch = nullptr;
    if ((rc = scratch_address(m.device, &scratch)) != KVS_OK) break;
    std::lock_guard<std::mutex> lk(g_image_mu);
    kvs::pack_chunk_meta(a, m, g_host_image);
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = stage_image(g_host_image, m.bytes, s);
    if (e != cudaSuccess) {
      rc = fail(KVS_E_CUDA, "%s: metadata staging: %s", op, cudaGetErrorString(e));
      break;
    }
    e = kvs::launch_chunk(kvs::chunk_params(a, m, scratch), s);
    if (e != cudaSuccess) rc = fail(KVS_E_CUDA, "%s: launch: %s", op, cudaGetErrorString(e));
  } while (false);
  if (prev >= 0 && prev != m.device) cudaSetDevice(prev);
  return rc;
}
