// kvs_noalloc.cu -- kvs_gather_chunk_noalloc: the chunk gather for callers that must not allocate.
//
// kvs_gather_chunk stages each call's metadata (member pointers, block sizes, region bases, block
// ids, header words) in a buffer it takes from the stream-ordered allocator. Some callers cannot
// allow that: a serving engine that has handed nearly all of HBM to its paged KV pool has no
// headroom for another allocation (and must not have its memory accounting disturbed), and a
// latency-critical restore path cannot afford cudaMalloc / cudaFree, which may synchronise the
// device. This entry point stages the same metadata in one fixed device array that lives in this
// file instead, so it never calls cudaMalloc, cudaMallocAsync, cudaFree or any allocating library
// routine. Every GPU that loads the library holds that array (kNoAllocScratchBytes) until exit.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "kvs.h"
#include "kvs_kernels.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = KVS_NOALLOC_SCRATCH_BYTES;
constexpr uint32_t kNoAllocTileBytes = 32u << 10;
constexpr int kMaxDevices = 64;

// Shared by every call on a device; each call overwrites the part it uses before its kernel reads
// it. Nothing in it needs to start at zero.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mu;
void *g_scratch_addr[kMaxDevices] = {};  // device address of g_noalloc_scratch, per device

thread_local uint8_t g_host_image[kNoAllocScratchBytes];  // host-side image of one call's metadata

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

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

}  // namespace

extern "C" int kvs_gather_chunk_noalloc(const uint64_t *member_ptrs, uint32_t n_ranks, uint32_t n_members,
                                        const uint64_t *member_block_bytes, const uint64_t *member_extent,
                                        const uint32_t *block_ids, uint32_t n_blocks, const uint64_t *region_bases,
                                        const uint32_t *header_words, uint32_t n_header_words, void *blob,
                                        uint64_t blob_bytes, void *stream) {
  const char *op = "kvcache gather (no-alloc)";
  if (n_ranks == 0) return fail(KVS_E_INVAL, "%s: rank_coords must not be empty", op);
  if (n_members == 0) return fail(KVS_E_INVAL, "%s: members must not be empty", op);
  if (n_blocks == 0) return fail(KVS_E_INVAL, "%s: block_ids must not be empty", op);
  if (!member_ptrs || !member_block_bytes || !member_extent || !block_ids || !region_bases || !blob ||
      (n_header_words && !header_words))
    return fail(KVS_E_INVAL, "%s: null argument", op);
  const uint64_t nrm = (uint64_t)n_ranks * n_members;
  // scratch layout: member ptrs | block bytes | region bases | tile prefix | block ids | blob ptr | header
  const size_t need = align16(8 * nrm) + 3 * align16(8ull * n_members + 8) + align16(8ull * n_blocks) + 16 +
                      align16(4ull * n_header_words);
  if (need > kNoAllocScratchBytes)
    return fail(KVS_E_INVAL,
                "%s: %u ranks x %u members, %u blocks and %u header words need %zu bytes of metadata, more than "
                "the %zu-byte scratch; use kvs_gather_chunk",
                op, n_ranks, n_members, n_blocks, n_header_words, need, kNoAllocScratchBytes);
  const uint32_t header_bytes = 4 * n_header_words;
  if (header_bytes % 32) return fail(KVS_E_INVAL, "%s: header must be 32-byte aligned, got %u B", op, header_bytes);
  if (header_bytes > blob_bytes)
    return fail(KVS_E_INVAL, "%s: %u B header exceeds the %llu B blob", op, header_bytes,
                (unsigned long long)blob_bytes);
  uint32_t max_block = 0;
  for (uint32_t i = 0; i < n_blocks; ++i) max_block = max_block > block_ids[i] ? max_block : block_ids[i];
  uint8_t *img = g_host_image;
  size_t off = 0;
  auto take = [&](size_t n) {
    const size_t o = off;
    off = align16(off + n);
    return o;
  };
  const size_t o_mp = take(8 * nrm), o_mb = take(8ull * n_members + 8), o_rb = take(8ull * n_members + 8);
  const size_t o_tp = take(8ull * n_members + 8), o_id = take(8ull * n_blocks), o_bl = take(8);
  const size_t o_hw = take(4ull * n_header_words);
  uint64_t *tile_prefix = reinterpret_cast<uint64_t *>(img + o_tp);
  tile_prefix[0] = 0;
  for (uint32_t m = 0; m < n_members; ++m) {
    const uint64_t sbb = member_block_bytes[m];
    if (sbb == 0 || sbb % 4)
      return fail(KVS_E_INVAL, "%s: member %u block bytes %llu must be nonzero and 4-byte aligned", op, m,
                  (unsigned long long)sbb);
    if (region_bases[m] % 32)
      return fail(KVS_E_INVAL, "%s: region base %llu must be 32-byte aligned", op, (unsigned long long)region_bases[m]);
    if (region_bases[m] < header_bytes)
      return fail(KVS_E_INVAL, "%s: member %u's region at %llu B overlaps the %u B header", op, m,
                  (unsigned long long)region_bases[m], header_bytes);
    if (((uint64_t)max_block + 1) * sbb > member_extent[m])
      return fail(KVS_E_INVAL, "%s: block %u reaches past member %u's %llu B shard", op, max_block, m,
                  (unsigned long long)member_extent[m]);
    const uint64_t end = region_bases[m] + (uint64_t)n_blocks * sbb * n_ranks;
    if (end > blob_bytes)
      return fail(KVS_E_INVAL, "%s: member %u's region ends at %llu B, past the %llu B blob", op, m,
                  (unsigned long long)end, (unsigned long long)blob_bytes);
    tile_prefix[m + 1] = tile_prefix[m] + (sbb + kNoAllocTileBytes - 1) / kNoAllocTileBytes;
  }
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, blob) != cudaSuccess || a.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return fail(KVS_E_INVAL, "%s: blob must be device memory", op);
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != a.device) cudaSetDevice(a.device);
  int rc = KVS_OK;
  do {
    for (uint64_t i = 0; i < nrm && rc == KVS_OK; ++i) {
      cudaPointerAttributes ma{};
      if (!member_ptrs[i] || cudaPointerGetAttributes(&ma, reinterpret_cast<const void *>(member_ptrs[i])) != cudaSuccess ||
          ma.type != cudaMemoryTypeDevice) {
        cudaGetLastError();
        rc = fail(KVS_E_INVAL, "%s: member tensor must be device memory", op);
      } else if (ma.device != a.device) {
        const cudaError_t pe = cudaDeviceEnablePeerAccess(ma.device, 0);
        if (pe == cudaErrorPeerAccessAlreadyEnabled)
          cudaGetLastError();
        else if (pe != cudaSuccess)
          rc = fail(KVS_E_CUDA, "%s: enable peer access %d->%d: %s", op, a.device, ma.device, cudaGetErrorString(pe));
      }
    }
    if (rc != KVS_OK) break;
    uint8_t *scratch = nullptr;
    if ((rc = scratch_address(a.device, &scratch)) != KVS_OK) break;
    std::memcpy(img + o_mp, member_ptrs, 8 * nrm);
    std::memcpy(img + o_mb, member_block_bytes, 8ull * n_members);
    std::memcpy(img + o_rb, region_bases, 8ull * n_members);
    int64_t *ids = reinterpret_cast<int64_t *>(img + o_id);
    for (uint32_t i = 0; i < n_blocks; ++i) ids[i] = block_ids[i];
    const uint64_t blob_addr = reinterpret_cast<uint64_t>(blob);
    std::memcpy(img + o_bl, &blob_addr, 8);
    if (n_header_words) std::memcpy(img + o_hw, header_words, 4ull * n_header_words);
    cudaStream_t s = (cudaStream_t)stream;
    // a copy from pageable host memory returns once the image has been staged, so the host image
    // can be reused by the next call
    cudaError_t e = cudaMemcpyAsync(scratch, img, off, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
      rc = fail(KVS_E_CUDA, "%s: metadata upload: %s", op, cudaGetErrorString(e));
      break;
    }
    kvs::ChunkCopyParams p{};
    p.member_ptrs = reinterpret_cast<const uint64_t *>(scratch + o_mp);
    p.member_bytes = reinterpret_cast<const uint64_t *>(scratch + o_mb);
    p.region_bases = reinterpret_cast<const uint64_t *>(scratch + o_rb);
    p.tile_prefix = reinterpret_cast<const uint64_t *>(scratch + o_tp);
    p.block_ids = reinterpret_cast<const int64_t *>(scratch + o_id);
    p.blob_ptrs = reinterpret_cast<const uint64_t *>(scratch + o_bl);
    p.header_words = reinterpret_cast<const uint32_t *>(scratch + o_hw);
    p.n_header_words = n_header_words;
    p.n_blobs = 1;
    p.blocks_per_blob = n_blocks;
    p.n_ranks = n_ranks;
    p.n_members = n_members;
    p.tile_bytes = kNoAllocTileBytes;
    p.tiles_per_combo = tile_prefix[n_members];
    p.total_tiles = (uint64_t)n_blocks * n_ranks * p.tiles_per_combo;
    p.to_blob = 1;
    e = kvs::launch_chunk_copy_tma(p, s);
    if (e != cudaSuccess) rc = fail(KVS_E_CUDA, "%s: launch: %s", op, cudaGetErrorString(e));
  } while (false);
  if (prev >= 0 && prev != a.device) cudaSetDevice(prev);
  return rc;
}
