// kvs_chunk_meta.cpp -- see kvs_chunk_meta.hpp.
#include "kvs_chunk_meta.hpp"

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "kvs.h"

namespace kvs {

namespace {

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  set_last_error(buf);
  return code;
}

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

// Offsets of the parts, in image order: member ptrs | block bytes | region bases | tile prefix |
// block ids | blob ptr | header words.
void layout(uint32_t n_ranks, uint32_t n_members, uint32_t n_blocks, uint32_t n_header_words, ChunkMeta *m) {
  size_t off = 0;
  auto take = [&](size_t n) {
    const size_t o = off;
    off = align16(off + n);
    return o;
  };
  m->o_member_ptrs = take(8ull * n_ranks * n_members);
  m->o_member_bytes = take(8ull * n_members);
  m->o_region_bases = take(8ull * n_members);
  m->o_tile_prefix = take(8ull * n_members + 8);
  m->o_block_ids = take(8ull * n_blocks);
  m->o_blob_ptr = take(8);
  m->o_header = take(4ull * n_header_words);
  m->bytes = off;
}

}  // namespace

size_t chunk_meta_bytes(uint32_t n_ranks, uint32_t n_members, uint32_t n_blocks, uint32_t n_header_words) {
  ChunkMeta m{};
  layout(n_ranks, n_members, n_blocks, n_header_words, &m);
  return m.bytes;
}

bool bulk_engine_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("KVS_COPY_ENGINE");
    return !(v && std::strcmp(v, "ldg") == 0);
  }();
  return on;
}

int check_chunk_args(const ChunkArgs &a, const char *op, ChunkMeta *m) {
  if (a.n_ranks == 0) return fail(KVS_E_INVAL, "%s: rank_coords must not be empty", op);
  if (a.n_members == 0) return fail(KVS_E_INVAL, "%s: members must not be empty", op);
  if (a.n_blocks == 0) return fail(KVS_E_INVAL, "%s: block_ids must not be empty", op);
  if (!a.member_ptrs || !a.member_block_bytes || !a.member_extent || !a.block_ids || !a.region_bases || !a.blob ||
      (a.to_blob && a.n_header_words && !a.header_words))
    return fail(KVS_E_INVAL, "%s: null argument", op);
  const uint32_t n_header = a.to_blob ? a.n_header_words : 0;
  const uint32_t header_bytes = 4 * n_header;
  if (header_bytes % 32) return fail(KVS_E_INVAL, "%s: header must be 32-byte aligned, got %u B", op, header_bytes);
  if (header_bytes > a.blob_bytes)
    return fail(KVS_E_INVAL, "%s: %u B header exceeds the %llu B blob", op, header_bytes,
                (unsigned long long)a.blob_bytes);
  uint32_t max_block = 0;
  for (uint32_t i = 0; i < a.n_blocks; ++i) max_block = max_block > a.block_ids[i] ? max_block : a.block_ids[i];
  uint64_t tiles = 0;
  for (uint32_t mi = 0; mi < a.n_members; ++mi) {
    const uint64_t sbb = a.member_block_bytes[mi];
    if (sbb == 0 || sbb % 4)
      return fail(KVS_E_INVAL, "%s: member %u block bytes %llu must be nonzero and 4-byte aligned", op, mi,
                  (unsigned long long)sbb);
    if (a.region_bases[mi] % 32)
      return fail(KVS_E_INVAL, "%s: region base %llu must be 32-byte aligned", op,
                  (unsigned long long)a.region_bases[mi]);
    if (a.region_bases[mi] < header_bytes)
      return fail(KVS_E_INVAL, "%s: member %u's region at %llu B overlaps the %u B header", op, mi,
                  (unsigned long long)a.region_bases[mi], header_bytes);
    if (((uint64_t)max_block + 1) * sbb > a.member_extent[mi])
      return fail(KVS_E_INVAL, "%s: block %u reaches past member %u's %llu B shard", op, max_block, mi,
                  (unsigned long long)a.member_extent[mi]);
    const uint64_t end = a.region_bases[mi] + (uint64_t)a.n_blocks * sbb * a.n_ranks;
    if (end > a.blob_bytes)
      return fail(KVS_E_INVAL, "%s: member %u's region ends at %llu B, past the %llu B blob", op, mi,
                  (unsigned long long)end, (unsigned long long)a.blob_bytes);
    for (uint32_t r = 0; r < a.n_ranks; ++r)
      if (!a.member_ptrs[(uint64_t)r * a.n_members + mi])
        return fail(KVS_E_INVAL, "%s: member %u of rank %u is null", op, mi, r);
    tiles += (sbb + kChunkTileBytes - 1) / kChunkTileBytes;
  }
  cudaPointerAttributes ba{};
  if (cudaPointerGetAttributes(&ba, a.blob) != cudaSuccess || ba.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return fail(KVS_E_INVAL, "%s: blob must be device memory", op);
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != ba.device) cudaSetDevice(ba.device);
  int rc = KVS_OK;
  // members on other GPUs are read / written over NVLink: enable peer access to their devices
  for (uint64_t i = 0; i < (uint64_t)a.n_ranks * a.n_members && rc == KVS_OK; ++i) {
    cudaPointerAttributes ma{};
    if (cudaPointerGetAttributes(&ma, reinterpret_cast<const void *>(a.member_ptrs[i])) != cudaSuccess ||
        ma.type != cudaMemoryTypeDevice) {
      cudaGetLastError();
      rc = fail(KVS_E_INVAL, "%s: member tensor must be device memory", op);
    } else if (ma.device != ba.device) {
      const cudaError_t pe = cudaDeviceEnablePeerAccess(ma.device, 0);
      if (pe == cudaErrorPeerAccessAlreadyEnabled)
        cudaGetLastError();
      else if (pe != cudaSuccess)
        rc = fail(KVS_E_CUDA, "%s: enable peer access %d->%d: %s", op, ba.device, ma.device, cudaGetErrorString(pe));
    }
  }
  if (prev >= 0 && prev != ba.device) cudaSetDevice(prev);
  if (rc != KVS_OK) return rc;
  layout(a.n_ranks, a.n_members, a.n_blocks, n_header, m);
  m->tiles_per_combo = tiles;
  m->device = ba.device;
  return KVS_OK;
}

void pack_chunk_meta(const ChunkArgs &a, const ChunkMeta &m, uint8_t *image) {
  std::memset(image, 0, m.bytes);
  std::memcpy(image + m.o_member_ptrs, a.member_ptrs, 8ull * a.n_ranks * a.n_members);
  std::memcpy(image + m.o_member_bytes, a.member_block_bytes, 8ull * a.n_members);
  std::memcpy(image + m.o_region_bases, a.region_bases, 8ull * a.n_members);
  uint64_t *prefix = reinterpret_cast<uint64_t *>(image + m.o_tile_prefix);
  prefix[0] = 0;
  for (uint32_t mi = 0; mi < a.n_members; ++mi)
    prefix[mi + 1] = prefix[mi] + (a.member_block_bytes[mi] + kChunkTileBytes - 1) / kChunkTileBytes;
  int64_t *ids = reinterpret_cast<int64_t *>(image + m.o_block_ids);
  for (uint32_t i = 0; i < a.n_blocks; ++i) ids[i] = a.block_ids[i];
  const uint64_t blob_addr = reinterpret_cast<uint64_t>(a.blob);
  std::memcpy(image + m.o_blob_ptr, &blob_addr, 8);
  if (a.to_blob && a.n_header_words) std::memcpy(image + m.o_header, a.header_words, 4ull * a.n_header_words);
}

ChunkCopyParams chunk_params(const ChunkArgs &a, const ChunkMeta &m, const uint8_t *meta) {
  ChunkCopyParams p{};
  p.member_ptrs = reinterpret_cast<const uint64_t *>(meta + m.o_member_ptrs);
  p.member_bytes = reinterpret_cast<const uint64_t *>(meta + m.o_member_bytes);
  p.region_bases = reinterpret_cast<const uint64_t *>(meta + m.o_region_bases);
  p.tile_prefix = reinterpret_cast<const uint64_t *>(meta + m.o_tile_prefix);
  p.block_ids = reinterpret_cast<const int64_t *>(meta + m.o_block_ids);
  p.blob_ptrs = reinterpret_cast<const uint64_t *>(meta + m.o_blob_ptr);
  p.header_words = reinterpret_cast<const uint32_t *>(meta + m.o_header);
  p.n_header_words = a.to_blob ? a.n_header_words : 0;
  p.n_blobs = 1;
  p.blocks_per_blob = a.n_blocks;
  p.n_ranks = a.n_ranks;
  p.n_members = a.n_members;
  p.tile_bytes = kChunkTileBytes;
  p.tiles_per_combo = m.tiles_per_combo;
  p.total_tiles = (uint64_t)a.n_blocks * a.n_ranks * m.tiles_per_combo;
  p.to_blob = a.to_blob;
  uint64_t mx = 0, sum = 0;
  for (uint32_t mi = 0; mi < a.n_members; ++mi) {
    mx = a.member_block_bytes[mi] > mx ? a.member_block_bytes[mi] : mx;
    sum += a.member_block_bytes[mi];
  }
  p.max_member_bytes = mx;
  p.payload_bytes = sum * a.n_blocks * a.n_ranks;
  return p;
}

cudaError_t launch_chunk(const ChunkCopyParams &p, cudaStream_t stream) {
  if (small_copy_suits(p)) return launch_chunk_copy_small(p, stream);
  if (bulk_engine_enabled()) return launch_chunk_copy_tma(p, stream);
  return launch_chunk_copy(p, stream);
}

}  // namespace kvs
