// kvs_chunk_meta.hpp -- argument checks, packed device metadata and launch of the chunk gather /
// scatter entry points (kvs_gather_chunk, kvs_scatter_chunk, kvs_gather_chunk_noalloc).
//
// The entry points differ only in where the packed metadata lives on the device (a stream-ordered
// allocation, or the fixed array of the allocation-free gather); the checks, the image layout and
// the copy-engine choice are shared here so they cannot drift apart. The checks follow the
// reference's gather / scatter validation (patch 0003 gather.hpp lines 9335-9453).
#pragma once

#include <cstddef>
#include <cstdint>

#include "kvs_kernels.cuh"

namespace kvs {

constexpr uint32_t kChunkTileBytes = 32u << 10;  // tile of the copy engines

struct ChunkArgs {
  const uint64_t *member_ptrs;  // [n_ranks * n_members]
  uint32_t n_ranks, n_members;
  const uint64_t *member_block_bytes, *member_extent;  // [n_members]
  const uint32_t *block_ids;
  uint32_t n_blocks;
  const uint64_t *region_bases;  // [n_members]
  const uint32_t *header_words;  // gather only
  uint32_t n_header_words;
  void *blob;
  uint64_t blob_bytes;
  int to_blob;  // 1 gather, 0 scatter
};

// Where each part sits in the packed image (16-byte aligned parts), and what the checks found.
struct ChunkMeta {
  size_t o_member_ptrs, o_member_bytes, o_region_bases, o_tile_prefix, o_block_ids, o_blob_ptr, o_header;
  size_t bytes;             // image size
  uint64_t tiles_per_combo; // tiles of one (chunk block, rank) over every member
  int device;               // GPU of the blob: the launch runs there
};

// Image size for these counts (no argument needs to be valid).
size_t chunk_meta_bytes(uint32_t n_ranks, uint32_t n_members, uint32_t n_blocks, uint32_t n_header_words);

// Checks every argument before any device access except the pointer queries, enables peer access
// from the blob's GPU to every member GPU, and fills `m`. On failure sets the thread-local error
// (text prefixed by `op`) and returns a KVS_E_* code. Calls no allocating routine.
int check_chunk_args(const ChunkArgs &a, const char *op, ChunkMeta *m);

// Writes the m.bytes-byte image into `image` (host memory).
void pack_chunk_meta(const ChunkArgs &a, const ChunkMeta &m, uint8_t *image);

// Copy-engine parameters whose arrays are the image at device address `meta`.
ChunkCopyParams chunk_params(const ChunkArgs &a, const ChunkMeta &m, const uint8_t *meta);

// Launches the copy with the runtime's engine choice: the one-wave engine for copies of at most
// small_copy_limit() bytes, else the bulk engine (both sides are device memory here), or 16-byte
// loads and stores when KVS_COPY_ENGINE=ldg.
cudaError_t launch_chunk(const ChunkCopyParams &p, cudaStream_t stream);

// Engine choice shared with the store runtime.
bool bulk_engine_enabled();

}  // namespace kvs
