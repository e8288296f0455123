// kvs_kernels.cuh -- device-side data structures and kernel launchers of the B200 KV block store.
//
// Four kernel families move every byte and answer every device-side lookup:
//   * chunk_copy: the paged-block gather (put) / scatter (get) engines. They move whole member
//     blocks between paged KV tensors and packed blobs (device slab values or caller blobs),
//     16-byte vectorised and coalesced: a one-wave grid with one CTA per 16 KiB piece for copies
//     up to 512 MiB, a persistent grid of one CTA per SM streaming 32 KiB tiles through a bulk-copy
//     ring for larger ones, and 16-byte loads and stores when a side is host memory.
//     It restates the byte layout of gather_tp_shards_to_chip / scatter_chunk_from_chip
//     (patch 0003 gather.hpp lines 9372-9453) for one GPU or for peer GPUs over NVLink.
//   * index_lookup: a warp-cooperative probe of the shard's device replica of the FNV-1a
//     open-addressed index (patch 0003 lines 9923-9963): 32 buckets per probe step, ballot
//     for empty / hash-matching lanes, and a 32-lane key compare against the directory row.
//   * apply_mutations: brings the device index replica up to date with the host directory
//     (bucket words, entry metadata, key rows) in stream order before any lookup reads it.
//   * paged_fill: token-granular fill of packed K/V rows of several requests into a paged cache
//     through page tables (moreh_paged_fill_cache_varlen, patch 0002 lines 106-421).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace kvs {

constexpr uint32_t kBucketEmpty = 0xFFFFFFFFu;      // reference kBucketDirSlotEmpty
constexpr uint32_t kBucketTombstone = 0xFFFFFFFEu;  // reference kBucketDirSlotTombstone
constexpr uint32_t kMaxKeyBytes = 128;              // reference kMaxPutKeyBytes
constexpr uint32_t kKeyRowWords = kMaxKeyBytes / 4; // 32 words = one per lane

// Device replica of one directory entry (16 bytes). location: 0 device, 1 host, 2 pending.
struct alignas(16) DevMeta {
  uint64_t value_off;
  uint32_t total_len;
  uint8_t valid;
  uint8_t location;
  uint8_t key_len;
  uint8_t pad;
};
static_assert(sizeof(DevMeta) == 16, "DevMeta is one 16-byte word");

// Lookup result per key (written by index_lookup).
enum LookupStatus : uint32_t {
  kMiss = 0,
  kHitDevice = 1,   // device-resident (or pending, which is device-readable)
  kHitHost = 2,     // host-only: the host tier serves it
  kLenMismatch = 3, // hit, but the stored value length differs from the expected block value
};

struct LookupOut {
  uint64_t value_off;
  uint32_t value_len;
  uint32_t status;
  uint32_t slot;
  uint32_t pad;
};

// Small calls carry their keys and block ids in the kernel parameters instead of an uploaded
// array (no host-to-device copy before the launch).
constexpr uint32_t kInlineKeys = 8;

// Parameters of one chunk_copy launch. All arrays are device-accessible.
struct ChunkCopyParams {
  const uint64_t *member_ptrs;   // [n_sets * n_ranks * n_members]
  const uint32_t *blob_sets;     // optional [n_blobs]: member set of each blob (nullptr: set 0)
  const uint64_t *member_bytes;  // [n_members] bytes of one block of the member
  const uint64_t *region_bases;  // [n_members] member region offset inside a blob
  const uint64_t *tile_prefix;   // [n_members + 1] tiles per member, prefix summed
  const int64_t *block_ids;      // [n_blobs * blocks_per_blob]; nullptr: inline_ids
  const uint64_t *blob_ptrs;     // [n_blobs] blob base addresses; 0 skips the blob; nullptr: inline_blobs
  const uint32_t *header_words;  // [n_header_words] (gather only)
  uint32_t n_header_words;
  uint32_t n_blobs;
  uint32_t blocks_per_blob;
  uint32_t n_ranks;
  uint32_t n_members;
  uint32_t tile_bytes;
  uint64_t tiles_per_combo;  // tile_prefix[n_members]
  uint64_t total_tiles;
  int to_blob;               // 1: members -> blob (gather), 0: blob -> members (scatter)
  unsigned int *timeout_flag;  // optional host-mapped word set to 1 if a bounded wait expires
  uint32_t wait_polls;       // polls of one bounded wait on a tile load (set by the launcher)
  int64_t inline_ids[kInlineKeys];  // block ids when block_ids is nullptr (n_blobs * blocks_per_blob <= 8)
  uint64_t inline_blobs[kInlineKeys];  // blob addresses when blob_ptrs is nullptr (n_blobs <= 8)
  // Host-side facts for the engine choice (no kernel reads them; 0 = not given, which keeps the
  // persistent engines): the largest member block in bytes, and the bytes the launch moves.
  uint64_t max_member_bytes;
  uint64_t payload_bytes;
};

struct LookupParams {
  const uint8_t *keys;      // n keys, `key_stride` bytes apart; nullptr: inline_keys (8-byte keys)
  const uint32_t *key_lens; // nullptr: every key is key_stride bytes
  uint32_t key_stride;
  uint32_t n;
  const uint64_t *buckets;  // (slot << 32) | hash
  uint32_t bucket_mask;
  const DevMeta *meta;
  const uint32_t *key_rows; // [max_keys][kKeyRowWords]
  uint32_t max_keys;
  uint64_t slab_base;       // device address of the slab
  uint64_t expected_len;    // 0: any length
  LookupOut *out;
  uint64_t *blob_ptrs;      // optional: slab_base + off for device hits, else 0
  uint64_t inline_keys[kInlineKeys];  // the keys when `keys` is nullptr (n <= 8, key_stride 8)
};

struct MutationParams {
  const uint64_t *bucket_writes;  // pairs {bucket index, bucket word}
  uint32_t n_bucket_writes;
  const uint64_t *meta_writes;    // triples {slot, meta word 0, meta word 1}
  uint32_t n_meta_writes;
  const uint32_t *key_writes;     // rows of {slot, kKeyRowWords words}
  uint32_t n_key_writes;
  uint64_t *buckets;
  DevMeta *meta;
  uint32_t *key_rows;
};

// Token-granular paged KV fill (moreh_paged_fill_cache_varlen): packed K/V rows of several
// requests into their paged cache blocks through page tables. All arrays are device memory.
// One launch fills up to kMaxFillLayers layers that share the requests and page tables; the
// layer's tensors come from FillLayers (k_fill etc. below are set per layer inside the kernels).
struct PagedFillParams {
  const uint8_t *k_fill, *v_fill;    // [n_heads][total_tokens][row_bytes]
  uint8_t *cache_k, *cache_v;        // [num_blocks][n_heads][block_size][row_bytes]
  const int32_t *cu_seqlens;         // [batch + 1], -1 padded
  const int32_t *page_table;         // [batch][max_blocks]
  const int32_t *start_positions;    // [batch]
  uint32_t n_heads, total_tokens, row_bytes, batch, max_blocks, num_blocks, block_size;
  unsigned int *out_of_range;        // optional: tokens skipped for a position or block out of range
                                     // (counted once per token, in the first layer)
  // Optional source of rows per request instead of the packed k_fill / v_fill: request r's value
  // (a raw-byte chunk blob) holds, for layer l, its K rows at req_src[r] + 2 l req_alloc[r] and its
  // V rows req_alloc[r] further on, one row_bytes row per token (one head: n_heads must be 1, and
  // row_bytes and the caches 16-byte aligned). req_src[r] already points past the value's header.
  // A launch covers layers layer0 .. layer0 + n_layers - 1 (its z index adds to layer0).
  const uint64_t *req_src;           // [batch] device addresses, or nullptr
  const uint64_t *req_alloc;         // [batch] bytes of one K (or V) region of the request's value
  uint32_t layer0;
};

constexpr uint32_t kMaxFillLayers = 64;
struct FillLayers {  // by value in the kernel parameters (2 KiB)
  const uint8_t *k_fill[kMaxFillLayers], *v_fill[kMaxFillLayers];
  uint8_t *cache_k[kMaxFillLayers], *cache_v[kMaxFillLayers];
};

// Launch helpers (return cudaError_t of the launch). `grid_ctas` = 0 picks the default
// persistent grid (SM count x resident CTAs per SM).
cudaError_t launch_chunk_copy(const ChunkCopyParams &p, cudaStream_t stream, int grid_ctas = 0);
// TMA bulk-copy variant (sources and destinations in device memory, this GPU's or a peer's).
cudaError_t launch_chunk_copy_tma(const ChunkCopyParams &p, cudaStream_t stream);
// One-wave variant for small copies: one CTA per 16 KiB of each (blob block, rank, member), every
// thread's loads issued before its stores, no tile walk. Needs p.max_member_bytes.
cudaError_t launch_chunk_copy_small(const ChunkCopyParams &p, cudaStream_t stream);
// Whether a copy goes to the one-wave variant: its facts are given, and either every member
// block is one 16 KiB piece or it moves at most small_copy_limit() bytes with a small grid. small_copy_limit() is 512 MiB unless
// KVS_SMALL_COPY_BYTES sets it (0 turns the variant off); set_small_copy_limit overrides both.
bool small_copy_suits(const ChunkCopyParams &p);
uint64_t small_copy_limit();
void set_small_copy_limit(uint64_t bytes);
// Counters of the bulk-copy engine on the current device (both 0 in normal operation): bounded
// waits on a tile load that expired, and CTAs that exited while one of their loads still had not
// landed after the full wait limit (the engine cannot be trusted after that).
cudaError_t read_tma_counters(unsigned int *expired, unsigned int *unsafe);
// Polls of the bulk-copy engine's bounded wait on each tile load for launches from now on (0
// expires every wait at once; a test of the expiry path uses it). default_copy_wait_polls() is
// the production limit.
void set_copy_wait_polls(uint32_t polls);
uint32_t default_copy_wait_polls();
cudaError_t launch_index_lookup(const LookupParams &p, cudaStream_t stream);
cudaError_t launch_apply_mutations(const MutationParams &p, cudaStream_t stream);
cudaError_t launch_paged_fill(const PagedFillParams &p, const FillLayers &layers, uint32_t n_layers,
                              cudaStream_t stream);
cudaError_t launch_echo(const uint8_t *in, uint8_t *out, uint32_t n, cudaStream_t stream);

// Request records of one hash-sharded step, bucketed on the GPU. Keys 0 .. n_get - 1 are gets,
// n_get .. n - 1 puts. Each key's owner is slot_shard[fnv1a32(key) % kPlacementSlots] (or
// fnv1a32(key) % world without a table). Record o (request_record_words(cap) int64 words) holds
// {gets, puts, op, 0}, then cap get keys, cap get block ids, cap put keys, cap put block ids, in
// batch order within each kind; unused words are zero. back[(o * 2 + kind) * cap + j] is the batch
// position (within its kind) of the j-th key of that kind in record o, counts[kind * world + o] the
// number of keys. *overflow is 0 after the launch, or 1 if a group had more than cap keys (it keeps
// its first cap keys).
constexpr uint32_t kPlacementSlots = 4096;
__host__ __device__ inline uint64_t request_record_words(uint32_t cap) { return 4 + 4ull * cap; }
struct BucketParams {
  const uint64_t *keys;
  const int64_t *ids;
  uint32_t n, n_get, world, cap;
  const int32_t *slot_shard;  // [kPlacementSlots] or nullptr
  int64_t op;
  int64_t *records;           // [world][request_record_words(cap)]
  int32_t *back;              // [world][2][cap]
  int32_t *counts;            // [2][world]
  uint32_t *overflow;         // one word
};
cudaError_t launch_bucket_requests(const BucketParams &p, cudaStream_t stream);

// Host-side FNV-1a 32 (the same function the device probe computes).
inline uint32_t fnv1a32(const uint8_t *key, uint32_t len) {
  uint32_t h = 2166136261u;
  for (uint32_t i = 0; i < len; ++i) {
    h ^= key[i];
    h *= 16777619u;
  }
  return h;
}

uint64_t kernel_launches();

// Sets the thread-local message kvs_last_error() returns (defined with the C ABI).
void set_last_error(const char *message);

}  // namespace kvs
