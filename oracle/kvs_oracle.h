/*
 * kvs_oracle.h -- CPU restatement of the kvcache_manager hot path (TEST INFRASTRUCTURE).
 *
 * This is the parity oracle for the B200 KV block store. It restates, in plain C, the
 * reference algorithms the GPU path must reproduce byte for byte:
 *
 *   - the chunked blob header and the paged-block gather/scatter byte layout
 *       (gather_tp_shards_to_chip / pack_local_shards, patch 0003 gather.hpp lines 9335-9453;
 *        RawByteCodec.device_chunk_plan, patch 0005 lines 12258-12310),
 *   - the raw-byte run planner and host gather/scatter
 *       (build_tp_interleaved_region_raw_mesh_runs, patch 0002 lines 1382-1410, 1545-1660),
 *   - the server directory: FNV-1a open-addressed index with backward-shift delete,
 *       buddy value heap, exact residency LRU, catalog LRU replacement, pending entries pinned
 *       until host write-through (patch 0003 lines 9912-10543, 11440-11700),
 *   - the authoritative host tier with a first-fit coalescing pool
 *       (src/native/ttnn/server_runtime/server_storage.cpp:66-116),
 *   - the put / get / exists / remove / move / flush contract (patch 0003 design.md
 *       sections 5-7, lines 7527-7683).
 *
 * Only tests/, the smoke check and bench.py's CPU-baseline leg may call into this library.
 * The product (tt-infinity_b200/) never links or loads it.
 *
 * Parity pins: the gather/scatter byte layout and blob header are pinned against golden
 * vectors produced by the reference's own Python test helpers (tests/golden/); the run
 * planner and the directory building blocks (hash index, buddy heap, residency LRU) are pinned
 * against the reference sources compiled here by oracle/build_ref.py into oracle/_ref/.
 */
#ifndef KVS_ORACLE_H
#define KVS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- constants restated from the reference wire/layout headers (patch 0003) ---- */
#define KVO_BLOB_MAGIC 0x524B564Eu        /* patch 0005:12023 RawByteCodec._MAGIC */
#define KVO_HEADER_ALIGN 32u              /* patch 0005:12240 HEADER_ALIGN */
#define KVO_UNIT_BYTES_DEFAULT 4288u      /* patch 0003:7100 kMaxChunkValueBytes */
#define KVO_MAX_KEY_BYTES 128u            /* patch 0003:6906 kMaxPutKeyBytes */
#define KVO_MAX_VALUE_BYTES_DEFAULT (64ull << 20) /* patch 0003:7109 */
#define KVO_BUCKET_EMPTY 0xFFFFFFFFu      /* patch 0003 layout.hpp kBucketDirSlotEmpty */
#define KVO_BUCKET_TOMBSTONE 0xFFFFFFFEu  /* patch 0003 layout.hpp kBucketDirSlotTombstone */
#define KVO_NONE 0xFFFFFFFFu              /* free-list / LRU terminator */
#define KVO_HEAP_FREE 0xFFFFFFFEu         /* kHeapBlockFree */
#define KVO_HEAP_CONT 0xFFFFFFFDu         /* kHeapBlockContinuation */
#define KVO_MAX_ORDERS 32u                /* kHeapAllocatorMaxOrders */

/* directory entry locations, patch 0003:6365-6367 */
#define KVO_LOC_DEVICE 0u
#define KVO_LOC_HOST 1u
#define KVO_LOC_PENDING 2u
#define KVO_ABSENT (-1)

/* return codes shared with the product's C ABI (include/kvs.h) */
#define KVO_OK 0
#define KVO_E_INVAL (-1)
#define KVO_E_NOSPACE (-3)
#define KVO_E_TOO_SMALL (-5)

const char *kvo_last_error(void);

/* ---- small arithmetic helpers ---- */
uint32_t kvo_fnv1a32(const uint8_t *key, uint32_t len);
uint32_t kvo_next_pow2(uint32_t x);
uint32_t kvo_hash_num_buckets(uint32_t max_keys);
uint32_t kvo_buddy_order_for_units(uint32_t units);
uint32_t kvo_floor_log2(uint32_t v);
uint64_t kvo_chunk_count(uint64_t bytes, uint32_t unit_bytes);

/* ---- blob header (patch 0005:12286-12296; gather test _gathered_plan) ----
 * words = [MAGIC, count, sizes[0..count)] zero padded to a 32-byte multiple.
 * Returns the word count written, or 0 if `cap` is too small. */
uint32_t kvo_header_words(uint32_t count, const uint32_t *sizes, uint32_t *out, uint32_t cap);

/* Standard chunk plan: n_layers layers, each contributing a K and a V member of
 * alloc = n_blocks * block_bytes bytes. Fills header words, region bases (2*n_layers
 * entries) and returns value_len. Restates RawByteCodec.device_chunk_plan. */
uint64_t kvo_chunk_plan(uint32_t n_layers, uint64_t alloc, uint32_t *words, uint32_t *n_words,
                        uint32_t words_cap, uint64_t *region_bases);

/* ---- gather / scatter (a4/a5) ----
 * members[r * n_members + m] is rank r's shard of member m. For member m, chunk block cb and
 * rank r, the member_bytes[m] bytes at block_ids[cb] * member_bytes[m] of members[r][m] land at
 * dst + region_bases[m] + cb * member_bytes[m] * n_ranks + r * member_bytes[m].
 * header_words (n_header_words) are written verbatim at dst. member_extent[m] bounds the
 * member buffers, dst_bytes bounds dst. Returns KVO_OK or KVO_E_INVAL (message via
 * kvo_last_error) without touching memory on error. */
int kvo_gather(const uint8_t *const *members, uint32_t n_ranks, uint32_t n_members,
               const uint64_t *member_bytes, const uint64_t *member_extent,
               const uint32_t *block_ids, uint32_t n_blocks, const uint64_t *region_bases,
               const uint32_t *header_words, uint32_t n_header_words, uint8_t *dst,
               uint64_t dst_bytes);
int kvo_scatter(const uint8_t *src, uint64_t src_bytes, uint8_t *const *members, uint32_t n_ranks,
                uint32_t n_members, const uint64_t *member_bytes, const uint64_t *member_extent,
                const uint32_t *block_ids, uint32_t n_blocks, const uint64_t *region_bases);

/* ---- chunk slot decode (a1): RawByteCodec._chunk_slots, patch 0005:12148-12168 ----
 * Returns KVO_OK and the first block / block count, or KVO_E_INVAL. */
int kvo_chunk_slots(const int64_t *slots, uint64_t n, uint32_t block_size, uint64_t *first_block,
                    uint64_t *n_blocks);

/* ---- raw run planner (a2), patch 0002:1382-1410, 1545-1660 ---- */
typedef struct {
  uint32_t shard_index;
  uint32_t device_byte_offset;
  uint32_t num_bytes;
  uint64_t host_byte_offset;
} kvo_run;

/* runs_out is n_members arrays laid out back to back with stride runs_cap; counts_out[m] gets
 * the run count of member m. Returns KVO_OK, or KVO_E_INVAL when the reference planner would
 * return nullopt, or KVO_E_NOSPACE if runs_cap is too small. */
int kvo_plan_tp_interleaved_runs(const int64_t *slots, uint64_t n_slots, const int64_t *starts,
                                 const int64_t *ends, const int64_t *memobj_slots,
                                 uint64_t n_chunks, const int64_t *member_alloc_bytes,
                                 const int64_t *region_bases, uint64_t n_members,
                                 int64_t shard_block_bytes, int64_t block_bytes, int64_t block_size,
                                 int64_t dp_size, int64_t blocks_per_dp, int64_t tp_size,
                                 kvo_run *runs_out, uint64_t runs_cap, uint64_t *counts_out);

/* Executes runs against shards (shard_ptrs[member * n_shards + shard_index]) and a host blob.
 * to_host=1 gathers shard -> host, to_host=0 scatters host -> shard. */
void kvo_apply_runs(const kvo_run *runs, uint64_t n_runs, uint8_t *const *shard_ptrs,
                    uint8_t *host, int to_host);

/* ---- the store (a7-a15) ---- */
typedef struct kvo_store kvo_store;

typedef struct {
  uint32_t max_keys;
  uint32_t unit_bytes;      /* value-heap unit U */
  uint64_t heap_bytes;      /* device value heap (the slab) */
  uint32_t max_key_bytes;   /* <= 128 */
  uint64_t max_value_bytes;
  uint64_t host_pool_bytes; /* first-fit pool; values that do not fit use a heap copy */
} kvo_config;

typedef struct {
  uint64_t live_device_bytes;
  uint64_t pending_device_bytes;
  uint64_t live_keys;
  uint64_t device_resident_keys;
  uint64_t allocation_calls;
  uint64_t allocation_successes;
  uint64_t allocation_failures;
  uint64_t victims_evicted;
  uint64_t catalog_replacements;
  uint64_t writes_through;
  uint64_t stale_commits;
  uint64_t host_serves;
  uint64_t admissions;
  uint64_t pool_values;
  uint64_t heap_values;
  uint32_t epoch;
  uint32_t issued;
  uint32_t committed;
} kvo_stats;

kvo_store *kvo_store_create(const kvo_config *cfg);
void kvo_store_destroy(kvo_store *s);

int kvo_put(kvo_store *s, const uint8_t *key, uint32_t key_len, const uint8_t *value,
            uint64_t len, int sync_commit);
int kvo_get(kvo_store *s, const uint8_t *key, uint32_t key_len, uint8_t *out, uint64_t capacity,
            int *found, uint64_t *value_len);
int kvo_exists(kvo_store *s, const uint8_t *key, uint32_t key_len, int *found);
int kvo_remove(kvo_store *s, const uint8_t *key, uint32_t key_len, int *removed);
int kvo_move_to_host(kvo_store *s, const uint8_t *key, uint32_t key_len);
int kvo_move_to_device(kvo_store *s, const uint8_t *key, uint32_t key_len);
int kvo_flush(kvo_store *s);

/* introspection: location code of a key (KVO_LOC_*), or KVO_ABSENT. No barrier, no recency. */
int kvo_location(kvo_store *s, const uint8_t *key, uint32_t key_len, uint64_t *value_off);
void kvo_get_stats(kvo_store *s, kvo_stats *out);
/* FNV index lookup only: returns the directory slot or KVO_BUCKET_EMPTY. */
uint32_t kvo_index_lookup(kvo_store *s, const uint8_t *key, uint32_t key_len);
/* raw views for white-box parity checks */
const uint32_t *kvo_buckets(kvo_store *s, uint32_t *n_buckets); /* pairs {hash, slot} */
uint32_t kvo_lru_order(kvo_store *s, uint32_t *slots_out, uint32_t cap); /* MRU -> LRU */

/* ---- paged-block put / get (the B200 block path; multi-threaded CPU baseline) ----
 * Block value layout (kvo_block_format): header [MAGIC, n_layers, layer bytes...] padded to 32 B,
 * then member blocks back to back in member order, each region 16-byte aligned. members[m] holds
 * n_pool_blocks blocks of member_bytes[m]; keys are 64-bit (stored as 8 little-endian bytes).
 * put gathers each block into the store's heap (write-through at the next commit barrier); get
 * scatters hits back. n_threads workers run the byte copies. */
uint64_t kvo_block_format(uint32_t n_members, uint32_t members_per_layer, const uint64_t *member_bytes,
                          uint32_t *words, uint32_t words_cap, uint32_t *n_words,
                          uint64_t *region_bases);
int kvo_put_blocks(kvo_store *s, uint8_t *const *members, uint32_t n_members, uint32_t members_per_layer,
                   const uint64_t *member_bytes, const uint64_t *keys, const uint32_t *block_ids,
                   uint32_t n, int n_threads);
int kvo_get_blocks(kvo_store *s, uint8_t *const *members, uint32_t n_members, uint32_t members_per_layer,
                   const uint64_t *member_bytes, const uint64_t *keys, const uint32_t *block_ids,
                   uint32_t n, uint8_t *found, int n_threads);

/* ---- token-granular paged KV fill (moreh_paged_fill_cache_varlen) ----
 * Restates the reader / writer kernels of moreh_paged_fill_cache_varlen (patch 0002,
 * reader_fill_cache_varlen.cpp and writer_fill_cache_varlen.cpp) one token at a time on row-major
 * buffers. k_fill / v_fill: [n_heads][total_tokens] rows of row_bytes; caches:
 * [num_blocks][n_heads][block_size] rows. cu_seqlens: batch + 1 offsets, padded with -1; the
 * valid total is the last entry before the padding. Token t (below that total and below
 * total_tokens) of request r = the last i with (uint32)cu[i] <= t goes to cache position
 * pos = t - cu[r] + start_positions[r], block page_table[r][pos / block_size], row pos % block_size,
 * for every head; a page-table entry of 0 (vLLM's null block) or below 0 skips the token. The
 * reference moves 32-token tiles, so both agree whenever request boundaries, start positions and
 * the block size are multiples of 32. Tokens whose position lies beyond the page-table row or whose
 * block is >= num_blocks (the reference would read or write out of bounds) are skipped and
 * counted in *out_of_range. */
int kvo_paged_fill_varlen(const uint8_t *k_fill, const uint8_t *v_fill, uint32_t n_heads, uint32_t total_tokens,
                          uint32_t row_bytes, const int32_t *cu_seqlens, uint32_t batch, const int32_t *page_table,
                          uint32_t max_blocks_per_seq, const int32_t *start_positions, uint8_t *cache_k,
                          uint8_t *cache_v, uint32_t num_blocks, uint32_t block_size, uint64_t *out_of_range);

#ifdef __cplusplus
}
#endif
#endif
