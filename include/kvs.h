/*
 * kvs.h -- C ABI of the B200 KV block store (kvcache_manager hot path).
 *
 * This is the drop-in boundary that replaces the reference's TTNN backend bridge
 * (src/backend_bridge.hpp:16-28, which pins the opaque ClientOperations ABI, version 4, of
 * third_party/tt-metal/patches/0003-kvcache-protocol-device-runtime.patch lines 3408-3531).
 * Every entry point takes plain pointers and sizes; device buffers are CUDA device pointers
 * (or any UVA pointer the CUDA device can address) and streams are cudaStream_t passed as
 * void*. No C++ or torch types cross this boundary.
 *
 * Conventions
 *   - Every function returns KVS_OK (0) or a negative KVS_E_* code; kvs_last_error() returns a
 *     thread-local message for the last failure on the calling thread. A get miss is not an
 *     error: *found is set to 0.
 *   - Calls on one client are serialised by the client; distinct clients may call
 *     concurrently. A shard (kvs_server) serialises the directory updates of all its clients.
 *   - Keys are 1..max_key_bytes (<= 128) bytes. The batched block calls take 64-bit keys
 *     (chained prefix-block hashes); a 64-bit key is stored as its 8 little-endian bytes, so
 *     kvs_put(key=&u64, key_len=8) and kvs_put_blocks(keys={u64}) name the same entry.
 *   - `stream` is the caller's stream: a call's device work starts after the work queued on it
 *     before the call and work queued on it after the call starts after the call's device work.
 *     A null stream is the legacy default stream (torch's default stream).
 *   - Ordering follows the reference (kvcache_manager/docs/design.md sections 5-6 in patch 0003,
 *     lines 7527-7683): a put
 *     returns once its bytes have landed in the device slab (on `stream`); host write-through
 *     finishes asynchronously; get, exists, delete, move and flush first wait for every issued
 *     put to be host-committed (the reference's COMMIT_BARRIER).
 */
#ifndef KVS_H
#define KVS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVS_ABI_VERSION 1

/* status codes */
#define KVS_OK 0
#define KVS_E_INVAL (-1)       /* invalid argument (reference: TT_FATAL on validation) */
#define KVS_E_CUDA (-2)        /* a CUDA call failed */
#define KVS_E_NOSPACE (-3)     /* no device-cache or catalog space even after forced commits */
#define KVS_E_TIMEOUT (-4)     /* a bounded wait expired */
#define KVS_E_TOO_SMALL (-5)   /* get: output capacity smaller than the stored value */
#define KVS_E_QUARANTINED (-6) /* an earlier indeterminate failure quarantined this handle */
#define KVS_E_CLOSED (-7)      /* the handle was closed */
#define KVS_E_FORMAT (-8)      /* stored value does not match the requested block layout */

/* location codes reported by kvs_location (reference layout.hpp kLocation*) */
#define KVS_LOC_DEVICE 0
#define KVS_LOC_HOST 1
#define KVS_LOC_PENDING 2
#define KVS_LOC_ABSENT (-1)

typedef struct kvs_server kvs_server; /* one store shard, owning one GPU's slab */
typedef struct kvs_client kvs_client; /* a client bound to one GPU and a set of shards */

/* Server construction knobs. Replaces the reference's env-parsed ServerRuntimeCore config
 * (src/native/ttnn/server_runtime/server.cpp:199-350; patch 0003 lines 5156-5380). */
typedef struct {
  int32_t device;           /* CUDA device ordinal that holds the slab and index */
  uint32_t max_keys;        /* catalog entries (KVM_SERVER_DRAM_MAX_KEYS) */
  uint32_t unit_bytes;      /* value-heap unit; 4288 = the reference's kMaxChunkValueBytes */
  uint32_t max_key_bytes;   /* <= 128 (KVM_SERVER_MAX_KEY_BYTES) */
  uint64_t heap_bytes;      /* device value slab (KVM_SERVER_DRAM_VALUE_HEAP_BYTES) */
  uint64_t host_pool_bytes; /* pinned host pool (KVM_SERVER_HOST_POOL_BYTES) */
  uint64_t max_value_bytes; /* per-value cap (KVM_COMMON_MAX_VALUE_BYTES) */
  uint32_t shard_id;        /* this shard's index in a hash-sharded group */
  uint32_t flags;           /* KVS_SERVER_* bits */
} kvs_server_config;

#define KVS_SERVER_PROFILE 1u /* collect move timing (KVM_SERVER_PROFILE) */

/* Paged KV layout the block calls gather from / scatter into. A value stored for one key is
 * the one-block chunk blob of the reference's raw-byte codec (patch 0005 lines 12258-12310):
 *   header words [0x524B564E, n_layers, bytes_of_layer(0) .. bytes_of_layer(n_layers-1)]
 *   zero padded to 32 bytes, then every member's block back to back in member order.
 * Members are grouped per layer (members_per_layer of them: K, V, and optionally per-block
 * scales), member m of layer l is member_ptrs[l * members_per_layer + m]. */
typedef struct {
  uint32_t n_members;                /* total members = n_layers * members_per_layer */
  uint32_t members_per_layer;        /* 2 for (K, V) */
  const uint64_t *member_ptrs;       /* [n_members] device pointers (host array) */
  const uint64_t *member_block_bytes;/* [n_members] bytes of one block of each member */
  uint64_t n_pool_blocks;            /* blocks per member tensor (bounds check) */
} kvs_block_layout;

typedef struct {
  uint64_t count;
  uint64_t prepare_ns;
  uint64_t program_ns;
  uint64_t enqueue_ns;
  uint64_t landed_wait_ns;
  uint64_t commit_wait_ns;
  uint64_t total_ns;
} kvs_put_profile; /* include/kvcache_manager/profiles.hpp:43-51 PutProfile */

typedef struct {
  uint64_t to_host_count, to_host_worker_ns, to_host_complete_ns, to_host_read_calls,
      to_host_read_bytes, to_host_read_passes, to_host_read_retries, to_host_read_io_ns,
      to_host_scatter_ns, to_host_device_pushes, to_device_count, to_device_worker_ns,
      to_device_complete_ns;
} kvs_move_profile; /* profiles.hpp:10-24 MoveProfile */

typedef struct {
  uint64_t allocation_calls, allocation_successes, allocation_failures, victim_scans,
      victims_evicted, lease_calls, lease_successes, lease_failures, lease_victim_scans,
      lease_victims_evicted, scan_cycles, lease_scan_cycles, allocation_cycles;
  uint32_t clock_mhz;
} kvs_allocator_profile; /* profiles.hpp:26-41 AllocatorProfile */

typedef struct {
  uint64_t live_device_bytes, pending_device_bytes, live_keys, device_resident_keys;
  uint64_t allocation_calls, allocation_successes, allocation_failures, victims_evicted;
  uint64_t catalog_replacements, writes_through, stale_commits, host_serves, admissions;
  uint64_t pool_values, heap_values;
  uint32_t epoch, issued, committed;
  uint64_t kernel_launches; /* kernels this shard's clients launched */
} kvs_stats;

/* ---- version / errors ---- */
int kvs_abi_version(void);        /* replaces client_operations_abi_version(), patch 0003:3439 */
const char *kvs_last_error(void); /* thread-local message of the last failure */

/* ---- server (one shard) ----  include/kvcache_manager/server.hpp:21-55 */
int kvs_server_config_default(kvs_server_config *cfg); /* defaults + KVM_* environment knobs */
int kvs_server_create(const kvs_server_config *cfg, kvs_server **out);
int kvs_server_destroy(kvs_server *s); /* drains write-through, then frees (Server::close) */
int kvs_server_is_ready(kvs_server *s, int *ready);
int kvs_server_moves_completed(kvs_server *s, uint64_t *out);
int kvs_server_move_profile(kvs_server *s, kvs_move_profile *out);
int kvs_server_allocator_profile(kvs_server *s, kvs_allocator_profile *out);
int kvs_server_stats(kvs_server *s, kvs_stats *out);
int kvs_server_device(kvs_server *s, int *device);
/* commit_barrier progress: issued and committed PUT counters (Server::test_put_drain_progress,
 * server.hpp:52) */
int kvs_server_put_drain_progress(kvs_server *s, uint32_t *issued, uint32_t *committed);
/* introspection for parity tests: location of a key (KVS_LOC_*), and its slab offset */
int kvs_server_location(kvs_server *s, const void *key, uint32_t key_len, int *location,
                        uint64_t *value_off);
/* copies the host directory's hash buckets ({hash, slot} pairs) and the device replica's */
int kvs_server_index_snapshot(kvs_server *s, uint32_t *host_pairs, uint32_t *device_pairs,
                              uint32_t cap_pairs, uint32_t *n_buckets);
/* residency LRU from MRU to LRU as directory slots */
int kvs_server_lru_order(kvs_server *s, uint32_t *slots, uint32_t cap, uint32_t *n);

/* ---- client ----  include/kvcache_manager/client.hpp:26-66 */
/* A client on `device` addressing `n_shards` shards; key k goes to shard fnv1a32(k) % n_shards
 * (the reference's worker groups, server.cpp:80-86, become hash shards across GPUs). */
int kvs_client_create(kvs_server *const *shards, uint32_t n_shards, int32_t device,
                      kvs_client **out);
int kvs_client_destroy(kvs_client *c); /* drains this client's puts, then frees (Client::close) */
int kvs_client_is_established(kvs_client *c, int *established);
int kvs_client_shard_of(kvs_client *c, const void *key, uint32_t key_len, uint32_t *shard);
/* PING: echo payload (<= 1024 bytes) through the device (Client::ping) */
int kvs_ping(kvs_client *c, const void *payload, uint32_t len, void *out, void *stream);

/* Client::put (patch 0003 lines 2533-2651): store value_len bytes at `value` (device memory)
 * under key. Returns after the bytes landed in the slab; sync_commit also waits for host
 * write-through. */
int kvs_put(kvs_client *c, const void *key, uint32_t key_len, const void *value,
            uint64_t value_len, int sync_commit, void *stream);
/* Client::put_batch: n independent puts in input order */
int kvs_put_batch(kvs_client *c, uint32_t n, const void *const *keys, const uint32_t *key_lens,
                  const void *const *values, const uint64_t *value_lens, int sync_commit,
                  void *stream);
/* Client::get (patch 0003 lines 2786-2891): on a hit, copy the value into out (capacity bytes)
 * and set *found=1, *value_len; a miss leaves out unchanged. */
int kvs_get(kvs_client *c, const void *key, uint32_t key_len, void *out, uint64_t capacity,
            int *found, uint64_t *value_len, void *stream);
/* Client::get_parallel (patch 0003 lines 2893-3125): clients[i] reads keys[i] into
 * out + i * stride; found[i] per key. */
int kvs_get_parallel(kvs_client *const *clients, uint32_t n, const void *const *keys,
                     const uint32_t *key_lens, void *out, uint64_t stride, uint64_t capacity,
                     uint8_t *found, void *stream);
int kvs_exists(kvs_client *c, const void *key, uint32_t key_len, int *found);
int kvs_delete(kvs_client *c, const void *key, uint32_t key_len, int *removed);
int kvs_move_to_host(kvs_client *c, const void *key, uint32_t key_len);
int kvs_move_to_device(kvs_client *c, const void *key, uint32_t key_len);
int kvs_flush(kvs_client *c);
int kvs_client_put_profile(kvs_client *c, kvs_put_profile *out);

/* ---- batched paged-block path (the B200 main path) ----
 * put: for each i, gather block block_ids[i] of every member into one blob value stored under
 *      keys[i] (one kernel for the whole batch). Replaces the connector's per-chunk
 *      gather_tp_shards_to_chip + Client.put sequence (patch 0005 lines 9653-9708).
 * get: look every key up in the shard's device hash index (warp-cooperative probe) and
 *      scatter each hit's members into block block_ids[i]; found[i] per key (host array).
 *      Misses leave their blocks untouched. Replaces Client.get + scatter_chunk_from_chip.
 * keys / block_ids / found are host arrays. */
int kvs_put_blocks(kvs_client *c, const kvs_block_layout *layout, uint32_t n,
                   const uint64_t *keys, const int64_t *block_ids, int sync_commit,
                   void *stream);
int kvs_get_blocks(kvs_client *c, const kvs_block_layout *layout, uint32_t n,
                   const uint64_t *keys, const int64_t *block_ids, uint8_t *found,
                   void *stream);
/* EXISTS over a batch of 64-bit keys through the device index; no recency update. */
int kvs_exists_batch(kvs_client *c, uint32_t n, const uint64_t *keys, uint8_t *found);

/* ---- chunk restore straight into a paged cache ----
 * The store side of the connector's batched restore. The reference fetches each chunk's K / V and
 * then fills the cache one layer per call with moreh_paged_fill_cache_varlen
 * (TTGPUConnector.batched_to_gpu and _paged_fill_layer_coalesced, patch 0005 lines 6780-6870 and
 * 11563-11770); here one paged-fill launch per 64 layers reads every chunk's rows where its value
 * lives (the slab, or the pinned host tier) and writes them token by token.
 * Key i names a raw-byte chunk value (patch 0005 lines 12258-12310): header words
 * [0x524B564E, n_layers, 2 alloc_i x n_layers] zero padded to 32 bytes, then per layer the K region
 * and the V region of alloc_i = ceil(tokens[i] / block_size) x block_size x row_bytes bytes each,
 * one row_bytes row per token (the chunk blob kvs_gather_chunk writes from caches whose block is
 * [block_size][row_bytes], e.g. vLLM's [num_blocks, block_size, heads, head_dim]). Row j < tokens[i]
 * of layer l goes to cache_ks[l] / cache_vs[l] ([num_blocks][block_size][row_bytes], 16-byte
 * aligned, row_bytes a multiple of 16) at position p = start_positions[i] + j: block
 * page_table[i * max_blocks_per_chunk + p / block_size], row p % block_size; entries <= 0 skip the
 * token, as in kvs_paged_fill_varlen. found[i] per key; a miss writes nothing; a stored value of
 * another length fails the call with KVS_E_FORMAT before any state changes. Each key is a get
 * (commit barrier first, recency, read-through admission, in key order). keys, key_lens, tokens,
 * page_table, start_positions and found are host arrays; the caches are device memory of the
 * client's GPU. Returns once the rows have landed. No counterpart entry point in the reference. */
int kvs_restore_chunks(kvs_client *c, uint32_t n, const void *const *keys, const uint32_t *key_lens,
                       const uint32_t *tokens, uint32_t n_layers, void *const *cache_ks, void *const *cache_vs,
                       uint32_t num_blocks, uint32_t block_size, uint32_t row_bytes, const int32_t *page_table,
                       uint32_t max_blocks_per_chunk, const int32_t *start_positions, uint8_t *found,
                       void *stream);

/* ---- hash sharding across processes (one process per GPU) ----
 * The reference serves several server worker groups behind one Fabric endpoint
 * (src/native/ttnn/server_runtime/server.cpp:80-86), each an independent directory; here each
 * shard is a process on its own GPU and the block bytes cross NVLink as kernel-issued P2P
 * stores. A step is bulk-synchronous (the host exchange runs on torch.distributed):
 *   1. clients send get and put keys to the owning shards;
 *   2. the owner serves the gets: lookup, then one scatter launch that stores each hit
 *      straight into the requesting process's paged pool (opened from IPC handles);
 *   3. the owner grants the puts (slab offsets), the clients gather their blocks straight into
 *      the owners' slabs, and after every client's copy has finished each owner starts the host
 *      write-through of what landed.
 * None of these has a counterpart entry point in the reference, whose shards share one process. */
typedef struct {
  uint8_t bytes[64];
} kvs_ipc_handle; /* a cudaIpcMemHandle_t */

/* IPC handle of the device allocation holding `ptr`, and ptr's offset inside it */
int kvs_ipc_export(const void *ptr, kvs_ipc_handle *handle, uint64_t *offset);
/* map another process's allocation on `device` (peer access enabled on first use) */
int kvs_ipc_open(int32_t device, const kvs_ipc_handle *handle, void **base);
int kvs_ipc_close(int32_t device, void *base);
/* the shard's value slab (a device allocation of its own, so its IPC offset is 0) */
int kvs_server_slab(kvs_server *s, void **base, uint64_t *bytes);

/* Owner side (a client whose only shard is the owner's). Gets of several requesters in one
 * call: key i is scattered into the paged pool layouts[sets[i]], whose member pointers may be
 * peer memory. Same semantics as kvs_get_blocks on the concatenated batch; every layout must
 * have the same member sizes. n == 0 still runs the commit barrier. */
int kvs_serve_gets(kvs_client *c, uint32_t n_sets, const kvs_block_layout *layouts, uint32_t n,
                   const uint32_t *sets, const int64_t *block_ids, const uint64_t *keys, uint8_t *found,
                   void *stream);
/* Owner side: the same gets delivered as whole values (header included), value i into
 * rows + i * value_len (this GPU's memory), for transports that move contiguous buffers. */
int kvs_serve_gets_packed(kvs_client *c, void *rows, uint64_t value_len, uint32_t n, const uint64_t *keys,
                          uint8_t *found, void *stream);
/* Owner side: publish puts in order (pending, pinned), returning each value's slab offset.
 * Stops early (n_granted < n) at a put whose space needs the host commit of a value that has
 * not landed yet; the rest are granted after kvs_puts_landed. KVS_E_NOSPACE if a value can
 * never fit. */
int kvs_grant_puts(kvs_client *c, uint32_t n, const uint64_t *keys, uint64_t value_len, uint64_t *slab_offsets,
                   uint32_t *n_granted);
/* Owner side: every granted value has been written (ordered before `stream`'s current work);
 * start their host write-through. */
int kvs_puts_landed(kvs_client *c, void *stream);

/* Client side: one copy launch between the layout's blocks (this GPU's memory) and explicit
 * value addresses (this GPU's or a peer's); to_blob 1 gathers (writes the value header too),
 * 0 scatters. Addresses are 16-byte aligned; a zero address skips the block. When every address
 * lies in a shard's slab or a mapping opened by kvs_ipc_open the bulk-copy engine moves the
 * bytes, otherwise plain 16-byte loads and stores (any memory the GPU can address). */
int kvs_copy_blocks(kvs_client *c, const kvs_block_layout *layout, uint32_t n, const int64_t *block_ids,
                    const uint64_t *blob_addrs, int to_blob, void *stream);
/* One copy launch between whole values at explicit addresses and contiguous rows:
 * to_rows 1 copies addrs[i] -> rows + i * value_len, 0 the reverse. */
int kvs_copy_values(kvs_client *c, void *rows, uint64_t value_len, uint32_t n, const uint64_t *addrs, int to_rows,
                    void *stream);

/* Client side: the request records of one sharded step, bucketed by owning shard on the GPU.
 * keys / ids: n keys and block ids, the first n_get gets, the rest puts. A key's owner is
 * slot_shard[fnv1a32(key) % 4096] (an int32 placement table), or fnv1a32(key) % world when
 * slot_shard is null; fnv1a32 runs over the key's 8 little-endian bytes, as kvs_client_shard_of's
 * does. records: world records of 4 + 4 x cap int64 words, record o = {gets, puts, op, 0, cap get
 * keys, cap get block ids, cap put keys, cap put block ids}, keys of each kind in batch order,
 * unused words zero (the layout the step's all-to-all sends). back: [world][2][cap] int32, the
 * batch position (within its kind) of each placed key; counts: [2][world] int32 keys per (kind,
 * owner); *overflow: 0, or 1 when an owner got more than cap keys of one kind (the first cap are
 * placed). Every pointer is device memory of `device`; asynchronous on `stream`. world <= 32.
 * The reference routes each request to its worker group on the host
 * (include/kvcache_manager/client.hpp:26-32); this is the GPU bucketing pass of the step. */
int kvs_bucket_requests(int32_t device, const uint64_t *keys, const int64_t *ids, uint32_t n, uint32_t n_get,
                        const int32_t *slot_shard, uint32_t world, uint32_t cap, int64_t op, int64_t *records,
                        int32_t *back, int32_t *counts, uint32_t *overflow, void *stream);

/* ---- token-granular paged KV fill ----
 * Replaces ttnn.experimental.moreh_paged_fill_cache_varlen (patch 0002 lines 106-421: reader /
 * writer kernels, validation at lines 441-545). k_fill / v_fill: [n_heads][total_tokens] rows of
 * row_bytes (one [1, H, T, D] tensor each); cache_k / cache_v: [num_blocks][n_heads][block_size]
 * rows; cu_seqlens: batch + 1 int32 offsets, padded with -1 after the valid ones; page_table:
 * [batch][max_blocks_per_seq] int32; start_positions: [batch] int32. Token t below the valid total
 * of request r (the last i with cu_seqlens[i] <= t) goes to cache position
 * p = t - cu_seqlens[r] + start_positions[r]: block page_table[r][p / block_size], row
 * p % block_size, every head. Entries <= 0 skip the token (vLLM's null block 0, -1 for unused
 * slots) as in the reference. The reference moves 32-token tiles; this fill moves single tokens
 * and equals it whenever boundaries, start positions and block_size are multiples of 32. A
 * position beyond the page-table row or a block >= num_blocks (the reference would read or write
 * out of bounds) skips the token and increments *out_of_range when given (a device word).
 * All arrays are device memory of one GPU; asynchronous on `stream`. */
int kvs_paged_fill_varlen(const void *k_fill, const void *v_fill, uint32_t n_heads, uint32_t total_tokens,
                          uint32_t row_bytes, const int32_t *cu_seqlens, uint32_t batch, const int32_t *page_table,
                          uint32_t max_blocks_per_seq, const int32_t *start_positions, void *cache_k, void *cache_v,
                          uint32_t num_blocks, uint32_t block_size, uint32_t *out_of_range, void *stream);
/* The same fill for n_layers layers that share the requests and page tables (no counterpart in
 * the reference, which fills one layer per call): layer l reads k_fills[l] / v_fills[l] and
 * writes cache_ks[l] / cache_vs[l], every layer of the same shapes. Up to 64 layers go in one
 * launch, so a restore of a whole model pays one kernel ramp instead of one per layer. Each
 * layer's result equals kvs_paged_fill_varlen on that layer; *out_of_range counts each skipped
 * token once (not once per layer). */
int kvs_paged_fill_varlen_layers(uint32_t n_layers, const void *const *k_fills, const void *const *v_fills,
                                 uint32_t n_heads, uint32_t total_tokens, uint32_t row_bytes,
                                 const int32_t *cu_seqlens, uint32_t batch, const int32_t *page_table,
                                 uint32_t max_blocks_per_seq, const int32_t *start_positions, void *const *cache_ks,
                                 void *const *cache_vs, uint32_t num_blocks, uint32_t block_size,
                                 uint32_t *out_of_range, void *stream);

/* ---- chunk gather / scatter ops ----
 * gather_tp_shards_to_chip / pack_local_shards (patch 0003 gather.hpp lines 9372-9417) and
 * their inverses scatter_chunk_from_chip / unpack_local_shards (9418-9453).
 * member_ptrs[r * n_members + m] is rank r's shard of member m (device or peer pointers);
 * for member m, chunk block cb and rank r, member_block_bytes[m] bytes at
 * block_ids[cb] * member_block_bytes[m] move to/from
 * blob + region_bases[m] + cb * member_block_bytes[m] * n_ranks + r * member_block_bytes[m].
 * gather writes header_words at the blob start. member_extent[m] bounds every member buffer,
 * blob_bytes bounds the blob; violations return KVS_E_INVAL before any access. Asynchronous on
 * `stream` (on the device of `blob`). */
int kvs_gather_chunk(const uint64_t *member_ptrs, uint32_t n_ranks, uint32_t n_members,
                     const uint64_t *member_block_bytes, const uint64_t *member_extent,
                     const uint32_t *block_ids, uint32_t n_blocks, const uint64_t *region_bases,
                     const uint32_t *header_words, uint32_t n_header_words, void *blob,
                     uint64_t blob_bytes, void *stream);
int kvs_scatter_chunk(const void *blob, uint64_t blob_bytes, const uint64_t *member_ptrs,
                      uint32_t n_ranks, uint32_t n_members, const uint64_t *member_block_bytes,
                      const uint64_t *member_extent, const uint32_t *block_ids,
                      uint32_t n_blocks, const uint64_t *region_bases, void *stream);

/* ---- chunk gather for callers that cannot allocate ----
 * No counterpart in the reference. Same arguments, validation and result as kvs_gather_chunk,
 * but the per-call metadata (member pointers, block sizes, region bases, block ids, header words)
 * is staged in one fixed device array compiled into the library instead of a buffer taken from
 * the CUDA allocator, so the call makes no cudaMalloc / cudaMallocAsync / cudaFree or other
 * allocating call. It exists for callers that must not allocate: serving engines that hand
 * nearly all HBM to their paged KV pool and leave no headroom (or must keep their memory
 * accounting exact), and latency-critical restore paths where an allocation could synchronise
 * the device.
 *   - The metadata reaches the array in the parameters of small staging kernels queued ahead of
 *     the copy (no host-to-device memory copy), so the calling thread never waits for earlier
 *     work on the stream.
 *   - Limit: the metadata must fit KVS_NOALLOC_SCRATCH_BYTES (8 x n_ranks x n_members
 *     + 24 x n_members + 8 x n_blocks + 4 x n_header_words bytes, each part rounded up to 16,
 *     about 64 KiB); larger requests fail with KVS_E_INVAL and a message naming the limit.
 *   - Every GPU that loads the library holds the array (64 KiB) until the process exits.
 *   - A copy whose bounded waits expired shows only in kvs_copy_engine_status.
 *   - The first call on a device looks up the array's device address; make that first call
 *     before any stream capture on that device.
 *   - All calls share the array and each call overwrites it: calls whose work overlaps on the
 *     GPU (different streams, or different host threads) race on it; issue them on one stream
 *     or order them with events. */
#define KVS_NOALLOC_SCRATCH_BYTES (64u * 1024u)
int kvs_gather_chunk_noalloc(const uint64_t *member_ptrs, uint32_t n_ranks, uint32_t n_members,
                             const uint64_t *member_block_bytes, const uint64_t *member_extent,
                             const uint32_t *block_ids, uint32_t n_blocks,
                             const uint64_t *region_bases, const uint32_t *header_words,
                             uint32_t n_header_words, void *blob, uint64_t blob_bytes,
                             void *stream);

/* kernels launched by this library since load (a launch counter for the benchmark) */
uint64_t kvs_kernel_launch_count(void);

/* ---- copy-engine health ----
 * Every wait of the bulk-copy engine on a tile load is bounded (the reference's device runtime
 * bounds its NoC waits the same way and reports a timeout instead of hanging). A wait that expires
 * stops its CTA's copy early: the CTA first lets every load it issued land (each with the full
 * limit), then exits, and the result is incomplete.
 *   - Store calls report it themselves: the next call that synchronises (get, get_blocks, exists,
 *     flush, a sync_commit put) returns KVS_E_TIMEOUT and quarantines the client, so every later
 *     call returns KVS_E_QUARANTINED (the reference's Quarantined state,
 *     src/client_operations_adapter.cpp:54-59).
 *   - The asynchronous chunk ops (kvs_gather_chunk, kvs_scatter_chunk, kvs_gather_chunk_noalloc)
 *     return before their kernel runs, so they report it only here: after synchronising the stream,
 *     a count that grew since the last read means the blobs or blocks of the calls in between are
 *     incomplete.
 * expired_waits: waits on `device` that expired since the library loaded. unsafe_exits: CTAs that
 * exited while a load of theirs still had not landed after the full limit (never seen in normal
 * operation; the engine on that device cannot be trusted afterwards). No counterpart in the
 * reference. */
int kvs_copy_engine_status(int32_t device, uint32_t *expired_waits, uint32_t *unsafe_exits);
/* Polls of each bounded tile-load wait for launches from now on, process-wide; a negative value
 * restores the default (2^22 polls). Tests of the expiry path pass 0, which expires a CTA's first
 * wait at once while its loads still land normally. No counterpart in the reference. */
int kvs_set_copy_wait_limit(int64_t polls);
/* Copies of at most this many bytes per launch take the one-wave copy engine (one CTA per 16 KiB
 * piece of each member block, all loads in flight at once: lower latency for a few blocks) instead
 * of the persistent engines, and so does any copy whose member blocks are at most 16 KiB each;
 * process-wide, for launches from now on. 0 turns the one-wave engine off; a negative value
 * restores the default (512 MiB, or KVS_SMALL_COPY_BYTES when set). Every engine moves the same
 * bytes: tests run their cases under each. No counterpart in the reference. */
int kvs_set_small_copy_limit(int64_t bytes);

/* Per-client kernel timing: with timing on, CUDA events bracket every gather (put) and scatter
 * (get) copy-engine launch on the client stream. kvs_client_timing waits for them, returns the
 * totals since the last call (and resets). bytes = payload bytes the kernels moved. */
typedef struct {
  uint64_t launches;
  uint64_t bytes;
  double total_ms;
} kvs_kernel_timing;
int kvs_client_set_timing(kvs_client *c, int enable);
int kvs_client_timing(kvs_client *c, kvs_kernel_timing *gather, kvs_kernel_timing *scatter);
/* The same for the host-tier copies of a get (timing on): admissions = copy launches that read
 * host-tier values over PCIe into their new slab blocks (bytes = whole values), serves = copy
 * launches that scatter host-tier hits into the paged pool (bytes = payload), from the slab block
 * their admission filled or, when no block could be allocated, from the pinned host copy. No
 * counterpart in the reference. */
int kvs_client_host_tier_timing(kvs_client *c, kvs_kernel_timing *admissions, kvs_kernel_timing *serves);
/* Per-shard write-through timing: with timing on, CUDA events on the shard's write-through stream
 * bracket each batch of device->host copies (one batch per put call). kvs_server_write_through_timing
 * waits for them and returns the totals since the last call (and resets): launches = batches,
 * bytes = bytes copied to the host tier, total_ms = the copies' device time. No counterpart in the
 * reference (its tiering thread keeps MoveProfile wall-clock totals, kvs_server_move_profile). */
int kvs_server_set_timing(kvs_server *s, int enable);
int kvs_server_write_through_timing(kvs_server *s, kvs_kernel_timing *out);

#ifdef __cplusplus
}
#endif
#endif /* KVS_H */
