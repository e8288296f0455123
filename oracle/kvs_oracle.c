/*
 * kvs_oracle.c -- CPU restatement of the kvcache_manager hot path (TEST INFRASTRUCTURE ONLY).
 *
 * See kvs_oracle.h for scope. Each function cites the reference code it restates. Citations
 * "P2:n", "P3:n", "P5:n" are line numbers inside the reference's tt-metal patch files
 * third_party/tt-metal/patches/000{2,3,5}-*.patch, where the reference keeps these sources.
 */
#define _GNU_SOURCE
#include "kvs_oracle.h"

#include <pthread.h>
#include <unistd.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static __thread char g_err[512];

static int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

const char *kvo_last_error(void) { return g_err; }

/* ------------------------------------------------------------------------------------------ */
/* helpers                                                                                    */
/* ------------------------------------------------------------------------------------------ */

/* FNV-1a 32-bit, P3:9912-9919 (offset basis 2166136261, prime 16777619). */
uint32_t kvo_fnv1a32(const uint8_t *key, uint32_t len) {
  uint32_t h = 2166136261u;
  for (uint32_t i = 0; i < len; ++i) {
    h ^= (uint32_t)key[i];
    h *= 16777619u;
  }
  return h;
}

/* layout.hpp next_pow2 / hash_num_buckets, P3:6398-6404: load factor <= 0.5. */
uint32_t kvo_next_pow2(uint32_t x) {
  uint32_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

uint32_t kvo_hash_num_buckets(uint32_t max_keys) {
  return kvo_next_pow2(max_keys ? max_keys * 2u : 2u);
}

/* P3:10059-10076 */
uint32_t kvo_floor_log2(uint32_t v) {
  uint32_t o = 0;
  while (v > 1) {
    v >>= 1;
    ++o;
  }
  return o;
}

uint32_t kvo_buddy_order_for_units(uint32_t units) {
  uint32_t order = 0, block = 1;
  while (block < units) {
    block <<= 1;
    ++order;
  }
  return order;
}

/* packet.hpp chunk_count_for, P3:7114 (generalised to 64-bit lengths and any unit). */
uint64_t kvo_chunk_count(uint64_t bytes, uint32_t unit_bytes) {
  return bytes == 0 ? 0 : 1 + (bytes - 1) / unit_bytes;
}

/* ------------------------------------------------------------------------------------------ */
/* blob header + chunk plan                                                                   */
/* ------------------------------------------------------------------------------------------ */

/* RawByteCodec.device_chunk_plan P5:12286-12291 and the gather test's _gathered_plan:
 * [MAGIC, count] + sizes, padded with zero words to a 32-byte multiple. */
uint32_t kvo_header_words(uint32_t count, const uint32_t *sizes, uint32_t *out, uint32_t cap) {
  uint32_t n = 2 + count;
  uint32_t pad = ((KVO_HEADER_ALIGN - (n * 4) % KVO_HEADER_ALIGN) % KVO_HEADER_ALIGN) / 4;
  if (n + pad > cap) return 0;
  out[0] = KVO_BLOB_MAGIC;
  out[1] = count;
  for (uint32_t i = 0; i < count; ++i) out[2 + i] = sizes[i];
  for (uint32_t i = 0; i < pad; ++i) out[n + i] = 0;
  return n + pad;
}

/* P5:12284-12306: members are K then V per layer; region_bases[2l] = hdr + l*2*alloc,
 * region_bases[2l+1] = that + alloc; value_len = hdr + n_layers*2*alloc. */
uint64_t kvo_chunk_plan(uint32_t n_layers, uint64_t alloc, uint32_t *words, uint32_t *n_words,
                        uint32_t words_cap, uint64_t *region_bases) {
  uint32_t *sizes = (uint32_t *)calloc(n_layers ? n_layers : 1, sizeof(uint32_t));
  for (uint32_t l = 0; l < n_layers; ++l) sizes[l] = (uint32_t)(2 * alloc);
  uint32_t nw = kvo_header_words(n_layers, sizes, words, words_cap);
  free(sizes);
  if (nw == 0) return 0;
  *n_words = nw;
  uint64_t hdr = 4ull * nw;
  for (uint32_t l = 0; l < n_layers; ++l) {
    region_bases[2 * l] = hdr + (uint64_t)l * 2 * alloc;
    region_bases[2 * l + 1] = region_bases[2 * l] + alloc;
  }
  return hdr + (uint64_t)n_layers * 2 * alloc;
}

/* ------------------------------------------------------------------------------------------ */
/* gather / scatter (a4 / a5)                                                                 */
/* ------------------------------------------------------------------------------------------ */

/* Validation restates validate_chunk, P3:8355-8470, for the B200 data model: members are
 * plain byte buffers with a known extent, and the 32-byte alignment rules of the reference
 * (a DRAM NoC read rounds down to 32 B) are kept for region bases and the header. Segment
 * sizes may be any multiple of 4 (per-member sizes also carry per-block fp32 scales). */
static int validate_chunk(uint32_t n_ranks, uint32_t n_members, const uint64_t *member_bytes,
                          const uint64_t *member_extent, const uint32_t *block_ids,
                          uint32_t n_blocks, const uint64_t *region_bases, uint32_t header_bytes,
                          uint64_t blob_bytes) {
  if (n_ranks == 0) return fail(KVO_E_INVAL, "rank_coords must not be empty");
  if (n_members == 0) return fail(KVO_E_INVAL, "members must not be empty");
  if (n_blocks == 0) return fail(KVO_E_INVAL, "block_ids must not be empty");
  if (header_bytes % 32 != 0)
    return fail(KVO_E_INVAL, "header must be 32-byte aligned, got %u B", header_bytes);
  if (header_bytes > blob_bytes)
    return fail(KVO_E_INVAL, "%u B header exceeds the %llu B blob", header_bytes,
                (unsigned long long)blob_bytes);
  uint32_t max_block = 0;
  for (uint32_t i = 0; i < n_blocks; ++i)
    if (block_ids[i] > max_block) max_block = block_ids[i];
  for (uint32_t m = 0; m < n_members; ++m) {
    uint64_t sbb = member_bytes[m];
    if (sbb == 0 || sbb % 4 != 0)
      return fail(KVO_E_INVAL, "member %u block bytes %llu must be nonzero and 4-byte aligned", m,
                  (unsigned long long)sbb);
    if (region_bases[m] % 32 != 0)
      return fail(KVO_E_INVAL, "region base %llu must be 32-byte aligned",
                  (unsigned long long)region_bases[m]);
    if (region_bases[m] < header_bytes)
      return fail(KVO_E_INVAL, "member %u's region at %llu B overlaps the %u B header", m,
                  (unsigned long long)region_bases[m], header_bytes);
    uint64_t source_end = ((uint64_t)max_block + 1) * sbb;
    if (source_end > member_extent[m])
      return fail(KVO_E_INVAL, "block %u reaches past member %u's %llu B shard", max_block, m,
                  (unsigned long long)member_extent[m]);
    uint64_t end = region_bases[m] + (uint64_t)n_blocks * sbb * n_ranks;
    if (end > blob_bytes)
      return fail(KVO_E_INVAL, "member %u's region ends at %llu B, past the %llu B blob", m,
                  (unsigned long long)end, (unsigned long long)blob_bytes);
  }
  return KVO_OK;
}

/* gather_push kernel semantics, P3:7745-7971 and gather.hpp P3:9372-9392: for member m,
 * chunk block cb, rank r: dst[region_bases[m] + cb*block_bytes + r*sbb] <- shard block. */
int kvo_gather(const uint8_t *const *members, uint32_t n_ranks, uint32_t n_members,
               const uint64_t *member_bytes, const uint64_t *member_extent,
               const uint32_t *block_ids, uint32_t n_blocks, const uint64_t *region_bases,
               const uint32_t *header_words, uint32_t n_header_words, uint8_t *dst,
               uint64_t dst_bytes) {
  int rc = validate_chunk(n_ranks, n_members, member_bytes, member_extent, block_ids, n_blocks,
                          region_bases, 4 * n_header_words, dst_bytes);
  if (rc) return rc;
  if (n_header_words) memcpy(dst, header_words, 4ull * n_header_words);
  for (uint32_t m = 0; m < n_members; ++m) {
    uint64_t sbb = member_bytes[m];
    uint64_t block_bytes = sbb * n_ranks;
    for (uint32_t cb = 0; cb < n_blocks; ++cb)
      for (uint32_t r = 0; r < n_ranks; ++r)
        memcpy(dst + region_bases[m] + cb * block_bytes + r * sbb,
               members[(uint64_t)r * n_members + m] + (uint64_t)block_ids[cb] * sbb, sbb);
  }
  return KVO_OK;
}

/* scatter_push kernel semantics, P3:8028-8247: exact inverse; blocks outside block_ids and
 * bytes outside the listed ranks' slices are untouched. */
int kvo_scatter(const uint8_t *src, uint64_t src_bytes, uint8_t *const *members, uint32_t n_ranks,
                uint32_t n_members, const uint64_t *member_bytes, const uint64_t *member_extent,
                const uint32_t *block_ids, uint32_t n_blocks, const uint64_t *region_bases) {
  int rc = validate_chunk(n_ranks, n_members, member_bytes, member_extent, block_ids, n_blocks,
                          region_bases, 0, src_bytes);
  if (rc) return rc;
  for (uint32_t m = 0; m < n_members; ++m) {
    uint64_t sbb = member_bytes[m];
    uint64_t block_bytes = sbb * n_ranks;
    for (uint32_t cb = 0; cb < n_blocks; ++cb)
      for (uint32_t r = 0; r < n_ranks; ++r)
        memcpy(members[(uint64_t)r * n_members + m] + (uint64_t)block_ids[cb] * sbb,
               src + region_bases[m] + cb * block_bytes + r * sbb, sbb);
  }
  return KVO_OK;
}

/* ------------------------------------------------------------------------------------------ */
/* slot decode + raw run planner                                                              */
/* ------------------------------------------------------------------------------------------ */

/* RawByteCodec._chunk_slots P5:12148-12163 and _n_blocks P5:12165-12166. */
int kvo_chunk_slots(const int64_t *slots, uint64_t n, uint32_t block_size, uint64_t *first_block,
                    uint64_t *n_blocks) {
  if (n == 0) return fail(KVO_E_INVAL, "raw-byte codec: empty slot_mapping slice");
  if (slots[0] < 0 || slots[0] % block_size != 0)
    return fail(KVO_E_INVAL,
                "raw-byte codec: chunk does not start on a cache-block boundary (first slot %lld, "
                "block_size %u)",
                (long long)slots[0], block_size);
  for (uint64_t i = 0; i < n; ++i)
    if (slots[i] != slots[0] + (int64_t)i)
      return fail(KVO_E_INVAL, "raw-byte codec: chunk slots must be sequential within one DP group");
  *first_block = (uint64_t)slots[0] / block_size;
  *n_blocks = (n + block_size - 1) / block_size;
  return KVO_OK;
}

static int fits_u32(int64_t v) { return v >= 0 && (uint64_t)v <= 0xFFFFFFFFull; }

/* append_region_raw_explicit_run, P2:1382-1410: append, merging with the previous run when
 * both the device and host ranges continue it on the same shard. */
static int append_run(kvo_run *runs, uint64_t *count, uint64_t cap, int64_t shard,
                      int64_t dev_off, int64_t bytes, int64_t host_off) {
  if (!fits_u32(shard) || !fits_u32(dev_off) || !fits_u32(bytes) || host_off < 0 || bytes <= 0)
    return KVO_E_INVAL;
  if (*count > 0) {
    kvo_run *p = &runs[*count - 1];
    if (p->shard_index == (uint32_t)shard &&
        (uint64_t)p->device_byte_offset + p->num_bytes == (uint64_t)dev_off &&
        p->host_byte_offset + p->num_bytes == (uint64_t)host_off &&
        (uint64_t)p->num_bytes + (uint64_t)bytes <= 0xFFFFFFFFull) {
      p->num_bytes += (uint32_t)bytes;
      return KVO_OK;
    }
  }
  if (*count >= cap) return KVO_E_NOSPACE;
  runs[*count].shard_index = (uint32_t)shard;
  runs[*count].device_byte_offset = (uint32_t)dev_off;
  runs[*count].num_bytes = (uint32_t)bytes;
  runs[*count].host_byte_offset = (uint64_t)host_off;
  ++*count;
  return KVO_OK;
}

/* build_tp_interleaved_region_raw_mesh_runs, P2:1545-1660. */
int kvo_plan_tp_interleaved_runs(const int64_t *slots, uint64_t n_slots, const int64_t *starts,
                                 const int64_t *ends, const int64_t *memobj_slots,
                                 uint64_t n_chunks, const int64_t *member_alloc_bytes,
                                 const int64_t *region_bases, uint64_t n_members,
                                 int64_t sbb, int64_t block_bytes, int64_t block_size,
                                 int64_t dp_size, int64_t blocks_per_dp, int64_t tp_size,
                                 kvo_run *runs_out, uint64_t runs_cap, uint64_t *counts_out) {
  if (n_chunks == 0 || n_members == 0) return fail(KVO_E_INVAL, "empty chunks or members");
  if (sbb <= 0 || block_bytes <= 0 || block_size <= 0 || dp_size <= 0 || blocks_per_dp <= 0 ||
      tp_size <= 0 || block_bytes != sbb * tp_size)
    return fail(KVO_E_INVAL, "invalid geometry");
  for (uint64_t m = 0; m < n_members; ++m) {
    counts_out[m] = 0;
    if (member_alloc_bytes[m] <= 0 || member_alloc_bytes[m] % block_bytes != 0)
      return fail(KVO_E_INVAL, "member alloc bytes not a multiple of block bytes");
  }
  const int64_t num_device_tensors = dp_size * tp_size;
  int64_t *blocks = (int64_t *)malloc(sizeof(int64_t) * (n_slots ? n_slots : 1));
  int rc = KVO_OK;
  for (uint64_t c = 0; c < n_chunks && rc == KVO_OK; ++c) {
    int64_t start = starts[c], end = ends[c];
    if (start < 0 || end < start || (uint64_t)end > n_slots) {
      rc = fail(KVO_E_INVAL, "chunk range out of bounds");
      break;
    }
    int64_t logical = end - start;
    if (logical == 0) continue;
    int64_t first = slots[start];
    if (first < 0 || first % block_size != 0) {
      rc = fail(KVO_E_INVAL, "chunk does not start on a block boundary");
      break;
    }
    uint64_t nb = 0;
    for (int64_t pos = 0; pos < logical; ++pos) {
      int64_t slot = slots[start + pos];
      if (slot < 0) {
        rc = fail(KVO_E_INVAL, "negative slot");
        break;
      }
      int64_t block = slot / block_size, intra = slot % block_size;
      if (intra != pos % block_size) {
        rc = fail(KVO_E_INVAL, "slot not aligned with its chunk position");
        break;
      }
      if (intra == 0)
        blocks[nb++] = block;
      else if (nb == 0 || blocks[nb - 1] != block) {
        rc = fail(KVO_E_INVAL, "slots leave their block mid-block");
        break;
      }
    }
    if (rc) break;
    for (uint64_t m = 0; m < n_members; ++m)
      if ((int64_t)nb > member_alloc_bytes[m] / block_bytes) {
        rc = fail(KVO_E_INVAL, "chunk has more blocks than the member allocation holds");
        break;
      }
    if (rc) break;
    for (uint64_t cb = 0; cb < nb && rc == KVO_OK; ++cb) {
      int64_t block = blocks[cb];
      int64_t dp = block / blocks_per_dp;
      int64_t local = block - dp * blocks_per_dp;
      if (dp < 0 || dp >= dp_size || local < 0 || local >= blocks_per_dp) {
        rc = fail(KVO_E_INVAL, "block outside the DP groups");
        break;
      }
      for (int64_t r = 0; r < tp_size && rc == KVO_OK; ++r) {
        int64_t shard = dp * tp_size + r;
        if (shard < 0 || shard >= num_device_tensors) {
          rc = fail(KVO_E_INVAL, "shard index out of range");
          break;
        }
        for (uint64_t m = 0; m < n_members; ++m) {
          int64_t host_off = region_bases[m] + memobj_slots[c] * member_alloc_bytes[m] +
                             (int64_t)cb * block_bytes + r * sbb;
          int a = append_run(runs_out + m * runs_cap, &counts_out[m], runs_cap, shard,
                             local * sbb, sbb, host_off);
          if (a == KVO_E_NOSPACE) {
            rc = fail(KVO_E_NOSPACE, "runs_cap too small");
            break;
          }
          if (a) {
            rc = fail(KVO_E_INVAL, "run does not fit the uint32 planner ABI");
            break;
          }
        }
      }
    }
  }
  free(blocks);
  return rc;
}

/* gather_region_raw_runs_to_torch / scatter_region_raw_runs_from_torch, P2:1846-1995: one
 * copy per run between a shard's bytes and the host blob. */
void kvo_apply_runs(const kvo_run *runs, uint64_t n_runs, uint8_t *const *shard_ptrs,
                    uint8_t *host, int to_host) {
  for (uint64_t i = 0; i < n_runs; ++i) {
    uint8_t *dev = shard_ptrs[runs[i].shard_index] + runs[i].device_byte_offset;
    uint8_t *h = host + runs[i].host_byte_offset;
    if (to_host)
      memcpy(h, dev, runs[i].num_bytes);
    else
      memcpy(dev, h, runs[i].num_bytes);
  }
}

/* ------------------------------------------------------------------------------------------ */
/* the store                                                                                  */
/* ------------------------------------------------------------------------------------------ */

/* Directory entry, layout.hpp P3:6352-6363 (value offset widened to 64 bits). */
typedef struct {
  uint32_t valid, key_len, total_len_lo, last_access;
  uint64_t value_off;
  uint32_t host_gen, location, order;
  uint64_t total_len;
  uint8_t key[KVO_MAX_KEY_BYTES];
} dir_entry;

typedef struct {
  uint32_t state, order, next, prev;
} heap_meta;

/* Host backing: server_impl.hpp HostValue {len, lease|bytes}; pool extents first-fit. */
typedef struct {
  int present;
  uint64_t len;
  int in_pool;
  uint64_t pool_unit, pool_units;
  uint8_t *heap;
} host_value;

typedef struct free_extent {
  uint64_t unit, units;
  struct free_extent *next; /* address ordered */
} free_extent;

typedef struct {
  uint32_t slot, token;
} fifo_item;

typedef struct {
  const uint8_t *src;
  uint8_t *dst;
  uint64_t len;
} copy_desc;

struct kvo_store {
  kvo_config cfg;
  uint32_t nb; /* buckets */
  uint32_t *buckets; /* nb pairs {hash, slot} */
  dir_entry *dir;
  /* catalog free slots, P3:10373-10413 */
  uint32_t next_unused, free_head;
  uint32_t *free_next;  /* intrusive free-slot list */
  uint8_t *free_queued;
  /* residency LRU, P3:10306-10372: head = MRU, tail = LRU */
  uint32_t *lru_prev, *lru_next;
  uint32_t lru_head, lru_tail, lru_count;
  /* buddy heap, P3:10078-10210 */
  uint8_t *heap;
  uint32_t num_units, max_order;
  heap_meta *hm;
  uint32_t free_head_by_order[KVO_MAX_ORDERS];
  uint64_t live_device_bytes, pending_device_bytes;
  uint32_t epoch;
  /* pending-host FIFO, P3:6322-6327 */
  fifo_item *fifo;
  uint32_t fifo_head, fifo_count;
  uint32_t next_token;
  uint32_t host_gen_counter;
  /* host tier */
  host_value *hv;
  uint8_t *pool;
  uint64_t pool_units_total;
  free_extent *pool_free;
  /* deferred copies (batched CPU baseline) */
  copy_desc *copies;
  uint64_t n_copies, copies_cap;
  int n_threads;
  kvo_stats st;
};

/* --- hash index: lookup / insert / backward-shift delete, P3:9923-10057 --- */

static int key_eq(const dir_entry *e, const uint8_t *key, uint32_t len) {
  return e->valid == 1 && e->key_len == len && memcmp(e->key, key, len) == 0;
}

static uint32_t idx_lookup(kvo_store *s, uint32_t h, const uint8_t *key, uint32_t len) {
  uint32_t mask = s->nb - 1, idx = h & mask;
  for (uint32_t probe = 0; probe < s->nb; ++probe) {
    uint32_t slot = s->buckets[2 * idx + 1];
    if (slot == KVO_BUCKET_EMPTY) return KVO_BUCKET_EMPTY;
    if (slot != KVO_BUCKET_TOMBSTONE && s->buckets[2 * idx] == h && key_eq(&s->dir[slot], key, len))
      return slot;
    idx = (idx + 1) & mask;
  }
  return KVO_BUCKET_EMPTY;
}

static void idx_insert(kvo_store *s, uint32_t h, uint32_t slot) {
  uint32_t mask = s->nb - 1, idx = h & mask;
  for (uint32_t probe = 0; probe < s->nb; ++probe) {
    uint32_t cur = s->buckets[2 * idx + 1];
    if (cur == KVO_BUCKET_EMPTY || cur == KVO_BUCKET_TOMBSTONE) {
      s->buckets[2 * idx] = h;
      s->buckets[2 * idx + 1] = slot;
      return;
    }
    idx = (idx + 1) & mask;
  }
  abort(); /* load factor <= 0.5 makes this unreachable */
}

static void idx_delete(kvo_store *s, uint32_t h, uint32_t target) {
  uint32_t mask = s->nb - 1, hole = h & mask;
  int found = 0;
  for (uint32_t probe = 0; probe < s->nb; ++probe) {
    uint32_t cur = s->buckets[2 * hole + 1];
    if (cur == KVO_BUCKET_EMPTY) return;
    if (cur == target && s->buckets[2 * hole] == h) {
      found = 1;
      break;
    }
    hole = (hole + 1) & mask;
  }
  if (!found) return;
  /* Knuth Alg. R: entry j moves into the hole unless its home lies cyclically in (hole, j]. */
  uint32_t j = hole;
  for (uint32_t scanned = 0; scanned < s->nb; ++scanned) {
    j = (j + 1) & mask;
    if (s->buckets[2 * j + 1] == KVO_BUCKET_EMPTY) break;
    uint32_t home = s->buckets[2 * j] & mask;
    int can_move = (hole <= j) ? (home <= hole || home > j) : (home <= hole && home > j);
    if (can_move) {
      s->buckets[2 * hole] = s->buckets[2 * j];
      s->buckets[2 * hole + 1] = s->buckets[2 * j + 1];
      hole = j;
    }
  }
  s->buckets[2 * hole + 1] = KVO_BUCKET_EMPTY;
}

/* --- buddy heap, P3:10078-10210 --- */

static void buddy_remove_free(kvo_store *s, uint32_t unit, uint32_t order) {
  heap_meta *b = &s->hm[unit];
  uint32_t next = b->next, prev = b->prev;
  if (prev == KVO_NONE)
    s->free_head_by_order[order] = next;
  else
    s->hm[prev].next = next;
  if (next != KVO_NONE) s->hm[next].prev = prev;
  b->state = KVO_HEAP_CONT;
  b->order = order;
  b->next = b->prev = KVO_NONE;
}

static void buddy_push_free(kvo_store *s, uint32_t unit, uint32_t order) {
  uint32_t old = s->free_head_by_order[order];
  s->hm[unit].state = KVO_HEAP_FREE;
  s->hm[unit].order = order;
  s->hm[unit].next = old;
  s->hm[unit].prev = KVO_NONE;
  if (old != KVO_NONE) s->hm[old].prev = unit;
  s->free_head_by_order[order] = unit;
}

static int buddy_allocate(kvo_store *s, uint32_t units, uint32_t owner, uint32_t *out_unit,
                          uint32_t *out_order) {
  uint32_t need = kvo_buddy_order_for_units(units);
  uint32_t order = need;
  while (order <= s->max_order && s->free_head_by_order[order] == KVO_NONE) ++order;
  if (order > s->max_order) return 0;
  uint32_t unit = s->free_head_by_order[order];
  buddy_remove_free(s, unit, order);
  while (order > need) {
    --order;
    buddy_push_free(s, unit + (1u << order), order);
  }
  s->hm[unit].state = owner;
  s->hm[unit].order = need;
  s->hm[unit].next = s->hm[unit].prev = KVO_NONE;
  *out_unit = unit;
  *out_order = need;
  return 1;
}

static void buddy_free(kvo_store *s, uint32_t unit, uint32_t order) {
  while (order < s->max_order) {
    uint32_t buddy = unit ^ (1u << order);
    if (buddy >= s->num_units) break;
    if (s->hm[buddy].state != KVO_HEAP_FREE || s->hm[buddy].order != order) break;
    buddy_remove_free(s, buddy, order);
    unit = buddy < unit ? buddy : unit;
    ++order;
  }
  buddy_push_free(s, unit, order);
}

/* --- residency LRU, P3:10306-10372 --- */

static void lru_remove(kvo_store *s, uint32_t slot) {
  uint32_t prev = s->lru_prev[slot], next = s->lru_next[slot];
  if (prev == KVO_NONE)
    s->lru_head = next;
  else
    s->lru_next[prev] = next;
  if (next == KVO_NONE)
    s->lru_tail = prev;
  else
    s->lru_prev[next] = prev;
  s->lru_prev[slot] = s->lru_next[slot] = KVO_NONE;
  --s->lru_count;
}

static void lru_insert_mru(kvo_store *s, uint32_t slot) {
  uint32_t old = s->lru_head;
  s->lru_prev[slot] = KVO_NONE;
  s->lru_next[slot] = old;
  if (old == KVO_NONE)
    s->lru_tail = slot;
  else
    s->lru_prev[old] = slot;
  s->lru_head = slot;
  ++s->lru_count;
}

static void lru_touch(kvo_store *s, uint32_t slot) {
  if (s->lru_head == slot) return;
  lru_remove(s, slot);
  lru_insert_mru(s, slot);
}

/* --- catalog slots, P3:10373-10413 --- */

static uint32_t catalog_claim(kvo_store *s) {
  if (s->free_head != KVO_NONE) {
    uint32_t slot = s->free_head;
    s->free_head = s->free_next[slot];
    s->free_queued[slot] = 0;
    return slot;
  }
  if (s->next_unused == s->cfg.max_keys) return KVO_BUCKET_EMPTY;
  return s->next_unused++;
}

static void catalog_release(kvo_store *s, uint32_t slot) {
  s->free_next[slot] = s->free_head;
  s->free_queued[slot] = 1;
  s->free_head = slot;
}

/* --- host tier: first-fit pool with coalescing, server_storage.cpp:66-116 --- */

static int pool_alloc(kvo_store *s, uint64_t units, uint64_t *unit_out) {
  if (s->pool == NULL || units == 0) return 0;
  free_extent **pp = &s->pool_free;
  while (*pp) {
    free_extent *e = *pp;
    if (e->units >= units) {
      *unit_out = e->unit;
      if (e->units == units) {
        *pp = e->next;
        free(e);
      } else {
        e->unit += units;
        e->units -= units;
      }
      return 1;
    }
    pp = &e->next;
  }
  return 0;
}

static void pool_release(kvo_store *s, uint64_t unit, uint64_t units) {
  if (units == 0) return;
  free_extent *prev = NULL, *cur = s->pool_free;
  while (cur && cur->unit < unit) {
    prev = cur;
    cur = cur->next;
  }
  if (cur && cur->unit == unit + units) { /* merge with the following extent */
    cur->unit = unit;
    cur->units += units;
    if (prev && prev->unit + prev->units == cur->unit) {
      prev->units += cur->units;
      prev->next = cur->next;
      free(cur);
    }
    return;
  }
  if (prev && prev->unit + prev->units == unit) {
    prev->units += units;
    return;
  }
  free_extent *e = (free_extent *)malloc(sizeof *e);
  e->unit = unit;
  e->units = units;
  e->next = cur;
  if (prev)
    prev->next = e;
  else
    s->pool_free = e;
}

static void host_drop(kvo_store *s, uint32_t slot) {
  host_value *h = &s->hv[slot];
  if (!h->present) return;
  if (h->in_pool)
    pool_release(s, h->pool_unit, h->pool_units);
  else
    free(h->heap);
  memset(h, 0, sizeof *h);
}

static uint8_t *host_bytes(kvo_store *s, uint32_t slot) {
  host_value *h = &s->hv[slot];
  return h->in_pool ? s->pool + h->pool_unit * s->cfg.unit_bytes : h->heap;
}

/* --- deferred (parallel) copies for the batched CPU baseline --- */

typedef struct {
  copy_desc *d;
  uint64_t n;
  uint64_t lo, hi; /* byte range of the flattened copy list */
} copy_task;

static void run_copy_range(copy_desc *d, uint64_t n, uint64_t lo, uint64_t hi) {
  uint64_t base = 0;
  for (uint64_t i = 0; i < n && base < hi; ++i) {
    uint64_t a = base, b = base + d[i].len;
    base = b;
    if (b <= lo) continue;
    uint64_t s0 = a < lo ? lo - a : 0, s1 = (b > hi ? hi : b) - a;
    memcpy(d[i].dst + s0, d[i].src + s0, s1 - s0);
  }
}

static void *copy_worker(void *arg) {
  copy_task *t = (copy_task *)arg;
  run_copy_range(t->d, t->n, t->lo, t->hi);
  return NULL;
}

static void flush_copies(kvo_store *s) {
  if (s->n_copies == 0) return;
  uint64_t total = 0;
  for (uint64_t i = 0; i < s->n_copies; ++i) total += s->copies[i].len;
  int nt = s->n_threads > 1 ? s->n_threads : 1;
  if (nt == 1 || total < (1u << 20)) {
    run_copy_range(s->copies, s->n_copies, 0, total);
  } else {
    pthread_t th[256];
    copy_task tk[256];
    if (nt > 256) nt = 256;
    uint64_t per = (total + nt - 1) / nt;
    per = (per + 4095) & ~4095ull;
    int launched = 0;
    for (int t = 0; t < nt; ++t) {
      uint64_t lo = (uint64_t)t * per, hi = lo + per > total ? total : lo + per;
      if (lo >= total) break;
      tk[t] = (copy_task){s->copies, s->n_copies, lo, hi};
      pthread_create(&th[t], NULL, copy_worker, &tk[t]);
      ++launched;
    }
    for (int t = 0; t < launched; ++t) pthread_join(th[t], NULL);
  }
  s->n_copies = 0;
}

static void copy_bytes(kvo_store *s, uint8_t *dst, const uint8_t *src, uint64_t len) {
  if (s->n_threads <= 0) { /* immediate mode (single-value API) */
    memcpy(dst, src, len);
    return;
  }
  if (s->n_copies == s->copies_cap) {
    s->copies_cap = s->copies_cap ? 2 * s->copies_cap : 1024;
    s->copies = (copy_desc *)realloc(s->copies, s->copies_cap * sizeof(copy_desc));
  }
  s->copies[s->n_copies++] = (copy_desc){src, dst, len};
}

/* --- allocation with LRU eviction, P3:10418-10543 --- */

static uint64_t block_bytes_of(kvo_store *s, uint32_t order) {
  return (uint64_t)s->cfg.unit_bytes << order;
}

static int find_oldest_device_victim(kvo_store *s, uint32_t *out) {
  uint32_t slot = s->lru_tail;
  for (uint32_t v = 0; slot != KVO_NONE && v < s->lru_count; ++v) {
    if (s->dir[slot].valid == 1 && s->dir[slot].location == KVO_LOC_DEVICE) {
      *out = slot;
      return 1;
    }
    slot = s->lru_prev[slot];
  }
  return 0;
}

static int evict_cached_block(kvo_store *s, uint32_t slot) {
  dir_entry *e = &s->dir[slot];
  if (e->valid != 1 || e->location != KVO_LOC_DEVICE) return 0;
  uint64_t bb = block_bytes_of(s, e->order);
  e->location = KVO_LOC_HOST;
  lru_remove(s, slot);
  buddy_free(s, (uint32_t)(e->value_off / s->cfg.unit_bytes), e->order);
  s->live_device_bytes = s->live_device_bytes >= bb ? s->live_device_bytes - bb : 0;
  return 1;
}

static int allocate_cache_block(kvo_store *s, uint64_t units, uint32_t owner, int allow_eviction,
                                uint32_t *out_unit, uint32_t *out_order) {
  s->st.allocation_calls++;
  if (units == 0 || units > s->num_units) {
    s->st.allocation_failures++;
    return 0;
  }
  uint64_t bb = block_bytes_of(s, kvo_buddy_order_for_units((uint32_t)units));
  if (bb > s->cfg.heap_bytes) {
    s->st.allocation_failures++;
    return 0;
  }
  for (uint32_t attempts = 0; attempts <= s->cfg.max_keys; ++attempts) {
    if (s->live_device_bytes <= s->cfg.heap_bytes - bb &&
        buddy_allocate(s, (uint32_t)units, owner, out_unit, out_order)) {
      s->st.allocation_successes++;
      return 1;
    }
    if (!allow_eviction || attempts == s->cfg.max_keys) break;
    uint32_t victim;
    if (!find_oldest_device_victim(s, &victim)) break;
    if (!evict_cached_block(s, victim)) break;
    s->st.victims_evicted++;
  }
  s->st.allocation_failures++;
  return 0;
}

/* --- write-through commit, P3:10747-10806 + server_tiering.cpp:36-64 --- */

static void write_through(kvo_store *s, uint32_t slot) {
  dir_entry *e = &s->dir[slot];
  host_drop(s, slot);
  host_value *h = &s->hv[slot];
  uint64_t units = kvo_chunk_count(e->total_len, s->cfg.unit_bytes);
  uint64_t unit;
  h->present = 1;
  h->len = e->total_len;
  if (pool_alloc(s, units, &unit)) {
    h->in_pool = 1;
    h->pool_unit = unit;
    h->pool_units = units;
    s->st.pool_values++;
  } else {
    h->in_pool = 0;
    h->heap = (uint8_t *)malloc(e->total_len);
    s->st.heap_values++;
  }
  copy_bytes(s, host_bytes(s, slot), s->heap + e->value_off, e->total_len);
  s->st.writes_through++;
}

/* commit_pending_put: stale tokens are consumed without creating host backing. */
static void commit_fifo_head(kvo_store *s) {
  fifo_item it = s->fifo[s->fifo_head];
  s->fifo_head = (s->fifo_head + 1) % s->cfg.max_keys;
  s->fifo_count--;
  s->st.committed++;
  dir_entry *e = &s->dir[it.slot];
  if (e->valid != 1 || e->location != KVO_LOC_PENDING || e->host_gen != it.token) {
    s->st.stale_commits++;
    return;
  }
  write_through(s, it.slot);
  uint32_t g = ++s->host_gen_counter;
  if (g == 0) g = ++s->host_gen_counter;
  e->host_gen = g;
  e->location = KVO_LOC_DEVICE;
  s->pending_device_bytes -= block_bytes_of(s, e->order);
}

/* COMMIT_BARRIER: wait until every issued PUT is host-committed (P3:2519-2531). */
static void commit_barrier(kvo_store *s) {
  flush_copies(s); /* landed data first */
  while (s->fifo_count) commit_fifo_head(s);
  flush_copies(s);
}

static int validate_key(kvo_store *s, const uint8_t *key, uint32_t len, const char *op) {
  (void)key;
  if (len == 0) return fail(KVO_E_INVAL, "%s: key must be non-empty", op);
  if (len > s->cfg.max_key_bytes)
    return fail(KVO_E_INVAL, "%s: key size %u exceeds Server max_key_bytes %u", op, len,
                s->cfg.max_key_bytes);
  return KVO_OK;
}

/* Zeroes a large arena with up to 16 threads, so its pages are faulted in before any timed use
 * (one thread faults in about 1 GB/s: a 15 GB store took 15 s). */
typedef struct {
  uint8_t *p;
  size_t n;
} zero_task;

static void *zero_worker(void *arg) {
  zero_task *t = (zero_task *)arg;
  memset(t->p, 0, t->n);
  return NULL;
}

static void parallel_zero(uint8_t *p, size_t bytes) {
  long ncpu = sysconf(_SC_NPROCESSORS_ONLN);
  int nt = bytes < (256u << 20) ? 1 : (int)(ncpu < 1 ? 1 : ncpu > 16 ? 16 : ncpu);
  pthread_t th[16];
  zero_task tk[16];
  const size_t per = (bytes + nt - 1) / nt;
  int launched = 0;
  for (int t = 0; t < nt; ++t) {
    const size_t lo = (size_t)t * per;
    if (lo >= bytes) break;
    tk[t].p = p + lo;
    tk[t].n = bytes - lo < per ? bytes - lo : per;
    if (t == nt - 1 || pthread_create(&th[t], NULL, zero_worker, &tk[t]) != 0)
      zero_worker(&tk[t]); /* the last piece (or one whose thread could not start) on this thread */
    else
      ++launched;
  }
  for (int t = 0; t < launched; ++t) pthread_join(th[t], NULL);
}

kvo_store *kvo_store_create(const kvo_config *cfg) {
  if (cfg->max_keys == 0 || cfg->unit_bytes == 0 || cfg->max_key_bytes == 0 ||
      cfg->max_key_bytes > KVO_MAX_KEY_BYTES || cfg->heap_bytes < cfg->unit_bytes) {
    fail(KVO_E_INVAL, "invalid store config");
    return NULL;
  }
  kvo_store *s = (kvo_store *)calloc(1, sizeof *s);
  s->cfg = *cfg;
  s->nb = kvo_hash_num_buckets(cfg->max_keys);
  s->buckets = (uint32_t *)malloc(8ull * s->nb);
  for (uint32_t b = 0; b < s->nb; ++b) {
    s->buckets[2 * b] = 0;
    s->buckets[2 * b + 1] = KVO_BUCKET_EMPTY;
  }
  s->dir = (dir_entry *)calloc(cfg->max_keys, sizeof(dir_entry));
  s->free_next = (uint32_t *)malloc(4ull * cfg->max_keys);
  s->free_queued = (uint8_t *)calloc(cfg->max_keys, 1);
  s->lru_prev = (uint32_t *)malloc(4ull * cfg->max_keys);
  s->lru_next = (uint32_t *)malloc(4ull * cfg->max_keys);
  for (uint32_t i = 0; i < cfg->max_keys; ++i) s->lru_prev[i] = s->lru_next[i] = KVO_NONE;
  s->lru_head = s->lru_tail = KVO_NONE;
  s->free_head = KVO_NONE;
  s->heap = (uint8_t *)malloc(cfg->heap_bytes);
  parallel_zero(s->heap, cfg->heap_bytes); /* fault the heap in up front, like a reserved arena */
  uint64_t nu = cfg->heap_bytes / cfg->unit_bytes;
  s->num_units = nu > 0xFFFFFFF0ull ? 0xFFFFFFF0u : (uint32_t)nu;
  s->max_order = kvo_floor_log2(s->num_units);
  s->hm = (heap_meta *)malloc(sizeof(heap_meta) * s->num_units);
  for (uint32_t o = 0; o < KVO_MAX_ORDERS; ++o) s->free_head_by_order[o] = KVO_NONE;
  /* seed aligned power-of-two free blocks, P3:11163-11180 */
  uint32_t first = 0, remaining = s->num_units;
  while (remaining) {
    uint32_t order = kvo_floor_log2(remaining);
    while (order != 0 && (first & ((1u << order) - 1u)) != 0) --order;
    buddy_push_free(s, first, order);
    first += 1u << order;
    remaining -= 1u << order;
  }
  s->fifo = (fifo_item *)malloc(sizeof(fifo_item) * cfg->max_keys);
  s->next_token = 1;
  s->hv = (host_value *)calloc(cfg->max_keys, sizeof(host_value));
  s->pool_units_total = cfg->host_pool_bytes / cfg->unit_bytes;
  if (s->pool_units_total) {
    s->pool = (uint8_t *)malloc(s->pool_units_total * cfg->unit_bytes);
    parallel_zero(s->pool, s->pool_units_total * cfg->unit_bytes);
    s->pool_free = (free_extent *)malloc(sizeof(free_extent));
    s->pool_free->unit = 0;
    s->pool_free->units = s->pool_units_total;
    s->pool_free->next = NULL;
  }
  return s;
}

void kvo_store_destroy(kvo_store *s) {
  if (!s) return;
  for (uint32_t i = 0; i < s->cfg.max_keys; ++i)
    if (s->hv[i].present && !s->hv[i].in_pool) free(s->hv[i].heap);
  while (s->pool_free) {
    free_extent *n = s->pool_free->next;
    free(s->pool_free);
    s->pool_free = n;
  }
  free(s->pool);
  free(s->hv);
  free(s->fifo);
  free(s->hm);
  free(s->heap);
  free(s->lru_prev);
  free(s->lru_next);
  free(s->free_next);
  free(s->free_queued);
  free(s->dir);
  free(s->buckets);
  free(s->copies);
  free(s);
}

/* PUT prepare + publish, P3:11440-11700 (selection, replacement, allocation) and
 * publish_pending_put P3:10681-10745. The speculative next-PUT lease of the Fabric wire
 * protocol is not modelled (it exists to overlap a Fabric grant round trip). When a pending
 * entry blocks the put (same key pending, or no evictable space), the FIFO head is committed
 * and the prepare retried, as force_put_host_commit does. The value bytes are copied from
 * `src` (or deferred into the parallel copy list). */
static int put_one(kvo_store *s, const uint8_t *key, uint32_t key_len, const uint8_t *src,
                   uint64_t len) {
  int rc = validate_key(s, key, key_len, "put");
  if (rc) return rc;
  if (len == 0) return fail(KVO_E_INVAL, "put: value_len_bytes must be > 0");
  if (len > s->cfg.max_value_bytes)
    return fail(KVO_E_INVAL, "put: value_len_bytes %llu exceeds max_value_bytes %llu",
                (unsigned long long)len, (unsigned long long)s->cfg.max_value_bytes);
  uint64_t units = kvo_chunk_count(len, s->cfg.unit_bytes);
  if (units > s->num_units)
    return fail(KVO_E_NOSPACE, "put: value of %llu B does not fit the value heap",
                (unsigned long long)len);
  uint32_t h = kvo_fnv1a32(key, key_len);
  for (;;) {
    int retry = 0;
    uint32_t slot = idx_lookup(s, h, key, key_len);
    if (slot != KVO_BUCKET_EMPTY) retry = s->dir[slot].location == KVO_LOC_PENDING;
    if (!retry && slot == KVO_BUCKET_EMPTY) slot = catalog_claim(s);
    if (!retry && slot == KVO_BUCKET_EMPTY) {
      /* catalog LRU replacement: oldest last_access among valid, non-pending entries */
      uint32_t oldest = 0, oldest_age = 0;
      int have = 0;
      for (uint32_t i = 0; i < s->cfg.max_keys; ++i) {
        dir_entry *e = &s->dir[i];
        if (e->valid != 1 || e->location == KVO_LOC_PENDING) continue;
        uint32_t age = s->epoch - e->last_access;
        if (!have || age > oldest_age) {
          have = 1;
          oldest_age = age;
          oldest = i;
        }
      }
      if (have) {
        slot = oldest;
        s->st.catalog_replacements++;
      } else
        retry = 1;
    }
    if (!retry) {
      dir_entry *old = &s->dir[slot];
      if (old->valid == 1) {
        idx_delete(s, kvo_fnv1a32(old->key, old->key_len), slot);
        if (old->location == KVO_LOC_DEVICE) {
          lru_remove(s, slot);
          uint64_t bb = block_bytes_of(s, old->order);
          buddy_free(s, (uint32_t)(old->value_off / s->cfg.unit_bytes), old->order);
          s->live_device_bytes = s->live_device_bytes >= bb ? s->live_device_bytes - bb : 0;
        }
        old->valid = 0;
        host_drop(s, slot);
      }
      uint32_t unit, order;
      if (allocate_cache_block(s, units, slot, 1, &unit, &order)) {
        dir_entry *e = &s->dir[slot];
        memset(e, 0, sizeof *e);
        uint32_t token = s->next_token++;
        if (s->next_token == 0) s->next_token = 1;
        e->valid = 1;
        e->key_len = key_len;
        e->total_len = len;
        e->total_len_lo = (uint32_t)len;
        e->last_access = ++s->epoch;
        e->value_off = (uint64_t)unit * s->cfg.unit_bytes;
        e->host_gen = token;
        e->location = KVO_LOC_PENDING;
        e->order = order;
        memcpy(e->key, key, key_len);
        copy_bytes(s, s->heap + e->value_off, src, len);
        idx_insert(s, h, slot);
        lru_insert_mru(s, slot);
        uint64_t bb = block_bytes_of(s, order);
        s->live_device_bytes += bb;
        s->pending_device_bytes += bb;
        s->fifo[(s->fifo_head + s->fifo_count) % s->cfg.max_keys] = (fifo_item){slot, token};
        s->fifo_count++;
        s->st.issued++;
        return KVO_OK;
      }
      catalog_release(s, slot);
      retry = 1;
    }
    if (!s->fifo_count)
      return fail(KVO_E_NOSPACE, "put: no device-cache space for a %llu B value",
                  (unsigned long long)len);
    flush_copies(s);
    commit_fifo_head(s); /* force_put_host_commit, then retry the prepare */
    /* force_put_host_commit returns after the head's host copy has landed: the retry may evict
     * the value just committed and hand its block to this put */
    flush_copies(s);
  }
}

int kvo_put(kvo_store *s, const uint8_t *key, uint32_t key_len, const uint8_t *value,
            uint64_t len, int sync_commit) {
  int rc = put_one(s, key, key_len, value, len);
  if (rc) return rc;
  if (sync_commit) commit_barrier(s);
  return KVO_OK;
}

/* GET, P3:2786-2891 (client) and the directory GET path P3:11756-12060: commit barrier,
 * lookup, output-size check before any stamp, epoch stamp, device hit -> LRU touch; host hit ->
 * read-through admission when a block can be allocated, else serve from host. A miss leaves
 * the output untouched. */
static int get_one(kvo_store *s, const uint8_t *key, uint32_t key_len, uint8_t *out,
                   uint64_t capacity, int *found, uint64_t *value_len, int deferred) {
  *found = 0;
  uint32_t slot = idx_lookup(s, kvo_fnv1a32(key, key_len), key, key_len);
  if (slot == KVO_BUCKET_EMPTY) return KVO_OK;
  dir_entry *e = &s->dir[slot];
  if (value_len) *value_len = e->total_len;
  if (e->total_len > capacity)
    return fail(KVO_E_TOO_SMALL, "get: out_tensor packed capacity %llu is smaller than the stored value",
                (unsigned long long)capacity);
  uint32_t epoch = ++s->epoch;
  if (e->location != KVO_LOC_HOST) {
    copy_bytes(s, out, s->heap + e->value_off, e->total_len);
    e->last_access = epoch;
    lru_touch(s, slot);
  } else {
    uint32_t unit, order;
    if (deferred) flush_copies(s); /* eviction may reuse a block an earlier copy reads */
    if (allocate_cache_block(s, kvo_chunk_count(e->total_len, s->cfg.unit_bytes), slot, 1, &unit,
                             &order)) {
      e->value_off = (uint64_t)unit * s->cfg.unit_bytes;
      e->location = KVO_LOC_DEVICE;
      e->order = order;
      e->last_access = epoch;
      lru_insert_mru(s, slot);
      s->live_device_bytes += block_bytes_of(s, order);
      copy_bytes(s, s->heap + e->value_off, host_bytes(s, slot), e->total_len);
      s->st.admissions++;
    } else {
      e->last_access = epoch;
    }
    copy_bytes(s, out, host_bytes(s, slot), e->total_len);
    s->st.host_serves++;
  }
  *found = 1;
  return KVO_OK;
}

int kvo_get(kvo_store *s, const uint8_t *key, uint32_t key_len, uint8_t *out, uint64_t capacity,
            int *found, uint64_t *value_len) {
  int rc = validate_key(s, key, key_len, "get");
  if (rc) return rc;
  commit_barrier(s);
  rc = get_one(s, key, key_len, out, capacity, found, value_len, 0);
  flush_copies(s);
  return rc;
}

/* EXISTS fuses the commit wait and does not update recency (P3 design, lines 7612-7619). */
int kvo_exists(kvo_store *s, const uint8_t *key, uint32_t key_len, int *found) {
  int rc = validate_key(s, key, key_len, "exists");
  if (rc) return rc;
  commit_barrier(s);
  *found = idx_lookup(s, kvo_fnv1a32(key, key_len), key, key_len) != KVO_BUCKET_EMPTY;
  return KVO_OK;
}

/* REMOVE, P3:11801-11849: drop the index mapping, free any device block (pending included),
 * clear the entry, recycle the slot, reclaim host backing. */
int kvo_remove(kvo_store *s, const uint8_t *key, uint32_t key_len, int *removed) {
  int rc = validate_key(s, key, key_len, "remove");
  if (rc) return rc;
  commit_barrier(s);
  *removed = 0;
  uint32_t h = kvo_fnv1a32(key, key_len);
  uint32_t slot = idx_lookup(s, h, key, key_len);
  if (slot == KVO_BUCKET_EMPTY) return KVO_OK;
  dir_entry *e = &s->dir[slot];
  idx_delete(s, h, slot);
  if (e->location != KVO_LOC_HOST) {
    lru_remove(s, slot);
    uint64_t bb = block_bytes_of(s, e->order);
    buddy_free(s, (uint32_t)(e->value_off / s->cfg.unit_bytes), e->order);
    s->live_device_bytes = s->live_device_bytes >= bb ? s->live_device_bytes - bb : 0;
    if (e->location == KVO_LOC_PENDING) s->pending_device_bytes -= bb;
  }
  e->valid = 0;
  catalog_release(s, slot);
  host_drop(s, slot);
  *removed = 1;
  return KVO_OK;
}

/* MOVE_TO_HOST: metadata-only eviction of a device-resident entry (P3:11851-11868). */
int kvo_move_to_host(kvo_store *s, const uint8_t *key, uint32_t key_len) {
  int rc = validate_key(s, key, key_len, "move");
  if (rc) return rc;
  commit_barrier(s);
  uint32_t slot = idx_lookup(s, kvo_fnv1a32(key, key_len), key, key_len);
  if (slot != KVO_BUCKET_EMPTY && s->dir[slot].location == KVO_LOC_DEVICE)
    evict_cached_block(s, slot);
  return KVO_OK;
}

/* MOVE_TO_DEVICE: best-effort admission of the authoritative host copy (P3:11869-11905);
 * committed admission updates access recency. */
int kvo_move_to_device(kvo_store *s, const uint8_t *key, uint32_t key_len) {
  int rc = validate_key(s, key, key_len, "move");
  if (rc) return rc;
  commit_barrier(s);
  uint32_t slot = idx_lookup(s, kvo_fnv1a32(key, key_len), key, key_len);
  if (slot == KVO_BUCKET_EMPTY || s->dir[slot].location != KVO_LOC_HOST) return KVO_OK;
  dir_entry *e = &s->dir[slot];
  uint32_t unit, order;
  if (allocate_cache_block(s, kvo_chunk_count(e->total_len, s->cfg.unit_bytes), slot, 1, &unit,
                           &order)) {
    e->value_off = (uint64_t)unit * s->cfg.unit_bytes;
    e->location = KVO_LOC_DEVICE;
    e->order = order;
    e->last_access = ++s->epoch;
    lru_insert_mru(s, slot);
    s->live_device_bytes += block_bytes_of(s, order);
    copy_bytes(s, s->heap + e->value_off, host_bytes(s, slot), e->total_len);
    s->st.admissions++;
  }
  return KVO_OK;
}

int kvo_flush(kvo_store *s) {
  commit_barrier(s);
  return KVO_OK;
}

int kvo_location(kvo_store *s, const uint8_t *key, uint32_t key_len, uint64_t *value_off) {
  uint32_t slot = idx_lookup(s, kvo_fnv1a32(key, key_len), key, key_len);
  if (slot == KVO_BUCKET_EMPTY) return KVO_ABSENT;
  if (value_off) *value_off = s->dir[slot].value_off;
  return (int)s->dir[slot].location;
}

uint32_t kvo_index_lookup(kvo_store *s, const uint8_t *key, uint32_t key_len) {
  return idx_lookup(s, kvo_fnv1a32(key, key_len), key, key_len);
}

const uint32_t *kvo_buckets(kvo_store *s, uint32_t *n_buckets) {
  *n_buckets = s->nb;
  return s->buckets;
}

uint32_t kvo_lru_order(kvo_store *s, uint32_t *out, uint32_t cap) {
  uint32_t n = 0;
  for (uint32_t slot = s->lru_head; slot != KVO_NONE && n < cap; slot = s->lru_next[slot])
    out[n++] = slot;
  return n;
}

void kvo_get_stats(kvo_store *s, kvo_stats *out) {
  kvo_stats st = s->st;
  st.live_device_bytes = s->live_device_bytes;
  st.pending_device_bytes = s->pending_device_bytes;
  st.epoch = s->epoch;
  st.live_keys = 0;
  st.device_resident_keys = 0;
  for (uint32_t i = 0; i < s->cfg.max_keys; ++i)
    if (s->dir[i].valid == 1) {
      st.live_keys++;
      if (s->dir[i].location != KVO_LOC_HOST) st.device_resident_keys++;
    }
  *out = st;
}

/* ------------------------------------------------------------------------------------------ */
/* batched paged-block put / get (CPU baseline of the reference host-DRAM path)               */
/* ------------------------------------------------------------------------------------------ */

/* Value of one block: the one-block chunk blob of RawByteCodec.device_chunk_plan
 * (P5:12284-12306) -- header [MAGIC, n_layers, layer bytes...] padded to 32 B, then every member's
 * block back to back (K0 V0 K1 V1 ...). Extra members per layer (per-block scales) extend the
 * same scheme; each member region starts 16-byte aligned, which is a no-op for K/V blocks. */
uint64_t kvo_block_format(uint32_t n_members, uint32_t members_per_layer, const uint64_t *member_bytes,
                          uint32_t *words, uint32_t words_cap, uint32_t *n_words,
                          uint64_t *region_bases) {
  if (members_per_layer == 0 || n_members % members_per_layer) return 0;
  uint32_t n_layers = n_members / members_per_layer;
  uint32_t nw = (2 + n_layers + 7) / 8 * 8;
  if (nw > words_cap) return 0;
  memset(words, 0, 4ull * nw);
  words[0] = KVO_BLOB_MAGIC;
  words[1] = n_layers;
  uint64_t off = 4ull * nw;
  for (uint32_t m = 0; m < n_members; ++m) {
    uint64_t start = off;
    region_bases[m] = off;
    off = (off + member_bytes[m] + 15) & ~15ull;
    words[2 + m / members_per_layer] += (uint32_t)(off - start);
  }
  *n_words = nw;
  return off;
}

typedef struct {
  uint32_t *words;
  uint32_t nw;
  uint64_t *rb;
  uint64_t value_len;
} block_fmt;

static int make_fmt(uint32_t n_members, uint32_t mpl, const uint64_t *mb, block_fmt *f) {
  f->words = (uint32_t *)malloc(4ull * (n_members + 16));
  f->rb = (uint64_t *)malloc(8ull * n_members);
  f->value_len = kvo_block_format(n_members, mpl, mb, f->words, n_members + 16, &f->nw, f->rb);
  if (!f->value_len) {
    free(f->words);
    free(f->rb);
    return fail(KVO_E_INVAL, "members must be whole layers of members_per_layer");
  }
  return KVO_OK;
}

static void free_fmt(block_fmt *f) {
  free(f->words);
  free(f->rb);
}

int kvo_put_blocks(kvo_store *s, uint8_t *const *members, uint32_t n_members, uint32_t members_per_layer,
                   const uint64_t *member_bytes, const uint64_t *keys, const uint32_t *block_ids,
                   uint32_t n, int n_threads) {
  block_fmt f;
  int rc = make_fmt(n_members, members_per_layer, member_bytes, &f);
  if (rc) return rc;
  s->n_threads = n_threads > 0 ? n_threads : 1;
  for (uint32_t i = 0; i < n && rc == KVO_OK; ++i) {
    uint8_t kb[8];
    memcpy(kb, &keys[i], 8);
    rc = put_one(s, kb, 8, NULL, f.value_len);
    if (rc) break;
    /* put_one queued one copy from NULL: replace it by header + per-member block copies */
    uint8_t *dst = s->copies[--s->n_copies].dst;
    memset(dst, 0, f.value_len);
    memcpy(dst, f.words, 4ull * f.nw);
    for (uint32_t m = 0; m < n_members; ++m)
      copy_bytes(s, dst + f.rb[m], members[m] + (uint64_t)block_ids[i] * member_bytes[m], member_bytes[m]);
  }
  flush_copies(s);
  s->n_threads = 0;
  free_fmt(&f);
  return rc;
}

int kvo_get_blocks(kvo_store *s, uint8_t *const *members, uint32_t n_members, uint32_t members_per_layer,
                   const uint64_t *member_bytes, const uint64_t *keys, const uint32_t *block_ids,
                   uint32_t n, uint8_t *found, int n_threads) {
  block_fmt f;
  int rc = make_fmt(n_members, members_per_layer, member_bytes, &f);
  if (rc) return rc;
  s->n_threads = n_threads > 0 ? n_threads : 1;
  commit_barrier(s);
  for (uint32_t i = 0; i < n && rc == KVO_OK; ++i) {
    uint8_t kb[8];
    memcpy(kb, &keys[i], 8);
    found[i] = 0;
    uint32_t slot = idx_lookup(s, kvo_fnv1a32(kb, 8), kb, 8);
    if (slot == KVO_BUCKET_EMPTY) continue;
    if (s->dir[slot].total_len != f.value_len) {
      rc = fail(KVO_E_INVAL, "get_blocks: stored value length %llu does not match the block layout",
                (unsigned long long)s->dir[slot].total_len);
      break;
    }
    int fnd = 0;
    rc = get_one(s, kb, 8, NULL, f.value_len, &fnd, NULL, 1);
    if (rc) break;
    /* replace the copy into NULL by per-member block copies from the same source; get_one may
     * have flushed the list before an admission, so search all of it */
    for (uint64_t c = 0; c < s->n_copies; ++c) {
      if (s->copies[c].dst != NULL) continue;
      const uint8_t *src = s->copies[c].src;
      s->copies[c] = s->copies[--s->n_copies];
      for (uint32_t m = 0; m < n_members; ++m)
        copy_bytes(s, members[m] + (uint64_t)block_ids[i] * member_bytes[m], src + f.rb[m], member_bytes[m]);
      break;
    }
    found[i] = (uint8_t)fnd;
  }
  flush_copies(s);
  s->n_threads = 0;
  free_fmt(&f);
  return rc;
}

/* --- token-granular paged KV fill: reader_fill_cache_varlen.cpp / writer_fill_cache_varlen.cpp
 * (patch 0002). The valid total is found as the reader does (the last cu entry that is not -1,
 * by bisection over [0, batch]); a token's request as the writer's find_request_idx does (the last
 * i in [0, batch] with cu[i] <= t, unsigned, so -1 padding never matches). --- */
static uint32_t fill_valid_total(const int32_t *cu, uint32_t batch) {
  uint32_t lo = 0, hi = batch;
  while (lo < hi) {
    uint32_t mid = (lo + hi + 1) >> 1;
    if ((uint32_t)cu[mid] != 0xFFFFFFFFu) lo = mid; else hi = mid - 1;
  }
  return (uint32_t)cu[lo];
}

static uint32_t fill_request_of(const int32_t *cu, uint32_t batch, uint32_t t) {
  uint32_t lo = 0, hi = batch;
  while (lo < hi) {
    uint32_t mid = (lo + hi + 1) >> 1;
    if ((uint32_t)cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

int kvo_paged_fill_varlen(const uint8_t *k_fill, const uint8_t *v_fill, uint32_t n_heads, uint32_t total_tokens,
                          uint32_t row_bytes, const int32_t *cu_seqlens, uint32_t batch, const int32_t *page_table,
                          uint32_t max_blocks_per_seq, const int32_t *start_positions, uint8_t *cache_k,
                          uint8_t *cache_v, uint32_t num_blocks, uint32_t block_size, uint64_t *out_of_range) {
  if (!k_fill || !v_fill || !cu_seqlens || !page_table || !start_positions || !cache_k || !cache_v || batch == 0 ||
      block_size == 0 || row_bytes == 0)
    return fail(KVO_E_INVAL, "paged_fill_varlen: invalid arguments");
  uint64_t oor = 0;
  uint32_t limit = fill_valid_total(cu_seqlens, batch);
  if (limit > total_tokens) limit = total_tokens;
  for (uint32_t t = 0; t < limit; ++t) {
    const uint32_t r = fill_request_of(cu_seqlens, batch, t);
    if (r >= batch) { ++oor; continue; }
    const uint32_t pos = t - (uint32_t)cu_seqlens[r] + (uint32_t)start_positions[r];
    const uint32_t vb = pos / block_size;
    if (vb >= max_blocks_per_seq) { ++oor; continue; }
    const int32_t phys = page_table[(uint64_t)r * max_blocks_per_seq + vb];
    if (phys <= 0) continue; /* null block or an unused / padded slot */
    if ((uint32_t)phys >= num_blocks) { ++oor; continue; }
    for (uint32_t h = 0; h < n_heads; ++h) {
      const uint64_t src = ((uint64_t)h * total_tokens + t) * row_bytes;
      const uint64_t dst = (((uint64_t)phys * n_heads + h) * block_size + pos % block_size) * row_bytes;
      memcpy(cache_k + dst, k_fill + src, row_bytes);
      memcpy(cache_v + dst, v_fill + src, row_bytes);
    }
  }
  if (out_of_range) *out_of_range = oor;
  return KVO_OK;
}
