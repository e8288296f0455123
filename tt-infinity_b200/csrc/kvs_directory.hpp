// kvs_directory.hpp -- the authoritative catalog of one store shard, on the host.
//
// The reference keeps this state in server DRAM and mutates it from one BRISC core
// (patch 0003 lines 9581-12412, "dram_worker_kernel"). On B200 the catalog decisions are made
// by this host-side class under the shard mutex, and every change that a device-side reader
// needs (hash buckets, entry location / offset / length, key rows) is recorded so the runtime
// can replay it into the shard's HBM index replica before the next kernel that reads it.
//
// Policies that must match the reference exactly, because they decide which values stay in
// the device cache (each restated from the reference):
//   * FNV-1a-32 open addressing, next_pow2(2 * max_keys) buckets, linear probe, every candidate
//     revalidated against the entry, backward-shift delete (patch 0003 lines 9912-10057);
//   * buddy value heap in `unit_bytes` units with LIFO free lists per order and aligned
//     power-of-two seeding (lines 10059-10210, 11163-11180);
//   * exact residency LRU (MRU insert on publish / admission, touch on device-hit GET); the
//     victim is the oldest *committed* device entry, pending entries are pinned
//     (lines 10306-10372, 10418-10543);
//   * catalog slots: recycled slot stack, then never-used slots, then replacement of the entry
//     with the oldest access epoch that is not pending (lines 10373-10413, 11487-11520);
//   * pending-host FIFO committed in issue order; stale tokens are consumed without backing.
#pragma once

#include <cstdint>
#include <cstring>
#include <deque>
#include <map>
#include <vector>

namespace kvs {

constexpr uint32_t kNone = 0xFFFFFFFFu;
constexpr uint8_t kLocDevice = 0, kLocHost = 1, kLocPending = 2;

struct DirConfig {
  uint32_t max_keys;
  uint32_t unit_bytes;
  uint32_t max_key_bytes;
  uint64_t heap_bytes;
  uint64_t max_value_bytes;
  uint64_t host_pool_units;  // pool size in units (0: no pool)
};

struct Entry {
  uint8_t valid = 0;
  uint8_t location = 0;
  uint8_t key_len = 0;
  uint32_t order = 0;
  uint32_t last_access = 0;
  uint32_t host_gen = 0;  // pending token while pending
  uint64_t value_off = 0;
  uint64_t total_len = 0;
  uint8_t key[128];
};

// Host backing of one committed value: a pool extent or a separately pinned buffer.
struct HostBacking {
  bool present = false;
  bool in_pool = false;
  uint64_t len = 0;
  uint64_t pool_unit = 0, pool_units = 0;
  uint8_t *heap = nullptr;
};

struct PendingPut {
  uint32_t slot, token;
  HostBacking backing;  // reserved at issue so the device->host copy can start at once
  int wt_batch;         // index of the write-through batch whose event covers this copy
};

struct DirStats {
  uint64_t allocation_calls = 0, allocation_successes = 0, allocation_failures = 0;
  uint64_t victim_scans = 0, victims_evicted = 0, catalog_replacements = 0;
  uint64_t writes_through = 0, stale_commits = 0, host_serves = 0, admissions = 0;
  uint64_t pool_values = 0, heap_values = 0;
  uint32_t issued = 0, committed = 0;
};

enum class Prepare { kGranted, kNeedCommit, kNoSpace };

struct Grant {
  uint32_t slot;
  uint32_t order;
  uint32_t token;
  uint64_t value_off;
};

class Directory {
 public:
  explicit Directory(const DirConfig &cfg);

  const DirConfig &config() const { return cfg_; }
  uint32_t num_buckets() const { return nb_; }
  uint32_t hash_of(const uint8_t *key, uint32_t len) const;
  uint32_t lookup(const uint8_t *key, uint32_t len) const;
  const Entry &entry(uint32_t slot) const { return dir_[slot]; }
  uint64_t block_bytes(uint32_t order) const { return (uint64_t)cfg_.unit_bytes << order; }
  uint64_t units_for(uint64_t len) const { return len == 0 ? 0 : 1 + (len - 1) / cfg_.unit_bytes; }

  // PUT prepare + publish. kNeedCommit: a pending entry blocks this put and the FIFO is not
  // empty -- commit the FIFO head and retry. kNoSpace: nothing left to commit.
  Prepare prepare_put(const uint8_t *key, uint32_t len, uint64_t value_len, Grant *out);
  // Pending-host FIFO.
  bool fifo_empty() const { return fifo_.empty(); }
  size_t fifo_size() const { return fifo_.size(); }
  PendingPut &fifo_head() { return fifo_.front(); }
  PendingPut &fifo_back() { return fifo_.back(); }
  std::deque<PendingPut> &fifo() { return fifo_; }
  // Commit the head: install its backing (returns false for a stale token, whose reserved
  // backing is handed back through *released for the caller to free).
  bool commit_head(HostBacking *released);

  // GET processing of a looked-up slot, in batch order. Returns the action taken.
  enum class GetAction { kDevice, kAdmit, kHostOnly };
  GetAction get_hit(uint32_t slot, uint64_t *admit_off);
  void remove(uint32_t slot);
  bool move_to_host(uint32_t slot);
  bool move_to_device(uint32_t slot, uint64_t *admit_off);

  // Host tier.
  HostBacking &backing(uint32_t slot) { return host_[slot]; }
  bool pool_alloc(uint64_t units, uint64_t *unit);
  void pool_release(uint64_t unit, uint64_t units);
  // Backings dropped by replacement / removal since the last call (caller frees heap ones).
  std::vector<HostBacking> take_dropped();

  // Device-replica change tracking.
  std::vector<uint32_t> take_dirty_buckets();
  std::vector<uint32_t> take_dirty_slots();
  std::vector<uint32_t> take_dirty_keys();
  void dirty_counts(size_t *buckets, size_t *slots, size_t *keys) const {
    *buckets = dirty_buckets_.size();
    *slots = dirty_slots_.size();
    *keys = dirty_keys_.size();
  }
  // Slots whose device copy was evicted since the last call.
  std::vector<uint32_t> take_evicted() {
    std::vector<uint32_t> out;
    out.swap(evicted_);
    return out;
  }
  uint64_t bucket_word(uint32_t b) const {
    return ((uint64_t)buckets_[2 * b + 1] << 32) | buckets_[2 * b];
  }
  const uint32_t *bucket_pairs() const { return buckets_.data(); }

  uint32_t lru_order(uint32_t *out, uint32_t cap) const;
  uint32_t lru_size() const { return lru_count_; }
  uint64_t live_device_bytes() const { return live_bytes_; }
  uint64_t pending_device_bytes() const { return pending_bytes_; }
  uint32_t epoch() const { return epoch_; }
  DirStats &stats() { return st_; }
  uint64_t live_keys(uint64_t *device_resident) const;

 private:
  // index
  uint32_t idx_lookup(uint32_t h, const uint8_t *key, uint32_t len) const;
  void idx_insert(uint32_t h, uint32_t slot);
  void idx_delete(uint32_t h, uint32_t slot);
  void set_bucket(uint32_t b, uint32_t hash, uint32_t slot);
  // heap
  void buddy_remove_free(uint32_t unit, uint32_t order);
  void buddy_push_free(uint32_t unit, uint32_t order);
  bool buddy_allocate(uint32_t units, uint32_t owner, uint32_t *unit, uint32_t *order);
  void buddy_free(uint32_t unit, uint32_t order);
  bool allocate_cache_block(uint64_t units, uint32_t owner, uint32_t *unit, uint32_t *order);
  bool evict(uint32_t slot);
  // lru
  void lru_remove(uint32_t slot);
  void lru_insert_mru(uint32_t slot);
  void lru_touch(uint32_t slot);
  // catalog
  uint32_t bump_epoch();
  void rec_unlink(uint32_t slot);
  void rec_touch(uint32_t slot);
  uint32_t oldest_replaceable() const;
  uint32_t catalog_claim();
  void catalog_release(uint32_t slot);
  void drop_backing(uint32_t slot);
  void mark_slot(uint32_t slot);

  DirConfig cfg_;
  uint32_t nb_;
  std::vector<uint32_t> buckets_;  // {hash, slot} pairs
  std::vector<Entry> dir_;
  uint32_t next_unused_ = 0, free_head_ = kNone;
  std::vector<uint32_t> free_next_;
  std::vector<uint32_t> lru_prev_, lru_next_;
  uint32_t lru_head_ = kNone, lru_tail_ = kNone, lru_count_ = 0;
  uint32_t num_units_, max_order_;
  struct HeapMeta {
    uint32_t state, order, next, prev;
  };
  std::vector<HeapMeta> hm_;
  uint32_t free_heads_[32];
  uint64_t live_bytes_ = 0, pending_bytes_ = 0;
  uint32_t epoch_ = 0;
  // Access order of the valid entries (head = least recently accessed) with a 64-bit copy of
  // each entry's access epoch: while every entry was accessed within the last 2^32 epochs, the
  // oldest non-pending entry from the head is the reference's replacement victim.
  uint64_t epoch64_ = 0;
  std::vector<uint64_t> access64_;
  std::vector<uint32_t> rec_prev_, rec_next_;
  std::vector<uint8_t> rec_linked_;
  uint32_t rec_head_ = kNone, rec_tail_ = kNone;
  uint32_t next_token_ = 1;
  std::deque<PendingPut> fifo_;  // front = oldest
  std::vector<HostBacking> host_;
  std::map<uint64_t, uint64_t> pool_free_;  // unit -> units, address ordered
  std::vector<HostBacking> dropped_;
  std::vector<uint32_t> dirty_buckets_, dirty_slots_, dirty_keys_, evicted_;
  std::vector<uint8_t> bucket_dirty_, slot_dirty_, key_dirty_;
  DirStats st_;
};

}  // namespace kvs
