// kvs_directory.cpp -- host catalog of one store shard. See kvs_directory.hpp.
#include "kvs_directory.hpp"

#include <algorithm>
#include <stdexcept>

#include "kvs_kernels.cuh"

namespace kvs {

namespace {
constexpr uint32_t kHeapFree = 0xFFFFFFFEu;
constexpr uint32_t kHeapCont = 0xFFFFFFFDu;

uint32_t floor_log2(uint32_t v) {
  uint32_t o = 0;
  while (v > 1) {
    v >>= 1;
    ++o;
  }
  return o;
}

uint32_t order_for_units(uint32_t units) {
  uint32_t o = 0, b = 1;
  while (b < units) {
    b <<= 1;
    ++o;
  }
  return o;
}

uint32_t next_pow2(uint32_t x) {
  uint32_t p = 1;
  while (p < x) p <<= 1;
  return p;
}
}  // namespace

Directory::Directory(const DirConfig &cfg) : cfg_(cfg) {
  if (cfg.max_keys == 0 || cfg.max_keys > (1u << 30)) throw std::invalid_argument("max_keys out of range");
  if (cfg.unit_bytes == 0 || cfg.unit_bytes % 16 != 0)
    throw std::invalid_argument("unit_bytes must be a nonzero multiple of 16");
  if (cfg.max_key_bytes == 0 || cfg.max_key_bytes > kMaxKeyBytes)
    throw std::invalid_argument("max_key_bytes must be 1..128");
  if (cfg.heap_bytes < cfg.unit_bytes) throw std::invalid_argument("heap smaller than one unit");
  nb_ = next_pow2(cfg.max_keys * 2u);
  buckets_.assign(2ull * nb_, 0);
  for (uint32_t b = 0; b < nb_; ++b) buckets_[2 * b + 1] = kBucketEmpty;
  dir_.resize(cfg.max_keys);
  access64_.assign(cfg.max_keys, 0);
  rec_prev_.assign(cfg.max_keys, kNone);
  rec_next_.assign(cfg.max_keys, kNone);
  rec_linked_.assign(cfg.max_keys, 0);
  free_next_.assign(cfg.max_keys, kNone);
  lru_prev_.assign(cfg.max_keys, kNone);
  lru_next_.assign(cfg.max_keys, kNone);
  const uint64_t nu = cfg.heap_bytes / cfg.unit_bytes;
  if (nu > 0xFFFFFFF0ull) throw std::invalid_argument("value heap has too many units");
  num_units_ = (uint32_t)nu;
  max_order_ = floor_log2(num_units_);
  hm_.resize(num_units_);
  for (auto &h : free_heads_) h = kNone;
  uint32_t first = 0, remaining = num_units_;
  while (remaining) {
    uint32_t order = floor_log2(remaining);
    while (order != 0 && (first & ((1u << order) - 1u)) != 0) --order;
    buddy_push_free(first, order);
    first += 1u << order;
    remaining -= 1u << order;
  }
  host_.resize(cfg.max_keys);
  if (cfg.host_pool_units) pool_free_.emplace(0, cfg.host_pool_units);
  bucket_dirty_.assign(nb_, 0);
  slot_dirty_.assign(cfg.max_keys, 0);
  key_dirty_.assign(cfg.max_keys, 0);
}

uint32_t Directory::hash_of(const uint8_t *key, uint32_t len) const { return fnv1a32(key, len); }

uint32_t Directory::lookup(const uint8_t *key, uint32_t len) const {
  return idx_lookup(hash_of(key, len), key, len);
}

// ---------------------------------------------------------------- index

void Directory::set_bucket(uint32_t b, uint32_t hash, uint32_t slot) {
  buckets_[2 * b] = hash;
  buckets_[2 * b + 1] = slot;
  if (!bucket_dirty_[b]) {
    bucket_dirty_[b] = 1;
    dirty_buckets_.push_back(b);
  }
}

uint32_t Directory::idx_lookup(uint32_t h, const uint8_t *key, uint32_t len) const {
  const uint32_t mask = nb_ - 1;
  uint32_t idx = h & mask;
  for (uint32_t probe = 0; probe < nb_; ++probe) {
    const uint32_t slot = buckets_[2 * idx + 1];
    if (slot == kBucketEmpty) return kBucketEmpty;
    if (slot != kBucketTombstone && buckets_[2 * idx] == h) {
      const Entry &e = dir_[slot];
      if (e.valid && e.key_len == len && std::memcmp(e.key, key, len) == 0) return slot;
    }
    idx = (idx + 1) & mask;
  }
  return kBucketEmpty;
}

void Directory::idx_insert(uint32_t h, uint32_t slot) {
  const uint32_t mask = nb_ - 1;
  uint32_t idx = h & mask;
  for (uint32_t probe = 0; probe < nb_; ++probe) {
    const uint32_t cur = buckets_[2 * idx + 1];
    if (cur == kBucketEmpty || cur == kBucketTombstone) {
      set_bucket(idx, h, slot);
      return;
    }
    idx = (idx + 1) & mask;
  }
  throw std::logic_error("hash index full despite load factor <= 0.5");
}

void Directory::idx_delete(uint32_t h, uint32_t target) {
  const uint32_t mask = nb_ - 1;
  uint32_t hole = h & mask;
  bool found = false;
  for (uint32_t probe = 0; probe < nb_; ++probe) {
    const uint32_t cur = buckets_[2 * hole + 1];
    if (cur == kBucketEmpty) return;
    if (cur == target && buckets_[2 * hole] == h) {
      found = true;
      break;
    }
    hole = (hole + 1) & mask;
  }
  if (!found) return;
  uint32_t j = hole;
  for (uint32_t scanned = 0; scanned < nb_; ++scanned) {
    j = (j + 1) & mask;
    if (buckets_[2 * j + 1] == kBucketEmpty) break;
    const uint32_t home = buckets_[2 * j] & mask;
    const bool can_move = (hole <= j) ? (home <= hole || home > j) : (home <= hole && home > j);
    if (can_move) {
      set_bucket(hole, buckets_[2 * j], buckets_[2 * j + 1]);
      hole = j;
    }
  }
  set_bucket(hole, buckets_[2 * hole], kBucketEmpty);
}

// ---------------------------------------------------------------- buddy heap

void Directory::buddy_remove_free(uint32_t unit, uint32_t order) {
  HeapMeta &b = hm_[unit];
  const uint32_t next = b.next, prev = b.prev;
  if (prev == kNone) free_heads_[order] = next; else hm_[prev].next = next;
  if (next != kNone) hm_[next].prev = prev;
  b = {kHeapCont, order, kNone, kNone};
}

void Directory::buddy_push_free(uint32_t unit, uint32_t order) {
  const uint32_t old = free_heads_[order];
  hm_[unit] = {kHeapFree, order, old, kNone};
  if (old != kNone) hm_[old].prev = unit;
  free_heads_[order] = unit;
}

bool Directory::buddy_allocate(uint32_t units, uint32_t owner, uint32_t *out_unit, uint32_t *out_order) {
  const uint32_t need = order_for_units(units);
  uint32_t order = need;
  while (order <= max_order_ && free_heads_[order] == kNone) ++order;
  if (order > max_order_) return false;
  const uint32_t unit = free_heads_[order];
  buddy_remove_free(unit, order);
  while (order > need) {
    --order;
    buddy_push_free(unit + (1u << order), order);
  }
  hm_[unit] = {owner, need, kNone, kNone};
  *out_unit = unit;
  *out_order = need;
  return true;
}

void Directory::buddy_free(uint32_t unit, uint32_t order) {
  while (order < max_order_) {
    const uint32_t buddy = unit ^ (1u << order);
    if (buddy >= num_units_) break;
    if (hm_[buddy].state != kHeapFree || hm_[buddy].order != order) break;
    buddy_remove_free(buddy, order);
    unit = std::min(unit, buddy);
    ++order;
  }
  buddy_push_free(unit, order);
}

bool Directory::evict(uint32_t slot) {
  Entry &e = dir_[slot];
  if (!e.valid || e.location != kLocDevice) return false;
  const uint64_t bb = block_bytes(e.order);
  e.location = kLocHost;
  mark_slot(slot);
  evicted_.push_back(slot);
  lru_remove(slot);
  buddy_free((uint32_t)(e.value_off / cfg_.unit_bytes), e.order);
  live_bytes_ = live_bytes_ >= bb ? live_bytes_ - bb : 0;
  return true;
}

bool Directory::allocate_cache_block(uint64_t units, uint32_t owner, uint32_t *unit, uint32_t *order) {
  st_.allocation_calls++;
  if (units == 0 || units > num_units_) {
    st_.allocation_failures++;
    return false;
  }
  const uint64_t bb = block_bytes(order_for_units((uint32_t)units));
  if (bb > cfg_.heap_bytes) {
    st_.allocation_failures++;
    return false;
  }
  for (uint32_t attempts = 0; attempts <= cfg_.max_keys; ++attempts) {
    if (live_bytes_ <= cfg_.heap_bytes - bb && buddy_allocate((uint32_t)units, owner, unit, order)) {
      st_.allocation_successes++;
      return true;
    }
    if (attempts == cfg_.max_keys) break;
    // oldest committed device-resident entry; pending entries are pinned
    st_.victim_scans++;
    uint32_t victim = kNone, s = lru_tail_;
    for (uint32_t v = 0; s != kNone && v < lru_count_; ++v) {
      if (dir_[s].valid && dir_[s].location == kLocDevice) {
        victim = s;
        break;
      }
      s = lru_prev_[s];
    }
    if (victim == kNone || !evict(victim)) break;
    st_.victims_evicted++;
  }
  st_.allocation_failures++;
  return false;
}

// ---------------------------------------------------------------- LRU

void Directory::lru_remove(uint32_t slot) {
  const uint32_t prev = lru_prev_[slot], next = lru_next_[slot];
  if (prev == kNone) lru_head_ = next; else lru_next_[prev] = next;
  if (next == kNone) lru_tail_ = prev; else lru_prev_[next] = prev;
  lru_prev_[slot] = lru_next_[slot] = kNone;
  --lru_count_;
}

void Directory::lru_insert_mru(uint32_t slot) {
  const uint32_t old = lru_head_;
  lru_prev_[slot] = kNone;
  lru_next_[slot] = old;
  if (old == kNone) lru_tail_ = slot; else lru_prev_[old] = slot;
  lru_head_ = slot;
  ++lru_count_;
}

void Directory::lru_touch(uint32_t slot) {
  if (lru_head_ == slot) return;
  lru_remove(slot);
  lru_insert_mru(slot);
}

uint32_t Directory::lru_order(uint32_t *out, uint32_t cap) const {
  uint32_t n = 0;
  for (uint32_t s = lru_head_; s != kNone && n < cap; s = lru_next_[s]) out[n++] = s;
  return n;
}

// ---------------------------------------------------------------- catalog

uint32_t Directory::catalog_claim() {
  if (free_head_ != kNone) {
    const uint32_t slot = free_head_;
    free_head_ = free_next_[slot];
    free_next_[slot] = kNone;
    return slot;
  }
  if (next_unused_ == cfg_.max_keys) return kBucketEmpty;
  return next_unused_++;
}

void Directory::catalog_release(uint32_t slot) {
  free_next_[slot] = free_head_;
  free_head_ = slot;
}

void Directory::mark_slot(uint32_t slot) {
  if (!slot_dirty_[slot]) {
    slot_dirty_[slot] = 1;
    dirty_slots_.push_back(slot);
  }
}

void Directory::drop_backing(uint32_t slot) {
  HostBacking &h = host_[slot];
  if (!h.present) return;
  if (h.in_pool)
    pool_release(h.pool_unit, h.pool_units);
  else
    dropped_.push_back(h);
  h = HostBacking{};
}

uint32_t Directory::bump_epoch() {
  ++epoch64_;
  return ++epoch_;
}

void Directory::rec_unlink(uint32_t slot) {
  if (!rec_linked_[slot]) return;
  const uint32_t p = rec_prev_[slot], n = rec_next_[slot];
  if (p != kNone) rec_next_[p] = n; else rec_head_ = n;
  if (n != kNone) rec_prev_[n] = p; else rec_tail_ = p;
  rec_prev_[slot] = rec_next_[slot] = kNone;
  rec_linked_[slot] = 0;
}

// The slot's entry was just given the newest access epoch: it moves to the tail.
void Directory::rec_touch(uint32_t slot) {
  rec_unlink(slot);
  rec_prev_[slot] = rec_tail_;
  rec_next_[slot] = kNone;
  if (rec_tail_ != kNone) rec_next_[rec_tail_] = slot; else rec_head_ = slot;
  rec_tail_ = slot;
  rec_linked_[slot] = 1;
  access64_[slot] = epoch64_;
}

// The catalog replacement victim (P3:10373-10413): the valid, non-pending entry with the largest
// 32-bit access age, epoch - last_access; kNone if every valid entry is pending. Access epochs are
// unique, so while the oldest entry is younger than 2^32 epochs the 32-bit ages order the entries
// as the access list does and the first non-pending entry from its head is the answer; past that
// the reference's wrap-around arithmetic decides, by its own scan over every slot.
uint32_t Directory::oldest_replaceable() const {
  if (rec_head_ == kNone) return kNone;
  if (epoch64_ - access64_[rec_head_] < (1ull << 32)) {
    for (uint32_t i = rec_head_; i != kNone; i = rec_next_[i])
      if (dir_[i].location != kLocPending) return i;
    return kNone;
  }
  uint32_t oldest = kNone, oldest_age = 0;
  for (uint32_t i = 0; i < cfg_.max_keys; ++i) {
    const Entry &e = dir_[i];
    if (!e.valid || e.location == kLocPending) continue;
    const uint32_t age = epoch_ - e.last_access;
    if (oldest == kNone || age > oldest_age) {
      oldest_age = age;
      oldest = i;
    }
  }
  return oldest;
}

Prepare Directory::prepare_put(const uint8_t *key, uint32_t len, uint64_t value_len, Grant *out) {
  const uint64_t units = units_for(value_len);
  const uint32_t h = hash_of(key, len);
  uint32_t slot = idx_lookup(h, key, len);
  bool retry = false;
  if (slot != kBucketEmpty) retry = dir_[slot].location == kLocPending;
  if (!retry && slot == kBucketEmpty) slot = catalog_claim();
  if (!retry && slot == kBucketEmpty) {
    const uint32_t oldest = oldest_replaceable();
    if (oldest != kNone) {
      slot = oldest;
      st_.catalog_replacements++;
    } else {
      retry = true;
    }
  }
  if (!retry) {
    Entry &old = dir_[slot];
    if (old.valid) {
      idx_delete(hash_of(old.key, old.key_len), slot);
      if (old.location == kLocDevice) {
        lru_remove(slot);
        const uint64_t bb = block_bytes(old.order);
        buddy_free((uint32_t)(old.value_off / cfg_.unit_bytes), old.order);
        live_bytes_ = live_bytes_ >= bb ? live_bytes_ - bb : 0;
      }
      old.valid = 0;
      rec_unlink(slot);
      mark_slot(slot);
      drop_backing(slot);
    }
    uint32_t unit, order;
    if (allocate_cache_block(units, slot, &unit, &order)) {
      Entry &e = dir_[slot];
      const uint32_t token = next_token_++;
      if (next_token_ == 0) next_token_ = 1;
      e.valid = 1;
      e.key_len = (uint8_t)len;
      e.total_len = value_len;
      e.last_access = bump_epoch();
      rec_touch(slot);
      e.value_off = (uint64_t)unit * cfg_.unit_bytes;
      e.host_gen = token;
      e.location = kLocPending;
      e.order = order;
      std::memset(e.key, 0, sizeof e.key);
      std::memcpy(e.key, key, len);
      mark_slot(slot);
      if (!key_dirty_[slot]) {
        key_dirty_[slot] = 1;
        dirty_keys_.push_back(slot);
      }
      idx_insert(h, slot);
      lru_insert_mru(slot);
      const uint64_t bb = block_bytes(order);
      live_bytes_ += bb;
      pending_bytes_ += bb;
      fifo_.push_back(PendingPut{slot, token, HostBacking{}, -1});
      st_.issued++;
      *out = Grant{slot, order, token, e.value_off};
      return Prepare::kGranted;
    }
    catalog_release(slot);
    retry = true;
  }
  return fifo_.empty() ? Prepare::kNoSpace : Prepare::kNeedCommit;
}

bool Directory::commit_head(HostBacking *released) {
  PendingPut it = fifo_.front();
  fifo_.pop_front();
  st_.committed++;
  Entry &e = dir_[it.slot];
  if (!e.valid || e.location != kLocPending || e.host_gen != it.token) {
    st_.stale_commits++;
    *released = it.backing;
    return false;
  }
  drop_backing(it.slot);
  host_[it.slot] = it.backing;
  host_[it.slot].present = true;
  st_.writes_through++;
  if (it.backing.in_pool) st_.pool_values++; else st_.heap_values++;
  e.host_gen = it.token;  // non-zero generation of the committed copy
  e.location = kLocDevice;
  mark_slot(it.slot);
  pending_bytes_ -= block_bytes(e.order);
  *released = HostBacking{};
  return true;
}

Directory::GetAction Directory::get_hit(uint32_t slot, uint64_t *admit_off) {
  Entry &e = dir_[slot];
  const uint32_t epoch = bump_epoch();
  rec_touch(slot);  // every branch below gives the entry this epoch
  if (e.location != kLocHost) {
    e.last_access = epoch;
    lru_touch(slot);
    return GetAction::kDevice;
  }
  st_.host_serves++;
  uint32_t unit, order;
  if (allocate_cache_block(units_for(e.total_len), slot, &unit, &order)) {
    e.value_off = (uint64_t)unit * cfg_.unit_bytes;
    e.location = kLocDevice;
    e.order = order;
    e.last_access = epoch;
    mark_slot(slot);
    lru_insert_mru(slot);
    live_bytes_ += block_bytes(order);
    st_.admissions++;
    *admit_off = e.value_off;
    return GetAction::kAdmit;
  }
  e.last_access = epoch;
  return GetAction::kHostOnly;
}

void Directory::remove(uint32_t slot) {
  Entry &e = dir_[slot];
  idx_delete(hash_of(e.key, e.key_len), slot);
  if (e.location != kLocHost) {
    lru_remove(slot);
    const uint64_t bb = block_bytes(e.order);
    buddy_free((uint32_t)(e.value_off / cfg_.unit_bytes), e.order);
    live_bytes_ = live_bytes_ >= bb ? live_bytes_ - bb : 0;
    if (e.location == kLocPending) pending_bytes_ -= bb;
  }
  e.valid = 0;
  rec_unlink(slot);
  mark_slot(slot);
  catalog_release(slot);
  drop_backing(slot);
}

bool Directory::move_to_host(uint32_t slot) {
  if (dir_[slot].location != kLocDevice) return false;
  return evict(slot);
}

bool Directory::move_to_device(uint32_t slot, uint64_t *admit_off) {
  Entry &e = dir_[slot];
  if (e.location != kLocHost) return false;
  uint32_t unit, order;
  if (!allocate_cache_block(units_for(e.total_len), slot, &unit, &order)) return false;
  e.value_off = (uint64_t)unit * cfg_.unit_bytes;
  e.location = kLocDevice;
  e.order = order;
  e.last_access = bump_epoch();
  rec_touch(slot);
  mark_slot(slot);
  lru_insert_mru(slot);
  live_bytes_ += block_bytes(order);
  st_.admissions++;
  *admit_off = e.value_off;
  return true;
}

// ---------------------------------------------------------------- host pool (first fit)

bool Directory::pool_alloc(uint64_t units, uint64_t *unit) {
  if (units == 0) return false;
  for (auto it = pool_free_.begin(); it != pool_free_.end(); ++it) {
    if (it->second < units) continue;
    const uint64_t u = it->first, left = it->second - units;
    pool_free_.erase(it);
    if (left) pool_free_.emplace(u + units, left);
    *unit = u;
    return true;
  }
  return false;
}

void Directory::pool_release(uint64_t unit, uint64_t units) {
  if (units == 0) return;
  auto next = pool_free_.lower_bound(unit);
  if (next != pool_free_.end() && next->first == unit + units) {
    units += next->second;
    next = pool_free_.erase(next);
  }
  if (next != pool_free_.begin()) {
    auto prev = std::prev(next);
    if (prev->first + prev->second == unit) {
      prev->second += units;
      return;
    }
  }
  pool_free_.emplace(unit, units);
}

std::vector<HostBacking> Directory::take_dropped() {
  std::vector<HostBacking> out;
  out.swap(dropped_);
  return out;
}

std::vector<uint32_t> Directory::take_dirty_buckets() {
  for (uint32_t b : dirty_buckets_) bucket_dirty_[b] = 0;
  std::vector<uint32_t> out;
  out.swap(dirty_buckets_);
  return out;
}

std::vector<uint32_t> Directory::take_dirty_slots() {
  for (uint32_t s : dirty_slots_) slot_dirty_[s] = 0;
  std::vector<uint32_t> out;
  out.swap(dirty_slots_);
  return out;
}

std::vector<uint32_t> Directory::take_dirty_keys() {
  for (uint32_t s : dirty_keys_) key_dirty_[s] = 0;
  std::vector<uint32_t> out;
  out.swap(dirty_keys_);
  return out;
}

uint64_t Directory::live_keys(uint64_t *device_resident) const {
  uint64_t n = 0, d = 0;
  for (const Entry &e : dir_)
    if (e.valid) {
      ++n;
      if (e.location != kLocHost) ++d;
    }
  if (device_resident) *device_resident = d;
  return n;
}

}  // namespace kvs
