// kvs_runtime.cpp -- store shards, clients and the C ABI (include/kvs.h).
//
// Execution model
//   * A shard (kvs_server) owns, on its GPU: the value slab (buddy heap of `unit_bytes` units),
//     the device replica of the hash index (bucket words, entry metadata, key rows), and a
//     write-through stream; on the host: the catalog (kvs::Directory) and the pinned host pool.
//   * A client owns a CUDA stream on its GPU and a pinned/device staging area. Every call
//     packs its metadata into the staging area, uploads it with one copy, and launches its
//     kernels on the client stream. Work that touches a shard is ordered across clients by an
//     event chain kept under the shard mutex: each call waits on the shard's last event before
//     launching and records a new one after. A get of at most kvs::kInlineKeys device-resident
//     blocks is the exception: the catalog answers its lookups and its one copy runs on the
//     caller's stream, which the call synchronises before returning (small_device_get).
//   * Copies take one of three engines (launch_copy): the one-wave engine for copies up to
//     kvs::small_copy_limit() bytes or of one-piece member blocks, the bulk-copy ring for larger
//     device-memory copies, and 16-byte loads and stores when a side is host memory.
//   * Host write-through is a device->host copy of each landed value on the shard's
//     write-through stream, ordered after the gather by an event; the pending-host FIFO entry
//     becomes committed at the next commit barrier (or earlier when allocation pressure forces
//     it), exactly in issue order.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "kvs.h"
#include "kvs_chunk_meta.hpp"
#include "kvs_directory.hpp"
#include "kvs_kernels.cuh"

using kvs::Directory;
using kvs::HostBacking;

namespace {

thread_local std::string g_err;

int set_err(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define CUDA_TRY(x)                                                                          \
  do {                                                                                       \
    cudaError_t e_ = (x);                                                                    \
    if (e_ != cudaSuccess) return set_err(KVS_E_CUDA, "%s failed: %s", #x, cudaGetErrorString(e_)); \
  } while (0)

#define TRY(x)              \
  do {                      \
    int rc_ = (x);          \
    if (rc_ != KVS_OK) return rc_; \
  } while (0)

// Device allocations the runtime knows: every shard's slab and every peer mapping opened from an
// IPC handle. A copy whose blob addresses all fall inside them may use the bulk-copy engine, which
// needs device memory on both sides (this GPU's or a peer's).
std::mutex g_ranges_mu;
std::map<uint64_t, uint64_t> g_ranges;  // base -> bytes

void dev_range_add(const void *base, uint64_t bytes) {
  std::lock_guard<std::mutex> lk(g_ranges_mu);
  g_ranges[reinterpret_cast<uint64_t>(base)] = bytes;
}

void dev_range_remove(const void *base) {
  std::lock_guard<std::mutex> lk(g_ranges_mu);
  g_ranges.erase(reinterpret_cast<uint64_t>(base));
}

bool dev_ranges_hold(const uint64_t *addrs, uint32_t n, uint64_t len) {
  std::lock_guard<std::mutex> lk(g_ranges_mu);
  for (uint32_t i = 0; i < n; ++i) {
    if (!addrs[i]) continue;  // a skipped blob
    auto it = g_ranges.upper_bound(addrs[i]);
    if (it == g_ranges.begin()) return false;
    --it;
    if (addrs[i] + len > it->first + it->second) return false;
  }
  return true;
}

uint64_t now_ns() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Growable pinned host + device staging area. One upload per call.
struct Staging {
  uint8_t *host = nullptr;
  uint8_t *host_dev = nullptr;  // device alias of the mapped host buffer (kernels write results here)
  uint8_t *dev = nullptr;
  size_t cap = 0, used = 0;
  cudaEvent_t uploaded = nullptr;  // last upload out of `host` finished

  int init() {
    CUDA_TRY(cudaEventCreateWithFlags(&uploaded, cudaEventDisableTiming));
    return KVS_OK;
  }
  // Start packing a new call: waits until the previous upload has left `host`.
  int begin(size_t need, cudaStream_t stream) {
    CUDA_TRY(cudaEventSynchronize(uploaded));
    used = 0;
    if (need > cap) {
      CUDA_TRY(cudaStreamSynchronize(stream));  // device staging may still be read
      if (host) cudaFreeHost(host);
      if (dev) cudaFree(dev);
      host = nullptr;
      dev = nullptr;
      size_t c = std::max<size_t>(need, 1 << 20);
      c = (c + 4095) & ~size_t(4095);
      CUDA_TRY(cudaHostAlloc(reinterpret_cast<void **>(&host), c, cudaHostAllocMapped | cudaHostAllocPortable));
      CUDA_TRY(cudaHostGetDevicePointer(reinterpret_cast<void **>(&host_dev), host, 0));
      CUDA_TRY(cudaMalloc(&dev, c));
      cap = c;
    }
    return KVS_OK;
  }
  // Reserve n bytes (16-byte aligned); returns the offset.
  size_t take(size_t n) {
    size_t off = (used + 15) & ~size_t(15);
    used = off + n;
    if (used > cap) {  // a sizing bug must never write past the buffer
      std::fprintf(stderr, "kvs: staging overflow (%zu > %zu)\n", used, cap);
      std::abort();
    }
    return off;
  }
  size_t push(const void *p, size_t n) {
    size_t off = take(n);
    if (n) std::memcpy(host + off, p, n);
    return off;
  }
  template <class T> T *h(size_t off) { return reinterpret_cast<T *>(host + off); }
  template <class T> T *d(size_t off) { return reinterpret_cast<T *>(dev + off); }
  template <class T> T *hd(size_t off) { return reinterpret_cast<T *>(host_dev + off); }
  int upload(cudaStream_t stream, size_t bytes) {
    if (bytes) CUDA_TRY(cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, stream));
    CUDA_TRY(cudaEventRecord(uploaded, stream));
    return KVS_OK;
  }
  void release() {
    if (uploaded) cudaEventSynchronize(uploaded);
    if (host) cudaFreeHost(host);
    if (dev) cudaFree(dev);
    if (uploaded) cudaEventDestroy(uploaded);
    host = dev = nullptr;
    uploaded = nullptr;
    cap = used = 0;
  }
};

uint64_t parse_env_u64(const char *name, uint64_t dflt, bool *bad) {
  const char *v = std::getenv(name);
  if (!v) return dflt;
  // exact unsigned decimal, like the reference's parse_u64_exact (patch 0003 lines 5156-5260)
  if (!*v) {
    *bad = true;
    return dflt;
  }
  uint64_t x = 0;
  for (const char *p = v; *p; ++p) {
    if (*p < '0' || *p > '9') {
      *bad = true;
      return dflt;
    }
    const uint64_t d = (uint64_t)(*p - '0');
    if (x > (UINT64_MAX - d) / 10) {
      *bad = true;
      return dflt;
    }
    x = x * 10 + d;
  }
  return x;
}

}  // namespace

// ============================================================================ shard

struct WtBatch {
  uint64_t id;
  cudaEvent_t done;
};

struct kvs_server {
  kvs_server_config cfg{};
  std::mutex mu;
  Directory *dir = nullptr;
  uint8_t *slab = nullptr;
  uint64_t *d_buckets = nullptr;
  kvs::DevMeta *d_meta = nullptr;
  uint32_t *d_keyrows = nullptr;
  uint8_t *pool = nullptr;
  uint8_t *pool_dev = nullptr;  // device alias of the mapped pool
  cudaStream_t wt_stream = nullptr;
  cudaEvent_t tail = nullptr;  // newest event of the shard's ordering chain (not owned)
  std::vector<WtBatch> wt_batches;
  std::vector<cudaEvent_t> free_events;
  uint64_t next_batch = 1;
  std::multimap<uint64_t, uint8_t *> heap_cache;  // recycled pinned buffers for off-pool values
  // Off-pool values live in pinned chunks of at least kHeapChunk bytes, handed out front to back
  // (one pinning call per chunk rather than per value); the chunks are freed with the shard.
  static constexpr uint64_t kHeapChunk = 256ull << 20;
  std::vector<uint8_t *> heap_chunks;
  uint8_t *heap_next = nullptr;
  uint64_t heap_left = 0;
  std::atomic<uint64_t> moves_completed{0};
  std::atomic<uint64_t> launches{0};
  kvs_move_profile mprof{};
  bool ready = false;
  bool quarantined = false;
  // remote puts (kvs_grant_puts): the newest `unlanded` FIFO entries wait for kvs_puts_landed;
  // grant_blocked: the last prepare asked for a commit of a value that had not landed
  uint32_t unlanded = 0;
  bool grant_blocked = false;

  uint64_t slab_base() const { return reinterpret_cast<uint64_t>(slab); }

  cudaEvent_t event_for_batch(uint64_t id) {
    for (auto &b : wt_batches)
      if (b.id == id) return b.done;
    return nullptr;
  }
  int new_batch(uint64_t *id, cudaEvent_t *ev) {
    cudaEvent_t e;
    if (!free_events.empty()) {
      e = free_events.back();
      free_events.pop_back();
    } else {
      CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    *id = next_batch++;
    wt_batches.push_back({*id, e});
    *ev = e;
    return KVS_OK;
  }
  void retire_batches() {
    // a batch is retired once no FIFO entry refers to it
    std::vector<WtBatch> keep;
    for (auto &b : wt_batches) {
      bool used = false;
      for (auto &p : dir->fifo())
        if ((uint64_t)p.wt_batch == b.id) {
          used = true;
          break;
        }
      if (used) keep.push_back(b); else free_events.push_back(b.done);
    }
    wt_batches.swap(keep);
  }
  uint8_t *host_ptr(const HostBacking &b) const {
    return b.in_pool ? pool + b.pool_unit * cfg.unit_bytes : b.heap;
  }
  // device alias of a host backing, for kernels that read the host tier directly over PCIe
  uint64_t device_alias(const HostBacking &b) const {
    if (b.in_pool) return reinterpret_cast<uint64_t>(pool_dev) + b.pool_unit * cfg.unit_bytes;
    void *d = nullptr;
    if (cudaHostGetDevicePointer(&d, b.heap, 0) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    return reinterpret_cast<uint64_t>(d);
  }
  int reserve_backing(uint64_t len, HostBacking *out) {
    HostBacking b;
    b.present = true;
    b.len = len;
    uint64_t unit;
    const uint64_t units = dir->units_for(len);
    if (pool && dir->pool_alloc(units, &unit)) {
      b.in_pool = true;
      b.pool_unit = unit;
      b.pool_units = units;
    } else {
      auto it = heap_cache.lower_bound(len);
      if (it != heap_cache.end() && it->first <= 2 * len) {
        b.heap = it->second;
        heap_cache.erase(it);
      } else {
        const uint64_t take = (len + 255) & ~uint64_t(255);
        if (take > heap_left) {
          void *p = nullptr;
          const uint64_t chunk = std::max(kHeapChunk, take);
          CUDA_TRY(cudaHostAlloc(&p, chunk, cudaHostAllocPortable | cudaHostAllocMapped));
          heap_chunks.push_back((uint8_t *)p);
          heap_next = (uint8_t *)p;
          heap_left = chunk;
        }
        b.heap = heap_next;
        heap_next += take;
        heap_left -= take;
      }
      b.len = len;
    }
    *out = b;
    return KVS_OK;
  }
  void release_backing(const HostBacking &b) {
    if (!b.present) return;
    if (b.in_pool)
      dir->pool_release(b.pool_unit, b.pool_units);
    else if (b.heap)
      heap_cache.emplace(b.len, b.heap);
  }
  void release_dropped() {
    for (auto &b : dir->take_dropped()) release_backing(b);
  }
  // Device->host copies of one write-through batch, coalesced: consecutive values of one length
  // whose slab blocks are evenly spaced and whose host extents are evenly spaced become one 2-D
  // copy, so a large put issues a handful of copy commands instead of one per value (thousands of
  // queued copies would block the issuing thread until the copy queue drains).
  struct WtRun {
    uint8_t *host;
    const uint8_t *slab;
    uint64_t len, host_pitch, slab_pitch, n;
  };
  std::vector<WtRun> wt_runs;
  bool in_pool(const uint8_t *p) const {
    return pool && p >= pool && p < pool + (cfg.host_pool_bytes / cfg.unit_bytes) * cfg.unit_bytes;
  }
  static constexpr uint64_t kWtMergeBelow = 8ull << 20;  // large values already make few commands
  void wt_add(uint8_t *host, const uint8_t *slab_ptr, uint64_t len) {
    // a 2-D copy spans the rows between its ends: merge only inside the one pinned pool allocation
    if (!wt_runs.empty() && len < kWtMergeBelow && in_pool(host) && in_pool(wt_runs.back().host)) {
      WtRun &r = wt_runs.back();
      if (r.len == len) {
        const uint8_t *last_slab = r.slab + (r.n - 1) * r.slab_pitch;
        uint8_t *last_host = r.host + (r.n - 1) * r.host_pitch;
        if (r.n == 1 && slab_ptr > r.slab && host > r.host && (uint64_t)(slab_ptr - r.slab) >= len &&
            (uint64_t)(host - r.host) >= len) {
          r.slab_pitch = (uint64_t)(slab_ptr - r.slab);
          r.host_pitch = (uint64_t)(host - r.host);
          r.n = 2;
          return;
        }
        if (r.n > 1 && slab_ptr == last_slab + r.slab_pitch && host == last_host + r.host_pitch) {
          r.n++;
          return;
        }
      }
    }
    wt_runs.push_back({host, slab_ptr, len, len, len, 1});
  }
  // Write-through timing (kvs_server_set_timing): events on the write-through stream around each
  // batch of device->host copies, so the copies' own duration is measured, not inferred.
  struct WtTimed {
    cudaEvent_t start, stop;
    uint64_t bytes;
  };
  bool wt_timing = false;
  std::vector<WtTimed> wt_timed;
  std::vector<cudaEvent_t> wt_timing_events;
  kvs_kernel_timing wt_acc{};
  cudaEvent_t timing_event() {
    if (!wt_timing_events.empty()) {
      cudaEvent_t e = wt_timing_events.back();
      wt_timing_events.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    return e;
  }
  void drain_wt_timing() {
    for (auto &t : wt_timed) {
      float ms = 0.f;
      if (cudaEventSynchronize(t.stop) == cudaSuccess && cudaEventElapsedTime(&ms, t.start, t.stop) == cudaSuccess) {
        wt_acc.launches++;
        wt_acc.bytes += t.bytes;
        wt_acc.total_ms += ms;
      } else {
        cudaGetLastError();
      }
      wt_timing_events.push_back(t.start);
      wt_timing_events.push_back(t.stop);
    }
    wt_timed.clear();
  }
  int wt_issue() {
    cudaEvent_t start = nullptr;
    uint64_t bytes = 0;
    if (wt_timing && !wt_runs.empty() && (start = timing_event()) != nullptr)
      CUDA_TRY(cudaEventRecord(start, wt_stream));
    for (const WtRun &r : wt_runs) {
      if (r.n == 1)
        CUDA_TRY(cudaMemcpyAsync(r.host, r.slab, r.len, cudaMemcpyDeviceToHost, wt_stream));
      else
        CUDA_TRY(cudaMemcpy2DAsync(r.host, r.host_pitch, r.slab, r.slab_pitch, r.len, r.n, cudaMemcpyDeviceToHost,
                                   wt_stream));
      bytes += r.len * r.n;
    }
    wt_runs.clear();
    if (start) {
      cudaEvent_t stop = timing_event();
      if (!stop) {
        wt_timing_events.push_back(start);
        return KVS_OK;
      }
      CUDA_TRY(cudaEventRecord(stop, wt_stream));
      wt_timed.push_back({start, stop, bytes});
    }
    return KVS_OK;
  }
  // Commit the FIFO head, waiting for its device->host copy.
  int commit_one() {
    auto &head = dir->fifo_head();
    if (head.wt_batch < 0)
      return set_err(KVS_E_INVAL, "shard %u: a granted remote put has not landed yet (kvs_puts_landed)", cfg.shard_id);
    cudaEvent_t ev = event_for_batch((uint64_t)head.wt_batch);
    const uint64_t t0 = now_ns();
    if (ev) CUDA_TRY(cudaEventSynchronize(ev));
    HostBacking released;
    const uint64_t len = head.backing.len;
    if (dir->commit_head(&released)) {
      mprof.to_host_count++;
      mprof.to_host_read_calls++;
      mprof.to_host_read_bytes += len;
      mprof.to_host_read_passes++;
      mprof.to_host_device_pushes++;
      const uint64_t dt = now_ns() - t0;
      mprof.to_host_worker_ns += dt;
      mprof.to_host_complete_ns += dt;
      moves_completed.fetch_add(1, std::memory_order_relaxed);
    } else {
      release_backing(released);
    }
    return KVS_OK;
  }
  // COMMIT_BARRIER: every issued put becomes host-committed, in issue order.
  int commit_all() {
    if (dir->fifo_empty()) return KVS_OK;
    if (unlanded)
      return set_err(KVS_E_INVAL, "shard %u: %u granted remote puts have not landed yet (kvs_puts_landed)",
                     cfg.shard_id, unlanded);
    cudaEvent_t last = event_for_batch((uint64_t)dir->fifo_back().wt_batch);
    if (last) CUDA_TRY(cudaEventSynchronize(last));
    while (!dir->fifo_empty()) TRY(commit_one());
    retire_batches();
    release_dropped();
    grant_blocked = false;  // the commit a stopped grant asked for has happened
    return KVS_OK;
  }
};

// ============================================================================ client

// Bumped whenever a peer mapping closes: member pointers checked before may now be invalid.
static std::atomic<uint64_t> g_mapping_generation{1};

struct kvs_client {
  int device = 0;
  std::vector<kvs_server *> shards;
  std::mutex mu;
  cudaStream_t stream = nullptr;
  cudaEvent_t entry_evt = nullptr, exit_evt = nullptr, landed_evt = nullptr;
  std::vector<cudaEvent_t> chain_evt;  // per shard
  Staging stage;
  Staging stage2;  // a get's second pass, packed while the first pass's results are still in flight
  // Device copy of the last block layout's arrays a get uploaded (member pointers, member block
  // bytes, region bases, tile prefix, back to back), and the host bytes it holds: small gets that
  // name the same layout read it from here instead of uploading it again.
  uint8_t *layout_dev = nullptr;
  size_t layout_cap = 0;
  std::vector<uint8_t> layout_key;
  bool closed = false, quarantined = false;
  kvs_put_profile prof{};
  std::vector<uint64_t> validated_members;
  uint64_t validated_generation = 0;  // g_mapping_generation when validated_members was checked
  // kernel timing (events around copy-engine launches)
  unsigned int *timeout_flag = nullptr;  // host-mapped word a copy kernel sets if a bounded wait expires
  bool timing = false;
  struct Timed {
    cudaEvent_t start, stop;
    int kind;  // 0 gather, 1 scatter, 2 admission (host -> slab), 3 host-tier serve (host -> pool)
    uint64_t bytes;
  };
  std::vector<Timed> timed;
  std::vector<cudaEvent_t> event_pool;
  kvs_kernel_timing acc[4]{};  // gather, scatter, host-tier admissions, host-tier serves
  cudaEvent_t pooled_event() {
    if (!event_pool.empty()) {
      cudaEvent_t e = event_pool.back();
      event_pool.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
  void time_begin(cudaEvent_t *start) { time_begin_on(start, stream); }
  void time_end(cudaEvent_t start, int kind, uint64_t bytes) { time_end_on(start, kind, bytes, stream); }
  // the same around a launch on stream `on` (the caller's stream, for instance)
  void time_begin_on(cudaEvent_t *start, cudaStream_t on) {
    *start = nullptr;
    if (!timing) return;
    *start = pooled_event();
    cudaEventRecord(*start, on);
  }
  void time_end_on(cudaEvent_t start, int kind, uint64_t bytes, cudaStream_t on) {
    if (!timing || !start) return;
    cudaEvent_t stop = pooled_event();
    cudaEventRecord(stop, on);
    timed.push_back({start, stop, kind, bytes});
  }
  void drain_timing() {
    for (auto &t : timed) {
      cudaEventSynchronize(t.stop);
      float ms = 0.f;
      cudaEventElapsedTime(&ms, t.start, t.stop);
      acc[t.kind].launches++;
      acc[t.kind].bytes += t.bytes;
      acc[t.kind].total_ms += ms;
      event_pool.push_back(t.start);
      event_pool.push_back(t.stop);
    }
    timed.clear();
  }
};

namespace {

// Copy-engine choice, for copies whose layout facts the caller gave (max_member_bytes,
// payload_bytes): the one-wave engine up to kvs::small_copy_limit() bytes, or at any size when
// every member block is one 16 KiB piece (kvs::small_copy_suits). Otherwise the TMA bulk engine for
// device memory (this GPU's or a peer's), and the LDG/STG engine when a side is host memory.
// KVS_COPY_ENGINE=ldg forces the LDG engine for the copies that do not take the one-wave engine.
bool tma_enabled() { return kvs::bulk_engine_enabled(); }

cudaError_t launch_copy(kvs::ChunkCopyParams p, cudaStream_t stream, bool device_memory_only,
                        unsigned int *timeout_flag) {
  p.timeout_flag = timeout_flag;
  if (kvs::small_copy_suits(p)) return kvs::launch_chunk_copy_small(p, stream);
  if (device_memory_only && tma_enabled()) return kvs::launch_chunk_copy_tma(p, stream);
  return kvs::launch_chunk_copy(p, stream);
}

// Sets the engine-choice facts of a copy of `combos` (blob block, rank) pairs over a layout whose
// member blocks are `member_bytes[0..n_members)`.
void set_copy_facts(kvs::ChunkCopyParams *p, const uint64_t *member_bytes, uint32_t n_members, uint64_t combos) {
  uint64_t mx = 0, sum = 0;
  for (uint32_t m = 0; m < n_members; ++m) {
    mx = member_bytes[m] > mx ? member_bytes[m] : mx;
    sum += member_bytes[m];
  }
  p->max_member_bytes = mx;
  p->payload_bytes = sum * combos;
}

// Bounded waits in the bulk engine that expired (never in normal operation) turn into an error.
// The kernel sets the client's host-mapped flag, read here after the call synchronised.
int check_tma_timeouts(kvs_client *c, const char *op) {
  if (c->timeout_flag && *reinterpret_cast<volatile unsigned int *>(c->timeout_flag))
    return set_err(KVS_E_TIMEOUT, "%s: copy-engine waits expired", op);
  return KVS_OK;
}

int check_client(kvs_client *c) {
  if (!c) return set_err(KVS_E_INVAL, "client handle is null");
  if (c->closed) return set_err(KVS_E_CLOSED, "client is closed");
  if (c->quarantined)
    return set_err(KVS_E_QUARANTINED, "client is quarantined after an indeterminate failure");
  return KVS_OK;
}

int validate_key(kvs_client *c, const void *key, uint32_t len, const char *op) {
  if (len == 0) return set_err(KVS_E_INVAL, "%s: key must be non-empty", op);
  uint32_t maxk = 128;
  for (auto *s : c->shards) maxk = std::min(maxk, s->cfg.max_key_bytes);
  if (len > maxk) return set_err(KVS_E_INVAL, "%s: key size %u exceeds Server max_key_bytes %u", op, len, maxk);
  if (!key) return set_err(KVS_E_INVAL, "%s: key pointer is null", op);
  return KVS_OK;
}

uint32_t shard_index(kvs_client *c, const uint8_t *key, uint32_t len) {
  if (c->shards.size() == 1) return 0;
  return kvs::fnv1a32(key, len) % (uint32_t)c->shards.size();
}

int check_device_ptr(kvs_client *c, const void *p, const char *op, const char *what) {
  cudaPointerAttributes a{};
  cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_err(KVS_E_INVAL, "%s: %s must use DEVICE storage", op, what);
  }
  if (a.type != cudaMemoryTypeDevice)
    return set_err(KVS_E_INVAL, "%s: %s must use DEVICE storage", op, what);
  if (a.type == cudaMemoryTypeDevice && a.device != c->device)
    return set_err(KVS_E_INVAL, "%s: %s must belong to the client device %d; got device %d", op, what,
                   c->device, a.device);
  return KVS_OK;
}

// Sorted, de-duplicated shard locks (get_parallel takes locks in address order, patch 0003
// client_operations_adapter.cpp:145-187).
struct ShardLocks {
  std::vector<kvs_server *> held;
  explicit ShardLocks(std::vector<kvs_server *> v) {
    std::sort(v.begin(), v.end());
    v.erase(std::unique(v.begin(), v.end()), v.end());
    for (auto *s : v) s->mu.lock();
    held = v;
  }
  ~ShardLocks() {
    for (auto it = held.rbegin(); it != held.rend(); ++it) (*it)->mu.unlock();
  }
};

// The client stream is non-blocking, so it is ordered with the caller's stream explicitly at entry
// and exit. A null handle is the legacy default stream (torch's default stream), not "no stream".
int begin_op(kvs_client *c, void *caller) {
  CUDA_TRY(cudaEventRecord(c->entry_evt, (cudaStream_t)caller));
  CUDA_TRY(cudaStreamWaitEvent(c->stream, c->entry_evt, 0));
  return KVS_OK;
}

int end_op(kvs_client *c, void *caller) {
  CUDA_TRY(cudaEventRecord(c->exit_evt, c->stream));
  CUDA_TRY(cudaStreamWaitEvent((cudaStream_t)caller, c->exit_evt, 0));
  return KVS_OK;
}

int chain_wait(kvs_client *c, kvs_server *s) {
  if (!s->tail) return KVS_OK;
  for (cudaEvent_t e : c->chain_evt)
    if (e == s->tail) return KVS_OK;  // recorded on this client's own stream: already ordered
  CUDA_TRY(cudaStreamWaitEvent(c->stream, s->tail, 0));
  return KVS_OK;
}

int chain_record(kvs_client *c, size_t shard_idx) {
  kvs_server *s = c->shards[shard_idx];
  CUDA_TRY(cudaEventRecord(c->chain_evt[shard_idx], c->stream));
  s->tail = c->chain_evt[shard_idx];
  return KVS_OK;
}

// Mutations of one shard's index replica, packed into the staging area.
struct PackedMutations {
  size_t buckets_off = 0, meta_off = 0, keys_off = 0;
  uint32_t nb = 0, nm = 0, nk = 0;
};

PackedMutations pack_mutations(kvs_server *s, Staging &st) {
  PackedMutations pm;
  auto buckets = s->dir->take_dirty_buckets();
  auto slots = s->dir->take_dirty_slots();
  auto keys = s->dir->take_dirty_keys();
  pm.nb = (uint32_t)buckets.size();
  pm.nm = (uint32_t)slots.size();
  pm.nk = (uint32_t)keys.size();
  pm.buckets_off = st.take(16ull * pm.nb);
  uint64_t *bw = st.h<uint64_t>(pm.buckets_off);
  for (size_t i = 0; i < buckets.size(); ++i) {
    bw[2 * i] = buckets[i];
    bw[2 * i + 1] = s->dir->bucket_word(buckets[i]);
  }
  pm.meta_off = st.take(24ull * pm.nm);
  uint64_t *mw = st.h<uint64_t>(pm.meta_off);
  for (size_t i = 0; i < slots.size(); ++i) {
    const kvs::Entry &e = s->dir->entry(slots[i]);
    kvs::DevMeta m{};
    m.value_off = e.value_off;
    m.total_len = (uint32_t)e.total_len;
    m.valid = e.valid;
    m.location = e.location;
    m.key_len = e.key_len;
    uint64_t words[2];
    std::memcpy(words, &m, 16);
    mw[3 * i] = slots[i];
    mw[3 * i + 1] = words[0];
    mw[3 * i + 2] = words[1];
  }
  pm.keys_off = st.take(4ull * (kvs::kKeyRowWords + 1) * pm.nk);
  uint32_t *kw = st.h<uint32_t>(pm.keys_off);
  for (size_t i = 0; i < keys.size(); ++i) {
    uint32_t *rec = kw + i * (kvs::kKeyRowWords + 1);
    rec[0] = keys[i];
    std::memcpy(rec + 1, s->dir->entry(keys[i]).key, kvs::kMaxKeyBytes);
  }
  return pm;
}

// Exact staging bytes pack_mutations will take for the shard's current dirty sets.
size_t mutation_upper_bound(kvs_server *s) {
  size_t nb, nm, nk;
  s->dir->dirty_counts(&nb, &nm, &nk);
  return 16 * nb + 24 * nm + 4ull * (kvs::kKeyRowWords + 1) * nk + 64;
}

int launch_mutations(kvs_client *c, kvs_server *s, const PackedMutations &pm, Staging *from = nullptr) {
  Staging &st = from ? *from : c->stage;
  kvs::MutationParams mp{};
  mp.bucket_writes = st.d<uint64_t>(pm.buckets_off);
  mp.n_bucket_writes = pm.nb;
  mp.meta_writes = st.d<uint64_t>(pm.meta_off);
  mp.n_meta_writes = pm.nm;
  mp.key_writes = st.d<uint32_t>(pm.keys_off);
  mp.n_key_writes = pm.nk;
  mp.buckets = s->d_buckets;
  mp.meta = s->d_meta;
  mp.key_rows = s->d_keyrows;
  CUDA_TRY(kvs::launch_apply_mutations(mp, c->stream));
  if (pm.nb + pm.nm + pm.nk) s->launches++;
  return KVS_OK;
}

// Block value format for a layout: header words + region bases + value length.
struct BlockFormat {
  std::vector<uint32_t> header;
  std::vector<uint64_t> region_bases;
  std::vector<uint64_t> tile_prefix;
  uint64_t value_len = 0;
};

constexpr uint32_t kTileBytes = 32 << 10;

// Block value layout: header [MAGIC, n_layers, layer bytes...] zero padded to 32 bytes, then the
// members back to back in member order, each member region starting on a 16-byte boundary (a
// no-op for K/V blocks, whose sizes are multiples of 16; it aligns members such as 4-byte
// per-block scales). Layer sizes in the header count the bytes the layer occupies.
int block_format(const kvs_block_layout *L, BlockFormat *f) {
  if (!L || L->n_members == 0 || !L->member_ptrs || !L->member_block_bytes)
    return set_err(KVS_E_INVAL, "block layout: members must not be empty");
  if (L->members_per_layer == 0 || L->n_members % L->members_per_layer)
    return set_err(KVS_E_INVAL, "block layout: %u members is not a whole number of %u-member layers",
                   L->n_members, L->members_per_layer);
  const uint32_t n_layers = L->n_members / L->members_per_layer;
  uint64_t hdr_words = 2 + n_layers;
  hdr_words = (hdr_words + 7) / 8 * 8;
  f->header.assign(hdr_words, 0);
  f->header[0] = 0x524B564Eu;
  f->header[1] = n_layers;
  uint64_t off = 4 * hdr_words;
  f->region_bases.resize(L->n_members);
  f->tile_prefix.assign(L->n_members + 1, 0);
  for (uint32_t m = 0; m < L->n_members; ++m) {
    const uint64_t b = L->member_block_bytes[m];
    if (b == 0 || b % 4)
      return set_err(KVS_E_INVAL, "block layout: member %u block bytes %llu must be nonzero and 4-byte aligned", m,
                     (unsigned long long)b);
    if (!L->member_ptrs[m]) return set_err(KVS_E_INVAL, "block layout: member %u pointer is null", m);
    const uint64_t start = off;
    f->region_bases[m] = off;
    off += b;
    off = (off + 15) & ~uint64_t(15);
    const uint32_t l = m / L->members_per_layer;
    const uint64_t sz = (uint64_t)f->header[2 + l] + (off - start);
    if (sz > 0xFFFFFFFFull) return set_err(KVS_E_INVAL, "block layout: layer %u exceeds the 32-bit header", l);
    f->header[2 + l] = (uint32_t)sz;
    f->tile_prefix[m + 1] = f->tile_prefix[m] + (b + kTileBytes - 1) / kTileBytes;
  }
  f->value_len = off;
  return KVS_OK;
}

// block_format through a per-thread cache of the last layout shape (member count, members per
// layer, member block bytes): the block calls of a serving loop name the same shape every time,
// so the format is built once per thread instead of once per call. Member pointers are checked
// for null on every call, as block_format does.
int cached_block_format(const kvs_block_layout *L, const BlockFormat **out) {
  thread_local BlockFormat fmt;
  thread_local std::vector<uint64_t> shape;  // {n_members, members_per_layer, block bytes...}
  if (L && L->n_members && L->member_ptrs && L->member_block_bytes && shape.size() == 2ull + L->n_members &&
      shape[0] == L->n_members && shape[1] == L->members_per_layer &&
      std::memcmp(shape.data() + 2, L->member_block_bytes, 8ull * L->n_members) == 0) {
    for (uint32_t m = 0; m < L->n_members; ++m)
      if (!L->member_ptrs[m]) return set_err(KVS_E_INVAL, "block layout: member %u pointer is null", m);
    *out = &fmt;
    return KVS_OK;
  }
  shape.clear();
  TRY(block_format(L, &fmt));
  shape.push_back(L->n_members);
  shape.push_back(L->members_per_layer);
  shape.insert(shape.end(), L->member_block_bytes, L->member_block_bytes + L->n_members);
  *out = &fmt;
  return KVS_OK;
}

int validate_layout_ptrs(kvs_client *c, const kvs_block_layout *L, const char *op) {
  std::vector<uint64_t> cur(L->member_ptrs, L->member_ptrs + L->n_members);
  const uint64_t gen = g_mapping_generation.load(std::memory_order_acquire);
  if (cur == c->validated_members && c->validated_generation == gen) return KVS_OK;
  for (uint32_t m = 0; m < L->n_members; ++m)
    TRY(check_device_ptr(c, reinterpret_cast<const void *>(L->member_ptrs[m]), op, "member tensor"));
  c->validated_members = cur;
  c->validated_generation = gen;
  return KVS_OK;
}

// ---------------------------------------------------------------------------- put machinery

// One item staged for a put: the slab destination and either a block id (block puts) or a
// source pointer and length (value puts).
struct PutItem {
  uint32_t shard;
  uint64_t blob;     // absolute slab address
  int64_t block_id;  // block puts
  uint64_t src, len; // value puts
  uint64_t slab_off;
};

struct PutBatch {
  kvs_client *c;
  const kvs_block_layout *layout;  // null for value puts
  const BlockFormat *fmt;
  std::vector<PutItem> items;
  std::vector<uint8_t> involved;  // per shard
};

// Launch everything staged so far: replica mutations, the gather, and write-through.
int flush_puts(PutBatch &b, cudaStream_t) {
  kvs_client *c = b.c;
  const size_t ns = c->shards.size();
  bool any_dirty = false;
  for (size_t i = 0; i < ns; ++i) any_dirty |= b.involved[i] != 0;
  if (b.items.empty() && !any_dirty) return KVS_OK;
  const uint64_t t0 = now_ns();
  size_t need = 4096 + b.items.size() * 64;
  if (b.layout) need += (size_t)b.layout->n_members * 40 + b.fmt->header.size() * 4;
  for (size_t i = 0; i < ns; ++i)
    if (b.involved[i]) need += mutation_upper_bound(c->shards[i]);
  need += 64ull * b.items.size();
  TRY(c->stage.begin(need, c->stream));
  Staging &st = c->stage;
  std::vector<PackedMutations> pms(ns);
  for (size_t i = 0; i < ns; ++i)
    if (b.involved[i]) pms[i] = pack_mutations(c->shards[i], st);
  size_t blobs_off = 0, ids_off = 0, mp_off = 0, mb_off = 0, rb_off = 0, tp_off = 0, hw_off = 0;
  const size_t n = b.items.size();
  if (b.layout) {
    blobs_off = st.take(8 * n);
    ids_off = st.take(8 * n);
    for (size_t i = 0; i < n; ++i) {
      st.h<uint64_t>(blobs_off)[i] = b.items[i].blob;
      st.h<int64_t>(ids_off)[i] = b.items[i].block_id;
    }
    mp_off = st.push(b.layout->member_ptrs, 8ull * b.layout->n_members);
    mb_off = st.push(b.layout->member_block_bytes, 8ull * b.layout->n_members);
    rb_off = st.push(b.fmt->region_bases.data(), 8ull * b.layout->n_members);
    tp_off = st.push(b.fmt->tile_prefix.data(), 8ull * (b.layout->n_members + 1));
    hw_off = st.push(b.fmt->header.data(), 4ull * b.fmt->header.size());
  } else {
    // value puts: per item {member ptr, bytes, region base 0, tile prefix 0..t, block 0, blob}
    blobs_off = st.take(48 * n);
    for (size_t i = 0; i < n; ++i) {
      uint64_t *r = st.h<uint64_t>(blobs_off) + 6 * i;
      r[0] = b.items[i].src;
      r[1] = b.items[i].len;
      r[2] = 0;
      r[3] = 0;
      r[4] = (b.items[i].len + kTileBytes - 1) / kTileBytes;
      r[5] = b.items[i].blob;
    }
    ids_off = st.take(8);
    *st.h<int64_t>(ids_off) = 0;
  }
  TRY(st.upload(c->stream, st.used));
  for (size_t i = 0; i < ns; ++i)
    if (b.involved[i]) TRY(chain_wait(c, c->shards[i]));
  for (size_t i = 0; i < ns; ++i)
    if (b.involved[i]) TRY(launch_mutations(c, c->shards[i], pms[i]));
  if (n) {
    if (b.layout) {
      kvs::ChunkCopyParams p{};
      p.member_ptrs = st.d<uint64_t>(mp_off);
      p.member_bytes = st.d<uint64_t>(mb_off);
      p.region_bases = st.d<uint64_t>(rb_off);
      p.tile_prefix = st.d<uint64_t>(tp_off);
      p.block_ids = st.d<int64_t>(ids_off);
      p.blob_ptrs = st.d<uint64_t>(blobs_off);
      p.header_words = st.d<uint32_t>(hw_off);
      p.n_header_words = (uint32_t)b.fmt->header.size();
      p.n_blobs = (uint32_t)n;
      p.blocks_per_blob = 1;
      p.n_ranks = 1;
      p.n_members = b.layout->n_members;
      p.tile_bytes = kTileBytes;
      p.tiles_per_combo = b.fmt->tile_prefix.back();
      p.total_tiles = (uint64_t)n * p.tiles_per_combo;
      p.to_blob = 1;
      set_copy_facts(&p, b.layout->member_block_bytes, b.layout->n_members, n);
      cudaEvent_t timed_start = nullptr;
      c->time_begin(&timed_start);
      CUDA_TRY(launch_copy(p, c->stream, true, c->timeout_flag));
      c->time_end(timed_start, 0, (uint64_t)n * (b.fmt->value_len - 4ull * b.fmt->header.size()));
    } else {
      for (size_t i = 0; i < n; ++i) {
        const size_t r = blobs_off + 48 * i;
        kvs::ChunkCopyParams p{};
        p.member_ptrs = st.d<uint64_t>(r);
        p.member_bytes = st.d<uint64_t>(r + 8);
        p.region_bases = st.d<uint64_t>(r + 16);
        p.tile_prefix = st.d<uint64_t>(r + 24);
        p.block_ids = st.d<int64_t>(ids_off);
        p.blob_ptrs = st.d<uint64_t>(r + 40);
        p.n_blobs = 1;
        p.blocks_per_blob = 1;
        p.n_ranks = 1;
        p.n_members = 1;
        p.tile_bytes = kTileBytes;
        p.tiles_per_combo = (b.items[i].len + kTileBytes - 1) / kTileBytes;
        p.total_tiles = p.tiles_per_combo;
        p.to_blob = 1;
        set_copy_facts(&p, &b.items[i].len, 1, 1);
        CUDA_TRY(launch_copy(p, c->stream, true, c->timeout_flag));
      }
    }
    for (size_t i = 0; i < ns; ++i)
      if (b.involved[i]) c->shards[i]->launches += b.layout ? 1 : n;
  }
  CUDA_TRY(cudaEventRecord(c->landed_evt, c->stream));
  for (size_t i = 0; i < ns; ++i)
    if (b.involved[i]) TRY(chain_record(c, i));
  const uint64_t t1 = now_ns();
  // write-through: one device->host copy per value on each shard's write-through stream
  std::vector<size_t> per_shard(ns, 0);
  for (auto &it : b.items) per_shard[it.shard]++;
  for (size_t si = 0; si < ns; ++si) {
    if (!per_shard[si]) continue;
    kvs_server *s = c->shards[si];
    DeviceGuard g(s->cfg.device);
    CUDA_TRY(cudaStreamWaitEvent(s->wt_stream, c->landed_evt, 0));
    uint64_t batch_id = 0;
    cudaEvent_t ev = nullptr;
    TRY(s->new_batch(&batch_id, &ev));
    auto &fifo = s->dir->fifo();
    size_t k = fifo.size() - per_shard[si];
    for (auto &it : b.items) {
      if (it.shard != si) continue;
      kvs::PendingPut &pp = fifo[k++];
      const uint64_t len = s->dir->entry(pp.slot).total_len;
      TRY(s->reserve_backing(len, &pp.backing));
      pp.wt_batch = (int)batch_id;
      s->wt_add(s->host_ptr(pp.backing), s->slab + it.slab_off, len);
    }
    TRY(s->wt_issue());
    CUDA_TRY(cudaEventRecord(ev, s->wt_stream));
  }
  c->prof.program_ns += t1 - t0;
  c->prof.enqueue_ns += now_ns() - t1;
  b.items.clear();
  return KVS_OK;
}

constexpr size_t kPutPieceBlocks = 512;

// Stage one put; drives forced commits when a pending entry blocks it.
int stage_put(PutBatch &b, uint32_t si, const uint8_t *key, uint32_t key_len, uint64_t value_len,
              int64_t block_id, uint64_t src) {
  kvs_server *s = b.c->shards[si];
  b.involved[si] = 1;
  for (;;) {
    kvs::Grant g;
    const kvs::Prepare r = s->dir->prepare_put(key, key_len, value_len, &g);
    if (r == kvs::Prepare::kGranted) {
      b.items.push_back(PutItem{si, s->slab_base() + g.value_off, block_id, src, value_len, g.value_off});
      return KVS_OK;
    }
    TRY(flush_puts(b, b.c->stream));
    if (r == kvs::Prepare::kNoSpace)
      return set_err(KVS_E_NOSPACE, "put: no device-cache space for a %llu B value", (unsigned long long)value_len);
    TRY(s->commit_one());  // force_put_host_commit, then retry the prepare
    s->retire_batches();
    s->release_dropped();
  }
}

int commit_barrier(kvs_client *c, const std::vector<uint8_t> &involved) {
  for (size_t i = 0; i < c->shards.size(); ++i)
    if (involved[i]) TRY(c->shards[i]->commit_all());
  // the write-through copies just waited for follow this client's gathers into those shards
  return check_tma_timeouts(c, "commit");
}

std::vector<kvs_server *> involved_servers(kvs_client *c, const std::vector<uint8_t> &inv) {
  std::vector<kvs_server *> v;
  for (size_t i = 0; i < c->shards.size(); ++i)
    if (inv[i]) v.push_back(c->shards[i]);
  return v;
}

int quarantine_on_error(kvs_client *c, int rc) {
  // a failed CUDA call or an expired copy-engine wait leaves the outcome indeterminate
  if ((rc == KVS_E_CUDA || rc == KVS_E_TIMEOUT) && c) c->quarantined = true;
  return rc;
}

// Copy one value staged by stage_value_copy (record at rec_off) with one copy launch. With
// device_memory_only both sides are device memory (bulk engine); otherwise the source is the
// pinned host tier read through its device alias (LDG engine).
int launch_value_copy(kvs_client *c, size_t rec_off, uint64_t len, bool device_memory_only) {
  kvs::ChunkCopyParams p{};
  p.member_ptrs = c->stage.d<uint64_t>(rec_off);
  p.member_bytes = c->stage.d<uint64_t>(rec_off + 8);
  p.region_bases = c->stage.d<uint64_t>(rec_off + 16);
  p.tile_prefix = c->stage.d<uint64_t>(rec_off + 24);
  p.block_ids = c->stage.d<int64_t>(rec_off + 48);
  p.blob_ptrs = c->stage.d<uint64_t>(rec_off + 40);
  p.n_blobs = 1;
  p.blocks_per_blob = 1;
  p.n_ranks = 1;
  p.n_members = 1;
  p.tile_bytes = kTileBytes;
  p.tiles_per_combo = (len + kTileBytes - 1) / kTileBytes;
  p.total_tiles = p.tiles_per_combo;
  p.to_blob = 0;
  if (device_memory_only) set_copy_facts(&p, &len, 1, 1);
  CUDA_TRY(launch_copy(p, c->stream, device_memory_only, c->timeout_flag));
  return KVS_OK;
}

// Record of a one-value copy src -> dst as a one-member scatter: {member ptr = dst, member bytes,
// region base 0, tile prefix {0, tiles}, blob ptr = src, block id 0}.
size_t stage_value_copy(Staging &st, uint64_t dst, uint64_t src, uint64_t len) {
  const size_t off = st.take(56);
  uint64_t *r = st.h<uint64_t>(off);
  r[0] = dst;
  r[1] = len;
  r[2] = 0;
  r[3] = 0;
  r[4] = (len + kTileBytes - 1) / kTileBytes;
  r[5] = src;
  r[6] = 0;  // block id
  return off;
}

}  // namespace

namespace kvs {
void set_last_error(const char *message) { g_err = message; }
}  // namespace kvs

// ============================================================================ C ABI

extern "C" {

int kvs_abi_version(void) { return KVS_ABI_VERSION; }

const char *kvs_last_error(void) { return g_err.c_str(); }

uint64_t kvs_kernel_launch_count(void) { return kvs::kernel_launches(); }

int kvs_copy_engine_status(int32_t device, uint32_t *expired_waits, uint32_t *unsafe_exits) {
  if (!expired_waits || !unsafe_exits) return set_err(KVS_E_INVAL, "copy_engine_status: null output");
  int ndev = 0;
  CUDA_TRY(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return set_err(KVS_E_INVAL, "device %d is not a visible CUDA device", device);
  DeviceGuard g(device);
  unsigned int expired = 0, unsafe = 0;
  CUDA_TRY(kvs::read_tma_counters(&expired, &unsafe));
  *expired_waits = expired;
  *unsafe_exits = unsafe;
  return KVS_OK;
}

int kvs_set_copy_wait_limit(int64_t polls) {
  if (polls > (int64_t)UINT32_MAX) return set_err(KVS_E_INVAL, "copy wait limit %lld exceeds 2^32 - 1 polls", (long long)polls);
  kvs::set_copy_wait_polls(polls < 0 ? kvs::default_copy_wait_polls() : (uint32_t)polls);
  return KVS_OK;
}

int kvs_set_small_copy_limit(int64_t bytes) {
  static const uint64_t initial = kvs::small_copy_limit();  // the default or KVS_SMALL_COPY_BYTES
  kvs::set_small_copy_limit(bytes < 0 ? initial : (uint64_t)bytes);
  return KVS_OK;
}

int kvs_server_config_default(kvs_server_config *cfg) {
  if (!cfg) return set_err(KVS_E_INVAL, "config is null");
  std::memset(cfg, 0, sizeof *cfg);
  bool bad = false;
  cfg->device = 0;
  cfg->max_keys = (uint32_t)parse_env_u64("KVM_SERVER_DRAM_MAX_KEYS", 1024, &bad);
  if (bad) return set_err(KVS_E_INVAL, "KVM_SERVER_DRAM_MAX_KEYS must be an unsigned decimal integer");
  cfg->heap_bytes = parse_env_u64("KVM_SERVER_DRAM_VALUE_HEAP_BYTES", 1434541824ull, &bad);
  if (bad) return set_err(KVS_E_INVAL, "KVM_SERVER_DRAM_VALUE_HEAP_BYTES must be an unsigned decimal integer");
  cfg->host_pool_bytes = parse_env_u64("KVM_SERVER_HOST_POOL_BYTES", 1ull << 30, &bad);
  if (bad) return set_err(KVS_E_INVAL, "KVM_SERVER_HOST_POOL_BYTES must be an unsigned decimal integer");
  cfg->max_value_bytes = parse_env_u64("KVM_COMMON_MAX_VALUE_BYTES", 64ull << 20, &bad);
  if (bad) return set_err(KVS_E_INVAL, "KVM_COMMON_MAX_VALUE_BYTES must be an unsigned decimal integer");
  cfg->max_key_bytes = (uint32_t)parse_env_u64("KVM_SERVER_MAX_KEY_BYTES", 128, &bad);
  if (bad) return set_err(KVS_E_INVAL, "KVM_SERVER_MAX_KEY_BYTES must be an unsigned decimal integer");
  cfg->unit_bytes = 4288;
  if (cfg->max_keys == 0 || cfg->max_keys > (1u << 26))
    return set_err(KVS_E_INVAL, "KVM_SERVER_DRAM_MAX_KEYS must be in 1..67108864");
  if (cfg->max_key_bytes == 0 || cfg->max_key_bytes > 128)
    return set_err(KVS_E_INVAL, "KVM_SERVER_MAX_KEY_BYTES must be in 1..128");
  if (cfg->max_value_bytes == 0) return set_err(KVS_E_INVAL, "KVM_COMMON_MAX_VALUE_BYTES must be > 0");
  return KVS_OK;
}

int kvs_server_create(const kvs_server_config *cfg_in, kvs_server **out) {
  if (!cfg_in || !out) return set_err(KVS_E_INVAL, "config and out must be non-null");
  *out = nullptr;
  kvs_server_config cfg = *cfg_in;
  if (cfg.unit_bytes == 0) cfg.unit_bytes = 4288;
  if (cfg.max_key_bytes == 0) cfg.max_key_bytes = 128;
  if (cfg.max_value_bytes == 0) cfg.max_value_bytes = 64ull << 20;
  if (cfg.max_keys == 0) return set_err(KVS_E_INVAL, "max_keys must be > 0");
  if (cfg.unit_bytes % 16) return set_err(KVS_E_INVAL, "unit_bytes must be a multiple of 16");
  if (cfg.max_key_bytes > 128) return set_err(KVS_E_INVAL, "max_key_bytes must be <= 128");
  if (cfg.heap_bytes < cfg.unit_bytes) return set_err(KVS_E_INVAL, "value heap smaller than one unit");
  if (cfg.heap_bytes / cfg.unit_bytes > 0xFFFFFFF0ull) return set_err(KVS_E_INVAL, "value heap has too many units");
  int ndev = 0;
  CUDA_TRY(cudaGetDeviceCount(&ndev));
  if (cfg.device < 0 || cfg.device >= ndev)
    return set_err(KVS_E_INVAL, "device %d is not a visible CUDA device (%d visible)", cfg.device, ndev);
  auto *s = new (std::nothrow) kvs_server();
  if (!s) return set_err(KVS_E_NOSPACE, "out of host memory");
  s->cfg = cfg;
  DeviceGuard g(cfg.device);
  auto fail = [&](int rc) {
    kvs_server_destroy(s);
    return rc;
  };
  try {
    kvs::DirConfig dc{cfg.max_keys, cfg.unit_bytes, cfg.max_key_bytes, cfg.heap_bytes, cfg.max_value_bytes,
                      cfg.host_pool_bytes / cfg.unit_bytes};
    s->dir = new Directory(dc);
  } catch (const std::exception &e) {
    return fail(set_err(KVS_E_INVAL, "server config: %s", e.what()));
  }
  cudaError_t e;
  if ((e = cudaMalloc(&s->slab, cfg.heap_bytes)) != cudaSuccess)
    return fail(set_err(KVS_E_NOSPACE, "slab of %llu B: %s", (unsigned long long)cfg.heap_bytes, cudaGetErrorString(e)));
  dev_range_add(s->slab, cfg.heap_bytes);
  const uint32_t nb = s->dir->num_buckets();
  if ((e = cudaMalloc(&s->d_buckets, 8ull * nb)) != cudaSuccess ||
      (e = cudaMalloc(&s->d_meta, sizeof(kvs::DevMeta) * cfg.max_keys)) != cudaSuccess ||
      (e = cudaMalloc(&s->d_keyrows, 4ull * kvs::kKeyRowWords * cfg.max_keys)) != cudaSuccess)
    return fail(set_err(KVS_E_NOSPACE, "index replica: %s", cudaGetErrorString(e)));
  // empty buckets are all-ones; metadata and key rows start zeroed
  if ((e = cudaMemset(s->d_buckets, 0xFF, 8ull * nb)) != cudaSuccess ||
      (e = cudaMemset(s->d_meta, 0, sizeof(kvs::DevMeta) * cfg.max_keys)) != cudaSuccess ||
      (e = cudaMemset(s->d_keyrows, 0, 4ull * kvs::kKeyRowWords * cfg.max_keys)) != cudaSuccess)
    return fail(set_err(KVS_E_CUDA, "index replica init: %s", cudaGetErrorString(e)));
  // the replica words are {hash, slot}: an empty bucket has slot 0xFFFFFFFF; hash is don't-care
  if (cfg.host_pool_bytes / cfg.unit_bytes) {
    const uint64_t bytes = (cfg.host_pool_bytes / cfg.unit_bytes) * cfg.unit_bytes;
    if ((e = cudaHostAlloc(&s->pool, bytes, cudaHostAllocPortable | cudaHostAllocMapped)) != cudaSuccess)
      return fail(set_err(KVS_E_NOSPACE, "host pool of %llu B: %s", (unsigned long long)bytes, cudaGetErrorString(e)));
    if ((e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&s->pool_dev), s->pool, 0)) != cudaSuccess)
      return fail(set_err(KVS_E_CUDA, "host pool device alias: %s", cudaGetErrorString(e)));
  }
  if ((e = cudaStreamCreateWithFlags(&s->wt_stream, cudaStreamNonBlocking)) != cudaSuccess)
    return fail(set_err(KVS_E_CUDA, "write-through stream: %s", cudaGetErrorString(e)));
  if ((e = cudaDeviceSynchronize()) != cudaSuccess)
    return fail(set_err(KVS_E_CUDA, "server init: %s", cudaGetErrorString(e)));
  s->ready = true;
  *out = s;
  return KVS_OK;
}

int kvs_server_destroy(kvs_server *s) {
  if (!s) return KVS_OK;
  int rc = KVS_OK;
  {
    std::lock_guard<std::mutex> lk(s->mu);
    DeviceGuard g(s->cfg.device);
    if (s->dir && s->wt_stream) {
      cudaStreamSynchronize(s->wt_stream);
      if (!s->dir->fifo_empty()) rc = s->commit_all();
    }
    if (s->wt_stream) cudaStreamSynchronize(s->wt_stream);
    s->drain_wt_timing();
    for (auto e : s->wt_timing_events) cudaEventDestroy(e);
    for (auto &b : s->wt_batches) cudaEventDestroy(b.done);
    for (auto e : s->free_events) cudaEventDestroy(e);
    for (uint8_t *chunk : s->heap_chunks) cudaFreeHost(chunk);  // every off-pool value lives in one
    if (s->wt_stream) cudaStreamDestroy(s->wt_stream);
    if (s->pool) cudaFreeHost(s->pool);
    if (s->d_keyrows) cudaFree(s->d_keyrows);
    if (s->d_meta) cudaFree(s->d_meta);
    if (s->d_buckets) cudaFree(s->d_buckets);
    if (s->slab) {
      dev_range_remove(s->slab);
      cudaFree(s->slab);
    }
    delete s->dir;
  }
  delete s;
  return rc;
}

int kvs_server_is_ready(kvs_server *s, int *ready) {
  if (!s || !ready) return set_err(KVS_E_INVAL, "null argument");
  *ready = s->ready && !s->quarantined;
  return KVS_OK;
}

int kvs_server_moves_completed(kvs_server *s, uint64_t *out) {
  if (!s || !out) return set_err(KVS_E_INVAL, "null argument");
  *out = s->moves_completed.load();
  return KVS_OK;
}

int kvs_server_move_profile(kvs_server *s, kvs_move_profile *out) {
  if (!s || !out) return set_err(KVS_E_INVAL, "null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  *out = s->mprof;
  return KVS_OK;
}

int kvs_server_allocator_profile(kvs_server *s, kvs_allocator_profile *out) {
  if (!s || !out) return set_err(KVS_E_INVAL, "null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  std::memset(out, 0, sizeof *out);
  auto &st = s->dir->stats();
  out->allocation_calls = st.allocation_calls;
  out->allocation_successes = st.allocation_successes;
  out->allocation_failures = st.allocation_failures;
  out->victim_scans = st.victim_scans;
  out->victims_evicted = st.victims_evicted;
  return KVS_OK;
}

int kvs_server_stats(kvs_server *s, kvs_stats *out) {
  if (!s || !out) return set_err(KVS_E_INVAL, "null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  std::memset(out, 0, sizeof *out);
  auto &st = s->dir->stats();
  out->live_device_bytes = s->dir->live_device_bytes();
  out->pending_device_bytes = s->dir->pending_device_bytes();
  out->live_keys = s->dir->live_keys(&out->device_resident_keys);
  out->allocation_calls = st.allocation_calls;
  out->allocation_successes = st.allocation_successes;
  out->allocation_failures = st.allocation_failures;
  out->victims_evicted = st.victims_evicted;
  out->catalog_replacements = st.catalog_replacements;
  out->writes_through = st.writes_through;
  out->stale_commits = st.stale_commits;
  out->host_serves = st.host_serves;
  out->admissions = st.admissions;
  out->pool_values = st.pool_values;
  out->heap_values = st.heap_values;
  out->epoch = s->dir->epoch();
  out->issued = st.issued;
  out->committed = st.committed;
  out->kernel_launches = s->launches.load();
  return KVS_OK;
}

int kvs_server_set_timing(kvs_server *s, int enable) {
  if (!s) return set_err(KVS_E_INVAL, "server handle is null");
  std::lock_guard<std::mutex> lk(s->mu);
  DeviceGuard g(s->cfg.device);
  s->wt_timing = enable != 0;
  return KVS_OK;
}

int kvs_server_write_through_timing(kvs_server *s, kvs_kernel_timing *out) {
  if (!s || !out) return set_err(KVS_E_INVAL, "server_write_through_timing: null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  DeviceGuard g(s->cfg.device);
  s->drain_wt_timing();
  *out = s->wt_acc;
  s->wt_acc = kvs_kernel_timing{};
  return KVS_OK;
}

int kvs_server_device(kvs_server *s, int *device) {
  if (!s || !device) return set_err(KVS_E_INVAL, "null argument");
  *device = s->cfg.device;
  return KVS_OK;
}

int kvs_server_put_drain_progress(kvs_server *s, uint32_t *issued, uint32_t *committed) {
  if (!s || !issued || !committed) return set_err(KVS_E_INVAL, "null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  *issued = s->dir->stats().issued;
  *committed = s->dir->stats().committed;
  return KVS_OK;
}

int kvs_server_location(kvs_server *s, const void *key, uint32_t key_len, int *location, uint64_t *value_off) {
  if (!s || !key || !location) return set_err(KVS_E_INVAL, "null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  const uint32_t slot = s->dir->lookup((const uint8_t *)key, key_len);
  if (slot == kvs::kBucketEmpty) {
    *location = KVS_LOC_ABSENT;
    return KVS_OK;
  }
  *location = s->dir->entry(slot).location;
  if (value_off) *value_off = s->dir->entry(slot).value_off;
  return KVS_OK;
}

int kvs_server_index_snapshot(kvs_server *s, uint32_t *host_pairs, uint32_t *device_pairs, uint32_t cap_pairs,
                              uint32_t *n_buckets) {
  if (!s || !n_buckets) return set_err(KVS_E_INVAL, "null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  const uint32_t nb = s->dir->num_buckets();
  *n_buckets = nb;
  if (cap_pairs < nb) return KVS_OK;
  DeviceGuard g(s->cfg.device);
  if (s->tail) CUDA_TRY(cudaEventSynchronize(s->tail));
  // replica updates that no device lookup has needed yet (small gets answer on the host) are
  // written now, so the snapshot shows the replica as the next probe will see it
  for (uint32_t b : s->dir->take_dirty_buckets()) {
    const uint64_t w = s->dir->bucket_word(b);
    CUDA_TRY(cudaMemcpy(s->d_buckets + b, &w, 8, cudaMemcpyHostToDevice));
  }
  for (uint32_t slot : s->dir->take_dirty_slots()) {
    const kvs::Entry &e = s->dir->entry(slot);
    kvs::DevMeta m{};
    m.value_off = e.value_off;
    m.total_len = (uint32_t)e.total_len;
    m.valid = e.valid;
    m.location = e.location;
    m.key_len = e.key_len;
    CUDA_TRY(cudaMemcpy(s->d_meta + slot, &m, sizeof m, cudaMemcpyHostToDevice));
  }
  for (uint32_t slot : s->dir->take_dirty_keys())
    CUDA_TRY(cudaMemcpy(s->d_keyrows + (uint64_t)slot * kvs::kKeyRowWords, s->dir->entry(slot).key,
                        kvs::kMaxKeyBytes, cudaMemcpyHostToDevice));
  if (host_pairs) std::memcpy(host_pairs, s->dir->bucket_pairs(), 8ull * nb);
  if (device_pairs) {
    std::vector<uint64_t> w(nb);
    CUDA_TRY(cudaMemcpy(w.data(), s->d_buckets, 8ull * nb, cudaMemcpyDeviceToHost));
    for (uint32_t b = 0; b < nb; ++b) {
      device_pairs[2 * b] = (uint32_t)w[b];
      device_pairs[2 * b + 1] = (uint32_t)(w[b] >> 32);
    }
  }
  return KVS_OK;
}

int kvs_server_lru_order(kvs_server *s, uint32_t *slots, uint32_t cap, uint32_t *n) {
  if (!s || !n) return set_err(KVS_E_INVAL, "null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  if (!slots) {  // size query
    *n = s->dir->lru_size();
    return KVS_OK;
  }
  *n = s->dir->lru_order(slots, cap);
  return KVS_OK;
}

// ---------------------------------------------------------------------------- client

int kvs_client_create(kvs_server *const *shards, uint32_t n_shards, int32_t device, kvs_client **out) {
  if (!out) return set_err(KVS_E_INVAL, "out is null");
  *out = nullptr;
  if (!shards || n_shards == 0) return set_err(KVS_E_INVAL, "a client needs at least one server shard");
  int ndev = 0;
  CUDA_TRY(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return set_err(KVS_E_INVAL, "device %d is not a visible CUDA device", device);
  for (uint32_t i = 0; i < n_shards; ++i)
    if (!shards[i]) return set_err(KVS_E_INVAL, "shard %u is null", i);
  auto *c = new (std::nothrow) kvs_client();
  if (!c) return set_err(KVS_E_NOSPACE, "out of host memory");
  c->device = device;
  c->shards.assign(shards, shards + n_shards);
  DeviceGuard g(device);
  // peer access to every remote shard's GPU: put / get kernels store and load over NVLink
  for (auto *s : c->shards) {
    if (s->cfg.device == device) continue;
    int can = 0;
    CUDA_TRY(cudaDeviceCanAccessPeer(&can, device, s->cfg.device));
    if (!can) {
      delete c;
      return set_err(KVS_E_INVAL, "device %d cannot access peer device %d", device, s->cfg.device);
    }
    cudaError_t e = cudaDeviceEnablePeerAccess(s->cfg.device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
    else if (e != cudaSuccess) {
      delete c;
      return set_err(KVS_E_CUDA, "enable peer access %d->%d: %s", device, s->cfg.device, cudaGetErrorString(e));
    }
  }
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->entry_evt, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->exit_evt, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->landed_evt, cudaEventDisableTiming);
  if (e == cudaSuccess)
    e = cudaHostAlloc(reinterpret_cast<void **>(&c->timeout_flag), 64, cudaHostAllocMapped | cudaHostAllocPortable);
  if (e == cudaSuccess) *c->timeout_flag = 0;
  c->chain_evt.assign(n_shards, nullptr);
  for (uint32_t i = 0; i < n_shards && e == cudaSuccess; ++i)
    e = cudaEventCreateWithFlags(&c->chain_evt[i], cudaEventDisableTiming);
  if (e != cudaSuccess || c->stage.init() != KVS_OK || c->stage2.init() != KVS_OK) {
    kvs_client_destroy(c);
    return set_err(KVS_E_CUDA, "client init: %s", cudaGetErrorString(e));
  }
  *out = c;
  return KVS_OK;
}

int kvs_client_destroy(kvs_client *c) {
  if (!c) return KVS_OK;
  int rc = KVS_OK;
  {
    std::lock_guard<std::mutex> lk(c->mu);
    DeviceGuard g(c->device);
    if (!c->closed && !c->quarantined && c->stream) {
      // drain every issued put of this client's shards (Client::close; kvcache_manager/docs/design.md section 8 in patch 0003)
      std::vector<uint8_t> inv(c->shards.size(), 1);
      ShardLocks locks(involved_servers(c, inv));
      rc = commit_barrier(c, inv);
      cudaStreamSynchronize(c->stream);
      for (size_t i = 0; i < c->shards.size(); ++i)
        if (c->shards[i]->tail == c->chain_evt[i]) {
          // keep the chain valid: hand the shard a completed chain position
          c->shards[i]->tail = nullptr;
        }
    } else if (c->stream) {
      cudaStreamSynchronize(c->stream);
      std::vector<kvs_server *> all(c->shards);
      ShardLocks locks(all);
      for (size_t i = 0; i < c->shards.size(); ++i)
        if (c->shards[i]->tail == c->chain_evt[i]) c->shards[i]->tail = nullptr;
    }
    c->closed = true;
    c->drain_timing();
    for (auto e : c->event_pool) cudaEventDestroy(e);
    if (c->timeout_flag) cudaFreeHost(c->timeout_flag);
    c->stage.release();
    c->stage2.release();
    if (c->layout_dev) cudaFree(c->layout_dev);
    for (auto e : c->chain_evt)
      if (e) cudaEventDestroy(e);
    if (c->entry_evt) cudaEventDestroy(c->entry_evt);
    if (c->exit_evt) cudaEventDestroy(c->exit_evt);
    if (c->landed_evt) cudaEventDestroy(c->landed_evt);
    if (c->stream) cudaStreamDestroy(c->stream);
  }
  delete c;
  return rc;
}

int kvs_client_is_established(kvs_client *c, int *established) {
  if (!c || !established) return set_err(KVS_E_INVAL, "null argument");
  *established = !c->closed && !c->quarantined;
  return KVS_OK;
}

int kvs_client_shard_of(kvs_client *c, const void *key, uint32_t key_len, uint32_t *shard) {
  if (!c || !key || !shard) return set_err(KVS_E_INVAL, "null argument");
  *shard = shard_index(c, (const uint8_t *)key, key_len);
  return KVS_OK;
}

int kvs_client_put_profile(kvs_client *c, kvs_put_profile *out) {
  if (!c || !out) return set_err(KVS_E_INVAL, "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  *out = c->prof;
  return KVS_OK;
}

int kvs_ping(kvs_client *c, const void *payload, uint32_t len, void *out, void *stream) {
  TRY(check_client(c));
  if (len > 1024) return set_err(KVS_E_INVAL, "ping: payload of %u bytes exceeds the 1024-byte limit", len);
  if (len && (!payload || !out)) return set_err(KVS_E_INVAL, "ping: null payload or output");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(begin_op(c, stream));
  TRY(c->stage.begin(4096, c->stream));
  const size_t in_off = c->stage.push(payload, len);
  const size_t out_off = c->stage.take(len);
  TRY(c->stage.upload(c->stream, c->stage.used));
  CUDA_TRY(kvs::launch_echo(c->stage.d<uint8_t>(in_off), c->stage.d<uint8_t>(out_off), len, c->stream));
  if (len) CUDA_TRY(cudaMemcpyAsync(out, c->stage.d<uint8_t>(out_off), len, cudaMemcpyDeviceToHost, c->stream));
  CUDA_TRY(cudaStreamSynchronize(c->stream));
  TRY(end_op(c, stream));
  return KVS_OK;
}

static int put_values(kvs_client *c, uint32_t n, const void *const *keys, const uint32_t *key_lens,
                      const void *const *values, const uint64_t *value_lens, int sync_commit, void *stream,
                      const char *op) {
  TRY(check_client(c));
  if (n && (!keys || !key_lens || !values || !value_lens)) return set_err(KVS_E_INVAL, "%s: null argument", op);
  const uint64_t t0 = now_ns();
  for (uint32_t i = 0; i < n; ++i) {
    TRY(validate_key(c, keys[i], key_lens[i], op));
    if (value_lens[i] == 0) return set_err(KVS_E_INVAL, "%s: value_len_bytes must be > 0", op);
    for (auto *s : c->shards)
      if (value_lens[i] > s->cfg.max_value_bytes)
        return set_err(KVS_E_INVAL, "%s: value_len_bytes %llu exceeds max_value_bytes %llu", op,
                       (unsigned long long)value_lens[i], (unsigned long long)s->cfg.max_value_bytes);
  }
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  for (uint32_t i = 0; i < n; ++i) TRY(check_device_ptr(c, values[i], op, "tensor"));
  std::vector<uint8_t> inv(c->shards.size(), 0);
  std::vector<uint32_t> si(n);
  for (uint32_t i = 0; i < n; ++i) {
    si[i] = shard_index(c, (const uint8_t *)keys[i], key_lens[i]);
    inv[si[i]] = 1;
  }
  ShardLocks locks(involved_servers(c, inv));
  TRY(begin_op(c, stream));
  PutBatch b{c, nullptr, nullptr, {}, std::vector<uint8_t>(c->shards.size(), 0)};
  const uint64_t t1 = now_ns();
  for (uint32_t i = 0; i < n; ++i)
    TRY(quarantine_on_error(c, stage_put(b, si[i], (const uint8_t *)keys[i], key_lens[i], value_lens[i], 0,
                                         reinterpret_cast<uint64_t>(values[i]))));
  c->prof.prepare_ns += now_ns() - t1;
  TRY(quarantine_on_error(c, flush_puts(b, c->stream)));
  const uint64_t t2 = now_ns();
  if (sync_commit) TRY(quarantine_on_error(c, commit_barrier(c, inv)));
  c->prof.commit_wait_ns += now_ns() - t2;
  TRY(end_op(c, stream));
  c->prof.count += n;
  c->prof.total_ns += now_ns() - t0;
  return KVS_OK;
}

int kvs_put(kvs_client *c, const void *key, uint32_t key_len, const void *value, uint64_t value_len,
            int sync_commit, void *stream) {
  return put_values(c, 1, &key, &key_len, &value, &value_len, sync_commit, stream, "put");
}

int kvs_put_batch(kvs_client *c, uint32_t n, const void *const *keys, const uint32_t *key_lens,
                  const void *const *values, const uint64_t *value_lens, int sync_commit, void *stream) {
  if (n > 128) return set_err(KVS_E_INVAL, "put_batch: %u items exceed the 128-descriptor limit", n);
  return put_values(c, n, keys, key_lens, values, value_lens, sync_commit, stream, "put_batch");
}

static int get_impl(kvs_client *c, const void *key, uint32_t key_len, void *out, uint64_t capacity, int *found,
                    uint64_t *value_len, void *stream) {
  TRY(check_client(c));
  if (!found) return set_err(KVS_E_INVAL, "get: found is null");
  *found = 0;
  TRY(validate_key(c, key, key_len, "get"));
  if (capacity == 0) return set_err(KVS_E_INVAL, "get: out_tensor packed byte size must be > 0");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(check_device_ptr(c, out, "get", "tensor"));
  const uint32_t si = shard_index(c, (const uint8_t *)key, key_len);
  kvs_server *s = c->shards[si];
  std::lock_guard<std::mutex> sl(s->mu);
  TRY(quarantine_on_error(c, s->commit_all()));  // GET preserves host-commit ordering first
  const uint32_t slot = s->dir->lookup((const uint8_t *)key, key_len);
  if (slot == kvs::kBucketEmpty) return KVS_OK;
  const kvs::Entry &e = s->dir->entry(slot);
  if (value_len) *value_len = e.total_len;
  if (e.total_len > capacity)
    return set_err(KVS_E_TOO_SMALL, "get: out_tensor packed capacity %llu is smaller than the stored value",
                   (unsigned long long)capacity);
  uint64_t admit_off = 0;
  const auto action = s->dir->get_hit(slot, &admit_off);
  const HostBacking &hb = s->dir->backing(slot);
  const uint64_t len = e.total_len;
  TRY(begin_op(c, stream));
  TRY(c->stage.begin(4096 + mutation_upper_bound(s), c->stream));
  PackedMutations pm = pack_mutations(s, c->stage);
  uint64_t src;
  if (action == Directory::GetAction::kHostOnly)
    src = s->device_alias(hb);  // mapped pinned memory, read over PCIe
  else
    src = s->slab_base() + e.value_off;
  const size_t rec = stage_value_copy(c->stage, reinterpret_cast<uint64_t>(out), src, len);
  TRY(c->stage.upload(c->stream, c->stage.used));
  TRY(chain_wait(c, s));
  TRY(quarantine_on_error(c, launch_mutations(c, s, pm)));
  if (action == Directory::GetAction::kAdmit)
    CUDA_TRY(cudaMemcpyAsync(s->slab + admit_off, s->host_ptr(hb), len, cudaMemcpyHostToDevice, c->stream));
  TRY(quarantine_on_error(c, launch_value_copy(c, rec, len, action != Directory::GetAction::kHostOnly)));
  s->launches++;
  TRY(chain_record(c, si));
  CUDA_TRY(cudaStreamSynchronize(c->stream));
  TRY(quarantine_on_error(c, check_tma_timeouts(c, "get")));
  if (action != Directory::GetAction::kDevice) {
    s->mprof.to_device_count++;
    s->moves_completed.fetch_add(1, std::memory_order_relaxed);
  }
  // no end_op: the client stream is idle after the synchronise, so the caller's stream has
  // nothing to wait for
  *found = 1;
  return KVS_OK;
}

int kvs_get(kvs_client *c, const void *key, uint32_t key_len, void *out, uint64_t capacity, int *found,
            uint64_t *value_len, void *stream) {
  return quarantine_on_error(c, get_impl(c, key, key_len, out, capacity, found, value_len, stream));
}

int kvs_get_parallel(kvs_client *const *clients, uint32_t n, const void *const *keys, const uint32_t *key_lens,
                     void *out, uint64_t stride, uint64_t capacity, uint8_t *found, void *stream) {
  if (n == 0 || !clients) return set_err(KVS_E_INVAL, "get_parallel: clients must not be empty");
  if (!keys || !key_lens || !found || !out) return set_err(KVS_E_INVAL, "get_parallel: null argument");
  for (uint32_t i = 0; i < n; ++i) {
    if (!clients[i]) return set_err(KVS_E_INVAL, "get_parallel: client %u is null", i);
    if (clients[i]->device != clients[0]->device)
      return set_err(KVS_E_INVAL, "get_parallel: all Clients must share one client device (client %u differs)", i);
  }
  for (uint32_t i = 0; i < n; ++i) {
    int f = 0;
    TRY(kvs_get(clients[i], keys[i], key_lens[i], (uint8_t *)out + i * stride, capacity, &f, nullptr, stream));
    found[i] = (uint8_t)f;
  }
  return KVS_OK;
}

static int single_key_op(kvs_client *c, const void *key, uint32_t key_len, const char *op,
                         kvs_server **s_out, uint32_t *slot_out, uint32_t *si_out) {
  TRY(check_client(c));
  TRY(validate_key(c, key, key_len, op));
  const uint32_t si = shard_index(c, (const uint8_t *)key, key_len);
  kvs_server *s = c->shards[si];
  TRY(quarantine_on_error(c, s->commit_all()));
  *s_out = s;
  *si_out = si;
  *slot_out = s->dir->lookup((const uint8_t *)key, key_len);
  return KVS_OK;
}

int kvs_exists(kvs_client *c, const void *key, uint32_t key_len, int *found) {
  if (!found) return set_err(KVS_E_INVAL, "exists: found is null");
  *found = 0;
  if (!c) return set_err(KVS_E_INVAL, "client handle is null");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(check_client(c));
  TRY(validate_key(c, key, key_len, "exists"));
  kvs_server *s = c->shards[shard_index(c, (const uint8_t *)key, key_len)];
  std::lock_guard<std::mutex> sl(s->mu);
  kvs_server *s2;
  uint32_t slot, si;
  TRY(single_key_op(c, key, key_len, "exists", &s2, &slot, &si));
  *found = slot != kvs::kBucketEmpty;
  return KVS_OK;
}

int kvs_delete(kvs_client *c, const void *key, uint32_t key_len, int *removed) {
  if (!removed) return set_err(KVS_E_INVAL, "delete: removed is null");
  *removed = 0;
  if (!c) return set_err(KVS_E_INVAL, "client handle is null");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(check_client(c));
  TRY(validate_key(c, key, key_len, "remove"));
  kvs_server *s = c->shards[shard_index(c, (const uint8_t *)key, key_len)];
  std::lock_guard<std::mutex> sl(s->mu);
  kvs_server *s2;
  uint32_t slot, si;
  TRY(single_key_op(c, key, key_len, "remove", &s2, &slot, &si));
  if (slot == kvs::kBucketEmpty) return KVS_OK;
  s->dir->remove(slot);
  s->release_dropped();
  *removed = 1;
  return KVS_OK;
}

int kvs_move_to_host(kvs_client *c, const void *key, uint32_t key_len) {
  if (!c) return set_err(KVS_E_INVAL, "client handle is null");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(check_client(c));
  TRY(validate_key(c, key, key_len, "move"));
  kvs_server *s = c->shards[shard_index(c, (const uint8_t *)key, key_len)];
  std::lock_guard<std::mutex> sl(s->mu);
  kvs_server *s2;
  uint32_t slot, si;
  TRY(single_key_op(c, key, key_len, "move", &s2, &slot, &si));
  if (slot != kvs::kBucketEmpty) s->dir->move_to_host(slot);
  return KVS_OK;
}

static int move_to_device_impl(kvs_client *c, const void *key, uint32_t key_len) {
  if (!c) return set_err(KVS_E_INVAL, "client handle is null");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(check_client(c));
  TRY(validate_key(c, key, key_len, "move"));
  const uint32_t si0 = shard_index(c, (const uint8_t *)key, key_len);
  kvs_server *s = c->shards[si0];
  std::lock_guard<std::mutex> sl(s->mu);
  kvs_server *s2;
  uint32_t slot, si;
  TRY(single_key_op(c, key, key_len, "move", &s2, &slot, &si));
  if (slot == kvs::kBucketEmpty) return KVS_OK;
  uint64_t off = 0;
  if (!s->dir->move_to_device(slot, &off)) return KVS_OK;
  const HostBacking &hb = s->dir->backing(slot);
  const uint64_t t0 = now_ns();
  TRY(c->stage.begin(4096 + mutation_upper_bound(s), c->stream));
  PackedMutations pm = pack_mutations(s, c->stage);
  TRY(c->stage.upload(c->stream, c->stage.used));
  TRY(chain_wait(c, s));
  TRY(quarantine_on_error(c, launch_mutations(c, s, pm)));
  CUDA_TRY(cudaMemcpyAsync(s->slab + off, s->host_ptr(hb), s->dir->entry(slot).total_len, cudaMemcpyHostToDevice,
                           c->stream));
  TRY(chain_record(c, si));
  CUDA_TRY(cudaStreamSynchronize(c->stream));
  s->mprof.to_device_count++;
  s->mprof.to_device_worker_ns += now_ns() - t0;
  s->mprof.to_device_complete_ns += now_ns() - t0;
  s->moves_completed.fetch_add(1, std::memory_order_relaxed);
  return KVS_OK;
}

int kvs_move_to_device(kvs_client *c, const void *key, uint32_t key_len) {
  return quarantine_on_error(c, move_to_device_impl(c, key, key_len));
}

int kvs_flush(kvs_client *c) {
  if (!c) return set_err(KVS_E_INVAL, "client handle is null");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(check_client(c));
  std::vector<uint8_t> inv(c->shards.size(), 1);
  ShardLocks locks(involved_servers(c, inv));
  return quarantine_on_error(c, commit_barrier(c, inv));
}

// ---------------------------------------------------------------------------- block path

static int check_blocks(const kvs_block_layout *L, uint32_t n, const uint64_t *keys, const int64_t *block_ids,
                        const char *op) {
  if (n == 0) return set_err(KVS_E_INVAL, "%s: empty batch", op);
  if (!keys || !block_ids) return set_err(KVS_E_INVAL, "%s: keys and block_ids must be non-null", op);
  for (uint32_t i = 0; i < n; ++i)
    if (block_ids[i] < 0 || (uint64_t)block_ids[i] >= L->n_pool_blocks)
      return set_err(KVS_E_INVAL, "%s: block id %lld at %u is outside the %llu-block pool", op,
                     (long long)block_ids[i], i, (unsigned long long)L->n_pool_blocks);
  return KVS_OK;
}

int kvs_put_blocks(kvs_client *c, const kvs_block_layout *layout, uint32_t n, const uint64_t *keys,
                   const int64_t *block_ids, int sync_commit, void *stream) {
  TRY(check_client(c));
  const BlockFormat *fmtp = nullptr;
  TRY(cached_block_format(layout, &fmtp));
  const BlockFormat &fmt = *fmtp;
  TRY(check_blocks(layout, n, keys, block_ids, "put_blocks"));
  for (auto *s : c->shards)
    if (fmt.value_len > s->cfg.max_value_bytes)
      return set_err(KVS_E_INVAL, "put_blocks: block value of %llu B exceeds max_value_bytes %llu",
                     (unsigned long long)fmt.value_len, (unsigned long long)s->cfg.max_value_bytes);
  const uint64_t t0 = now_ns();
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(validate_layout_ptrs(c, layout, "put_blocks"));
  std::vector<uint8_t> inv(c->shards.size(), 0);
  std::vector<uint32_t> si(n);
  for (uint32_t i = 0; i < n; ++i) {
    si[i] = shard_index(c, (const uint8_t *)&keys[i], 8);
    inv[si[i]] = 1;
  }
  ShardLocks locks(involved_servers(c, inv));
  TRY(begin_op(c, stream));
  PutBatch b{c, layout, &fmt, {}, std::vector<uint8_t>(c->shards.size(), 0)};
  b.items.reserve(n);
  const uint64_t t1 = now_ns();
  uint64_t piece_ns = 0;  // time in the pieces' flushes, which the put profile counts as program time
  for (uint32_t i = 0; i < n; ++i) {
    TRY(quarantine_on_error(c, stage_put(b, si[i], (const uint8_t *)&keys[i], 8, fmt.value_len, block_ids[i], 0)));
    // a large batch launches its gather every kPutPieceBlocks blocks, so the device copies one
    // piece while the host prepares the next (the catalog sees the same sequence either way)
    if (b.items.size() >= kPutPieceBlocks && i + 1 < n) {
      const uint64_t f0 = now_ns();
      TRY(quarantine_on_error(c, flush_puts(b, c->stream)));
      piece_ns += now_ns() - f0;
    }
  }
  c->prof.prepare_ns += now_ns() - t1 - piece_ns;
  TRY(quarantine_on_error(c, flush_puts(b, c->stream)));
  const uint64_t t2 = now_ns();
  if (sync_commit) TRY(quarantine_on_error(c, commit_barrier(c, inv)));
  c->prof.commit_wait_ns += now_ns() - t2;
  TRY(end_op(c, stream));
  c->prof.count += n;
  c->prof.total_ns += now_ns() - t0;
  return KVS_OK;
}

// Keys of a batch ordered by shard (stable), so each shard's device lookup reads one contiguous
// run. perm[j] is the batch position of the j-th key in shard order.
struct ShardOrder {
  std::vector<uint32_t> perm;
  std::vector<uint32_t> run_begin, run_shard;  // runs of one shard in `perm` order
};

static ShardOrder order_by_shard(const std::vector<uint32_t> &si, size_t n_shards) {
  ShardOrder o;
  const uint32_t n = (uint32_t)si.size();
  o.perm.resize(n);
  if (n_shards == 1) {
    for (uint32_t i = 0; i < n; ++i) o.perm[i] = i;
    o.run_begin = {0, n};
    o.run_shard = {0};
    return o;
  }
  std::vector<uint32_t> count(n_shards + 1, 0);
  for (uint32_t x : si) count[x + 1]++;
  for (size_t k = 0; k < n_shards; ++k) count[k + 1] += count[k];
  std::vector<uint32_t> pos(count.begin(), count.end() - 1);
  for (uint32_t i = 0; i < n; ++i) o.perm[pos[si[i]]++] = i;
  for (size_t k = 0; k < n_shards; ++k)
    if (count[k + 1] > count[k]) {
      o.run_begin.push_back(count[k]);
      o.run_shard.push_back((uint32_t)k);
    }
  o.run_begin.push_back(n);
  return o;
}

// Probe parameters for n 8-byte keys of shard s (d_keys nullptr: the caller fills inline_keys).
static kvs::LookupParams lookup_params(kvs_server *s, const uint8_t *d_keys, uint32_t n, kvs::LookupOut *d_out,
                                       uint64_t *d_blob, uint64_t expected_len) {
  kvs::LookupParams lp{};
  lp.keys = d_keys;
  lp.key_lens = nullptr;
  lp.key_stride = 8;
  lp.n = n;
  lp.buckets = s->d_buckets;
  lp.bucket_mask = s->dir->num_buckets() - 1;
  lp.meta = s->d_meta;
  lp.key_rows = s->d_keyrows;
  lp.max_keys = s->cfg.max_keys;
  lp.slab_base = s->slab_base();
  lp.expected_len = expected_len;
  lp.out = d_out;
  lp.blob_ptrs = d_blob;
  return lp;
}

// Launch the device index probe for every shard run. keys/out/blob arrays are in shard order.
static int launch_lookups(kvs_client *c, const ShardOrder &o, const uint8_t *d_keys, kvs::LookupOut *d_out,
                          uint64_t *d_blob, uint64_t expected_len) {
  for (size_t r = 0; r + 1 < o.run_begin.size(); ++r) {
    const uint32_t b0 = o.run_begin[r], b1 = o.run_begin[r + 1];
    kvs_server *s = c->shards[o.run_shard[r]];
    const kvs::LookupParams lp = lookup_params(s, d_keys + 8ull * b0, b1 - b0, d_out + b0,
                                               d_blob ? d_blob + b0 : nullptr, expected_len);
    CUDA_TRY(kvs::launch_index_lookup(lp, c->stream));
    s->launches++;
  }
  return KVS_OK;
}

// Destination side of a block get: the value format, the member block sizes, and one or more
// member sets (one per requesting paged pool; the owner of a shard serving several processes
// scatters into each requester's pool over NVLink in one launch).
struct GetTarget {
  const BlockFormat *fmt;
  uint32_t n_members;
  const uint64_t *member_bytes;  // [n_members]
  uint32_t n_sets;
  const uint64_t *member_ptrs;   // [n_sets * n_members]
  const uint32_t *sets;          // [n] member set of each key, or nullptr (set 0)
};

// Gets of at most kInlineKeys keys on one shard whose hits are all device-resident: the host
// catalog, which every get consults anyway, answers the few lookups in well under a microsecond,
// so the scatter launches at once with the block ids and slab addresses in its parameters -- no
// probe kernel, replica update or host-to-device copy goes before it, and the device replica's
// pending updates wait for the next probe. A host-tier hit or a length mismatch leaves *served = 0
// and the catalog untouched, and the general path runs. Runs after the commit barrier, with the
// shard locked and the layout's arrays on the device (c->layout_dev).
static int small_device_get(kvs_client *c, const GetTarget &t, uint32_t n, const uint64_t *keys,
                            const int64_t *block_ids, uint32_t shard, uint8_t *found, void *stream, int *served) {
  *served = 0;
  kvs_server *s = c->shards[shard];
  const BlockFormat &fmt = *t.fmt;
  uint32_t slots[kvs::kInlineKeys];
  for (uint32_t i = 0; i < n; ++i) {
    slots[i] = s->dir->lookup((const uint8_t *)&keys[i], 8);
    if (slots[i] == kvs::kBucketEmpty) continue;
    const kvs::Entry &e = s->dir->entry(slots[i]);
    if (e.total_len != fmt.value_len || e.location == kvs::kLocHost) return KVS_OK;
  }
  *served = 1;
  kvs::ChunkCopyParams p{};
  uint64_t payload_per_block = 0, hits = 0;
  for (uint32_t m = 0; m < t.n_members; ++m) payload_per_block += t.member_bytes[m];
  s->dir->take_evicted();
  for (uint32_t i = 0; i < n; ++i) {
    found[i] = 0;
    p.inline_ids[i] = block_ids[i];
    p.inline_blobs[i] = 0;  // a miss copies nothing
    if (slots[i] == kvs::kBucketEmpty) continue;
    uint64_t off = 0;
    // recency in batch order, as the general path applies it: a device-resident hit moves to MRU
    if (s->dir->get_hit(slots[i], &off) != Directory::GetAction::kDevice || !s->dir->take_evicted().empty())
      return set_err(KVS_E_CUDA, "get_blocks: catalog placed device-resident key %u off the device", i);
    p.inline_blobs[i] = s->slab_base() + s->dir->entry(slots[i]).value_off;
    found[i] = 1;
    ++hits;
  }
  if (!hits) return KVS_OK;  // every key missed: nothing to copy, no device work to order
  // The copy runs on the caller's stream, so it starts after the caller's earlier work on the
  // destination blocks, and the call synchronises that stream before it returns. Device work of
  // other clients on this shard is ordered first through the shard's event chain; the shard stays
  // locked until the copy has finished, so the chain needs no new position.
  cudaStream_t cs = (cudaStream_t)stream;
  if (s->tail && std::find(c->chain_evt.begin(), c->chain_evt.end(), s->tail) == c->chain_evt.end())
    CUDA_TRY(cudaStreamWaitEvent(cs, s->tail, 0));
  const size_t lay_mb = 8ull * t.n_members, lay_rb = lay_mb + 8ull * t.n_members, lay_tp = lay_rb + 8ull * t.n_members;
  p.member_ptrs = reinterpret_cast<const uint64_t *>(c->layout_dev);
  p.member_bytes = reinterpret_cast<const uint64_t *>(c->layout_dev + lay_mb);
  p.region_bases = reinterpret_cast<const uint64_t *>(c->layout_dev + lay_rb);
  p.tile_prefix = reinterpret_cast<const uint64_t *>(c->layout_dev + lay_tp);
  p.block_ids = nullptr;
  p.blob_ptrs = nullptr;
  p.n_blobs = n;
  p.blocks_per_blob = 1;
  p.n_ranks = 1;
  p.n_members = t.n_members;
  p.tile_bytes = kTileBytes;
  p.tiles_per_combo = fmt.tile_prefix.back();
  p.total_tiles = (uint64_t)n * p.tiles_per_combo;
  p.to_blob = 0;
  set_copy_facts(&p, t.member_bytes, t.n_members, n);
  cudaEvent_t t0 = nullptr;
  c->time_begin_on(&t0, cs);
  CUDA_TRY(launch_copy(p, cs, true, c->timeout_flag));
  c->time_end_on(t0, 1, hits * payload_per_block, cs);
  s->launches++;
  CUDA_TRY(cudaStreamSynchronize(cs));
  TRY(check_tma_timeouts(c, "get_blocks"));
  return KVS_OK;
}

static int get_blocks_impl(kvs_client *c, const GetTarget &t, uint32_t n, const uint64_t *keys,
                           const int64_t *block_ids, uint8_t *found, void *stream) {
  const BlockFormat &fmt = *t.fmt;
  const size_t ns = c->shards.size();
  std::vector<uint8_t> inv(ns, 0);
  std::vector<uint32_t> si(n);
  for (uint32_t i = 0; i < n; ++i) {
    si[i] = shard_index(c, (const uint8_t *)&keys[i], 8);
    inv[si[i]] = 1;
  }
  const ShardOrder ord = order_by_shard(si, ns);
  ShardLocks locks(involved_servers(c, inv));
  TRY(quarantine_on_error(c, commit_barrier(c, inv)));  // GET preserves host-commit ordering first
  const uint64_t ptr_bytes = 8ull * t.n_sets * t.n_members;
  // the layout arrays, back to back as the device copy holds them
  const size_t lay_mb = ptr_bytes, lay_rb = lay_mb + 8ull * t.n_members, lay_tp = lay_rb + 8ull * t.n_members;
  const size_t lay_bytes = lay_tp + 8ull * (t.n_members + 1);
  thread_local std::vector<uint8_t> lay;
  lay.resize(lay_bytes);
  std::memcpy(lay.data(), t.member_ptrs, ptr_bytes);
  std::memcpy(lay.data() + lay_mb, t.member_bytes, 8ull * t.n_members);
  std::memcpy(lay.data() + lay_rb, fmt.region_bases.data(), 8ull * t.n_members);
  std::memcpy(lay.data() + lay_tp, fmt.tile_prefix.data(), 8ull * (t.n_members + 1));
  // A small get on one shard with a layout already on the device needs no host-to-device copy:
  // its keys and block ids travel in the kernel parameters.
  const bool layout_cached = !t.sets && c->layout_key.size() == lay_bytes &&
                             std::memcmp(c->layout_key.data(), lay.data(), lay_bytes) == 0;
  if (layout_cached && n <= kvs::kInlineKeys && ord.run_shard.size() == 1) {
    int served = 0;
    const int rc = small_device_get(c, t, n, keys, block_ids, ord.run_shard[0], found, stream, &served);
    if (served || rc != KVS_OK) return rc;
  }
  TRY(begin_op(c, stream));
  // ---- pass 1: replica update, device lookup, scatter of device hits
  Staging &st = c->stage;
  size_t need = 4096 + 68ull * n + ptr_bytes + 32ull * t.n_members;
  for (size_t i = 0; i < ns; ++i)
    if (inv[i]) need += mutation_upper_bound(c->shards[i]);
  TRY(st.begin(need, c->stream));
  // with no index updates to apply either, the probe's keys travel in its parameters too
  bool inline_call = layout_cached && n <= kvs::kInlineKeys && ord.run_shard.size() == 1;
  if (inline_call) {
    size_t nb, nm, nk;
    c->shards[ord.run_shard[0]]->dir->dirty_counts(&nb, &nm, &nk);
    inline_call = nb + nm + nk == 0;
  }
  std::vector<PackedMutations> pms(ns);
  size_t keys_off = 0, ids_off = 0, sets_off = 0, lay_off = 0;
  const uint8_t *lay_dev = c->layout_dev;
  if (!inline_call) {
    for (size_t i = 0; i < ns; ++i)
      if (inv[i]) pms[i] = pack_mutations(c->shards[i], st);
    keys_off = st.take(8ull * n);
    ids_off = st.take(8ull * n);
    for (uint32_t j = 0; j < n; ++j) {
      st.h<uint64_t>(keys_off)[j] = keys[ord.perm[j]];
      st.h<int64_t>(ids_off)[j] = block_ids[ord.perm[j]];
    }
    if (t.sets) {
      sets_off = st.take(4ull * n);
      for (uint32_t j = 0; j < n; ++j) st.h<uint32_t>(sets_off)[j] = t.sets[ord.perm[j]];
    }
    lay_off = st.push(lay.data(), lay_bytes);
    lay_dev = st.d<uint8_t>(lay_off);
  }
  const size_t upload_bytes = st.used;
  const size_t out_off = st.take(sizeof(kvs::LookupOut) * n);
  const size_t blob_off = st.take(8ull * n);
  if (!inline_call) {
    TRY(st.upload(c->stream, upload_bytes));
    if (!t.sets && !layout_cached) {  // keep the layout on the device for the next small gets
      if (lay_bytes > c->layout_cap) {
        CUDA_TRY(cudaStreamSynchronize(c->stream));  // the old copy may still be read
        if (c->layout_dev) cudaFree(c->layout_dev);
        c->layout_dev = nullptr;
        c->layout_cap = 0;
        c->layout_key.clear();
        CUDA_TRY(cudaMalloc(&c->layout_dev, std::max<size_t>(lay_bytes, 16 << 10)));
        c->layout_cap = std::max<size_t>(lay_bytes, 16 << 10);
      }
      CUDA_TRY(cudaMemcpyAsync(c->layout_dev, st.d<uint8_t>(lay_off), lay_bytes, cudaMemcpyDeviceToDevice,
                               c->stream));
      c->layout_key.assign(lay.begin(), lay.end());
    }
  }
  for (size_t i = 0; i < ns; ++i)
    if (inv[i]) TRY(chain_wait(c, c->shards[i]));
  if (inline_call) {
    kvs_server *s = c->shards[ord.run_shard[0]];
    kvs::LookupParams lp = lookup_params(s, nullptr, n, st.hd<kvs::LookupOut>(out_off), st.d<uint64_t>(blob_off),
                                         fmt.value_len);
    for (uint32_t j = 0; j < n; ++j) lp.inline_keys[j] = keys[ord.perm[j]];
    CUDA_TRY(kvs::launch_index_lookup(lp, c->stream));
    s->launches++;
  } else {
    for (size_t i = 0; i < ns; ++i)
      if (inv[i]) TRY(quarantine_on_error(c, launch_mutations(c, c->shards[i], pms[i])));
    TRY(quarantine_on_error(c, launch_lookups(c, ord, st.d<uint8_t>(keys_off), st.hd<kvs::LookupOut>(out_off),
                                              st.d<uint64_t>(blob_off), fmt.value_len)));
  }
  kvs::ChunkCopyParams p{};
  p.member_ptrs = reinterpret_cast<const uint64_t *>(lay_dev);
  p.blob_sets = t.sets ? st.d<uint32_t>(sets_off) : nullptr;
  p.member_bytes = reinterpret_cast<const uint64_t *>(lay_dev + lay_mb);
  p.region_bases = reinterpret_cast<const uint64_t *>(lay_dev + lay_rb);
  p.tile_prefix = reinterpret_cast<const uint64_t *>(lay_dev + lay_tp);
  if (inline_call) {
    p.block_ids = nullptr;
    for (uint32_t j = 0; j < n; ++j) p.inline_ids[j] = block_ids[ord.perm[j]];
  } else {
    p.block_ids = st.d<int64_t>(ids_off);
  }
  p.blob_ptrs = st.d<uint64_t>(blob_off);
  p.n_blobs = n;
  p.blocks_per_blob = 1;
  p.n_ranks = 1;
  p.n_members = t.n_members;
  p.tile_bytes = kTileBytes;
  p.tiles_per_combo = fmt.tile_prefix.back();
  p.total_tiles = (uint64_t)n * p.tiles_per_combo;
  p.to_blob = 0;
  set_copy_facts(&p, t.member_bytes, t.n_members, n);
  uint64_t payload_per_block = 0;
  for (uint32_t m = 0; m < t.n_members; ++m) payload_per_block += t.member_bytes[m];
  cudaEvent_t t0 = nullptr;
  c->time_begin(&t0);
  CUDA_TRY(launch_copy(p, c->stream, true, c->timeout_flag));
  c->time_end(t0, 1, (uint64_t)n * payload_per_block);  // misses copy nothing; corrected below
  for (size_t i = 0; i < ns; ++i)
    if (inv[i]) c->shards[i]->launches++;
  for (size_t i = 0; i < ns; ++i)
    if (inv[i]) TRY(chain_record(c, i));
  // While the GPU works: the authoritative host lookups decide every outcome (the device replica
  // mirrors the catalog, so a key the catalog places on the host tier is one pass 1 did not
  // deliver). The device results are checked against them once, after the last pass.
  std::vector<uint32_t> host_slot(n);
  std::vector<kvs::LookupOut> res(n);
  for (uint32_t i = 0; i < n; ++i) {
    kvs_server *s = c->shards[si[i]];
    host_slot[i] = s->dir->lookup((const uint8_t *)&keys[i], 8);
    kvs::LookupOut &r = res[i];
    r.status = kvs::kMiss;
    r.slot = host_slot[i];
    if (host_slot[i] == kvs::kBucketEmpty) continue;
    const kvs::Entry &e = s->dir->entry(host_slot[i]);
    r.value_len = (uint32_t)e.total_len;
    if (e.total_len != fmt.value_len)
      r.status = kvs::kLenMismatch;
    else
      r.status = e.location == kvs::kLocHost ? kvs::kHitHost : kvs::kHitDevice;
  }
  int format_error = -1;
  for (uint32_t i = 0; i < n && format_error < 0; ++i)
    if (res[i].status == kvs::kLenMismatch) format_error = (int)i;
  if (c->timing && !c->timed.empty() && c->timed.back().kind == 1) {
    uint64_t hits = 0;
    for (uint32_t i = 0; i < n; ++i) hits += res[i].status == kvs::kHitDevice;
    c->timed.back().bytes = hits * payload_per_block;
  }
  // ---- host processing in batch order: recency, read-through admission
  struct Late {
    uint32_t i, shard, slot;
    uint64_t admit_dst;  // slab address filled from the host copy (0: none)
    const uint8_t *host;
    uint64_t len;
    bool scatter;  // pass 1 did not deliver it (host-tier hit)
    uint64_t host_dev;  // device alias of the host copy
    uint64_t slab_src;  // pass 2 scatters from this slab block (0: from the host copy)
    bool moved;  // a host-tier serve (counted as a move to the device side)
  };
  std::vector<Late> late;
  // (shard, slot) -> late entries that read the slot's slab block in pass 2
  std::multimap<std::pair<uint32_t, uint32_t>, size_t> reads;
  for (size_t i = 0; i < ns; ++i)
    if (inv[i]) c->shards[i]->dir->take_evicted();
  for (uint32_t i = 0; i < n; ++i) {
    found[i] = 0;
    if (res[i].status == kvs::kMiss || res[i].status == kvs::kLenMismatch) continue;
    kvs_server *s = c->shards[si[i]];
    uint64_t off = 0;
    const auto action = s->dir->get_hit(host_slot[i], &off);
    found[i] = 1;
    // a block admitted earlier in this batch and just evicted again: the gets that were to read
    // it read the host copy instead, and its admission copy is dropped
    for (uint32_t ev : s->dir->take_evicted()) {
      auto range = reads.equal_range({si[i], ev});
      for (auto it = range.first; it != range.second; ++it) {
        late[it->second].admit_dst = 0;
        late[it->second].slab_src = 0;
      }
      reads.erase(range.first, range.second);
    }
    const HostBacking &hb = s->dir->backing(host_slot[i]);
    Late L{i, si[i], host_slot[i], 0, s->host_ptr(hb), s->dir->entry(host_slot[i]).total_len,
           res[i].status == kvs::kHitHost, s->device_alias(hb), 0, true};
    if (action == Directory::GetAction::kDevice) {
      if (!L.scatter) continue;  // delivered by pass 1
      // pass 1 saw the host tier, and an earlier get of this batch has admitted the value since:
      // read the block that admission fills
      L.slab_src = s->slab_base() + s->dir->entry(host_slot[i]).value_off;
      L.moved = false;
      reads.insert({{si[i], host_slot[i]}, late.size()});
    } else if (action == Directory::GetAction::kAdmit) {
      L.admit_dst = L.slab_src = s->slab_base() + off;
      reads.insert({{si[i], host_slot[i]}, late.size()});
    }
    late.push_back(L);
  }
  if (!late.empty()) {
    // ---- pass 2, queued behind pass 1 on the client stream from the second staging area:
    // replica update, admissions (host -> slab), scatter of host-tier hits
    Staging &st2 = c->stage2;
    size_t need2 = 4096 + 72ull * late.size() + ptr_bytes + 32ull * t.n_members;
    for (size_t i = 0; i < ns; ++i)
      if (inv[i]) need2 += mutation_upper_bound(c->shards[i]);
    TRY(st2.begin(need2, c->stream));
    std::vector<PackedMutations> pms2(ns);
    for (size_t i = 0; i < ns; ++i)
      if (inv[i]) pms2[i] = pack_mutations(c->shards[i], st2);
    size_t nscatter = 0;
    for (auto &L : late) nscatter += L.scatter;
    const size_t blobs2 = st2.take(8 * std::max<size_t>(nscatter, 1));
    const size_t ids2 = st2.take(8 * std::max<size_t>(nscatter, 1));
    const size_t sets2 = st2.take(4 * std::max<size_t>(nscatter, 1));
    size_t k = 0;
    for (auto &L : late)
      if (L.scatter) {
        // values in the slab (admitted in this batch) are scattered from their block, others
        // from host memory
        st2.h<uint64_t>(blobs2)[k] = L.slab_src ? L.slab_src : L.host_dev;
        st2.h<int64_t>(ids2)[k] = block_ids[L.i];
        st2.h<uint32_t>(sets2)[k] = t.sets ? t.sets[L.i] : 0;
        ++k;
      }
    const size_t mp2 = st2.push(t.member_ptrs, ptr_bytes);
    const size_t mb2 = st2.push(t.member_bytes, 8ull * t.n_members);
    const size_t rb2 = st2.push(fmt.region_bases.data(), 8ull * t.n_members);
    const size_t tp2 = st2.push(fmt.tile_prefix.data(), 8ull * (t.n_members + 1));
    // admissions as one copy list: value a goes from its pinned host copy (device alias) to its
    // new slab block; each value is its own one-member set whose member pointer is the block
    size_t n_admit = 0;
    for (auto &L : late) n_admit += (L.admit_dst && L.host_dev);
    const size_t adm_dst = st2.take(8 * std::max<size_t>(n_admit, 1));
    const size_t adm_src = st2.take(8 * std::max<size_t>(n_admit, 1));
    const size_t adm_set = st2.take(4 * std::max<size_t>(n_admit, 1));
    const size_t adm_ids = st2.take(8 * std::max<size_t>(n_admit, 1));
    const uint64_t adm_meta[5] = {fmt.value_len, 0, 0, (fmt.value_len + kTileBytes - 1) / kTileBytes, 0};
    const size_t adm_m = st2.push(adm_meta, sizeof adm_meta);
    {
      size_t a = 0;
      for (auto &L : late)
        if (L.admit_dst && L.host_dev) {
          st2.h<uint64_t>(adm_dst)[a] = L.admit_dst;
          st2.h<uint64_t>(adm_src)[a] = L.host_dev;
          st2.h<uint32_t>(adm_set)[a] = (uint32_t)a;
          st2.h<int64_t>(adm_ids)[a] = 0;
          ++a;
        }
    }
    TRY(st2.upload(c->stream, st2.used));
    for (size_t i = 0; i < ns; ++i)
      if (inv[i]) TRY(chain_wait(c, c->shards[i]));
    for (size_t i = 0; i < ns; ++i)
      if (inv[i]) TRY(quarantine_on_error(c, launch_mutations(c, c->shards[i], pms2[i], &st2)));
    if (n_admit) {
      kvs::ChunkCopyParams a{};
      a.member_ptrs = st2.d<uint64_t>(adm_dst);
      a.blob_sets = st2.d<uint32_t>(adm_set);
      a.member_bytes = st2.d<uint64_t>(adm_m);
      a.region_bases = st2.d<uint64_t>(adm_m + 8);
      a.tile_prefix = st2.d<uint64_t>(adm_m + 16);
      a.block_ids = st2.d<int64_t>(adm_ids);
      a.blob_ptrs = st2.d<uint64_t>(adm_src);
      a.n_blobs = (uint32_t)n_admit;
      a.blocks_per_blob = 1;
      a.n_ranks = 1;
      a.n_members = 1;
      a.tile_bytes = kTileBytes;
      a.tiles_per_combo = adm_meta[3];
      a.total_tiles = (uint64_t)n_admit * a.tiles_per_combo;
      a.to_blob = 0;
      cudaEvent_t ta = nullptr;
      c->time_begin(&ta);
      CUDA_TRY(launch_copy(a, c->stream, false, c->timeout_flag));  // the source is host memory
      c->time_end(ta, 2, (uint64_t)n_admit * fmt.value_len);
    }
    for (auto &L : late)
      if (L.admit_dst && !L.host_dev)  // no device alias: a copy-engine copy
        CUDA_TRY(cudaMemcpyAsync(reinterpret_cast<void *>(L.admit_dst), L.host, L.len, cudaMemcpyHostToDevice,
                                 c->stream));
    if (nscatter) {
      kvs::ChunkCopyParams q = p;
      q.member_ptrs = st2.d<uint64_t>(mp2);
      q.blob_sets = t.sets ? st2.d<uint32_t>(sets2) : nullptr;
      q.member_bytes = st2.d<uint64_t>(mb2);
      q.region_bases = st2.d<uint64_t>(rb2);
      q.tile_prefix = st2.d<uint64_t>(tp2);
      q.block_ids = st2.d<int64_t>(ids2);
      q.blob_ptrs = st2.d<uint64_t>(blobs2);
      q.n_blobs = (uint32_t)nscatter;
      q.total_tiles = (uint64_t)nscatter * q.tiles_per_combo;
      q.max_member_bytes = q.payload_bytes = 0;  // sources may be pinned host memory: LDG engine
      cudaEvent_t tq = nullptr;
      c->time_begin(&tq);
      CUDA_TRY(launch_copy(q, c->stream, false, c->timeout_flag));
      c->time_end(tq, 3, (uint64_t)nscatter * payload_per_block);
    }
    for (size_t i = 0; i < ns; ++i)
      if (inv[i]) TRY(chain_record(c, i));
    for (auto &L : late) {
      if (!L.moved) continue;
      kvs_server *s = c->shards[L.shard];
      s->mprof.to_device_count++;
      s->moves_completed.fetch_add(1, std::memory_order_relaxed);
    }
  }
  CUDA_TRY(cudaStreamSynchronize(c->stream));
  TRY(quarantine_on_error(c, check_tma_timeouts(c, "get_blocks")));
  // the device probe must have found exactly what the catalog holds
  for (uint32_t j = 0; j < n; ++j) {
    const kvs::LookupOut &d = st.h<kvs::LookupOut>(out_off)[j];
    const uint32_t i = ord.perm[j];
    const bool dev_hit = d.status != kvs::kMiss;
    const bool host_hit = host_slot[i] != kvs::kBucketEmpty;
    if (dev_hit != host_hit || (dev_hit && (d.slot != host_slot[i] || d.status != res[i].status))) {
      c->quarantined = true;
      return set_err(KVS_E_CUDA, "get_blocks: device index replica disagrees with the catalog for key %u", i);
    }
  }
  // no end_op: the client stream is idle after the synchronise above
  if (format_error >= 0)
    return set_err(KVS_E_FORMAT, "get_blocks: stored value for key %d has length %u, the block layout needs %llu",
                   format_error, res[format_error].value_len, (unsigned long long)fmt.value_len);
  return KVS_OK;
}

// ---------------------------------------------------------------------------- chunk restore

// Restore of n chunk values straight into a paged cache (kvs_restore_chunks in kvs.h): the catalog
// decides every outcome in key order as a sequence of gets would (commit barrier, recency,
// read-through admission); then one paged-fill launch per 64 layers reads each chunk's K / V rows
// where the value lives -- its slab block, or its pinned host copy when no block could be
// allocated or a later admission of the same call took the block again.
static int restore_chunks_impl(kvs_client *c, uint32_t n, const void *const *keys, const uint32_t *key_lens,
                               const uint32_t *tokens, uint32_t n_layers, void *const *cache_ks,
                               void *const *cache_vs, uint32_t num_blocks, uint32_t block_size, uint32_t row_bytes,
                               const int32_t *page_table, uint32_t max_blocks, const int32_t *start_positions,
                               uint8_t *found, void *stream) {
  const char *op = "restore_chunks";
  if (n == 0) return KVS_OK;
  if (!keys || !key_lens || !tokens || !cache_ks || !cache_vs || !page_table || !start_positions || !found)
    return set_err(KVS_E_INVAL, "%s: null argument", op);
  if (n_layers == 0 || block_size == 0 || max_blocks == 0 || num_blocks == 0)
    return set_err(KVS_E_INVAL, "%s: n_layers, block_size, max_blocks_per_chunk and num_blocks must be > 0", op);
  if (row_bytes == 0 || row_bytes % 16)
    return set_err(KVS_E_INVAL, "%s: row_bytes %u must be a nonzero multiple of 16", op, row_bytes);
  for (uint32_t i = 0; i < n; ++i) TRY(validate_key(c, keys[i], key_lens[i], op));
  for (uint32_t l = 0; l < n_layers; ++l) {
    if (((reinterpret_cast<uint64_t>(cache_ks[l]) | reinterpret_cast<uint64_t>(cache_vs[l])) & 15u) != 0)
      return set_err(KVS_E_INVAL, "%s: cache tensors of layer %u must be 16-byte aligned", op, l);
    TRY(check_device_ptr(c, cache_ks[l], op, "cache_k"));
    TRY(check_device_ptr(c, cache_vs[l], op, "cache_v"));
  }
  // value layout of the raw-byte chunk codec: header [MAGIC, n_layers, 2 alloc x n_layers] padded
  // to 32 bytes, then per layer K (alloc bytes) and V (alloc bytes)
  const uint64_t hdr = 4ull * (((2ull + n_layers) + 7) / 8 * 8);
  std::vector<uint64_t> alloc(n), vlen(n);
  for (uint32_t i = 0; i < n; ++i) {
    alloc[i] = (uint64_t)((tokens[i] + block_size - 1) / block_size) * block_size * row_bytes;
    vlen[i] = hdr + 2ull * n_layers * alloc[i];
  }
  const size_t ns = c->shards.size();
  std::vector<uint8_t> inv(ns, 0);
  std::vector<uint32_t> si(n);
  for (uint32_t i = 0; i < n; ++i) {
    si[i] = shard_index(c, (const uint8_t *)keys[i], key_lens[i]);
    inv[si[i]] = 1;
  }
  ShardLocks locks(involved_servers(c, inv));
  TRY(quarantine_on_error(c, commit_barrier(c, inv)));
  // every length is checked before any recency changes, as one failed get leaves the store as it was
  std::vector<uint32_t> slot(n);
  for (uint32_t i = 0; i < n; ++i) {
    kvs_server *s = c->shards[si[i]];
    slot[i] = s->dir->lookup((const uint8_t *)keys[i], key_lens[i]);
    if (slot[i] != kvs::kBucketEmpty && s->dir->entry(slot[i]).total_len != vlen[i])
      return set_err(KVS_E_FORMAT, "%s: stored value for key %u has length %llu, a %u-token chunk of %u layers needs %llu",
                     op, i, (unsigned long long)s->dir->entry(slot[i]).total_len, tokens[i], n_layers,
                     (unsigned long long)vlen[i]);
  }
  struct Src {
    uint32_t i, shard, slot;
    uint64_t slab;       // slab address the value is read from (0: its host copy)
    uint64_t host_dev;   // device alias of the host copy
    const uint8_t *host; // the host copy (admissions copy from it)
    bool admit;          // the slab block is filled from the host copy first
  };
  std::vector<Src> src;
  std::multimap<std::pair<uint32_t, uint32_t>, size_t> reads;  // (shard, slot) -> src entries on its block
  for (size_t k = 0; k < ns; ++k)
    if (inv[k]) c->shards[k]->dir->take_evicted();
  for (uint32_t i = 0; i < n; ++i) {
    found[i] = 0;
    if (slot[i] == kvs::kBucketEmpty) continue;
    kvs_server *s = c->shards[si[i]];
    uint64_t off = 0;
    const auto action = s->dir->get_hit(slot[i], &off);
    // a block this call reads and a later admission just took: read that value's host copy
    for (uint32_t ev : s->dir->take_evicted()) {
      auto range = reads.equal_range({si[i], ev});
      for (auto it = range.first; it != range.second; ++it) {
        src[it->second].slab = 0;
        src[it->second].admit = false;
      }
      reads.erase(range.first, range.second);
    }
    const HostBacking &hb = s->dir->backing(slot[i]);
    Src r{i, si[i], slot[i], 0, s->device_alias(hb), s->host_ptr(hb), false};
    if (action == Directory::GetAction::kDevice) {
      r.slab = s->slab_base() + s->dir->entry(slot[i]).value_off;
    } else if (action == Directory::GetAction::kAdmit) {
      r.slab = s->slab_base() + off;
      r.admit = true;
      s->mprof.to_device_count++;
      s->moves_completed.fetch_add(1, std::memory_order_relaxed);
    } else {
      s->mprof.to_device_count++;
      s->moves_completed.fetch_add(1, std::memory_order_relaxed);
    }
    if (r.slab) reads.insert({{si[i], slot[i]}, src.size()});
    found[i] = 1;
    src.push_back(r);
  }
  for (const Src &r : src)
    if (!r.slab && !r.host_dev)
      return set_err(KVS_E_CUDA, "%s: the host copy of key %u has no device alias", op, r.i);
  if (src.empty()) return KVS_OK;  // every key missed
  const uint32_t nr = (uint32_t)src.size();
  TRY(begin_op(c, stream));
  Staging &st = c->stage;
  TRY(st.begin(4096 + 32ull * nr + 4ull * nr * max_blocks, c->stream));
  const size_t cu_off = st.take(4ull * (nr + 1)), pt_off = st.take(4ull * nr * max_blocks);
  const size_t sp_off = st.take(4ull * nr), rs_off = st.take(8ull * nr), ra_off = st.take(8ull * nr);
  int32_t *cu = st.h<int32_t>(cu_off);
  cu[0] = 0;
  uint64_t payload = 0, total = 0;
  for (uint32_t k = 0; k < nr; ++k) {
    const Src &r = src[k];
    total += tokens[r.i];
    if (total > 0x7FFFFFFFull) return set_err(KVS_E_INVAL, "%s: more than 2^31 tokens in one call", op);
    cu[k + 1] = (int32_t)total;
    std::memcpy(st.h<int32_t>(pt_off) + (uint64_t)k * max_blocks, page_table + (uint64_t)r.i * max_blocks,
                4ull * max_blocks);
    st.h<int32_t>(sp_off)[k] = start_positions[r.i];
    st.h<uint64_t>(rs_off)[k] = (r.slab ? r.slab : r.host_dev) + hdr;
    st.h<uint64_t>(ra_off)[k] = alloc[r.i];
    payload += 2ull * n_layers * tokens[r.i] * row_bytes;
  }
  TRY(st.upload(c->stream, st.used));
  for (size_t k = 0; k < ns; ++k)
    if (inv[k]) TRY(chain_wait(c, c->shards[k]));
  // read-through admissions first: host copy -> the value's new slab block
  for (const Src &r : src)
    if (r.admit && r.slab)
      CUDA_TRY(cudaMemcpyAsync(reinterpret_cast<void *>(r.slab), r.host, vlen[r.i], cudaMemcpyHostToDevice, c->stream));
  kvs::PagedFillParams fp{};
  fp.cu_seqlens = st.d<int32_t>(cu_off);
  fp.page_table = st.d<int32_t>(pt_off);
  fp.start_positions = st.d<int32_t>(sp_off);
  fp.req_src = st.d<uint64_t>(rs_off);
  fp.req_alloc = st.d<uint64_t>(ra_off);
  fp.n_heads = 1;
  fp.total_tokens = (uint32_t)total;
  fp.row_bytes = row_bytes;
  fp.batch = nr;
  fp.max_blocks = max_blocks;
  fp.num_blocks = num_blocks;
  fp.block_size = block_size;
  cudaEvent_t t0 = nullptr;
  c->time_begin(&t0);
  for (uint32_t l0 = 0; l0 < n_layers; l0 += kvs::kMaxFillLayers) {
    const uint32_t nl = std::min<uint32_t>(kvs::kMaxFillLayers, n_layers - l0);
    kvs::FillLayers L{};
    for (uint32_t l = 0; l < nl; ++l) {
      L.cache_k[l] = static_cast<uint8_t *>(cache_ks[l0 + l]);
      L.cache_v[l] = static_cast<uint8_t *>(cache_vs[l0 + l]);
    }
    fp.layer0 = l0;
    CUDA_TRY(kvs::launch_paged_fill(fp, L, nl, c->stream));
  }
  c->time_end(t0, 1, payload);
  for (size_t k = 0; k < ns; ++k)
    if (inv[k]) {
      c->shards[k]->launches++;
      TRY(chain_record(c, k));
    }
  CUDA_TRY(cudaStreamSynchronize(c->stream));
  TRY(check_tma_timeouts(c, op));
  // no end_op: the client stream is idle after the synchronise
  return KVS_OK;
}

int kvs_restore_chunks(kvs_client *c, uint32_t n, const void *const *keys, const uint32_t *key_lens,
                       const uint32_t *tokens, uint32_t n_layers, void *const *cache_ks, void *const *cache_vs,
                       uint32_t num_blocks, uint32_t block_size, uint32_t row_bytes, const int32_t *page_table,
                       uint32_t max_blocks_per_chunk, const int32_t *start_positions, uint8_t *found, void *stream) {
  TRY(check_client(c));
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  return quarantine_on_error(c, restore_chunks_impl(c, n, keys, key_lens, tokens, n_layers, cache_ks, cache_vs,
                                                    num_blocks, block_size, row_bytes, page_table,
                                                    max_blocks_per_chunk, start_positions, found, stream));
}

int kvs_get_blocks(kvs_client *c, const kvs_block_layout *layout, uint32_t n, const uint64_t *keys,
                   const int64_t *block_ids, uint8_t *found, void *stream) {
  TRY(check_client(c));
  if (!found) return set_err(KVS_E_INVAL, "get_blocks: found is null");
  const BlockFormat *fmt = nullptr;
  TRY(cached_block_format(layout, &fmt));
  TRY(check_blocks(layout, n, keys, block_ids, "get_blocks"));
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(validate_layout_ptrs(c, layout, "get_blocks"));
  GetTarget t{fmt, layout->n_members, layout->member_block_bytes, 1, layout->member_ptrs, nullptr};
  return quarantine_on_error(c, get_blocks_impl(c, t, n, keys, block_ids, found, stream));
}

static int exists_batch_impl(kvs_client *c, uint32_t n, const uint64_t *keys, uint8_t *found) {
  TRY(check_client(c));
  if (n == 0) return KVS_OK;
  if (!keys || !found) return set_err(KVS_E_INVAL, "exists_batch: null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  const size_t ns = c->shards.size();
  std::vector<uint8_t> inv(ns, 0);
  std::vector<uint32_t> si(n);
  for (uint32_t i = 0; i < n; ++i) {
    si[i] = shard_index(c, (const uint8_t *)&keys[i], 8);
    inv[si[i]] = 1;
  }
  const ShardOrder ord = order_by_shard(si, ns);
  ShardLocks locks(involved_servers(c, inv));
  TRY(quarantine_on_error(c, commit_barrier(c, inv)));  // EXISTS fuses the commit wait
  Staging &st = c->stage;
  size_t need = 4096 + 48ull * n;
  for (size_t i = 0; i < ns; ++i)
    if (inv[i]) need += mutation_upper_bound(c->shards[i]);
  TRY(st.begin(need, c->stream));
  std::vector<PackedMutations> pms(ns);
  for (size_t i = 0; i < ns; ++i)
    if (inv[i]) pms[i] = pack_mutations(c->shards[i], st);
  const size_t keys_off = st.take(8ull * n);
  for (uint32_t j = 0; j < n; ++j) st.h<uint64_t>(keys_off)[j] = keys[ord.perm[j]];
  const size_t upload_bytes = st.used;
  const size_t out_off = st.take(sizeof(kvs::LookupOut) * n);
  TRY(st.upload(c->stream, upload_bytes));
  for (size_t i = 0; i < ns; ++i)
    if (inv[i]) TRY(chain_wait(c, c->shards[i]));
  for (size_t i = 0; i < ns; ++i)
    if (inv[i]) TRY(quarantine_on_error(c, launch_mutations(c, c->shards[i], pms[i])));
  TRY(quarantine_on_error(c, launch_lookups(c, ord, st.d<uint8_t>(keys_off), st.hd<kvs::LookupOut>(out_off), nullptr, 0)));
  for (size_t i = 0; i < ns; ++i)
    if (inv[i]) TRY(chain_record(c, i));
  CUDA_TRY(cudaStreamSynchronize(c->stream));
  for (uint32_t j = 0; j < n; ++j) {
    const uint32_t i = ord.perm[j];
    found[i] = st.h<kvs::LookupOut>(out_off)[j].status != kvs::kMiss;
    const bool host_hit = c->shards[si[i]]->dir->lookup((const uint8_t *)&keys[i], 8) != kvs::kBucketEmpty;
    if ((bool)found[i] != host_hit) {
      c->quarantined = true;
      return set_err(KVS_E_CUDA, "exists_batch: device index replica disagrees with the catalog for key %u", i);
    }
  }
  return KVS_OK;
}

int kvs_exists_batch(kvs_client *c, uint32_t n, const uint64_t *keys, uint8_t *found) {
  return quarantine_on_error(c, exists_batch_impl(c, n, keys, found));
}

// ---------------------------------------------------------------------------- shards in other processes

namespace {

// cuMemGetAddressRange through the runtime's driver entry point (no link against libcuda).
typedef CUresult (*GetAddressRangeFn)(CUdeviceptr *base, size_t *size, CUdeviceptr ptr);

GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return (GetAddressRangeFn) nullptr;
    }
    return reinterpret_cast<GetAddressRangeFn>(f);
  }();
  return fn;
}

// Member pointers of the requesters' pools that were checked to be device memory.
std::mutex g_checked_mu;
std::vector<uint64_t> g_checked_members;

int check_member_sets(const kvs_block_layout *layouts, uint32_t n_sets, const char *op) {
  std::lock_guard<std::mutex> lk(g_checked_mu);
  for (uint32_t s = 0; s < n_sets; ++s)
    for (uint32_t m = 0; m < layouts[s].n_members; ++m) {
      const uint64_t ptr = layouts[s].member_ptrs[m];
      if (std::find(g_checked_members.begin(), g_checked_members.end(), ptr) != g_checked_members.end()) continue;
      cudaPointerAttributes a{};
      if (cudaPointerGetAttributes(&a, reinterpret_cast<const void *>(ptr)) != cudaSuccess ||
          a.type != cudaMemoryTypeDevice) {
        cudaGetLastError();
        return set_err(KVS_E_INVAL, "%s: member %u of pool %u must be device memory (this GPU's or a peer's)", op, m,
                       s);
      }
      g_checked_members.push_back(ptr);
    }
  return KVS_OK;
}

int owner_shard(kvs_client *c, const char *op, kvs_server **s) {
  TRY(check_client(c));
  if (c->shards.size() != 1)
    return set_err(KVS_E_INVAL, "%s: the owner's client must have exactly one shard (has %zu)", op, c->shards.size());
  *s = c->shards[0];
  return KVS_OK;
}

// One copy launch between whole values at `addrs` and rows of `value_len` bytes (raw values, no
// header). to_rows: addrs[i] -> rows[i].
int copy_values_launch(kvs_client *c, uint64_t rows, uint64_t value_len, uint32_t n, const uint64_t *addrs,
                       int to_rows) {
  Staging &st = c->stage;
  TRY(st.begin(4096 + 16ull * n, c->stream));
  const size_t blobs = st.push(addrs, 8ull * n);
  const size_t ids = st.take(8ull * n);
  for (uint32_t i = 0; i < n; ++i) st.h<int64_t>(ids)[i] = i;
  const uint64_t meta[5] = {rows, value_len, 0, 0, (value_len + kTileBytes - 1) / kTileBytes};
  const size_t mo = st.push(meta, sizeof meta);
  TRY(st.upload(c->stream, st.used));
  kvs::ChunkCopyParams p{};
  p.member_ptrs = st.d<uint64_t>(mo);
  p.member_bytes = st.d<uint64_t>(mo + 8);
  p.region_bases = st.d<uint64_t>(mo + 16);
  p.tile_prefix = st.d<uint64_t>(mo + 24);
  p.block_ids = st.d<int64_t>(ids);
  p.blob_ptrs = st.d<uint64_t>(blobs);
  p.n_blobs = n;
  p.blocks_per_blob = 1;
  p.n_ranks = 1;
  p.n_members = 1;
  p.tile_bytes = kTileBytes;
  p.tiles_per_combo = meta[4];
  p.total_tiles = (uint64_t)n * p.tiles_per_combo;
  p.to_blob = to_rows ? 0 : 1;
  set_copy_facts(&p, &value_len, 1, n);
  // rows are this GPU's memory (checked by the caller): the bulk engine when every value address
  // lies in a known slab or peer mapping
  CUDA_TRY(launch_copy(p, c->stream, dev_ranges_hold(addrs, n, value_len), c->timeout_flag));
  return KVS_OK;
}

}  // namespace

int kvs_ipc_export(const void *ptr, kvs_ipc_handle *handle, uint64_t *offset) {
  if (!ptr || !handle || !offset) return set_err(KVS_E_INVAL, "ipc_export: null argument");
  static_assert(sizeof(kvs_ipc_handle) == sizeof(cudaIpcMemHandle_t), "kvs_ipc_handle is a cudaIpcMemHandle_t");
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess || a.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return set_err(KVS_E_INVAL, "ipc_export: pointer is not device memory");
  }
  DeviceGuard g(a.device);
  GetAddressRangeFn range = address_range_fn();
  if (!range) return set_err(KVS_E_CUDA, "ipc_export: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_err(KVS_E_INVAL, "ipc_export: no device allocation contains the pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_err(KVS_E_INVAL, "ipc_export: %s (the allocation must come from cudaMalloc)", cudaGetErrorString(e));
  }
  std::memcpy(handle->bytes, &h, sizeof h);
  *offset = reinterpret_cast<uint64_t>(ptr) - (uint64_t)base;
  return KVS_OK;
}

int kvs_ipc_open(int32_t device, const kvs_ipc_handle *handle, void **base) {
  if (!handle || !base) return set_err(KVS_E_INVAL, "ipc_open: null argument");
  *base = nullptr;
  DeviceGuard g(device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof h);
  cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_err(KVS_E_CUDA, "ipc_open: %s", cudaGetErrorString(e));
  }
  GetAddressRangeFn range = address_range_fn();
  CUdeviceptr b = 0;
  size_t size = 0;
  if (range && range(&b, &size, reinterpret_cast<CUdeviceptr>(*base)) == CUDA_SUCCESS)
    dev_range_add(reinterpret_cast<void *>(b), size);
  return KVS_OK;
}

int kvs_ipc_close(int32_t device, void *base) {
  if (!base) return KVS_OK;
  DeviceGuard g(device);
  {
    // pointers inside the closed mapping are no longer known device memory
    std::lock_guard<std::mutex> lk(g_checked_mu);
    g_checked_members.clear();
  }
  g_mapping_generation.fetch_add(1, std::memory_order_acq_rel);
  dev_range_remove(base);
  CUDA_TRY(cudaIpcCloseMemHandle(base));
  return KVS_OK;
}

int kvs_server_slab(kvs_server *s, void **base, uint64_t *bytes) {
  if (!s || !base || !bytes) return set_err(KVS_E_INVAL, "server_slab: null argument");
  *base = s->slab;
  *bytes = s->cfg.heap_bytes;
  return KVS_OK;
}

int kvs_serve_gets(kvs_client *c, uint32_t n_sets, const kvs_block_layout *layouts, uint32_t n, const uint32_t *sets,
                   const int64_t *block_ids, const uint64_t *keys, uint8_t *found, void *stream) {
  kvs_server *s = nullptr;
  TRY(owner_shard(c, "serve_gets", &s));
  if (n_sets == 0 || !layouts) return set_err(KVS_E_INVAL, "serve_gets: at least one pool layout is required");
  BlockFormat fmt;
  TRY(block_format(&layouts[0], &fmt));
  for (uint32_t k = 1; k < n_sets; ++k) {
    const kvs_block_layout &L = layouts[k];
    BlockFormat fk;
    TRY(block_format(&L, &fk));  // validates pointers and sizes of every layout
    bool same = L.n_members == layouts[0].n_members && L.members_per_layer == layouts[0].members_per_layer;
    for (uint32_t m = 0; same && m < L.n_members; ++m) same = L.member_block_bytes[m] == layouts[0].member_block_bytes[m];
    if (!same) return set_err(KVS_E_INVAL, "serve_gets: pool %u has other member sizes than pool 0", k);
  }
  if (n && (!sets || !block_ids || !keys || !found)) return set_err(KVS_E_INVAL, "serve_gets: null argument");
  for (uint32_t i = 0; i < n; ++i) {
    if (sets[i] >= n_sets) return set_err(KVS_E_INVAL, "serve_gets: pool %u of key %u out of range", sets[i], i);
    if (block_ids[i] < 0 || (uint64_t)block_ids[i] >= layouts[sets[i]].n_pool_blocks)
      return set_err(KVS_E_INVAL, "serve_gets: block id %lld at %u is outside the %llu-block pool",
                     (long long)block_ids[i], i, (unsigned long long)layouts[sets[i]].n_pool_blocks);
  }
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  if (n == 0) {
    std::lock_guard<std::mutex> sl(s->mu);
    return quarantine_on_error(c, s->commit_all());
  }
  TRY(check_member_sets(layouts, n_sets, "serve_gets"));
  const uint32_t nm = layouts[0].n_members;
  std::vector<uint64_t> ptrs((size_t)n_sets * nm);
  for (uint32_t k = 0; k < n_sets; ++k)
    std::memcpy(ptrs.data() + (size_t)k * nm, layouts[k].member_ptrs, 8ull * nm);
  GetTarget t{&fmt, nm, layouts[0].member_block_bytes, n_sets, ptrs.data(), sets};
  return quarantine_on_error(c, get_blocks_impl(c, t, n, keys, block_ids, found, stream));
}

int kvs_serve_gets_packed(kvs_client *c, void *rows, uint64_t value_len, uint32_t n, const uint64_t *keys,
                          uint8_t *found, void *stream) {
  kvs_server *s = nullptr;
  TRY(owner_shard(c, "serve_gets_packed", &s));
  if (value_len == 0 || value_len % 4) return set_err(KVS_E_INVAL, "serve_gets_packed: value_len must be a nonzero multiple of 4");
  if (n && (!rows || !keys || !found)) return set_err(KVS_E_INVAL, "serve_gets_packed: null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  if (n == 0) {
    std::lock_guard<std::mutex> sl(s->mu);
    return quarantine_on_error(c, s->commit_all());
  }
  TRY(check_device_ptr(c, rows, "serve_gets_packed", "rows"));
  BlockFormat fmt;  // a whole value is one member region at offset 0
  fmt.region_bases = {0};
  fmt.tile_prefix = {0, (value_len + kTileBytes - 1) / kTileBytes};
  fmt.value_len = value_len;
  const uint64_t member_bytes = value_len, member_ptr = reinterpret_cast<uint64_t>(rows);
  std::vector<int64_t> ids(n);
  for (uint32_t i = 0; i < n; ++i) ids[i] = i;
  GetTarget t{&fmt, 1, &member_bytes, 1, &member_ptr, nullptr};
  return quarantine_on_error(c, get_blocks_impl(c, t, n, keys, ids.data(), found, stream));
}

int kvs_grant_puts(kvs_client *c, uint32_t n, const uint64_t *keys, uint64_t value_len, uint64_t *slab_offsets,
                   uint32_t *n_granted) {
  kvs_server *s = nullptr;
  TRY(owner_shard(c, "grant_puts", &s));
  if (!n_granted) return set_err(KVS_E_INVAL, "grant_puts: n_granted is null");
  *n_granted = 0;
  if (n && (!keys || !slab_offsets)) return set_err(KVS_E_INVAL, "grant_puts: null argument");
  if (value_len == 0 || value_len > s->cfg.max_value_bytes)
    return set_err(KVS_E_INVAL, "grant_puts: value of %llu B is outside (0, max_value_bytes %llu]",
                   (unsigned long long)value_len, (unsigned long long)s->cfg.max_value_bytes);
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  std::lock_guard<std::mutex> sl(s->mu);
  if (s->grant_blocked) {
    // the prepare that stopped the last grant asked for this commit; its value has landed since
    s->grant_blocked = false;
    if (!s->dir->fifo_empty() && s->dir->fifo_head().wt_batch >= 0) {
      TRY(quarantine_on_error(c, s->commit_one()));
      s->retire_batches();
      s->release_dropped();
    }
  }
  uint32_t i = 0;
  for (; i < n; ++i) {
    bool granted = false;
    for (;;) {
      kvs::Grant gr;
      const kvs::Prepare r = s->dir->prepare_put((const uint8_t *)&keys[i], 8, value_len, &gr);
      if (r == kvs::Prepare::kGranted) {
        slab_offsets[i] = gr.value_off;
        s->unlanded++;
        granted = true;
        break;
      }
      if (r == kvs::Prepare::kNoSpace) {
        *n_granted = i;
        return set_err(KVS_E_NOSPACE, "grant_puts: no device-cache space for a %llu B value",
                       (unsigned long long)value_len);
      }
      if (s->dir->fifo_head().wt_batch < 0) {
        s->grant_blocked = true;  // force_put_host_commit of a value still in flight: next round
        break;
      }
      TRY(quarantine_on_error(c, s->commit_one()));  // force_put_host_commit, then retry the prepare
      s->retire_batches();
      s->release_dropped();
    }
    if (!granted) break;
  }
  *n_granted = i;
  return KVS_OK;
}

static int puts_landed_impl(kvs_client *c, void *stream) {
  kvs_server *s = nullptr;
  TRY(owner_shard(c, "puts_landed", &s));
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  std::lock_guard<std::mutex> sl(s->mu);
  if (!s->unlanded) return KVS_OK;
  auto &fifo = s->dir->fifo();
  if (fifo.size() < s->unlanded) {
    c->quarantined = true;
    return set_err(KVS_E_CUDA, "puts_landed: the pending FIFO lost granted entries");
  }
  CUDA_TRY(cudaEventRecord(c->landed_evt, stream ? (cudaStream_t)stream : c->stream));
  CUDA_TRY(cudaStreamWaitEvent(s->wt_stream, c->landed_evt, 0));
  uint64_t batch_id = 0;
  cudaEvent_t ev = nullptr;
  TRY(s->new_batch(&batch_id, &ev));
  for (size_t k = fifo.size() - s->unlanded; k < fifo.size(); ++k) {
    kvs::PendingPut &pp = fifo[k];
    const kvs::Entry &e = s->dir->entry(pp.slot);
    TRY(s->reserve_backing(e.total_len, &pp.backing));
    pp.wt_batch = (int)batch_id;
    s->wt_add(s->host_ptr(pp.backing), s->slab + e.value_off, e.total_len);
  }
  TRY(s->wt_issue());
  CUDA_TRY(cudaEventRecord(ev, s->wt_stream));
  s->unlanded = 0;
  return KVS_OK;
}

int kvs_puts_landed(kvs_client *c, void *stream) {
  return quarantine_on_error(c, puts_landed_impl(c, stream));
}

static int copy_blocks_impl(kvs_client *c, const kvs_block_layout *layout, uint32_t n, const int64_t *block_ids,
                            const uint64_t *blob_addrs, int to_blob, void *stream) {
  TRY(check_client(c));
  BlockFormat fmt;
  TRY(block_format(layout, &fmt));
  if (n == 0) return KVS_OK;
  if (!block_ids || !blob_addrs) return set_err(KVS_E_INVAL, "copy_blocks: null argument");
  for (uint32_t i = 0; i < n; ++i) {
    if (block_ids[i] < 0 || (uint64_t)block_ids[i] >= layout->n_pool_blocks)
      return set_err(KVS_E_INVAL, "copy_blocks: block id %lld at %u is outside the %llu-block pool",
                     (long long)block_ids[i], i, (unsigned long long)layout->n_pool_blocks);
    if (blob_addrs[i] & 15u) return set_err(KVS_E_INVAL, "copy_blocks: value address %u is not 16-byte aligned", i);
  }
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(validate_layout_ptrs(c, layout, "copy_blocks"));
  TRY(begin_op(c, stream));
  Staging &st = c->stage;
  TRY(st.begin(4096 + 16ull * n + 40ull * layout->n_members + 4ull * fmt.header.size(), c->stream));
  const size_t blobs = st.push(blob_addrs, 8ull * n);
  const size_t ids = st.push(block_ids, 8ull * n);
  const size_t mp = st.push(layout->member_ptrs, 8ull * layout->n_members);
  const size_t mb = st.push(layout->member_block_bytes, 8ull * layout->n_members);
  const size_t rb = st.push(fmt.region_bases.data(), 8ull * layout->n_members);
  const size_t tp = st.push(fmt.tile_prefix.data(), 8ull * (layout->n_members + 1));
  const size_t hw = st.push(fmt.header.data(), 4ull * fmt.header.size());
  TRY(st.upload(c->stream, st.used));
  kvs::ChunkCopyParams p{};
  p.member_ptrs = st.d<uint64_t>(mp);
  p.member_bytes = st.d<uint64_t>(mb);
  p.region_bases = st.d<uint64_t>(rb);
  p.tile_prefix = st.d<uint64_t>(tp);
  p.block_ids = st.d<int64_t>(ids);
  p.blob_ptrs = st.d<uint64_t>(blobs);
  p.header_words = st.d<uint32_t>(hw);
  p.n_header_words = to_blob ? (uint32_t)fmt.header.size() : 0;
  p.n_blobs = n;
  p.blocks_per_blob = 1;
  p.n_ranks = 1;
  p.n_members = layout->n_members;
  p.tile_bytes = kTileBytes;
  p.tiles_per_combo = fmt.tile_prefix.back();
  p.total_tiles = (uint64_t)n * p.tiles_per_combo;
  p.to_blob = to_blob ? 1 : 0;
  set_copy_facts(&p, layout->member_block_bytes, layout->n_members, n);
  uint64_t payload = 0;
  for (uint32_t m = 0; m < layout->n_members; ++m) payload += layout->member_block_bytes[m];
  cudaEvent_t t0 = nullptr;
  c->time_begin(&t0);
  // members are this GPU's memory (validated): the bulk engine when every value address lies in a
  // known slab or peer mapping, plain loads and stores otherwise
  CUDA_TRY(launch_copy(p, c->stream, dev_ranges_hold(blob_addrs, n, fmt.value_len), c->timeout_flag));
  c->time_end(t0, to_blob ? 0 : 1, (uint64_t)n * payload);
  TRY(end_op(c, stream));
  return KVS_OK;
}

int kvs_copy_blocks(kvs_client *c, const kvs_block_layout *layout, uint32_t n, const int64_t *block_ids,
                    const uint64_t *blob_addrs, int to_blob, void *stream) {
  return quarantine_on_error(c, copy_blocks_impl(c, layout, n, block_ids, blob_addrs, to_blob, stream));
}

int kvs_bucket_requests(int32_t device, const uint64_t *keys, const int64_t *ids, uint32_t n, uint32_t n_get,
                        const int32_t *slot_shard, uint32_t world, uint32_t cap, int64_t op, int64_t *records,
                        int32_t *back, int32_t *counts, uint32_t *overflow, void *stream) {
  if (world == 0 || world > 32) return set_err(KVS_E_INVAL, "bucket_requests: world %u outside 1..32", world);
  if (cap == 0) return set_err(KVS_E_INVAL, "bucket_requests: cap must be positive");
  if (n_get > n) return set_err(KVS_E_INVAL, "bucket_requests: %u gets of %u keys", n_get, n);
  if ((n && (!keys || !ids)) || !records || !back || !counts || !overflow)
    return set_err(KVS_E_INVAL, "bucket_requests: null argument");
  const void *ptrs[] = {keys, ids, slot_shard, records, back, counts, overflow};
  for (const void *q : ptrs) {
    if (!q) continue;
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, q) != cudaSuccess || a.type != cudaMemoryTypeDevice || a.device != device) {
      cudaGetLastError();
      return set_err(KVS_E_INVAL, "bucket_requests: every array must be device memory of device %d", device);
    }
  }
  DeviceGuard g(device);
  kvs::BucketParams p{keys, ids, n, n_get, world, cap, slot_shard, op, records, back, counts, overflow};
  CUDA_TRY(kvs::launch_bucket_requests(p, (cudaStream_t)stream));
  return KVS_OK;
}

int kvs_copy_values(kvs_client *c, void *rows, uint64_t value_len, uint32_t n, const uint64_t *addrs, int to_rows,
                    void *stream) {
  TRY(check_client(c));
  if (n == 0) return KVS_OK;
  if (!rows || !addrs || value_len == 0) return set_err(KVS_E_INVAL, "copy_values: null argument or empty value");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  TRY(check_device_ptr(c, rows, "copy_values", "rows"));
  TRY(begin_op(c, stream));
  TRY(copy_values_launch(c, reinterpret_cast<uint64_t>(rows), value_len, n, addrs, to_rows));
  TRY(end_op(c, stream));
  return KVS_OK;
}

int kvs_client_set_timing(kvs_client *c, int enable) {
  if (!c) return set_err(KVS_E_INVAL, "client handle is null");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  c->drain_timing();
  c->timing = enable != 0;
  return KVS_OK;
}

int kvs_client_timing(kvs_client *c, kvs_kernel_timing *gather, kvs_kernel_timing *scatter) {
  if (!c) return set_err(KVS_E_INVAL, "client handle is null");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  c->drain_timing();
  if (gather) *gather = c->acc[0];
  if (scatter) *scatter = c->acc[1];
  c->acc[0] = kvs_kernel_timing{};
  c->acc[1] = kvs_kernel_timing{};
  return KVS_OK;
}

int kvs_client_host_tier_timing(kvs_client *c, kvs_kernel_timing *admissions, kvs_kernel_timing *serves) {
  if (!c) return set_err(KVS_E_INVAL, "client handle is null");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g(c->device);
  c->drain_timing();
  if (admissions) *admissions = c->acc[2];
  if (serves) *serves = c->acc[3];
  c->acc[2] = kvs_kernel_timing{};
  c->acc[3] = kvs_kernel_timing{};
  return KVS_OK;
}

// ---------------------------------------------------------------------------- chunk ops

static int chunk_op(const uint64_t *member_ptrs, uint32_t n_ranks, uint32_t n_members,
                    const uint64_t *member_block_bytes, const uint64_t *member_extent, const uint32_t *block_ids,
                    uint32_t n_blocks, const uint64_t *region_bases, const uint32_t *header_words,
                    uint32_t n_header_words, void *blob, uint64_t blob_bytes, void *stream, int to_blob,
                    const char *op) {
  const kvs::ChunkArgs a{member_ptrs, n_ranks,      n_members,      member_block_bytes, member_extent, block_ids,
                         n_blocks,    region_bases, header_words,   n_header_words,     blob,          blob_bytes,
                         to_blob};
  kvs::ChunkMeta m{};
  TRY(kvs::check_chunk_args(a, op, &m));
  DeviceGuard g(m.device);
  // per-call device metadata: allocated from the stream-ordered pool (cudaMallocAsync)
  std::vector<uint8_t> image(m.bytes);
  kvs::pack_chunk_meta(a, m, image.data());
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t *dbuf = nullptr;
  CUDA_TRY(cudaMallocAsync(&dbuf, m.bytes, s));
  CUDA_TRY(cudaMemcpyAsync(dbuf, image.data(), m.bytes, cudaMemcpyHostToDevice, s));
  CUDA_TRY(kvs::launch_chunk(kvs::chunk_params(a, m, dbuf), s));
  CUDA_TRY(cudaFreeAsync(dbuf, s));
  // the host image was consumed by a pageable copy, which returns once the image is staged
  return KVS_OK;
}

static int paged_fill_impl(uint32_t n_layers, const void *const *k_fills, const void *const *v_fills, uint32_t n_heads,
                           uint32_t total_tokens, uint32_t row_bytes, const int32_t *cu_seqlens, uint32_t batch,
                           const int32_t *page_table, uint32_t max_blocks_per_seq, const int32_t *start_positions,
                           void *const *cache_ks, void *const *cache_vs, uint32_t num_blocks, uint32_t block_size,
                           uint32_t *out_of_range, void *stream, const char *op) {
  if (n_layers == 0) return KVS_OK;
  if (!k_fills || !v_fills || !cache_ks || !cache_vs) return set_err(KVS_E_INVAL, "%s: layer arrays are null", op);
  if (batch == 0) return set_err(KVS_E_INVAL, "%s: page_table must have at least one row", op);
  if (block_size == 0 || row_bytes == 0 || n_heads == 0)
    return set_err(KVS_E_INVAL, "%s: block_size, head row bytes and num_kv_heads must be > 0", op);
  if (max_blocks_per_seq > num_blocks)
    return set_err(KVS_E_INVAL, "%s: max_num_blocks_per_seq (%u) must be <= max_num_blocks (%u)", op,
                   max_blocks_per_seq, num_blocks);
  int device = -1;
  auto on_device = [&](const void *ptr, const char *name, uint32_t layer) -> int {
    cudaPointerAttributes a{};
    if (!ptr || cudaPointerGetAttributes(&a, ptr) != cudaSuccess || a.type != cudaMemoryTypeDevice) {
      cudaGetLastError();
      if (n_layers > 1) return set_err(KVS_E_INVAL, "%s: %s of layer %u must be on device!", op, name, layer);
      return set_err(KVS_E_INVAL, "%s: %s must be on device!", op, name);
    }
    if (device < 0) device = a.device;
    if (a.device != device) return set_err(KVS_E_INVAL, "%s: All tensors must be on the same device!", op);
    return KVS_OK;
  };
  for (uint32_t l = 0; l < n_layers; ++l) {
    TRY(on_device(k_fills[l], "k_fill_value", l));
    TRY(on_device(v_fills[l], "v_fill_value", l));
    if (l == 0) {
      TRY(on_device(cu_seqlens, "cu_seqlens", 0));
      TRY(on_device(page_table, "page_table", 0));
      TRY(on_device(start_positions, "start_positions", 0));
    }
    TRY(on_device(cache_ks[l], "cache_k", l));
    TRY(on_device(cache_vs[l], "cache_v", l));
  }
  DeviceGuard g(device);
  kvs::PagedFillParams p{};
  p.cu_seqlens = cu_seqlens;
  p.page_table = page_table;
  p.start_positions = start_positions;
  p.n_heads = n_heads;
  p.total_tokens = total_tokens;
  p.row_bytes = row_bytes;
  p.batch = batch;
  p.max_blocks = max_blocks_per_seq;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  for (uint32_t l0 = 0; l0 < n_layers; l0 += kvs::kMaxFillLayers) {
    const uint32_t nl = std::min<uint32_t>(kvs::kMaxFillLayers, n_layers - l0);
    kvs::FillLayers L{};
    for (uint32_t l = 0; l < nl; ++l) {
      L.k_fill[l] = static_cast<const uint8_t *>(k_fills[l0 + l]);
      L.v_fill[l] = static_cast<const uint8_t *>(v_fills[l0 + l]);
      L.cache_k[l] = static_cast<uint8_t *>(cache_ks[l0 + l]);
      L.cache_v[l] = static_cast<uint8_t *>(cache_vs[l0 + l]);
    }
    p.out_of_range = l0 == 0 ? out_of_range : nullptr;  // counted once per token
    CUDA_TRY(kvs::launch_paged_fill(p, L, nl, static_cast<cudaStream_t>(stream)));
  }
  return KVS_OK;
}

int kvs_paged_fill_varlen(const void *k_fill, const void *v_fill, uint32_t n_heads, uint32_t total_tokens,
                          uint32_t row_bytes, const int32_t *cu_seqlens, uint32_t batch, const int32_t *page_table,
                          uint32_t max_blocks_per_seq, const int32_t *start_positions, void *cache_k, void *cache_v,
                          uint32_t num_blocks, uint32_t block_size, uint32_t *out_of_range, void *stream) {
  return paged_fill_impl(1, &k_fill, &v_fill, n_heads, total_tokens, row_bytes, cu_seqlens, batch, page_table,
                         max_blocks_per_seq, start_positions, &cache_k, &cache_v, num_blocks, block_size, out_of_range,
                         stream, "paged_fill_varlen");
}

int kvs_paged_fill_varlen_layers(uint32_t n_layers, const void *const *k_fills, const void *const *v_fills,
                                 uint32_t n_heads, uint32_t total_tokens, uint32_t row_bytes,
                                 const int32_t *cu_seqlens, uint32_t batch, const int32_t *page_table,
                                 uint32_t max_blocks_per_seq, const int32_t *start_positions, void *const *cache_ks,
                                 void *const *cache_vs, uint32_t num_blocks, uint32_t block_size,
                                 uint32_t *out_of_range, void *stream) {
  return paged_fill_impl(n_layers, k_fills, v_fills, n_heads, total_tokens, row_bytes, cu_seqlens, batch, page_table,
                         max_blocks_per_seq, start_positions, cache_ks, cache_vs, num_blocks, block_size, out_of_range,
                         stream, "paged_fill_varlen_layers");
}

int kvs_gather_chunk(const uint64_t *member_ptrs, uint32_t n_ranks, uint32_t n_members,
                     const uint64_t *member_block_bytes, const uint64_t *member_extent, const uint32_t *block_ids,
                     uint32_t n_blocks, const uint64_t *region_bases, const uint32_t *header_words,
                     uint32_t n_header_words, void *blob, uint64_t blob_bytes, void *stream) {
  return chunk_op(member_ptrs, n_ranks, n_members, member_block_bytes, member_extent, block_ids, n_blocks,
                  region_bases, header_words, n_header_words, blob, blob_bytes, stream, 1, "kvcache gather");
}

int kvs_scatter_chunk(const void *blob, uint64_t blob_bytes, const uint64_t *member_ptrs, uint32_t n_ranks,
                      uint32_t n_members, const uint64_t *member_block_bytes, const uint64_t *member_extent,
                      const uint32_t *block_ids, uint32_t n_blocks, const uint64_t *region_bases, void *stream) {
  return chunk_op(member_ptrs, n_ranks, n_members, member_block_bytes, member_extent, block_ids, n_blocks,
                  region_bases, nullptr, 0, const_cast<void *>(blob), blob_bytes, stream, 0, "kvcache scatter");
}

}  // extern "C"
