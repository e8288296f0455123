"""The product's shard catalog (tt-infinity_b200/csrc/kvs_directory.cpp) against the oracle store
(oracle/kvs_oracle.c), both compiled for the host: random put / get / exists / remove / move /
flush sequences under eviction and catalog pressure, the catalog driven in the order the runtime
drives it (kvs_runtime.cpp: prepare, forced commit of the FIFO head, host backing reserved when a
put is issued, commit barrier before every get / exists / remove / move / flush). After every
operation each key's residency, the counters, the LRU order and the hash buckets must be equal.
The split of host copies between the pinned pool and separate buffers is not compared: the
runtime reserves a copy when the put is issued (so the device->host copy can start at once), the
reference when it commits. Needs g++, gcc and the CUDA headers, no GPU."""

import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "tt-infinity_b200" / "csrc"
ORACLE = ROOT / "oracle"
CUDA_INC = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"

DRIVER = r"""
#include "kvs_directory.hpp"
extern "C" {
#include "kvs_oracle.h"
}
#include <cstdio>
#include <cstdlib>
#include <random>
#include <string>
#include <vector>
using namespace kvs;

// The runtime's orchestration of one shard's catalog (kvs_server in kvs_runtime.cpp), host side.
struct Shard {
  Directory d;
  size_t staged = 0;  // granted puts not yet flushed (their FIFO entries are the newest)
  explicit Shard(const DirConfig &c) : d(c) {}
  HostBacking reserve(uint64_t len) {
    HostBacking b;
    b.present = true;
    b.len = len;
    uint64_t unit;
    const uint64_t units = d.units_for(len);
    if (d.config().host_pool_units && d.pool_alloc(units, &unit)) {
      b.in_pool = true;
      b.pool_unit = unit;
      b.pool_units = units;
    } else {
      b.heap = reinterpret_cast<uint8_t *>(16);  // stands for a separately pinned buffer
    }
    return b;
  }
  void release(const HostBacking &b) {
    if (b.present && b.in_pool) d.pool_release(b.pool_unit, b.pool_units);
  }
  void release_dropped() {
    for (auto &b : d.take_dropped()) release(b);
  }
  void flush() {  // flush_puts: every staged put gets its host backing, in FIFO order
    auto &fifo = d.fifo();
    for (size_t k = fifo.size() - staged; k < fifo.size(); ++k) {
      fifo[k].backing = reserve(d.entry(fifo[k].slot).total_len);
      fifo[k].wt_batch = 0;
    }
    staged = 0;
  }
  void commit_one() {
    HostBacking released;
    if (!d.commit_head(&released)) release(released);
  }
  void commit_all() {
    while (!d.fifo_empty()) commit_one();
    release_dropped();
  }
  bool put(const std::string &k, uint64_t len) {  // stage_put + flush_puts
    for (;;) {
      Grant g;
      const Prepare r = d.prepare_put((const uint8_t *)k.data(), (uint32_t)k.size(), len, &g);
      if (r == Prepare::kGranted) { ++staged; flush(); return true; }
      flush();
      if (r == Prepare::kNoSpace) return false;
      commit_one();
      release_dropped();
    }
  }
  uint32_t lookup(const std::string &k) { return d.lookup((const uint8_t *)k.data(), (uint32_t)k.size()); }
};

static int fail(const char *what, uint32_t op, long long a, long long b) {
  std::printf("op %u: %s differs (product %lld, oracle %lld)\n", op, what, a, b);
  return 1;
}

int main(int argc, char **argv) {
  const uint64_t seed = std::strtoull(argv[1], nullptr, 10);
  const uint32_t max_keys = (uint32_t)std::strtoul(argv[2], nullptr, 10);
  const uint32_t heap_units = (uint32_t)std::strtoul(argv[3], nullptr, 10);
  const uint32_t pool_units = (uint32_t)std::strtoul(argv[4], nullptr, 10);
  const uint32_t ops = (uint32_t)std::strtoul(argv[5], nullptr, 10);
  const uint32_t U = 4288;
  DirConfig dc{max_keys, U, 128, (uint64_t)heap_units * U, 1u << 20, pool_units};
  Shard p(dc);
  kvo_config oc{max_keys, U, (uint64_t)heap_units * U, 128, 1u << 20, (uint64_t)pool_units * U};
  kvo_store *o = kvo_store_create(&oc);
  if (!o) { std::printf("oracle: %s\n", kvo_last_error()); return 2; }
  std::vector<std::string> keys;
  for (uint32_t i = 0; i < 3 * max_keys; ++i) keys.push_back("key-" + std::to_string(i * 7919u % 100003u));
  std::vector<uint8_t> value(8 * U, 0x5A), out(8 * U);
  std::mt19937_64 rng(seed);
  std::vector<uint32_t> lp(max_keys), lo(max_keys);
  for (uint32_t op = 0; op < ops; ++op) {
    const uint32_t r = (uint32_t)(rng() % 100);
    const std::string &k = keys[rng() % keys.size()];
    const uint8_t *kb = (const uint8_t *)k.data();
    const uint32_t kl = (uint32_t)k.size();
    if (r < 40) {
      const uint64_t len = 1 + rng() % (6 * U);
      const bool ok = p.put(k, len);
      const int rc = kvo_put(o, kb, kl, value.data(), len, 0);
      if (ok != (rc == 0)) return fail("put outcome", op, ok, rc);
    } else if (r < 65) {
      p.commit_all();
      const uint32_t slot = p.lookup(k);
      int found = 0;
      uint64_t vlen = 0;
      kvo_get(o, kb, kl, out.data(), out.size(), &found, &vlen);
      if ((slot != kNone) != (found != 0)) return fail("get found", op, slot != kNone, found);
      if (slot != kNone) { uint64_t off; p.d.get_hit(slot, &off); }
    } else if (r < 72) {
      p.commit_all();
      int found = 0;
      kvo_exists(o, kb, kl, &found);
      if ((p.lookup(k) != kNone) != (found != 0)) return fail("exists", op, p.lookup(k) != kNone, found);
    } else if (r < 79) {
      p.commit_all();
      const uint32_t slot = p.lookup(k);
      if (slot != kNone) { p.d.remove(slot); p.release_dropped(); }
      int removed = 0;
      kvo_remove(o, kb, kl, &removed);
      if ((slot != kNone) != (removed != 0)) return fail("remove", op, slot != kNone, removed);
    } else if (r < 87) {
      p.commit_all();
      const uint32_t slot = p.lookup(k);
      if (slot != kNone) p.d.move_to_host(slot);
      kvo_move_to_host(o, kb, kl);
    } else if (r < 95) {
      p.commit_all();
      const uint32_t slot = p.lookup(k);
      if (slot != kNone) { uint64_t off; p.d.move_to_device(slot, &off); }
      kvo_move_to_device(o, kb, kl);
    } else {
      p.commit_all();
      kvo_flush(o);
    }
    // residency of every key
    for (const std::string &q : keys) {
      const uint32_t slot = p.lookup(q);
      const int lp_ = slot == kNone ? -1 : (int)p.d.entry(slot).location;
      const int lo_ = kvo_location(o, (const uint8_t *)q.data(), (uint32_t)q.size(), nullptr);
      if (lp_ != lo_) return fail(("location of " + q).c_str(), op, lp_, lo_);
    }
    // counters
    kvo_stats os;
    kvo_get_stats(o, &os);
    DirStats &ps = p.d.stats();
    uint64_t dev_keys = 0;
    const uint64_t live = p.d.live_keys(&dev_keys);
    const long long pv[] = {(long long)p.d.live_device_bytes(), (long long)p.d.pending_device_bytes(), (long long)live,
                            (long long)dev_keys, (long long)ps.allocation_calls, (long long)ps.allocation_successes,
                            (long long)ps.allocation_failures, (long long)ps.victims_evicted,
                            (long long)ps.catalog_replacements, (long long)ps.writes_through,
                            (long long)ps.stale_commits, (long long)ps.host_serves, (long long)ps.admissions,
                            (long long)p.d.epoch(), (long long)ps.issued, (long long)ps.committed};
    const long long ov[] = {(long long)os.live_device_bytes, (long long)os.pending_device_bytes, (long long)os.live_keys,
                            (long long)os.device_resident_keys, (long long)os.allocation_calls,
                            (long long)os.allocation_successes, (long long)os.allocation_failures,
                            (long long)os.victims_evicted, (long long)os.catalog_replacements,
                            (long long)os.writes_through, (long long)os.stale_commits, (long long)os.host_serves,
                            (long long)os.admissions, (long long)os.epoch, (long long)os.issued,
                            (long long)os.committed};
    const char *names[] = {"live_device_bytes", "pending_device_bytes", "live_keys", "device_resident_keys",
                           "allocation_calls", "allocation_successes", "allocation_failures", "victims_evicted",
                           "catalog_replacements", "writes_through", "stale_commits", "host_serves", "admissions",
                           "epoch", "issued", "committed"};
    for (int i = 0; i < 16; ++i)
      if (pv[i] != ov[i]) return fail(names[i], op, pv[i], ov[i]);
    // LRU order and hash buckets
    const uint32_t np_ = p.d.lru_order(lp.data(), max_keys), no_ = kvo_lru_order(o, lo.data(), max_keys);
    if (np_ != no_) return fail("LRU length", op, np_, no_);
    for (uint32_t i = 0; i < np_; ++i)
      if (lp[i] != lo[i]) return fail("LRU order", op, lp[i], lo[i]);
    uint32_t nbo = 0;
    const uint32_t *bo = kvo_buckets(o, &nbo);
    if (nbo != p.d.num_buckets()) return fail("bucket count", op, p.d.num_buckets(), nbo);
    const uint32_t *bp = p.d.bucket_pairs();
    for (uint32_t i = 0; i < 2 * nbo; ++i)
      if (bp[i] != bo[i]) return fail("bucket word", op, bp[i], bo[i]);
  }
  kvo_store_destroy(o);
  std::printf("ok\n");
  return 0;
}
"""


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    if shutil.which("g++") is None or shutil.which("gcc") is None or not (CUDA_INC / "cuda_runtime.h").exists():
        pytest.skip("needs g++, gcc and the CUDA headers")
    d = tmp_path_factory.mktemp("dirdiff")
    (d / "driver.cpp").write_text(DRIVER)
    run = lambda *a: subprocess.run(list(a), check=True, capture_output=True, timeout=300)
    run("gcc", "-O2", "-std=c11", "-pthread", f"-I{ORACLE}", "-c", str(ORACLE / "kvs_oracle.c"), "-o", str(d / "o.o"))
    run("g++", "-O2", "-std=c++17", "-pthread", f"-I{CSRC}", f"-I{ORACLE}", f"-I{CUDA_INC}", str(d / "driver.cpp"),
        str(CSRC / "kvs_directory.cpp"), str(d / "o.o"), "-o", str(d / "driver"))
    return d / "driver"


@pytest.mark.parametrize("seed,max_keys,heap_units,pool_units", [
    (1, 16, 24, 40),     # small catalog and slab: replacement, eviction, forced commits
    (2, 24, 64, 16),     # host pool smaller than the live set: separately pinned copies
    (3, 48, 40, 400),    # more keys than the slab holds: host-tier serves and admissions
    (4, 64, 256, 0),     # no host pool at all
])
def test_catalog_matches_oracle(driver, seed, max_keys, heap_units, pool_units):
    r = subprocess.run([str(driver), str(seed), str(max_keys), str(heap_units), str(pool_units), "3000"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-2000:]
