// CPU test of the host-only helpers of hb_host.h with stubbed CUDA / NCCL
// calls: the per-context cache of a device symbol's address, and the
// deadline loop of a ring call.  Built and run by tests/test_host_native.py;
// prints "ok" and exits 0 when every check holds.
#include <cstdio>
#include <cstdlib>

#include "hb_host.h"

static int failures = 0;
#define CHECK(c)                                                   \
  do {                                                             \
    if (!(c)) {                                                    \
      std::printf("FAILED line %d: %s\n", __LINE__, #c);           \
      ++failures;                                                  \
    }                                                              \
  } while (0)

// a fake device: its current context id (0 = none) and the address its
// module gives the symbol in that context
struct FakeDevice {
  unsigned long long ctx = 0;
  unsigned long long next_ctx = 100;
  int lookups = 0;
  int fail_with = 0;
  int ctx_id(unsigned long long* id) {
    if (!ctx) return 1;
    *id = ctx;
    return 0;
  }
  int lookup(void** p) {
    ++lookups;
    if (fail_with) return fail_with;
    if (!ctx) ctx = next_ctx++;  // the runtime makes the primary context current
    *p = reinterpret_cast<void*>(0x10000 * ctx);
    return 0;
  }
};

static void symbol_cache() {
  hb::SymbolCache cache;
  FakeDevice d;
  auto id = [&](unsigned long long* x) { return d.ctx_id(x); };
  auto look = [&](void** p) { return d.lookup(p); };
  void* a = nullptr;
  // no context yet: the lookup creates it, the entry is keyed on it
  CHECK(cache.get(0, id, look, &a) == 0);
  CHECK(a == reinterpret_cast<void*>(0x10000 * 100));
  CHECK(d.lookups == 1);
  // same context: served from the cache
  void* b = nullptr;
  CHECK(cache.get(0, id, look, &b) == 0 && b == a && d.lookups == 1);
  // the context ends and a new one starts (cudaDeviceReset): looked up again
  d.ctx = 0;
  void* c = nullptr;
  CHECK(cache.get(0, id, look, &c) == 0);
  CHECK(c == reinterpret_cast<void*>(0x10000 * 101) && d.lookups == 2);
  CHECK(cache.get(0, id, look, &c) == 0 && d.lookups == 2);
  // another device has its own entry
  FakeDevice d1;
  d1.ctx = 7;
  auto id1 = [&](unsigned long long* x) { return d1.ctx_id(x); };
  auto look1 = [&](void** p) { return d1.lookup(p); };
  void* e = nullptr;
  CHECK(cache.get(1, id1, look1, &e) == 0 && e == reinterpret_cast<void*>(0x10000 * 7));
  CHECK(cache.get(0, id, look, &c) == 0 && c == reinterpret_cast<void*>(0x10000 * 101));
  CHECK(d.lookups == 2 && d1.lookups == 1);
  // a failing lookup is returned unchanged and caches nothing
  FakeDevice d2;
  d2.ctx = 9;
  d2.fail_with = 4;
  auto id2 = [&](unsigned long long* x) { return d2.ctx_id(x); };
  auto look2 = [&](void** p) { return d2.lookup(p); };
  void* f = nullptr;
  CHECK(cache.get(2, id2, look2, &f) == 4);
  d2.fail_with = 0;
  CHECK(cache.get(2, id2, look2, &f) == 0 && f == reinterpret_cast<void*>(0x10000 * 9));
  CHECK(d2.lookups == 2);
  // devices outside the table
  CHECK(cache.get(-1, id, look, &f) == -1);
  CHECK(cache.get(hb::SymbolCache::kMaxDevices, id, look, &f) == -1);
  CHECK(cache.lookups() == 4);
}

struct FakeRing {
  double t = 0;
  int polls = 0, sleeps = 0;
  int done_after = -1;       // poll count at which the stream completes (-1: never)
  int comm_error_after = -1;  // poll count from which the communicator reports an error
  int query_error_at = -1;
  int poll() {
    ++polls;
    if (polls == query_error_at) return 2;
    return done_after >= 0 && polls >= done_after ? 0 : 1;
  }
  bool comm_error() const { return comm_error_after >= 0 && polls >= comm_error_after; }
  double now() const { return t; }
  void sleep() {
    ++sleeps;
    t += 0.1;
  }
};

static hb::WaitResult run(FakeRing& r, double timeout) {
  return hb::wait_with_deadline([&] { return r.poll(); }, [&] { return r.comm_error(); },
                                [&] { return r.now(); }, [&] { r.sleep(); }, timeout);
}

static void deadline() {
  {  // completes on the fourth poll
    FakeRing r;
    r.done_after = 4;
    CHECK(run(r, 10.0) == hb::WaitResult::kDone);
    CHECK(r.polls == 4 && r.sleeps == 3);
  }
  {  // never completes: gives up once more than 1 s has passed
    FakeRing r;
    CHECK(run(r, 1.0) == hb::WaitResult::kTimeout);
    CHECK(r.t > 1.0 && r.t < 1.25);
  }
  {  // zero timeout, complete at once
    FakeRing r;
    r.done_after = 1;
    CHECK(run(r, 0.0) == hb::WaitResult::kDone && r.sleeps == 0);
  }
  {  // zero timeout, still running: ends at the first check after one poll interval
    FakeRing r;
    CHECK(run(r, 0.0) == hb::WaitResult::kTimeout && r.sleeps == 1);
  }
  {  // a peer's failure shows as an asynchronous communicator error
    FakeRing r;
    r.comm_error_after = 3;
    CHECK(run(r, 10.0) == hb::WaitResult::kCommError && r.polls == 3);
  }
  {  // complete, but the communicator failed: still an error
    FakeRing r;
    r.done_after = 2;
    r.comm_error_after = 1;
    CHECK(run(r, 10.0) == hb::WaitResult::kCommError);
  }
  {  // the stream query fails (a sticky device error)
    FakeRing r;
    r.query_error_at = 2;
    CHECK(run(r, 10.0) == hb::WaitResult::kQueryError && r.polls == 2);
  }
}

int main() {
  symbol_cache();
  deadline();
  if (failures) return 1;
  std::printf("ok\n");
  return 0;
}
