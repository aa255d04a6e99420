// hb_host.h -- host-only helpers with no CUDA dependency, so that their
// logic can be tested on a machine without a GPU (tests/native/): the
// per-context cache of a device symbol's address and the deadline loop of a
// multi-GPU call.  The CUDA and NCCL calls they drive are passed in.
#pragma once

#include <chrono>
#include <cstdint>
#include <mutex>
#include <thread>

namespace hb {

// Device address of one file-scope __device__ array, per device, cached
// against the CUDA context it was looked up in.  A module is loaded once per
// context, so the address is only valid in that context: after
// cudaDeviceReset (or any other end of the primary context) the next
// lookup on the device sees a new context id and asks again, instead of
// handing a kernel an address that is no longer mapped.
//
//   ctx_id(unsigned long long* id) -> int : 0 with the current context's
//       unique id (non-zero), non-zero when there is no current context;
//   lookup(void** addr) -> int : 0 with the address in the current context
//       (it makes the device's primary context current if none was), else an
//       error code that get() returns unchanged.
class SymbolCache {
 public:
  static constexpr int kMaxDevices = 64;

  template <class CtxId, class Lookup>
  int get(int dev, CtxId ctx_id, Lookup lookup, void** out) {
    if (dev < 0 || dev >= kMaxDevices) return -1;
    unsigned long long id = 0;
    const bool have_ctx = ctx_id(&id) == 0 && id != 0;
    std::lock_guard<std::mutex> lock(mu_);
    Slot& s = slot_[dev];
    if (have_ctx && s.addr && s.ctx == id) {
      *out = s.addr;
      return 0;
    }
    void* p = nullptr;
    const int e = lookup(&p);
    if (e != 0) return e;
    if (!have_ctx && (ctx_id(&id) != 0 || id == 0)) {
      *out = p;  // no context id to key the entry on: use it, keep nothing
      return 0;
    }
    s.ctx = id;
    s.addr = p;
    ++lookups_;
    *out = p;
    return 0;
  }

  // Lookups that filled a slot (for tests).
  long lookups() const { return lookups_; }

 private:
  struct Slot {
    unsigned long long ctx = 0;
    void* addr = nullptr;
  };
  std::mutex mu_;
  Slot slot_[kMaxDevices];
  long lookups_ = 0;
};

// Outcome of a host wait on a multi-GPU call.
enum class WaitResult { kDone, kTimeout, kCommError, kQueryError };

// Polls `poll()` (0: the work is complete, 1: still running, other: the
// query failed) and `comm_error()` (true once the communicator reports an
// asynchronous error) until the work completes, an error shows, or
// `timeout_s` seconds have passed on `now()` (seconds, monotonic).  Between
// polls it calls sleep_for_poll().  The caller aborts the communicator on
// kTimeout and kCommError, so that peers waiting on this rank end too.
template <class Poll, class CommError, class Now, class Sleep>
WaitResult wait_with_deadline(Poll poll, CommError comm_error, Now now, Sleep sleep_for_poll,
                              double timeout_s) {
  const double t0 = now();
  for (;;) {
    const int p = poll();
    if (p == 0) return comm_error() ? WaitResult::kCommError : WaitResult::kDone;
    if (p != 1) return WaitResult::kQueryError;
    if (comm_error()) return WaitResult::kCommError;
    if (now() - t0 > timeout_s) return WaitResult::kTimeout;
    sleep_for_poll();
  }
}

inline double monotonic_seconds() {
  using namespace std::chrono;
  return duration<double>(steady_clock::now().time_since_epoch()).count();
}

inline void sleep_poll_interval() { std::this_thread::sleep_for(std::chrono::microseconds(50)); }

}  // namespace hb
