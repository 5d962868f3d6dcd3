// global_policy.h - host-side choice, per global layer, between the bf16 speculative pass (one launch, plus
// a fixup launch that recomputes the CTAs it marked) and the exact two-pass kernel (one launch).
//
// The speculative pass wins when few CTAs need the recompute: at ViT-H shapes it costs 0.87x the exact
// kernel, and each recomputed CTA costs a full exact CTA on top of it. So above a recompute share of about
// 0.13 the exact kernel alone is faster. Such shares show up with large rel-pos tables (std 2 and
// activations std 2: 91 % of CTAs). The share is data-dependent and differs per layer, so the choice is
// kept per layer, keyed by the device and the rel-pos table's address (each layer has its own table).
//
// Measuring: a speculative call that measures points the fixup kernel at its own device counter (zeroed
// first on the call's stream), then copies that counter into pinned host memory and records an event.
// A later call on the same layer reads it once the event has completed, and never waits for it. The
// first call on a layer and every kMeasureEvery-th speculative call measure. Above kExactShare the layer
// switches to the exact kernel for kExactCalls calls, after which the speculative pass is tried (and
// measured) again. A stream that is capturing a CUDA graph replays the current choice: no measurement,
// no event query, and the exact-call count does not advance.
// No counterpart in the reference (its kernels have no speculative pass).
#pragma once
#include <cuda_runtime.h>

#include <mutex>
#include <stdint.h>

#include "common.cuh"

namespace samrs {

class GlobalPolicy {
 public:
  static constexpr double kExactShare = 0.15;
  static constexpr int kExactCalls = 32;
  static constexpr int kMeasureEvery = 16;
  static constexpr int kSlots = kPolicySlots;  // layers tracked per device (by table address)
  static constexpr int kMaxDevices = 64;

  // What one call launches: the exact kernel, or the speculative pass whose fixup counts into `slot`
  // (nullptr: no measurement this call).
  struct Choice {
    bool exact = false;
    unsigned long long* slot = nullptr;
    int index = -1;
  };

  // Decide for the call on `table` with `ctas` CTAs on stream `st` of device `dev`. If the returned choice
  // measures, the caller must launch and then call `after_launch` (same stream) on every path.
  Choice choose(int dev, const void* table, unsigned long long ctas, cudaStream_t st) {
    Choice c;
    if (dev < 0 || dev >= kMaxDevices) return c;
    Dev& d = devs_[dev];
    std::lock_guard<std::mutex> lock(d.mu);
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    const cudaError_t ce = cudaStreamIsCapturing(st, &cs);
    if (ce != cudaSuccess) (void)cudaGetLastError();
    if (ce != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
      // Inside a graph capture: replay the layer's current choice. No set-up, event query, copy or counter
      // update (such calls are not allowed while a stream captures in the global mode).
      const int i = d.ready ? find(d, table) : -1;
      c.exact = i >= 0 && d.entries[i].exact_left > 0;
      return c;
    }
    if (!d.ready && !init(d, dev)) return c;
    const int i = find_or_claim(d, table);
    if (i < 0) return c;  // every slot this table may use has a read-back in flight: no measurement
    Entry& e = d.entries[i];
    e.last_use = ++d.clock;
    consume(d, i);
    if (e.exact_left > 0) {
      if (--e.exact_left == 0) e.since_measure = kMeasureEvery;  // probe on the next call
      c.exact = true;
      return c;
    }
    if (e.pending) return c;
    if (++e.since_measure < kMeasureEvery) return c;
    e.since_measure = 0;
    if (cudaMemsetAsync(d.dev_slots + i, 0, sizeof(unsigned long long), st) != cudaSuccess) {
      (void)cudaGetLastError();
      return c;
    }
    e.ctas = ctas;
    c.slot = d.dev_slots + i;
    c.index = i;
    return c;
  }

  // After the launches of a measuring call: queue the read-back of its counter.
  void after_launch(int dev, const Choice& c, cudaStream_t st) {
    if (c.index < 0 || dev < 0 || dev >= kMaxDevices) return;
    Dev& d = devs_[dev];
    std::lock_guard<std::mutex> lock(d.mu);
    Entry& e = d.entries[c.index];
    if (cudaMemcpyAsync(d.host + c.index, d.dev_slots + c.index, sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                        st) == cudaSuccess &&
        cudaEventRecord(e.done, st) == cudaSuccess)
      e.pending = true;
    else
      (void)cudaGetLastError();
  }

  // The last measured recompute share of the layer using `table` (-1 if none), and whether its next call
  // launches the exact kernel. For tests and diagnostics.
  void state(int dev, const void* table, double* share, int* exact) {
    *share = -1.0;
    *exact = 0;
    if (dev < 0 || dev >= kMaxDevices) return;
    Dev& d = devs_[dev];
    std::lock_guard<std::mutex> lock(d.mu);
    if (!d.ready) return;
    const int i = find(d, table);
    if (i < 0) return;
    Entry& e = d.entries[i];
    consume(d, i);
    *share = e.last_share;
    *exact = e.exact_left > 0;
  }

  // Forget every layer's history on device `dev` (the next call on each layer measures again). Waits for
  // read-backs still in flight.
  void reset(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return;
    Dev& d = devs_[dev];
    std::lock_guard<std::mutex> lock(d.mu);
    if (!d.ready) return;
    for (int i = 0; i < kSlots; ++i) {
      if (d.entries[i].pending) cudaEventSynchronize(d.entries[i].done);
      cudaEvent_t ev = d.entries[i].done;
      d.entries[i] = Entry();
      d.entries[i].done = ev;
    }
  }

 private:
  struct Entry {
    const void* table = nullptr;
    cudaEvent_t done = nullptr;
    bool pending = false;   // a read-back is queued and not yet consumed
    int since_measure = kMeasureEvery - 1;  // speculative calls since the last measurement (first call measures)
    int exact_left = 0;     // calls left on the exact kernel
    unsigned long long ctas = 0;  // CTAs of the measured call
    double last_share = -1.0;
    unsigned long long last_use = 0;
  };
  struct Dev {
    std::mutex mu;
    bool ready = false;
    bool failed = false;  // set up failed once: the device keeps the speculative pass, unmeasured
    unsigned long long* dev_slots = nullptr;  // the device's g_policy_counts
    unsigned long long* host = nullptr;       // its row of the page-locked host mirror
    unsigned long long clock = 0;             // call counter for the least-recently-used choice
    Entry entries[kSlots];
  };

  // A table may use the kWays slots from its hash onwards (open addressing within a short window).
  static constexpr int kWays = 8;
  static int slot_of(const void* table) { return (int)((reinterpret_cast<uintptr_t>(table) >> 8) % kSlots); }

  static int find(Dev& d, const void* table) {
    for (int k = 0, i = slot_of(table); k < kWays; ++k, i = (i + 1) % kSlots)
      if (d.entries[i].table == table) return i;
    return -1;
  }

  // The table's slot, or a new one for it: an empty slot of its window, else the least recently used one
  // without a read-back in flight (-1 if there is none).
  static int find_or_claim(Dev& d, const void* table) {
    const int hit = find(d, table);
    if (hit >= 0) return hit;
    int victim = -1;
    for (int k = 0, i = slot_of(table); k < kWays; ++k, i = (i + 1) % kSlots) {
      const Entry& e = d.entries[i];
      if (e.table == nullptr) {
        victim = i;
        break;
      }
      if (!e.pending && (victim < 0 || e.last_use < d.entries[victim].last_use)) victim = i;
    }
    if (victim < 0) return -1;
    cudaEvent_t ev = d.entries[victim].done;
    d.entries[victim] = Entry();
    d.entries[victim].done = ev;
    d.entries[victim].table = table;
    return victim;
  }

  // Takes in a completed read-back of slot i: the share of the measured call's CTAs that were recomputed,
  // and the switch to the exact kernel above kExactShare.
  static void consume(Dev& d, int i) {
    Entry& e = d.entries[i];
    if (!e.pending || cudaEventQuery(e.done) != cudaSuccess) return;
    e.pending = false;
    e.last_share = e.ctas ? (double)d.host[i] / (double)e.ctas : 0.0;
    if (e.last_share > kExactShare) e.exact_left = kExactCalls;
  }

  // Nothing is allocated: the device counters are a module global, and the host mirror is a static array
  // page-locked once per process (so that the read-back copies are asynchronous).
  bool init(Dev& d, int dev) {
    if (d.failed) return false;
    d.failed = true;  // until every resource below exists
    std::call_once(host_once_, [this]() {
      host_ok_ = cudaHostRegister(host_mirror_, sizeof(host_mirror_), cudaHostRegisterPortable) == cudaSuccess;
    });
    void* p = nullptr;
    if (!host_ok_ || cudaGetSymbolAddress(&p, g_policy_counts) != cudaSuccess) {
      (void)cudaGetLastError();  // must not surface as the launch error of the kernels that follow
      return false;
    }
    d.dev_slots = static_cast<unsigned long long*>(p);
    d.host = host_mirror_[dev];
    for (int i = 0; i < kSlots; ++i) {
      if (cudaEventCreateWithFlags(&d.entries[i].done, cudaEventDisableTiming) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
      }
    }
    d.ready = true;
    d.failed = false;
    return true;
  }

  Dev devs_[kMaxDevices];
  alignas(4096) unsigned long long host_mirror_[kMaxDevices][kSlots] = {};
  std::once_flag host_once_;
  bool host_ok_ = false;
};

inline GlobalPolicy& global_policy() {
  static GlobalPolicy p;
  return p;
}

}  // namespace samrs
