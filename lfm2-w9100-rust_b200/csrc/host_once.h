#pragma once
// Per-device one-time host setup. Kernel attributes (the dynamic shared memory
// limit, the carveout) are set on the current device's copy of a kernel, so a
// process that drives several GPUs must set them once on each.
#include <cuda_runtime.h>

#include <mutex>

namespace lfm {

// Runs f() the first time the calling thread's current device reaches this
// call site (`done` and `mu` are the call site's statics). Thread-safe.
template <class F>
inline void once_per_device(unsigned long long& done, std::mutex& mu, F&& f) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = (dev >= 0 && dev < 64) ? 1ull << dev : 0ull;
  std::lock_guard<std::mutex> lock(mu);
  if (bit && (done & bit)) return;
  f();
  done |= bit;
}

}  // namespace lfm
