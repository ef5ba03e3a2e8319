// Host-side caches of the library's launch set-up (SM counts, kernel
// attributes, occupancy, tensor maps).  Every cache is kept per device
// ordinal and every lookup or update holds one process-wide lock, so the
// library may be called from several host threads and for several devices in
// one process.
#pragma once

#include <cuda_runtime.h>

#include <mutex>

namespace hc {

constexpr int kMaxDevices = 64;

inline std::mutex& host_lock() {
  static std::mutex m;
  return m;
}

// Ordinal of the calling thread's current device, or -1 (query failed or an
// ordinal beyond kMaxDevices).
inline int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) return -1;
  return d;
}

// SM count of device `dev` (queried once; 148 if the query fails).
inline int device_sms(int dev) {
  static int sms[kMaxDevices] = {0};
  if (dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> g(host_lock());
  if (sms[dev] <= 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    sms[dev] = n;
  }
  return sms[dev];
}

// A small per-device map from a launch shape (one integer key) to a value,
// e.g. dynamic shared-memory bytes -> co-resident CTAs.  Callers hold
// host_lock() around find/put.
template <int N>
struct ShapeCache {
  long long key[kMaxDevices][N];
  long long val[kMaxDevices][N];
  int n[kMaxDevices] = {0};
  bool find(int dev, long long k, long long& v) const {
    for (int i = 0; i < n[dev]; ++i)
      if (key[dev][i] == k) {
        v = val[dev][i];
        return true;
      }
    return false;
  }
  void put(int dev, long long k, long long v) {
    if (n[dev] < N) {
      key[dev][n[dev]] = k;
      val[dev][n[dev]] = v;
      ++n[dev];
    }
  }
};

}  // namespace hc
