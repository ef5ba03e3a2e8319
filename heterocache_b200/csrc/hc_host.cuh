// Host-side caches of the library's launch set-up (SM counts, kernel
// attributes, occupancy, tensor maps).  Every cache is kept per device
// ordinal and every lookup or update holds one process-wide lock, so the
// library may be called from several host threads and for several devices in
// one process.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "heterocache_b200.h"

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

// cuTensorMapEncodeTiled through the runtime's driver entry point (looked up
// once), or null if the driver does not provide it.
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Tensor map of a pool viewed as a 2-D [rows, 128] array of 16-bit elements
// (rows = n_blocks * 256), boxes of box_rows rows x 64 elements, 128-byte
// swizzle.  Encoded once per (device, pool address, rows, dtype, box) and
// cached; false if it cannot be encoded.
inline bool pool_tensor_map(CUtensorMap* out, const void* base, long long rows, int dtype, int box_rows) {
  struct Entry { int dev; const void* base; long long rows; int dtype, box; CUtensorMap map; };
  static Entry cache[256];
  static int n = 0, next = 0;
  const int dev = current_device();
  auto encode = tensor_map_encoder();
  if (dev < 0 || !encode) return false;
  std::lock_guard<std::mutex> g(host_lock());
  for (int i = 0; i < n; ++i)
    if (cache[i].dev == dev && cache[i].base == base && cache[i].rows == rows && cache[i].dtype == dtype &&
        cache[i].box == box_rows) {
      *out = cache[i].map;
      return true;
    }
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)HC_HEAD_DIM, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)HC_HEAD_DIM * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType ty =
      dtype == HC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (encode(&map, ty, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  Entry& e = cache[n < 256 ? n++ : (next++ % 256)];
  e.dev = dev;
  e.base = base;
  e.rows = rows;
  e.dtype = dtype;
  e.box = box_rows;
  e.map = map;
  *out = map;
  return true;
}

// Tensor map of a strided [bsz, heads, L, 128] array of 16-bit elements (element
// strides sb, sh, st), boxes of box_rows tokens x 64 elements of one (batch,
// head), 128-byte swizzle; rows past L read as zeros.  False if it cannot be
// encoded (e.g. a stride the TMA unit does not accept).
inline bool dense_tensor_map(CUtensorMap* out, const void* base, int bsz, int heads, int L, int64_t sb, int64_t sh,
                             int64_t st, int dtype, int box_rows) {
  auto encode = tensor_map_encoder();
  if (!encode || bsz <= 0 || heads <= 0 || L <= 0) return false;
  // a dimension of extent 1 is never stepped over: give it a valid stride
  if (heads == 1) sh = st * L;
  if (bsz == 1) sb = sh * heads;
  const cuuint64_t dims[4] = {(cuuint64_t)HC_HEAD_DIM, (cuuint64_t)L, (cuuint64_t)heads, (cuuint64_t)bsz};
  const cuuint64_t strides[3] = {(cuuint64_t)st * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType ty =
      dtype == HC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode(out, ty, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace hc
