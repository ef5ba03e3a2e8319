// Shared device helpers for the sm_100a compressed-KV attention path.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "heterocache_b200.h"

namespace hc {

constexpr int kPage = HC_PAGE_SIZE;
constexpr int kD = HC_HEAD_DIM;

// ---------------------------------------------------------------------------
// Element traits.  `rnd` rounds an fp32 value to the element type and back
// (round to nearest even), which is how the reference's tensors in the model
// dtype hold every intermediate.  `key` maps a value that is exactly
// representable in the element type to an unsigned integer whose order is the
// value's order (the radix-select key); kKeyBits is its width.
template <typename T> struct Elem;

template <> struct Elem<float> {
  static constexpr int kKeyBits = 32;
  __device__ __forceinline__ static float to_f(float x) { return x; }
  __device__ __forceinline__ static float from_f(float x) { return x; }
  __device__ __forceinline__ static float rnd(float x) { return x; }
  __device__ __forceinline__ static float pack(float x) { return x; }
  __device__ __forceinline__ static void rnd2(float&, float&) {}
  __device__ __forceinline__ static uint32_t key(float x) {
    uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  }
  __device__ __forceinline__ static float unkey(uint32_t k) {
    uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(b);
  }
};

template <> struct Elem<__nv_bfloat16> {
  static constexpr int kKeyBits = 16;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  __device__ __forceinline__ static float rnd(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
  // two values with one packed conversion (half the conversion-unit work)
  __device__ __forceinline__ static void rnd2(float& a, float& b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(&h);
    a = __uint_as_float(w << 16);
    b = __uint_as_float(w & 0xffff0000u);
  }
  // x already holds a bf16 value: keep its upper half
  __device__ __forceinline__ static __nv_bfloat16 pack(float x) {
    return __ushort_as_bfloat16((unsigned short)(__float_as_uint(x) >> 16));
  }
  // a and b already hold bf16 values: a in the low half, b in the high half
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    return __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x7632);
  }
  // any two floats, rounded to nearest: a in the low half, b in the high half
  __device__ __forceinline__ static uint32_t cvt2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint32_t key(float x) {
    uint32_t b = __float_as_uint(x) >> 16;  // exact: x is a bf16 value
    return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
  }
  __device__ __forceinline__ static float unkey(uint32_t k) {
    uint32_t b = (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu);
    return __uint_as_float(b << 16);
  }
};

template <> struct Elem<__half> {
  static constexpr int kKeyBits = 16;
  __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
  __device__ __forceinline__ static float rnd(float x) { return __half2float(__float2half_rn(x)); }
  __device__ __forceinline__ static __half pack(float x) { return __float2half_rn(x); }  // exact
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {  // exact: f16 values
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint32_t cvt2(float a, float b) { return pack2(a, b); }  // rounds to nearest
  __device__ __forceinline__ static void rnd2(float& a, float& b) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 f = __half22float2(h);
    a = f.x;
    b = f.y;
  }
  __device__ __forceinline__ static uint32_t key(float x) {
    uint32_t b = (uint32_t)__half_as_ushort(__float2half_rn(x));  // exact: x is an f16 value
    return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
  }
  __device__ __forceinline__ static float unkey(uint32_t k) {
    uint32_t b = (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu);
    return __half2float(__ushort_as_half((unsigned short)b));
  }
};

// Unpack two 16-bit elements of a 32-bit word to fp32.
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t w);
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}

// ---------------------------------------------------------------------------
// Warp-level tensor-core product D += A(16x16) * B(16x8), fp32 accumulate.
template <typename T> __device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                                                uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1);
template <> __device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1,
                                                                     uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <> __device__ __forceinline__ void mma16816<__half>(float (&d)[4], uint32_t a0, uint32_t a1,
                                                              uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// x / y rounded to nearest-even, for a divisor y known in advance with
// r = 1/y rounded to nearest: Markstein's correction step (P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Dev. 34(1), 1990): q = x*r, the exact residual
// e = x - q*y from one fused multiply-add, then q + e*r.  Branch-free.  It is
// exact for every fp32 x when y is 3, 5, 7 or 9, and for every bf16 / f16 x
// divided by sqrt(128) whose quotient is a normal number (so callers send
// |x| < 2^-120 to IEEE division); the unit tests check both exhaustively.
__device__ __forceinline__ float div_known(float x, float y, float r) {
  const float q = x * r;
  const float e = fmaf(-q, y, x);
  return fmaf(e, r, q);
}

__device__ __forceinline__ uint4 ldg128(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint2 ldg64(const void* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }

// Streaming load that does not allocate in L1 (data read once).
// L2 policy for data read once per step and larger than L2 (key/value
// streams): its lines are evicted first, so that it does not push the
// kernels' code, page tables and scratch out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
// Streaming load with an L2 policy (l2_evict_first_policy).
__device__ __forceinline__ uint4 ld_stream128(const void* p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ uint4 ld_stream128(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ld_stream64(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

__device__ __forceinline__ void set_err(int32_t* err, int code) {
  if (err) atomicOr(err, 1 << code);
}

// 2^x on the multi-function unit (ex2.approx.ftz: relative error about
// 2^-22, far below the 16-bit rounding the probabilities get; 2^-inf = 0).
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// Grid barrier for cooperative launches (all CTAs co-resident).  Monotonic
// arrival counter: barrier number e completes when count >= e * nblocks
// (+ `extra`, an injected arrival that never comes: 0 in normal use).
// Every wait is bounded (limit_ns, by default kBarrierTimeoutNs); on timeout
// the CTA sets `abort` and HC_ERR_TIMEOUT and every CTA leaves the kernel at
// its next barrier.  The state resets itself: after the final barrier each
// CTA increments `depart`, and the last to depart zeroes the counters (an
// aborted launch leaves the state for the caller to zero).
struct GridBarrier {
  unsigned int count;
  unsigned int depart;
  unsigned int abort;
  unsigned int pad;
};

constexpr uint64_t kBarrierTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Returns false if the grid aborted (caller must return).
__device__ __forceinline__ bool grid_sync(GridBarrier* gb, unsigned int nblocks, unsigned int& epoch,
                                          int32_t* err, uint64_t limit_ns = kBarrierTimeoutNs,
                                          unsigned int extra = 0u) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    epoch += 1;
    const unsigned int target = epoch * nblocks + extra;
    // release-add: the CTA's writes (ordered before by the block barrier)
    // become visible to every CTA that acquires the count
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(&gb->count), "r"(1u) : "memory");
    int ok = 1;
    uint64_t t0 = 0;
    unsigned int spins = 0;
    while (true) {
      if (ld_acquire_u32(&gb->count) >= target) break;
      if ((++spins & 31u) == 0) {
        if (ld_acquire_u32(&gb->abort)) { ok = 0; break; }
        uint64_t now = globaltimer_ns();
        if (t0 == 0) t0 = now;
        else if (now - t0 > limit_ns) {
          atomicExch(&gb->abort, 1u);
          set_err(err, HC_ERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
      __nanosleep(20);
    }
    __threadfence();
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Call once per CTA after its last grid_sync (only if no abort happened).
__device__ __forceinline__ void grid_depart(GridBarrier* gb, unsigned int nblocks) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int d = atomicAdd(&gb->depart, 1u);
    if (d == nblocks - 1) {
      gb->count = 0;
      gb->depart = 0;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA engine) helpers.  Every wait is bounded
// (limit_ns, by default kMbarTimeoutNs); callers turn a timeout into
// HC_ERR_TIMEOUT.
constexpr uint64_t kMbarTimeoutNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Retire an mbarrier before its memory is initialised again (no arrival or
// wait may be pending on it).
__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kMbarTimeoutNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}
// The same, with the waiting thread suspended (up to `hint_ns` per try, woken
// when the phase completes) instead of spinning: for roles that wait while
// other warps of the SM need the issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_sleep(bar, parity, 2000u)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
  return r;
}
// Store two 8x8 16-bit matrices held in the mma accumulator layout (lane l:
// row l/4, columns 2(l%4), 2(l%4)+1 of each), transposed: memory row j of
// matrix m (address from lane 8m + j) receives column j.
__device__ __forceinline__ void stmatrix2_trans(uint32_t addr, uint32_t m0, uint32_t m1) {
  asm volatile("stmatrix.sync.aligned.m8n8.x2.trans.shared.b16 [%0], {%1, %2};\n" ::"r"(addr), "r"(m0), "r"(m1)
               : "memory");
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 r;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "r"(addr));
  return r;
}
// Programmatic dependent launch: the dependent grid may start before this one
// ends (trigger) and waits for its completion and memory (wait).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024).
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) s_warp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  total = s_warp[nw - 1];
  int base = wid > 0 ? s_warp[wid - 1] : 0;
  int excl = base + x - v;
  __syncthreads();
  return excl;
}

}  // namespace hc
