// Causal prefill attention on the 5th-generation tensor cores (sm_100a).
//
// Replaces the prefill attention of the patched Llama / Qwen2 attention
// (flash-attn's varlen forward over the uncompressed prompt,
// heterocache/llama_model.py:353-361, heterocache/qwen_model.py:161-169):
//   out[b, t, h, :] = softmax_j<=t(q[b,h,t] . k[b,h/G,j] * scale) v[b,h/G,j]
// grouped-query (query head h reads KV head h / G), 16-bit q/k/v, fp32
// accumulation, 16-bit output.
//
// One CTA per (128-query tile, query head, batch row); the tiles with the
// longest causal spans are launched first.  Roles (12 warps):
//   warp 0, lane 0: TMA producer of the query tile and the key tiles (a
//     three-stage ring, each stage released as soon as its scores are
//     computed); warp 2, lane 0: producer of the value tiles (two stages,
//     released by O += P V).  128-token tiles, 64-dim boxes, 128-byte
//     swizzle; the maps cover this GPU's memory only, no multicast;
//   warp 1: allocates the tensor memory (512 columns: two score
//     accumulators of 128 columns, the output accumulator, two P buffers
//     of 64 columns); lane 0 issues the MMAs
//       S_j = Q K_j^T  (M = 128 queries, N = 128 keys, A and B K-major)
//       O  += P_j V_j  (M = 128 queries, N = 128 dims; A = P_j from tensor
//                       memory, written there by the softmax warps; B = V_j,
//                       MN-major as loaded)
//     S_{j+1} is issued before O += P_j V_j, so the tensor core computes the
//     next scores while the softmax warps work on the current ones;
//   warps 4-11: softmax, two threads per query row (= TMEM lane), one for
//     each half of the row's keys and output dims: read S_j, mask the
//     diagonal tile, trade the halves' maxima, running max in the log2
//     domain, P = exp2(s * scale - m) into tensor memory in the 16-bit type
//     (two buffers: writing P_{j+1} waits only for O += P_{j-1} V_{j-1}).
//     O and the row sum are rescaled only when the max has grown by more
//     than 8 (a factor 256) since the last rescale: P stays below 256 and
//     the final division uses the same reference, so most tiles leave O
//     alone.  At the end O / l goes out.
//   warp 3 has no role.
// Every wait is bounded; a wait that gives up marks the launch failed
// (HC_ERR_TIMEOUT), its role stops, copies and MMAs in flight are waited for
// (bounded) and the tensor memory is released before the CTA exits.
#include <cstring>

#include "hc_host.cuh"
#include "hc_params.cuh"
#include "umma.cuh"

namespace hc {

constexpr int kPaSoftmaxWarps = 8;
constexpr int kPaThreads = (4 + kPaSoftmaxWarps) * 32;
constexpr int kPaTile = 128;
constexpr int kPaBox = 128 * 128;         // bytes: 128 rows x 64 16-bit elements
constexpr int kPaTileBytes = 2 * kPaBox;  // one 128 x 128 tile
constexpr int kPaTmemCols = 512;
constexpr int kPaKStages = 3, kPaVStages = 2;
// tensor-memory columns: S buffers at 0 and 128, O at 256, P buffers at 384
// and 448 (64 columns: 128 16-bit keys per lane)
constexpr uint32_t kPaColO = 256, kPaColP = 384;
// dynamic shared memory: 1024 bytes of alignment slack, Q, the K stages, the
// V stages
constexpr size_t kPaSmem = 1024 + (size_t)(1 + kPaKStages + kPaVStages) * kPaTileBytes;

__device__ __forceinline__ void tma_load_4d_plain(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                                  uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

// 2^x on the multi-function unit (ex2.approx.ftz: relative error about
// 2^-22, far below the 16-bit rounding P gets; 2^-inf = 0).
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__global__ void __launch_bounds__(kPaThreads, 1)
    prefill_attn_kernel(const PAParams p, const __grid_constant__ CUtensorMap tmq,
                        const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ __align__(16) unsigned char smem_dyn[];
  // the swizzle phase comes from address bits 7-9: buffers on 1024-byte
  // boundaries (the launch reserves the slack)
  unsigned char* sq = smem_dyn + ((1024 - (smem_u32(smem_dyn) & 1023)) & 1023);
  unsigned char* sk = sq + kPaTileBytes;
  unsigned char* sv = sk + kPaKStages * kPaTileBytes;
  // o_done[b]: completions of O += P_j V_j for j of parity b (two barriers, so
  // that a wait for the one before last cannot be passed by the last)
  __shared__ __align__(8) uint64_t q_full, k_full[kPaKStages], k_empty[kPaKStages], v_full[kPaVStages],
      v_empty[kPaVStages], s_full[2], s_free[2], p_ready, o_done[2], x_bar;
  __shared__ float s_hmax[2][2][kPaTile], s_hsum[2][kPaTile];  // halves' row maxima and sums
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail, s_kissued, s_vissued;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hb = p.H * p.bsz;
  const int qt = p.n_qt - 1 - (int)(blockIdx.x / hb);
  const int rem = (int)(blockIdx.x % hb);
  const int h = rem % p.H, b = rem / p.H;
  const int kvh = h / p.G;
  const int q0 = qt * kPaTile;
  const int nkv = qt + 1;  // causal: key tiles 0..qt

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kPaKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kPaVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], kPaSoftmaxWarps);
    }
    mbar_init(&p_ready, kPaSoftmaxWarps);
    mbar_init(&o_done[0], 1);
    mbar_init(&o_done[1], 1);
    mbar_init(&x_bar, kPaSoftmaxWarps);
    s_fail = 0;
    s_kissued = s_vissued = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, (uint32_t)kPaTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0 || warp == 2) {
    // ---- TMA producers: warp 0 the query and key tiles, warp 2 the values
    if (lane == 0) {
      const bool keys = warp == 0;
      const int NS = keys ? kPaKStages : kPaVStages;
      uint64_t* full = keys ? k_full : v_full;
      uint64_t* empty = keys ? k_empty : v_empty;
      unsigned char* ring = keys ? sk : sv;
      const CUtensorMap* map = keys ? &tmk : &tmv;
      int issued = 0;
      if (keys) {
        mbar_arrive_expect_tx(&q_full, (uint32_t)kPaTileBytes);
        tma_load_4d_plain(sq, &tmq, 0, q0, h, b, &q_full);
        tma_load_4d_plain(sq + kPaBox, &tmq, 64, q0, h, b, &q_full);
      }
      for (int j = 0; j < nkv; ++j) {
        const int s = j % NS;
        if (!mbar_wait_sleep(&empty[s], ((j / NS) & 1) ^ 1, p.wait_ns)) {
          atomicExch(&s_fail, 1);
          break;
        }
        unsigned char* dst = ring + s * kPaTileBytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)kPaTileBytes);
        tma_load_4d_plain(dst, map, 0, j * kPaTile, kvh, b, &full[s]);
        tma_load_4d_plain(dst + kPaBox, map, 64, j * kPaTile, kvh, b, &full[s]);
        issued = j + 1;
      }
      if (keys) s_kissued = issued;
      else s_vissued = issued;
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      const uint32_t id_s = idesc_f16_m128(kBf16, 128);
      const uint32_t id_o = idesc_f16_m128(kBf16, 128) | kIdescBMajorMN;
      const uint32_t aq = smem_u32(sq);
      int last_s = -1, last_pv = -1;
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1, ks = j % kPaKStages;
        if (!mbar_wait(&k_full[ks], (j / kPaKStages) & 1, p.wait_ns)) return false;
        if (!mbar_wait(&s_free[s], ((j >> 1) & 1) ^ 1, p.wait_ns)) return false;
        tc_fence_after();
        const uint32_t bk = smem_u32(sk + ks * kPaTileBytes);
        const uint32_t d = tmem + (uint32_t)(s * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * kPaBox + (kk & 3) * 32);
          umma_f16(d, smem_desc_sw128(aq + off), smem_desc_sw128(bk + off), id_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[s]);
        umma_commit(&k_empty[ks]);
        last_s = j;
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int vs = j % kPaVStages;
        if (!mbar_wait(&v_full[vs], (j / kPaVStages) & 1, p.wait_ns)) return false;
        if (!mbar_wait(&p_ready, j & 1, p.wait_ns)) return false;
        tc_fence_after();
        const uint32_t bv = smem_u32(sv + vs * kPaTileBytes);
        const uint32_t d = tmem + kPaColO;
        const uint32_t pa = tmem + kPaColP + (uint32_t)((j & 1) * 64);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // A = P_j, keys 16kk.. (8 columns each); B = V, key rows 16kk..
          // (128 bytes a row, the second 64 dims one box further)
          umma_f16_ts(d, pa + (uint32_t)(8 * kk), smem_desc_sw128_mn(bv + (uint32_t)(kk * 16 * 128), kPaBox), id_o,
                      (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[j & 1]);
        umma_commit(&v_empty[vs]);
        last_pv = j;
        return true;
      };
      bool ok = mbar_wait_sleep(&q_full, 0, p.wait_ns);
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nkv; ++j) {
        if (j + 1 < nkv) ok = issue_s(j + 1);
        if (ok) ok = issue_pv(j);
      }
      if (!ok) atomicExch(&s_fail, 1);
      // every MMA issued has completed before the tensor memory is released
      if (last_s >= 0) (void)mbar_wait_sleep(&s_full[last_s & 1], (last_s >> 1) & 1, p.wait_ns);
      if (last_pv >= 0) (void)mbar_wait_sleep(&o_done[last_pv & 1], (last_pv >> 1) & 1, p.wait_ns);
    }
  } else if (warp >= 4) {
    // ---- softmax and output: two threads per query row (TMEM lane), warps
    // 4-7 the columns 0-63 of S (keys) and of O (dims), warps 8-11 the
    // columns 64-127; the two halves of a row trade their maxima (and at the
    // end their sums) through shared memory, meeting on an mbarrier
    const int quarter = warp & 3, half = (warp - 4) >> 2;
    const int row = 32 * quarter + lane;
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    const int col0 = 64 * half;
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    auto meet = [&](int k) -> bool {  // both halves' values of exchange k are in
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_bar);
      return mbar_wait(&x_bar, k & 1, p.wait_ns);
    };
    for (int j = 0; j < nkv; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1, p.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // this half of the row's scores: two loads in flight, then one wait
      // (the registers are read only after it)
      uint32_t xr[64];
      tmem_ld32(tmem + lane_off + (uint32_t)(s * 128 + col0), xr);
      tmem_ld32(tmem + lane_off + (uint32_t)(s * 128 + col0 + 32), xr + 32);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[s]);
      float x[64];
#pragma unroll
      for (int k = 0; k < 64; ++k) x[k] = __uint_as_float(xr[k]);
      if (j == qt) {  // the diagonal tile hides keys after the row
#pragma unroll
        for (int k = 0; k < 64; ++k)
          if (col0 + k > row) x[k] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int k = 0; k < 64; ++k) mx = fmaxf(mx, x[k]);
      s_hmax[j & 1][half][row] = mx;
      if (!meet(j)) {
        ok = false;
        break;
      }
      mx = fmaxf(mx, s_hmax[j & 1][half ^ 1][row]);
      const float m_new = fmaxf(m_used, mx * sl2);  // log2 domain (scale > 0)
      const bool resc = j > 0 && m_new > m_used + 8.f;  // the same in both halves
      const bool any_resc = __any_sync(0xffffffffu, resc);
      if (j == 0) m_used = m_new;
      if (any_resc) {
        // O += P_{j-1} V_{j-1} (and every product before it) has completed:
        // O is stable, and P's buffer (last read by O += P_{j-2} V_{j-2}) free
        if (!mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, p.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha = resc ? exp2_approx(m_used - m_new) : 1.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[16];
          const uint32_t ta = tmem + lane_off + kPaColO + (uint32_t)(col0 + 16 * c);
          tmem_ld16(ta, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
          tmem_st16(ta, v);
        }
        tmem_st_wait();
        if (resc) {
          l *= alpha;
          m_used = m_new;
        }
      } else if (j >= 2) {
        // P's buffer was last read by O += P_{j-2} V_{j-2}
        if (!mbar_wait(&o_done[j & 1], ((j - 2) >> 1) & 1, p.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // P = exp2(s * scale_log2 - m) in the 16-bit type into this half's 32
      // columns of P buffer j & 1, keys in pairs (masked scores give
      // exp2(-inf) = 0)
      const float nm = -m_used;
      float ps = 0.f;
      uint32_t pw[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float e0 = exp2_approx(fmaf(x[2 * c], sl2, nm));
        const float e1 = exp2_approx(fmaf(x[2 * c + 1], sl2, nm));
        ps += e0 + e1;
        pw[c] = Elem<T>::cvt2(e0, e1);
      }
      tmem_st32(tmem + lane_off + kPaColP + (uint32_t)((j & 1) * 64 + 32 * half), pw);
      l += ps;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready);
    }
    if (ok) ok = mbar_wait(&o_done[(nkv - 1) & 1], ((nkv - 1) >> 1) & 1, p.wait_ns);
    if (ok) {
      s_hsum[half][row] = l;
      ok = meet(nkv);
    }
    if (!ok) {
      atomicExch(&s_fail, 1);
    } else {
      tc_fence_after();
      const float lt = l + s_hsum[half ^ 1][row];
      const int t = q0 + row;
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      T* dst = reinterpret_cast<T*>(p.out) + (int64_t)b * p.osb + (int64_t)h * p.osh + (int64_t)t * p.ost + col0;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[16];
        tmem_ld16(tmem + lane_off + kPaColO + (uint32_t)(col0 + 16 * c), v);
        tmem_ld_wait();
        if (t < p.L) {
          uint4 w0, w1;
          w0.x = Elem<T>::cvt2(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv);
          w0.y = Elem<T>::cvt2(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv);
          w0.z = Elem<T>::cvt2(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv);
          w0.w = Elem<T>::cvt2(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv);
          w1.x = Elem<T>::cvt2(__uint_as_float(v[8]) * inv, __uint_as_float(v[9]) * inv);
          w1.y = Elem<T>::cvt2(__uint_as_float(v[10]) * inv, __uint_as_float(v[11]) * inv);
          w1.z = Elem<T>::cvt2(__uint_as_float(v[12]) * inv, __uint_as_float(v[13]) * inv);
          w1.w = Elem<T>::cvt2(__uint_as_float(v[14]) * inv, __uint_as_float(v[15]) * inv);
          *reinterpret_cast<uint4*>(dst + 16 * c) = w0;
          *reinterpret_cast<uint4*>(dst + 16 * c + 8) = w1;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && s_fail) {
    set_err(p.err, HC_ERR_TIMEOUT);
    // the copies still in flight (at most the last tile of each stage, and
    // the query tile) land before the CTA's shared memory is released
    (void)mbar_wait_sleep(&q_full, 0, p.wait_ns);
    for (int j = max(0, s_kissued - kPaKStages); j < s_kissued; ++j)
      (void)mbar_wait_sleep(&k_full[j % kPaKStages], (j / kPaKStages) & 1, p.wait_ns);
    for (int j = max(0, s_vissued - kPaVStages); j < s_vissued; ++j)
      (void)mbar_wait_sleep(&v_full[j % kPaVStages], (j / kPaVStages) & 1, p.wait_ns);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)kPaTmemCols);
  }
}

template <typename T>
static int prefill_attn_launch(const PAParams& p, const CUtensorMap* maps, cudaStream_t st) {
  auto kern = prefill_attn_kernel<T>;
  static bool attr_set[kMaxDevices];
  const int dev = current_device();
  if (dev < 0) return HC_ERR_CUDA;
  {
    std::lock_guard<std::mutex> g(host_lock());
    if (!attr_set[dev]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPaSmem) != cudaSuccess)
        return HC_ERR_CUDA;
      attr_set[dev] = true;
    }
  }
  const long long grid = (long long)p.n_qt * p.H * p.bsz;
  if (grid <= 0) return HC_OK;
  if (grid > 0x7fffffffLL) return HC_ERR_UNSUPPORTED;
  prefill_attn_kernel<T><<<(unsigned int)grid, kPaThreads, kPaSmem, st>>>(p, maps[0], maps[1], maps[2]);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

int prefill_attn_dispatch(int dtype, PAParams& p, const void* q, int64_t qsb, int64_t qsh, int64_t qst,
                          const void* k, int64_t ksb, int64_t ksh, int64_t kst, const void* v, int64_t vsb,
                          int64_t vsh, int64_t vst, cudaStream_t st) {
  if (dtype != HC_BF16 && dtype != HC_F16) return HC_ERR_UNSUPPORTED;
  CUtensorMap maps[3];
  std::memset(maps, 0, sizeof(maps));
  if (!dense_tensor_map(&maps[0], q, p.bsz, p.H, p.L, qsb, qsh, qst, dtype, kPaTile) ||
      !dense_tensor_map(&maps[1], k, p.bsz, p.KV, p.L, ksb, ksh, kst, dtype, kPaTile) ||
      !dense_tensor_map(&maps[2], v, p.bsz, p.KV, p.L, vsb, vsh, vst, dtype, kPaTile))
    return HC_ERR_INVALID;
  p.n_qt = (p.L + kPaTile - 1) / kPaTile;
  p.wait_ns = wait_limit_ns(kMbarTimeoutNs);
  return dtype == HC_BF16 ? prefill_attn_launch<__nv_bfloat16>(p, maps, st) : prefill_attn_launch<__half>(p, maps, st);
}

}  // namespace hc
