// Causal prefill attention on the 5th-generation tensor cores (sm_100a).
//
// Replaces the prefill attention of the patched Llama / Qwen2 attention
// (flash-attn's varlen forward over the uncompressed prompt,
// heterocache/llama_model.py:353-361, heterocache/qwen_model.py:161-169):
//   out[b, t, h, :] = softmax_j<=t(q[b,h,t] . k[b,h/G,j] * scale) v[b,h/G,j]
// grouped-query (query head h reads KV head h / G), 16-bit q/k/v, fp32
// accumulation, 16-bit output.
//
// One CTA per (pair of consecutive 128-query tiles A and B, query head,
// batch row): each key/value tile fetched into shared memory serves 256
// queries, half the L2 traffic per FLOP of one tile per CTA.  Pairs with
// the longest causal spans are launched first.  Roles (12 warps):
//   warp 0, lane 0: TMA producer of the two query tiles and the key tiles
//     (three stages, a stage released once both tiles' scores are computed);
//   warp 2, lane 0: producer of the value tiles (two stages, released by the
//     second O += P V).  128-token tiles, 64-dim boxes, 128-byte swizzle;
//     the maps cover this GPU's memory only, no multicast;
//   warp 1: allocates the tensor memory -- per tile an S accumulator of 128
//     columns (P is written over its first 64 columns once S is read) and
//     an O accumulator of 128 columns -- and lane 0 issues the MMAs
//       S_X = Q_X K_j^T  (M = 128 queries, N = 128 keys, A and B K-major)
//       O_X += P_X V_j   (M = 128 queries, N = 128 dims; A = P_X from tensor
//                         memory, B = V_j MN-major as loaded)
//     in the order S_A S_B | PV_A S_A' | PV_B S_B' | ..., so the tensor core
//     works on one tile while the softmax warps work on the other;
//   warps 4-7 (tile A) and 8-11 (tile B): softmax, one query row per thread
//     (= TMEM lane): the row max over the tile from a first pass over S
//     (masked on the diagonal tile), running max in the log2 domain, then
//     P = exp2(s * scale - m) in the 16-bit type written over S.  O and the
//     row sum are rescaled only when the max has grown by more than 8 (a
//     factor 256) since the last rescale: P stays below 256 and the final
//     division uses the same reference, so most tiles leave O alone.  At the
//     end O / l goes out.
//   warp 3 has no role.
// Tensor-core MMAs issued by one thread execute in order, so S_X of the next
// key tile, which overwrites P_X, follows the O += P_X V that reads it.
// Every wait is bounded; a wait that gives up marks the launch failed
// (HC_ERR_TIMEOUT), its role stops, copies and MMAs in flight are waited for
// (bounded) and the tensor memory is released before the CTA exits.
#include <cstring>

#include "hc_host.cuh"
#include "hc_params.cuh"
#include "umma.cuh"

namespace hc {

constexpr int kPaThreads = 12 * 32;
constexpr int kPaTile = 128;
constexpr int kPaBox = 128 * 128;         // bytes: 128 rows x 64 16-bit elements
constexpr int kPaTileBytes = 2 * kPaBox;  // one 128 x 128 tile
constexpr int kPaTmemCols = 512;
constexpr int kPaKStages = 3, kPaVStages = 2;
// tensor-memory columns: S_X (P_X in its first 64) at 128 * X, O_X at
// 256 + 128 * X (X = 0 for tile A, 1 for tile B)
constexpr uint32_t kPaColS = 0, kPaColO = 256;
// dynamic shared memory: 1024 bytes of alignment slack, Q_A, Q_B, the K
// stages, the V stages
constexpr size_t kPaSmem = 1024 + (size_t)(2 + kPaKStages + kPaVStages) * kPaTileBytes;

__device__ __forceinline__ void tma_load_4d_plain(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                                  uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kPaThreads, 1)
    prefill_attn_kernel(const PAParams p, const __grid_constant__ CUtensorMap tmq,
                        const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ __align__(16) unsigned char smem_dyn[];
  // the swizzle phase comes from address bits 7-9: buffers on 1024-byte
  // boundaries (the launch reserves the slack)
  unsigned char* sq = smem_dyn + ((1024 - (smem_u32(smem_dyn) & 1023)) & 1023);  // Q_A, then Q_B
  unsigned char* sk = sq + 2 * kPaTileBytes;
  unsigned char* sv = sk + kPaKStages * kPaTileBytes;
  // per tile X: s_full[X] (S_X computed), p_ready[X] (P_X written, O_X
  // rescaled), o_done[X] (O_X += P_X V completed); one phase per key tile
  __shared__ __align__(8) uint64_t q_full, k_full[kPaKStages], k_empty[kPaKStages], v_full[kPaVStages],
      v_empty[kPaVStages], s_full[2], p_ready[2], o_done[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail, s_kissued, s_vissued;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hb = p.H * p.bsz;
  const int npair = (p.n_qt + 1) >> 1;
  const int pi = npair - 1 - (int)(blockIdx.x / hb);
  const int rem = (int)(blockIdx.x % hb);
  const int h = rem % p.H, b = rem / p.H;
  const int kvh = h / p.G;
  const int qa0 = 2 * pi * kPaTile, qb0 = qa0 + kPaTile;
  const bool bact = qb0 < p.L;  // tile B holds queries
  const int nA = 2 * pi + 1;    // key tiles of A: 0..2pi; of B: 0..2pi+1
  const int nB = bact ? nA + 1 : 0;
  const int nkv = bact ? nB : nA;

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
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_ready[x], 4);
      mbar_init(&o_done[x], 1);
    }
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
    // ---- TMA producers: warp 0 the query tiles and the key tiles, warp 2
    // the value tiles
    if (lane == 0) {
      const bool keys = warp == 0;
      const int NS = keys ? kPaKStages : kPaVStages;
      uint64_t* full = keys ? k_full : v_full;
      uint64_t* empty = keys ? k_empty : v_empty;
      unsigned char* ring = keys ? sk : sv;
      const CUtensorMap* map = keys ? &tmk : &tmv;
      int issued = 0;
      if (keys) {
        // rows past L read as zeros; tile B only when it holds queries
        mbar_arrive_expect_tx(&q_full, (uint32_t)((bact ? 2 : 1) * kPaTileBytes));
        tma_load_4d_plain(sq, &tmq, 0, qa0, h, b, &q_full);
        tma_load_4d_plain(sq + kPaBox, &tmq, 64, qa0, h, b, &q_full);
        if (bact) {
          tma_load_4d_plain(sq + kPaTileBytes, &tmq, 0, qb0, h, b, &q_full);
          tma_load_4d_plain(sq + kPaTileBytes + kPaBox, &tmq, 64, qb0, h, b, &q_full);
        }
      }
      // an injected stall (hc_set_wait_limits) loads no key tile: every wait
      // on one runs out, for tests of the timeout path
      const int ntiles = (keys && p.stall) ? 0 : nkv;
      for (int j = 0; j < ntiles; ++j) {
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
      int kw = -1, vw = -1;        // last key / value tile waited for
      int last_s[2] = {-1, -1}, last_pv[2] = {-1, -1};
      auto wait_k = [&](int j) -> bool {
        if (j <= kw) return true;
        if (!mbar_wait(&k_full[j % kPaKStages], (j / kPaKStages) & 1, p.wait_ns)) return false;
        kw = j;
        return true;
      };
      auto wait_v = [&](int j) -> bool {
        if (j <= vw) return true;
        if (!mbar_wait(&v_full[j % kPaVStages], (j / kPaVStages) & 1, p.wait_ns)) return false;
        vw = j;
        return true;
      };
      // S_X = Q_X K_j^T into S_X's columns
      auto issue_s = [&](int x, int j) -> bool {
        if (!wait_k(j)) return false;
        tc_fence_after();
        const uint32_t aq = smem_u32(sq + x * kPaTileBytes);
        const uint32_t bk = smem_u32(sk + (j % kPaKStages) * kPaTileBytes);
        const uint32_t d = tmem + kPaColS + (uint32_t)(128 * x);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * kPaBox + (kk & 3) * 32);
          umma_f16(d, smem_desc_sw128(aq + off), smem_desc_sw128(bk + off), id_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[x]);
        last_s[x] = j;
        return true;
      };
      // O_X += P_X V_j, P_X in the first 64 columns of S_X
      auto issue_pv = [&](int x, int j) -> bool {
        if (!wait_v(j)) return false;
        if (!mbar_wait(&p_ready[x], j & 1, p.wait_ns)) return false;
        tc_fence_after();
        const uint32_t bv = smem_u32(sv + (j % kPaVStages) * kPaTileBytes);
        const uint32_t d = tmem + kPaColO + (uint32_t)(128 * x);
        const uint32_t pa = tmem + kPaColS + (uint32_t)(128 * x);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // A = P_X, keys 16kk.. (8 columns each); B = V, key rows 16kk..
          // (128 bytes a row, the second 64 dims one box further)
          umma_f16_ts(d, pa + (uint32_t)(8 * kk), smem_desc_sw128_mn(bv + (uint32_t)(kk * 16 * 128), kPaBox), id_o,
                      (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[x]);
        last_pv[x] = j;
        return true;
      };
      bool ok = mbar_wait_sleep(&q_full, 0, p.wait_ns);
      if (ok) ok = issue_s(0, 0);
      if (ok && bact) ok = issue_s(1, 0);
      if (ok) umma_commit(&k_empty[0]);
      for (int j = 0; ok && j < nkv; ++j) {
        if (j < nA) {
          ok = issue_pv(0, j);
          if (ok && j + 1 < nA) ok = issue_s(0, j + 1);
        }
        if (ok && bact) ok = issue_pv(1, j);
        if (ok) umma_commit(&v_empty[j % kPaVStages]);
        if (ok && bact && j + 1 < nB) ok = issue_s(1, j + 1);
        if (ok && j + 1 < nkv) umma_commit(&k_empty[(j + 1) % kPaKStages]);
      }
      if (!ok) atomicExch(&s_fail, 1);
      // every MMA issued has completed before the tensor memory is released
      for (int x = 0; x < 2; ++x) {
        if (last_s[x] >= 0) (void)mbar_wait_sleep(&s_full[x], last_s[x] & 1, p.wait_ns);
        if (last_pv[x] >= 0) (void)mbar_wait_sleep(&o_done[x], last_pv[x] & 1, p.wait_ns);
      }
    }
  } else if (warp >= 4) {
    // ---- softmax and output: warps 4-7 tile A, 8-11 tile B, one query row
    // per thread (TMEM lane)
    const int x = (warp - 4) >> 2;
    const int n = x ? nB : nA;                 // key tiles of this tile
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t cs = tmem + lane_off + kPaColS + (uint32_t)(128 * x);
    const uint32_t co = tmem + lane_off + kPaColO + (uint32_t)(128 * x);
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!mbar_wait(&s_full[x], j & 1, p.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = j == n - 1;  // the diagonal tile hides keys after the row
      // pass 1: the row max over the tile (two loads in flight per wait; the
      // registers are read only after the wait)
      float mx = -INFINITY;
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        uint32_t v[64];
        tmem_ld32(cs + (uint32_t)(64 * c2), v);
        tmem_ld32(cs + (uint32_t)(64 * c2 + 32), v + 32);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float s = (diag && 64 * c2 + i > row) ? -INFINITY : __uint_as_float(v[i]);
          mx = fmaxf(mx, s);
        }
      }
      const float m_new = fmaxf(m_used, mx * sl2);  // log2 domain (scale > 0)
      const bool resc = j > 0 && m_new > m_used + 8.f;
      if (j == 0) m_used = m_new;
      if (__any_sync(0xffffffffu, resc)) {
        // O_X += P_X V_{j-1} has completed: O_X is stable (measured: this
        // wait also keeps the common path fast, 0.97 against 0.72 PFLOP/s
        // without it at 32K)
        if (!mbar_wait(&o_done[x], (j - 1) & 1, p.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha = resc ? exp2_approx(m_used - m_new) : 1.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(co + (uint32_t)(32 * c), v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
          tmem_st32(co + (uint32_t)(32 * c), v);
        }
        if (resc) {
          l *= alpha;
          m_used = m_new;
        }
      }
      // pass 2: P = exp2(s * scale_log2 - m) in the 16-bit type, keys in
      // pairs, written over S: the 32 keys of chunk c go to columns
      // 16c..16c+15, whose scores were read in an earlier (or this) chunk
      const float nm = -m_used;
      float ps = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(cs + (uint32_t)(32 * c), v);
        tmem_ld_wait();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int k0 = 32 * c + 2 * i;
          const float s0 = (diag && k0 > row) ? -INFINITY : __uint_as_float(v[2 * i]);
          const float s1 = (diag && k0 + 1 > row) ? -INFINITY : __uint_as_float(v[2 * i + 1]);
          const float e0 = exp2_approx(fmaf(s0, sl2, nm));
          const float e1 = exp2_approx(fmaf(s1, sl2, nm));
          ps += e0 + e1;
          w[i] = Elem<T>::cvt2(e0, e1);
        }
        tmem_st16(cs + (uint32_t)(16 * c), w);
      }
      l += ps;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[x]);
    }
    if (n > 0) {
      if (ok) ok = mbar_wait(&o_done[x], (n - 1) & 1, p.wait_ns);
      if (!ok) {
        atomicExch(&s_fail, 1);
      } else {
        tc_fence_after();
        const int t = (x ? qb0 : qa0) + row;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* dst = reinterpret_cast<T*>(p.out) + (int64_t)b * p.osb + (int64_t)h * p.osh + (int64_t)t * p.ost;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(co + (uint32_t)(32 * c), v);
          tmem_ld_wait();
          if (t < p.L) {
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              uint4 w;
              w.x = Elem<T>::cvt2(__uint_as_float(v[8 * q4]) * inv, __uint_as_float(v[8 * q4 + 1]) * inv);
              w.y = Elem<T>::cvt2(__uint_as_float(v[8 * q4 + 2]) * inv, __uint_as_float(v[8 * q4 + 3]) * inv);
              w.z = Elem<T>::cvt2(__uint_as_float(v[8 * q4 + 4]) * inv, __uint_as_float(v[8 * q4 + 5]) * inv);
              w.w = Elem<T>::cvt2(__uint_as_float(v[8 * q4 + 6]) * inv, __uint_as_float(v[8 * q4 + 7]) * inv);
              *reinterpret_cast<uint4*>(dst + 32 * c + 8 * q4) = w;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && s_fail) {
    set_err(p.err, HC_ERR_TIMEOUT);
    // the copies still in flight (at most the last tile of each stage, and
    // the query tiles) land before the CTA's shared memory is released
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
  const long long grid = (long long)((p.n_qt + 1) / 2) * p.H * p.bsz;
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
  p.stall = injected_stall();
  return dtype == HC_BF16 ? prefill_attn_launch<__nv_bfloat16>(p, maps, st) : prefill_attn_launch<__half>(p, maps, st);
}

}  // namespace hc
