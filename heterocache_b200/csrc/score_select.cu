// Fused token scoring + budgeted top-k for the three selection stages of the
// HeteroCache path, one cooperative launch each:
//
//   prefill select  (heterocache/cache_utils.py:782-882): compressed heads,
//                   top keep_len[h] positions -> written to the head's pages.
//   pivot init      (heterocache/cache_utils.py:1149-1190): pivot heads,
//                   top-K_base positions -> reference set (positions + bitmap).
//   drift check     (heterocache/cache_utils.py:1007-1082): S buffered decode
//                   queries per pivot, top-K_base per step, overlap with the
//                   reference set, median, trigger; top-max_len positions of
//                   the last step for the retrieval.
//
// One "job" is one (batch row, KV head).  Each job's L tokens are split into
// contiguous ranges of T tokens, one CTA per range.  Phases, separated by
// grid barriers:
//   1. logits of every query row for the CTA's tokens (plus a 16-token margin
//      each side for the pooling halo) -> shared memory; per-row partial
//      max / sum-of-exp over the CTA's own tokens -> workspace.
//   2. global softmax statistics; p = dtype(exp(x - M) / sum); window sum;
//      pooling; max over the GQA group -> one orderable key per token and
//      score row.
//   3. radix select of the k-th largest key per select (8-bit digits; 2
//      rounds for 16-bit dtypes, 4 for fp32) with global histograms.
//   4. per-CTA counts of keys above / equal to the threshold; ranks in
//      position order (ties at the threshold go to the lowest positions), so
//      the selected positions come out ascending without a sort.
//   5. the stage's epilogue (page writes / reference set / overlap + trigger).
//
// Rounding points follow the reference exactly: q.K^T rounded to the model
// dtype, then divided by sqrt(d) and rounded, fp32 softmax rounded to the
// dtype, the window sum rounded, the pooling output rounded.
#include <cstring>

#include "hc_host.cuh"
#include "hc_params.cuh"
#include "umma.cuh"

namespace hc {



// Kernel parameter carrying a drift-check batch (DRIFT mode only).
template <int MODE>
using BatchOf = typename std::conditional<MODE == MODE_DRIFT, DriftBatch, NoBatch>::type;

// DRIFT mode: the job's result locations.
struct DriftView {
  uint32_t* bitmap;
  int32_t* ref_pos;
  int32_t* trigger;
  int32_t* retr;
  int retr_cap;
  float* coeffs;
  double* median;
  int max_len;
};

struct JobInfo {
  int b, h, job, part, t0, t1;
  // DRIFT mode: page ids of the CTA's token range, staged in shared memory
  // (npages == 0: look them up in the block table)
  const int* pages;
  int page0, npages;
};

constexpr int kMaxPages = 64;

__device__ __forceinline__ JobInfo job_info(const ScoreParams& p) {
  JobInfo ji;
  ji.job = blockIdx.x / p.cpj;
  ji.part = blockIdx.x % p.cpj;
  if (p.mode == MODE_PREFILL) {
    ji.b = ji.job / p.nh;
    ji.h = ji.job % p.nh;
  } else if (p.mode == MODE_PIVOT) {
    ji.b = ji.job / p.nh;
    ji.h = p.first_head + ji.job % p.nh;
  } else {
    ji.b = 0;
    ji.h = p.job_heads ? p.job_heads[ji.job] : 0;  // a batch sets it from the job
  }
  ji.t0 = ji.part * p.T;
  ji.t1 = min(p.L, ji.t0 + p.T);
  ji.pages = nullptr;
  ji.page0 = ji.npages = 0;
  return ji;
}

// Address of key row t of the job (dense tensor or paged pool).
template <typename T>
__device__ __forceinline__ const T* key_row(const ScoreParams& p, const JobInfo& ji, int t) {
  if (p.mode == MODE_DRIFT) {
    int blk;
    if (ji.npages) {
      // rows past the staged range (a tile's tail beyond the CTA's keys) only
      // feed discarded logits: clamp them to the last staged page
      const int i = min((t >> 8) - ji.page0, ji.npages - 1);
      blk = ji.pages[i];  // validated when staged (-1: reported, read page 0)
      if (blk < 0) blk = 0;
    } else {
      const int row = ji.b * p.KV + ji.h;
      blk = p.bt[(int64_t)row * p.max_blocks + (t >> 8)];
      if (blk < 0 || blk >= p.n_blocks) {  // keep the address inside the pool; report
        set_err(p.err, HC_ERR_RANGE);
        blk = 0;
      }
    }
    return reinterpret_cast<const T*>(p.k_pool) + ((int64_t)blk * kPage + (t & (kPage - 1))) * kD;
  }
  return reinterpret_cast<const T*>(p.k) + ji.b * p.ksb + (int64_t)ji.h * p.ksh + (int64_t)t * p.kst;
}

// Query row qi = (s*G + g)*W + w of the job.
template <typename T>
__device__ __forceinline__ const T* query_row(const ScoreParams& p, const JobInfo& ji, int qi) {
  int w = qi % p.W;
  int sg = qi / p.W;
  int g = sg % p.G;
  int s = sg / p.G;
  int tok = p.q_tok0 + s + w;
  return reinterpret_cast<const T*>(p.q) + ji.b * p.qsb + (int64_t)(ji.h * p.G + g) * p.qsh + (int64_t)tok * p.qst;
}

__device__ __forceinline__ bool masked(const ScoreParams& p, int qi, int t) {
  if (t >= p.L) return true;
  if (p.W > 1) {
    int w = qi % p.W;
    return t > p.L - p.W + w;
  }
  return false;
}

// IEEE division for the rare operands the known-divisor path cannot take,
// out of line so that the hot loops that may need it stay small.
__device__ __noinline__ float div_ieee(float x, float y) { return __fdiv_rn(x, y); }

// 0 < |x| < 2^-120: operands whose quotient by sqrt(d) may be subnormal.
__device__ __forceinline__ bool tiny_nonzero(float x) {
  return (__float_as_uint(x) & 0x7fffffffu) - 1u < 0x037fffffu;
}

// sqrt(128) in fp32: the divisor of every logit (head dim 128).  For bf16
// logits, rnd(x * r) with r the correctly rounded 1 / sqrt(128) equals
// rnd(x / sqrt(128)) with the correctly rounded division, for every finite
// bf16 x (all 2^16 bit patterns checked, tests/test_scale_exact.py), so bf16
// models scale with one multiply.  fp16 (52 of its values round differently)
// and fp32 keep the division.
constexpr float kSqrtD = 11.313708305358887f;
template <typename T>
__device__ __forceinline__ bool scale_by_recip(float y) {
  return std::is_same<T, __nv_bfloat16>::value && y == kSqrtD;
}

// Logit in the model dtype: rnd(rnd(q.k) / sqrt(d)), the division correctly
// rounded.  16-bit models divide by the known divisor with one residual
// correction (tiny nonzero operands take IEEE division; the sign of a zero
// quotient is restored from the operand, as IEEE division keeps it), or for
// bf16 and d = 128 multiply (above); fp32 models always use IEEE division.
template <typename T>
__device__ __forceinline__ float scale_logit(float acc, float y, float r) {
  const float x = Elem<T>::rnd(acc);
  if constexpr (std::is_same<T, float>::value) {
    return __fdiv_rn(x, y);
  } else {
    if (scale_by_recip<T>(y)) return Elem<T>::rnd(x * r);
    float q = copysignf(div_known(x, y, r), x);
    if (__builtin_expect(tiny_nonzero(x), 0)) q = div_ieee(x, y);
    return Elem<T>::rnd(q);
  }
}

// The same for the two logits of a pair, with packed conversions.
template <typename T>
__device__ __forceinline__ void scale_logit2(float& a, float& b, float y, float r) {
  if constexpr (std::is_same<T, float>::value) {
    a = __fdiv_rn(a, y);
    b = __fdiv_rn(b, y);
  } else {
    Elem<T>::rnd2(a, b);
    if (scale_by_recip<T>(y)) {
      float qa = a * r, qb = b * r;
      Elem<T>::rnd2(qa, qb);
      a = qa;
      b = qb;
      return;
    }
    float qa = copysignf(div_known(a, y, r), a), qb = copysignf(div_known(b, y, r), b);
    if (__builtin_expect(tiny_nonzero(a) || tiny_nonzero(b), 0)) {
      if (tiny_nonzero(a)) qa = div_ieee(a, y);
      if (tiny_nonzero(b)) qb = div_ieee(b, y);
    }
    Elem<T>::rnd2(qa, qb);
    a = qa;
    b = qb;
  }
}

// ---------------------------------------------------------------------------
// Phase 1, tensor-core path (16-bit dtypes, Rq <= 8*NT): a warp computes the
// logits of 16 tokens x 8*NT query rows per iteration with m16n8k16 MMAs.
// A = 16 key rows (tokens), B = query rows^T.  The head dimension is read in
// a permuted order so that each thread loads 16 contiguous bytes per row; the
// query fragments use the same permutation, so the dot products are exact
// sums over all 128 dims.
//
// The B fragments (query rows) stay in registers for NT <= 2.  For more rows
// they would take 16*NT registers of the 128 a thread of the 512-thread CTA
// has and spill; they go to shared memory instead, in per-lane order
// (fragment word pair [nt][k-step][lane], so a warp's 8-byte loads are
// conflict-free), filled once per CTA.
// exp for the row sums: the same exp the probabilities use
template <typename T>
__device__ __forceinline__ float row_exp(float x) {
  if constexpr (std::is_same<T, float>::value) return expf(x);
  else return __expf(x);
}

// Softmax probability of logit x with row max M, row sum of exp S and its
// rounded reciprocal R, in fp32 (the reference's softmax(dtype=float32)).
// fp32 models use the accurate exp and an IEEE division.  16-bit models
// multiply by the reciprocal (as the CPU softmax the reference runs does) and
// round to their dtype right after, so they use the fast exp: over every
// 16-bit parity test (5.5 M scored positions) the fast and the accurate exp
// give the same rate of scores that differ from the oracle's by one rounding
// step (0.021 % and 0.021 %), and the accurate one costs 5.6 us per drift
// check at 128K (47.5 vs 53.1 us, measured).
template <typename T>
__device__ __forceinline__ float softmax_prob(float x, float M, float S, float R) {
  if constexpr (std::is_same<T, float>::value) return __fdiv_rn(expf(x - M), S);
  else return __expf(x - M) * R;
}

// Running (max, sum of exp(x - max)) of one score row over the logits a
// thread produces, two at a time: the sum is rescaled when the max grows.
template <typename T>
__device__ __forceinline__ void online_add2(float& m, float& sum, float x0, float x1) {
  const float tm = fmaxf(x0, x1);
  if (tm == -INFINITY) return;
  if (tm > m) {
    sum *= row_exp<T>(m - tm);  // 0 while m is still -inf
    m = tm;
  }
  sum += row_exp<T>(x0 - m) + row_exp<T>(x1 - m);
}
// Merge of two such pairs (m2, s2) into (m, s).
template <typename T>
__device__ __forceinline__ void online_merge(float& m, float& sum, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  sum = (m == -INFINITY ? 0.f : sum * row_exp<T>(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * row_exp<T>(m2 - mn));
  m = mn;
}

constexpr int kMaxNT = 5;
// the mma path's per-warp row sums sit in the upper part of each warp's
// kMaxRq-entry row of wmax (its rows number at most 8 * kMaxNT)
constexpr int kWarpSumOff = 128;
static_assert(kWarpSumOff >= 8 * kMaxNT && kWarpSumOff + 8 * kMaxNT <= kMaxRq, "wmax layout");

// Logits in global memory leave a warp through `stg` (kSWarps tiles of
// kStgBytes, free shared memory during phase 1): stmatrix transposes a
// tile's 16 tokens x 8*NT rows into rows of kStgRow bytes (16 bytes of padding
// keep the eight row addresses of a matrix on distinct banks), then each row
// goes out as two 16-byte stores.
constexpr int kStgRow = 48;
constexpr int kStgBytes = 8 * kMaxNT * kStgRow;

// GLOBAL: the logits buffer is global memory (else shared memory).
template <typename T, int NT, bool GLOBAL, typename Pre>
__device__ void logits_mma(const ScoreParams& p, const JobInfo& ji, T* lg, float* wmax, uint32_t* dummy,
                           uint2* s_qf, unsigned char* stg, Pre&& pre) {
  constexpr bool QS = NT > 2;  // query fragments in shared memory (s_qf: kMaxNT * 8 * 32 entries)
  static_assert(NT <= kMaxNT, "query tiles");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  uint32_t qb[QS ? 1 : NT][8][2];
  if constexpr (QS) {
    for (int i = threadIdx.x; i < NT * 8 * 32; i += kSThreads) {
      const int nt = i >> 8, ks = (i >> 5) & 7, ln = i & 31;
      const int qi = nt * 8 + (ln >> 2);
      uint2 w2 = make_uint2(0u, 0u);
      if (qi < p.Rq) w2 = ldg64(query_row<T>(p, ji, qi) + 32 * (ks >> 1) + 8 * (ln & 3) + 4 * (ks & 1));
      s_qf[i] = w2;
    }
  } else {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      int qi = nt * 8 + gid;
      const T* qr = qi < p.Rq ? query_row<T>(p, ji, qi) : nullptr;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          uint2 w2 = make_uint2(0u, 0u);
          if (qr) w2 = ldg64(qr + 32 * s + 8 * tig + 4 * u);
          qb[nt][2 * s + u][0] = w2.x;
          qb[nt][2 * s + u][1] = w2.y;
        }
      }
    }
  }
  pre();  // block-wide work that overlaps the query loads
  if constexpr (QS) __syncthreads();  // the fragments are in shared memory
  // per query row: running max and, for logits in global memory, sum of exp
  // over the CTA's own tokens (saving a second pass over the logits)
  float rmax[NT][2], rsum[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    rmax[nt][0] = rmax[nt][1] = -INFINITY;
    rsum[nt][0] = rsum[nt][1] = 0.f;
  }
  const float r_sqrt = __frcp_rn(p.sqrt_d);

  const int lo = max(0, ji.t0 - kMargin);
  const int hi = min(p.L, ji.t1 + kMargin);
  const int base = ji.t0 - kMargin;  // lg column 0 <-> token base
  // Tiles whose 16 tokens all lie in [t0, t1) (no window mask, logits in
  // shared memory) store their logits transposed with stmatrix: lane 8h + j
  // addresses query row nt*8 + j at the tile's token 8h.  Rows past Rq go to
  // a scratch word.  Column offsets are multiples of 16 tokens (t0 is a
  // multiple of 32, lo = t0 - 16 or 0) and TB a multiple of 8, so every row
  // address is 16-byte aligned.
  const bool fast_ok = !GLOBAL && p.W == 1;
  // global logits: staged stores (W == 1: no in-window mask)
  const bool stage_ok = GLOBAL && p.W == 1 && stg != nullptr;
  unsigned char* my_stg = stg ? stg + warp * kStgBytes : nullptr;
  const uint32_t stg_row = stg ? smem_u32(my_stg) + (uint32_t)((lane & 7) * kStgRow + 16 * ((lane >> 3) & 1)) : 0u;
  uint32_t st_row[NT];
  unsigned int st_valid = 0u;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int qi = nt * 8 + (lane & 7);
    st_row[nt] = smem_u32(lg) + 2u * (uint32_t)(qi * p.TB - base + 8 * ((lane >> 3) & 1));
    if (qi < p.Rq) st_valid |= 1u << nt;
  }
  const uint32_t st_dummy = smem_u32(dummy);
  const uint64_t pol = l2_evict_first_policy();  // the keys are read once
  // Two key tiles in flight per warp: each iteration first issues the loads
  // of the warp's next tile, then computes on the current one.
  constexpr int kStep = kSWarps * 16;
  auto load_tile = [&](int t, uint4 (&a)[4], uint4 (&b)[4]) {
    const T* ra = key_row<T>(p, ji, min(t + gid, p.L - 1));
    const T* rb = key_row<T>(p, ji, min(t + gid + 8, p.L - 1));
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      a[s] = ld_stream128(ra + 32 * s + 8 * tig, pol);
      b[s] = ld_stream128(rb + 32 * s + 8 * tig, pol);
    }
  };
  uint4 na[4], nb[4];
  if (lo + warp * 16 < hi) load_tile(lo + warp * 16, na, nb);
  for (int tg = lo + warp * 16; tg < hi; tg += kStep) {
    uint4 ka[4], kb[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      ka[s] = na[s];
      kb[s] = nb[s];
    }
    if (tg + kStep < hi) load_tile(tg + kStep, na, nb);
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        uint2 b0, b1;
        if constexpr (QS) {
          b0 = s_qf[((nt * 8 + 2 * s) << 5) + lane];
          b1 = s_qf[((nt * 8 + 2 * s + 1) << 5) + lane];
        } else {
          b0 = make_uint2(qb[nt][2 * s][0], qb[nt][2 * s][1]);
          b1 = make_uint2(qb[nt][2 * s + 1][0], qb[nt][2 * s + 1][1]);
        }
        mma16816<T>(acc[nt], ka[s].x, kb[s].x, ka[s].y, kb[s].y, b0.x, b0.y);
        mma16816<T>(acc[nt], ka[s].z, kb[s].z, ka[s].w, kb[s].w, b1.x, b1.y);
      }
    }
    if (!GLOBAL && fast_ok && tg >= ji.t0 && tg + 16 <= ji.t1) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        scale_logit2<T>(acc[nt][0], acc[nt][1], p.sqrt_d, r_sqrt);
        scale_logit2<T>(acc[nt][2], acc[nt][3], p.sqrt_d, r_sqrt);
        // logits in shared memory: the exp sums come from a pass over them
        rmax[nt][0] = fmaxf(rmax[nt][0], fmaxf(acc[nt][0], acc[nt][2]));
        rmax[nt][1] = fmaxf(rmax[nt][1], fmaxf(acc[nt][1], acc[nt][3]));
        const uint32_t a = ((st_valid >> nt) & 1u) ? st_row[nt] + 2u * (uint32_t)tg : st_dummy;
        stmatrix2_trans(a, Elem<T>::pack2(acc[nt][0], acc[nt][1]), Elem<T>::pack2(acc[nt][2], acc[nt][3]));
      }
      continue;
    }
    if (GLOBAL && stage_ok && tg + 16 <= hi) {
      // tiles are wholly own tokens or wholly margin (t0, t1 and lo are
      // multiples of 16 apart)
      const bool own_tile = tg >= ji.t0 && tg + 16 <= ji.t1;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        scale_logit2<T>(acc[nt][0], acc[nt][1], p.sqrt_d, r_sqrt);
        scale_logit2<T>(acc[nt][2], acc[nt][3], p.sqrt_d, r_sqrt);
        if (own_tile) {
          online_add2<T>(rmax[nt][0], rsum[nt][0], acc[nt][0], acc[nt][2]);
          online_add2<T>(rmax[nt][1], rsum[nt][1], acc[nt][1], acc[nt][3]);
        }
        stmatrix2_trans(stg_row + (uint32_t)(nt * 8 * kStgRow), Elem<T>::pack2(acc[nt][0], acc[nt][1]),
                        Elem<T>::pack2(acc[nt][2], acc[nt][3]));
      }
      __syncwarp();
      T* dst = lg + (tg - base);
#pragma unroll
      for (int i0 = 0; i0 < NT * 16; i0 += 32) {
        const int i = i0 + lane;
        const int row = i >> 1, half = i & 1;
        if (i < NT * 16 && row < p.Rq)
          *reinterpret_cast<uint4*>(dst + (int64_t)row * p.TB + 8 * half) =
              *reinterpret_cast<const uint4*>(my_stg + row * kStgRow + 16 * half);
      }
      __syncwarp();
      continue;
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      scale_logit2<T>(acc[nt][0], acc[nt][1], p.sqrt_d, r_sqrt);
      scale_logit2<T>(acc[nt][2], acc[nt][3], p.sqrt_d, r_sqrt);
      float own[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = nt * 8 + 2 * tig + (e & 1);
        const int t = tg + gid + ((e >> 1) << 3);
        own[e] = -INFINITY;
        if (qi >= p.Rq || t >= hi) continue;
        float x = acc[nt][e];
        if (masked(p, qi, t)) x = -INFINITY;
        lg[(int64_t)qi * p.TB + (t - base)] = Elem<T>::pack(x);
        if (t >= ji.t0 && t < ji.t1) own[e] = x;
      }
      if constexpr (GLOBAL) {
        online_add2<T>(rmax[nt][0], rsum[nt][0], own[0], own[2]);
        online_add2<T>(rmax[nt][1], rsum[nt][1], own[1], own[3]);
      } else {
        rmax[nt][0] = fmaxf(rmax[nt][0], fmaxf(own[0], own[2]));
        rmax[nt][1] = fmaxf(rmax[nt][1], fmaxf(own[1], own[3]));
      }
    }
  }
  // merge the running pairs over the 8 lanes sharing tig, then publish:
  // wmax[warp][qi] the warp's row max, wmax[warp][kWarpSumOff + qi] its sum
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float m = rmax[nt][c], sm = rsum[nt][c];
      if constexpr (GLOBAL) {
#pragma unroll
        for (int o = 4; o <= 16; o <<= 1)
          online_merge<T>(m, sm, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, sm, o));
      } else {
#pragma unroll
        for (int o = 4; o <= 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      }
      const int qi = nt * 8 + 2 * tig + c;
      if (gid == 0 && qi < p.Rq) {
        wmax[warp * kMaxRq + qi] = m;
        wmax[warp * kMaxRq + kWarpSumOff + qi] = sm;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Phase 1 and the window sums, tcgen05 path (16-bit dtypes, launches of more
// than 40 query rows: observation windows).  The CTA's keys stream through
// shared memory twice, in tiles of 128 tokens loaded by TMA, and the tensor
// core recomputes the logits on each pass (K = 128 dims in eight 16-deep
// steps) into one of two tensor-memory accumulators; no logit is stored:
//
//  * PASS_STATS: D[query row, token] = Q . K_tile^T (M = 128 query rows per
//    row block, N = 128 tokens).  A thread reads one query row's logits of 32
//    tokens per load (its TMEM lane is the row), rounds and scales them as
//    the other paths do, and keeps that row's running (max, sum of exp) over
//    the CTA's own tokens; the warps of a lane quarter split the token
//    columns, and after the pass their pairs are merged in warp order into
//    the CTA's softmax partials (p.part).  Margin tiles are not loaded.
//  * PASS_SUMS, after the grid-wide softmax statistics: D[token, query row]
//    = K_tile . Q^T (M = 128 tokens, N = NP query rows).  A thread holds one
//    token's logits of every row of a score row's window, turns them into
//    probabilities rounded to the dtype, adds them in window order (w = 0 ..
//    W-1, fp32) and stores the rounded window sum -- the probability itself
//    when W = 1 -- into row sg of the compact buffer lg [S * G][TB], for the
//    CTA's tokens and the pooling margins either side (16-row tiles; rows
//    16..127 of such a tile are left over from earlier tiles and discarded).
//
// The CTA's token range [t0, t1) is a multiple of 128 tokens from a
// 128-aligned t0 (a tile never crosses a 256-token page).
//
// All 16 warps read the accumulators, four per TMEM lane quarter (a warp may
// only read lanes 32 * (warp % 4) .. + 31), so every quarter's share of a
// tile is split four ways.  There are no producer or MMA warps: at the start
// of tile i (its MMAs seen complete) lane 0 of warp i % 16 refills tile i's
// stage with tile i + NS, and lane 0 of warp (i + 8) % 16 issues the MMAs of
// tile i + D into the accumulator that tile i + D - NB used, once every warp
// has released it; with NB = 4 accumulators (where the tensor memory holds
// them) D = 2, so the MMAs run two tiles ahead of the readers and wait for a
// release two tiles old; with 2, D = 1.  Every wait is bounded; a wait that gives up
// marks the launch failed (HC_ERR_TIMEOUT) and the warps stop, copies and
// MMAs still in flight are waited for (bounded) and the tensor memory is
// released before the pass ends; after a failed statistics pass the sums
// pass does nothing.  Each pass initialises its own mbarriers (the previous
// pass's copies, MMAs and arrivals have all completed).
constexpr int kUStage = 2 * 128 * 128;  // bytes of one stage: two 128-row x 128-byte boxes
constexpr int kMaxStages = 6;
constexpr int kUBox = 128 * 128;

constexpr int kUAcc = 4;  // tensor-memory accumulators at most

struct UmmaSmem {
  uint64_t full[kMaxStages], accf[kUAcc], acce[kUAcc];
  uint32_t tmem;
  int issued, consumed, mma_last, fail;
  int pages[kMaxPages];  // drift checks: page ids of the CTA's keys
};

enum { PASS_STATS = 0, PASS_SUMS = 1 };

// Rows of the query operand in shared memory: NP for the sums pass's B
// operand, whole 128-row blocks for the statistics pass's A operand.
__host__ __device__ constexpr int umma_query_rows(int Rq) { return (Rq + 127) / 128 * 128; }

// Eight logits: x holds q.k dot products (fp32) and receives rnd(rnd(x) /
// sqrt(d)) as scale_logit does (bf16 and d = 128: one multiply each), else
// branch-free except for one vote-free fix-up branch taken when any operand
// is 0 or tiny (the fast division does not keep the sign of a zero; a
// subnormal quotient needs IEEE division).
template <typename T>
__device__ __forceinline__ void scale_logit8(float* x, float y, float r) {
#pragma unroll
  for (int j = 0; j < 8; j += 2) Elem<T>::rnd2(x[j], x[j + 1]);
  if (scale_by_recip<T>(y)) {
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      float a = x[j] * r, b = x[j + 1] * r;
      Elem<T>::rnd2(a, b);
      x[j] = a;
      x[j + 1] = b;
    }
    return;
  }
  float q[8];
  bool fix = false;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    q[j] = div_known(x[j], y, r);
    fix |= (__float_as_uint(x[j]) & 0x7fffffffu) < 0x03800000u;  // |x| < 2^-120, zeros included
  }
  if (__builtin_expect(fix, 0)) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t a = __float_as_uint(x[j]) & 0x7fffffffu;
      if (a == 0u) q[j] = x[j];
      else if (a < 0x03800000u) q[j] = div_ieee(x[j], y);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    Elem<T>::rnd2(q[j], q[j + 1]);
    x[j] = q[j];
    x[j + 1] = q[j + 1];
  }
}

// One pass (see above).  wpart: PASS_STATS's per-warp row pairs [4][kMaxRq]
// (memory of the later phases, free here).  s_rowM / s_rowS / s_rowR:
// PASS_SUMS's global row statistics.
template <typename T, int MODE, int PASS>
__device__ void umma_pass(const ScoreParams& p, const JobInfo& ji, T* lg, unsigned char* stages,
                          unsigned char* qop, UmmaSmem& u, const CUtensorMap* tm_rows, const CUtensorMap* tm_edge,
                          float2* wpart, const float* s_rowM, const float* s_rowS, const float* s_rowR) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int NS = p.n_stages, NP = p.NP, Rq = p.Rq;
  const int QR = umma_query_rows(Rq);
  const int nrb = QR >> 7;  // 128-row blocks of query rows
  const int lo = max(0, ji.t0 - kMargin), hi = min(p.L, ji.t1 + kMargin);
  constexpr bool kMargins = PASS == PASS_SUMS;
  const bool left = kMargins && ji.t0 > 0, right = kMargins && ji.t1 < p.L;
  const int nmain = (ji.t1 - ji.t0 + 127) >> 7;
  const int ntiles = (left ? 1 : 0) + nmain + (right ? 1 : 0);
  auto tile_of = [&](int i, int& start, int& rows) {
    if (left) {
      if (i == 0) { start = ji.t0 - kMargin; rows = kMargin; return; }
      --i;
    }
    if (i < nmain) { start = ji.t0 + 128 * i; rows = 128; return; }
    start = ji.t1;
    rows = kMargin;
  };
  // accumulators: NB buffers of 128 columns per row block (statistics) or of
  // NP columns (sums), as many as the 512 columns hold up to kUAcc and no
  // more than the stages (so that an MMA's keys were requested a tile ago)
  const int acc_cols = PASS == PASS_STATS ? QR : NP;
  const int NB = min(min(kUAcc, 512 / acc_cols), NS);
  uint32_t ncols = 32;
  while (ncols < (uint32_t)(NB * acc_cols)) ncols <<= 1;
  // ---- set-up: this pass's barriers
  if (threadIdx.x == 0) {
    if (PASS == PASS_SUMS) {
      // retire the statistics pass's barriers (its accumulator count)
      const int nb_a = min(min(kUAcc, 512 / QR), NS);
      for (int s = 0; s < NS; ++s) mbar_inval(&u.full[s]);
      for (int b = 0; b < nb_a; ++b) {
        mbar_inval(&u.accf[b]);
        mbar_inval(&u.acce[b]);
      }
    }
    for (int s = 0; s < NS; ++s) mbar_init(&u.full[s], 1);
    for (int b = 0; b < NB; ++b) {
      mbar_init(&u.accf[b], 1);
      mbar_init(&u.acce[b], kSWarps);
    }
    if (PASS == PASS_STATS) u.fail = 0;
    u.issued = u.consumed = 0;
    u.mma_last = -1;
    fence_mbar_init();
  }
  // the ring held the statistics pass's row pairs (generic stores) before the
  // copies of this pass write it
  if (PASS == PASS_SUMS) fence_proxy_async_smem();
  __syncthreads();
  if (PASS == PASS_SUMS && u.fail) return;  // the statistics pass gave up (block-uniform)

  // drift checks: the page ids of the CTA's keys, loaded by warp 0 at once
  // (kMaxPages of them; beyond that each tile reads its own)
  int npg = 0, pg0 = 0;
  if constexpr (MODE == MODE_DRIFT) {
    pg0 = lo >> 8;
    npg = ((hi - 1) >> 8) - pg0 + 1;
    if (npg <= kMaxPages) {
      if (warp == 0) {
        const int row = ji.b * p.KV + ji.h;
        for (int j = lane; j < npg; j += 32) {
          int blk = p.bt[(int64_t)row * p.max_blocks + pg0 + j];
          if (blk < 0 || blk >= p.n_blocks) {
            set_err(p.err, HC_ERR_RANGE);
            blk = 0;  // keep the copy inside the pool (the launch reports the error)
          }
          u.pages[j] = blk;
        }
        __syncwarp();
      }
    } else {
      npg = 0;
    }
  }
  // thread 0: TMA copies of tile i into its stage
  auto load_tile = [&](int i) {
    const int s = i % NS;
    int start, rows;
    tile_of(i, start, rows);
    const CUtensorMap* m = rows == 128 ? tm_rows : tm_edge;
    unsigned char* dst = stages + (size_t)s * kUStage;
    const uint64_t pol = l2_evict_first_policy();
    mbar_arrive_expect_tx(&u.full[s], (uint32_t)rows * 256u);
    if constexpr (MODE == MODE_DRIFT) {
      int blk;
      if (npg) {
        blk = u.pages[min((start >> 8) - pg0, npg - 1)];
      } else {
        blk = p.bt[(int64_t)(ji.b * p.KV + ji.h) * p.max_blocks + (start >> 8)];
        if (blk < 0 || blk >= p.n_blocks) {  // reported; read page 0 instead
          set_err(p.err, HC_ERR_RANGE);
          blk = 0;
        }
      }
      const int y = blk * kPage + (start & (kPage - 1));
      tma_load_2d(dst, m, 0, y, &u.full[s], pol);
      tma_load_2d(dst + kUBox, m, 64, y, &u.full[s], pol);
    } else {
      tma_load_4d(dst, m, 0, start, ji.h, ji.b, &u.full[s], pol);
      tma_load_4d(dst + kUBox, m, 64, start, ji.h, ji.b, &u.full[s], pol);
    }
    u.issued = i + 1;
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < min(ntiles, NS); ++i) load_tile(i);
  // tensor memory and (first pass) the query operand, while the first tiles load
  if (warp == 1) {
    tmem_alloc(&u.tmem, ncols);
    if (PASS == PASS_SUMS) tmem_relinquish();  // the CTA's last allocation
  }
  if (PASS == PASS_STATS) {
    // query rows: QR rows x 128 dims, K-major, 128-byte swizzle, rows past
    // Rq zero; the two 64-dim halves QR * 128 bytes apart
    for (int i = threadIdx.x; i < QR * 16; i += kSThreads) {
      const int r = i >> 4, c16 = i & 15;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < Rq) v = ldg128(query_row<T>(p, ji, r) + 8 * c16);
      *reinterpret_cast<uint4*>(qop + (c16 >> 3) * (QR * 128) + swz128(r, c16 & 7)) = v;
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = u.tmem;
  // thread 0: the MMAs of tile i into its accumulator, once its keys are in
  const uint32_t idesc =
      idesc_f16_m128(std::is_same<T, __nv_bfloat16>::value, PASS == PASS_STATS ? 128 : NP);
  auto issue_mma = [&](int i) {
    const int s = i % NS, b = i % NB;
    if (!mbar_wait(&u.full[s], (i / NS) & 1, p.wait_ns)) {
      atomicExch(&u.fail, 1);
      return;
    }
    u.consumed = i + 1;
    tc_fence_after();
    const uint32_t q0 = smem_u32(qop);
    const uint32_t k0 = smem_u32(stages + (size_t)s * kUStage);
    const uint32_t d = tmem + (uint32_t)(b * acc_cols);
    if (PASS == PASS_STATS) {
      for (int rb = 0; rb < nrb; ++rb) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t ao = q0 + (kk >> 2) * (QR * 128) + rb * (128 * 128) + (kk & 3) * 32;
          const uint32_t bo = k0 + (kk >> 2) * kUBox + (kk & 3) * 32;
          umma_f16(d + (uint32_t)(rb * 128), smem_desc_sw128(ao), smem_desc_sw128(bo), idesc, kk > 0 ? 1u : 0u);
        }
      }
    } else {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t ao = k0 + (kk >> 2) * kUBox + (kk & 3) * 32;
        const uint32_t bo = q0 + (kk >> 2) * (QR * 128) + (kk & 3) * 32;
        umma_f16(d, smem_desc_sw128(ao), smem_desc_sw128(bo), idesc, kk > 0 ? 1u : 0u);
      }
    }
    umma_commit(&u.accf[b]);
    u.mma_last = i;
  };
  // MMAs run D tiles ahead of the tile being read: the first D now
  const int D = max(1, NB - 2);
  if (threadIdx.x == 0)
    for (int i = 0; i < min(ntiles, D) && !u.fail; ++i) issue_mma(i);

  // ---- every warp: read the accumulators tile by tile
  const int q4 = warp & 3, k = warp >> 2;  // lane quarter, index among its four warps
  const uint32_t lane_off = (uint32_t)(32 * q4) << 16;
  // launch constants in registers (the loops store through pointers the
  // compiler cannot separate from the parameter block)
  const int W = p.W, L = p.L, TB = p.TB, t1 = ji.t1;
  const float sqd = p.sqrt_d, r_sqrt = __frcp_rn(sqd);
  float rm[2] = {-INFINITY, -INFINITY}, rs[2] = {0.f, 0.f};  // statistics: (max, sum) per row block
  for (int i = 0; i < ntiles; ++i) {
    const int b = i % NB;
    int start, rows;
    tile_of(i, start, rows);
    const bool ok = mbar_wait_sleep(&u.accf[b], (i / NB) & 1, p.wait_ns);
    if (!ok) atomicExch(&u.fail, 1);
    tc_fence_after();
    // the duties of tile i rotate over the warps (issuing a tile's copies or
    // MMAs takes a fraction of a microsecond of one thread, which would
    // otherwise hold back one warp on every tile):
    if (ok && lane == 0) {
      // warp i % 16: tile i's MMAs have read its stage, refill it with tile
      // i + NS
      if (warp == (i & (kSWarps - 1)) && i + NS < ntiles) load_tile(i + NS);
      // warp (i + 8) % 16: the MMAs of tile i + D into the accumulator tile
      // i + D - NB used, once every warp has released it (D tiles ahead, so
      // that the wait is for a tile the slowest warp finished a while ago)
      const int j = i + D;
      if (warp == ((i + kSWarps / 2) & (kSWarps - 1)) && j < ntiles) {
        const int r = j - NB;
        if (r >= 0 && !mbar_wait(&u.acce[r % NB], (r / NB) & 1, p.wait_ns)) {
          atomicExch(&u.fail, 1);
        } else {
          tc_fence_after();
          issue_mma(j);
        }
      }
    }
    if (ok && PASS == PASS_STATS) {
      // work items (row block, 32-token chunk), dealt over the quarter's warps
      for (int it = k; it < 4 * nrb; it += 4) {
        const int rb = it >> 2, kc = it & 3;
        if (rb * 128 + 32 * q4 >= Rq) continue;  // no row on this warp's lanes (warp-uniform)
        const int qi = rb * 128 + 32 * q4 + lane;
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + (uint32_t)(b * acc_cols + rb * 128 + 32 * kc), v);
        tmem_ld_wait();
        float x[4][8];
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j >> 3][j & 7] = __uint_as_float(v[j]);
#pragma unroll
        for (int c = 0; c < 4; ++c) scale_logit8<T>(x[c], sqd, r_sqrt);
        // tokens counted: the CTA's own (t < t1) that the row may see (in an
        // observation window row qi = sg * W + w sees t <= L - W + w)
        const int tk = start + 32 * kc;
        const int lim = W > 1 ? min(t1, L - W + qi % W + 1) : t1;
        if (tk + 32 > lim) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (tk + j >= lim) x[j >> 3][j & 7] = -INFINITY;
        }
        // the chunk's max as a tree (short dependency chains)
        float m8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) m8[j] = fmaxf(fmaxf(x[0][j], x[1][j]), fmaxf(x[2][j], x[3][j]));
#pragma unroll
        for (int j = 0; j < 4; ++j) m8[j] = fmaxf(m8[j], m8[j + 4]);
        const float cm = fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3]));
        if (cm != -INFINITY) {
          float& M = rm[rb];
          float& S = rs[rb];
          if (cm > M) {
            S *= exp2_approx((M - cm) * kLog2e);  // 0 while M is still -inf
            M = cm;
          }
          // exp(x - M) as 2^(x log2 e - M log2 e), one multiply-add each
          const float nm = -M * kLog2e;
          float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int j = 0; j < 32; ++j) s4[j & 3] += exp2_approx(fmaf(x[j >> 3][j & 7], kLog2e, nm));
          S += (s4[0] + s4[1]) + (s4[2] + s4[3]);
        }
      }
    } else if (ok) {
      // sums: thread = token; the quarter's warps take score rows sg = k,
      // k + 4, ... (window columns sg * W .. + W - 1)
      const int r = 32 * q4 + lane;
      const int t = start + r;
      const bool valid = r < rows && t >= lo && t < hi;
      const int nsg = Rq / W;
      const int base = ji.t0 - kMargin;
      // per-column checks only where a chunk straddles a window's edge (W not
      // a multiple of 8) or a token of the tile is masked for some row
      // (t > L - W); tile-uniform
      const bool checked = (W & 7) != 0 || (W > 1 && start + rows - 1 > L - W);
      for (int sg = k; sg < nsg; sg += 4) {
        const int c0 = sg * W, c1 = c0 + W;
        float acc = 0.f;
        for (int cb = c0 & ~7; cb < c1; cb += 32) {
          // 32 columns in one load where they lie in the window, else up to
          // four 8-column loads; one wait
          const int nl = min(4, (c1 - cb + 7) >> 3);
          uint32_t v[4][8];
          if (nl == 4 && cb >= c0) {
            tmem_ld32(tmem + lane_off + (uint32_t)(b * acc_cols + cb), &v[0][0]);
          } else {
#pragma unroll
            for (int c = 0; c < 4; ++c)
              if (c < nl) tmem_ld8(tmem + lane_off + (uint32_t)(b * acc_cols + cb + 8 * c), v[c]);
          }
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              if (c >= nl) break;
              float x[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) x[j] = __uint_as_float(v[c][j]);
              scale_logit8<T>(x, sqd, r_sqrt);
              const int q8 = cb + 8 * c;  // first query row of the chunk (8-aligned)
              const float4 Ma = *reinterpret_cast<const float4*>(s_rowM + q8);
              const float4 Mb = *reinterpret_cast<const float4*>(s_rowM + q8 + 4);
              const float4 Ra = *reinterpret_cast<const float4*>(s_rowR + q8);
              const float4 Rb = *reinterpret_cast<const float4*>(s_rowR + q8 + 4);
              const float Mv[8] = {Ma.x, Ma.y, Ma.z, Ma.w, Mb.x, Mb.y, Mb.z, Mb.w};
              const float Rv[8] = {Ra.x, Ra.y, Ra.z, Ra.w, Rb.x, Rb.y, Rb.z, Rb.w};
              float pr[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) pr[j] = softmax_prob<T>(x[j], Mv[j], s_rowS[q8 + j], Rv[j]);
              if (checked) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int qi = q8 + j;
                  // outside this window, or masked: no contribution
                  if (qi < c0 || qi >= c1 || (W > 1 && t > L - W + (qi - c0))) pr[j] = 0.f;
                }
              }
#pragma unroll
              for (int j = 0; j < 8; j += 2) Elem<T>::rnd2(pr[j], pr[j + 1]);
#pragma unroll
              for (int j = 0; j < 8; ++j) acc += pr[j];
            }
          }
        }
        if (valid) lg[(int64_t)sg * TB + (t - base)] = Elem<T>::from_f(acc);
      }
    }
    // release the accumulator
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&u.acce[b]);
    if (!ok) break;
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && u.fail) {
    set_err(p.err, HC_ERR_TIMEOUT);
    // copies still in flight land before the stages can be reused, and the
    // last MMAs issued into each accumulator complete before it is released
    for (int i = u.consumed; i < u.issued; ++i) (void)mbar_wait_sleep(&u.full[i % NS], (i / NS) & 1, p.wait_ns);
    for (int i = max(0, u.mma_last - NB + 1); i <= u.mma_last; ++i)
      (void)mbar_wait_sleep(&u.accf[i % NB], (i / NB) & 1, p.wait_ns);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
  if (PASS == PASS_STATS) {
    // the ring is idle: each warp's row pairs, then per row the merge of its
    // quarter's four warps in warp order into the CTA's partial
    for (int rb = 0; rb < nrb; ++rb) {
      const int qi = rb * 128 + 32 * q4 + lane;
      if (qi < Rq) wpart[k * kMaxRq + qi] = make_float2(rm[rb], rs[rb]);
    }
    __syncthreads();
    for (int qi = threadIdx.x; qi < Rq; qi += kSThreads) {
      float M = -INFINITY, S = 0.f;
#pragma unroll
      for (int kw = 0; kw < 4; ++kw) {
        const float2 v = wpart[kw * kMaxRq + qi];
        online_merge<T>(M, S, v.x, v.y);
      }
      p.part[((size_t)ji.job * p.Rq + qi) * p.cpj + ji.part] = make_float2(M, S);
    }
  }
}

// Phase 1, CUDA-core path (fp32, or many query rows): 32-token tiles of keys
// staged in shared memory (rows padded to 129 floats), lanes over tokens.
template <typename T>
__device__ void logits_fma(const ScoreParams& p, const JobInfo& ji, T* lg, float* wmax, float* sq, float* sk) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < p.Rq * kD; i += kSThreads) {
    int qi = i / kD, d = i % kD;
    sq[i] = Elem<T>::to_f(query_row<T>(p, ji, qi)[d]);
  }
  float rmax[kMaxRq / kSWarps];
  for (int i = 0; i < kMaxRq / kSWarps; ++i) rmax[i] = -INFINITY;
  const float r_sqrt = __frcp_rn(p.sqrt_d);
  const int lo = max(0, ji.t0 - kMargin);
  const int hi = min(p.L, ji.t1 + kMargin);
  const int base = ji.t0 - kMargin;
  for (int tt = lo; tt < hi; tt += 32) {
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * kD; i += kSThreads) {
      int r = i / kD, d = i % kD;
      int t = min(tt + r, p.L - 1);
      sk[r * (kD + 1) + d] = Elem<T>::to_f(key_row<T>(p, ji, t)[d]);
    }
    __syncthreads();
    const int t = tt + lane;
    int slot = 0;
    for (int qi = warp; qi < p.Rq; qi += kSWarps, ++slot) {
      const float* qr = sq + qi * kD;
      const float* kr = sk + lane * (kD + 1);
      float acc = 0.f;
#pragma unroll 8
      for (int d = 0; d < kD; ++d) acc = fmaf(qr[d], kr[d], acc);
      if (t < hi) {
        float x = scale_logit<T>(acc, p.sqrt_d, r_sqrt);
        if (masked(p, qi, t)) x = -INFINITY;
        lg[(int64_t)qi * p.TB + (t - base)] = Elem<T>::pack(x);
        if (t >= ji.t0 && t < ji.t1) rmax[slot] = fmaxf(rmax[slot], x);
      }
    }
  }
  int slot = 0;
  for (int qi = warp; qi < p.Rq; qi += kSWarps, ++slot) {
    float m = rmax[slot];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) {
      for (int w = 0; w < kSWarps; ++w) wmax[w * kMaxRq + qi] = (w == warp) ? m : -INFINITY;
    }
  }
}

// Eight consecutive elements (16-byte aligned for 16-bit types, 32-byte for
// fp32) as fp32.
template <typename T>
__device__ __forceinline__ void ld8(const T* src, float* v) {
  if constexpr (std::is_same<T, float>::value) {
    const float4 a = reinterpret_cast<const float4*>(src)[0];
    const float4 b = reinterpret_cast<const float4*>(src)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 w = *reinterpret_cast<const uint4*>(src);
    float2 f;
    f = unpack2<T>(w.x); v[0] = f.x; v[1] = f.y;
    f = unpack2<T>(w.y); v[2] = f.x; v[3] = f.y;
    f = unpack2<T>(w.z); v[4] = f.x; v[5] = f.y;
    f = unpack2<T>(w.w); v[6] = f.x; v[7] = f.y;
  }
}

// Add one to bin `tag` of the shared histogram for every lane whose `valid`
// is set.  Plain shared-memory atomics: combining lanes with equal tags into
// one atomic first (a warp match) was slower (an 8-check drift batch at 128K:
// 173 against 169 us, measured).
__device__ __forceinline__ void hist_add_warp(unsigned int* h, bool valid, unsigned int tag) {
  if (valid) atomicAdd(&h[tag], 1u);
}

// Phase 2, pooled scores.  A group of GP lanes (GP = G rounded up to a power
// of two) takes 8 consecutive tokens of one score row, one query head of the
// GQA group per lane: the lane reads the 8 tokens and their neighbours (24
// elements, three 16-byte loads), turns them into rounded probabilities
// (INLINE: from the logits with the row's max, sum and reciprocal; else they
// already are), pools them in the reference's order ((((p0+p1)+p2)+p3)+p4,
// divided by the kernel size, count_include_pad; or max), and the group
// takes the max over its lanes with butterfly shuffles.  Each lane then
// keys 8/GP of the tokens into shared memory and into the round-0 radix
// histogram of their score row.
template <typename T, int HALO, bool INLINE>
__device__ void pooled_keys8(const ScoreParams& p, const JobInfo& ji, const T* lg, unsigned int* keys,
                             unsigned int* lhist, const float* s_rowM, const float* s_rowS, const float* s_rowR) {
  constexpr int KB = Elem<T>::kKeyBits;
  constexpr float KS = (float)(2 * HALO + 1);
  const int base = ji.t0 - kMargin;
  const int ntok = ji.t1 - ji.t0;
  const int nchunk = (ntok + 7) >> 3;
  const int lgp = p.G <= 1 ? 0 : p.G <= 2 ? 1 : p.G <= 4 ? 2 : 3;
  const int GP = 1 << lgp;
  const int items = p.S * nchunk * GP;
  const bool avg = p.pooling == HC_AVGPOOL;
  const float pad = avg ? 0.f : -INFINITY;
  const float rKS = __frcp_rn(KS);
  // ci / nchunk as a multiply-high, exact while ci * nchunk < 2^32 (ci <
  // S * nchunk); a slice of one chunk (multiplier 2^32) or a very long slice
  // divides plainly
  const bool by_magic = nchunk > 1 && (unsigned long long)p.S * nchunk * nchunk < (1ull << 32);
  const unsigned int magic = by_magic ? 0xffffffffu / (unsigned int)nchunk + 1u : 0u;
  for (int i0 = 0; i0 < items; i0 += kSThreads) {
    const int it = i0 + threadIdx.x;
    const bool on = it < items;
    const int gl = it & (GP - 1);
    const int ci = on ? it >> lgp : 0;
    const int s = by_magic ? (int)__umulhi((unsigned int)ci, magic) : ci / nchunk;
    const int c = ji.t0 + 8 * (ci - s * nchunk);
    float best[8];
#pragma unroll
    for (int o = 0; o < 8; ++o) best[o] = -INFINITY;
    if (on && gl < p.G) {
      const int qi = (s * p.G + gl) * p.W;
      const T* src = lg + (int64_t)qi * p.TB + (c - base);
      float w[24];
      ld8<T>(src - 8, w);
      ld8<T>(src, w + 8);
      ld8<T>(src + 8, w + 16);
      if (INLINE) {
        const float M = s_rowM[qi], S = s_rowS[qi], R = s_rowR[qi];
#pragma unroll
        for (int i = 8 - HALO; i < 16 + HALO; ++i)
          w[i] = (w[i] == -INFINITY) ? 0.f : softmax_prob<T>(w[i], M, S, R);
        // rounded to the dtype in pairs (one packed conversion each)
#pragma unroll
        for (int i = 8 - HALO; i < 16 + HALO; i += 2) {
          if (i + 1 < 16 + HALO) Elem<T>::rnd2(w[i], w[i + 1]);
          else w[i] = Elem<T>::rnd(w[i]);
        }
      }
      if (c - HALO < 0 || c + 8 + HALO > p.Lsel) {
#pragma unroll
        for (int i = 8 - HALO; i < 16 + HALO; ++i) {
          const int t = c - 8 + i;
          if (t < 0 || t >= p.Lsel) w[i] = pad;
        }
      }
#pragma unroll
      for (int o = 0; o < 8; ++o) {
        float v = w[8 + o - HALO];
        if (avg) {
#pragma unroll
          for (int j = 1; j <= 2 * HALO; ++j) v += w[8 + o - HALO + j];
          if constexpr (std::is_same<T, float>::value) v = __fdiv_rn(v, KS);
          else v = div_known(v, KS, rKS);
        } else {
#pragma unroll
          for (int j = 1; j <= 2 * HALO; ++j) v = fmaxf(v, w[8 + o - HALO + j]);
        }
        best[o] = v;
      }
      if (avg) {  // pooled averages rounded to the dtype (max pooling keeps dtype values)
#pragma unroll
        for (int o = 0; o < 8; o += 2) Elem<T>::rnd2(best[o], best[o + 1]);
      }
    }
    // max over the group's lanes (groups are aligned within a warp) as a
    // reduce-scatter: in the round with lane mask m each lane keeps one half
    // of its values (the upper half if gl & m) and takes the max with its
    // partner's copy of that half; after log2(GP) rounds lane gl holds the
    // group maxima of tokens gl*8/GP .. (gl+1)*8/GP - 1 in best[0 ..)
    auto rs_round = [&](auto half, int m) {  // half: a compile-time 4, 2 or 1
      constexpr int H = decltype(half)::value;
      const bool upper = (gl & m) != 0;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const float send = upper ? best[i] : best[i + H];
        const float keep = upper ? best[i + H] : best[i];
        best[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, m));
      }
    };
    if (GP >= 2) rs_round(std::integral_constant<int, 4>{}, GP >> 1);  // GP is uniform over the warp
    if (GP >= 4) rs_round(std::integral_constant<int, 2>{}, GP >> 2);
    if (GP >= 8) rs_round(std::integral_constant<int, 1>{}, GP >> 3);
    // lane gl keys its 8/GP consecutive tokens
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j * GP >= 8) break;
      const int o = gl * (8 / GP) + j;
      const float v = best[j];
      const bool valid = on && c + o < ji.t1 && c + o < p.Lsel;
      const unsigned int key = valid ? Elem<T>::key(v) : 0u;
      if (on) {
        keys[s * p.T + (c - ji.t0) + o] = key;
        if (valid && p.out_scores)
          reinterpret_cast<T*>(p.out_scores)[(size_t)ji.job * p.out_job_stride + (size_t)s * p.L + c + o] = Elem<T>::pack(v);
      }
      hist_add_warp(lhist, valid, ((unsigned int)s << 8) | (key >> (KB - 8)));
    }
  }
}

// Phase 2, pooled scores for kernels wider than 7 (probabilities and window
// sums already in place): one thread per (score row, token).
template <typename T>
__device__ void pooled_keys_wide(const ScoreParams& p, const JobInfo& ji, const T* lg, unsigned int* keys,
                                 unsigned int* lhist) {
  constexpr int KB = Elem<T>::kKeyBits;
  const int base = ji.t0 - kMargin;
  const int ntok = ji.t1 - ji.t0;
  for (int i0 = 0; i0 < p.S * ntok; i0 += kSThreads) {
    const int i = i0 + threadIdx.x;
    const bool on = i < p.S * ntok;
    const int s = on ? i / ntok : 0, t = ji.t0 + (on ? i % ntok : 0);
    const bool valid = on && t < p.Lsel;
    unsigned int key = 0u;
    if (valid) {
      float best = -INFINITY;
      for (int g = 0; g < p.G; ++g) {
        const T* row = lg + (int64_t)((s * p.G + g) * p.W) * p.TB - base;
        float v;
        if (p.pooling == HC_AVGPOOL) {
          float acc = 0.f;
          for (int j = t - p.halo; j <= t + p.halo; ++j)
            if (j >= 0 && j < p.Lsel) acc += Elem<T>::to_f(row[j]);
          v = Elem<T>::rnd(acc / (float)p.ksize);
        } else {
          v = -INFINITY;
          for (int j = t - p.halo; j <= t + p.halo; ++j)
            if (j >= 0 && j < p.Lsel) v = fmaxf(v, Elem<T>::to_f(row[j]));
        }
        best = fmaxf(best, v);
      }
      key = Elem<T>::key(best);
      keys[s * p.T + (t - ji.t0)] = key;
      if (p.out_scores) {
        T* os = reinterpret_cast<T*>(p.out_scores);
        os[(size_t)ji.job * p.out_job_stride + (size_t)s * p.L + t] = Elem<T>::from_f(best);
      }
    }
    if (on && !valid) keys[s * p.T + (t - ji.t0)] = 0u;
    hist_add_warp(lhist, valid, ((unsigned int)s << 8) | (key >> (KB - 8)));
  }
}

// Find the 8-bit digit bin holding the rem-th largest key (rem >= 1).
// Returns the bin; `above` = number of keys in higher bins.  One warp.
__device__ __forceinline__ int find_bin(const unsigned int* h, unsigned int rem, unsigned int& above) {
  const int lane = threadIdx.x & 31;
  unsigned int c[8];
  unsigned int tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c[i] = h[lane * 8 + i];
    tot += c[i];
  }
  // inclusive suffix sum over lanes (lane 31 holds the highest bins)
  unsigned int suf = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    unsigned int y = __shfl_down_sync(0xffffffffu, suf, o);
    if (lane + o < 32) suf += y;
  }
  unsigned int above_lane = suf - tot;  // keys in lanes > lane
  int found = -1;
  unsigned int ab = 0;
  if (above_lane < rem && suf >= rem) {
    unsigned int run = above_lane;
    for (int i = 7; i >= 0; --i) {
      if (run + c[i] >= rem) {
        found = lane * 8 + i;
        ab = run;
        break;
      }
      run += c[i];
    }
  }
  unsigned int msk = __ballot_sync(0xffffffffu, found >= 0);
  int src = msk ? (__ffs(msk) - 1) : 0;
  int bin = __shfl_sync(0xffffffffu, found, src);
  above = __shfl_sync(0xffffffffu, ab, src);
  return bin;
}

// One instantiation per mode: the mode (and, outside prefill, the window of
// one query per row) are compile-time constants in a local copy of the
// parameters, so each instantiation carries only its own mode's code.
template <typename T, int MODE>
__global__ void __launch_bounds__(kSThreads, 1)
    score_select_kernel(const ScoreParams pin, const __grid_constant__ CUtensorMap tm_rows,
                        const __grid_constant__ CUtensorMap tm_edge,
                        const __grid_constant__ BatchOf<MODE> batch) {
  ScoreParams p = pin;
  p.mode = MODE;
  if constexpr (MODE != MODE_PREFILL) p.W = 1;
  if (MODE != MODE_PREFILL || p.Lsel <= 0 || p.Lsel > p.L) p.Lsel = p.L;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ __align__(16) float s_rowM[kMaxRq], s_rowInv[kMaxRq], s_rowR[kMaxRq];  // 16-byte loads (tcgen05 sums)
  __shared__ unsigned int s_prefix[kMaxSel], s_mask[kMaxSel], s_rem[kMaxSel], s_k[kMaxSel];
  __shared__ int s_sel_row[kMaxSel];
  __shared__ int2 s_wcnt[kMaxSel][kSWarps];
  __shared__ int s_base[kMaxSel], s_eqoff[kMaxSel];
  __shared__ int s_wsel[kMaxSel][kSWarps], s_weq[kMaxSel][kSWarps];
  __shared__ unsigned int s_gtc[kMaxSel];
  __shared__ unsigned int s_ov[kMaxRows];
  __shared__ uint32_t s_refw[kRefWords];
  __shared__ int s_trigger;

  constexpr int KB = Elem<T>::kKeyBits;
  constexpr int ROUNDS = KB / 8;
  __shared__ int s_pages[kMaxPages];
  __shared__ __align__(16) uint32_t s_dummy[4];  // sink of stmatrix rows past Rq
  // query fragments of the tensor-core logits for more than 16 query rows
  __shared__ uint2 s_qfrag[std::is_same<T, float>::value ? 1 : kMaxNT * 8 * 32];
  JobInfo ji = job_info(p);
  p.out_job_stride = (int64_t)p.S * p.L;
  // DRIFT, batch: the job's query buffer, pool, page table and score output
  // replace the launch-wide ones
  if constexpr (MODE == MODE_DRIFT) {
    if (batch.n > 0) {
      const DriftJob& d = batch.job[ji.job];
      p.out_scores = d.out_scores;
      p.out_job_stride = 0;
      ji.h = d.head;
      p.q = d.q;
      p.qst = d.qst;
      p.qsh = d.qsh;
      p.k_pool = d.k_pool;
      p.bt = d.bt;
      p.n_blocks = d.n_blocks;
      p.max_blocks = d.max_blocks;
    }
  }
  // DRIFT: where this job's results go -- rows of the job-indexed arrays of
  // one hc_drift_check launch, or the job's own descriptor in a batch
  // (formed where used: parameter-space and cached loads, no live registers)
  auto drift_view = [&]() {
    DriftView dv{};
    if constexpr (MODE == MODE_DRIFT) {
      if (batch.n > 0) {
        const DriftJob& d = batch.job[ji.job];
        dv.bitmap = d.bitmap;
        dv.ref_pos = d.ref_pos;
        dv.trigger = d.trigger;
        dv.retr = d.retr;
        dv.retr_cap = d.max_len;
        dv.coeffs = d.coeffs;
        dv.median = d.median;
        dv.max_len = d.max_len;
      } else {
        const int slot = p.ref_slots[ji.job];
        dv.bitmap = p.ref_bitmap + (size_t)slot * p.bitmap_words;
        dv.ref_pos = p.ref_positions + (size_t)slot * p.topk;
        dv.trigger = p.trigger + ji.job;
        dv.retr = p.retrieve_positions + (size_t)ji.job * p.max_len_cap;
        dv.retr_cap = p.max_len_cap;
        dv.coeffs = p.coeffs ? p.coeffs + (size_t)ji.job * p.S : nullptr;
        dv.median = p.median ? p.median + ji.job : nullptr;
        dv.max_len = p.max_len[ji.job];
      }
    }
    return dv;
  };
  const int nblocks = gridDim.x;
  unsigned int epoch = 0;

  // ---- shared memory carve-up.  The logits buffer: every query row's
  // logits, or on the tcgen05 path (which stores no logits) one window-summed
  // probability row per score row
  unsigned char* sp = smem;
  const int lg_rows = p.umma ? p.S * p.G : p.Rq;
  T* lg;
  if (p.logits_in_smem) {
    lg = reinterpret_cast<T*>(sp);
    sp += ((size_t)lg_rows * p.TB * sizeof(T) + 15) & ~(size_t)15;
  } else {
    lg = reinterpret_cast<T*>(p.glogits) + (size_t)blockIdx.x * lg_rows * p.TB;
  }
  // tcgen05 path: the query operand, then the ring of key stages, 1024-byte
  // aligned (the launch reserves the slack); the ring is idle between the two
  // passes and dead after the second, so the arrays of the later phases
  // (keys, histograms, row partials) share its memory
  __shared__ UmmaSmem s_umma;
  unsigned char* u_stages = nullptr;
  unsigned char* u_qop = nullptr;
  if (p.umma) {
    const uint32_t a = smem_u32(sp);
    u_qop = sp + ((1024u - (a & 1023u)) & 1023u);
    u_stages = u_qop + (size_t)umma_query_rows(p.Rq) * 256;
    sp = u_stages;
  }
  unsigned int* keys = reinterpret_cast<unsigned int*>(sp);
  sp += (size_t)p.S * p.T * sizeof(unsigned int);
  unsigned int* lhist = reinterpret_cast<unsigned int*>(sp);
  sp += (size_t)kMaxSel * 256 * sizeof(unsigned int);
  float* wmax = reinterpret_cast<float*>(sp);
  sp += (size_t)kSWarps * kMaxRq * sizeof(float);
  float* sq = reinterpret_cast<float*>(sp);  // fma path only

  // ---- phase 1 on the tensor cores comes first, so that its key stream
  // starts before any other global access of the launch (the page ids are
  // read per tile by the TMA producer)
  constexpr bool kTensor = !std::is_same<T, float>::value;
  bool used_mma = false, used_umma = false;
  if constexpr (kTensor) {
    if (p.umma) {
      // the CTA's softmax partials (max, sum of exp) per query row, into p.part
      umma_pass<T, MODE, PASS_STATS>(p, ji, lg, u_stages, u_qop, s_umma, &tm_rows, &tm_edge,
                                     reinterpret_cast<float2*>(wmax), nullptr, nullptr, nullptr);
      used_mma = used_umma = true;
    }
  }

  // ---- zero the per-launch accumulators (ordered before use by barrier 1)
  if (ji.part == 0) {
    unsigned int* hj = p.hist + (size_t)ji.job * kMaxSel * ROUNDS * 256;
    for (int i = threadIdx.x; i < kMaxSel * ROUNDS * 256; i += kSThreads) hj[i] = 0u;
    if (p.mode == MODE_DRIFT && threadIdx.x < p.S) p.overlap[ji.job * kMaxRows + threadIdx.x] = 0u;
  }
  if (p.mode == MODE_DRIFT) {
    // the reference bitmap is only rewritten after the last grid barrier
    if (threadIdx.x < kMaxRows) s_ov[threadIdx.x] = 0u;
    const uint32_t* bm = drift_view().bitmap;
    const int wbeg = ji.t0 >> 5, nwords = ((ji.t1 + 31) >> 5) - wbeg;
    if (nwords <= kRefWords)
      for (int w = threadIdx.x; w < nwords; w += kSThreads) s_refw[w] = bm[wbeg + w];
  }

  // the page ids of this CTA's keys, once (instead of one dependent load per
  // tile); the tensor-core path runs this after issuing its query loads
  auto stage_pages = [&]() {
    if (p.mode != MODE_DRIFT) return;
    const int lo = max(0, ji.t0 - kMargin), hi = min(p.L, ji.t1 + kMargin);
    const int pg0 = lo >> 8, npg = ((hi - 1) >> 8) - pg0 + 1;
    if (npg <= kMaxPages) {
      const int row = ji.b * p.KV + ji.h;
      for (int i = threadIdx.x; i < npg; i += kSThreads) {
        int blk = p.bt[(int64_t)row * p.max_blocks + pg0 + i];
        if (blk < 0 || blk >= p.n_blocks) {
          set_err(p.err, HC_ERR_RANGE);
          blk = -1;
        }
        s_pages[i] = blk;
      }
      ji.pages = s_pages;
      ji.page0 = pg0;
      ji.npages = npg;
    }
    __syncthreads();
  };

  // ---- phase 1, legacy paths: logits
  // staging of global logits: the keys' array is free until the pooling pass
  unsigned char* stg = (!p.logits_in_smem && (size_t)p.S * p.T * sizeof(unsigned int) >= (size_t)kSWarps * kStgBytes)
                           ? reinterpret_cast<unsigned char*>(keys) : nullptr;
  if constexpr (kTensor) {
    if (used_umma) {
    } else if (p.Rq <= 8) { (p.logits_in_smem ? logits_mma<T, 1, false>(p, ji, lg, wmax, s_dummy, s_qfrag, stg, stage_pages)
                       : logits_mma<T, 1, true>(p, ji, lg, wmax, s_dummy, s_qfrag, stg, stage_pages)); used_mma = true; }
    else if (p.Rq <= 16) { (p.logits_in_smem ? logits_mma<T, 2, false>(p, ji, lg, wmax, s_dummy, s_qfrag, stg, stage_pages)
                       : logits_mma<T, 2, true>(p, ji, lg, wmax, s_dummy, s_qfrag, stg, stage_pages)); used_mma = true; }
    else if (p.Rq <= 24) { (p.logits_in_smem ? logits_mma<T, 3, false>(p, ji, lg, wmax, s_dummy, s_qfrag, stg, stage_pages)
                       : logits_mma<T, 3, true>(p, ji, lg, wmax, s_dummy, s_qfrag, stg, stage_pages)); used_mma = true; }
    else if (p.Rq <= 32) { (p.logits_in_smem ? logits_mma<T, 4, false>(p, ji, lg, wmax, s_dummy, s_qfrag, stg, stage_pages)
                       : logits_mma<T, 4, true>(p, ji, lg, wmax, s_dummy, s_qfrag, stg, stage_pages)); used_mma = true; }
    else if (p.Rq <= 40) { (p.logits_in_smem ? logits_mma<T, 5, false>(p, ji, lg, wmax, s_dummy, s_qfrag, stg, stage_pages)
                       : logits_mma<T, 5, true>(p, ji, lg, wmax, s_dummy, s_qfrag, stg, stage_pages)); used_mma = true; }
  }
  if (!used_mma) {
    stage_pages();
    float* sk = sq + p.Rq * kD;
    logits_fma<T>(p, ji, lg, wmax, sq, sk);
  }
  // the logits pass also summed exp (mma.sync path, logits in global memory;
  // the tcgen05 statistics pass published the CTA's partials itself)
  const bool online_sums = used_umma || (used_mma && !p.logits_in_smem);
  __syncthreads();
  if (!used_umma) {
    for (int qi = threadIdx.x; qi < p.Rq; qi += kSThreads) {
      float m = -INFINITY;
      for (int w = 0; w < kSWarps; ++w) m = fmaxf(m, wmax[w * kMaxRq + qi]);
      s_rowM[qi] = m;
      if (online_sums) {
        // the mma.sync path brought each warp's row sum along: rescale the
        // warps' sums to the CTA's max, in warp order
        float sum = 0.f;
        for (int w = 0; w < kSWarps; ++w) {
          const float mw = wmax[w * kMaxRq + qi];
          if (mw != -INFINITY) sum += wmax[w * kMaxRq + kWarpSumOff + qi] * row_exp<T>(mw - m);
        }
        p.part[((size_t)ji.job * p.Rq + qi) * p.cpj + ji.part] = make_float2(m, sum);
      }
    }
  }
  __syncthreads();
  // partial sum of exp over own tokens (four independent accumulators): one
  // warp per row; with fewer rows than warps (prefill and pivot launches) a
  // row's tokens are split into nch chunks so that every warp has work, and
  // the chunk sums of a row are added in a fixed order (the per-warp maxima
  // in wmax were consumed above, so it holds the chunk sums)
  if (!online_sums) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int base = ji.t0 - kMargin;
    auto exp_sum = [&](int qi, float m, int tb, int te) {
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
      if (m != -INFINITY) {
        const T* row = lg + (int64_t)qi * p.TB - base;
        for (int t = tb + lane; t < te; t += 128) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int tu = t + 32 * u;
            if (tu < te) s4[u] += row_exp<T>(Elem<T>::to_f(row[tu]) - m);
          }
        }
      }
      float s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      return s;
    };
    if (p.Rq >= kSWarps) {
      for (int qi = warp; qi < p.Rq; qi += kSWarps) {
        const float m = s_rowM[qi];
        const float s = exp_sum(qi, m, ji.t0, ji.t1);
        if (lane == 0) p.part[((size_t)ji.job * p.Rq + qi) * p.cpj + ji.part] = make_float2(m, s);
      }
    } else {
      const int nch = min(4, kSWarps / p.Rq);
      const int clen = (((ji.t1 - ji.t0 + nch - 1) / nch) + 127) / 128 * 128;  // a multiple of 128
      float* csum = wmax;  // [Rq][nch]
      for (int it = warp; it < p.Rq * nch; it += kSWarps) {
        const int qi = it / nch, qc = it - qi * nch;
        const int tb = ji.t0 + qc * clen;
        const float s = exp_sum(qi, s_rowM[qi], tb, min(ji.t1, tb + clen));
        if (lane == 0) csum[it] = s;
      }
      __syncthreads();  // p.Rq is uniform over the block
      for (int qi = threadIdx.x; qi < p.Rq; qi += kSThreads) {
        float s = 0.f;
        for (int c = 0; c < nch; ++c) s += csum[qi * nch + c];
        p.part[((size_t)ji.job * p.Rq + qi) * p.cpj + ji.part] = make_float2(s_rowM[qi], s);
      }
    }
  }
  if (!grid_sync(p.gb, nblocks, epoch, p.err, p.wait_ns, p.stall)) return;

  // ---- phase 2: global softmax statistics, probabilities, pooling, keys
  {
    // two rows per warp (a half-warp each), lanes over the job's CTAs (a
    // row's partials are contiguous): each lane issues all its loads (up to
    // 16 CTAs' partials) before using them, then an online merge of the
    // (max, sum of exp) pairs
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hl = lane & 15;
    const float2* pj = p.part + (size_t)ji.job * p.Rq * p.cpj;
    for (int q0 = 2 * warp; q0 < p.Rq; q0 += 2 * kSWarps) {
      const int qi = q0 + (lane >> 4);
      const bool row_ok = qi < p.Rq;
      float M = -INFINITY, S = 0.f;
      for (int c0 = 0; c0 < p.cpj; c0 += 256) {
        float2 v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int c = c0 + hl + 16 * j;
          v[j] = (row_ok && c < p.cpj) ? __ldcg(&pj[(size_t)qi * p.cpj + c]) : make_float2(-INFINITY, 0.f);
        }
        float Mb = M;
#pragma unroll
        for (int j = 0; j < 16; ++j) Mb = fmaxf(Mb, v[j].x);
        if (Mb != -INFINITY) {
          float acc = M == -INFINITY ? 0.f : S * row_exp<T>(M - Mb);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc += v[j].x == -INFINITY ? 0.f : v[j].y * row_exp<T>(v[j].x - Mb);
          S = acc;
          M = Mb;
        }
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        const float M2 = __shfl_xor_sync(0xffffffffu, M, o);
        const float S2 = __shfl_xor_sync(0xffffffffu, S, o);
        const float Mn = fmaxf(M, M2);
        if (Mn != -INFINITY) {
          S = (M == -INFINITY ? 0.f : S * row_exp<T>(M - Mn)) + (M2 == -INFINITY ? 0.f : S2 * row_exp<T>(M2 - Mn));
          M = Mn;
        }
      }
      if (hl == 0 && row_ok) {
        s_rowM[qi] = M;
        s_rowInv[qi] = S;
        s_rowR[qi] = __frcp_rn(S);
      }
    }
  }
  __syncthreads();
  if constexpr (kTensor) {
    if (used_umma) {
      // second pass over the keys: one window-summed probability row per
      // score row in lg (row sg, so the pooling below reads it as W = 1)
      umma_pass<T, MODE, PASS_SUMS>(p, ji, lg, u_stages, u_qop, s_umma, &tm_rows, &tm_edge, nullptr, s_rowM,
                                    s_rowInv, s_rowR);
      p.W = 1;
    }
  }
  // zero the round-0 histograms (one per score row) before the pooling pass
  for (int i = threadIdx.x; i < kMaxSel * 256; i += kSThreads) lhist[i] = 0u;
  __syncthreads();
  if (!used_umma && p.W == 1 && p.halo <= 3) {
    // probabilities computed inline from the logits
    switch (p.halo) {
      case 0: pooled_keys8<T, 0, true>(p, ji, lg, keys, lhist, s_rowM, s_rowInv, s_rowR); break;
      case 1: pooled_keys8<T, 1, true>(p, ji, lg, keys, lhist, s_rowM, s_rowInv, s_rowR); break;
      case 2: pooled_keys8<T, 2, true>(p, ji, lg, keys, lhist, s_rowM, s_rowInv, s_rowR); break;
      default: pooled_keys8<T, 3, true>(p, ji, lg, keys, lhist, s_rowM, s_rowInv, s_rowR); break;
    }
  } else {
    // probabilities and window sums in place (the tcgen05 path wrote them)
    const int base = ji.t0 - kMargin;
    const int lo = max(0, ji.t0 - p.halo), hi = min(p.L, ji.t1 + p.halo);
    const int span = used_umma ? 0 : hi - lo;
    for (int i = threadIdx.x; i < p.Rq * span; i += kSThreads) {
      int qi = i / span, t = lo + i % span;
      T* cell = lg + (int64_t)qi * p.TB + (t - base);
      float x = Elem<T>::to_f(*cell);
      float pr = (x == -INFINITY) ? 0.f : softmax_prob<T>(x, s_rowM[qi], s_rowInv[qi], s_rowR[qi]);
      *cell = Elem<T>::from_f(pr);
    }
    __syncthreads();
    if (p.W > 1 && !used_umma) {
      const int nsg = p.S * p.G;
      for (int i = threadIdx.x; i < nsg * span; i += kSThreads) {
        int sg = i / span, t = lo + i % span;
        float acc = 0.f;
        for (int w = 0; w < p.W; ++w) acc += Elem<T>::to_f(lg[(int64_t)(sg * p.W + w) * p.TB + (t - base)]);
        // row (sg, w=W-1) is read last above; park the sum in a scratch row
        // that no other (sg', t') of this loop reads: row sg*W + 0 is only
        // read by the thread handling (sg, t) itself.
        lg[(int64_t)(sg * p.W) * p.TB + (t - base)] = Elem<T>::from_f(acc);
      }
      __syncthreads();
    }
    switch (p.halo) {
      case 0: pooled_keys8<T, 0, false>(p, ji, lg, keys, lhist, s_rowM, s_rowInv, s_rowR); break;
      case 1: pooled_keys8<T, 1, false>(p, ji, lg, keys, lhist, s_rowM, s_rowInv, s_rowR); break;
      case 2: pooled_keys8<T, 2, false>(p, ji, lg, keys, lhist, s_rowM, s_rowInv, s_rowR); break;
      case 3: pooled_keys8<T, 3, false>(p, ji, lg, keys, lhist, s_rowM, s_rowInv, s_rowR); break;
      default: pooled_keys_wide<T>(p, ji, lg, keys, lhist); break;
    }
  }
  // select descriptors
  if (threadIdx.x < p.nsel) {
    const int sel = threadIdx.x;
    int k, row;
    if (p.mode == MODE_PREFILL) { k = p.keep_lens ? p.keep_lens[ji.h] : p.keep_const; row = 0; }
    else if (p.mode == MODE_PIVOT) { k = p.topk; row = 0; }
    else if (sel < p.S) { k = p.topk; row = sel; }
    else { k = drift_view().max_len; row = p.S - 1; }
    s_sel_row[sel] = row;
    s_k[sel] = (unsigned int)max(k, 0);
    s_prefix[sel] = 0u;
    s_mask[sel] = 0u;
    s_rem[sel] = (unsigned int)max(k, 0);
    s_gtc[sel] = 0u;
  }
  __syncthreads();

  // ---- phase 3: radix select, 8-bit digits from the top.  The round-0
  // histograms (per score row) came out of the pooling pass.  In the last
  // round every CTA also publishes, per select and digit b, how many of its
  // keys are above and equal to prefix|b, so that after the final barrier
  // each CTA knows how many tokens the CTAs before it select.
  const int ntok = ji.t1 - ji.t0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = 0; r < ROUNDS; ++r) {
    const int shift = KB - 8 * (r + 1);
    const bool last = r == ROUNDS - 1;
    if (r == 0) {
      for (int i = threadIdx.x; i < p.S * 256; i += kSThreads) {
        const unsigned int c = lhist[i];
        if (c) atomicAdd(&p.hist[(((size_t)ji.job * kMaxSel + i / 256) * ROUNDS) * 256 + (i % 256)], c);
      }
    } else {
      for (int i = threadIdx.x; i < p.nsel * 256; i += kSThreads) lhist[i] = 0u;
      __syncthreads();
      for (int sel = 0; sel < p.nsel; ++sel) {
        const unsigned int k = s_k[sel];
        if (k == 0u || k >= (unsigned int)p.Lsel) continue;  // trivial selects
        const unsigned int pre = s_prefix[sel], msk = s_mask[sel];
        const unsigned int* kr = keys + s_sel_row[sel] * p.T;
        unsigned int ngt = 0;
        // below the top digit the keys of one prefix spread over many bins:
        // plain shared-memory atomics (a warp-level match costs more here)
        for (int c0 = 0; c0 < ntok; c0 += kSThreads) {
          const int i = c0 + threadIdx.x;
          const unsigned int key = i < ntok ? kr[i] : 0u;
          ngt += __popc(__ballot_sync(0xffffffffu, i < ntok && (key & msk) > pre));
          if (i < ntok && (key & msk) == pre) atomicAdd(&lhist[sel * 256 + ((key >> shift) & 255u)], 1u);
        }
        if (last && lane == 0 && ngt) atomicAdd(&s_gtc[sel], ngt);
      }
      __syncthreads();
      unsigned int* gh = p.hist + ((size_t)ji.job * kMaxSel * ROUNDS + r) * 256;
      for (int i = threadIdx.x; i < p.nsel * 256; i += kSThreads) {
        const unsigned int c = lhist[i];
        if (c) atomicAdd(&gh[(size_t)(i / 256) * ROUNDS * 256 + (i % 256)], c);
      }
      if (last) {
        // per digit b: (keys above prefix|b, keys equal to it), one warp per select
        for (int sel = warp; sel < p.nsel; sel += kSWarps) {
          const unsigned int k = s_k[sel];
          if (k == 0u || k >= (unsigned int)p.Lsel) continue;
          unsigned int c8[8], tot = 0;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            c8[i] = lhist[sel * 256 + lane * 8 + i];
            tot += c8[i];
          }
          unsigned int suf = tot;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const unsigned int y = __shfl_down_sync(0xffffffffu, suf, o);
            if (lane + o < 32) suf += y;
          }
          unsigned int run = s_gtc[sel] + (suf - tot);
          int2* dst = p.cnt + (((size_t)ji.job * kMaxSel + sel) * 256 + lane * 8) * p.cpj + ji.part;
#pragma unroll
          for (int i = 7; i >= 0; --i) {
            dst[(size_t)i * p.cpj] = make_int2((int)run, (int)c8[i]);
            run += c8[i];
          }
        }
      }
    }
    if (!grid_sync(p.gb, nblocks, epoch, p.err, p.wait_ns, p.stall)) return;
    // stage the job's global histograms of this round (one load round);
    // round 0 was counted per score row
    for (int i = threadIdx.x; i < p.nsel * 256; i += kSThreads) {
      const int sel = i / 256;
      const int slot = r == 0 ? s_sel_row[sel] : sel;
      lhist[i] = __ldcg(&p.hist[(((size_t)ji.job * kMaxSel + slot) * ROUNDS + r) * 256 + (i % 256)]);
    }
    __syncthreads();
    // one warp per select
    for (int sel = warp; sel < p.nsel; sel += kSWarps) {
      const unsigned int k = s_k[sel];
      if (k == 0u || k >= (unsigned int)p.Lsel) continue;
      unsigned int above;
      int bin = find_bin(lhist + sel * 256, s_rem[sel], above);
      if (lane == 0) {
        s_rem[sel] -= above;
        s_prefix[sel] |= ((unsigned int)bin) << shift;
        s_mask[sel] |= 255u << shift;
      }
    }
    __syncthreads();
  }

  // ---- phase 4: where this CTA's selected tokens start.  For a select with
  // threshold key thr and `need` keys equal to thr still to take (in position
  // order), the CTAs before this one select gt_before + min(need, eq_before).
  for (int sel = warp; sel < p.nsel; sel += kSWarps) {
    const unsigned int k = s_k[sel];
    long long gtb = 0, eqb = 0;
    if (k >= (unsigned int)p.Lsel) {
      gtb = min((long long)ji.part * p.T, (long long)p.Lsel);  // everything eligible before is selected
    } else if (k > 0u) {
      const int b = (int)(s_prefix[sel] & 255u);
      const int2* cj = p.cnt + (((size_t)ji.job * kMaxSel + sel) * 256 + b) * p.cpj;
      for (int c0 = 0; c0 < ji.part; c0 += 256) {
        int2 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int c = c0 + lane + 32 * j;
          v[j] = c < ji.part ? __ldcg(&cj[c]) : make_int2(0, 0);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          gtb += v[j].x;
          eqb += v[j].y;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        gtb += __shfl_xor_sync(0xffffffffu, gtb, o);
        eqb += __shfl_xor_sync(0xffffffffu, eqb, o);
      }
    }
    if (lane == 0) {
      s_base[sel] = (int)gtb;
      s_eqoff[sel] = (int)min(eqb, (long long)0x7fffffff);
    }
  }
  // thresholds: trivial selects take everything / nothing
  if (threadIdx.x < p.nsel) {
    const int sel = threadIdx.x;
    const unsigned int k = s_k[sel];
    // take everything: every key at or above 0 (all of them), or, with
    // ineligible positions (key 0), every key above 1 (scores are
    // non-negative, so eligible keys are at least the key of +0)
    if (k >= (unsigned int)p.Lsel) {
      if (p.Lsel == p.L) { s_prefix[sel] = 0u; s_rem[sel] = 0x7fffffffu; }
      else { s_prefix[sel] = 1u; s_rem[sel] = 0u; }
    }
    else if (k == 0u) { s_prefix[sel] = 0xffffffffu; s_rem[sel] = 0u; }
  }
  __syncthreads();
  // Each warp owns a contiguous, 32-aligned slice of the CTA's tokens, so
  // ranks in position order need no block-wide scans: per 32 tokens one
  // ballot for "above", one for "equal", and popc of the lanes below.
  const int TW = ((ntok + kSWarps - 1) / kSWarps + 31) & ~31;
  const int w0 = min(ntok, warp * TW), w1 = min(ntok, w0 + TW);
  const unsigned int lt_mask = (1u << lane) - 1u;
  for (int sel = 0; sel < p.nsel; ++sel) {
    const unsigned int thr = s_prefix[sel];
    const unsigned int* kr = keys + s_sel_row[sel] * p.T;
    int ngt = 0, neq = 0;
    for (int c = w0; c < w1; c += 32) {
      const int i = c + lane;
      const unsigned int key = i < w1 ? kr[i] : 0u;
      ngt += __popc(__ballot_sync(0xffffffffu, i < w1 && key > thr));
      neq += __popc(__ballot_sync(0xffffffffu, i < w1 && key == thr));
    }
    if (lane == 0) s_wcnt[sel][warp] = make_int2(ngt, neq);
  }
  __syncthreads();
  // per-warp starting (selected rank, equal keys seen)
  if (threadIdx.x < p.nsel * kSWarps) {
    const int sel = threadIdx.x / kSWarps, w = threadIdx.x % kSWarps;
    long long gt = s_base[sel], eq = s_eqoff[sel];
    for (int x = 0; x < w; ++x) {
      gt += s_wcnt[sel][x].x;
      eq += s_wcnt[sel][x].y;
    }
    const long long need = (long long)s_rem[sel];
    s_wsel[sel][w] = (int)(gt + (eq < need ? eq : need));
    s_weq[sel][w] = (int)min(eq, (long long)0x7fffffff);
  }
  __syncthreads();

  // ---- phase 5: epilogues
  // Walk this warp's slice in position order; for select `sel` every lane
  // gets its token (or -1 past the slice) and its rank (or -1).  Warp-uniform.
  auto rank_pass = [&](int sel, auto&& fn) {
    const unsigned int thr = s_prefix[sel];
    const long long need = (long long)s_rem[sel];
    const unsigned int* kr = keys + s_sel_row[sel] * p.T;
    long long run_eq = s_weq[sel][warp];
    int run_sel = s_wsel[sel][warp];
    for (int c = w0; c < w1; c += 32) {
      const int i = c + lane;
      const bool in = i < w1;
      const unsigned int key = in ? kr[i] : 0u;
      const unsigned int gtm = __ballot_sync(0xffffffffu, in && key > thr);
      const unsigned int eqm = __ballot_sync(0xffffffffu, in && key == thr);
      const bool is_eq = (eqm >> lane) & 1u;
      const bool sel_me = ((gtm >> lane) & 1u) || (is_eq && run_eq + __popc(eqm & lt_mask) < need);
      const unsigned int selm = __ballot_sync(0xffffffffu, sel_me);
      fn(in ? ji.t0 + i : -1, sel_me ? run_sel + __popc(selm & lt_mask) : -1, c);
      run_sel += __popc(selm);
      run_eq += __popc(eqm);
    }
  };
  // Same walk, one call per 32-token chunk with the selection mask and the
  // rank of the chunk's first selected token (warp-uniform).
  auto rank_walk = [&](int sel, auto&& fnw) {
    const unsigned int thr = s_prefix[sel];
    const long long need = (long long)s_rem[sel];
    const unsigned int* kr = keys + s_sel_row[sel] * p.T;
    long long run_eq = s_weq[sel][warp];
    int run_sel = s_wsel[sel][warp];
    for (int c = w0; c < w1; c += 32) {
      const int i = c + lane;
      const bool in = i < w1;
      const unsigned int key = in ? kr[i] : 0u;
      const unsigned int gtm = __ballot_sync(0xffffffffu, in && key > thr);
      const unsigned int eqm = __ballot_sync(0xffffffffu, in && key == thr);
      const bool is_eq = (eqm >> lane) & 1u;
      const bool sel_me = ((gtm >> lane) & 1u) || (is_eq && run_eq + __popc(eqm & lt_mask) < need);
      const unsigned int selm = __ballot_sync(0xffffffffu, sel_me);
      fnw(c, selm, run_sel);
      run_sel += __popc(selm);
      run_eq += __popc(eqm);
    }
  };

  if (p.mode == MODE_PREFILL) {
    const int kk = (int)s_k[0];  // <= L (the host clamps keep lengths)
    const int row = ji.b * p.KV + ji.h;
    // 1. the job's kept positions in rank order -> the workspace list (and
    //    out_indices when asked for)
    int32_t* plist = p.keep_pos + (size_t)ji.job * p.L;
    rank_walk(0, [&](int c, unsigned int selm, int r0) {
      if ((selm >> lane) & 1u) {
        const int rank = r0 + __popc(selm & lt_mask);
        if (rank < kk) {
          plist[rank] = ji.t0 + c + lane;
          if (p.out_indices) p.out_indices[(size_t)ji.job * p.max_keep + rank] = ji.t0 + c + lane;
        }
      }
    });
    if (p.heads_len && ji.part == 0 && threadIdx.x == 0) p.heads_len[row] = kk;
    if (p.out_indices && ji.part == p.cpj - 1) {
      for (int i = kk + threadIdx.x; i < p.max_keep; i += kSThreads)
        p.out_indices[(size_t)ji.job * p.max_keep + i] = -1;
    }
    // 2. every job's list is complete
    if (!grid_sync(p.gb, nblocks, epoch, p.err, p.wait_ns, p.stall)) return;
    // 3. kept K/V rows to their pages: the rows of all jobs (in job, then
    //    rank order) split into equal contiguous shares, one per CTA, so that
    //    CTAs whose tokens hold many kept positions do not set the end.
    //    Flat slots from each row's first page (prefill pages are contiguous),
    //    or, with a dense output, rows from job * out_job_rows.  Each job's
    //    kept rows are followed by its last `tail` rows (SnapKV's window).
    constexpr int CH = kD * (int)sizeof(T) / 16;  // 16-byte chunks per row
    constexpr int PER = (2 * CH + 31) / 32;        // chunks per lane per row (K and V)
    constexpr int NQ = std::is_same<T, float>::value ? 4 : 8;  // rows in flight per warp
    auto keep_of = [&](int h) { return min(max(p.keep_lens ? p.keep_lens[h] : p.keep_const, 0), p.Lsel); };
    long long total = 0;
    for (int jb = 0; jb < p.n_jobs; ++jb) total += keep_of(jb % p.nh) + p.tail;
    const long long share = (total + nblocks - 1) / nblocks;
    const long long g0 = (long long)blockIdx.x * share, g1 = min(total, g0 + share);
    long long off = 0;
    for (int jb = 0; jb < p.n_jobs && off < g1; ++jb) {
      const int bj = jb / p.nh, hj = jb % p.nh;
      const int keepj = keep_of(hj);
      const int nj = keepj + p.tail;
      const long long a = max(g0, off), e = min(g1, off + nj);
      if (a < e) {
        T* kdst;
        T* vdst;
        bool ok;
        if (p.out_job_rows > 0) {
          ok = nj <= p.out_job_rows;
          kdst = reinterpret_cast<T*>(p.k_pool_out) + (int64_t)jb * p.out_job_rows * kD;
          vdst = reinterpret_cast<T*>(p.v_pool_out) + (int64_t)jb * p.out_job_rows * kD;
        } else {
          const int rowj = bj * p.KV + hj;
          const int start = p.bt[(int64_t)rowj * p.max_blocks];
          ok = !(start < 0 || (int64_t)start * kPage + nj > (int64_t)p.n_blocks * kPage);
          kdst = reinterpret_cast<T*>(p.k_pool_out) + (int64_t)max(start, 0) * kPage * kD;
          vdst = reinterpret_cast<T*>(p.v_pool_out) + (int64_t)max(start, 0) * kPage * kD;
        }
        if (!ok) {
          if (threadIdx.x == 0) set_err(p.err, HC_ERR_RANGE);
        } else {
          const int32_t* pl = p.keep_pos + (size_t)jb * p.L;
          const T* kbase = reinterpret_cast<const T*>(p.k) + bj * p.ksb + (int64_t)hj * p.ksh;
          const T* vbase = reinterpret_cast<const T*>(p.v) + bj * p.vsb + (int64_t)hj * p.vsh;
          const int r_lo = (int)(a - off), r_hi = (int)(e - off);
          for (int rb = r_lo + warp * NQ; rb < r_hi; rb += kSWarps * NQ) {
            int tt[NQ];
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
              const int r = rb + q;
              tt[q] = r >= r_hi ? -1 : r < keepj ? __ldcg(pl + r) : p.L - p.tail + (r - keepj);
            }
            uint4 buf[NQ][PER];
#pragma unroll
            for (int q = 0; q < NQ; ++q)
#pragma unroll
              for (int x8 = 0; x8 < PER; ++x8) {
                const int x = lane + 32 * x8;
                if (tt[q] >= 0 && tt[q] < p.L && x < 2 * CH) {
                  const T* src = x < CH ? kbase + (int64_t)tt[q] * p.kst : vbase + (int64_t)tt[q] * p.vst;
                  buf[q][x8] = ldg128(reinterpret_cast<const uint4*>(src) + (x % CH));
                }
              }
#pragma unroll
            for (int q = 0; q < NQ; ++q)
#pragma unroll
              for (int x8 = 0; x8 < PER; ++x8) {
                const int x = lane + 32 * x8;
                if (tt[q] >= 0 && tt[q] < p.L && x < 2 * CH) {
                  T* dst = (x < CH ? kdst : vdst) + (int64_t)(rb + q) * kD;
                  reinterpret_cast<uint4*>(dst)[x % CH] = buf[q][x8];
                }
              }
          }
        }
      }
      off += nj;
    }
  } else if (p.mode == MODE_PIVOT) {
    const int slot = ji.job;
    const int kk = (int)s_k[0];
    uint32_t* bm = p.ref_bitmap + (size_t)slot * p.bitmap_words;
    rank_pass(0, [&](int t, int rank, int c) {
      const bool sel = rank >= 0 && rank < kk;
      if (sel) p.ref_positions[(size_t)slot * p.topk + rank] = t;
      const unsigned int bits = __ballot_sync(0xffffffffu, sel);
      if (lane == 0) bm[(ji.t0 + c) >> 5] = bits;
    });
  } else {
    // drift: overlap of each step's top-k with the reference bitmap
    uint32_t* bm = drift_view().bitmap;
    // this CTA's words of the reference bitmap were staged at kernel start
    const int wbeg = ji.t0 >> 5, nwords = ((ji.t1 + 31) >> 5) - wbeg;
    const bool staged = nwords <= kRefWords;
    // every selected token counts (a select takes exactly min(k, L) tokens);
    // 32-token chunks are bitmap words
    for (int sel = 0; sel < p.S; ++sel) {
      unsigned int local = 0;
      rank_walk(sel, [&](int c, unsigned int selm, int) {
        const int wi = (ji.t0 + c) >> 5;
        const uint32_t word = staged ? s_refw[wi - wbeg] : bm[wi];
        local += __popc(selm & word);
      });
      if (lane == 0 && local) atomicAdd(&s_ov[sel], local);
    }
    // retrieval list: last step's top-max_len, ascending
    {
      const int sel = p.S;
      const DriftView dv = drift_view();
      const int kk = min((int)s_k[sel], dv.retr_cap);
      rank_pass(sel, [&](int t, int rank, int) {
        if (rank >= 0 && rank < kk) dv.retr[rank] = t;
      });
    }
    __syncthreads();
    if (threadIdx.x < p.S && s_ov[threadIdx.x])
      atomicAdd(&p.overlap[ji.job * kMaxRows + threadIdx.x], s_ov[threadIdx.x]);
    if (!grid_sync(p.gb, nblocks, epoch, p.err, p.wait_ns, p.stall)) return;
    if (threadIdx.x < p.S) s_ov[threadIdx.x] = __ldcg(&p.overlap[ji.job * kMaxRows + threadIdx.x]);
    __syncthreads();
    if (threadIdx.x == 0) {
      float c[kMaxRows];
      const float kf = (float)p.topk;
      for (int s = 0; s < p.S; ++s) c[s] = __fdiv_rn((float)s_ov[s], kf);
      float srt[kMaxRows];
      for (int s = 0; s < p.S; ++s) srt[s] = c[s];
      for (int a = 1; a < p.S; ++a)
        for (int b = a; b > 0 && srt[b - 1] > srt[b]; --b) {
          float tmp = srt[b]; srt[b] = srt[b - 1]; srt[b - 1] = tmp;
        }
      double med = (p.S & 1) ? (double)srt[p.S / 2]
                             : ((double)srt[p.S / 2 - 1] + (double)srt[p.S / 2]) / 2.0;
      const int trig = med < p.threshold;
      s_trigger = trig;
      if (ji.part == 0) {
        const DriftView dv = drift_view();
        *dv.trigger = trig;
        if (dv.coeffs) for (int s = 0; s < p.S; ++s) dv.coeffs[s] = c[s];
        if (dv.median) *dv.median = med;
      }
    }
    __syncthreads();
    if (s_trigger) {
      const int sel = p.S - 1;
      const int kk = (int)s_k[sel];
      int32_t* ref_pos = drift_view().ref_pos;
      rank_pass(sel, [&](int t, int rank, int c) {
        const bool on = rank >= 0 && rank < kk;
        if (on) ref_pos[rank] = t;
        const unsigned int bits = __ballot_sync(0xffffffffu, on);
        if (lane == 0) bm[(ji.t0 + c) >> 5] = bits;
      });
    }
  }
  grid_depart(p.gb, nblocks);
}

// ---------------------------------------------------------------------------
// Host side.
struct ScorePlan {
  int cpj, T, TB, grid;
  size_t smem, logits_bytes;
  bool logits_in_smem;
  bool umma;  // tcgen05 logits: tokens per CTA a multiple of 128
  int n_stages, NP, tmem_cols;
};

static int num_sms() { return device_sms(current_device()); }

// Dynamic shared memory a launch may use (the opt-in limit less the kernel's
// static shared memory, with room to spare).
constexpr size_t kDynSmemCap = 203 * 1024;

template <typename T>
static size_t smem_bytes(int Rq, int S, int T_, int TB, bool logits_in_smem, bool fma) {
  size_t b = 0;
  if (logits_in_smem) b += ((size_t)Rq * TB * sizeof(T) + 15) & ~(size_t)15;
  b += (size_t)S * T_ * sizeof(unsigned int);
  b += (size_t)kMaxSel * 256 * sizeof(unsigned int);
  b += (size_t)kSWarps * kMaxRq * sizeof(float);
  if (fma) b += (size_t)Rq * kD * sizeof(float) + 32 * (kD + 1) * sizeof(float);
  return b;
}

static size_t elem_size(int dtype) { return dtype == HC_F32 ? 4 : 2; }

// Plan the partition: as many CTAs per job as fit co-resident (1 per SM),
// token ranges a multiple of 32 (bitmap words stay CTA-private), of 128 for
// the tcgen05 path (whole key tiles).
//
// Logits paths, 16-bit dtypes: up to 40 query rows (one observation window:
// pivot sets, drift checks, HeteroCache prefill selection) the mma.sync path,
// whose plain vector loads stream the keys faster than the TMA ring at these
// row counts (measured at 128K tokens: drift check 49.7 vs 53.7 us, pivot set
// 27.5 vs 31.5 us, the key stream being the limit of both); more rows (an
// observation window of W > 1 queries) the tcgen05 path, when the keys'
// tensor maps could be made (3.4x faster than the CUDA-core path at W = 32).
// The tcgen05 path takes 2-6 shared-memory stages of 128 keys plus the query
// operand; its logits stay in shared memory when that leaves four stages.
// fp32: the CUDA-core path.
// lg_rows: rows of the logits buffer on the tcgen05 path (one window-summed
// row per score row; Rq when not given).
static ScorePlan plan_score(int dtype, int n_jobs, int L, int Rq, int S, int ctas_per_sm, bool umma,
                            int lg_rows = 0) {
  ScorePlan pl;
  pl.umma = umma && dtype != HC_F32 && Rq > 40;
  const int gran = pl.umma ? 128 : 32;
  const int max_ctas = num_sms() * ctas_per_sm;
  int cpj = max(1, max_ctas / max(n_jobs, 1));
  cpj = min(cpj, (L + gran - 1) / gran);
  int T_ = ((L + cpj - 1) / cpj + gran - 1) / gran * gran;
  cpj = (L + T_ - 1) / T_;
  pl.cpj = cpj;
  pl.T = T_;
  pl.TB = T_ + 2 * kMargin;
  pl.grid = cpj * n_jobs;
  const size_t es = elem_size(dtype);
  const size_t with = (size_t)Rq * pl.TB * es;
  pl.n_stages = pl.NP = pl.tmem_cols = 0;
  if (pl.umma) {
    pl.NP = max(16, (Rq + 15) / 16 * 16);
    pl.tmem_cols = 32;
    while (pl.tmem_cols < 2 * pl.NP) pl.tmem_cols *= 2;
    // the stage ring shares memory with the later phases' arrays
    const size_t later = smem_bytes<float>(Rq, S, T_, pl.TB, false, false);
    const size_t fixed = 1024 + (size_t)umma_query_rows(Rq) * 256;
    const size_t lgr = (size_t)(lg_rows > 0 ? lg_rows : Rq);
    const size_t lgb = (lgr * pl.TB * es + 15) & ~(size_t)15;
    auto stages_for = [&](bool lsm) {
      const size_t used = fixed + (lsm ? lgb : 0);
      return used >= kDynSmemCap ? 0 : (int)min((size_t)kMaxStages, (kDynSmemCap - used) / kUStage);
    };
    // logits in shared memory if that leaves at least four stages
    pl.logits_in_smem = stages_for(true) >= 4;
    pl.n_stages = stages_for(pl.logits_in_smem);
    const size_t region = max((size_t)pl.n_stages * kUStage, later);
    const size_t total = fixed + (pl.logits_in_smem ? lgb : 0) + region;
    if (pl.n_stages >= 2 && total <= kDynSmemCap) {
      pl.smem = total;
      pl.logits_bytes = pl.logits_in_smem ? 0 : (size_t)pl.grid * lgr * pl.TB * es;
      return pl;
    }
    pl.umma = false;  // no room: the legacy paths (128-token ranges are valid there too)
  }
  const bool fma = dtype == HC_F32 || Rq > 40;
  size_t rest = smem_bytes<float>(Rq, S, T_, pl.TB, false, fma);
  pl.logits_in_smem = (with + rest + 64) <= kDynSmemCap;
  pl.smem = rest + (pl.logits_in_smem ? ((with + 15) & ~(size_t)15) : 0);
  pl.logits_bytes = pl.logits_in_smem ? 0 : (size_t)pl.grid * Rq * pl.TB * es;
  return pl;
}

struct ScoreWs {
  size_t off_gb, off_part, off_hist, off_cnt, off_overlap, off_logits, off_keep, total;
};

static ScoreWs score_ws_layout(int n_jobs, const ScorePlan& pl, int Rq, int L) {
  ScoreWs w;
  size_t o = 0;
  auto take = [&](size_t n) { size_t r = o; o += (n + 255) & ~(size_t)255; return r; };
  w.off_gb = take(sizeof(GridBarrier));
  w.off_part = take((size_t)n_jobs * pl.cpj * Rq * sizeof(float2));
  w.off_hist = take((size_t)n_jobs * kMaxSel * 4 * 256 * sizeof(unsigned int));
  w.off_cnt = take((size_t)n_jobs * kMaxSel * pl.cpj * 256 * sizeof(int2));
  w.off_overlap = take((size_t)n_jobs * kMaxRows * sizeof(unsigned int));
  w.off_logits = take(pl.logits_bytes);
  w.off_keep = take((size_t)n_jobs * L * sizeof(int32_t));
  w.total = o;
  return w;
}

template <typename T, int MODE>
static int launch_score_mode(ScoreParams& p, const ScorePlan& pl, const CUtensorMap* maps, void* ws,
                             size_t ws_bytes, cudaStream_t st, const DriftBatch* batch) {
  ScoreWs w = score_ws_layout(p.n_jobs, pl, p.Rq, p.L);
  if (!ws || ws_bytes < w.total) return HC_ERR_WORKSPACE;
  unsigned char* base = reinterpret_cast<unsigned char*>(ws);
  p.gb = reinterpret_cast<GridBarrier*>(base + w.off_gb);
  p.part = reinterpret_cast<float2*>(base + w.off_part);
  p.hist = reinterpret_cast<unsigned int*>(base + w.off_hist);
  p.cnt = reinterpret_cast<int2*>(base + w.off_cnt);
  p.overlap = reinterpret_cast<unsigned int*>(base + w.off_overlap);
  p.glogits = pl.logits_in_smem ? nullptr : (void*)(base + w.off_logits);
  p.keep_pos = reinterpret_cast<int32_t*>(base + w.off_keep);
  p.logits_in_smem = pl.logits_in_smem ? 1 : 0;
  p.wait_ns = wait_limit_ns(kBarrierTimeoutNs);
  p.stall = injected_stall();
  p.cpj = pl.cpj;
  p.T = pl.T;
  p.TB = pl.TB;
  p.umma = pl.umma ? 1 : 0;
  p.n_stages = pl.n_stages;
  p.NP = pl.NP;
  p.tmem_cols = pl.tmem_cols;
  auto kern = score_select_kernel<T, MODE>;
  // Attribute and occupancy queries are made once per device and shared-memory
  // size and cached, so a launch issues no non-stream CUDA call (graph capture
  // safe after the first launch of a given shape).
  static bool attr_set[kMaxDevices];
  static ShapeCache<16> occs;
  const int dev = current_device();
  if (dev < 0) return HC_ERR_CUDA;
  int occ = -1;
  {
    std::lock_guard<std::mutex> g(host_lock());
    if (!attr_set[dev]) {
      int optin = 0;
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return HC_ERR_CUDA;
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               optin - (int)fa.sharedSizeBytes) != cudaSuccess)
        return HC_ERR_CUDA;
      attr_set[dev] = true;
    }
    long long v = 0;
    if (occs.find(dev, (long long)pl.smem, v)) {
      occ = (int)v;
    } else {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kSThreads, pl.smem) != cudaSuccess)
        return HC_ERR_CUDA;
      occs.put(dev, (long long)pl.smem, occ);
    }
  }
  if ((long long)occ * num_sms() < pl.grid) return HC_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  BatchOf<MODE> bp;
  if constexpr (MODE == MODE_DRIFT) {
    if (batch) bp = *batch;
    else bp.n = 0;
  } else {
    bp.n = 0;
  }
  if (cudaLaunchKernelEx(&cfg, kern, p, maps[0], maps[1], bp) != cudaSuccess) return HC_ERR_CUDA;
  return HC_OK;
}

template <typename T>
static int launch_score(ScoreParams& p, const ScorePlan& pl, const CUtensorMap* maps, void* ws, size_t ws_bytes,
                        cudaStream_t st, const DriftBatch* batch) {
  switch (p.mode) {
    case MODE_PREFILL: return launch_score_mode<T, MODE_PREFILL>(p, pl, maps, ws, ws_bytes, st, nullptr);
    case MODE_PIVOT: return launch_score_mode<T, MODE_PIVOT>(p, pl, maps, ws, ws_bytes, st, nullptr);
    case MODE_DRIFT: return launch_score_mode<T, MODE_DRIFT>(p, pl, maps, ws, ws_bytes, st, batch);
    default: return HC_ERR_INVALID;
  }
}

// Tensor maps of the keys for the tcgen05 path: 128-row tiles and 16-row
// margin tiles, over the paged pool (drift checks) or the dense [bsz, KV, L,
// 128] keys (prefill scoring, pivot sets).  False if either cannot be made.
static bool key_tensor_maps(const ScoreParams& p, int dtype, CUtensorMap* maps) {
  if (p.mode == MODE_DRIFT) {
    const long long rows = (long long)p.n_blocks * kPage;
    return pool_tensor_map(&maps[0], p.k_pool, rows, dtype, 128) &&
           pool_tensor_map(&maps[1], p.k_pool, rows, dtype, kMargin);
  }
  const int bsz = p.n_jobs / max(p.nh, 1);
  return dense_tensor_map(&maps[0], p.k, bsz, p.KV, p.L, p.ksb, p.ksh, p.kst, dtype, 128) &&
         dense_tensor_map(&maps[1], p.k, bsz, p.KV, p.L, p.ksb, p.ksh, p.kst, dtype, kMargin);
}

template <typename T>
static int run_score(ScoreParams& p, void* ws, size_t ws_bytes, cudaStream_t st, const DriftBatch* batch) {
  constexpr bool f32 = std::is_same<T, float>::value;
  const int dtype = f32 ? HC_F32 : std::is_same<T, __half>::value ? HC_F16 : HC_BF16;
  CUtensorMap maps[2];
  std::memset(maps, 0, sizeof(maps));
  // a batch's jobs read different pools, and its query rows (steps x groups
  // <= 40) take the mma.sync path, which needs no tensor maps: measured on a
  // batch of 8 checks at 128K, the tcgen05 path's logits took 3.4x as long
  const bool umma = !f32 && !batch && key_tensor_maps(p, dtype, maps);
  // one 512-thread CTA per SM
  ScorePlan pl = plan_score(dtype, p.n_jobs, p.L, p.Rq, p.S, 1, umma, p.S * p.G);
  return launch_score<T>(p, pl, maps, ws, ws_bytes, st, batch);
}

// Large enough for either plan (whether the keys' tensor maps can be made is
// known only at launch).
size_t score_workspace_size(int dtype, int n_jobs, int L, int Rq, int S) {
  // the tcgen05 plan's buffer holds between one and Rq rows (score rows are
  // not known here): reserve Rq rows in global memory, whichever it picks
  ScorePlan a = plan_score(dtype, n_jobs, L, Rq, S, 1, true);
  if (a.umma) a.logits_bytes = (size_t)a.grid * Rq * a.TB * elem_size(dtype);
  const ScorePlan b = plan_score(dtype, n_jobs, L, Rq, S, 1, false);
  return max(score_ws_layout(n_jobs, a, Rq, L).total, score_ws_layout(n_jobs, b, Rq, L).total);
}

// Drift checks per batch launch when the caller does not say.
constexpr int kDriftBatchDefault = 8;

int drift_batch_per_launch(int dtype, int n_jobs, int L, int Rq, int S, int want) {
  if (n_jobs <= 0 || L <= 0 || Rq <= 0 || S <= 0) return 0;
  int per = want > 0 ? want : kDriftBatchDefault;
  per = min(min(per, kDriftBatchMax), n_jobs);
  while (per > 1 && plan_score(dtype, per, L, Rq, S, 1, false).smem > kDynSmemCap) --per;
  return per;
}

int score_dispatch(int dtype, ScoreParams& p, void* ws, size_t ws_bytes, cudaStream_t st, const DriftBatch* batch) {
  if (batch && (p.mode != MODE_DRIFT || batch->n != p.n_jobs || batch->n < 1 || batch->n > kDriftBatchMax))
    return HC_ERR_INVALID;
  switch (dtype) {
    case HC_F32: return run_score<float>(p, ws, ws_bytes, st, batch);
    case HC_BF16: return run_score<__nv_bfloat16>(p, ws, ws_bytes, st, batch);
    case HC_F16: return run_score<__half>(p, ws, ws_bytes, st, batch);
    default: return HC_ERR_DTYPE;
  }
}

}  // namespace hc
