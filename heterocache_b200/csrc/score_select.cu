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
#include "hc_params.cuh"

namespace hc {



struct JobInfo {
  int b, h, job, part, t0, t1;
};

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
    ji.h = p.job_heads[ji.job];
  }
  ji.t0 = ji.part * p.T;
  ji.t1 = min(p.L, ji.t0 + p.T);
  return ji;
}

// Address of key row t of the job (dense tensor or paged pool).
template <typename T>
__device__ __forceinline__ const T* key_row(const ScoreParams& p, const JobInfo& ji, int t) {
  if (p.mode == MODE_DRIFT) {
    int row = ji.b * p.KV + ji.h;
    int blk = p.bt[(int64_t)row * p.max_blocks + (t >> 8)];
    if (blk < 0 || blk >= p.n_blocks) {  // keep the address inside the pool; report
      set_err(p.err, HC_ERR_RANGE);
      blk = 0;
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

// ---------------------------------------------------------------------------
// Phase 1, tensor-core path (16-bit dtypes, Rq <= 8*NT): a warp computes the
// logits of 16 tokens x 8*NT query rows per iteration with m16n8k16 MMAs.
// A = 16 key rows (tokens), B = query rows^T.  The head dimension is read in
// a permuted order so that each thread loads 16 contiguous bytes per row; the
// query fragments use the same permutation, so the dot products are exact
// sums over all 128 dims.
template <typename T, int NT>
__device__ void logits_mma(const ScoreParams& p, const JobInfo& ji, T* lg, float* wmax) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  uint32_t qb[NT][8][2];
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
  float rmax[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) rmax[nt][0] = rmax[nt][1] = -INFINITY;

  const int lo = max(0, ji.t0 - kMargin);
  const int hi = min(p.L, ji.t1 + kMargin);
  const int base = ji.t0 - kMargin;  // lg column 0 <-> token base
  for (int tg = lo + warp * 16; tg < hi; tg += kSWarps * 16) {
    const int ta = min(tg + gid, p.L - 1), tb = min(tg + gid + 8, p.L - 1);
    const T* ra = key_row<T>(p, ji, ta);
    const T* rb = key_row<T>(p, ji, tb);
    uint4 ka[4], kb[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      ka[s] = ld_stream128(ra + 32 * s + 8 * tig);
      kb[s] = ld_stream128(rb + 32 * s + 8 * tig);
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma16816<T>(acc[nt], ka[s].x, kb[s].x, ka[s].y, kb[s].y, qb[nt][2 * s][0], qb[nt][2 * s][1]);
        mma16816<T>(acc[nt], ka[s].z, kb[s].z, ka[s].w, kb[s].w, qb[nt][2 * s + 1][0], qb[nt][2 * s + 1][1]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = nt * 8 + 2 * tig + (e & 1);
        const int t = tg + gid + ((e >> 1) << 3);
        if (qi >= p.Rq || t >= hi) continue;
        float x = Elem<T>::rnd(Elem<T>::rnd(acc[nt][e]) / p.sqrt_d);
        if (masked(p, qi, t)) x = -INFINITY;
        lg[(int64_t)qi * p.TB + (t - base)] = Elem<T>::from_f(x);
        if (t >= ji.t0 && t < ji.t1) rmax[nt][e & 1] = fmaxf(rmax[nt][e & 1], x);
      }
    }
  }
  // reduce the running maxima over the 8 lanes sharing tig, then publish
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float m = rmax[nt][c];
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
      const int qi = nt * 8 + 2 * tig + c;
      if (gid == 0 && qi < p.Rq) wmax[warp * kMaxRq + qi] = m;
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
        float x = Elem<T>::rnd(Elem<T>::rnd(acc) / p.sqrt_d);
        if (masked(p, qi, t)) x = -INFINITY;
        lg[(int64_t)qi * p.TB + (t - base)] = Elem<T>::from_f(x);
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

// Softmax probability of logit x with row max M and row sum of exp S, in
// fp32 (the reference's softmax(dtype=float32)).  fp32 models use the
// accurate exp and an IEEE division; 16-bit models round the result to
// their dtype right after, so the fast exp (a few ulp of fp32) and the
// reciprocal are used there.
template <typename T>
__device__ __forceinline__ float softmax_prob(float x, float M, float S) {
  if constexpr (std::is_same<T, float>::value) return expf(x - M) / S;
  else return __expf(x - M) * __frcp_rn(S);
}

// Phase 2 for W == 1 and pooling half-width HALO <= 3, fused: each thread
// takes a strip of 8 output tokens of one score row, computes the rounded
// probabilities of the strip plus halo once per query head, pools each
// output in the reference's order ((((p0+p1)+p2)+p3)+p4, divided by the
// kernel size, count_include_pad) and keeps the max over the GQA group.
template <typename T, int HALO>
__device__ void pooled_keys_fused(const ScoreParams& p, const JobInfo& ji, const T* lg, unsigned int* keys,
                                  const float* s_rowM, const float* s_rowS) {
  constexpr int SW = 8;
  constexpr int NP = SW + 2 * HALO;
  constexpr float KS = (float)(2 * HALO + 1);
  const int base = ji.t0 - kMargin;
  const int ntok = ji.t1 - ji.t0;
  const int nstrip = (ntok + SW - 1) / SW;
  for (int it = threadIdx.x; it < p.S * nstrip; it += kSThreads) {
    const int s = it / nstrip;
    const int t0 = ji.t0 + (it - s * nstrip) * SW;
    float best[SW];
#pragma unroll
    for (int o = 0; o < SW; ++o) best[o] = -INFINITY;
    for (int g = 0; g < p.G; ++g) {
      const int qi = s * p.G + g;
      const float M = s_rowM[qi], S = s_rowS[qi];
      const T* row = lg + (int64_t)qi * p.TB - base;
      float pv[NP];
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int t = t0 - HALO + j;
        float v = p.pooling == HC_AVGPOOL ? 0.f : -INFINITY;  // padding
        if (t >= 0 && t < p.L) {
          const float x = Elem<T>::to_f(row[t]);
          v = (x == -INFINITY) ? 0.f : Elem<T>::rnd(softmax_prob<T>(x, M, S));
        }
        pv[j] = v;
      }
#pragma unroll
      for (int o = 0; o < SW; ++o) {
        float v;
        if (p.pooling == HC_AVGPOOL) {
          float acc = pv[o];
#pragma unroll
          for (int j = 1; j <= 2 * HALO; ++j) acc += pv[o + j];
          v = Elem<T>::rnd(acc / KS);
        } else {
          v = pv[o];
#pragma unroll
          for (int j = 1; j <= 2 * HALO; ++j) v = fmaxf(v, pv[o + j]);
        }
        best[o] = fmaxf(best[o], v);
      }
    }
#pragma unroll
    for (int o = 0; o < SW; ++o) {
      const int t = t0 + o;
      if (t < ji.t1) {
        keys[s * p.T + (t - ji.t0)] = Elem<T>::key(best[o]);
        if (p.out_scores)
          reinterpret_cast<T*>(p.out_scores)[((size_t)ji.job * p.S + s) * p.L + t] = Elem<T>::from_f(best[o]);
      }
    }
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

template <typename T>
__global__ void __launch_bounds__(kSThreads, 1) score_select_kernel(ScoreParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float s_rowM[kMaxRq], s_rowInv[kMaxRq];
  __shared__ unsigned int s_prefix[kMaxSel], s_mask[kMaxSel], s_rem[kMaxSel], s_k[kMaxSel];
  __shared__ int s_sel_row[kMaxSel];
  __shared__ int2 s_wcnt[kMaxSel][kSWarps];
  __shared__ int s_base[kMaxSel], s_eqoff[kMaxSel];
  __shared__ unsigned int s_ov[kMaxRows];
  __shared__ uint32_t s_refw[kRefWords];
  __shared__ int s_trigger;

  constexpr int KB = Elem<T>::kKeyBits;
  constexpr int ROUNDS = KB / 8;
  const JobInfo ji = job_info(p);
  const int nblocks = gridDim.x;
  unsigned int epoch = 0;

  // ---- shared memory carve-up
  unsigned char* sp = smem;
  T* lg;
  if (p.logits_in_smem) {
    lg = reinterpret_cast<T*>(sp);
    sp += ((size_t)p.Rq * p.TB * sizeof(T) + 15) & ~(size_t)15;
  } else {
    lg = reinterpret_cast<T*>(p.glogits) + (size_t)blockIdx.x * p.Rq * p.TB;
  }
  unsigned int* keys = reinterpret_cast<unsigned int*>(sp);
  sp += (size_t)p.S * p.T * sizeof(unsigned int);
  unsigned int* lhist = reinterpret_cast<unsigned int*>(sp);
  sp += (size_t)kMaxSel * 256 * sizeof(unsigned int);
  float* wmax = reinterpret_cast<float*>(sp);
  sp += (size_t)kSWarps * kMaxRq * sizeof(float);
  float* sq = reinterpret_cast<float*>(sp);  // fma path only

  // ---- zero the per-launch accumulators (ordered before use by barrier 1)
  if (ji.part == 0) {
    unsigned int* hj = p.hist + (size_t)ji.job * kMaxSel * ROUNDS * 256;
    for (int i = threadIdx.x; i < kMaxSel * ROUNDS * 256; i += kSThreads) hj[i] = 0u;
    if (p.mode == MODE_DRIFT && threadIdx.x < p.S) p.overlap[ji.job * kMaxRows + threadIdx.x] = 0u;
  }

  // ---- phase 1: logits
  constexpr bool kTensor = !std::is_same<T, float>::value;
  bool used_mma = false;
  if constexpr (kTensor) {
    if (p.Rq <= 8) { logits_mma<T, 1>(p, ji, lg, wmax); used_mma = true; }
    else if (p.Rq <= 16) { logits_mma<T, 2>(p, ji, lg, wmax); used_mma = true; }
    else if (p.Rq <= 24) { logits_mma<T, 3>(p, ji, lg, wmax); used_mma = true; }
    else if (p.Rq <= 32) { logits_mma<T, 4>(p, ji, lg, wmax); used_mma = true; }
    else if (p.Rq <= 40) { logits_mma<T, 5>(p, ji, lg, wmax); used_mma = true; }
  }
  if (!used_mma) {
    float* sk = sq + p.Rq * kD;
    logits_fma<T>(p, ji, lg, wmax, sq, sk);
  }
  __syncthreads();
  for (int qi = threadIdx.x; qi < p.Rq; qi += kSThreads) {
    float m = -INFINITY;
    for (int w = 0; w < kSWarps; ++w) m = fmaxf(m, wmax[w * kMaxRq + qi]);
    s_rowM[qi] = m;
  }
  __syncthreads();
  // partial sum of exp over own tokens
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int base = ji.t0 - kMargin;
    for (int qi = warp; qi < p.Rq; qi += kSWarps) {
      const float m = s_rowM[qi];
      float s = 0.f;
      if (m != -INFINITY) {
        for (int t = ji.t0 + lane; t < ji.t1; t += 32) {
          float x = Elem<T>::to_f(lg[(int64_t)qi * p.TB + (t - base)]);
          s += expf(x - m);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) p.part[((size_t)ji.job * p.cpj + ji.part) * p.Rq + qi] = make_float2(m, s);
    }
  }
  if (!grid_sync(p.gb, nblocks, epoch, p.err)) return;

  // ---- phase 2: global softmax statistics, probabilities, pooling, keys
  {
    // one warp per query row, lanes over the job's CTAs
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float2* pj = p.part + (size_t)ji.job * p.cpj * p.Rq;
    for (int qi = warp; qi < p.Rq; qi += kSWarps) {
      float M = -INFINITY;
      for (int c = lane; c < p.cpj; c += 32) M = fmaxf(M, pj[c * p.Rq + qi].x);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      float S = 0.f;
      for (int c = lane; c < p.cpj; c += 32) {
        const float2 v = pj[c * p.Rq + qi];
        if (v.x != -INFINITY) S += v.y * expf(v.x - M);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
      if (lane == 0) {
        s_rowM[qi] = M;
        s_rowInv[qi] = S;
      }
    }
  }
  __syncthreads();
  const bool fused = p.W == 1 && p.halo >= 1 && p.halo <= 3;
  if (fused) {
    switch (p.halo) {
      case 1: pooled_keys_fused<T, 1>(p, ji, lg, keys, s_rowM, s_rowInv); break;
      case 2: pooled_keys_fused<T, 2>(p, ji, lg, keys, s_rowM, s_rowInv); break;
      default: pooled_keys_fused<T, 3>(p, ji, lg, keys, s_rowM, s_rowInv); break;
    }
  } else {
    const int base = ji.t0 - kMargin;
    const int lo = max(0, ji.t0 - p.halo), hi = min(p.L, ji.t1 + p.halo);
    const int span = hi - lo;
    for (int i = threadIdx.x; i < p.Rq * span; i += kSThreads) {
      int qi = i / span, t = lo + i % span;
      T* cell = lg + (int64_t)qi * p.TB + (t - base);
      float x = Elem<T>::to_f(*cell);
      float pr = (x == -INFINITY) ? 0.f : softmax_prob<T>(x, s_rowM[qi], s_rowInv[qi]);
      *cell = Elem<T>::from_f(pr);
    }
    __syncthreads();
    if (p.W > 1) {
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
    // pooled, GQA-max keys for own tokens
    const int ntok = ji.t1 - ji.t0;
    for (int i = threadIdx.x; i < p.S * ntok; i += kSThreads) {
      int s = i / ntok, t = ji.t0 + i % ntok;
      float best = -INFINITY;
      for (int g = 0; g < p.G; ++g) {
        const T* row = lg + (int64_t)((s * p.G + g) * p.W) * p.TB - base;
        float v;
        if (p.pooling == HC_AVGPOOL) {
          float acc = 0.f;
          for (int j = t - p.halo; j <= t + p.halo; ++j)
            if (j >= 0 && j < p.L) acc += Elem<T>::to_f(row[j]);
          v = Elem<T>::rnd(acc / (float)p.ksize);
        } else {
          v = -INFINITY;
          for (int j = t - p.halo; j <= t + p.halo; ++j)
            if (j >= 0 && j < p.L) v = fmaxf(v, Elem<T>::to_f(row[j]));
        }
        best = fmaxf(best, v);
      }
      keys[s * p.T + (t - ji.t0)] = Elem<T>::key(best);
      if (p.out_scores) {
        T* os = reinterpret_cast<T*>(p.out_scores);
        os[((size_t)ji.job * p.S + s) * p.L + t] = Elem<T>::from_f(best);
      }
    }
  }
  // select descriptors
  if (threadIdx.x < p.nsel) {
    const int sel = threadIdx.x;
    int k, row;
    if (p.mode == MODE_PREFILL) { k = p.keep_lens[ji.h]; row = 0; }
    else if (p.mode == MODE_PIVOT) { k = p.topk; row = 0; }
    else if (sel < p.S) { k = p.topk; row = sel; }
    else { k = p.max_len[ji.job]; row = p.S - 1; }
    s_sel_row[sel] = row;
    s_k[sel] = (unsigned int)max(k, 0);
    s_prefix[sel] = 0u;
    s_mask[sel] = 0u;
    s_rem[sel] = (unsigned int)max(k, 0);
  }
  __syncthreads();

  // ---- phase 3: radix select
  const int ntok = ji.t1 - ji.t0;
  for (int r = 0; r < ROUNDS; ++r) {
    const int shift = KB - 8 * (r + 1);
    for (int i = threadIdx.x; i < p.nsel * 256; i += kSThreads) lhist[i] = 0u;
    __syncthreads();
    for (int sel = 0; sel < p.nsel; ++sel) {
      const unsigned int k = s_k[sel];
      if (k == 0u || k >= (unsigned int)p.L) continue;  // trivial selects
      const unsigned int pre = s_prefix[sel], msk = s_mask[sel];
      const unsigned int* kr = keys + s_sel_row[sel] * p.T;
      for (int i = threadIdx.x; i < ntok; i += kSThreads) {
        unsigned int key = kr[i];
        if ((key & msk) == pre) atomicAdd(&lhist[sel * 256 + ((key >> shift) & 255u)], 1u);
      }
    }
    __syncthreads();
    unsigned int* gh = p.hist + ((size_t)ji.job * kMaxSel * ROUNDS + r) * 256;
    for (int i = threadIdx.x; i < p.nsel * 256; i += kSThreads) {
      unsigned int c = lhist[i];
      if (c) atomicAdd(&gh[(size_t)(i / 256) * ROUNDS * 256 + (i % 256)], c);
    }
    if (!grid_sync(p.gb, nblocks, epoch, p.err)) return;
    {
      // one warp per select
      const int warp = threadIdx.x >> 5;
      for (int sel = warp; sel < p.nsel; sel += kSWarps) {
        const unsigned int k = s_k[sel];
        if (k == 0u || k >= (unsigned int)p.L) continue;
        unsigned int above;
        int bin = find_bin(gh + (size_t)sel * ROUNDS * 256, s_rem[sel], above);
        if ((threadIdx.x & 31) == 0) {
          s_rem[sel] -= above;
          s_prefix[sel] |= ((unsigned int)bin) << shift;
          s_mask[sel] |= 255u << shift;
        }
      }
    }
    __syncthreads();
  }
  // thresholds: trivial selects take everything / nothing
  if (threadIdx.x < p.nsel) {
    const int sel = threadIdx.x;
    const unsigned int k = s_k[sel];
    if (k >= (unsigned int)p.L) { s_prefix[sel] = 0u; s_rem[sel] = 0x7fffffffu; }
    else if (k == 0u) { s_prefix[sel] = 0xffffffffu; s_rem[sel] = 0u; }
  }
  __syncthreads();

  // ---- phase 4: counts of keys above / at each threshold, per warp slice
  // Each warp owns a contiguous, 32-aligned slice of the CTA's tokens, so
  // ranks in position order need no block-wide scans: per 32 tokens one
  // ballot for "above", one for "equal", and popc of the lanes below.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
  if (threadIdx.x < p.nsel) {
    int gt = 0, eq = 0;
    for (int w = 0; w < kSWarps; ++w) {
      gt += s_wcnt[threadIdx.x][w].x;
      eq += s_wcnt[threadIdx.x][w].y;
    }
    p.cnt[((size_t)ji.job * kMaxSel + threadIdx.x) * p.cpj + ji.part] = make_int2(gt, eq);
  }
  if (!grid_sync(p.gb, nblocks, epoch, p.err)) return;
  // Rank offsets of this CTA: over the job's earlier CTAs c < part, the
  // selected count is n_gt(c) + clamp(need - eq_before(c), 0, n_eq(c)).
  // One warp per select, lanes over c with a carried warp scan.
  for (int sel = warp; sel < p.nsel; sel += kSWarps) {
    const int2* cj = p.cnt + ((size_t)ji.job * kMaxSel + sel) * p.cpj;
    const long long need = (long long)s_rem[sel];
    long long carry_eq = 0, base = 0;
    for (int c0 = 0; c0 < ji.part; c0 += 32) {
      const int c = c0 + lane;
      const int2 v = c < ji.part ? cj[c] : make_int2(0, 0);
      int incl = v.y;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      long long eqsel = need - (carry_eq + incl - v.y);
      eqsel = eqsel < 0 ? 0 : (eqsel > v.y ? v.y : eqsel);
      int contrib = v.x + (int)eqsel;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) contrib += __shfl_xor_sync(0xffffffffu, contrib, o);
      carry_eq += __shfl_sync(0xffffffffu, incl, 31);
      base += contrib;
    }
    if (lane == 0) {
      s_base[sel] = (int)base;
      s_eqoff[sel] = (int)min(carry_eq, (long long)0x7fffffff);
    }
  }
  __syncthreads();

  // ---- phase 5: epilogues
  // Walk this warp's slice in position order; for select `sel` every lane
  // gets its token (or -1 past the slice) and its rank (or -1).  Warp-uniform.
  auto rank_pass = [&](int sel, auto&& fn) {
    const unsigned int thr = s_prefix[sel];
    const long long need = (long long)s_rem[sel];
    const unsigned int* kr = keys + s_sel_row[sel] * p.T;
    long long run_eq = s_eqoff[sel];
    int run_sel = s_base[sel];
    for (int w = 0; w < warp; ++w) {  // warps before this one in the CTA
      const int2 v = s_wcnt[sel][w];
      long long e = need - run_eq;
      e = e < 0 ? 0 : (e > v.y ? v.y : e);
      run_sel += v.x + (int)e;
      run_eq += v.y;
    }
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
    long long run_eq = s_eqoff[sel];
    int run_sel = s_base[sel];
    for (int w = 0; w < warp; ++w) {
      const int2 v = s_wcnt[sel][w];
      long long e = need - run_eq;
      e = e < 0 ? 0 : (e > v.y ? v.y : e);
      run_sel += v.x + (int)e;
      run_eq += v.y;
    }
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
    const int kk = (int)s_k[0];
    const int row = ji.b * p.KV + ji.h;
    // flat slots from the row's first page (the row's prefill pages are contiguous)
    const int start = p.bt[(int64_t)row * p.max_blocks];
    const bool start_ok = start >= 0 && (int64_t)start * kPage + kk <= (int64_t)p.n_blocks * kPage;
    if (!start_ok && kk > 0 && threadIdx.x == 0 && ji.part == 0) set_err(p.err, HC_ERR_RANGE);
    const T* kbase = reinterpret_cast<const T*>(p.k) + ji.b * p.ksb + (int64_t)ji.h * p.ksh;
    const T* vbase = reinterpret_cast<const T*>(p.v) + ji.b * p.vsb + (int64_t)ji.h * p.vsh;
    T* kdst = reinterpret_cast<T*>(p.k_pool_out) + (int64_t)start * kPage * kD;
    T* vdst = reinterpret_cast<T*>(p.v_pool_out) + (int64_t)start * kPage * kD;
    constexpr int CH = kD * (int)sizeof(T) / 16;  // 16-byte chunks per row
    constexpr int PER = (2 * CH + 31) / 32;        // chunks per lane per token (K and V)
    rank_walk(0, [&](int c, unsigned int selm, int r0) {
      if (p.out_indices && ((selm >> lane) & 1u)) {
        const int rank = r0 + __popc(selm & lt_mask);
        if (rank < kk) p.out_indices[(size_t)ji.job * p.max_keep + rank] = ji.t0 + c + lane;
      }
      if (!start_ok) return;
      // warp-cooperative row copies, 4 tokens in flight
      unsigned int m = selm;
      int r = r0;
      while (m) {
        int tt[4], rr[4];
        int nb = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          tt[q] = -1;
          rr[q] = kk;
          if (m) {
            const int j = __ffs(m) - 1;
            m &= m - 1;
            tt[q] = ji.t0 + c + j;
            rr[q] = r++;
            ++nb;
          }
        }
        uint4 buf[4][PER];
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int e = 0; e < PER; ++e) {
            const int x = lane + 32 * e;
            if (q < nb && rr[q] < kk && x < 2 * CH) {
              const T* src = x < CH ? kbase + (int64_t)tt[q] * p.kst : vbase + (int64_t)tt[q] * p.vst;
              buf[q][e] = ldg128(reinterpret_cast<const uint4*>(src) + (x % CH));
            }
          }
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int e = 0; e < PER; ++e) {
            const int x = lane + 32 * e;
            if (q < nb && rr[q] < kk && x < 2 * CH) {
              T* dst = (x < CH ? kdst : vdst) + (int64_t)rr[q] * kD;
              reinterpret_cast<uint4*>(dst)[x % CH] = buf[q][e];
            }
          }
      }
    });
    if (ji.part == 0 && threadIdx.x == 0) p.heads_len[row] = kk;
    if (p.out_indices && ji.part == p.cpj - 1) {
      for (int i = kk + threadIdx.x; i < p.max_keep; i += kSThreads)
        p.out_indices[(size_t)ji.job * p.max_keep + i] = -1;
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
    const int slot = p.ref_slots[ji.job];
    uint32_t* bm = p.ref_bitmap + (size_t)slot * p.bitmap_words;
    if (threadIdx.x < kMaxRows) s_ov[threadIdx.x] = 0u;
    // this CTA's words of the reference bitmap, staged in shared memory
    const int wbeg = ji.t0 >> 5, nwords = ((ji.t1 + 31) >> 5) - wbeg;
    const bool staged = nwords <= kRefWords;
    if (staged)
      for (int w = threadIdx.x; w < nwords; w += kSThreads) s_refw[w] = bm[wbeg + w];
    __syncthreads();
    for (int sel = 0; sel < p.S; ++sel) {
      const int kk = (int)s_k[sel];
      unsigned int local = 0;
      rank_pass(sel, [&](int t, int rank, int) {
        if (rank >= 0 && rank < kk) {
          const uint32_t word = staged ? s_refw[(t >> 5) - wbeg] : bm[t >> 5];
          local += (word >> (t & 31)) & 1u;
        }
      });
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
      if (lane == 0 && local) atomicAdd(&s_ov[sel], local);
    }
    // retrieval list: last step's top-max_len, ascending
    {
      const int sel = p.S;
      const int kk = min((int)s_k[sel], p.max_len_cap);
      rank_pass(sel, [&](int t, int rank, int) {
        if (rank >= 0 && rank < kk) p.retrieve_positions[(size_t)ji.job * p.max_len_cap + rank] = t;
      });
    }
    __syncthreads();
    if (threadIdx.x < p.S && s_ov[threadIdx.x])
      atomicAdd(&p.overlap[ji.job * kMaxRows + threadIdx.x], s_ov[threadIdx.x]);
    if (!grid_sync(p.gb, nblocks, epoch, p.err)) return;
    if (threadIdx.x == 0) {
      float c[kMaxRows];
      const float kf = (float)p.topk;
      for (int s = 0; s < p.S; ++s) c[s] = __fdiv_rn((float)p.overlap[ji.job * kMaxRows + s], kf);
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
        p.trigger[ji.job] = trig;
        if (p.coeffs) for (int s = 0; s < p.S; ++s) p.coeffs[ji.job * p.S + s] = c[s];
        if (p.median) p.median[ji.job] = med;
      }
    }
    __syncthreads();
    if (s_trigger) {
      const int sel = p.S - 1;
      const int kk = (int)s_k[sel];
      rank_pass(sel, [&](int t, int rank, int c) {
        const bool on = rank >= 0 && rank < kk;
        if (on) p.ref_positions[(size_t)slot * p.topk + rank] = t;
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
};

static int g_num_sms = 0;

static int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

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

static bool uses_fma(int dtype, int Rq) { return dtype == HC_F32 || Rq > 40; }

static size_t elem_size(int dtype) { return dtype == HC_F32 ? 4 : 2; }

// Plan the partition: as many CTAs per job as fit co-resident (2 per SM by
// default), token ranges a multiple of 32 (bitmap words stay CTA-private).
static ScorePlan plan_score(int dtype, int n_jobs, int L, int Rq, int S, int ctas_per_sm) {
  ScorePlan pl;
  const int max_ctas = num_sms() * ctas_per_sm;
  int cpj = max(1, max_ctas / max(n_jobs, 1));
  cpj = min(cpj, (L + 31) / 32);
  int T_ = ((L + cpj - 1) / cpj + 31) / 32 * 32;
  cpj = (L + T_ - 1) / T_;
  pl.cpj = cpj;
  pl.T = T_;
  pl.TB = T_ + 2 * kMargin;
  pl.grid = cpj * n_jobs;
  const bool fma = uses_fma(dtype, Rq);
  const size_t es = elem_size(dtype);
  size_t with = (size_t)Rq * pl.TB * es;
  size_t rest = smem_bytes<float>(Rq, S, T_, pl.TB, false, fma);
  pl.logits_in_smem = (with + rest + 64) <= 200 * 1024;
  pl.smem = rest + (pl.logits_in_smem ? ((with + 15) & ~(size_t)15) : 0);
  pl.logits_bytes = pl.logits_in_smem ? 0 : (size_t)pl.grid * Rq * pl.TB * es;
  return pl;
}

struct ScoreWs {
  size_t off_gb, off_part, off_hist, off_cnt, off_overlap, off_logits, total;
};

static ScoreWs score_ws_layout(int n_jobs, const ScorePlan& pl, int Rq) {
  ScoreWs w;
  size_t o = 0;
  auto take = [&](size_t n) { size_t r = o; o += (n + 255) & ~(size_t)255; return r; };
  w.off_gb = take(sizeof(GridBarrier));
  w.off_part = take((size_t)n_jobs * pl.cpj * Rq * sizeof(float2));
  w.off_hist = take((size_t)n_jobs * kMaxSel * 4 * 256 * sizeof(unsigned int));
  w.off_cnt = take((size_t)n_jobs * kMaxSel * pl.cpj * sizeof(int2));
  w.off_overlap = take((size_t)n_jobs * kMaxRows * sizeof(unsigned int));
  w.off_logits = take(pl.logits_bytes);
  w.total = o;
  return w;
}

template <typename T>
static int launch_score(ScoreParams& p, const ScorePlan& pl, void* ws, size_t ws_bytes, cudaStream_t st) {
  ScoreWs w = score_ws_layout(p.n_jobs, pl, p.Rq);
  if (!ws || ws_bytes < w.total) return HC_ERR_WORKSPACE;
  unsigned char* base = reinterpret_cast<unsigned char*>(ws);
  p.gb = reinterpret_cast<GridBarrier*>(base + w.off_gb);
  p.part = reinterpret_cast<float2*>(base + w.off_part);
  p.hist = reinterpret_cast<unsigned int*>(base + w.off_hist);
  p.cnt = reinterpret_cast<int2*>(base + w.off_cnt);
  p.overlap = reinterpret_cast<unsigned int*>(base + w.off_overlap);
  p.glogits = pl.logits_in_smem ? nullptr : (void*)(base + w.off_logits);
  p.logits_in_smem = pl.logits_in_smem ? 1 : 0;
  p.cpj = pl.cpj;
  p.T = pl.T;
  p.TB = pl.TB;
  auto kern = score_select_kernel<T>;
  // Attribute and occupancy queries are made once per shared-memory size and
  // cached, so a launch issues no non-stream CUDA call (graph capture safe
  // after the first launch of a given shape).
  static bool attr_set = false;
  static int cache_smem[16], cache_occ[16], n_cache = 0;
  if (!attr_set) {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return HC_ERR_CUDA;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)fa.sharedSizeBytes) != cudaSuccess)
      return HC_ERR_CUDA;
    attr_set = true;
  }
  int occ = -1;
  for (int i = 0; i < n_cache; ++i)
    if (cache_smem[i] == (int)pl.smem) occ = cache_occ[i];
  if (occ < 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kSThreads, pl.smem) != cudaSuccess)
      return HC_ERR_CUDA;
    if (n_cache < 16) {
      cache_smem[n_cache] = (int)pl.smem;
      cache_occ[n_cache] = occ;
      ++n_cache;
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
  if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return HC_ERR_CUDA;
  return HC_OK;
}

template <typename T>
static int run_score(ScoreParams& p, void* ws, size_t ws_bytes, cudaStream_t st) {
  // one 512-thread CTA per SM
  ScorePlan pl = plan_score(std::is_same<T, float>::value ? HC_F32 : HC_BF16, p.n_jobs, p.L, p.Rq, p.S, 1);
  return launch_score<T>(p, pl, ws, ws_bytes, st);
}

size_t score_workspace_size(int dtype, int n_jobs, int L, int Rq, int S) {
  ScorePlan pl = plan_score(dtype, n_jobs, L, Rq, S, 1);
  return score_ws_layout(n_jobs, pl, Rq).total;
}

int score_dispatch(int dtype, ScoreParams& p, void* ws, size_t ws_bytes, cudaStream_t st) {
  switch (dtype) {
    case HC_F32: return run_score<float>(p, ws, ws_bytes, st);
    case HC_BF16: return run_score<__nv_bfloat16>(p, ws, ws_bytes, st);
    case HC_F16: return run_score<__half>(p, ws, ws_bytes, st);
    default: return HC_ERR_DTYPE;
  }
}

}  // namespace hc
