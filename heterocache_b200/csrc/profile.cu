// Offline head profiler (tools/get_cluster.py): the top-k positions of each
// head's last-query attention row as a bitmap, and intersection counts of
// such bitmaps.  The host side (classification, star clustering, allocation)
// is heterocache_b200/profiler.py.
//
// get_head_topk_exact (tools/get_cluster.py:13-60), per (batch row, head):
//   row  = attn[b, h, -1, :use_len]; with GQA dumps (all query heads saved)
//          the mean over the head's G query heads, in the dump's dtype
//          (fp32 sum in head order, divided by G, rounded to the dtype)
//   pool = avg_pool1d(row.float(), k = min(5, use_len), padding = k // 2,
//          stride 1, count_include_pad): ((((x0 + x1) + x2) + x3) + x4) / k
//   set  = topk(pool, min(topk, len(pool)))
// Equal pooled values at the k-th place go to the lowest positions (torch's
// topk leaves the order of equal values unspecified).
#include "hc_host.cuh"
#include "hc_params.cuh"

namespace hc {

constexpr int kPThreads = 512;
constexpr int kPWarps = kPThreads / 32;

// fp32 -> uint32 with the same order
__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct ProfileParams {
  const void* attn;
  int64_t sb, sh, sq, st;
  int q_last;     // query row read (the last)
  int He, G;      // effective heads, query heads averaged per effective head
  int use_len;    // positions of the row used
  int ksz, pad;   // pooling kernel size and padding
  int plen;       // pooled length
  int k;          // top-k size (<= plen)
  uint32_t* bits; // [rows][words]
  int64_t words;
  uint32_t* keys; // workspace: [rows][plen]
};

// The row value at position i (0 outside [0, use_len)): the head's own value
// or the dtype-rounded mean over its group.
template <typename T>
__device__ __forceinline__ float row_value(const ProfileParams& p, const T* base, int i) {
  if (i < 0 || i >= p.use_len) return 0.f;
  const T* x = base + (int64_t)i * p.st;
  if (p.G == 1) return Elem<T>::to_f(x[0]);
  float s = Elem<T>::to_f(x[0]);
  for (int g = 1; g < p.G; ++g) s += Elem<T>::to_f(x[(int64_t)g * p.sh]);
  return Elem<T>::rnd(__fdiv_rn(s, (float)p.G));
}

// One CTA per (batch row, effective head): pooled keys, a 4-round radix
// select of the k-th largest, then the bitmap, one 32-position word per warp
// and step.
template <typename T>
__global__ void __launch_bounds__(kPThreads) profile_topk_kernel(const ProfileParams p) {
  const int row = blockIdx.x;
  const int b = row / p.He, h = row % p.He;
  const T* base = reinterpret_cast<const T*>(p.attn) + (int64_t)b * p.sb + (int64_t)h * p.G * p.sh +
                  (int64_t)p.q_last * p.sq;
  uint32_t* keys = p.keys + (int64_t)row * p.plen;
  uint32_t* bits = p.bits + (int64_t)row * p.words;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ unsigned int hist[256];
  __shared__ unsigned int s_sel[2];  // threshold key, equal keys still to take
  __shared__ unsigned int s_wcnt[kPWarps];

  // ---- pooled keys (the window summed in order, zeros outside the row)
  for (int t = threadIdx.x; t < p.plen; t += kPThreads) {
    float s = 0.f;
    for (int j = 0; j < p.ksz; ++j) s += row_value<T>(p, base, t - p.pad + j);
    keys[t] = order_key(__fdiv_rn(s, (float)p.ksz));
  }
  __syncthreads();

  // ---- radix select: the k-th largest key, 8 bits a round from the top
  unsigned int prefix = 0u, mask = 0u, rem = (unsigned int)p.k;
  if (p.k > 0) {
    for (int r = 0; r < 4; ++r) {
      const int shift = 24 - 8 * r;
      for (int i = threadIdx.x; i < 256; i += kPThreads) hist[i] = 0u;
      __syncthreads();
      for (int t = threadIdx.x; t < p.plen; t += kPThreads) {
        const uint32_t key = keys[t];
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (warp == 0) {
        // lane l holds bins 8l .. 8l+7; suffix sums over lanes from the top
        unsigned int c[8], tot = 0u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          c[i] = hist[lane * 8 + i];
          tot += c[i];
        }
        unsigned int suf = tot;  // keys in bins >= 8 * lane
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned int y = __shfl_down_sync(0xffffffffu, suf, o);
          if (lane + o < 32) suf += y;
        }
        const unsigned int above_lane = suf - tot;  // keys in bins above this lane's
        // the lane whose bins hold the rem-th largest: above_lane < rem <= suf
        const bool mine = above_lane < rem && rem <= suf;
        const unsigned int who = __ballot_sync(0xffffffffu, mine);
        if (mine && lane == __ffs(who) - 1) {
          unsigned int above = above_lane;
          int bin = lane * 8 + 7;
          for (; bin > lane * 8; --bin) {
            if (above + c[bin - lane * 8] >= rem) break;
            above += c[bin - lane * 8];
          }
          s_sel[0] = (unsigned int)bin;
          s_sel[1] = rem - above;
        }
      }
      __syncthreads();
      prefix |= s_sel[0] << shift;
      mask |= 255u << shift;
      rem = s_sel[1];
      __syncthreads();
    }
  }
  const uint32_t thr = prefix;
  const unsigned int need = rem;  // keys equal to thr to take (lowest positions first)

  // ---- bitmap: key > thr, or equal and among the first `need` equal ones
  unsigned int eq_before = 0u;  // equal keys at earlier positions (same in every thread)
  for (int64_t w0 = 0; w0 < p.words; w0 += kPWarps) {
    const int64_t w = w0 + warp;
    const int64_t t = w * 32 + lane;
    const bool in = p.k > 0 && w < p.words && t < p.plen;
    const uint32_t key = in ? keys[t] : 0u;
    const unsigned int gt = __ballot_sync(0xffffffffu, in && key > thr);
    const unsigned int eq = __ballot_sync(0xffffffffu, in && key == thr);
    if (lane == 0) s_wcnt[warp] = __popc(eq);
    __syncthreads();
    unsigned int before = eq_before;
    for (int i = 0; i < warp; ++i) before += s_wcnt[i];
    const unsigned int rank = before + __popc(eq & ((1u << lane) - 1u));
    const unsigned int sel = __ballot_sync(0xffffffffu, ((eq >> lane) & 1u) && rank < need);
    if (lane == 0 && w < p.words) bits[w] = gt | sel;
    for (int i = 0; i < kPWarps; ++i) eq_before += s_wcnt[i];
    __syncthreads();
  }
}

// counts[p] = popcount(a[i] & b[j]) over `words` words: all (i, j) pairs, p =
// i * nb + j, or (diagonal) i == j, p = i.  One warp per pair.
__global__ void __launch_bounds__(256) profile_overlap_kernel(const uint32_t* __restrict__ a, int64_t as,
                                                              int na, const uint32_t* __restrict__ b, int64_t bs,
                                                              int nb, int64_t words, int diagonal,
                                                              int32_t* __restrict__ counts) {
  const int lane = threadIdx.x & 31;
  const int64_t pair = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t npairs = diagonal ? (int64_t)na : (int64_t)na * nb;
  if (pair >= npairs) return;
  const int64_t i = diagonal ? pair : pair / nb, j = diagonal ? pair : pair % nb;
  const uint32_t* x = a + i * as;
  const uint32_t* y = b + j * bs;
  int c = 0;
  for (int64_t w = lane; w < words; w += 32) c += __popc(__ldg(x + w) & __ldg(y + w));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if (lane == 0) counts[pair] = c;
}

size_t profile_topk_ws_bytes(int rows, int plen) { return (size_t)rows * (size_t)max(plen, 1) * sizeof(uint32_t); }

int profile_topk_dispatch(int dtype, const void* attn, int64_t sb, int64_t sh, int64_t sq, int64_t st, int q_last,
                          int bsz, int He, int G, int use_len, int topk, uint32_t* bits, int64_t words, void* ws,
                          size_t ws_bytes, cudaStream_t s) {
  ProfileParams p;
  p.attn = attn;
  p.sb = sb;
  p.sh = sh;
  p.sq = sq;
  p.st = st;
  p.q_last = q_last;
  p.He = He;
  p.G = G;
  p.use_len = use_len;
  p.ksz = min(5, use_len);
  p.pad = p.ksz / 2;
  p.plen = use_len + 2 * p.pad - p.ksz + 1;
  p.k = min(topk, p.plen);
  p.bits = bits;
  p.words = words;
  const int rows = bsz * He;
  if (ws_bytes < profile_topk_ws_bytes(rows, p.plen) || !ws) return HC_ERR_WORKSPACE;
  p.keys = reinterpret_cast<uint32_t*>(ws);
  switch (dtype) {
    case HC_F32: profile_topk_kernel<float><<<rows, kPThreads, 0, s>>>(p); break;
    case HC_F16: profile_topk_kernel<__half><<<rows, kPThreads, 0, s>>>(p); break;
    case HC_BF16: profile_topk_kernel<__nv_bfloat16><<<rows, kPThreads, 0, s>>>(p); break;
    default: return HC_ERR_DTYPE;
  }
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

int profile_overlap_dispatch(const uint32_t* a, int64_t as, int na, const uint32_t* b, int64_t bs, int nb,
                             int64_t words, int diagonal, int32_t* counts, cudaStream_t s) {
  const int64_t npairs = diagonal ? (int64_t)na : (int64_t)na * nb;
  if (npairs == 0) return HC_OK;
  const int64_t blocks = (npairs + 7) / 8;
  if (blocks > 0x7fffffff) return HC_ERR_INVALID;
  profile_overlap_kernel<<<(unsigned int)blocks, 256, 0, s>>>(a, as, na, b, bs, nb, words, diagonal, counts);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

}  // namespace hc
