// Split-K paged flash-decode over ragged per-(batch, KV head) lengths.
//
// Replaces flash_attn_with_kvcache(q[bsz*KV, 1, G, D], k_pool, v_pool,
// cache_seqlens=heads_len, block_table, causal=False) as called by the
// patched attention (heterocache/llama_model.py:370-397,
// heterocache/qwen_model.py:181-206).
//
// Work split: every row's length is padded to a multiple of 16 and the rows
// are laid end to end; the grid (a fixed number of CTAs per SM) cuts that
// flattened token space into equal spans, so every CTA streams the same
// number of KV bytes whatever the per-head budgets are.  A CTA's span covers
// one or more row pieces; per piece the 4 warps take 16-token groups (a group
// never crosses a 256-token page), keep an online softmax per query head,
// and are merged in shared memory into one partial (m, l, o[G][D]) stored at
// slot (cta + row).  A second kernel merges each row's partials.
//
// Per 16-token group a warp issues 8 x 16-byte key loads and 16 x 8-byte
// value loads per lane (coalesced 256-byte rows), computes q.K^T for the G
// query heads with two m16n8k16 MMAs per 16 dims (queries on M, padded to 16;
// tokens on N), and accumulates P.V on the CUDA cores with each lane owning 4
// of the 128 output dims.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <utility>

#include "hc_host.cuh"
#include "hc_params.cuh"
#include "umma.cuh"

namespace hc {



// Padded prefix of row lengths into s_start[0..R]; returns total.
__device__ __forceinline__ int row_prefix(const FDParams& p, int* s_start, int* s_warp, int* s_len = nullptr) {
  int carry = 0;
  for (int c0 = 0; c0 < p.R; c0 += blockDim.x) {
    int r = c0 + threadIdx.x;
    int len = r < p.R ? p.heads_len[r] : 0;
    len = len < 0 ? 0 : len;
    if (s_len && r < p.R) s_len[r] = len;
    int l16 = (len + p.gran - 1) / p.gran * p.gran;
    int tot;
    int ex = block_exclusive_scan(l16, s_warp, tot);
    if (r < p.R) s_start[r] = carry + ex;
    carry += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) s_start[p.R] = carry;
  __syncthreads();
  return carry;
}

__device__ __forceinline__ int span_of(int total, int nctas, int gran) {
  int s = (total + nctas - 1) / nctas;
  return (s + gran - 1) / gran * gran;
}

template <typename T>
struct WarpState {
  float m, l;           // for query head gid (identical across the 4 lanes of a gid)
  float o[kGMax][4];    // dims 4*lane .. 4*lane+3 for every query head
};

template <typename T>
__device__ __forceinline__ void fd_group_compute(const FDParams& p, WarpState<T>& st, const uint32_t (&qa)[8][2],
                                                 const uint4 (&kf)[2][4], const uint2 (&vf)[16], int valid,
                                                 float* sp, float* sc);

// 16-bit dtypes: tensor-core q.K^T, loads from global memory.
template <typename T>
__device__ __forceinline__ void fd_group_mma(const FDParams& p, WarpState<T>& st, const uint32_t (&qa)[8][2],
                                             const T* kbase, const T* vbase, int valid, float* sp, float* sc) {
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  uint4 kf[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int s = 0; s < 4; ++s) kf[nt][s] = ld_stream128(kbase + (8 * nt + gid) * kD + 32 * s + 8 * tig);
  uint2 vf[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) vf[i] = ld_stream64(vbase + i * kD + 4 * lane);
  fd_group_compute<T>(p, st, qa, kf, vf, valid, sp, sc);
}

// The math of one 16-token group given its key fragments (kf: the lane's
// 16-byte slices of rows gid and gid+8, dims 32s+8tig..) and value slices
// (vf: dims 4*lane.. of the 16 rows).
template <typename T>
__device__ __forceinline__ void fd_group_compute(const FDParams& p, WarpState<T>& st, const uint32_t (&qa)[8][2],
                                                 const uint4 (&kf)[2][4], const uint2 (&vf)[16], int valid,
                                                 float* sp, float* sc) {
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  float acc[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
  for (int s = 0; s < 4; ++s)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      mma16816<T>(acc[nt], qa[2 * s][0], 0u, qa[2 * s][1], 0u, kf[nt][s].x, kf[nt][s].y);
      mma16816<T>(acc[nt], qa[2 * s + 1][0], 0u, qa[2 * s + 1][1], 0u, kf[nt][s].z, kf[nt][s].w);
    }
  float sv[4];
  float mx = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = 8 * nt + 2 * tig + e;
      float x = t < valid ? acc[nt][e] * p.scale_log2 : -INFINITY;
      sv[nt * 2 + e] = x;
      mx = fmaxf(mx, x);
    }
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  const float mnew = fmaxf(st.m, mx);
  const float corr = (mnew == -INFINITY) ? 1.f : exp2f(st.m - mnew);
  float rs = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float pv = (sv[i] == -INFINITY) ? 0.f : exp2f(sv[i] - mnew);
    sv[i] = pv;
    rs += pv;
  }
  rs += __shfl_xor_sync(0xffffffffu, rs, 1);
  rs += __shfl_xor_sync(0xffffffffu, rs, 2);
  st.l = st.l * corr + rs;
  st.m = mnew;
  if (gid < p.G) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sp[gid * 16 + 8 * nt + 2 * tig] = sv[nt * 2];
      sp[gid * 16 + 8 * nt + 2 * tig + 1] = sv[nt * 2 + 1];
    }
    if (tig == 0) sc[gid] = corr;
  }
  __syncwarp();
#pragma unroll
  for (int g = 0; g < kGMax; ++g) {
    if (g < p.G) {
      const float c = sc[g];
#pragma unroll
      for (int j = 0; j < 4; ++j) st.o[g][j] *= c;
    }
  }
#pragma unroll
  for (int i4 = 0; i4 < 16; i4 += 4) {
    float2 va[4], vb[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      va[j] = unpack2<T>(vf[i4 + j].x);
      vb[j] = unpack2<T>(vf[i4 + j].y);
    }
#pragma unroll
    for (int g = 0; g < kGMax; ++g) {
      if (g < p.G) {
        const float4 pv = *reinterpret_cast<const float4*>(&sp[g * 16 + i4]);
        const float pj[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          st.o[g][0] = fmaf(pj[j], va[j].x, st.o[g][0]);
          st.o[g][1] = fmaf(pj[j], va[j].y, st.o[g][1]);
          st.o[g][2] = fmaf(pj[j], vb[j].x, st.o[g][2]);
          st.o[g][3] = fmaf(pj[j], vb[j].y, st.o[g][3]);
        }
      }
    }
  }
  __syncwarp();
}

// fp32: lanes over dims, warp all-reduce per (query head, token).
__device__ __forceinline__ void fd_group_f32(const FDParams& p, WarpState<float>& st, const float (&qf)[kGMax][4],
                                             const float* kbase, const float* vbase, int valid, float (&mrow)[kGMax],
                                             float (&lrow)[kGMax]) {
  const int lane = threadIdx.x & 31;
  for (int i = 0; i < 16; ++i) {
    if (i >= valid) break;
    const float4 k4 = *reinterpret_cast<const float4*>(kbase + i * kD + 4 * lane);
    const float4 v4 = *reinterpret_cast<const float4*>(vbase + i * kD + 4 * lane);
#pragma unroll
    for (int g = 0; g < kGMax; ++g) {
      if (g >= p.G) continue;
      float s = qf[g][0] * k4.x + qf[g][1] * k4.y + qf[g][2] * k4.z + qf[g][3] * k4.w;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      s *= p.scale_log2;
      const float mnew = fmaxf(mrow[g], s);
      const float corr = exp2f(mrow[g] - mnew);
      const float pv = exp2f(s - mnew);
      lrow[g] = lrow[g] * corr + pv;
      mrow[g] = mnew;
      st.o[g][0] = st.o[g][0] * corr + pv * v4.x;
      st.o[g][1] = st.o[g][1] * corr + pv * v4.y;
      st.o[g][2] = st.o[g][2] * corr + pv * v4.z;
      st.o[g][3] = st.o[g][3] * corr + pv * v4.w;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kFThreads) flash_decode_kernel(FDParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int* s_start = reinterpret_cast<int*>(smem_raw);
  __shared__ int s_warp[32];
  __shared__ __align__(16) float s_p[kFWarps][kGMax * 16];
  __shared__ float s_c[kFWarps][kGMax];
  __shared__ float s_m[kFWarps][kGMax], s_l[kFWarps][kGMax];
  __shared__ float s_o[kFWarps][kGMax][kD];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  pdl_wait();  // as in the TMA kernel
  pdl_trigger();
  const int total = row_prefix(p, s_start, s_warp);
  const int span = span_of(total, gridDim.x, p.gran);
  const int beg = blockIdx.x * span;
  if (beg >= total) return;
  const int end = min(total, beg + span);
  // first row with s_start[r+1] > beg
  int lo = 0, hi = p.R - 1;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (s_start[mid + 1] > beg) hi = mid; else lo = mid + 1;
  }
  for (int r = lo; r < p.R && s_start[r] < end; ++r) {
    const int rs = s_start[r], re = s_start[r + 1];
    if (re <= beg || re == rs) continue;
    const int a = max(rs, beg) - rs, bnd = min(re, end) - rs;
    const int len = p.heads_len[r];
    const int b = r / p.KV, h = r % p.KV;
    const T* qrow0 = reinterpret_cast<const T*>(p.q) + b * p.qsb + (int64_t)(h * p.G) * p.qsh;

    WarpState<T> st;
    st.m = -INFINITY;
    st.l = 0.f;
#pragma unroll
    for (int g = 0; g < kGMax; ++g) st.o[g][0] = st.o[g][1] = st.o[g][2] = st.o[g][3] = 0.f;

    if constexpr (std::is_same<T, float>::value) {
      float qf[kGMax][4];
      float mrow[kGMax], lrow[kGMax];
#pragma unroll
      for (int g = 0; g < kGMax; ++g) {
        mrow[g] = -INFINITY;
        lrow[g] = 0.f;
        if (g < p.G) {
          float4 q4 = *reinterpret_cast<const float4*>(qrow0 + g * p.qsh + 4 * lane);
          qf[g][0] = q4.x; qf[g][1] = q4.y; qf[g][2] = q4.z; qf[g][3] = q4.w;
        } else {
          qf[g][0] = qf[g][1] = qf[g][2] = qf[g][3] = 0.f;
        }
      }
      for (int t16 = a + warp * 16; t16 < bnd; t16 += kFWarps * 16) {
        const int page = t16 >> 8;
        int blk = page < p.max_blocks ? p.bt[(int64_t)r * p.max_blocks + page] : -1;
        if (blk < 0 || blk >= p.n_blocks) { set_err(p.err, HC_ERR_RANGE); continue; }
        const int64_t off = ((int64_t)blk * kPage + (t16 & (kPage - 1))) * kD;
        fd_group_f32(p, st, qf, reinterpret_cast<const float*>(p.kp) + off,
                     reinterpret_cast<const float*>(p.vp) + off, min(16, len - t16), mrow, lrow);
      }
      if (lane == 0) {
        for (int g = 0; g < kGMax; ++g) { s_m[warp][g] = mrow[g]; s_l[warp][g] = lrow[g]; }
      }
    } else {
      uint32_t qa[8][2];
      const T* qg = qrow0 + (gid < p.G ? gid : 0) * p.qsh;
#pragma unroll
      for (int s = 0; s < 4; ++s)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          uint2 w = gid < p.G ? ldg64(qg + 32 * s + 8 * tig + 4 * u) : make_uint2(0u, 0u);
          qa[2 * s + u][0] = w.x;
          qa[2 * s + u][1] = w.y;
        }
      for (int t16 = a + warp * 16; t16 < bnd; t16 += kFWarps * 16) {
        const int page = t16 >> 8;
        int blk = page < p.max_blocks ? p.bt[(int64_t)r * p.max_blocks + page] : -1;
        if (blk < 0 || blk >= p.n_blocks) { set_err(p.err, HC_ERR_RANGE); continue; }
        const int64_t off = ((int64_t)blk * kPage + (t16 & (kPage - 1))) * kD;
        fd_group_mma<T>(p, st, qa, reinterpret_cast<const T*>(p.kp) + off, reinterpret_cast<const T*>(p.vp) + off,
                        min(16, len - t16), s_p[warp], s_c[warp]);
      }
      if (tig == 0 && gid < kGMax) {
        s_m[warp][gid] = st.m;
        s_l[warp][gid] = st.l;
      }
    }
#pragma unroll
    for (int g = 0; g < kGMax; ++g)
      if (g < p.G)
        *reinterpret_cast<float4*>(&s_o[warp][g][4 * lane]) = make_float4(st.o[g][0], st.o[g][1], st.o[g][2], st.o[g][3]);
    __syncthreads();
    // merge the 4 warps: thread d owns output dim d
    const int d = threadIdx.x;
    const int slot = blockIdx.x + r;
    for (int g = 0; g < p.G; ++g) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kFWarps; ++w) M = fmaxf(M, s_m[w][g]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kFWarps; ++w) {
        const float f = (s_m[w][g] == -INFINITY) ? 0.f : exp2f(s_m[w][g] - M);
        L += f * s_l[w][g];
        O += f * s_o[w][g][d];
      }
      p.part_o[((size_t)slot * p.G + g) * kD + d] = O;
      if (d == 0) p.part_ml[(size_t)slot * p.G + g] = make_float2(M, L);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Pipelined tensor-core variant for 16-bit pools.
//
// Rows are padded to 64 tokens and the flattened space is cut into 64-token
// tiles (a tile never crosses a page: 256 % 64 == 0).  Warp kTConsumers is the
// producer: one lane loads each tile with four TMA tensor copies (keys and
// values, dims 0-63 and 64-127, each a 64-row x 128-byte box with the 128-byte
// swizzle) into a ring of kTStages shared-memory stages, completion counted on
// the stage's "full" mbarrier.  Consumer warp w takes tokens 16w..16w+15 of a
// tile:
//   S  = Q K^T   m16n8k16, A = query rows (registers), B = key rows (ldmatrix)
//   O^T += V^T P^T  m16n8k16, A = value rows transposed (ldmatrix.trans),
//                 B = the probabilities straight from S's accumulators
// and releases the stage on its "empty" mbarrier.  The swizzle makes every
// ldmatrix conflict-free.  All waits are bounded; after a timeout a warp
// stops waiting but keeps the same control flow (so the consumers' named
// barriers still meet) and the producer waits, bounded, for the copies it
// issued before it exits.
constexpr int kTTile = 64;
constexpr int kTStages = 3;
constexpr int kTConsumers = 4;
constexpr int kTThreads = (kTConsumers + 1) * 32;
constexpr int kTBox = kTTile * 64 * 2;  // bytes of one 64-row x 64-element box

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// The K/V stream is read with the evict-first L2 policy (l2_evict_first_policy),
// through tma_load_2d (umma.cuh).
// Address of 16-byte chunk `chunk` (0..15 over the 128 dims) of tile row
// `row` (0..63), for a stage whose first box starts at `base` (1024-aligned).
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int chunk) {
  return base + (chunk >> 3) * kTBox + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct TcState {
  float m, l;       // query row gid (same on the 4 lanes of the row)
  float ot[8][4];   // O^T: dims 16mt+gid(+8), queries 2tig, 2tig+1
};

// One 16-token group; kst/vst = shared addresses of the stage's key/value
// boxes, tok0 = first tile row of the group, valid = tokens to use.
template <typename T>
__device__ __forceinline__ void fd_group_tc(const FDParams& p, TcState& st, const uint32_t (&qa)[8][2],
                                            uint32_t kst, uint32_t vst, int tok0, int valid) {
  const int lane = threadIdx.x & 31;
  const int tig = lane & 3;
  const int mi = lane >> 3, j = lane & 7;
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const int krow = tok0 + 8 * (mi >> 1) + j;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    uint32_t b[4];
    ldsm_x4(b, swz(kst, krow, 2 * ks + (mi & 1)));
    mma16816<T>(acc[0], qa[ks][0], 0u, qa[ks][1], 0u, b[0], b[1]);
    mma16816<T>(acc[1], qa[ks][0], 0u, qa[ks][1], 0u, b[2], b[3]);
  }
  float sv[4];
  float mx = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = 8 * nt + 2 * tig + e;
      const float x = t < valid ? acc[nt][e] * p.scale_log2 : -INFINITY;
      sv[nt * 2 + e] = x;
      mx = fmaxf(mx, x);
    }
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  const float mnew = fmaxf(st.m, mx);
  const float corr = (mnew == -INFINITY) ? 1.f : exp2f(st.m - mnew);
  float rs = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float pv = (sv[i] == -INFINITY) ? 0.f : exp2f(sv[i] - mnew);
    sv[i] = pv;
    rs += pv;
  }
  rs += __shfl_xor_sync(0xffffffffu, rs, 1);
  rs += __shfl_xor_sync(0xffffffffu, rs, 2);
  st.l = st.l * corr + rs;
  st.m = mnew;
  // rescale O^T columns (queries 2tig, 2tig+1) by their rows' corrections
  const float c0 = __shfl_sync(0xffffffffu, corr, 8 * tig);
  const float c1 = __shfl_sync(0xffffffffu, corr, 8 * tig + 4);
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    st.ot[mt][0] *= c0;
    st.ot[mt][1] *= c1;
    st.ot[mt][2] *= c0;
    st.ot[mt][3] *= c1;
  }
  // P^T as the B operand: tokens 2tig.. (n-tile 0) and 8+2tig.. (n-tile 1)
  const uint32_t b0 = pack2<T>(sv[0], sv[1]);
  const uint32_t b1 = pack2<T>(sv[2], sv[3]);
  const int vrow = tok0 + 8 * (mi >> 1) + j;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    uint32_t a[4];
    ldsm_x4_t(a, swz(vst, vrow, 2 * mt + (mi & 1)));
    // a[0]: dims 16mt..+7 x tokens 0-7, a[1]: dims +8.. x tokens 0-7,
    // a[2]: dims 16mt.. x tokens 8-15, a[3]: dims +8.. x tokens 8-15
    mma16816<T>(st.ot[mt], a[0], a[1], a[2], a[3], b0, b1);
  }
}

__host__ __device__ constexpr int fd_round4(int n) { return (n + 3) & ~3; }

// Dynamic shared memory of the TMA kernel: 1024 bytes of alignment slack,
// the stages, row starts and lengths, and the per-warp partial outputs.
__host__ __device__ constexpr size_t fd_tma_smem(int R, int G) {
  return 1024 + (size_t)kTStages * 4 * kTBox + (size_t)(fd_round4(R + 1) + fd_round4(R)) * sizeof(int) +
         (size_t)kTConsumers * G * kD * sizeof(float);
}

template <typename T>
__global__ void __launch_bounds__(kTThreads, 2)
    flash_decode_tma_kernel(FDParams p, const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv) {
  constexpr int kStageBytes = 4 * kTBox;  // K box 0, K box 1, V box 0, V box 1
  extern __shared__ __align__(16) unsigned char smem_dyn[];
  // the 128-byte swizzle pattern is taken from address bits 4-9: stages start
  // on a 1024-byte boundary (the launch reserves 1024 bytes of slack)
  unsigned char* smem_raw = smem_dyn + ((1024 - (smem_u32(smem_dyn) & 1023)) & 1023);
  unsigned char* stages = smem_raw;
  int* s_start = reinterpret_cast<int*>(smem_raw + (size_t)kTStages * kStageBytes);
  int* s_len = s_start + fd_round4(p.R + 1);
  float* s_ob = reinterpret_cast<float*>(s_len + fd_round4(p.R));
  auto s_o = [&](int w, int g) { return s_ob + ((size_t)w * p.G + g) * kD; };
  __shared__ __align__(8) uint64_t full_bar[kTStages], empty_bar[kTStages];
  __shared__ int s_tile_ok[kTStages];  // page id of the stage's tile was valid
  __shared__ int s_warp[32];
  __shared__ float s_m[kTConsumers][kGMax], s_l[kTConsumers][kGMax];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  // programmatic dependent launch: wait for the kernel before (the page
  // append) to finish, then let the combine get resident; it reads row
  // lengths before its own wait and waits for this grid's partials
  pdl_wait();
  pdl_trigger();
  const int total = row_prefix(p, s_start, s_warp, s_len);
  const int span = span_of(total, gridDim.x, kTTile);
  const int beg = blockIdx.x * span;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kTConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (beg >= total) return;
  const int end = min(total, beg + span);
  const int ntiles = (end - beg) / kTTile;
  int r0 = 0, hi = p.R - 1;  // first row with s_start[r+1] > beg
  while (r0 < hi) {
    const int mid = (r0 + hi) >> 1;
    if (s_start[mid + 1] > beg) hi = mid; else r0 = mid + 1;
  }

  if (warp == kTConsumers) {
    // ---- producer
    if (lane == 0) {
      int r = r0, issued = 0;
      bool dead = false;
      const uint64_t pol = l2_evict_first_policy();
      for (int i = 0; i < ntiles; ++i) {
        const int s = i % kTStages;
        if (!mbar_wait(&empty_bar[s], ((i / kTStages) & 1) ^ 1, p.wait_ns)) {
          set_err(p.err, HC_ERR_TIMEOUT);
          dead = true;
          break;
        }
        const int tok = beg + i * kTTile;
        while (s_start[r + 1] <= tok) ++r;
        const int t = tok - s_start[r];
        const int page = t >> 8;
        const int blk = page < p.max_blocks ? p.bt[(int64_t)r * p.max_blocks + page] : -1;
        if (blk < 0 || blk >= p.n_blocks) {  // consumers skip this tile
          set_err(p.err, HC_ERR_RANGE);
          s_tile_ok[s] = 0;
          mbar_arrive(&full_bar[s]);  // release: orders the flag before the consumers' wait
          continue;
        }
        s_tile_ok[s] = 1;
        const int y = blk * kPage + (t & (kPage - 1));
        unsigned char* dst = stages + (size_t)s * kStageBytes;
        mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
        tma_load_2d(dst, &tmk, 0, y, &full_bar[s], pol);
        tma_load_2d(dst + kTBox, &tmk, 64, y, &full_bar[s], pol);
        tma_load_2d(dst + 2 * kTBox, &tmv, 0, y, &full_bar[s], pol);
        tma_load_2d(dst + 3 * kTBox, &tmv, 64, y, &full_bar[s], pol);
        issued = i + 1;
      }
      if (dead) {  // let the copies this CTA issued land before it exits
        for (int i = max(0, issued - kTStages); i < issued; ++i)
          (void)mbar_wait(&full_bar[i % kTStages], (i / kTStages) & 1, p.wait_ns);
      }
    }
    return;
  }

  // ---- consumers
  TcState st;
  uint32_t qa[8][2];
  int cur = -1;
  bool dead = false;
  auto reset_state = [&]() {
    st.m = -INFINITY;
    st.l = 0.f;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) st.ot[mt][0] = st.ot[mt][1] = st.ot[mt][2] = st.ot[mt][3] = 0.f;
  };
  auto load_q = [&](int r) {
    const int b = r / p.KV, h = r % p.KV;
    const T* qg = reinterpret_cast<const T*>(p.q) + b * p.qsb + (int64_t)(h * p.G + (gid < p.G ? gid : 0)) * p.qsh;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = gid < p.G ? __ldg(reinterpret_cast<const uint32_t*>(qg + 16 * ks + 2 * tig)) : 0u;
      qa[ks][1] = gid < p.G ? __ldg(reinterpret_cast<const uint32_t*>(qg + 16 * ks + 8 + 2 * tig)) : 0u;
    }
  };
  // merge the consumer warps' states of row r into partial slot (cta + r)
  auto flush = [&](int r) {
    if (tig == 0 && gid < kGMax) {
      s_m[warp][gid] = st.m;
      s_l[warp][gid] = st.l;
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = 2 * tig + (e & 1);
        const int d = 16 * mt + gid + 8 * (e >> 1);
        if (q < p.G) s_o(warp, q)[d] = st.ot[mt][e];
      }
    named_bar_sync(1, kTConsumers * 32);
    const int slot = blockIdx.x + r;
    for (int e = threadIdx.x; e < p.G * kD; e += kTConsumers * 32) {
      const int g = e / kD, d = e % kD;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kTConsumers; ++w) M = fmaxf(M, s_m[w][g]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kTConsumers; ++w) {
        const float f = (s_m[w][g] == -INFINITY) ? 0.f : exp2f(s_m[w][g] - M);
        L += f * s_l[w][g];
        O += f * s_o(w, g)[d];
      }
      p.part_o[((size_t)slot * p.G + g) * kD + d] = O;
      if (d == 0) p.part_ml[(size_t)slot * p.G + g] = make_float2(M, L);
    }
    named_bar_sync(1, kTConsumers * 32);
  };

  int r = r0;
  for (int i = 0; i < ntiles; ++i) {
    const int s = i % kTStages;
    const int tok = beg + i * kTTile;
    while (s_start[r + 1] <= tok) ++r;
    if (r != cur) {
      if (cur >= 0) flush(cur);
      load_q(r);
      reset_state();
      cur = r;
    }
    if (!dead && !mbar_wait(&full_bar[s], (i / kTStages) & 1, p.wait_ns)) {
      if (lane == 0) set_err(p.err, HC_ERR_TIMEOUT);
      dead = true;
    }
    if (!dead) {
      const int t = tok - s_start[r];
      const int valid = s_tile_ok[s] ? min(16, s_len[r] - t - 16 * warp) : 0;
      if (valid > 0) {
        const uint32_t kst = smem_u32(stages + (size_t)s * kStageBytes);
        fd_group_tc<T>(p, st, qa, kst, kst + 2 * kTBox, 16 * warp, valid);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);
    }
  }
  if (cur >= 0) flush(cur);
}

// Merge of one (row, query head, 32-dim slice of the output): four CTAs per
// (row, query head), so that the merge after the decode kernel's last CTA is
// spread over 4 x R x G CTAs, each loading a quarter of every partial.  One
// load round: lanes in groups of 8 (one 16-byte quarter of the slice each)
// take a partial, 4 per warp and 8 warps, 4 deep: 128 partials (rows of up
// to 131072 tokens at the decode grid's spans); the partial's (m, l) comes
// with it (a broadcast load); then the block maximum, each thread rescales
// its own partials, and the 32 groups' sums are added in shared memory.
constexpr int kCThreads = 256;
constexpr int kCSlices = 4;
constexpr int kCSliceDims = kD / kCSlices;  // 32

template <typename T>
__global__ void __launch_bounds__(kCThreads) flash_combine_kernel(FDParams p, int nctas) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int* s_start = reinterpret_cast<int*>(smem_raw);
  // LG lanes per partial group (16 bytes of the slice each), GPW groups a warp
  constexpr int LG = kCSliceDims / 4, GPW = 32 / LG;
  constexpr int NW = kCThreads / 32, NG = NW * GPW, DEPTH = 128 / NG;
  __shared__ int s_warp[32];
  __shared__ float s_red[NW], s_redl[NW];
  __shared__ float s_mrun;  // running maximum over the rounds of 128 partials
  __shared__ float4 s_acc[NG][kCSliceDims / 4];
  const int total = row_prefix(p, s_start, s_warp);
  const int span = span_of(total, nctas, p.gran);
  const int rg = blockIdx.x / kCSlices, sl = blockIdx.x % kCSlices;
  const int r = rg / p.G, g = rg % p.G;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / LG, q4 = lane % LG;  // partial group within the warp, 16-byte piece of the slice
  const int d0 = kCSliceDims * sl;           // the slice's first dim
  T* out = reinterpret_cast<T*>(p.out) + ((size_t)r * p.G + g) * kD + d0;
  // the output element d of this slice, here and in the mirrors (peer GPUs'
  // gathered outputs, written over NVLink), then a system-scope fence so that
  // a later step barrier publishes them
  auto store = [&](int d, float x) {
    const T val = Elem<T>::from_f(x);
    out[d] = val;
    if (p.n_mirror > 0) {
      const int64_t off = (int64_t)(r / p.KV) * p.mirror_sb + ((int64_t)(r % p.KV) * p.G + g) * kD + d0 + d;
      for (int m = 0; m < p.n_mirror; ++m) reinterpret_cast<T*>(p.mirror[m])[off] = val;
      __threadfence_system();
    }
  };
  const int rs = s_start[r], re = s_start[r + 1];
  // the step's token not in the pages yet: its score (log2 domain) and value.
  // q and k_new come from before the decode kernel, which started after they
  // were complete, so they are read ahead of the wait.
  const bool has_new = p.k_new != nullptr;
  if (p.q_stage && threadIdx.x < kCSliceDims) {  // the query row into the drift-check buffer
    const int h = r % p.KV;
    const T* qrow = reinterpret_cast<const T*>(p.q) + (int64_t)(h * p.G + g) * p.qsh;
    reinterpret_cast<T*>(p.q_stage)[(int64_t)(h * p.G + g) * kD + d0 + threadIdx.x] = qrow[d0 + threadIdx.x];
  }
  float s_new = -INFINITY, v_new_d = 0.f;
  if (has_new) {
    const int b = r / p.KV, h = r % p.KV;
    const T* qrow = reinterpret_cast<const T*>(p.q) + b * p.qsb + (int64_t)(h * p.G + g) * p.qsh;
    const T* krow = reinterpret_cast<const T*>(p.k_new) + b * p.kn_sb + (int64_t)h * p.kn_sh;
    float prod = threadIdx.x < kD ? Elem<T>::to_f(qrow[threadIdx.x]) * Elem<T>::to_f(krow[threadIdx.x]) : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) prod += __shfl_xor_sync(0xffffffffu, prod, o);
    if (lane == 0) s_red[warp] = prod;
    __syncthreads();
    float dot = 0.f;
#pragma unroll
    for (int w = 0; w < kD / 32; ++w) dot += s_red[w];
    s_new = dot * p.scale_log2;
    if (threadIdx.x < kCSliceDims)
      v_new_d = Elem<T>::to_f(
          reinterpret_cast<const T*>(p.v_new)[b * p.vn_sb + (int64_t)h * p.vn_sh + d0 + threadIdx.x]);
    __syncthreads();
  }
  if (re == rs || span == 0) {  // no pages: the new token alone, or nothing
    if (threadIdx.x < kCSliceDims) store(threadIdx.x, has_new ? v_new_d : 0.f);
    return;
  }
  const int c0 = rs / span, n = (re - 1) / span - c0 + 1;
  const size_t slot0 = (size_t)(c0 + r);
  // the partials are written by the decode kernel launched just before
  pdl_wait();
  pdl_trigger();  // the next kernel may get resident; it waits for this grid
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float Lw = 0.f;
  for (int cb0 = 0; cb0 < n; cb0 += NG * DEPTH) {
    float4 o[DEPTH];
    float2 ml[DEPTH];
#pragma unroll
    for (int u = 0; u < DEPTH; ++u) {
      const int c = cb0 + (warp * GPW + sub) + u * NG;
      const bool ok = c < n;
      ml[u] = ok ? p.part_ml[(slot0 + c) * p.G + g] : make_float2(-INFINITY, 0.f);
      o[u] = ok ? *reinterpret_cast<const float4*>(p.part_o + ((slot0 + c) * p.G + g) * kD + d0 + 4 * q4)
                : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mw = -INFINITY;
#pragma unroll
    for (int u = 0; u < DEPTH; ++u) mw = fmaxf(mw, ml[u].x);
#pragma unroll
    for (int off = LG; off < 32; off <<= 1) mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, off));
    if (lane == 0) s_red[warp] = mw;
    __syncthreads();
    float M = cb0 == 0 ? s_new : s_mrun;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, s_red[w]);
    // rescale what earlier rounds accumulated (more than 128 partials only)
    if (cb0 > 0) {
      const float fo = (s_mrun == -INFINITY) ? 0.f : exp2f(s_mrun - M);
      acc.x *= fo; acc.y *= fo; acc.z *= fo; acc.w *= fo;
      Lw *= fo;
    }
#pragma unroll
    for (int u = 0; u < DEPTH; ++u) {
      const float f = (ml[u].x == -INFINITY) ? 0.f : exp2f(ml[u].x - M);
      Lw = fmaf(f, ml[u].y, Lw);
      acc.x = fmaf(f, o[u].x, acc.x);
      acc.y = fmaf(f, o[u].y, acc.y);
      acc.z = fmaf(f, o[u].z, acc.z);
      acc.w = fmaf(f, o[u].w, acc.w);
    }
    __syncthreads();  // every warp has read s_red and s_mrun
    if (threadIdx.x == 0) s_mrun = M;
  }
  __syncthreads();
  const float M = s_mrun;
  // the normaliser: every lane of a group holds its group's sum; one per group
#pragma unroll
  for (int off = LG; off < 32; off <<= 1) Lw += __shfl_xor_sync(0xffffffffu, Lw, off);
  if (lane == 0) s_redl[warp] = Lw;
  s_acc[warp * GPW + sub][q4] = acc;
  __syncthreads();
  const float f_new = has_new ? exp2f(s_new - M) : 0.f;  // the new token's weight (its l is 1)
  float L = f_new;
#pragma unroll
  for (int w = 0; w < NW; ++w) L += s_redl[w];
  if (threadIdx.x < kCSliceDims) {
    const int d = threadIdx.x;
    float O = f_new * v_new_d;
#pragma unroll
    for (int k = 0; k < NG; ++k) O += reinterpret_cast<const float*>(&s_acc[k][d / 4])[d % 4];
    store(d, L > 0.f ? O / L : 0.f);
  }
}

// ---------------------------------------------------------------------------
// Step barrier of a head-sharded cache's GPUs (the output mirrors above make
// the all-gather of head outputs part of the attention's combine).  One warp:
// lane 0 takes the next value of the rank's counter; lane q < world stores it
// into slot `rank` of rank q's flags (release, system scope: after the
// mirrored stores of earlier kernels), then lane q waits until slot q of this
// rank's flags reaches it (acquire).  Every wait is bounded: after the limit
// the lane ORs HC_ERR_TIMEOUT into err and returns.
__device__ __forceinline__ void st_release_sys(int32_t* a, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;\n" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* a) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];\n" : "=r"(v) : "l"(a) : "memory");
  return v;
}

struct PeerFlags {
  int32_t* f[kMaxPeers];
};

__global__ void __launch_bounds__(32) peer_barrier_kernel(int rank, int world, PeerFlags flags, int32_t* counter,
                                                          int32_t* err, uint64_t wait_ns) {
  const int lane = threadIdx.x;
  int32_t v = 0;
  if (lane == 0) {
    v = *counter + 1;
    *counter = v;
  }
  v = __shfl_sync(0xffffffffu, v, 0);
  __threadfence_system();
  if (lane < world) st_release_sys(flags.f[lane] + rank, v);
  if (lane < world && lane != rank) {
    const int32_t* mine = flags.f[rank] + lane;
    if (ld_acquire_sys(mine) < v) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(mine) < v) {
        if (globaltimer_ns() - t0 > wait_ns) {
          set_err(err, HC_ERR_TIMEOUT);
          return;
        }
        __nanosleep(64);
      }
    }
  }
}

int peer_barrier_dispatch(int rank, int world, int32_t* const* peer_flags, int32_t* counter, int32_t* err,
                          cudaStream_t st) {
  PeerFlags f;
  for (int i = 0; i < kMaxPeers; ++i) f.f[i] = i < world ? peer_flags[i] : nullptr;
  peer_barrier_kernel<<<1, 32, 0, st>>>(rank, world, f, counter, err, wait_limit_ns(kBarrierTimeoutNs));
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

// Concatenation of up to kMaxPutSegs int32 segments stored into up to
// kMaxPeers destinations (other ranks' buffers mapped through CUDA IPC):
// word i of the concatenation goes to dst[d][i] for every d.  Each thread
// fences its stores at system scope, so a peer barrier issued after this
// kernel on the same stream publishes them.
struct PutArgs {
  const int32_t* src[kMaxPutSegs];
  int64_t end[kMaxPutSegs];  // running word count through segment s
  int32_t* dst[kMaxPeers];
  int n_seg, n_dst;
};

__global__ void __launch_bounds__(256) peer_put_kernel(PutArgs a) {
  const int64_t total = a.end[a.n_seg - 1];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    int s = 0;
    while (i >= a.end[s]) ++s;  // n_seg <= kMaxPutSegs
    const int64_t j = i - (s ? a.end[s - 1] : 0);
    const int32_t w = a.src[s][j];
    for (int d = 0; d < a.n_dst; ++d) a.dst[d][i] = w;
  }
  __threadfence_system();
}

int peer_put_dispatch(int n_seg, const int32_t* const* srcs, const int64_t* seg_words, int n_dst,
                      int32_t* const* dsts, cudaStream_t st) {
  PutArgs a;
  std::memset(&a, 0, sizeof(a));
  int64_t run = 0;
  for (int s = 0; s < n_seg; ++s) {
    a.src[s] = srcs[s];
    run += seg_words[s];
    a.end[s] = run;
  }
  for (int d = 0; d < n_dst; ++d) a.dst[d] = dsts[d];
  a.n_seg = n_seg;
  a.n_dst = n_dst;
  if (run == 0 || n_dst == 0) return HC_OK;
  const int64_t blocks = (run + 255) / 256;
  const int grid = (int)(blocks < 64 ? blocks : 64);
  peer_put_kernel<<<grid, 256, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

// Co-resident CTAs of the fp32 decode kernel on the current device (cached
// per device).
static int fd_grid(int dtype) {
  static int cached[kMaxDevices][3];
  const int dev = current_device();
  if (dev < 0) return 0;
  {
    std::lock_guard<std::mutex> g(host_lock());
    if (cached[dev][dtype]) return cached[dev][dtype];
  }
  const int sms = device_sms(dev);
  int occ = 0;
  size_t dsm = (kMaxRowsFD + 1) * sizeof(int);
  switch (dtype) {
    case HC_F32: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, flash_decode_kernel<float>, kFThreads, dsm); break;
    case HC_BF16: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, flash_decode_kernel<__nv_bfloat16>, kFThreads, dsm); break;
    default: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, flash_decode_kernel<__half>, kFThreads, dsm); break;
  }
  if (occ <= 0) occ = 1;
  std::lock_guard<std::mutex> g(host_lock());
  cached[dev][dtype] = sms * occ;
  return cached[dev][dtype];
}

size_t flash_decode_ws_bytes(int R, int G) {
  const size_t slots = (size_t)148 * 32 + R;
  return slots * G * kD * sizeof(float) + slots * G * sizeof(float2) + 256;
}

template <typename T>
static int fd_combine(FDParams& p, int grid, cudaStream_t st) {
  // launched as a programmatic dependent of the decode kernel: its CTAs may
  // start early and wait (griddepcontrol.wait) for the partials
  const size_t csm = (((size_t)(p.R + 1) * sizeof(int) + 15) & ~(size_t)15);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.R * p.G * kCSlices);
  cfg.blockDim = dim3(kCThreads);
  cfg.dynamicSmemBytes = csm;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, flash_combine_kernel<T>, p, grid) != cudaSuccess) return HC_ERR_CUDA;
  return HC_OK;
}

// Launch with programmatic stream serialization: the grid may start while the
// previous kernel in the stream drains; every kernel launched this way
// executes griddepcontrol.wait before it reads anything.
template <typename... KArgs, typename... Args>
static cudaError_t pdl_launch(void (*kern)(KArgs...), int grid, int threads, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// fp32 pools: the global-load kernel, rows padded to 16.
static int fd_launch_f32(FDParams& p, void* ws, size_t ws_bytes, cudaStream_t st) {
  const int grid = fd_grid(HC_F32);
  const size_t slots = (size_t)grid + p.R;
  if (!ws || ws_bytes < slots * p.G * kD * sizeof(float) + slots * p.G * sizeof(float2)) return HC_ERR_WORKSPACE;
  p.part_o = reinterpret_cast<float*>(ws);
  p.part_ml = reinterpret_cast<float2*>(reinterpret_cast<unsigned char*>(ws) + slots * p.G * kD * sizeof(float));
  p.gran = 16;
  if (pdl_launch(flash_decode_kernel<float>, grid, kFThreads, (size_t)(p.R + 1) * sizeof(int), st, p) != cudaSuccess)
    return HC_ERR_CUDA;
  return fd_combine<float>(p, grid, st);
}

// Co-resident CTAs of the 16-bit TMA decode kernel for `dsm` bytes of dynamic
// shared memory on the current device, 0 if it cannot run.  The kernel's
// shared-memory limit is raised and the occupancy queried once per device and
// size; later calls make no CUDA call but cudaGetDevice.
template <typename T>
static int fd_tma_grid(size_t dsm) {
  static bool attr_set[kMaxDevices];
  static ShapeCache<8> grids;
  auto kern = flash_decode_tma_kernel<T>;
  const int dev = current_device();
  if (dev < 0) return 0;
  std::lock_guard<std::mutex> g(host_lock());
  long long v = 0;
  if (attr_set[dev] && grids.find(dev, (long long)dsm, v)) return (int)v;
  if (!attr_set[dev]) {
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes) !=
        cudaSuccess)
      return 0;
    attr_set[dev] = true;
  }
  int occ = 0, sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kTThreads, dsm) != cudaSuccess || occ <= 0) return 0;
  grids.put(dev, (long long)dsm, (long long)sms * occ);
  return sms * occ;
}

// 16-bit pools: the TMA pipeline, rows padded to 64.
template <typename T>
static int fd_launch_tma(FDParams& p, void* ws, size_t ws_bytes, cudaStream_t st) {
  auto kern = flash_decode_tma_kernel<T>;
  const int dtype = std::is_same<T, __nv_bfloat16>::value ? HC_BF16 : HC_F16;
  CUtensorMap tmk, tmv;
  const long long rows = (long long)p.n_blocks * kPage;
  if (!pool_tensor_map(&tmk, p.kp, rows, dtype, kTTile)) return HC_ERR_CUDA;
  if (!pool_tensor_map(&tmv, p.vp, rows, dtype, kTTile)) return HC_ERR_CUDA;
  const size_t dsm = fd_tma_smem(p.R, p.G);
  const int grid = fd_tma_grid<T>(dsm);
  if (grid <= 0) return HC_ERR_UNSUPPORTED;
  const size_t slots = (size_t)grid + p.R;
  if (!ws || ws_bytes < slots * p.G * kD * sizeof(float) + slots * p.G * sizeof(float2)) return HC_ERR_WORKSPACE;
  p.part_o = reinterpret_cast<float*>(ws);
  p.part_ml = reinterpret_cast<float2*>(reinterpret_cast<unsigned char*>(ws) + slots * p.G * kD * sizeof(float));
  p.gran = kTTile;
  if (pdl_launch(kern, grid, kTThreads, dsm, st, p, tmk, tmv) != cudaSuccess) return HC_ERR_CUDA;
  return fd_combine<T>(p, grid, st);
}

// ---------------------------------------------------------------------------
// Fixed scratch for hc_flash_decode_noalloc: the split-K partials live in this
// module-scope array instead of a caller workspace.  Host code must not use
// the symbol as a device address; the address is fetched with
// cudaGetSymbolAddress once per device (on that device's first call).
static __device__ __align__(256) unsigned char g_noalloc_scratch[HC_NOALLOC_SCRATCH_BYTES];
static void* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Partials bytes one hc_flash_decode launch writes: (grid + rows) slots of
// G x (128 + 2) floats, the grid being the device's co-resident CTA count
// (from the same per-device cache the launch uses).  0 if the kernel cannot
// run.
static size_t flash_decode_scratch_need(int dtype, int R, int G) {
  int grid = 0;
  switch (dtype) {
    case HC_F32: grid = fd_grid(HC_F32); break;
    case HC_BF16: grid = fd_tma_grid<__nv_bfloat16>(fd_tma_smem(R, G)); break;
    case HC_F16: grid = fd_tma_grid<__half>(fd_tma_smem(R, G)); break;
    default: return 0;
  }
  if (grid <= 0) return 0;
  const size_t slots = (size_t)grid + R;
  return slots * G * kD * sizeof(float) + slots * G * sizeof(float2);
}

int flash_decode_noalloc_dispatch(int dtype, FDParams& p, cudaStream_t st, size_t* need_out) {
  // the same argument checks, in the same order, as flash_decode_dispatch
  if (p.R <= 0 || p.R > kMaxRowsFD) return HC_ERR_UNSUPPORTED;
  if (p.G <= 0 || p.G > kGMax) return HC_ERR_UNSUPPORTED;
  if (dtype != HC_F32 && dtype != HC_BF16 && dtype != HC_F16) return HC_ERR_DTYPE;
  const int dev = current_device();
  if (dev < 0) return HC_ERR_UNSUPPORTED;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> g(host_lock());
    if (!g_noalloc_ptr[dev]) {
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return HC_ERR_CUDA;
      g_noalloc_ptr[dev] = ptr;
    }
    scratch = g_noalloc_ptr[dev];
  }
  const size_t need = flash_decode_scratch_need(dtype, p.R, p.G);
  if (need_out) *need_out = need;
  if (need == 0) return HC_ERR_UNSUPPORTED;
  if (need > (size_t)HC_NOALLOC_SCRATCH_BYTES) return HC_ERR_WORKSPACE;
  return flash_decode_dispatch(dtype, p, scratch, HC_NOALLOC_SCRATCH_BYTES, st);
}

int flash_decode_dispatch(int dtype, FDParams& p, void* ws, size_t ws_bytes, cudaStream_t st) {
  p.wait_ns = wait_limit_ns(kMbarTimeoutNs);
  if (p.R <= 0 || p.R > kMaxRowsFD) return HC_ERR_UNSUPPORTED;
  if (p.G <= 0 || p.G > kGMax) return HC_ERR_UNSUPPORTED;
  switch (dtype) {
    case HC_F32: return fd_launch_f32(p, ws, ws_bytes, st);
    case HC_BF16: return fd_launch_tma<__nv_bfloat16>(p, ws, ws_bytes, st);
    case HC_F16: return fd_launch_tma<__half>(p, ws, ws_bytes, st);
    default: return HC_ERR_DTYPE;
  }
}

}  // namespace hc
