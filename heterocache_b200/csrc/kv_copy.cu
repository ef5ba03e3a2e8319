// Page writes of the HeteroCache path that are plain data movement:
//   prefill keep-head copy   (heterocache/cache_utils.py:914-937)
//   decode append            (heterocache/cache_utils.py:970-1005)
//   satellite retrieval      (heterocache/cache_utils.py:1084-1147)
// All three move whole 128-element rows with 16-byte vector accesses.
#include "hc_host.cuh"
#include "hc_params.cuh"

namespace hc {

// ---------------------------------------------------------------------------
// Prefill: copy keep heads' [L, D] rows into their pages; heads_len = L.
template <typename T>
__global__ void __launch_bounds__(256) prefill_keep_kernel(const T* __restrict__ k, const T* __restrict__ v,
                                                           int64_t sb, int64_t sh, int64_t st, int64_t vsb,
                                                           int64_t vsh, int64_t vst, int L, int KV,
                                                           const int32_t* __restrict__ keep_heads, T* k_pool,
                                                           T* v_pool, int n_blocks, const int32_t* __restrict__ bt,
                                                           int max_blocks, int32_t* heads_len, int32_t* err) {
  constexpr int CH = kD * sizeof(T) / 16;  // 16-byte chunks per row
  constexpr int RPP = 256 / CH;            // rows per pass
  const int b = blockIdx.z, i = blockIdx.y;
  const int h = keep_heads[i];
  const int row = b * KV + h;
  const int c = threadIdx.x % CH;
  const int t0 = blockIdx.x * 64;
  for (int t = t0 + threadIdx.x / CH; t < min(L, t0 + 64); t += RPP) {
    const int page = t >> 8;
    const int blk = page < max_blocks ? bt[(int64_t)row * max_blocks + page] : -1;
    if (blk < 0 || blk >= n_blocks) {
      if (c == 0) set_err(err, HC_ERR_RANGE);
      continue;
    }
    const int64_t src = b * sb + (int64_t)h * sh + (int64_t)t * st;
    const int64_t vsrc = b * vsb + (int64_t)h * vsh + (int64_t)t * vst;
    const int64_t dst = ((int64_t)blk * kPage + (t & (kPage - 1))) * kD;
    reinterpret_cast<uint4*>(k_pool + dst)[c] = ldg128(reinterpret_cast<const uint4*>(k + src) + c);
    reinterpret_cast<uint4*>(v_pool + dst)[c] = ldg128(reinterpret_cast<const uint4*>(v + vsrc) + c);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) heads_len[row] = L;
}

// ---------------------------------------------------------------------------
// Decode append.  One CTA; rows that need a page take one from the free list
// in row order (the reference assigns free_blocks[ptr:ptr+n] to the rows of
// the boolean mask in order).  Launched as a programmatic dependent: it waits
// for the previous kernel's results, then lets the attention kernel after it
// get resident.  With q_stage set it also stores the step's query rows.
constexpr int kAppendThreads = 256;

template <typename T>
__device__ __forceinline__ void append_row_copies(const T* k, const T* v, int64_t sb, int64_t sh, int64_t vsb,
                                                  int64_t vsh, int KV, T* k_pool, T* v_pool, int R,
                                                  const int* s_phys, const int* s_off) {
  constexpr int CH = kD * sizeof(T) / 16;
  for (int i = threadIdx.x; i < R * 2 * CH; i += kAppendThreads) {
    const int r = i / (2 * CH), x = i % (2 * CH);
    const int phys = s_phys[r];
    if (phys < 0) continue;
    const int b = r / KV, h = r % KV, c = x % CH;
    const int64_t dst = ((int64_t)phys * kPage + s_off[r]) * kD;
    if (x < CH)
      reinterpret_cast<uint4*>(k_pool + dst)[c] = ldg128(reinterpret_cast<const uint4*>(k + b * sb + (int64_t)h * sh) + c);
    else
      reinterpret_cast<uint4*>(v_pool + dst)[c] = ldg128(reinterpret_cast<const uint4*>(v + b * vsb + (int64_t)h * vsh) + c);
  }
}

template <typename T>
__global__ void __launch_bounds__(kAppendThreads) decode_append_kernel(
    const T* __restrict__ k, const T* __restrict__ v, int64_t sb, int64_t sh, int64_t vsb, int64_t vsh, int R, int KV,
    T* k_pool, T* v_pool, int n_blocks, int32_t* bt, int max_blocks, int32_t* heads_len,
    const int32_t* __restrict__ free_blocks, int n_free, int32_t* free_ptr, const T* __restrict__ q, int64_t qsh,
    int nq, T* q_stage, int32_t* err) {
  constexpr int CH = kD * sizeof(T) / 16;
  __shared__ int s_warp[32];
  __shared__ int s_total, s_fail;
  __shared__ int s_phys[32], s_off[32];
  pdl_wait();
  pdl_trigger();
  // the step's query rows for the drift check (independent of the page work)
  for (int i = threadIdx.x; i < nq * CH; i += kAppendThreads)
    reinterpret_cast<uint4*>(q_stage)[i] = ldg128(reinterpret_cast<const uint4*>(q + (int64_t)(i / CH) * qsh) + i % CH);
  if (R <= 32) {
    // one warp does the bookkeeping: ballots replace the block scans
    if (threadIdx.x < 32) {
      const int r = threadIdx.x;
      const int base_ptr = *free_ptr;
      int len = 0, blk = 0, phys = -1, need = 0, fail = 0;
      if (r < R) {
        len = heads_len[r];
        blk = len >> 8;
        if (len < 0 || blk >= max_blocks) {
          fail = HC_ERR_RANGE;
        } else {
          phys = bt[(int64_t)r * max_blocks + blk];
          need = phys == -1;
          if (phys < -1 || phys >= n_blocks) fail = HC_ERR_RANGE;
        }
      }
      const unsigned int needm = __ballot_sync(0xffffffffu, need);
      const int total = __popc(needm);
      int f = __ballot_sync(0xffffffffu, fail != 0) ? HC_ERR_RANGE : 0;
      if (!f && (base_ptr < 0 || base_ptr + total > n_free)) f = HC_ERR_OOM;
      bool ok = r < R && !f;
      if (ok && need) {
        phys = free_blocks[base_ptr + __popc(needm & ((1u << r) - 1u))];
        if (phys < 0 || phys >= n_blocks) {  // corrupt free list: leave the row untouched
          set_err(err, HC_ERR_RANGE);
          ok = false;
        } else {
          bt[(int64_t)r * max_blocks + blk] = phys;
        }
      }
      if (ok) heads_len[r] = len + 1;
      s_phys[r] = ok ? phys : -1;
      s_off[r] = len & (kPage - 1);
      if (r == 0) {
        s_fail = f;
        if (f) set_err(err, f);
        else *free_ptr = base_ptr + total;
      }
    }
    __syncthreads();
    if (s_fail) return;
    append_row_copies<T>(k, v, sb, sh, vsb, vsh, KV, k_pool, v_pool, R, s_phys, s_off);
    return;
  }
  const int base_ptr = *free_ptr;
  int carry = 0;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  // pass 1: count needed pages and detect range errors
  for (int c0 = 0; c0 < R; c0 += blockDim.x) {
    const int r = c0 + threadIdx.x;
    int need = 0;
    if (r < R) {
      const int len = heads_len[r];
      const int blk = len >> 8;
      if (len < 0 || blk >= max_blocks) {
        atomicExch(&s_fail, HC_ERR_RANGE);
      } else {
        const int phys = bt[(int64_t)r * max_blocks + blk];
        need = phys == -1;
        if (phys < -1 || phys >= n_blocks) atomicExch(&s_fail, HC_ERR_RANGE);
      }
    }
    int tot;
    block_exclusive_scan(need, s_warp, tot);
    carry += tot;
  }
  if (threadIdx.x == 0) {
    s_total = carry;
    if (!s_fail && (base_ptr < 0 || base_ptr + carry > n_free)) s_fail = HC_ERR_OOM;
  }
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0) set_err(err, s_fail);
    return;
  }
  // pass 2: allocate in row order and write the rows
  carry = 0;
  for (int c0 = 0; c0 < R; c0 += blockDim.x) {
    const int r = c0 + threadIdx.x;
    int need = 0, len = 0, blk = 0, phys = 0;
    if (r < R) {
      len = heads_len[r];
      blk = len >> 8;
      phys = bt[(int64_t)r * max_blocks + blk];
      need = phys == -1;
    }
    int tot;
    const int ex = block_exclusive_scan(need, s_warp, tot);
    bool ok = r < R;
    if (ok && need) {
      phys = free_blocks[base_ptr + carry + ex];
      if (phys < 0 || phys >= n_blocks) {  // corrupt free list: leave the row untouched
        set_err(err, HC_ERR_RANGE);
        ok = false;
      } else {
        bt[(int64_t)r * max_blocks + blk] = phys;
      }
    }
    if (ok) {
      const int b = r / KV, h = r % KV;
      const uint4* ks = reinterpret_cast<const uint4*>(k + b * sb + (int64_t)h * sh);
      const uint4* vs = reinterpret_cast<const uint4*>(v + b * vsb + (int64_t)h * vsh);
      const int64_t dst = ((int64_t)phys * kPage + (len & (kPage - 1))) * kD;
      uint4* kd = reinterpret_cast<uint4*>(k_pool + dst);
      uint4* vd = reinterpret_cast<uint4*>(v_pool + dst);
#pragma unroll 4
      for (int c = 0; c < CH; ++c) {
        kd[c] = ks[c];
        vd[c] = vs[c];
      }
      heads_len[r] = len + 1;
    }
    carry += tot;
  }
  if (threadIdx.x == 0) *free_ptr = base_ptr + s_total;
}

// ---------------------------------------------------------------------------
// Retrieval gather: full tier (device or pinned host memory) -> satellite pages.
// Work items of 64 rows of one member, K and V, taken by a grid of at most
// one wave that strides over them (members whose pivot did not trigger cost
// one check per item, not a CTA launch each).  In an item each thread copies
// one 16-byte chunk of NP rows: all position loads, then all row loads, then
// the stores (two dependent load rounds).
template <typename T>
__global__ void __launch_bounds__(256) retrieve_kernel(const int32_t* __restrict__ member_job,
                                                       const int32_t* __restrict__ member_head,
                                                       const int32_t* __restrict__ member_len,
                                                       const int32_t* __restrict__ trigger,
                                                       const int32_t* __restrict__ positions, int pos_stride,
                                                       const T* full_k, const T* full_v, int64_t fsh, int64_t fst,
                                                       T* k_pool, T* v_pool, int n_blocks,
                                                       const int32_t* __restrict__ bt, int max_blocks, int32_t* err,
                                                       int n_members, int items_per_member) {
  constexpr int CH = kD * sizeof(T) / 16;  // 16-byte chunks per row
  constexpr int RPP = 256 / CH;            // rows per pass of the CTA
  constexpr int NP = 64 / RPP;             // passes (rows per thread)
  // programmatic dependent launch: the trigger and positions come from the
  // drift check just before; the next kernel may get resident meanwhile
  pdl_wait();
  pdl_trigger();
  const uint64_t pol = l2_evict_first_policy();  // full-tier rows are read once
  const int n_items = n_members * items_per_member;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int m = item / items_per_member, blk = item % items_per_member;
    const int job = member_job[m];
    if (!trigger[job]) continue;
    const int n = member_len[m];
    if (blk * 64 >= n) continue;
    const int h = member_head[m];
    const int start = bt[(int64_t)h * max_blocks];
    if (start < 0) continue;
    if ((int64_t)start * kPage + n > (int64_t)n_blocks * kPage) {
      if (threadIdx.x == 0 && blk == 0) set_err(err, HC_ERR_RANGE);
      continue;
    }
    const int c = threadIdx.x % CH;
    const int i0 = blk * 64 + threadIdx.x / CH;
    int pos[NP];
    unsigned int rows = 0u;  // bit u: row i0 + u*RPP is one of the member's
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      const int i = i0 + u * RPP;
      pos[u] = -1;
      if (i < n) {
        pos[u] = positions[(size_t)job * pos_stride + i];
        rows |= 1u << u;
      }
    }
    uint4 kr[NP], vr[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      if (pos[u] >= 0) {
        const int64_t src = (int64_t)h * fsh + (int64_t)pos[u] * fst;
        kr[u] = ld_stream128(reinterpret_cast<const uint4*>(full_k + src) + c, pol);
        vr[u] = ld_stream128(reinterpret_cast<const uint4*>(full_v + src) + c, pol);
      }
    }
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      const int i = i0 + u * RPP;
      if (!((rows >> u) & 1u)) continue;
      if (pos[u] < 0) {
        if (c == 0) set_err(err, HC_ERR_RANGE);
        continue;
      }
      const int64_t dst = ((int64_t)start * kPage + i) * kD;
      reinterpret_cast<uint4*>(k_pool + dst)[c] = kr[u];
      reinterpret_cast<uint4*>(v_pool + dst)[c] = vr[u];
    }
  }
}

// ---------------------------------------------------------------------------
// Delta retrieval (pinned-host tier).  Same result as retrieve_kernel, but
// rows a satellite already holds are copied on the device and only the other
// rows cross the host link.  Each member m keeps a slot map: slot_pos[m][i] is
// the full-tier position held in slot i, for i < reuse_len[m].  Those slots lie
// below the satellite's prefill keep length, which only prefill selection and
// retrieval write (decode appends start at that length), so the map stays
// exact.  The map (kept indices, then retrieval lists) and every new list are
// ascending, so a binary search finds a new position's old slot.
//   pass 1 (delta_stage_kernel): per new slot i, the old slot holding its
//     position (or -1) -> stage_src[off[m] + i]; held rows -> staging row
//     off[m] + i.
//   pass 2 (delta_write_kernel): every new slot from the staging area or the
//     tier; then slot_pos[m][i] = new position for i < reuse_len[m].
// Two launches: a slot can be the source of another slot that overwrites it.
// Both passes skip the same work items (trigger off, unmapped or out-of-range
// member), so pass 2 only reads what pass 1 wrote.

// Old slot of `pos` among the ascending old[0, n), or -1.
__device__ __forceinline__ int find_slot(const int32_t* old, int n, int pos) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(old + mid) < pos) lo = mid + 1;
    else hi = mid;
  }
  return (lo < n && __ldg(old + lo) == pos) ? lo : -1;
}

struct DeltaArgs {
  const int32_t* member_job;
  const int32_t* member_head;
  const int32_t* member_len;
  const int32_t* member_off;
  const int32_t* reuse_len;
  const int32_t* trigger;
  const int32_t* positions;
  int pos_stride;
  int32_t* slot_pos;
  int slot_stride;
  const void* full_k;
  const void* full_v;
  int64_t fsh, fst;
  void* k_pool;
  void* v_pool;
  int n_blocks;
  const int32_t* bt;
  int max_blocks;
  void* stage_k;
  void* stage_v;
  int32_t* stage_src;
  int64_t stage_rows;
  int32_t* err;
  int n_members, items_per_member;
};

// Work item -> member geometry; false: nothing to do for this item.  Errors
// are reported by pass 1 only (pass 2 takes the same decisions).
struct DeltaItem {
  int m, job, n, h, start, off, R;
};
__device__ __forceinline__ bool delta_item(const DeltaArgs& a, int item, bool report, DeltaItem& it) {
  it.m = item / a.items_per_member;
  const int blk = item % a.items_per_member;
  it.job = a.member_job[it.m];
  if (!a.trigger[it.job]) return false;
  it.n = a.member_len[it.m];
  if (blk * 64 >= it.n) return false;
  it.h = a.member_head[it.m];
  it.start = a.bt[(int64_t)it.h * a.max_blocks];
  if (it.start < 0) return false;
  it.off = a.member_off[it.m];
  it.R = min(a.reuse_len[it.m], min(it.n, a.slot_stride));
  if ((int64_t)it.start * kPage + it.n > (int64_t)a.n_blocks * kPage || it.off < 0 ||
      (int64_t)it.off + it.n > a.stage_rows) {
    if (report && threadIdx.x == 0 && blk == 0) set_err(a.err, HC_ERR_RANGE);
    return false;
  }
  return true;
}

template <typename T>
__global__ void __launch_bounds__(256) delta_stage_kernel(const DeltaArgs a) {
  constexpr int CH = kD * sizeof(T) / 16;  // 16-byte chunks per row
  constexpr int RPP = 256 / CH;            // rows per pass of the CTA
  constexpr int NP = 64 / RPP;             // passes (rows per thread)
  pdl_wait();
  pdl_trigger();
  const T* kp = reinterpret_cast<const T*>(a.k_pool);
  const T* vp = reinterpret_cast<const T*>(a.v_pool);
  T* sk = reinterpret_cast<T*>(a.stage_k);
  T* sv = reinterpret_cast<T*>(a.stage_v);
  const int n_items = a.n_members * a.items_per_member;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    DeltaItem it;
    if (!delta_item(a, item, true, it)) continue;
    const int c = threadIdx.x % CH;
    const int i0 = (item % a.items_per_member) * 64 + threadIdx.x / CH;
    const int32_t* old = a.slot_pos + (int64_t)it.m * a.slot_stride;
    int src[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      const int i = i0 + u * RPP;
      src[u] = -1;
      if (i < it.n) {
        const int pos = a.positions[(size_t)it.job * a.pos_stride + i];
        if (pos >= 0) src[u] = find_slot(old, it.R, pos);
      }
    }
    uint4 kr[NP], vr[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      if (src[u] >= 0) {
        const int64_t row = ((int64_t)it.start * kPage + src[u]) * kD;
        kr[u] = ld_stream128(reinterpret_cast<const uint4*>(kp + row) + c);
        vr[u] = ld_stream128(reinterpret_cast<const uint4*>(vp + row) + c);
      }
    }
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      const int i = i0 + u * RPP;
      if (i >= it.n) continue;
      if (c == 0) a.stage_src[it.off + i] = src[u];
      if (src[u] >= 0) {
        const int64_t row = ((int64_t)it.off + i) * kD;
        reinterpret_cast<uint4*>(sk + row)[c] = kr[u];
        reinterpret_cast<uint4*>(sv + row)[c] = vr[u];
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) delta_write_kernel(const DeltaArgs a) {
  constexpr int CH = kD * sizeof(T) / 16;
  constexpr int RPP = 256 / CH;
  constexpr int NP = 64 / RPP;
  pdl_wait();  // pass 1 complete: staging rows, sources and the old map read
  pdl_trigger();
  const uint64_t pol = l2_evict_first_policy();  // full-tier rows are read once
  const T* fk = reinterpret_cast<const T*>(a.full_k);
  const T* fv = reinterpret_cast<const T*>(a.full_v);
  const T* sk = reinterpret_cast<const T*>(a.stage_k);
  const T* sv = reinterpret_cast<const T*>(a.stage_v);
  T* kp = reinterpret_cast<T*>(a.k_pool);
  T* vp = reinterpret_cast<T*>(a.v_pool);
  const int n_items = a.n_members * a.items_per_member;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    DeltaItem it;
    if (!delta_item(a, item, false, it)) continue;
    const int c = threadIdx.x % CH;
    const int i0 = (item % a.items_per_member) * 64 + threadIdx.x / CH;
    int pos[NP], src[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      const int i = i0 + u * RPP;
      pos[u] = -1;
      src[u] = -1;
      if (i < it.n) {
        pos[u] = a.positions[(size_t)it.job * a.pos_stride + i];
        src[u] = a.stage_src[it.off + i];
      }
    }
    uint4 kr[NP], vr[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      if (src[u] >= 0) {
        const int64_t row = ((int64_t)it.off + i0 + u * RPP) * kD;
        kr[u] = ld_stream128(reinterpret_cast<const uint4*>(sk + row) + c);
        vr[u] = ld_stream128(reinterpret_cast<const uint4*>(sv + row) + c);
      } else if (pos[u] >= 0) {
        const int64_t row = (int64_t)it.h * a.fsh + (int64_t)pos[u] * a.fst;
        kr[u] = ld_stream128(reinterpret_cast<const uint4*>(fk + row) + c, pol);
        vr[u] = ld_stream128(reinterpret_cast<const uint4*>(fv + row) + c, pol);
      }
    }
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      const int i = i0 + u * RPP;
      if (i >= it.n) continue;
      if (pos[u] < 0) {
        if (c == 0) set_err(a.err, HC_ERR_RANGE);
        continue;
      }
      const int64_t dst = ((int64_t)it.start * kPage + i) * kD;
      reinterpret_cast<uint4*>(kp + dst)[c] = kr[u];
      reinterpret_cast<uint4*>(vp + dst)[c] = vr[u];
      if (c == 0 && i < it.R) a.slot_pos[(int64_t)it.m * a.slot_stride + i] = pos[u];
    }
  }
}

// ---------------------------------------------------------------------------
template <typename T>
static int prefill_keep_t(int bsz, int KV, int L, const int32_t* keep, int n_keep, const void* k, const void* v,
                          int64_t sb, int64_t sh, int64_t st, int64_t vsb, int64_t vsh, int64_t vst, void* kp,
                          void* vp, int nb, const int32_t* bt, int mb, int32_t* hl, int32_t* err, cudaStream_t s) {
  dim3 grid((L + 63) / 64, n_keep, bsz);
  prefill_keep_kernel<T><<<grid, 256, 0, s>>>((const T*)k, (const T*)v, sb, sh, st, vsb, vsh, vst, L, KV, keep,
                                              (T*)kp, (T*)vp, nb, bt, mb, hl, err);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

int prefill_keep_dispatch(int dtype, int bsz, int KV, int L, const int32_t* keep, int n_keep, const void* k,
                          const void* v, int64_t sb, int64_t sh, int64_t st, int64_t vsb, int64_t vsh, int64_t vst,
                          void* kp, void* vp, int nb, const int32_t* bt, int mb, int32_t* hl, int32_t* err,
                          cudaStream_t s) {
  switch (dtype) {
    case HC_F32:
      return prefill_keep_t<float>(bsz, KV, L, keep, n_keep, k, v, sb, sh, st, vsb, vsh, vst, kp, vp, nb, bt, mb, hl,
                                   err, s);
    case HC_BF16:
      return prefill_keep_t<__nv_bfloat16>(bsz, KV, L, keep, n_keep, k, v, sb, sh, st, vsb, vsh, vst, kp, vp, nb, bt,
                                           mb, hl, err, s);
    case HC_F16:
      return prefill_keep_t<__half>(bsz, KV, L, keep, n_keep, k, v, sb, sh, st, vsb, vsh, vst, kp, vp, nb, bt, mb, hl,
                                    err, s);
    default: return HC_ERR_DTYPE;
  }
}

template <typename T>
static int append_t(int R, int KV, const void* k, const void* v, int64_t sb, int64_t sh, int64_t vsb, int64_t vsh,
                    void* kp, void* vp, int nb, int32_t* bt, int mb, int32_t* hl, const int32_t* fb, int nf,
                    int32_t* fp, const void* q, int64_t qsh, int nq, void* q_stage, int32_t* err, cudaStream_t s) {
  // programmatic dependent launch: the kernel starts while the previous one
  // drains and waits (griddepcontrol.wait) before touching any data
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kAppendThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_append_kernel<T>, (const T*)k, (const T*)v, sb, sh, vsb, vsh, R,
                                           KV, (T*)kp, (T*)vp, nb, bt, mb, hl, fb, nf, fp, (const T*)q, qsh, nq,
                                           (T*)q_stage, err);
  return e == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

int decode_append_dispatch(int dtype, int R, int KV, const void* k, const void* v, int64_t sb, int64_t sh,
                           int64_t vsb, int64_t vsh, void* kp, void* vp, int nb, int32_t* bt, int mb, int32_t* hl,
                           const int32_t* fb, int nf, int32_t* fp, const void* q, int64_t qsh, int nq, void* q_stage,
                           int32_t* err, cudaStream_t s) {
  switch (dtype) {
    case HC_F32:
      return append_t<float>(R, KV, k, v, sb, sh, vsb, vsh, kp, vp, nb, bt, mb, hl, fb, nf, fp, q, qsh, nq, q_stage, err,
                             s);
    case HC_BF16:
      return append_t<__nv_bfloat16>(R, KV, k, v, sb, sh, vsb, vsh, kp, vp, nb, bt, mb, hl, fb, nf, fp, q, qsh, nq,
                                     q_stage, err, s);
    case HC_F16:
      return append_t<__half>(R, KV, k, v, sb, sh, vsb, vsh, kp, vp, nb, bt, mb, hl, fb, nf, fp, q, qsh, nq, q_stage,
                              err, s);
    default: return HC_ERR_DTYPE;
  }
}

template <typename T>
static int retrieve_t(int n_members, const int32_t* mj, const int32_t* mh, const int32_t* ml, int max_len,
                      const int32_t* trig, const int32_t* pos, int pos_stride, const void* fk, const void* fv,
                      int64_t fsh, int64_t fst, void* kp, void* vp, int nb, const int32_t* bt, int mb, int32_t* err,
                      cudaStream_t s) {
  if (n_members == 0 || max_len <= 0) return HC_OK;
  // one wave: 8 CTAs of 256 threads per SM
  const int sms = device_sms(current_device());
  const int per_member = (max_len + 63) / 64;
  const long long items = (long long)per_member * n_members;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(items < 8LL * sms ? items : 8LL * sms));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (items > 0x7fffffffLL) return HC_ERR_UNSUPPORTED;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, retrieve_kernel<T>, mj, mh, ml, trig, pos, pos_stride, (const T*)fk,
                                           (const T*)fv, fsh, fst, (T*)kp, (T*)vp, nb, bt, mb, err, n_members,
                                           per_member);
  return e == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

template <typename T>
static int retrieve_delta_t(DeltaArgs& a, int max_len, cudaStream_t s) {
  if (a.n_members == 0 || max_len <= 0) return HC_OK;
  const int sms = device_sms(current_device());
  a.items_per_member = (max_len + 63) / 64;
  const long long items = (long long)a.items_per_member * a.n_members;
  if (items > 0x7fffffffLL) return HC_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(items < 8LL * sms ? items : 8LL * sms));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, delta_stage_kernel<T>, a) != cudaSuccess) return HC_ERR_CUDA;
  if (cudaLaunchKernelEx(&cfg, delta_write_kernel<T>, a) != cudaSuccess) return HC_ERR_CUDA;
  return HC_OK;
}

int retrieve_delta_dispatch(int dtype, const int32_t* mj, const int32_t* mh, const int32_t* ml, const int32_t* moff,
                            const int32_t* reuse, int n_members, int max_len, const int32_t* trig, const int32_t* pos,
                            int pos_stride, int32_t* slot_pos, int slot_stride, const void* fk, const void* fv,
                            int64_t fsh, int64_t fst, void* kp, void* vp, int nb, const int32_t* bt, int mb,
                            void* stage_k, void* stage_v, int32_t* stage_src, int64_t stage_rows, int32_t* err,
                            cudaStream_t s) {
  DeltaArgs a;
  a.member_job = mj;
  a.member_head = mh;
  a.member_len = ml;
  a.member_off = moff;
  a.reuse_len = reuse;
  a.trigger = trig;
  a.positions = pos;
  a.pos_stride = pos_stride;
  a.slot_pos = slot_pos;
  a.slot_stride = slot_stride;
  a.full_k = fk;
  a.full_v = fv;
  a.fsh = fsh;
  a.fst = fst;
  a.k_pool = kp;
  a.v_pool = vp;
  a.n_blocks = nb;
  a.bt = bt;
  a.max_blocks = mb;
  a.stage_k = stage_k;
  a.stage_v = stage_v;
  a.stage_src = stage_src;
  a.stage_rows = stage_rows;
  a.err = err;
  a.n_members = n_members;
  a.items_per_member = 0;
  switch (dtype) {
    case HC_F32: return retrieve_delta_t<float>(a, max_len, s);
    case HC_BF16: return retrieve_delta_t<__nv_bfloat16>(a, max_len, s);
    case HC_F16: return retrieve_delta_t<__half>(a, max_len, s);
    default: return HC_ERR_DTYPE;
  }
}

int retrieve_dispatch(int dtype, int n_members, const int32_t* mj, const int32_t* mh, const int32_t* ml, int max_len,
                      const int32_t* trig, const int32_t* pos, int pos_stride, const void* fk, const void* fv,
                      int64_t fsh, int64_t fst, void* kp, void* vp, int nb, const int32_t* bt, int mb, int32_t* err,
                      cudaStream_t s) {
  switch (dtype) {
    case HC_F32: return retrieve_t<float>(n_members, mj, mh, ml, max_len, trig, pos, pos_stride, fk, fv, fsh, fst, kp, vp, nb, bt, mb, err, s);
    case HC_BF16: return retrieve_t<__nv_bfloat16>(n_members, mj, mh, ml, max_len, trig, pos, pos_stride, fk, fv, fsh, fst, kp, vp, nb, bt, mb, err, s);
    case HC_F16: return retrieve_t<__half>(n_members, mj, mh, ml, max_len, trig, pos, pos_stride, fk, fv, fsh, fst, kp, vp, nb, bt, mb, err, s);
    default: return HC_ERR_DTYPE;
  }
}

}  // namespace hc
