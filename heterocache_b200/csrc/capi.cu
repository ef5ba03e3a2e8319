// extern "C" boundary: argument validation, parameter packing, dispatch.
#include <cmath>
#include <cstring>

#include <cstdio>

#include <algorithm>
#include <atomic>
#include <mutex>

#include <cuda.h>

#include "hc_params.cuh"

namespace hc {

static std::atomic<unsigned long long> g_wait_limit_ns{0};
static std::atomic<int> g_stall{0};

uint64_t wait_limit_ns(uint64_t dflt) {
  const unsigned long long v = g_wait_limit_ns.load(std::memory_order_relaxed);
  return v ? (uint64_t)v : dflt;
}

unsigned int injected_stall() { return g_stall.load(std::memory_order_relaxed) ? 1u : 0u; }

}  // namespace hc

namespace {

thread_local char g_last_err[256] = {0};

int note_cuda(int rc) {
  if (rc == HC_ERR_CUDA) {
    cudaError_t e = cudaGetLastError();
    std::snprintf(g_last_err, sizeof(g_last_err), "%s", cudaGetErrorString(e));
  }
  return rc;
}

bool valid_dtype(int dtype) { return dtype == HC_F32 || dtype == HC_BF16 || dtype == HC_F16; }
int elem_bytes(int dtype) { return dtype == HC_F32 ? 4 : 2; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
// Row strides must keep every 128-element row 16-byte aligned.
bool stride_ok(int dtype, int64_t s) { return (s * elem_bytes(dtype)) % 16 == 0; }

float div_sqrt_d(int head_dim) { return (float)std::sqrt((double)head_dim); }

}  // namespace

extern "C" {

int hc_abi_version(void) { return HC_ABI_VERSION; }

const char* hc_status_string(int status) {
  switch (status) {
    case HC_OK: return "ok";
    case HC_ERR_INVALID: return "invalid argument";
    case HC_ERR_DTYPE: return "unsupported dtype";
    case HC_ERR_OOM: return "decode free list exhausted";
    case HC_ERR_RANGE: return "page-table entry or index out of range";
    case HC_ERR_CUDA: return "CUDA error";
    case HC_ERR_WORKSPACE: return "workspace missing or too small";
    case HC_ERR_TIMEOUT: return "device-side wait timed out";
    case HC_ERR_UNSUPPORTED: return "unsupported configuration";
    default: return "unknown status";
  }
}

const char* hc_last_cuda_error(void) { return g_last_err; }

int hc_set_wait_limits(unsigned long long limit_ns, int inject_stall) {
  hc::g_wait_limit_ns.store(limit_ns, std::memory_order_relaxed);
  hc::g_stall.store(inject_stall ? 1 : 0, std::memory_order_relaxed);
  return HC_OK;
}

int hc_prefill_keep(int dtype, int bsz, int num_kv_heads, int seq_len, int head_dim, const int32_t* keep_heads,
                    int n_keep, const void* k, const void* v, int64_t sb, int64_t sh, int64_t st, int64_t vsb,
                    int64_t vsh, int64_t vst, void* k_pool, void* v_pool, int n_pool_blocks,
                    const int32_t* block_table, int max_blocks, int32_t* heads_len, int32_t* err_flag,
                    void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || bsz <= 0 || num_kv_heads <= 0 || seq_len <= 0 || n_keep < 0) return HC_ERR_INVALID;
  if (n_keep == 0) return HC_OK;
  if (!aligned16(k) || !aligned16(v) || !aligned16(k_pool) || !aligned16(v_pool)) return HC_ERR_INVALID;
  if (!stride_ok(dtype, sb) || !stride_ok(dtype, sh) || !stride_ok(dtype, st) || !stride_ok(dtype, vsb) ||
      !stride_ok(dtype, vsh) || !stride_ok(dtype, vst))
    return HC_ERR_INVALID;
  return note_cuda(hc::prefill_keep_dispatch(dtype, bsz, num_kv_heads, seq_len, keep_heads, n_keep, k, v, sb, sh, st,
                                             vsb, vsh, vst, k_pool, v_pool, n_pool_blocks, block_table, max_blocks,
                                             heads_len, err_flag, (cudaStream_t)stream));
}

size_t hc_prefill_select_workspace_size(int dtype, int bsz, int n_heads, int seq_len, int groups, int window) {
  if (bsz <= 0 || n_heads <= 0 || seq_len <= 0) return 0;
  return hc::score_workspace_size(dtype, bsz * n_heads, seq_len, groups * window, 1);
}

int hc_prefill_select(int dtype, int bsz, int num_kv_heads, int groups, int seq_len, int head_dim, int n_heads,
                      int window, int pooling, int kernel_size, const void* q, int64_t qsb, int64_t qsh, int64_t qst,
                      const void* k, const void* v, int64_t sb, int64_t sh, int64_t st, int64_t vsb, int64_t vsh,
                      int64_t vst, const int32_t* keep_lens,
                      int max_keep, void* k_pool, void* v_pool, int n_pool_blocks, const int32_t* block_table,
                      int max_blocks, int32_t* heads_len, int32_t* out_indices, void* out_scores, void* workspace,
                      size_t workspace_bytes, int32_t* err_flag, void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || bsz <= 0 || num_kv_heads <= 0 || groups <= 0 || seq_len <= 0) return HC_ERR_INVALID;
  if (n_heads < 0 || n_heads > num_kv_heads) return HC_ERR_INVALID;
  if (n_heads == 0) return HC_OK;
  if (window < 1 || window > seq_len) return HC_ERR_INVALID;
  if (pooling != HC_AVGPOOL && pooling != HC_MAXPOOL) return HC_ERR_INVALID;
  if (kernel_size < 1 || (kernel_size & 1) == 0 || kernel_size / 2 > 16) return HC_ERR_INVALID;
  if (groups * window > 256) return HC_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(k_pool) || !aligned16(v_pool))
    return HC_ERR_INVALID;
  if (!stride_ok(dtype, qsb) || !stride_ok(dtype, qsh) || !stride_ok(dtype, qst) || !stride_ok(dtype, sb) ||
      !stride_ok(dtype, sh) || !stride_ok(dtype, st) || !stride_ok(dtype, vsb) || !stride_ok(dtype, vsh) ||
      !stride_ok(dtype, vst))
    return HC_ERR_INVALID;
  hc::ScoreParams p;
  std::memset(&p, 0, sizeof(p));
  p.mode = hc::MODE_PREFILL;
  p.vsb = vsb;
  p.vsh = vsh;
  p.vst = vst;
  p.L = seq_len;
  p.G = groups;
  p.W = window;
  p.S = 1;
  p.Rq = groups * window;
  p.pooling = pooling;
  p.ksize = kernel_size;
  p.halo = kernel_size / 2;
  p.sqrt_d = div_sqrt_d(head_dim);
  p.n_jobs = bsz * n_heads;
  p.KV = num_kv_heads;
  p.nh = n_heads;
  p.nsel = 1;
  p.keep_lens = keep_lens;
  p.q = q;
  p.qsb = qsb;
  p.qsh = qsh;
  p.qst = qst;
  p.q_tok0 = seq_len - window;
  p.k = k;
  p.v = v;
  p.ksb = sb;
  p.ksh = sh;
  p.kst = st;
  p.bt = block_table;
  p.max_blocks = max_blocks;
  p.n_blocks = n_pool_blocks;
  p.k_pool_out = k_pool;
  p.v_pool_out = v_pool;
  p.heads_len = heads_len;
  p.out_indices = out_indices;
  p.max_keep = max_keep;
  p.out_scores = out_scores;
  p.err = err_flag;
  return note_cuda(hc::score_dispatch(dtype, p, workspace, workspace_bytes, (cudaStream_t)stream));
}

size_t hc_snapkv_update_kv_workspace_size(int dtype, int bsz, int num_heads, int seq_len, int window) {
  if (bsz <= 0 || num_heads <= 0 || seq_len <= 0 || window <= 0) return 0;
  return hc::score_workspace_size(dtype, bsz * num_heads, seq_len, window, 1);
}

int hc_snapkv_update_kv(int dtype, int bsz, int num_heads, int seq_len, int head_dim, int window, int pooling,
                        int kernel_size, int capacity, const void* q, int64_t qsb, int64_t qsh, int64_t qst,
                        const void* k, const void* v, int64_t sb, int64_t sh, int64_t st, int64_t vsb, int64_t vsh,
                        int64_t vst, void* out_k, void* out_v, int32_t* out_indices, void* out_scores,
                        void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || bsz <= 0 || num_heads <= 0 || seq_len <= 0) return HC_ERR_INVALID;
  if (window < 1 || window >= seq_len) return HC_ERR_INVALID;
  if (capacity < window || capacity > seq_len) return HC_ERR_INVALID;
  if (pooling != HC_AVGPOOL && pooling != HC_MAXPOOL) return HC_ERR_INVALID;
  if (kernel_size < 1 || (kernel_size & 1) == 0 || kernel_size / 2 > 16) return HC_ERR_INVALID;
  if (window > 256) return HC_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out_k) || !aligned16(out_v))
    return HC_ERR_INVALID;
  if (!stride_ok(dtype, qsb) || !stride_ok(dtype, qsh) || !stride_ok(dtype, qst) || !stride_ok(dtype, sb) ||
      !stride_ok(dtype, sh) || !stride_ok(dtype, st) || !stride_ok(dtype, vsb) || !stride_ok(dtype, vsh) ||
      !stride_ok(dtype, vst))
    return HC_ERR_INVALID;
  hc::ScoreParams p;
  std::memset(&p, 0, sizeof(p));
  p.mode = hc::MODE_PREFILL;
  p.L = seq_len;
  p.Lsel = seq_len - window;
  p.G = 1;
  p.W = window;
  p.S = 1;
  p.Rq = window;
  p.pooling = pooling;
  p.ksize = kernel_size;
  p.halo = kernel_size / 2;
  p.sqrt_d = div_sqrt_d(head_dim);
  p.n_jobs = bsz * num_heads;
  p.KV = num_heads;
  p.nh = num_heads;
  p.nsel = 1;
  p.keep_lens = nullptr;
  p.keep_const = capacity - window;
  p.tail = window;
  p.out_job_rows = capacity;
  p.q = q;
  p.qsb = qsb;
  p.qsh = qsh;
  p.qst = qst;
  p.q_tok0 = seq_len - window;
  p.k = k;
  p.v = v;
  p.ksb = sb;
  p.ksh = sh;
  p.kst = st;
  p.vsb = vsb;
  p.vsh = vsh;
  p.vst = vst;
  p.k_pool_out = out_k;
  p.v_pool_out = out_v;
  p.heads_len = nullptr;
  p.out_indices = out_indices;
  p.max_keep = capacity - window;
  p.out_scores = out_scores;
  p.err = err_flag;
  return note_cuda(hc::score_dispatch(dtype, p, workspace, workspace_bytes, (cudaStream_t)stream));
}

size_t hc_pivot_init_workspace_size(int dtype, int bsz, int n_pivots, int seq_len, int groups) {
  if (bsz <= 0 || n_pivots <= 0 || seq_len <= 0) return 0;
  return hc::score_workspace_size(dtype, bsz * n_pivots, seq_len, groups, 1);
}

int hc_pivot_init(int dtype, int bsz, int num_kv_heads, int groups, int seq_len, int head_dim, int first_pivot,
                  int n_pivots, int pooling, int kernel_size, int topk, const void* q, int64_t qsb, int64_t qsh,
                  int64_t qst, const void* k, int64_t sb, int64_t sh, int64_t st, int32_t* ref_positions,
                  uint32_t* ref_bitmap, void* out_scores, void* workspace, size_t workspace_bytes, int32_t* err_flag,
                  void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || bsz <= 0 || num_kv_heads <= 0 || groups <= 0 || seq_len <= 0) return HC_ERR_INVALID;
  if (n_pivots == 0) return HC_OK;
  if (n_pivots < 0 || first_pivot < 0 || first_pivot + n_pivots > num_kv_heads) return HC_ERR_INVALID;
  if (topk < 0 || topk > seq_len) return HC_ERR_INVALID;
  if (pooling != HC_AVGPOOL && pooling != HC_MAXPOOL) return HC_ERR_INVALID;
  if (kernel_size < 1 || (kernel_size & 1) == 0 || kernel_size / 2 > 16) return HC_ERR_INVALID;
  if (groups > 256) return HC_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k)) return HC_ERR_INVALID;
  if (!stride_ok(dtype, qsb) || !stride_ok(dtype, qsh) || !stride_ok(dtype, qst) || !stride_ok(dtype, sb) ||
      !stride_ok(dtype, sh) || !stride_ok(dtype, st))
    return HC_ERR_INVALID;
  hc::ScoreParams p;
  std::memset(&p, 0, sizeof(p));
  p.mode = hc::MODE_PIVOT;
  p.L = seq_len;
  p.G = groups;
  p.W = 1;
  p.S = 1;
  p.Rq = groups;
  p.pooling = pooling;
  p.ksize = kernel_size;
  p.halo = kernel_size / 2;
  p.sqrt_d = div_sqrt_d(head_dim);
  p.n_jobs = bsz * n_pivots;
  p.KV = num_kv_heads;
  p.nh = n_pivots;
  p.first_head = first_pivot;
  p.nsel = 1;
  p.topk = topk;
  p.q = q;
  p.qsb = qsb;
  p.qsh = qsh;
  p.qst = qst;
  p.q_tok0 = seq_len - 1;
  p.k = k;
  p.ksb = sb;
  p.ksh = sh;
  p.kst = st;
  p.ref_positions = ref_positions;
  p.ref_bitmap = ref_bitmap;
  p.bitmap_words = (seq_len + 31) / 32;
  p.out_scores = out_scores;
  p.err = err_flag;
  return note_cuda(hc::score_dispatch(dtype, p, workspace, workspace_bytes, (cudaStream_t)stream));
}

int hc_decode_append(int dtype, int bsz, int num_kv_heads, int head_dim, const void* k, const void* v, int64_t sb,
                     int64_t sh, int64_t vsb, int64_t vsh, void* k_pool, void* v_pool, int n_pool_blocks,
                     int32_t* block_table, int max_blocks, int32_t* heads_len, const int32_t* free_blocks, int n_free,
                     int32_t* free_ptr, const void* q, int64_t qsh, int n_q_heads, void* q_stage, int32_t* err_flag,
                     void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || bsz <= 0 || num_kv_heads <= 0 || max_blocks <= 0 || n_free < 0)
    return HC_ERR_INVALID;
  if (!aligned16(k) || !aligned16(v) || !aligned16(k_pool) || !aligned16(v_pool)) return HC_ERR_INVALID;
  if (!stride_ok(dtype, sb) || !stride_ok(dtype, sh) || !stride_ok(dtype, vsb) || !stride_ok(dtype, vsh))
    return HC_ERR_INVALID;
  if (q_stage) {
    if (bsz != 1 || !q || n_q_heads <= 0 || !aligned16(q) || !aligned16(q_stage) || !stride_ok(dtype, qsh))
      return HC_ERR_INVALID;
  } else {
    n_q_heads = 0;
  }
  return note_cuda(hc::decode_append_dispatch(dtype, bsz * num_kv_heads, num_kv_heads, k, v, sb, sh, vsb, vsh, k_pool,
                                              v_pool, n_pool_blocks, block_table, max_blocks, heads_len, free_blocks,
                                              n_free, free_ptr, q, qsh, n_q_heads, q_stage, err_flag,
                                              (cudaStream_t)stream));
}

size_t hc_flash_decode_workspace_size(int bsz, int num_kv_heads, int groups, int head_dim) {
  (void)head_dim;
  if (bsz <= 0 || num_kv_heads <= 0 || groups <= 0) return 0;
  return hc::flash_decode_ws_bytes(bsz * num_kv_heads, groups);
}

int hc_flash_decode(int dtype, int bsz, int num_kv_heads, int groups, int head_dim, const void* q, int64_t qsb,
                    int64_t qsh, const void* k_pool, const void* v_pool, int n_pool_blocks,
                    const int32_t* block_table, int max_blocks, const int32_t* heads_len, float scale, void* out, long long total_tokens_hint, void* workspace,
                    size_t workspace_bytes, int32_t* err_flag, void* stream) {
  (void)total_tokens_hint;
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || bsz <= 0 || num_kv_heads <= 0 || groups <= 0 || max_blocks <= 0)
    return HC_ERR_INVALID;
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(out)) return HC_ERR_INVALID;
  if (!stride_ok(dtype, qsb) || !stride_ok(dtype, qsh)) return HC_ERR_INVALID;
  hc::FDParams p;
  std::memset(&p, 0, sizeof(p));
  p.q = q;
  p.qsb = qsb;
  p.qsh = qsh;
  p.kp = k_pool;
  p.vp = v_pool;
  p.bt = block_table;
  p.max_blocks = max_blocks;
  p.n_blocks = n_pool_blocks;
  p.heads_len = heads_len;
  p.R = bsz * num_kv_heads;
  p.KV = num_kv_heads;
  p.G = groups;
  const float sc = scale > 0.f ? scale : (float)(1.0 / std::sqrt((double)head_dim));
  p.scale_log2 = sc * 1.4426950408889634f;
  p.out = out;
  p.err = err_flag;
  return note_cuda(hc::flash_decode_dispatch(dtype, p, workspace, workspace_bytes, (cudaStream_t)stream));
}

}  // extern "C"

namespace {
// The parameters of a decode launch that also attends to the step's new token
// (hc_flash_decode_with_new, hc_flash_decode_peer); HC_OK or the error.
int with_new_params(hc::FDParams& p, int dtype, int bsz, int num_kv_heads, int groups, int head_dim, const void* q,
                    int64_t qsb, int64_t qsh, const void* k_pool, const void* v_pool, int n_pool_blocks,
                    const int32_t* block_table, int max_blocks, const int32_t* heads_len, const void* k_new,
                    const void* v_new, int64_t kn_sb, int64_t kn_sh, int64_t vn_sb, int64_t vn_sh, float scale,
                    void* out, void* q_stage, int32_t* err_flag, bool need_new = true) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || bsz <= 0 || num_kv_heads <= 0 || groups <= 0 || max_blocks <= 0)
    return HC_ERR_INVALID;
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(out)) return HC_ERR_INVALID;
  if (need_new ? (!k_new || !v_new) : (!k_new != !v_new)) return HC_ERR_INVALID;
  if (q_stage && (bsz != 1 || !k_new)) return HC_ERR_INVALID;
  if (!stride_ok(dtype, qsb) || !stride_ok(dtype, qsh)) return HC_ERR_INVALID;
  std::memset(&p, 0, sizeof(p));
  p.q = q;
  p.qsb = qsb;
  p.qsh = qsh;
  p.kp = k_pool;
  p.vp = v_pool;
  p.bt = block_table;
  p.max_blocks = max_blocks;
  p.n_blocks = n_pool_blocks;
  p.heads_len = heads_len;
  p.R = bsz * num_kv_heads;
  p.KV = num_kv_heads;
  p.G = groups;
  const float sc = scale > 0.f ? scale : (float)(1.0 / std::sqrt((double)head_dim));
  p.scale_log2 = sc * 1.4426950408889634f;
  p.out = out;
  p.err = err_flag;
  p.k_new = k_new;
  p.v_new = v_new;
  p.kn_sb = kn_sb;
  p.kn_sh = kn_sh;
  p.vn_sb = vn_sb;
  p.vn_sh = vn_sh;
  p.q_stage = q_stage;
  return HC_OK;
}
}  // namespace

extern "C" {

int hc_flash_decode_with_new(int dtype, int bsz, int num_kv_heads, int groups, int head_dim, const void* q,
                             int64_t qsb, int64_t qsh, const void* k_pool, const void* v_pool, int n_pool_blocks,
                             const int32_t* block_table, int max_blocks, const int32_t* heads_len,
                             const void* k_new, const void* v_new, int64_t kn_sb, int64_t kn_sh, int64_t vn_sb,
                             int64_t vn_sh, float scale, void* out, void* q_stage, void* workspace,
                             size_t workspace_bytes, int32_t* err_flag, void* stream) {
  hc::FDParams p;
  const int rc = with_new_params(p, dtype, bsz, num_kv_heads, groups, head_dim, q, qsb, qsh, k_pool, v_pool,
                                 n_pool_blocks, block_table, max_blocks, heads_len, k_new, v_new, kn_sb, kn_sh,
                                 vn_sb, vn_sh, scale, out, q_stage, err_flag);
  if (rc != HC_OK) return rc;
  return note_cuda(hc::flash_decode_dispatch(dtype, p, workspace, workspace_bytes, (cudaStream_t)stream));
}

int hc_flash_decode_peer(int dtype, int bsz, int num_kv_heads, int groups, int head_dim, const void* q,
                         int64_t qsb, int64_t qsh, const void* k_pool, const void* v_pool, int n_pool_blocks,
                         const int32_t* block_table, int max_blocks, const int32_t* heads_len, const void* k_new,
                         const void* v_new, int64_t kn_sb, int64_t kn_sh, int64_t vn_sb, int64_t vn_sh, float scale,
                         void* out, void* q_stage, int n_mirrors, void* const* mirrors, int64_t mirror_batch_stride,
                         void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream) {
  hc::FDParams p;
  const int rc = with_new_params(p, dtype, bsz, num_kv_heads, groups, head_dim, q, qsb, qsh, k_pool, v_pool,
                                 n_pool_blocks, block_table, max_blocks, heads_len, k_new, v_new, kn_sb, kn_sh,
                                 vn_sb, vn_sh, scale, out, q_stage, err_flag, false);
  if (rc != HC_OK) return rc;
  if (n_mirrors < 0 || n_mirrors > HC_MAX_PEERS || (n_mirrors > 0 && !mirrors)) return HC_ERR_INVALID;
  if (n_mirrors > 0 && mirror_batch_stride < (int64_t)num_kv_heads * groups * head_dim && bsz > 1)
    return HC_ERR_INVALID;
  for (int m = 0; m < n_mirrors; ++m) {
    if (!mirrors[m] || (reinterpret_cast<uintptr_t>(mirrors[m]) % elem_bytes(dtype)) != 0) return HC_ERR_INVALID;
    p.mirror[m] = mirrors[m];
  }
  p.n_mirror = n_mirrors;
  p.mirror_sb = mirror_batch_stride;
  return note_cuda(hc::flash_decode_dispatch(dtype, p, workspace, workspace_bytes, (cudaStream_t)stream));
}

int hc_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) return HC_ERR_INVALID;
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static GetRange get_range = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_range = reinterpret_cast<GetRange>(f);
  });
  if (!get_range) return HC_ERR_UNSUPPORTED;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (get_range(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS) return HC_ERR_INVALID;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return note_cuda(HC_ERR_CUDA);
  std::memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)((CUdeviceptr)ptr - base);
  return HC_OK;
}

int hc_ipc_open(const void* handle, void** base) {
  if (!handle || !base) return HC_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return note_cuda(HC_ERR_CUDA);
  // the mapping must be known to this process as device memory
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess || a.type != cudaMemoryTypeDevice) {
    (void)cudaGetLastError();
    (void)cudaIpcCloseMemHandle(p);
    return HC_ERR_UNSUPPORTED;
  }
  *base = p;
  return HC_OK;
}

int hc_ipc_close(void* base) {
  if (!base) return HC_ERR_INVALID;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? HC_OK : note_cuda(HC_ERR_CUDA);
}

int hc_enable_peer_access(int peer_device) {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceCount(&n) != cudaSuccess) return note_cuda(HC_ERR_CUDA);
  if (peer_device < 0 || peer_device >= n) return HC_ERR_INVALID;
  if (peer_device == dev) return HC_OK;
  int can = 0;
  if (cudaDeviceCanAccessPeer(&can, dev, peer_device) != cudaSuccess) return note_cuda(HC_ERR_CUDA);
  if (!can) return HC_ERR_UNSUPPORTED;
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();  // not an error here
    return HC_OK;
  }
  return e == cudaSuccess ? HC_OK : note_cuda(HC_ERR_CUDA);
}

int hc_peer_barrier(int rank, int world, int32_t* const* peer_flags, int32_t* counter, int32_t* err_flag,
                    void* stream) {
  if (world <= 0 || world > HC_MAX_PEERS || rank < 0 || rank >= world || !peer_flags || !counter || !err_flag)
    return HC_ERR_INVALID;
  for (int r = 0; r < world; ++r)
    if (!peer_flags[r] || (reinterpret_cast<uintptr_t>(peer_flags[r]) & 3u) != 0) return HC_ERR_INVALID;
  return note_cuda(hc::peer_barrier_dispatch(rank, world, peer_flags, counter, err_flag, (cudaStream_t)stream));
}

int hc_peer_put(int n_segments, const int32_t* const* segments, const int64_t* segment_words, int n_dst,
                int32_t* const* dsts, void* stream) {
  if (n_segments <= 0 || n_segments > HC_MAX_PUT_SEGMENTS || n_dst < 0 || n_dst > HC_MAX_PEERS || !segments ||
      !segment_words || (n_dst > 0 && !dsts))
    return HC_ERR_INVALID;
  for (int s = 0; s < n_segments; ++s)
    if (segment_words[s] < 0 || (segment_words[s] > 0 && !segments[s])) return HC_ERR_INVALID;
  for (int d = 0; d < n_dst; ++d)
    if (!dsts[d] || (reinterpret_cast<uintptr_t>(dsts[d]) & 3u) != 0) return HC_ERR_INVALID;
  return note_cuda(hc::peer_put_dispatch(n_segments, segments, segment_words, n_dst, dsts, (cudaStream_t)stream));
}

int hc_flash_decode_noalloc(int dtype, int bsz, int num_kv_heads, int groups, int head_dim, const void* q,
                            int64_t qsb, int64_t qsh, const void* k_pool, const void* v_pool, int n_pool_blocks,
                            const int32_t* block_table, int max_blocks, const int32_t* heads_len, float scale,
                            void* out, int32_t* err_flag, void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || bsz <= 0 || num_kv_heads <= 0 || groups <= 0 || max_blocks <= 0)
    return HC_ERR_INVALID;
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(out)) return HC_ERR_INVALID;
  if (!stride_ok(dtype, qsb) || !stride_ok(dtype, qsh)) return HC_ERR_INVALID;
  hc::FDParams p;
  std::memset(&p, 0, sizeof(p));
  p.q = q;
  p.qsb = qsb;
  p.qsh = qsh;
  p.kp = k_pool;
  p.vp = v_pool;
  p.bt = block_table;
  p.max_blocks = max_blocks;
  p.n_blocks = n_pool_blocks;
  p.heads_len = heads_len;
  p.R = bsz * num_kv_heads;
  p.KV = num_kv_heads;
  p.G = groups;
  const float sc = scale > 0.f ? scale : (float)(1.0 / std::sqrt((double)head_dim));
  p.scale_log2 = sc * 1.4426950408889634f;
  p.out = out;
  p.err = err_flag;
  size_t need = 0;
  const int rc = hc::flash_decode_noalloc_dispatch(dtype, p, (cudaStream_t)stream, &need);
  if (rc == HC_ERR_WORKSPACE)
    std::snprintf(g_last_err, sizeof(g_last_err),
                  "hc_flash_decode_noalloc: %zu bytes of partials needed, the fixed scratch holds %u", need,
                  (unsigned)HC_NOALLOC_SCRATCH_BYTES);
  return note_cuda(rc);
}

size_t hc_drift_check_workspace_size(int dtype, int n_jobs, int steps, int seq_len, int groups) {
  if (n_jobs <= 0 || steps <= 0 || seq_len <= 0) return 0;
  return hc::score_workspace_size(dtype, n_jobs, seq_len, steps * groups, steps);
}

int hc_drift_check(int dtype, int num_kv_heads, int groups, int head_dim, int steps, int seq_len, int pooling,
                   int kernel_size, int topk, double threshold, const void* qbuf, int64_t qss, int64_t qsh,
                   const void* k_pool, int n_pool_blocks, const int32_t* block_table, int max_blocks, int n_jobs,
                   const int32_t* pivot_heads, const int32_t* ref_slots, const int32_t* max_len, int max_len_cap,
                   uint32_t* ref_bitmap, int32_t* ref_positions, int32_t* trigger, float* coeffs, double* median,
                   int32_t* retrieve_positions, void* out_scores, void* workspace, size_t workspace_bytes,
                   int32_t* err_flag, void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || num_kv_heads <= 0 || groups <= 0 || seq_len <= 0) return HC_ERR_INVALID;
  if (n_jobs == 0) return HC_OK;
  if (n_jobs < 0 || steps < 1 || steps > 7) return steps > 7 ? HC_ERR_UNSUPPORTED : HC_ERR_INVALID;
  if (topk < 0 || topk > seq_len || max_len_cap < 0) return HC_ERR_INVALID;
  if (pooling != HC_AVGPOOL && pooling != HC_MAXPOOL) return HC_ERR_INVALID;
  if (kernel_size < 1 || (kernel_size & 1) == 0 || kernel_size / 2 > 16) return HC_ERR_INVALID;
  if (steps * groups > 256) return HC_ERR_UNSUPPORTED;
  if (!aligned16(qbuf) || !aligned16(k_pool)) return HC_ERR_INVALID;
  if (!stride_ok(dtype, qss) || !stride_ok(dtype, qsh)) return HC_ERR_INVALID;
  if ((seq_len + HC_PAGE_SIZE - 1) / HC_PAGE_SIZE > max_blocks) return HC_ERR_INVALID;
  hc::ScoreParams p;
  std::memset(&p, 0, sizeof(p));
  p.mode = hc::MODE_DRIFT;
  p.L = seq_len;
  p.G = groups;
  p.W = 1;
  p.S = steps;
  p.Rq = steps * groups;
  p.pooling = pooling;
  p.ksize = kernel_size;
  p.halo = kernel_size / 2;
  p.sqrt_d = div_sqrt_d(head_dim);
  p.n_jobs = n_jobs;
  p.KV = num_kv_heads;
  p.nh = n_jobs;
  p.nsel = steps + 1;
  p.job_heads = pivot_heads;
  p.topk = topk;
  p.max_len = max_len;
  p.q = qbuf;
  p.qsb = 0;
  p.qsh = qsh;
  p.qst = qss;
  p.q_tok0 = 0;
  p.k_pool = k_pool;
  p.bt = block_table;
  p.max_blocks = max_blocks;
  p.n_blocks = n_pool_blocks;
  p.ref_slots = ref_slots;
  p.ref_bitmap = ref_bitmap;
  p.ref_positions = ref_positions;
  p.bitmap_words = (seq_len + 31) / 32;
  p.trigger = trigger;
  p.coeffs = coeffs;
  p.median = median;
  p.retrieve_positions = retrieve_positions;
  p.max_len_cap = max_len_cap;
  p.threshold = threshold;
  p.out_scores = out_scores;
  p.err = err_flag;
  return note_cuda(hc::score_dispatch(dtype, p, workspace, workspace_bytes, (cudaStream_t)stream));
}

int hc_prefill_attention(int dtype, int bsz, int num_heads, int num_kv_heads, int seq_len, int head_dim,
                         const void* q, int64_t qsb, int64_t qsh, int64_t qst, const void* k, int64_t ksb,
                         int64_t ksh, int64_t kst, const void* v, int64_t vsb, int64_t vsh, int64_t vst, float scale,
                         void* out, int64_t osb, int64_t osh, int64_t ost, int32_t* err_flag, void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (dtype == HC_F32) return HC_ERR_UNSUPPORTED;
  if (head_dim != HC_HEAD_DIM || bsz <= 0 || num_heads <= 0 || num_kv_heads <= 0 || seq_len < 0) return HC_ERR_INVALID;
  if (num_heads % num_kv_heads != 0) return HC_ERR_INVALID;
  if (seq_len == 0) return HC_OK;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return HC_ERR_INVALID;
  const int64_t strides[] = {qsb, qsh, qst, ksb, ksh, kst, vsb, vsh, vst, osb, osh, ost};
  for (int64_t x : strides)
    if (x <= 0 || !stride_ok(dtype, x)) return HC_ERR_INVALID;
  hc::PAParams p;
  std::memset(&p, 0, sizeof(p));
  p.out = out;
  p.osb = osb;
  p.osh = osh;
  p.ost = ost;
  p.L = seq_len;
  p.H = num_heads;
  p.KV = num_kv_heads;
  p.G = num_heads / num_kv_heads;
  p.bsz = bsz;
  const double sc = scale > 0.f ? (double)scale : 1.0 / std::sqrt((double)head_dim);
  p.scale_log2 = (float)(sc * 1.4426950408889634);
  p.err = err_flag;
  return note_cuda(hc::prefill_attn_dispatch(dtype, p, q, qsb, qsh, qst, k, ksb, ksh, kst, v, vsb, vsh, vst,
                                             (cudaStream_t)stream));
}

int hc_drift_check_batch_per_launch(int dtype, int n_jobs, int steps, int seq_len, int groups,
                                    int jobs_per_launch) {
  if (!valid_dtype(dtype) || steps < 1 || steps > 7 || groups <= 0 || steps * groups > 256) return 0;
  return hc::drift_batch_per_launch(dtype, n_jobs, seq_len, steps * groups, steps, jobs_per_launch);
}

size_t hc_drift_check_batch_workspace_size(int dtype, int n_jobs, int steps, int seq_len, int groups,
                                           int jobs_per_launch) {
  const int per = hc_drift_check_batch_per_launch(dtype, n_jobs, steps, seq_len, groups, jobs_per_launch);
  if (per <= 0) return 0;
  // the launches take `per` jobs, the last one the remainder
  size_t ws = hc::score_workspace_size(dtype, per, seq_len, steps * groups, steps);
  const int rem = n_jobs % per;
  if (rem) ws = std::max(ws, hc::score_workspace_size(dtype, rem, seq_len, steps * groups, steps));
  return ws;
}

int hc_drift_check_batch(int dtype, int num_kv_heads, int groups, int head_dim, int steps, int seq_len, int pooling,
                         int kernel_size, int topk, double threshold, const hc_drift_job* jobs, int n_jobs,
                         int jobs_per_launch, void* workspace, size_t workspace_bytes, int32_t* err_flag,
                         void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || num_kv_heads <= 0 || groups <= 0 || seq_len <= 0) return HC_ERR_INVALID;
  if (n_jobs == 0) return HC_OK;
  if (n_jobs < 0 || !jobs || steps < 1 || steps > 7) return steps > 7 ? HC_ERR_UNSUPPORTED : HC_ERR_INVALID;
  if (topk < 0 || topk > seq_len) return HC_ERR_INVALID;
  if (pooling != HC_AVGPOOL && pooling != HC_MAXPOOL) return HC_ERR_INVALID;
  if (kernel_size < 1 || (kernel_size & 1) == 0 || kernel_size / 2 > 16) return HC_ERR_INVALID;
  if (steps * groups > 256) return HC_ERR_UNSUPPORTED;
  const int pages = (seq_len + HC_PAGE_SIZE - 1) / HC_PAGE_SIZE;
  for (int j = 0; j < n_jobs; ++j) {
    const hc_drift_job& d = jobs[j];
    if (!aligned16(d.qbuf) || !aligned16(d.k_pool) || !d.block_table || d.n_pool_blocks <= 0) return HC_ERR_INVALID;
    if (!stride_ok(dtype, d.qss) || !stride_ok(dtype, d.qsh)) return HC_ERR_INVALID;
    if (pages > d.max_blocks || d.pivot_head < 0 || d.pivot_head >= num_kv_heads) return HC_ERR_INVALID;
    if (d.max_len < 0 || d.max_len > seq_len || (d.max_len > 0 && !d.retrieve_positions)) return HC_ERR_INVALID;
    if (!d.ref_bitmap || (topk > 0 && !d.ref_positions) || !d.trigger) return HC_ERR_INVALID;
    for (int i = 0; i < j; ++i)
      if (jobs[i].ref_bitmap == d.ref_bitmap) return HC_ERR_INVALID;
  }
  const int per = hc::drift_batch_per_launch(dtype, n_jobs, seq_len, steps * groups, steps, jobs_per_launch);
  if (per <= 0) return HC_ERR_INVALID;
  for (int j0 = 0; j0 < n_jobs; j0 += per) {
    const int n = std::min(per, n_jobs - j0);
    hc::DriftBatch b;
    std::memset(&b, 0, sizeof(b));
    b.n = n;
    for (int i = 0; i < n; ++i) {
      const hc_drift_job& d = jobs[j0 + i];
      hc::DriftJob& o = b.job[i];
      o.q = d.qbuf;
      o.qst = d.qss;
      o.qsh = d.qsh;
      o.k_pool = d.k_pool;
      o.bt = d.block_table;
      o.n_blocks = d.n_pool_blocks;
      o.max_blocks = d.max_blocks;
      o.head = d.pivot_head;
      o.max_len = d.max_len;
      o.bitmap = d.ref_bitmap;
      o.ref_pos = d.ref_positions;
      o.trigger = d.trigger;
      o.retr = d.retrieve_positions;
      o.coeffs = d.coeffs;
      o.median = d.median;
      o.out_scores = d.out_scores;
    }
    hc::ScoreParams p;
    std::memset(&p, 0, sizeof(p));
    p.mode = hc::MODE_DRIFT;
    p.L = seq_len;
    p.G = groups;
    p.W = 1;
    p.S = steps;
    p.Rq = steps * groups;
    p.pooling = pooling;
    p.ksize = kernel_size;
    p.halo = kernel_size / 2;
    p.sqrt_d = div_sqrt_d(head_dim);
    p.n_jobs = n;
    p.KV = num_kv_heads;
    p.nh = n;
    p.nsel = steps + 1;
    p.topk = topk;
    p.bitmap_words = (seq_len + 31) / 32;
    p.threshold = threshold;
    p.err = err_flag;
    const int rc = hc::score_dispatch(dtype, p, workspace, workspace_bytes, (cudaStream_t)stream, &b);
    if (rc != HC_OK) return note_cuda(rc);
  }
  return HC_OK;
}

int hc_retrieve(int dtype, int num_kv_heads, int head_dim, int n_members, const int32_t* member_job,
                const int32_t* member_head, const int32_t* member_len, int max_member_len, const int32_t* trigger,
                const int32_t* retrieve_positions, int retrieve_stride, const void* full_k, const void* full_v,
                int64_t fsh, int64_t fst, void* k_pool, void* v_pool, int n_pool_blocks,
                const int32_t* block_table, int max_blocks, int32_t* err_flag, void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || num_kv_heads <= 0 || n_members < 0 || max_blocks <= 0) return HC_ERR_INVALID;
  if (n_members == 0) return HC_OK;
  if (!aligned16(full_k) || !aligned16(full_v) || !aligned16(k_pool) || !aligned16(v_pool)) return HC_ERR_INVALID;
  if (!stride_ok(dtype, fsh) || !stride_ok(dtype, fst)) return HC_ERR_INVALID;
  return note_cuda(hc::retrieve_dispatch(dtype, n_members, member_job, member_head, member_len, max_member_len,
                                         trigger, retrieve_positions, retrieve_stride, full_k, full_v, fsh, fst,
                                         k_pool, v_pool, n_pool_blocks, block_table, max_blocks, err_flag,
                                         (cudaStream_t)stream));
}

int hc_retrieve_delta(int dtype, int num_kv_heads, int head_dim, int n_members, const int32_t* member_job,
                      const int32_t* member_head, const int32_t* member_len, const int32_t* member_stage_offset,
                      const int32_t* reuse_len, int max_member_len, const int32_t* trigger,
                      const int32_t* retrieve_positions, int retrieve_stride, int32_t* slot_positions,
                      int slot_stride, const void* full_k, const void* full_v, int64_t fsh, int64_t fst,
                      void* k_pool, void* v_pool, int n_pool_blocks, const int32_t* block_table, int max_blocks,
                      void* stage_k, void* stage_v, int32_t* stage_src, int64_t stage_rows, int32_t* err_flag,
                      void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (head_dim != HC_HEAD_DIM || num_kv_heads <= 0 || n_members < 0 || max_blocks <= 0 || slot_stride < 0 ||
      stage_rows < 0)
    return HC_ERR_INVALID;
  if (n_members == 0) return HC_OK;
  if (!aligned16(full_k) || !aligned16(full_v) || !aligned16(k_pool) || !aligned16(v_pool) ||
      !aligned16(stage_k) || !aligned16(stage_v))
    return HC_ERR_INVALID;
  if (!stride_ok(dtype, fsh) || !stride_ok(dtype, fst)) return HC_ERR_INVALID;
  return note_cuda(hc::retrieve_delta_dispatch(dtype, member_job, member_head, member_len, member_stage_offset,
                                               reuse_len, n_members, max_member_len, trigger, retrieve_positions,
                                               retrieve_stride, slot_positions, slot_stride, full_k, full_v, fsh, fst,
                                               k_pool, v_pool, n_pool_blocks, block_table, max_blocks, stage_k,
                                               stage_v, stage_src, stage_rows, err_flag, (cudaStream_t)stream));
}

size_t hc_profile_topk_workspace_size(int bsz, int effective_heads, int use_len) {
  if (bsz <= 0 || effective_heads <= 0 || use_len <= 0) return 0;
  return hc::profile_topk_ws_bytes(bsz * effective_heads, use_len + 1);
}

int hc_profile_topk(int dtype, int bsz, int saved_heads, int groups, int q_len, int seq_len, const void* attn,
                    int64_t sb, int64_t sh, int64_t sq, int64_t st, int use_len, int topk, uint32_t* bitmaps,
                    int64_t words, void* workspace, size_t workspace_bytes, void* stream) {
  if (!valid_dtype(dtype)) return HC_ERR_DTYPE;
  if (bsz < 0 || saved_heads <= 0 || groups <= 0 || saved_heads % groups != 0 || q_len <= 0 || seq_len < 0 ||
      use_len < 0 || use_len > seq_len || topk < 0 || words < 0)
    return HC_ERR_INVALID;
  const int He = saved_heads / groups;
  const int64_t rows = (int64_t)bsz * He;
  if (rows == 0) return HC_OK;
  if (!bitmaps) return HC_ERR_INVALID;
  if (rows > 0x7fffffff) return HC_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  if (use_len == 0) {  // every set empty
    if (words == 0) return HC_OK;
    return note_cuda(cudaMemsetAsync(bitmaps, 0, (size_t)rows * words * sizeof(uint32_t), s) == cudaSuccess
                         ? HC_OK : HC_ERR_CUDA);
  }
  const int ksz = use_len < 5 ? use_len : 5;
  const int plen = use_len + 2 * (ksz / 2) - ksz + 1;
  if (words < (plen + 31) / 32) return HC_ERR_INVALID;
  if (!attn || sb <= 0 || sh <= 0 || sq <= 0 || st <= 0) return HC_ERR_INVALID;
  return note_cuda(hc::profile_topk_dispatch(dtype, attn, sb, sh, sq, st, q_len - 1, bsz, He, groups, use_len, topk,
                                             bitmaps, words, workspace, workspace_bytes, s));
}

int hc_profile_overlap(const uint32_t* a, int64_t a_stride, int na, const uint32_t* b, int64_t b_stride, int nb,
                       int64_t words, int diagonal, int32_t* counts, void* stream) {
  if (na < 0 || nb < 0 || words < 0 || (diagonal && na != nb)) return HC_ERR_INVALID;
  if (na == 0 || nb == 0) return HC_OK;
  if (!a || !b || !counts || a_stride < words || b_stride < words) return HC_ERR_INVALID;
  return note_cuda(hc::profile_overlap_dispatch(a, a_stride, na, b, b_stride, nb, words, diagonal, counts,
                                                (cudaStream_t)stream));
}

}  // extern "C"
