// Launch parameter blocks and host dispatch entry points shared by the
// kernels and the C ABI layer.
#pragma once

#include <type_traits>

#include "hc_common.cuh"

namespace hc {

// ---- fused scoring / selection (score_select.cu)
constexpr int kSThreads = 512;  // one CTA per SM (cooperative grid)
constexpr int kRefWords = 512;  // reference-bitmap words staged per CTA (16K tokens)
constexpr int kSWarps = kSThreads / 32;
constexpr int kMargin = 16;
constexpr int kMaxSel = 8;
constexpr int kMaxRq = 256;
constexpr int kMaxRows = 7;

enum { MODE_PREFILL = 0, MODE_PIVOT = 1, MODE_DRIFT = 2 };

struct ScoreParams {
  int mode, L, G, W, S, Rq, pooling, ksize, halo;
  float sqrt_d;
  int n_jobs, cpj, T, TB, KV, nh, first_head, nsel;
  const int32_t* job_heads;
  const int32_t* keep_lens;
  int topk;
  const int32_t* max_len;
  const void* q;
  int64_t qsb, qsh, qst;
  int q_tok0;
  const void* k;
  const void* v;
  int64_t ksb, ksh, kst;
  int64_t vsb, vsh, vst;
  const void* k_pool;
  const int32_t* bt;
  int max_blocks;
  int n_blocks;
  void* k_pool_out;
  void* v_pool_out;
  int32_t* heads_len;
  int32_t* out_indices;
  int32_t* keep_pos;  // workspace: prefill kept positions [job][rank] (set at launch)
  int max_keep;
  // PREFILL only.  Lsel: positions [0, Lsel) are pooled and may be selected
  // (L for HeteroCache; L - window for SnapKV, whose window rows are kept
  // whole).  keep_const: the keep length of every head when keep_lens is
  // null.  tail: the last `tail` key/value rows follow each head's kept rows.
  // out_job_rows > 0: dense output, job j's rows start at row j*out_job_rows
  // of k_pool_out / v_pool_out (else flat slots from the row's first page).
  int Lsel;
  int keep_const;
  int tail;
  int64_t out_job_rows;
  void* out_scores;
  int64_t out_job_stride;  // elements between jobs' score rows (set in the kernel)
  const int32_t* ref_slots;
  uint32_t* ref_bitmap;
  int32_t* ref_positions;
  int bitmap_words;
  int32_t* trigger;
  float* coeffs;
  double* median;
  int32_t* retrieve_positions;
  int max_len_cap;
  double threshold;
  GridBarrier* gb;
  float2* part;
  unsigned int* hist;
  int2* cnt;
  unsigned int* overlap;
  void* glogits;
  int logits_in_smem;
  // tensor-core logits (16-bit dtypes): tcgen05.mma from TMA-fed key tiles;
  // n_stages shared-memory stages of 128 keys, NP query rows padded to 16,
  // tmem_cols tensor-memory columns (two accumulators of NP columns)
  int umma, n_stages, NP, tmem_cols;
  int32_t* err;
  uint64_t wait_ns;    // grid-barrier wait limit (set at dispatch)
  unsigned int stall;  // injected grid-barrier arrival that never comes (tests of the timeout path)
};

// A batch of drift checks (hc_drift_check_batch): per job its own query
// buffer, key pool, page table, reference set and outputs.  Passed to the
// kernel by value (kernel parameter space), so a captured graph holds it.
struct DriftJob {
  const void* q;
  int64_t qst, qsh;
  const void* k_pool;
  const int32_t* bt;
  int n_blocks, max_blocks;
  int head, max_len;
  uint32_t* bitmap;   // reference bitmap row
  int32_t* ref_pos;   // reference position row (topk entries)
  int32_t* trigger;   // one entry
  int32_t* retr;      // max_len entries
  float* coeffs;      // S entries or null
  double* median;     // one entry or null
  void* out_scores;   // [S, L] pooled scores or null
};
constexpr int kDriftBatchMax = 16;
struct DriftBatch {
  int n;  // 0: a single hc_drift_check launch (job-indexed arrays of ScoreParams)
  DriftJob job[kDriftBatchMax];
};
struct NoBatch {
  int n;
};

// Process-wide limits of the device-side waits (hc_set_wait_limits): the
// limit to use given a wait's default, and the injected stall (0 or 1).
uint64_t wait_limit_ns(uint64_t dflt);
unsigned int injected_stall();

size_t score_workspace_size(int dtype, int n_jobs, int L, int Rq, int S);
// Jobs per drift-check batch launch: `want` (or the default when <= 0),
// capped at kDriftBatchMax and n_jobs, lowered until the plan's shared memory
// fits.
int drift_batch_per_launch(int dtype, int n_jobs, int L, int Rq, int S, int want);
// batch: the jobs of one drift-check batch launch (MODE_DRIFT, p.n_jobs ==
// batch->n), else null.
int score_dispatch(int dtype, ScoreParams& p, void* ws, size_t ws_bytes, cudaStream_t st,
                   const DriftBatch* batch = nullptr);

// ---- paged flash-decode (decode_attn.cu)
constexpr int kMaxPeers = 8;  // GPUs of one node a head-sharded output is mirrored to
constexpr int kFThreads = 128;
constexpr int kFWarps = 4;
constexpr int kGMax = 8;
constexpr int kMaxRowsFD = 4096;

struct FDParams {
  const void* q;
  int64_t qsb, qsh;
  const void* kp;
  const void* vp;
  const int32_t* bt;
  int max_blocks;
  int n_blocks;
  const int32_t* heads_len;
  int R, KV, G;
  int gran;  // rows are padded to, and CTA spans cut at, multiples of this many tokens
  float scale_log2;
  float* part_o;
  float2* part_ml;
  // optional: one more token per row, not in the pages yet (k_new/v_new
  // [bsz, KV, 1, D] with batch and head strides); the combine merges it
  const void* k_new;
  const void* v_new;
  int64_t kn_sb, kn_sh, vn_sb, vn_sh;
  // optional (batch of one): the combine also stores the query rows here [H, D]
  void* q_stage;
  void* out;
  // optional: copies of the output in other GPUs' memory (peer pointers over
  // NVLink): element (b, query head j, d) also goes to mirror[m] + b *
  // mirror_sb + j * D + d
  int n_mirror;
  int64_t mirror_sb;
  void* mirror[kMaxPeers];
  int32_t* err;
  uint64_t wait_ns;  // mbarrier wait limit (set at dispatch)
};

size_t flash_decode_ws_bytes(int R, int G);
// One step barrier across the GPUs of a head-sharded cache: the caller's
// counter + 1 stored into slot `rank` of every rank's flags, then a wait
// until every slot of this rank's flags holds at least that value.
constexpr int kMaxPutSegs = 4;
int peer_put_dispatch(int n_seg, const int32_t* const* srcs, const int64_t* seg_words, int n_dst,
                      int32_t* const* dsts, cudaStream_t st);
int peer_barrier_dispatch(int rank, int world, int32_t* const* peer_flags, int32_t* counter, int32_t* err,
                          cudaStream_t st);
int flash_decode_dispatch(int dtype, FDParams& p, void* ws, size_t ws_bytes, cudaStream_t st);
int flash_decode_noalloc_dispatch(int dtype, FDParams& p, cudaStream_t st, size_t* need_out);

// ---- causal prefill attention (prefill_attn.cu)
struct PAParams {
  void* out;
  int64_t osb, osh, ost;  // element strides of out [bsz, heads, L, D] (any order)
  int L, H, KV, G, bsz;
  int n_qt;               // 128-query tiles (set at dispatch)
  float scale_log2;       // softmax scale times log2(e)
  int32_t* err;
  uint64_t wait_ns;       // mbarrier wait limit (set at dispatch)
  unsigned int stall;     // injected stall: no key tile is loaded (tests of the timeout path)
};
int prefill_attn_dispatch(int dtype, PAParams& p, const void* q, int64_t qsb, int64_t qsh, int64_t qst,
                          const void* k, int64_t ksb, int64_t ksh, int64_t kst, const void* v, int64_t vsb,
                          int64_t vsh, int64_t vst, cudaStream_t st);

// ---- page copies (kv_copy.cu)
int prefill_keep_dispatch(int dtype, int bsz, int KV, int L, const int32_t* keep, int n_keep, const void* k,
                          const void* v, int64_t sb, int64_t sh, int64_t st, int64_t vsb, int64_t vsh, int64_t vst,
                          void* kp, void* vp, int nblocks, const int32_t* bt, int mb, int32_t* hl, int32_t* err,
                          cudaStream_t s);
int decode_append_dispatch(int dtype, int R, int KV, const void* k, const void* v, int64_t sb, int64_t sh,
                           int64_t vsb, int64_t vsh, void* kp, void* vp, int nblocks, int32_t* bt, int mb, int32_t* hl,
                           const int32_t* fb, int nf, int32_t* fp, const void* q, int64_t qsh, int nq, void* q_stage,
                           int32_t* err, cudaStream_t s);
int retrieve_dispatch(int dtype, int n_members, const int32_t* mj, const int32_t* mh, const int32_t* ml, int max_len,
                      const int32_t* trig, const int32_t* pos, int pos_stride, const void* fk, const void* fv,
                      int64_t fsh, int64_t fst, void* kp, void* vp, int nblocks, const int32_t* bt, int mb,
                      int32_t* err, cudaStream_t s);

int retrieve_delta_dispatch(int dtype, const int32_t* mj, const int32_t* mh, const int32_t* ml, const int32_t* moff,
                            const int32_t* reuse, int n_members, int max_len, const int32_t* trig, const int32_t* pos,
                            int pos_stride, int32_t* slot_pos, int slot_stride, const void* fk, const void* fv,
                            int64_t fsh, int64_t fst, void* kp, void* vp, int nb, const int32_t* bt, int mb,
                            void* stage_k, void* stage_v, int32_t* stage_src, int64_t stage_rows, int32_t* err,
                            cudaStream_t s);

// ---- offline head profiler (profile.cu)
size_t profile_topk_ws_bytes(int rows, int plen);
int profile_topk_dispatch(int dtype, const void* attn, int64_t sb, int64_t sh, int64_t sq, int64_t st, int q_last,
                          int bsz, int He, int G, int use_len, int topk, uint32_t* bits, int64_t words, void* ws,
                          size_t ws_bytes, cudaStream_t s);
int profile_overlap_dispatch(const uint32_t* a, int64_t as, int na, const uint32_t* b, int64_t bs, int nb,
                             int64_t words, int diagonal, int32_t* counts, cudaStream_t s);

}  // namespace hc
