/*
 * heterocache_b200.h -- C ABI of the B200 (sm_100a) compressed-KV attention path.
 *
 * One entry point per operation of HeteroCache's cache object and patched
 * attention (ponytaill/HeteroCache, heterocache/cache_utils.py and
 * heterocache/llama_model.py).  Every argument is a plain pointer, size,
 * stride or scalar; no framework type crosses this boundary.
 *
 * Conventions
 *   - All tensor pointers are device pointers (or, where stated, host memory
 *     the GPU can address: pinned host memory under unified addressing).
 *   - Strides are in ELEMENTS; the innermost (head_dim) stride is always 1.
 *   - A "row" of the page table is one (batch, kv-head) pair: row = b*KV + h.
 *   - Pages hold HC_PAGE_SIZE tokens; a pool is [n_blocks, 256, 1, head_dim],
 *     i.e. token (page p, slot s) lives at element ((p*256)+s)*head_dim.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *   - Return value: HC_OK or an hc_status code.  Launch errors return
 *     HC_ERR_CUDA; conditions detected on the device (free list exhausted,
 *     page-table entry out of range, a bounded wait that gave up) are OR-ed
 *     into the caller's int32 `err_flag` on the device and read back by the
 *     caller after the stream has progressed.
 *   - Every op that needs scratch takes a caller-owned workspace; query its
 *     size with the matching *_workspace_size function.  Workspaces must be
 *     zero-filled once when first allocated (the grid barrier they hold
 *     resets itself after each launch).
 *   - Only head_dim == 128 is supported (Llama-3.x and Qwen2.x).
 *   - n_pool_blocks is the pool's first dimension; every page id read from a
 *     block table is checked against it on the device (out of range ->
 *     HC_ERR_RANGE in err_flag, the access is skipped).
 */
#ifndef HETEROCACHE_B200_H
#define HETEROCACHE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HC_PAGE_SIZE 256
#define HC_HEAD_DIM 128
#define HC_ABI_VERSION 1

typedef enum hc_status {
  HC_OK = 0,
  HC_ERR_INVALID = 1,     /* bad shape, size or argument */
  HC_ERR_DTYPE = 2,       /* unsupported element type */
  HC_ERR_OOM = 3,         /* decode free list exhausted ("Layer N OOM.") */
  HC_ERR_RANGE = 4,       /* page-table entry or index out of range */
  HC_ERR_CUDA = 5,        /* CUDA runtime error at launch */
  HC_ERR_WORKSPACE = 6,   /* workspace missing or too small */
  HC_ERR_TIMEOUT = 7,     /* a bounded device-side wait gave up */
  HC_ERR_UNSUPPORTED = 8  /* valid request outside what this build implements */
} hc_status;

typedef enum hc_dtype { HC_F32 = 0, HC_BF16 = 1, HC_F16 = 2 } hc_dtype;
typedef enum hc_pooling { HC_AVGPOOL = 0, HC_MAXPOOL = 1 } hc_pooling;

/* Library identity and diagnostics. */
int hc_abi_version(void);
const char* hc_status_string(int status);
/* Last CUDA error string seen by this library on the calling thread. */
const char* hc_last_cuda_error(void);

/* Limits of the device-side waits.  Every wait of this library's kernels --
 * the scoring kernels' grid barriers, flash-decode's mbarrier waits on its
 * TMA ring -- gives up after `limit_ns` nanoseconds, ORs HC_ERR_TIMEOUT into
 * the launch's err_flag and leaves the kernel (no wait is unbounded).
 * limit_ns = 0 restores the defaults (2 s for a grid barrier, 1 s for an
 * mbarrier).  inject_stall != 0 makes every grid barrier of the scoring
 * kernels wait for one arrival that never comes, and the prefill attention
 * load no key tile, so the limit runs out:
 * fault injection for tests of the timeout path (a workspace of a launch
 * that timed out must be zero-filled again before its next use).  Process-
 * wide, for launches made after the call (a captured graph keeps the values
 * of its capture).  No counterpart in the reference, whose waits are those
 * of PyTorch and flash-attn.  Returns HC_OK. */
int hc_set_wait_limits(unsigned long long limit_ns, int inject_stall);

/* ---------------------------------------------------------------------------
 * Prefill: keep-head copy.  Replaces the prefill branch of HeteroCache.update
 * (heterocache/cache_utils.py:900-937): the volatile and pivot heads are
 * copied whole into their pages and heads_len[row] = L.
 *   k: [bsz, KV, L, D] strided (sb, sh, st); v likewise with (vsb, vsh, vst).
 *   keep_heads: device int32[n_keep].
 */
int hc_prefill_keep(int dtype, int bsz, int num_kv_heads, int seq_len, int head_dim,
                    const int32_t* keep_heads, int n_keep,
                    const void* k, const void* v, int64_t sb, int64_t sh, int64_t st,
                    int64_t vsb, int64_t vsh, int64_t vst,
                    void* k_pool, void* v_pool, int n_pool_blocks, const int32_t* block_table,
                    int max_blocks, int32_t* heads_len, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Prefill: compressed-head selection.  Replaces HeteroCache.prefill_select
 * (heterocache/cache_utils.py:782-882) and, for window > 1, the observation
 * window scoring of SnapKVCluster.update_kv (heterocache/kv_cluster.py:160-178).
 * Heads 0..n_heads-1 (anchor + satellite, which the role order puts first)
 * are scored from the last `window` queries of their G query heads; head h
 * keeps its top keep_lens[h] positions, written in ascending position order
 * from flat pool slot block_table[row, 0]*256 on (the prefill pages of a row
 * are contiguous, as the reference lays them out and writes them,
 * cache_utils.py:735-747 and :862-877); heads_len[row] = keep_lens[h].
 *   q: [bsz, H, L, D] strided (qsb, qsh, qst), k: [bsz, KV, L, D] strided
 *   (sb, sh, st), v: same shape strided (vsb, vsh, vst).  Only query token
 *   positions L - window .. L - 1 are read (q's token axis aligned with k's);
 *   a caller holding only the last queries passes q rebased by that many
 *   positions so that those reads stay inside its buffer.
 *   keep_lens: device int32[n_heads].
 *   out_indices (optional, may be NULL): int32 [bsz, n_heads, max_keep],
 *     kept positions ascending, -1 padded.
 *   out_scores (optional, may be NULL): [bsz, n_heads, L] pooled scores in
 *     the model dtype (the values the selection ranks).
 */
size_t hc_prefill_select_workspace_size(int dtype, int bsz, int n_heads, int seq_len, int groups, int window);
int hc_prefill_select(int dtype, int bsz, int num_kv_heads, int groups, int seq_len, int head_dim,
                      int n_heads, int window, int pooling, int kernel_size,
                      const void* q, int64_t qsb, int64_t qsh, int64_t qst,
                      const void* k, const void* v, int64_t sb, int64_t sh, int64_t st,
                      int64_t vsb, int64_t vsh, int64_t vst,
                      const int32_t* keep_lens, int max_keep,
                      void* k_pool, void* v_pool, int n_pool_blocks, const int32_t* block_table,
                      int max_blocks, int32_t* heads_len, int32_t* out_indices, void* out_scores,
                      void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Prefill: SnapKV compression of one layer.  Replaces
 * SnapKVCluster.update_kv (heterocache/kv_cluster.py:155-199) once the
 * caller has decided to compress (capacity <= seq_len; the reference returns
 * its inputs unchanged otherwise).  For every (batch row, head): the last
 * `window` queries score all seq_len keys (q.K^T / sqrt(D) in the model
 * dtype, the in-window causal mask, fp32 softmax cast to the dtype), the
 * window rows are summed, the sums of positions 0 .. seq_len-window-1 are
 * pooled (avg_pool1d with count_include_pad, or max_pool1d; kernel_size odd,
 * padding kernel_size/2) and the top (capacity - window) of them are kept.
 *   q: [bsz, H, L, D] strided (qsb, qsh, qst; only the last `window`
 *   positions are read, aligned with k as in hc_prefill_select); k, v:
 *   [bsz, H, L, D] strided (one key head per query head, as the reference's
 *   matmul requires).
 *   out_k, out_v: contiguous [bsz, H, capacity, D]: per head the kept rows
 *   in ascending position order, then the last `window` rows.  (The
 *   reference orders the kept rows by descending score; attention over the
 *   rows does not depend on their order.)
 *   out_indices (optional): int32 [bsz, H, capacity - window], kept
 *   positions ascending.  out_scores (optional): [bsz, H, L] pooled scores in
 *   the model dtype at positions 0 .. L-window-1 (the rest is not written).
 * Ties at the k-th score go to the lowest positions (torch.topk leaves their
 * order unspecified).  1 <= window < seq_len, window <= 256,
 * window <= capacity <= seq_len.
 */
size_t hc_snapkv_update_kv_workspace_size(int dtype, int bsz, int num_heads, int seq_len, int window);
int hc_snapkv_update_kv(int dtype, int bsz, int num_heads, int seq_len, int head_dim, int window, int pooling,
                        int kernel_size, int capacity,
                        const void* q, int64_t qsb, int64_t qsh, int64_t qst,
                        const void* k, const void* v, int64_t sb, int64_t sh, int64_t st,
                        int64_t vsb, int64_t vsh, int64_t vst,
                        void* out_k, void* out_v, int32_t* out_indices, void* out_scores,
                        void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Prefill: pivot reference sets.  Replaces HeteroCache.init_coefficient
 * (heterocache/cache_utils.py:1149-1190): pivot heads first_pivot ..
 * first_pivot+n_pivots-1 (contiguous after the role permutation) are scored
 * from the last query and their top-`topk` positions become the reference
 * set, stored both as ascending positions ref_positions [bsz, n_pivots, topk]
 * and as a bitmap ref_bitmap [bsz, n_pivots, ceil(L/32)] (uint32 words).
 * q is read at token position L - 1 only (as in hc_prefill_select).
 */
size_t hc_pivot_init_workspace_size(int dtype, int bsz, int n_pivots, int seq_len, int groups);
int hc_pivot_init(int dtype, int bsz, int num_kv_heads, int groups, int seq_len, int head_dim,
                  int first_pivot, int n_pivots, int pooling, int kernel_size, int topk,
                  const void* q, int64_t qsb, int64_t qsh, int64_t qst,
                  const void* k, int64_t sb, int64_t sh, int64_t st,
                  int32_t* ref_positions, uint32_t* ref_bitmap, void* out_scores,
                  void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Decode: append one token per row.  Replaces the decode branch of
 * HeteroCache.update (heterocache/cache_utils.py:970-1005).  Rows whose next
 * slot falls in an unmapped page (-1) take pages from free_blocks in row
 * order starting at *free_ptr (device int32); if the free list would
 * overflow nothing is written and HC_ERR_OOM is OR-ed into err_flag.
 *   k: [bsz, KV, 1, D] strided (sb, sh); v likewise with (vsb, vsh).
 * Optionally (q_stage non-null, bsz == 1) the same launch also stores the
 * step's query q [1, n_q_heads, 1, D] (head stride qsh) into q_stage
 * [n_q_heads, D]: the slot of the per-step query buffer that decode_select
 * keeps for the drift check (heterocache/cache_utils.py:1011-1017 appends
 * each decode query and concatenates decode_step of them), so that store
 * costs no launch of its own.
 */
int hc_decode_append(int dtype, int bsz, int num_kv_heads, int head_dim,
                     const void* k, const void* v, int64_t sb, int64_t sh, int64_t vsb, int64_t vsh,
                     void* k_pool, void* v_pool, int n_pool_blocks, int32_t* block_table, int max_blocks,
                     int32_t* heads_len, const int32_t* free_blocks, int n_free, int32_t* free_ptr,
                     const void* q, int64_t qsh, int n_q_heads, void* q_stage,
                     int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Decode attention.  Replaces the flash_attn_with_kvcache call of the patched
 * attention (heterocache/llama_model.py:370-397, qwen_model.py:181-206):
 * non-causal attention of each row's G query heads over its first
 * heads_len[row] tokens, through the page table.  Split-K over a balanced
 * partition of all rows' tokens, then a per-row combine.
 *   q: [bsz, H, 1, D] strided (qsb, qsh); out: [bsz, H, D] contiguous
 *   (== [bsz, 1, H*D]).  scale <= 0 selects 1/sqrt(D).
 *   total_tokens_hint: sum of heads_len if the caller knows it (sizes the
 *   grid), else 0.
 */
size_t hc_flash_decode_workspace_size(int bsz, int num_kv_heads, int groups, int head_dim);
int hc_flash_decode(int dtype, int bsz, int num_kv_heads, int groups, int head_dim,
                    const void* q, int64_t qsb, int64_t qsh,
                    const void* k_pool, const void* v_pool, int n_pool_blocks, const int32_t* block_table,
                    int max_blocks, const int32_t* heads_len, float scale, void* out, long long total_tokens_hint,
                    void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Decode attention over each row's pages plus the step's own token, which is
 * not in the pages yet: the form of flash_attn_with_kvcache that takes the
 * new k and v with the cache (the call the patched attention makes is
 * llama_model.py:382-389 / qwen_model.py:194-201, after HeteroCache.update
 * has appended).  Row r attends over its heads_len[r] page tokens and
 * k_new/v_new [bsz, KV, 1, D] (batch strides kn_sb / vn_sb, head strides
 * kn_sh / vn_sh); the pages are not written, so the caller appends the token
 * afterwards (hc_decode_append) -- which lets that append run off the
 * attention's critical path.  q_stage: NULL, or (bsz 1 only) a [H,
 * head_dim] buffer in the query dtype into which the call also stores the
 * step's query rows -- the decode-step query buffer the drift check reads
 * (heterocache/cache_utils.py:1011-1017 collects the last decode_step
 * queries), so the check need not wait for the deferred append.  Arguments
 * otherwise as hc_flash_decode.
 */
int hc_flash_decode_with_new(int dtype, int bsz, int num_kv_heads, int groups, int head_dim,
                             const void* q, int64_t qsb, int64_t qsh,
                             const void* k_pool, const void* v_pool, int n_pool_blocks,
                             const int32_t* block_table, int max_blocks, const int32_t* heads_len,
                             const void* k_new, const void* v_new, int64_t kn_sb, int64_t kn_sh,
                             int64_t vn_sb, int64_t vn_sh, float scale, void* out, void* q_stage,
                             void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Head-sharded decode: the all-gather of head outputs done by the attention
 * kernels themselves.  Replaces the NCCL all-gather of per-rank head outputs
 * (the head-sharded mode has no reference counterpart: the reference runs
 * one GPU; its attention output feeds o_proj, llama_model.py:398-405).
 *
 * hc_flash_decode_peer: hc_flash_decode_with_new (k_new / v_new may both be
 * NULL: hc_flash_decode then, without q_stage), whose combine kernel also
 * stores every output element into n_mirrors other buffers (up to
 * HC_MAX_PEERS device pointers, typically other GPUs' memory mapped with
 * CUDA IPC, written over NVLink): element (b, query head j, d) goes to
 * mirrors[m] + b * mirror_batch_stride + j * head_dim + d (elements).  A
 * rank of a head-sharded cache passes, for every rank, the address of its
 * own heads' rows in that rank's gathered output.  The stores are fenced at
 * system scope; hc_peer_barrier publishes them.
 *
 * hc_peer_barrier: step barrier of `world` ranks, one launch per rank, each
 * on its own GPU (never several ranks on one GPU: they would wait on each
 * other's launches).  peer_flags[r] is rank r's int32 flag array (at least
 * `world` entries, zero at start, the same order on every rank); counter is
 * this rank's own int32 (zero at start).  The kernel stores counter + 1 into
 * slot `rank` of every rank's flags (release, system scope) and waits until
 * every slot of peer_flags[rank] holds at least that value (acquire); all
 * ranks must issue the same number of barriers.  A wait that exceeds the
 * limit of hc_set_wait_limits (default 2 s) ORs HC_ERR_TIMEOUT into err_flag
 * and returns.  Issue one before a step's mirrored stores (every rank has
 * finished reading the previous step's gathered output) and one after them
 * (every rank's output rows have landed everywhere).
 */
#define HC_MAX_PEERS 8
/* Lets kernels on the current device read and write memory that lives on
 * peer_device (cudaDeviceEnablePeerAccess), e.g. another rank's buffer mapped
 * with CUDA IPC under that device: HC_OK (also when already enabled or the
 * same device), HC_ERR_UNSUPPORTED when the two devices cannot reach each
 * other.  Call before handing such addresses to hc_flash_decode_peer or
 * hc_peer_barrier. */
int hc_enable_peer_access(int peer_device);
/* CUDA IPC of one rank's buffers, for the output mirrors and flags above.
 * hc_ipc_export: the 64-byte handle (HC_IPC_HANDLE_BYTES) of the device
 * allocation that holds `ptr` (a caching allocator's segment) and ptr's byte
 * offset in it.  hc_ipc_open (in another process): maps that allocation for
 * the current device, enabling peer access as needed, and returns its base
 * (add the offset); one open per allocation and process, undone by
 * hc_ipc_close. */
#define HC_IPC_HANDLE_BYTES 64
int hc_ipc_export(const void* ptr, void* handle, int64_t* offset);
int hc_ipc_open(const void* handle, void** base);
int hc_ipc_close(void* base);
int hc_flash_decode_peer(int dtype, int bsz, int num_kv_heads, int groups, int head_dim,
                         const void* q, int64_t qsb, int64_t qsh,
                         const void* k_pool, const void* v_pool, int n_pool_blocks,
                         const int32_t* block_table, int max_blocks, const int32_t* heads_len,
                         const void* k_new, const void* v_new, int64_t kn_sb, int64_t kn_sh,
                         int64_t vn_sb, int64_t vn_sh, float scale, void* out, void* q_stage,
                         int n_mirrors, void* const* mirrors, int64_t mirror_batch_stride,
                         void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream);
int hc_peer_barrier(int rank, int world, int32_t* const* peer_flags, int32_t* counter, int32_t* err_flag,
                    void* stream);
/* hc_peer_put: the broadcast of a pivot's trigger and position list
 * (replaces the torch.distributed.broadcast a head-sharded rank would issue;
 * the reference runs one GPU and reads the list in place,
 * heterocache/cache_utils.py:1084-1101).  Stores the concatenation of
 * n_segments int32 segments (up to HC_MAX_PUT_SEGMENTS; segment s:
 * segment_words[s] words at segments[s], device memory) into each of n_dst
 * destinations (up to HC_MAX_PEERS device pointers, 4-byte aligned, e.g.
 * other ranks' buffers mapped with hc_ipc_open), fenced at system scope: an
 * hc_peer_barrier issued after it on the same stream publishes the words to
 * the destinations' ranks.  Nothing is launched when there is no word or no
 * destination. */
#define HC_MAX_PUT_SEGMENTS 4
int hc_peer_put(int n_segments, const int32_t* const* segments, const int64_t* segment_words, int n_dst,
                int32_t* const* dsts, void* stream);

/* ---------------------------------------------------------------------------
 * Decode attention without a workspace.  No counterpart in the reference:
 * this is an addition for callers that cannot allocate device memory, such as
 * a host program whose device memory is entirely owned by another allocator,
 * or a language binding with no device allocator to call, and that therefore
 * cannot pass the workspace hc_flash_decode asks for.
 *
 * Same arguments, result and errors as hc_flash_decode, minus the workspace:
 * the split-K partials go to a fixed array of HC_NOALLOC_SCRATCH_BYTES that
 * the library defines at file scope in device memory.  Every GPU that loads
 * the library holds that array until the process exits.  The entry point
 * allocates nothing (no cudaMalloc, no cudaFree, no allocating library call).
 *   - The first call on a device looks the array's device address up
 *     (cudaGetSymbolAddress, with that device current); make that first
 *     call before any stream capture.
 *   - Requests whose partials need more than HC_NOALLOC_SCRATCH_BYTES (many
 *     rows: about 1700 batch*KV rows for 4 query heads per KV head, about 700
 *     for 8) return HC_ERR_WORKSPACE and launch nothing.
 *   - All calls share the one array, and it keeps what the last call wrote.
 *     Nothing in it has to start at zero (every partial is written before it
 *     is read).  Calls that overlap on the GPU -- on different streams, or
 *     from different host threads without ordering -- race on it; order them.
 */
#define HC_NOALLOC_SCRATCH_BYTES (4u << 20)
int hc_flash_decode_noalloc(int dtype, int bsz, int num_kv_heads, int groups, int head_dim,
                            const void* q, int64_t qsb, int64_t qsh,
                            const void* k_pool, const void* v_pool, int n_pool_blocks,
                            const int32_t* block_table, int max_blocks, const int32_t* heads_len,
                            float scale, void* out, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Decode: pivot drift check.  Replaces the scoring and overlap part of
 * HeteroCache.decode_select (heterocache/cache_utils.py:1007-1082) for
 * batch size 1.  For each job j (a pivot with at least one satellite):
 *   - score the S buffered queries of the pivot's G query heads against the
 *     pivot's first seq_len keys (read through its page-table row);
 *   - per step, top-`topk` positions and their overlap with the reference
 *     bitmap; coefficient = overlap/topk (fp32); median over the S steps;
 *   - trigger[j] = median < threshold.  On trigger the reference set slot
 *     becomes the last step's top-`topk` set (bitmap and ascending positions).
 *   - always: retrieve_positions[j, 0..max_len[j]) = the last step's
 *     top-max_len[j] positions in ascending order.
 *   qbuf: [S, H, D] strided (qss, qsh).  pivot_heads, ref_slots, max_len:
 *   device int32[n_jobs].  coeffs: float[n_jobs, S] (optional), median:
 *   double[n_jobs] (optional).
 */
size_t hc_drift_check_workspace_size(int dtype, int n_jobs, int steps, int seq_len, int groups);
int hc_drift_check(int dtype, int num_kv_heads, int groups, int head_dim, int steps, int seq_len,
                   int pooling, int kernel_size, int topk, double threshold,
                   const void* qbuf, int64_t qss, int64_t qsh,
                   const void* k_pool, int n_pool_blocks, const int32_t* block_table, int max_blocks,
                   int n_jobs, const int32_t* pivot_heads, const int32_t* ref_slots,
                   const int32_t* max_len, int max_len_cap,
                   uint32_t* ref_bitmap, int32_t* ref_positions,
                   int32_t* trigger, float* coeffs, double* median,
                   int32_t* retrieve_positions, void* out_scores,
                   void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Decode: a batch of drift checks in few launches.  Each job is the
 * computation of hc_drift_check for one pivot, with its own query buffer,
 * key pool, page table, reference set and outputs -- e.g. the checks of all
 * layers that fall due in one decode step, which the reference runs one
 * layer at a time (HeteroCache.decode_select, heterocache/cache_utils.py:
 * 1007-1082).  dtype, geometry, steps, seq_len, pooling, kernel_size, topk
 * and threshold are common to all jobs.
 *   jobs: HOST array of n_jobs descriptors, read during the call (the
 *   pointers in them are device memory).  The call launches
 *   ceil(n_jobs / per_launch) kernels on `stream`, in job order, per_launch =
 *   hc_drift_check_batch_per_launch(...).  Two jobs must not share a
 *   reference bitmap row.  The workspace is reused by the launches in turn.
 */
#define HC_DRIFT_BATCH_MAX 16
typedef struct hc_drift_job {
  const void* qbuf;            /* [S, H, D] strided, 16-byte aligned */
  int64_t qss, qsh;            /* element strides of qbuf's step and head dims */
  const void* k_pool;          /* the job's key pool [n_pool_blocks, 256, D] */
  const int32_t* block_table;  /* [num_kv_heads, max_blocks] */
  int n_pool_blocks, max_blocks;
  int pivot_head;              /* the KV head scored */
  int max_len;                 /* retrieval list length (0..seq_len) */
  uint32_t* ref_bitmap;        /* the pivot's reference bitmap: ceil(seq_len/32) words */
  int32_t* ref_positions;      /* the pivot's reference set: topk int32 */
  int32_t* trigger;            /* one int32 */
  int32_t* retrieve_positions; /* max_len int32 (the last step's top-max_len, ascending) */
  float* coeffs;               /* steps floats, or null */
  double* median;              /* one double, or null */
  void* out_scores;            /* [steps, seq_len] pooled scores (dtype), or null */
} hc_drift_job;
/* Jobs per launch: jobs_per_launch (1..HC_DRIFT_BATCH_MAX), or the
 * library's choice when <= 0, lowered until a launch's shared memory fits;
 * 0 for invalid sizes. */
int hc_drift_check_batch_per_launch(int dtype, int n_jobs, int steps, int seq_len, int groups,
                                    int jobs_per_launch);
size_t hc_drift_check_batch_workspace_size(int dtype, int n_jobs, int steps, int seq_len, int groups,
                                           int jobs_per_launch);
int hc_drift_check_batch(int dtype, int num_kv_heads, int groups, int head_dim, int steps, int seq_len,
                         int pooling, int kernel_size, int topk, double threshold,
                         const hc_drift_job* jobs, int n_jobs, int jobs_per_launch,
                         void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Prefill: causal attention over the uncompressed prompt.  Replaces the
 * flash-attn forward of the patched attention's prefill branch
 * (heterocache/llama_model.py:353-361, heterocache/qwen_model.py:161-169):
 *   out[b, h, t, :] = sum_{j <= t} softmax_j(q[b,h,t] . k[b,h/G,j] * scale) v[b,h/G,j]
 * with G = num_heads / num_kv_heads (grouped-query), fp32 accumulation,
 * output in the input dtype.  16-bit dtypes only (HC_ERR_UNSUPPORTED for
 * fp32).  scale <= 0 selects 1/sqrt(D).
 *   q: [bsz, num_heads, seq_len, D] strided (qsb, qsh, qst); k, v:
 *   [bsz, num_kv_heads, seq_len, D] strided; out: strided (osb, osh, ost) --
 *   e.g. [bsz, seq_len, num_heads, D] for the o_proj input.  All strides
 *   positive multiples of 16 bytes, pointers 16-byte aligned.
 */
int hc_prefill_attention(int dtype, int bsz, int num_heads, int num_kv_heads, int seq_len, int head_dim,
                         const void* q, int64_t qsb, int64_t qsh, int64_t qst,
                         const void* k, int64_t ksb, int64_t ksh, int64_t kst,
                         const void* v, int64_t vsb, int64_t vsh, int64_t vst,
                         float scale, void* out, int64_t osb, int64_t osh, int64_t ost,
                         int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Decode: satellite retrieval.  Replaces the retrieval part of
 * HeteroCache.decode_select (heterocache/cache_utils.py:1084-1147) for batch
 * size 1.  For member m (job member_job[m], KV head member_head[m],
 * member_len[m] tokens): if trigger[job] is set, copy rows
 * retrieve_positions[job, i] (i < member_len[m]) of that head from the full
 * tier into the pool at flat slot block_table[row, 0]*256 + i.
 * The full tier (full_k/full_v, [1, KV, L, D] strided) may be device memory
 * or pinned host memory (read directly over the host link).
 */
int hc_retrieve(int dtype, int num_kv_heads, int head_dim, int n_members,
                const int32_t* member_job, const int32_t* member_head, const int32_t* member_len,
                int max_member_len, const int32_t* trigger, const int32_t* retrieve_positions,
                int retrieve_stride,
                const void* full_k, const void* full_v, int64_t fsh, int64_t fst,
                void* k_pool, void* v_pool, int n_pool_blocks, const int32_t* block_table, int max_blocks,
                int32_t* err_flag, void* stream);

/* ---------------------------------------------------------------------------
 * Decode: satellite retrieval from a pinned-host full tier, moving only the
 * rows a satellite does not already hold.  Same pool contents as
 * hc_retrieve (heterocache/cache_utils.py:1084-1147, the host-tier branch
 * real_offload=True at :1095-1123); the reference copies every row over the
 * host link.
 *   slot_positions [n_members, slot_stride] int32: for member m, the full-tier
 *     position held in flat slot i, i < reuse_len[m] (ascending).  The caller
 *     seeds it with the satellite's prefill kept indices and must choose
 *     reuse_len[m] <= min(the satellite's prefill keep length, member_len[m]);
 *     this call keeps it up to date.
 *   stage_k/stage_v [stage_rows, D], stage_src int32 [stage_rows]: device
 *     scratch; member m uses rows member_stage_offset[m] + [0, member_len[m]).
 * Two launches on `stream`: rows found in the slot map are copied from the
 * pool to the staging area, then every slot is written from the staging area
 * or from the tier.  Members whose pivot did not trigger do nothing.
 */
int hc_retrieve_delta(int dtype, int num_kv_heads, int head_dim, int n_members,
                      const int32_t* member_job, const int32_t* member_head, const int32_t* member_len,
                      const int32_t* member_stage_offset, const int32_t* reuse_len, int max_member_len,
                      const int32_t* trigger, const int32_t* retrieve_positions, int retrieve_stride,
                      int32_t* slot_positions, int slot_stride,
                      const void* full_k, const void* full_v, int64_t fsh, int64_t fst,
                      void* k_pool, void* v_pool, int n_pool_blocks, const int32_t* block_table, int max_blocks,
                      void* stage_k, void* stage_v, int32_t* stage_src, int64_t stage_rows,
                      int32_t* err_flag, void* stream);

/*
 * Offline head profiler: top-k sets of the heads' last-query attention rows
 * (replaces get_head_topk_exact, tools/get_cluster.py:13-60, which the
 * profiler runs once per dumped layer and step).
 *   attn: one dump, [bsz, saved_heads, q_len, seq_len] with element strides
 *     (sb, sh, sq, st); only query row q_len - 1 is read.
 *   groups: 1, or num_q_heads / num_kv_heads when a GQA model's dump holds
 *     every query head (the reference's `is_gqa and num_saved_heads ==
 *     num_q_heads`): effective head h is then the mean of saved heads
 *     h * groups .. + groups - 1, taken in the dump's dtype (fp32 sum in head
 *     order divided by groups, rounded to the dtype).
 *   use_len: positions used, min(max_length, seq_len) (the reference's
 *     `[..., :max_length]`); 0 leaves every set empty.
 * Per (batch row, effective head): avg_pool1d over the row as fp32 with
 * kernel k = min(5, use_len), padding k / 2, stride 1 (zero padding counted),
 * then the top min(topk, pooled length) positions, equal values at the
 * boundary taken at the lowest positions.  Written as bitmaps
 * [bsz][saved_heads / groups][words] (bit t of word t / 32, LSB first);
 * words >= ceil((use_len + 1) / 32); bits past the pooled length are 0.
 * Workspace: hc_profile_topk_workspace_size bytes.  dtype: HC_F32 (the fp32
 * mean of more than 4 heads may differ from torch's, whose summation order is
 * vectorized, by one unit in the last place), HC_F16 or HC_BF16.
 */
size_t hc_profile_topk_workspace_size(int bsz, int effective_heads, int use_len);
int hc_profile_topk(int dtype, int bsz, int saved_heads, int groups, int q_len, int seq_len,
                    const void* attn, int64_t sb, int64_t sh, int64_t sq, int64_t st,
                    int use_len, int topk, uint32_t* bitmaps, int64_t words,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Intersection sizes of top-k bitmaps (the numerators of
 * calculate_overlap_ratio, tools/get_cluster.py:62-69): counts[i * nb + j] =
 * |a_i & b_j| for every pair, or with diagonal != 0 counts[i] = |a_i & b_i|
 * (na == nb).  a_i starts at a + i * a_stride words, b_j likewise.
 */
int hc_profile_overlap(const uint32_t* a, int64_t a_stride, int na, const uint32_t* b, int64_t b_stride, int nb,
                       int64_t words, int diagonal, int32_t* counts, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* HETEROCACHE_B200_H */
