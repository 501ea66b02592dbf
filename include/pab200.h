/*
 * pab200.h — C ABI of the B200 (sm_100a) paged-attention decode library
 * (libpab200.so).
 *
 * The reference (lashhw/pagedattention) is a Python package whose paged
 * decode path is a Python wrapper over two Triton kernels:
 *   flash_attn_with_kvcache_wrapper_triton   src/kernel_triton.py:181-307
 *     ├─ host chunk planner                  src/kernel_triton.py:206-243
 *     ├─ _paged_attention_decode_split_kernel src/kernel_triton.py:8-117
 *     └─ _paged_attention_decode_reduce_kernel src/kernel_triton.py:120-174
 * with the eager PyTorch path (src/kernel_eager.py:29-56) as its numerics
 * reference and the argument contract in src/common.py:1-29.  This header is
 * the native boundary that replaces that wrapper: plain device pointers,
 * element strides and sizes, no framework types.  The Python mirror of the
 * reference interface (pagedattention_b200/kernel_b200.py) binds it with
 * ctypes.
 *
 * Conventions
 *  - Every pointer in pab200_decode_args is a DEVICE pointer on the current
 *    CUDA device.  Strides are in ELEMENTS, not bytes.
 *  - Calls are asynchronous on `stream`; the library never synchronises the
 *    device.  It allocates device memory only in the exchange-buffer set-up
 *    calls (pab200_exchange_buffer_create/open) and keeps no per-call state
 *    outside the caller's workspace, with one exception:
 *    pab200_decode_noalloc() runs on a fixed scratch array that is part of
 *    the library image (one per device) and whose contents persist from one
 *    call to the next.
 *  - Consecutive calls on one stream may share a workspace whatever their
 *    shapes.  A call's kernels may start while the previous call's kernels
 *    on the stream are still running (programmatic dependent launch), but
 *    until that call has finished they only read their inputs (lengths,
 *    block table, query, cache) and their own shared memory: every write to
 *    the workspace, the outputs or the cache comes after it.  Two calls that
 *    can overlap in time on the GPU (different streams with no ordering
 *    between them) must not share a workspace.
 *  - Return value: PAB200_OK (0) or a negative pab200_status code; the text of
 *    the last error on the calling thread is available from
 *    pab200_last_error().
 */
#ifndef PAB200_H_
#define PAB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PAB200_ABI_VERSION 1

/* Status codes. */
typedef enum pab200_status {
  PAB200_OK = 0,
  PAB200_ERR_INVALID_ARGUMENT = -1, /* bad shape, size or null pointer       */
  PAB200_ERR_UNSUPPORTED = -2,      /* valid but not built: dtype, D, bs, G  */
  PAB200_ERR_WORKSPACE = -3,        /* workspace missing or too small        */
  PAB200_ERR_ALIGNMENT = -4,        /* pointer or stride alignment           */
  PAB200_ERR_CUDA = -5              /* CUDA runtime / driver error           */
} pab200_status;

/* Element type of q, k_cache, v_cache and out. */
typedef enum pab200_dtype {
  PAB200_DTYPE_BF16 = 0,
  PAB200_DTYPE_F16 = 1,
  PAB200_DTYPE_F32 = 2 /* only as the output type of pab200_merge_states */
} pab200_dtype;

/* Physical layout of k_cache / v_cache.
 *  PAB200_LAYOUT_PAGES: [num_pages, block_size, head_size]; one page holds one
 *    (sequence, kv head)'s block of tokens — the reference layout,
 *    src/common.py:6-7.  A vLLM-style [num_blocks, num_kv_heads, block_size,
 *    head_size] ("HND") pool is the same memory seen as num_blocks*num_kv_heads
 *    pages, addressed with bt_page_mul = num_kv_heads, bt_page_add = 1.
 *  PAB200_LAYOUT_NHD: [num_pages, block_size, num_kv_heads, head_size]; one
 *    page holds a block of tokens for all kv heads (the layout the reference's
 *    vLLM adapter hands to flash-attn, src/kernel_vllm.py:17-26). */
typedef enum pab200_layout {
  PAB200_LAYOUT_PAGES = 0,
  PAB200_LAYOUT_NHD = 1
} pab200_layout;

/* Device-side error bits, accumulated in the workspace status word and read
 * with pab200_read_status(). */
#define PAB200_STATUS_BAD_PAGE_ID 0x1u   /* page id outside [0, num_pages)    */
#define PAB200_STATUS_SEQLEN_CLAMP 0x2u  /* seqlen > max_blocks*block_size    */
#define PAB200_STATUS_NEG_SEQLEN 0x4u    /* seqlen < 0 (treated as 0)         */
#define PAB200_STATUS_WAIT_TIMEOUT 0x8u  /* a pipeline wait hit its time limit */
#define PAB200_STATUS_APPEND_FULL 0x10u  /* kv append: no page slot left (L >= max_blocks*block_size) */

/* Arguments of one batched paged decode call.
 *
 * For sequence s in [0, num_seqs), kv head h in [0, num_kv_heads) and query
 * head g in [0, G), G = num_q_heads / num_kv_heads, the call computes
 *   out[s, h*G+g, :] = softmax(q[s, h*G+g, :] . K_{s,h}^T * softmax_scale) V_{s,h}
 * where K_{s,h}, V_{s,h} are the first L = seqlens(s,h) tokens of the pages
 *   page(s,h,i) = block_table[s*bt_stride_b + h*bt_stride_h + i*bt_stride_i]
 *                 * bt_page_mul + h * bt_page_add,      i < ceil(L/block_size)
 *   seqlens(s,h) = seqlens[s*seqlens_stride_b + h*seqlens_stride_h].
 * A sequence with L == 0 yields zeros.  This is the contract of
 * src/common.py:1-14 (with the reference's batch==1 restriction lifted: its
 * flattened [1, B*Hkv] form is the same call with num_seqs = 1). */
typedef struct pab200_decode_args {
  void* out;                 /* [num_seqs, num_q_heads, head_size], dtype    */
  const void* q;             /* [num_seqs, num_q_heads, head_size], dtype    */
  const void* k_cache;       /* see pab200_layout; contiguous                */
  const void* v_cache;       /* same shape as k_cache                        */
  const int32_t* seqlens;    /* cache_seqlens / context_lens                 */
  const int32_t* block_table;

  int32_t dtype;             /* pab200_dtype (BF16 or F16)                   */
  int32_t layout;            /* pab200_layout                                */
  int32_t num_seqs;          /* B                                            */
  int32_t num_q_heads;       /* Hq; G = Hq/Hkv with G*D <= 2048, or G <= 32
                                at D <= 128                                  */
  int32_t num_kv_heads;      /* Hkv                                          */
  int32_t head_size;         /* D: 64, 128 or 256                            */
  int32_t block_size;        /* tokens per page: 8, 16, 32 or 64             */
  int32_t max_blocks;        /* block-table entries per (seq, kv head)       */
  int64_t num_pages;         /* leading extent of k_cache / v_cache          */

  int64_t q_stride_b, q_stride_h;       /* head_size stride must be 1  */
  int64_t out_stride_b, out_stride_h;   /* head_size stride must be 1  */
  int64_t seqlens_stride_b, seqlens_stride_h;  /* h stride 0 => per-seq len */
  int64_t bt_stride_b, bt_stride_h, bt_stride_i;
  int32_t bt_page_mul, bt_page_add;

  float softmax_scale;
  /* Reference meaning (src/kernel_triton.py:206-209): target number of KV
   * chunks per kv head.  0 or 1: the library sizes the split to the device
   * (balanced token ranges over every resident warp).  n > 1: at most
   * num_seqs*num_kv_heads*n ranges. */
  int32_t num_splits;

  /* Optional cross-device mode.  When state_o is non-null the call writes,
   * instead of `out`, the normalised fp32 output state_o[s, h*G+g, :]
   * ([num_seqs, num_q_heads, head_size], contiguous) and its log-sum-exp
   * state_lse[s, h*G+g] (natural log of sum_t exp(score_t)); an empty range
   * gives o = 0, lse = -inf.  pab200_merge_states() combines such states. */
  float* state_o;
  float* state_lse;

  /* Optional cudaEvent_t handles recorded on `stream` immediately before and
   * after the main decode kernel (for kernel-only timing); may be null. */
  void* event_before;
  void* event_after;
} pab200_decode_args;

/* Bytes of workspace pab200_decode() needs for these arguments on the
 * current device (0 if the arguments are invalid; see pab200_last_error()).
 * Replaces the partial-buffer allocations of src/kernel_triton.py:232-243.
 * It grows with num_seqs * num_kv_heads and with the query group: a few MB
 * for the batches of the benchmark workloads, ~30 MB for 256 sequences x 8
 * kv heads x 8 query heads at head_size 128. */
size_t pab200_decode_workspace_size(const pab200_decode_args* args);

/* Number of kernel launches pab200_decode() makes for these arguments on the
 * current device: 3 (planner, decode, reduce), or 0 if the arguments are
 * invalid.  The reference makes 2 (plus host work, src/kernel_triton.py:
 * 245-305). */
int pab200_decode_launch_count(const pab200_decode_args* args);

/* Paged-attention decode.  Replaces flash_attn_with_kvcache_wrapper_triton
 * (src/kernel_triton.py:181-307: planner + split kernel + reduce kernel) with
 * launches on `stream`: a device-side planner (no host sync), the split-KV
 * decode kernel and a log-sum-exp reduce kernel for the heads it split
 * across warps (scheduled early by programmatic dependent launch).  Results
 * do not depend on run-time scheduling: repeated calls are bit-identical.  `workspace` is a device buffer
 * of at least pab200_decode_workspace_size() bytes, 256-byte aligned; its
 * contents need no initialisation.  `stream` is a cudaStream_t (0 = legacy
 * default stream). */
int pab200_decode(const pab200_decode_args* args, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Size of the fixed device scratch used by pab200_decode_noalloc(): 16 MiB. */
#define PAB200_NOALLOC_SCRATCH_BYTES (16u << 20)

/* pab200_decode() for callers that cannot allocate device memory.  No
 * counterpart in the reference.
 *
 * Some hosts of this library have no device allocator to hand a workspace
 * from: a plain C or foreign-language binding with no CUDA memory manager of
 * its own, or an engine whose pooling allocator has already reserved all free
 * device memory, so that a fresh cudaMalloc would fail (and where cudaMalloc /
 * cudaFree would also stall the device on every call).  This entry point takes
 * the same arguments as pab200_decode() minus the workspace and uses instead a
 * scratch array of PAB200_NOALLOC_SCRATCH_BYTES that is part of the library
 * image: every GPU that loads the library holds it until the process exits.
 * It calls no allocating routine.
 *
 * Limits and rules:
 *  - The plan is fitted to the scratch: where pab200_decode_workspace_size()
 *    exceeds PAB200_NOALLOC_SCRATCH_BYTES, the call first uses fewer
 *    run-time tail chunks per warp (results then agree with pab200_decode()
 *    to rounding, not bit for bit, because split heads merge their partial
 *    states in another grouping); calls that do not fit even without tail
 *    chunks fail with PAB200_ERR_WORKSPACE.  Use pab200_decode() with a
 *    caller workspace for those.
 *  - The first call on a device, made with that device current, looks up the
 *    scratch array's device address; make that first call before any stream
 *    capture begins.
 *  - All calls on a device share the one scratch array and it keeps the last
 *    call's contents (the planner kernel of every call re-initialises the
 *    parts that must start at zero).  Calls queued on ONE stream are ordered
 *    correctly whatever their shapes (a call writes to the scratch only
 *    after the previous call on the stream has finished).  Calls that can
 *    overlap on the GPU (different streams without ordering between them,
 *    or several host threads on different streams) race: serialise them.
 *  - pab200_read_status() does not see this scratch; device status bits of
 *    these calls are not reported. */
int pab200_decode_noalloc(const pab200_decode_args* args, void* stream);

/* The north-star signature paged_attention(out, query, key_cache,
 * value_cache, block_tables, context_lens, scale, block_size) over the
 * reference page layout: out/query [num_seqs, num_q_heads, head_size]
 * contiguous, caches [num_pages, block_size, head_size] contiguous,
 * block_tables [num_seqs, num_kv_heads, max_blocks] contiguous int32,
 * context_lens [num_seqs, num_kv_heads] contiguous int32.  Same semantics
 * and workspace rules as pab200_decode(); num_splits is 0 (the device-sized
 * split).  pab200_paged_attention_workspace_size() gives the workspace it
 * needs. */
int pab200_paged_attention(void* out, const void* query, const void* key_cache,
                           const void* value_cache, const int32_t* block_tables,
                           const int32_t* context_lens, float scale,
                           int32_t block_size, int32_t dtype, int32_t num_seqs,
                           int32_t num_q_heads, int32_t num_kv_heads,
                           int32_t head_size, int32_t max_blocks,
                           int64_t num_pages, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Workspace bytes pab200_paged_attention() needs for these sizes on the
 * current device (0 if they are invalid; see pab200_last_error()), without
 * the pointers: what the flat binding of the reference's decode wrapper
 * (src/kernel_triton.py:181-307, whose partial buffers it replaces,
 * :232-243) sizes its cached workspace with. */
size_t pab200_paged_attention_workspace_size(int32_t dtype, int32_t num_seqs,
                                             int32_t num_q_heads, int32_t num_kv_heads,
                                             int32_t head_size, int32_t block_size,
                                             int32_t max_blocks, int64_t num_pages);

/* Merge num_states partial attention states (o, lse) into `out`, the
 * log-sum-exp combination of src/kernel_triton.py:120-174 applied across
 * devices: out[r] = sum_i exp(lse_i[r] - LSE[r]) o_i[r], LSE[r] =
 * log sum_i exp(lse_i[r]); states with lse = -inf carry no weight and rows
 * whose states are all empty give zeros.  State i's outputs are the fp32 rows
 * state_o + i*o_stride ([rows, head_size], contiguous) and its log-sum-exps
 * state_lse + i*lse_stride ([rows]); strides are in floats, o_stride a
 * multiple of 4.  `out`: [rows, head_size] with row stride out_stride_row
 * (elements), type out_dtype (BF16, F16 or F32). */
int pab200_merge_states(const float* state_o, int64_t o_stride,
                        const float* state_lse, int64_t lse_stride,
                        int32_t num_states, int64_t rows, int32_t head_size,
                        void* out, int64_t out_stride_row, int32_t out_dtype,
                        void* stream);

/* Bytes of the exchange buffer each rank needs for pab200_exchange_merge():
 * two parities of `world` packed states, every float stored as a 64-bit
 * {value, epoch} word, plus one epoch counter per exchange block.  Each rank
 * allocates its buffer once (pab200_exchange_buffer_create, zero-filled) and
 * maps every peer's buffer into its address space (CUDA IPC); all ranks must
 * use the same `world`, `rows` and `head_size`. */
size_t pab200_exchange_buffer_bytes(int32_t world, int64_t rows, int32_t head_size);

/* Setup of the exchange buffers (once per process group and shape; these
 * are the only calls of the library that allocate or map device memory).
 *  create:  cudaMalloc `bytes` on the current device, zero-fill it, and write
 *           its CUDA IPC handle (64 bytes) to `ipc_handle`.
 *  open:    map a peer's buffer, given its handle, into this process on the
 *           current device (peer access enabled on first use).
 *  reset:   zero-fill a buffer (stream-ordered), e.g. on every rank after a
 *           timed-out exchange.
 *  close:   unmap a buffer mapped with open.
 *  destroy: free a buffer made by create (after every peer closed it). */
int pab200_exchange_buffer_create(size_t bytes, void** buf, void* ipc_handle);
int pab200_exchange_buffer_open(const void* ipc_handle, void** peer_buf);
int pab200_exchange_buffer_reset(void* buf, size_t bytes, void* stream);
int pab200_exchange_buffer_close(void* peer_buf);
int pab200_exchange_buffer_destroy(void* buf);

/* Context split across the GPUs of one node, fused exchange + merge: the
 * all-gather of partial states and the log-sum-exp merge of
 * src/kernel_triton.py:120-174 in one kernel over peer memory.  `state` is
 * this rank's packed state (o [rows, head_size] fp32, then lse [rows], the
 * layout paged_attention_states writes, `rows` padded to a multiple of 4);
 * `bufs` is a DEVICE array of `world` pointers to the exchange buffers of
 * ranks 0..world-1 as mapped in this process (bufs[rank] is this rank's own).
 * The kernel stores `state` into every peer's buffer over NVLink, each value
 * in one 64-bit word with the call's epoch, then writes out[rows, head_size]
 * (row stride out_stride_row, type out_dtype) from its own memory once every
 * peer's words of the same call have arrived.  A wait longer than
 * wait_limit_ns sets PAB200_STATUS_WAIT_TIMEOUT in *status and merges what
 * is there.  Every rank must call it the same number of times; after a
 * timeout all ranks must zero their buffers (pab200_exchange_buffer_reset)
 * before the next call.  No multicast objects or multimem instructions are
 * used. */
int pab200_exchange_merge(const float* state, void* const* bufs, int32_t rank,
                          int32_t world, int64_t rows, int32_t head_size,
                          void* out, int64_t out_stride_row, int32_t out_dtype,
                          int64_t wait_limit_ns, uint32_t* status, void* stream);

/* Context split across GPUs, decode and exchange in one call: the same as
 * pab200_decode(args) in state mode followed by pab200_exchange_merge() of
 * that state, with the reduce kernel of the decode folded into the exchange
 * kernel (each exchange block first merges the partial states of its own
 * rows whose heads the decode split, then exchanges).  One launch fewer and
 * no separate merge pass per call.  args->state_o / state_lse must be this
 * rank's packed state (lse stored right after o, the layout
 * pab200_exchange_merge() reads); `workspace` and the exchange arguments
 * follow pab200_decode() and pab200_exchange_merge().  The reference has no
 * multi-device code: this replaces an all-gather of the states followed by
 * the reduce of src/kernel_triton.py:120-174 applied across devices. */
int pab200_decode_exchange(const pab200_decode_args* args, void* workspace,
                           size_t workspace_bytes, void* const* bufs, int32_t rank,
                           int32_t world, void* out, int64_t out_stride_row, int32_t out_dtype,
                           int64_t wait_limit_ns, uint32_t* status, void* stream);

/* Arguments of pab200_kv_append(): the step before a decode, writing each
 * (sequence, kv head)'s new token into its page.  Cache layout, block-table
 * addressing and seqlens strides mean what they mean in pab200_decode_args. */
typedef struct pab200_kv_append_args {
  void* k_cache;             /* see pab200_layout                              */
  void* v_cache;
  const void* k_new;         /* [num_seqs, num_kv_heads, head_size], dtype     */
  const void* v_new;
  int32_t* seqlens;          /* current lengths L; L + 1 afterwards if increment */
  const int32_t* block_table;
  uint32_t* status;          /* device word: PAB200_STATUS_* bits ORed in; may be null */

  int32_t dtype, layout;
  int32_t num_seqs, num_kv_heads, head_size, block_size, max_blocks;
  int64_t num_pages;
  int64_t new_stride_b, new_stride_h;          /* of k_new / v_new; head_size stride 1 */
  int64_t seqlens_stride_b, seqlens_stride_h;  /* h stride 0 => per-seq length        */
  int64_t bt_stride_b, bt_stride_h, bt_stride_i;
  int32_t bt_page_mul, bt_page_add;
  int32_t increment;         /* 1: seqlens[s, h] += 1 after the write             */
} pab200_kv_append_args;

/* KV append.  No counterpart in the reference (its decode only reads the
 * cache; its benchmark fills the cache once, scripts/benchmark.py:101-108):
 * for every (sequence s, kv head h) with current length L = seqlens(s,h),
 * writes k_new[s,h,:] / v_new[s,h,:] into row L % block_size of page
 * page(s,h,L / block_size) (the addressing of pab200_decode_args) and, with
 * increment, stores L + 1.  A slot past max_blocks sets
 * PAB200_STATUS_APPEND_FULL, a page id outside [0, num_pages) sets
 * PAB200_STATUS_BAD_PAGE_ID, and that (s, h) is left untouched (length
 * included).  With a per-sequence length (seqlens_stride_h == 0) the length
 * is incremented once per sequence.  One launch, asynchronous on `stream`. */
int pab200_kv_append(const pab200_kv_append_args* args, void* stream);

/* Append, then decode, in one call: the same as pab200_kv_append(app)
 * followed by pab200_decode(args) on the same stream, with the append done
 * by the decode call's planner (one launch fewer per serving step, and it
 * keeps the planner's overlap with the previous call).  `app` must address
 * the caches, block table and lengths of `args` (same pointers, layout and
 * strides; PAB200_ERR_INVALID_ARGUMENT otherwise); its status pointer is
 * ignored: append bits go to the workspace status word.  The step's
 * flash-attn-style counterpart is flash_attn_with_kvcache(..., k, v, ...);
 * the reference wrapper (src/common.py:1-14) has no append. */
int pab200_decode_append(const pab200_decode_args* args, const pab200_kv_append_args* app,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Copy the device status word of `workspace` (the PAB200_STATUS_* bits raised
 * by the most recent pab200_decode call on it) to *status_out.  Synchronises
 * `stream`. */
int pab200_read_status(const void* workspace, uint32_t* status_out,
                       void* stream);

/* Static text for a pab200_status code. */
const char* pab200_strerror(int status);

/* Detail of the last failed call on this thread ("" if none). */
const char* pab200_last_error(void);

/* PAB200_ABI_VERSION of the loaded library. */
int pab200_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PAB200_H_ */
