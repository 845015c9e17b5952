/*
 * dsai.h — C ABI of the B200 (sm_100a) DSA lightning indexer.
 *
 * The operator: for every row b and token t in [0, seq_lens[b]) with
 *   page = block_table[b, t/64], slot = t % 64,
 *   S[h]       = sum_d q[b,h,d] * K[page,slot,d]          (e4m3 x e4m3, fp32 accumulate)
 *   logit[b,t] = scale[page,slot] * sum_h ReLU(S[h]) * weights[b,h]
 *   out[b,:]   = physical slot ids (page*64 + slot) of the 2048 largest logits,
 *                rows with seq_len <= 2048 get ids of t = 0..seq_len-1 in
 *                token order followed by -1 padding.
 *
 * Each entry point below replaces a piece of the reference's interface; the
 * citation is given beside it (paths inside the reference project).
 *
 * Page layout in the index-K cache (k_cache, declared [num_pages,64,1,132] u8):
 *   bytes [0, 8192)     64 tokens x 128 e4m3 values, token-major
 *   bytes [8192, 8448)  64 little-endian fp32 scales
 *
 * All pointers are device pointers unless stated otherwise. Calls are
 * asynchronous on `stream` and never synchronise the host; nothing is read
 * back from the device.  Every function returns 0 (DSAI_OK) on success or a
 * negative DSAI_E* code; dsai_last_error() gives the message of the last
 * failure on the calling thread.
 */
#ifndef DSAI_H_
#define DSAI_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DSAI_API __attribute__((visibility("default")))
#else
#define DSAI_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DSAI_NUM_HEADS 64
#define DSAI_HEAD_DIM 128
#define DSAI_PAGE_SIZE 64
#define DSAI_TOPK 2048
#define DSAI_ATTN_HEADS 16     /* sparse MLA attention: query heads */
#define DSAI_ATTN_CKV_DIM 512  /* compressed KV (latent) dimension */
#define DSAI_ATTN_KPE_DIM 64   /* rotary key dimension */
#define DSAI_PAGE_BYTES 8448
#define DSAI_SCALE_OFFSET 8192

/* Return codes. */
#define DSAI_OK 0
#define DSAI_E_INVALID (-1)   /* bad argument: null pointer, negative size, misalignment */
#define DSAI_E_WORKSPACE (-2) /* workspace missing or smaller than dsai_workspace_size() */
#define DSAI_E_CUDA (-3)      /* a CUDA runtime / driver call failed */
#define DSAI_E_UNSUPPORTED (-4) /* device is not sm_100 or the library was built without it */

/* Element types of dsai_write_k's new keys. */
#define DSAI_DTYPE_F32 0
#define DSAI_DTYPE_BF16 1

/* Device status bits, accumulated in the workspace header by the kernels and
 * read with dsai_read_status().  They never stop a call: the kernels clamp
 * or zero-fill and carry on, so the output stays well defined. */
#define DSAI_STATUS_SEQLEN_CLAMPED 0x1 /* a seq_len was < 0 or > max_pages*64 */
#define DSAI_STATUS_BAD_PAGE 0x2       /* a block_table entry was outside [0, num_pages) */
#define DSAI_STATUS_WAIT_TIMEOUT 0x4   /* a bounded on-chip wait gave up */
#define DSAI_STATUS_BAD_INDEX 0x8      /* sparse attention: a sparse index outside [-1, num_pages*64) */

/* Flags for dsai_args.flags. */
#define DSAI_FLAG_SCORE_ALL_ROWS 0x1 /* also score rows with seq_len <= 2048 (debug logits) */
/* Launch the call's kernels as one cached CUDA graph: the executable graph is
 * kept per (device, stream, launch plan = kernels, grids, blocks, shared
 * memory), captured on the first call of a plan, and later calls write their
 * pointers and sizes into its kernel nodes and launch it (no re-capture).
 * The reference's host entry point replays every call from such a cache
 * (solution/python/kernel.cu:1101-1199, :1389-1478).  Ignored (the kernels
 * are launched directly) when ev_after_score is set, when the caller's
 * stream is itself capturing, for the opt-in fused launch, and once 64 plans
 * are cached. */
#define DSAI_FLAG_GRAPH 0x2

typedef struct dsai_args {
  const void* q;             /* [rows, 64, 128] float8_e4m3fn                         */
  const void* k_cache;       /* [num_pages, 64, 1, 132] uint8, 8448 B per page         */
  const float* weights;      /* [rows, 64] fp32                                        */
  const int32_t* seq_lens;   /* [rows] int32                                           */
  const int32_t* block_table;/* [rows, max_pages] int32                                */
  int32_t* topk_indices;     /* [rows, 2048] int32, written                            */
  float* logits_out;         /* optional [rows, max_pages*64] fp32; NULL = internal    */
  int32_t rows;
  int32_t max_pages;
  int32_t num_pages;
  int32_t flags;             /* DSAI_FLAG_*                                            */
  void* ev_after_score;      /* optional cudaEvent_t recorded after the scoring launch */
  int32_t rows_per_seq;      /* 0 or 1: rows independent.  2-4: consecutive groups of
                                that many rows are query tokens of one sequence (multi-
                                query decode, next-n / MTP, causal prefill rows): they
                                must agree on block_table over every page each of them
                                reaches, and each group's K pages are read once, through
                                the block_table row of its longest row.  rows must be a
                                multiple of it.  No counterpart in the reference, whose
                                rows are always scored one by one
                                (solution/python/kernel.cu:1208-1479).              */
} dsai_args;

/* Bytes of device workspace dsai_run needs for these sizes (256-B aligned
 * base required): a status header, per row a 4096-bin histogram with four
 * counters and a 4096-entry list of (key, id) pairs, and the fp32 logits.
 * Replaces the reference's per-device fp16 logits scratch
 * (solution/python/kernel.cu:1299-1323).  A workspace serves one call at a
 * time: calls that may overlap on the GPU need separate workspaces. */
DSAI_API size_t dsai_workspace_size(int32_t rows, int32_t max_pages);

/* Zero a workspace (status word, histograms and counters).  Call once after
 * allocating it; every call leaves them zero again, and the status
 * word is sticky until dsai_read_status. */
DSAI_API int dsai_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* The indexer, destination-passing.  Replaces the reference's extension op
 * `run` / dsa_topk_indexer_cuda (solution/python/kernel.cu:1208-1479) that
 * solution.py::kernel (solution/python/solution.py:25-26) forwards to, and the
 * TVM-FFI export `kernel` (solution/cuda/kernel.cu:430-507). */
DSAI_API int dsai_run(const dsai_args* args, void* workspace, size_t workspace_bytes,
             void* stream);

/* Executable graphs held by the DSAI_FLAG_GRAPH cache (all devices and
 * streams).  The reference keeps its cache internal
 * (solution/python/kernel.cu:1133-1199); exported here so that callers and
 * tests can see whether calls replay a cached plan or capture new ones. */
DSAI_API int dsai_graph_cache_entries(void);

/* Per-row top-2048 as (fp32 score, token index + token_offset) pairs, for a
 * caller that merges several partial rows (a long row split by page range
 * across GPUs).  Rows with seq_len <= 2048 give all their tokens, padded with
 * (-inf, -1).  No reference counterpart: the reference is single-GPU; this
 * is the local half of the page-range split. */
DSAI_API int dsai_run_pairs(const dsai_args* args, int32_t token_offset,
                   float* out_scores, int32_t* out_tokens, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Merge n_cand (score, token) candidates of ONE row into its top-2048
 * physical slot ids, using that row's full block table (bt_row, max_pages
 * entries) and its seq_len.  Token -1 marks padding.  When the row has
 * seq_len <= 2048 the output is token order then -1, as dsai_run gives.
 * No reference counterpart (the merge half of the page-range split). */
DSAI_API int dsai_merge_pairs(const float* scores, const int32_t* tokens, int32_t n_cand,
                     const int32_t* bt_row, int32_t max_pages,
                     const int32_t* seq_len, int32_t* out, void* stream);

/* The indexer for callers that cannot allocate device memory (a host that
 * owns all device allocations and forbids plugins to call cudaMalloc, a
 * serving loop that bans allocation after warm-up, a binding without a
 * device allocator).  Same arguments and results as dsai_run, but no
 * workspace: it uses a 16 MiB device array built into the library, held on
 * every GPU that loads it until the process exits.  Calls needing more than
 * 16 MiB of workspace (dsai_workspace_size) fail with DSAI_E_WORKSPACE.
 * The first call on a device looks up and zeroes the array (make it before
 * any stream capture).  All calls on a device share the array: calls whose
 * work can overlap on the GPU race and must be serialised.  No counterpart
 * in the reference. */
DSAI_API int dsai_run_noalloc(const dsai_args* args, void* stream);

/* The status word of dsai_run_noalloc's built-in array on the current
 * device, as dsai_read_status gives it for a workspace: copied to
 * *status_out (host), then cleared; 0 before the first call on the device.
 * Synchronises `stream`.  No counterpart in the reference. */
DSAI_API int dsai_noalloc_read_status(void* stream, int32_t* status_out);

/* Index-K cache writer: quantises n_tokens new keys k_new [n_tokens, 128]
 * (fp32 or bf16, row-major) to e4m3 with one fp32 scale per token
 * (scale = max(max_d |k|, 1e-12) / 448, values clamp(k / scale, +-448),
 * round to nearest even) and stores token i at physical slot id
 * slot_ids[i] = page*64 + slot of k_cache (the page layout above): 128 bytes
 * at page*8448 + slot*128 and the scale at page*8448 + 8192 + slot*4.  Ids of
 * -1 and ids outside [0, num_pages*64) are skipped.  k_new 16-B (fp32) or
 * 8-B (bf16) aligned, k_cache 16-B aligned.  Two tokens with the same id race.
 * No counterpart in the reference, which reads this cache but does not
 * write it; the format is the one it reads (solution/python/kernel.cu:29-40). */
DSAI_API int dsai_write_k(const void* k_new, int32_t dtype, const int32_t* slot_ids, int32_t n_tokens,
                          void* k_cache, int32_t num_pages, void* stream);

/* Copy the workspace status word to *status_out (host), then clear it.
 * Synchronises `stream`. */
DSAI_API int dsai_read_status(void* workspace, void* stream, int32_t* status_out);

/* Sparse MLA attention over the indexer's output: the operator after the
 * indexer in a DSA decode step (dsa_sparse_attention_h16_ckv512_kpe64_
 * topk2048_ps64).  No counterpart in this reference, which names it as the
 * next stage (final_writeup.md:27-41); its published definition is
 * flashinfer 0.6.11.post2 `_dsa_paged_reference`.  For token t and head h,
 * over the entries i of sparse_indices[t] that are not -1 (flat slot ids
 * page*64 + slot, as dsai_run writes them):
 *   s_i = (q_nope[t,h] . ckv[i] + q_pe[t,h] . kpe[i]) * sm_scale
 *   output[t,h] = sum_i softmax(s)_i ckv[i]   (bf16)
 *   lse[t,h]    = log2(sum_i exp(s_i))        (fp32; -inf, with output 0,
 *                                              when no entry is valid)
 * Indices outside [0, num_pages*64) other than -1 count as padding and set
 * DSAI_STATUS_BAD_INDEX in the workspace status word. */
typedef struct dsai_attn_args {
  const void* q_nope;            /* [T, 16, 512] bf16                          */
  const void* q_pe;              /* [T, 16, 64] bf16                           */
  const void* ckv_cache;         /* [num_pages, 64, 512] bf16                  */
  const void* kpe_cache;         /* [num_pages, 64, 64] bf16                   */
  const int32_t* sparse_indices; /* [T, 2048] int32                            */
  void* output;                  /* [T, 16, 512] bf16, written                 */
  float* lse;                    /* [T, 16] fp32 (base 2), written             */
  float sm_scale;
  int32_t num_tokens;            /* T (at most 65535)                          */
  int32_t num_pages;
} dsai_attn_args;

/* Bytes of workspace dsai_sparse_attn needs for num_tokens on the current
 * device (256-B header with the status word, plus the per-split partial
 * results when tokens are split across CTAs).  Zero the header once after
 * allocating; the status word is sticky until dsai_read_status. */
DSAI_API size_t dsai_sparse_attn_workspace_size(int32_t num_tokens);

/* The sparse attention, destination-passing, on `stream`. */
DSAI_API int dsai_sparse_attn(const dsai_attn_args* args, void* workspace, size_t workspace_bytes,
                              void* stream);

/* Self-test of failure detection: launches one kernel that waits on an
 * on-chip barrier nothing will complete, bounded by timeout_ns (at most 1 s);
 * the wait gives up and sets DSAI_STATUS_WAIT_TIMEOUT in the workspace status
 * word, as a stalled indexer kernel would, and the context stays usable.
 * Read the result with dsai_read_status.  No reference counterpart (the
 * reference's waits spin without bound, solution/python/tcgen05_ptx.h:164-167). */
DSAI_API int dsai_selftest_wait_timeout(void* workspace, uint64_t timeout_ns, void* stream);

/* Message of the last failure on this thread ("" if none). */
DSAI_API const char* dsai_last_error(void);

/* Library version string. */
DSAI_API const char* dsai_version(void);

#ifdef __cplusplus
}
#endif

#endif /* DSAI_H_ */
