// launch.h — internal launchers of the indexer kernels (host side).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace dsai {

struct ScoreLaunch {
  const float* weights;
  const int32_t* seq_lens;
  const int32_t* block_table;
  float* logits;      // [rows, ld]
  uint32_t* hist;     // [rows, kHistStride] first-digit histograms (zero on entry)
  int* status;
  int rows;
  int max_pages;
  int num_pages;
  int ld;             // row stride of logits in floats (max_pages * 64)
  int row_base;       // first row of this launch inside the q tensor map
  int score_all;
  int grid;
};

// Scores every scored row's tokens into `logits`.  The tensor maps describe
// q ([rows*64, 128] u8, SW128), the K pages ([num_pages, 64, 128] u8, SW128)
// and the per-token scales ([num_pages, 64] f32).
cudaError_t launch_score(const ScoreLaunch& p, const CUtensorMap& tmap_q, const CUtensorMap& tmap_k,
                         const CUtensorMap& tmap_s, cudaStream_t stream);

// The same scoring for groups of `rows_per_group` (2-4) consecutive rows that
// read one block-table row (the group's longest row's): each K tile is staged
// once and multiplied against the whole group.  `p.rows` is a multiple of
// rows_per_group; `p.grid` is the number of CTAs (one per SM).
cudaError_t launch_score_groups(const ScoreLaunch& p, int rows_per_group, const CUtensorMap& tmap_q,
                                const CUtensorMap& tmap_k, const CUtensorMap& tmap_s, cudaStream_t stream);

struct FusedLaunch {
  const float* weights;
  const int32_t* seq_lens;
  const int32_t* block_table;
  float* logits;      // [rows, ld]
  uint32_t* hist;     // [rows, kHistStride] (zero on entry, left zero)
  int* ws;            // workspace header (status word and the selectors' control words)
  int32_t* out_ids;   // [rows, 2048]
  int rows;           // at most kMaxRowsPerLaunch
  int max_pages;
  int num_pages;
  int ld;
  int score_all;
  int keep_logits;    // 1: `logits` is the caller's buffer (left holding the logits)
  int sms;
};

// Scoring and top-2048 selection of many rows in one persistent launch
// (fused.cu): scorer CTAs over an interleaved tile schedule, selector CTAs
// that select each row as soon as its scoring completes.  Opt-in:
// fused_enabled() is true only with DSAI_FUSED=1 in the environment (it is
// slower than the two-launch path on the benchmark shapes).
// `logits` must hold fused_logits_sentinel() in every 32-bit word the call
// writes (rows x seq_len) on entry; without keep_logits the call leaves it so.
bool fused_enabled();
uint32_t fused_logits_sentinel();
cudaError_t launch_fused(const FusedLaunch& p, const CUtensorMap& tmap_q, const CUtensorMap& tmap_k,
                         const CUtensorMap& tmap_s, cudaStream_t stream);

struct AttnLaunch {
  const void* q_nope;
  const void* q_pe;
  const void* ckv;
  const void* kpe;
  const int32_t* idx;
  void* out;
  float* lse;
  void* workspace;   // 256-B status header, then the split partials
  float sm_scale;
  int num_tokens;
  int num_slots;
};

// Sparse MLA attention (attn.cu): splits per token and workspace bytes for
// the current device, and the launch (attention kernel, then the combine
// kernel when a token is split).
int attn_splits(int num_tokens);
size_t attn_workspace_bytes(int num_tokens);
cudaError_t launch_attn(const AttnLaunch& a, cudaStream_t stream);

struct SelectLaunch {
  const float* logits;  // [rows, ld]
  int ld;
  uint32_t* hist;       // [rows, kHistStride] from the scoring launch; cleared here
  uint32_t* cand;       // [rows, 2, kSplitCap] pivot-bin lists of the split selection
  const int32_t* seq_lens;
  const int32_t* block_table;
  int rows;
  int max_pages;
  int* status;
  // Output: either physical ids, or (score, token + token_offset) pairs.
  int32_t* out_ids;
  float* out_scores;
  int32_t* out_tokens;
  int32_t token_offset;
  int sms;              // SMs of the device (sizes the clusters)
};

// Shape of the selection launch: threads per CTA and CTAs per row (the
// cluster size).
struct SelectShape {
  int threads;
  int cluster;
};
SelectShape select_shape(int rows, int max_pages, int sms);

cudaError_t launch_select(const SelectLaunch& p, cudaStream_t stream);

cudaError_t launch_short_rows(const int32_t* seq_lens, const int32_t* block_table, int rows,
                              int max_pages, int32_t* out, cudaStream_t stream);

cudaError_t launch_wait_selftest(int* status, unsigned long long timeout_ns, cudaStream_t stream);

cudaError_t launch_merge(const float* scores, const int32_t* tokens, int n_cand,
                         const int32_t* bt_row, int max_pages, const int32_t* seq_len,
                         int32_t* out, cudaStream_t stream);

// Index-K cache writer (csrc/writer.cu): quantises n new keys (fp32, or bf16
// when bf16) and stores them at their physical slot ids.
cudaError_t launch_write_k(const void* k_new, bool bf16, const int32_t* slot_ids, int n, uint8_t* k_cache,
                           int num_pages, cudaStream_t stream);

// Records `msg` as the calling thread's dsai_last_error() and returns code.
int set_last_error(int code, const char* msg);

int score_smem_bytes();
int select_smem_bytes();

}  // namespace dsai
