// Launchers of the per-layer and speculation kernels (internal).
//
// Every per-row kernel works on a set of "rows": a row is one token of one
// stream at one position. Rows are described by a device array of RowInfo;
// the number of active rows is static (M) or read from device memory (m_dev)
// when it is produced on the device inside a CUDA graph. Each stream has its
// own KV cache (StreamKV); many streams can share one forward pass.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "tp.cuh"

namespace rai {

constexpr int kMaxRowsPerStream = 33;  // max_draft <= 32 (rai run's --lookup-k limit) + 1
constexpr int kScoreChunk = 256;       // positions per attention-score CTA
constexpr int kSegRows = 16;           // max rows per attention segment
// Rows per segment in a decode step: a stream's verify rows (1 .. k+1 of
// them) are cut into pieces this long so every attention CTA carries about
// the same work; prompt rows (uniform) use kSegRows.
constexpr int kStepSegRows = 2;

struct RowInfo {
  int pos;     // position of the row's token
  int stream;  // index into the StreamKV / StreamStep arrays
};

// A run of rows of one stream at consecutive positions pos0 .. pos0 + nrows - 1
// (nrows <= kSegRows): the unit the attention kernels share K/V reads over.
struct AttnSeg {
  int row0;
  int nrows;
  int stream;
  int pos0;
};

// One stream's cache: [layer][kv_head][max_ctx][head_dim] f32.
struct StreamKV {
  float* k;
  float* v;
  int max_ctx;
  int pad;
};

// One stream's state in a decode step. The host writes pos and ctx_len; the
// kernels write the rest; the host reads it back once per step.
struct StreamStep {
  int pos, ctx_len;
  int n_rows;   // verify rows: drafted + 1
  int drafted;
  int ngram;    // matched n-gram length, 0 = none
  int accepted, produced;
  int row0;     // first compacted row of this stream in the step's forward
  uint32_t tokens[kMaxRowsPerStream];  // [last, draft_0 .. draft_{k-1}]
  uint32_t out[kMaxRowsPerStream];     // produced tokens
  // Sampled acceptance: the decoder's seed and its step count (the
  // random-number counter of this step).
  uint32_t rng_seed_lo, rng_seed_hi, rng_step_lo, rng_step_hi;
};

// Dynamic shared memory the attention kernels may use (the opt-in limit of
// 227 KB less static shared memory and a margin).
constexpr size_t kAttnMaxSmem = 224 * 1024;

// Raise the dynamic shared-memory limit of the attention kernels (once per
// process, before any stream capture).
cudaError_t init_layer_attributes();

// epoch (tensor parallelism, may be null): [0] += 1 per forward, [1] += 1
// when it ends in logits.
cudaError_t launch_embed(const uint32_t* ids, const int* m_dev, int M, const uint8_t* codes,
                         const uint8_t* params, int vocab, int hidden, int gs, float embed_scale,
                         float* out, uint32_t* err, cudaStream_t s, uint32_t* epoch = nullptr,
                         bool with_logits = false);
cudaError_t launch_qkv_post(float* qkv, int ld, float* q_out, int nh, int nkv, int hd, const float* qn,
                            const float* kn, int qk_mode, float eps, const float* rope_cos,
                            const float* rope_sin, const StreamKV* kv, int layer, const RowInfo* rows,
                            const int* m_dev, int M, cudaStream_t s);
// Attention over each row's own stream cache (positions 0..pos inclusive).
// segs: the rows grouped into segments (*nseg_dev of them when set, else
// nseg_max); seg_rows bounds nrows over the segments. scores:
// [M][nh][n_alloc] f32 scratch (holds p on return).
size_t attention_n_chunks(int n_alloc);
cudaError_t launch_attention(const float* q, float* out, const StreamKV* kv, int layer, const RowInfo* rows,
                             const int* m_dev, int M, const AttnSeg* segs, const int* nseg_dev, int nseg_max,
                             int seg_rows, int nh, int nkv, int hd, float scale, float softcap, float* scores,
                             int n_alloc, const ExpfTable& et, uint32_t* err, cudaStream_t s);
// Group host rows into segments (runs of one stream at consecutive
// positions, at most seg_len <= kSegRows long); returns the count (<= M).
int build_segments(const RowInfo* rows, int M, int seg_len, AttnSeg* segs);
// Tensor parallelism: logits are vocabulary rows vocab_off.. of the model and
// the keys go to every rank's best[] (peers, n_peers of them, own included).
cudaError_t launch_argmax(const float* logits, int vocab, const int* m_dev, int M, unsigned long long* best,
                          cudaStream_t s, int vocab_off = 0, unsigned long long* const* peers = nullptr,
                          int n_peers = 0);
// Draft search for each of n streams; ctx for stream i at ctx + i * ctx_cap.
cudaError_t launch_ngram(const uint32_t* ctx, int ctx_cap, StreamStep* st, const StreamKV* kv, int n,
                         int max_draft, int max_ngram, int min_ngram, cudaStream_t s);
// Compact the streams' verify rows: rows / ids / *m_active, attention
// segments / *n_segs; zero best[].
cudaError_t launch_plan(StreamStep* st, int n, RowInfo* rows, uint32_t* ids, int* m_active, AttnSeg* segs,
                        int* n_segs, int seg_len, unsigned long long* best, int best_len, cudaStream_t s);
// Sampled acceptance (temperature > 0) of every stream from its verify rows'
// logits (vocab wide): accept / correction / bonus tokens and counts, as
// launch_accept does for greedy.
// draft_logits (optional, one stream): the draft model's logits per draft
// row for speculative decoding; null = the point mass of prompt lookup.
cudaError_t launch_sample_accept(StreamStep* st, int n, const float* logits, int vocab, float temperature,
                                 cudaStream_t s, const float* draft_logits = nullptr);
// out[i] = expf_host of the float with bit pattern first + i (i < n): the
// library's reproduction of the host libm expf, for an exhaustive check.
cudaError_t launch_expf_range(uint32_t first, size_t n, float* out, const ExpfTable& et, cudaStream_t s);
// With tp (world > 1) and slot >= 0, best[] is awaited as exchange `slot`.
cudaError_t launch_accept(StreamStep* st, int n, const unsigned long long* best, cudaStream_t s,
                          const TpLink* tp = nullptr, int slot = -1, uint32_t* err = nullptr);

}  // namespace rai
