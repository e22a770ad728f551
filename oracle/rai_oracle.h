// CPU oracle for the prompt-lookup decode path (TEST INFRASTRUCTURE ONLY).
//
// An intrinsic-for-intrinsic C++ restatement of rai-infer's AVX2/FMA/F16C
// kernels, KV cache and LookupDecoder (greedy acceptance), used as the parity
// checker for the CUDA path and as the timed CPU baseline. Only tests/,
// __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may
// load it. Each function names the reference lines it follows.
//
// Parity pin: the reference is Rust and cannot be built in this container
// (no cargo). The oracle is pinned against the reference's own known-answer
// tests and golden fixtures (tests/golden/, tests/test_oracle_golden.py).
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- kernels (rai-infer/src/gemm.rs, layers.rs, lookup.rs) ---- */
void orc_quantize_input(const float* x, size_t cols, size_t group_size, int8_t* even,
                        int8_t* odd, float* scales, float* sums);
void orc_w4a8_matmul(float* out, const uint8_t* nibbles, const uint8_t* params,
                     const float* input, size_t rows, size_t cols, size_t tokens,
                     size_t group_size);
void orc_tied_lm_head(float* logits, const float* hidden, const uint8_t* data,
                      const uint8_t* params, size_t vocab, size_t hidden_size,
                      size_t group_size);
void orc_embed_lookup(float* out, size_t token, const uint8_t* data, const uint8_t* params,
                      size_t vocab, size_t hidden_size, size_t group_size);
void orc_rms_norm(float* out, const float* in, const float* w, size_t n, float eps);
void orc_rms_norm_with_residual(float* normed, float* residual, const float* hidden,
                                const float* w, size_t n, float eps);
void orc_rms_norm_heads(float* x, size_t num_heads, size_t head_dim, const float* w, float eps);
int orc_rope_table(float* cos_t, float* sin_t, size_t head_dim, size_t max_ctx, float theta,
                   int rope_type, float factor, float low, float high, uint32_t orig_max);
void orc_rope_apply(float* heads, size_t num_heads, size_t head_dim, const float* cos_row,
                    const float* sin_row);
void orc_silu_mul(float* gate, const float* up, size_t n);
void orc_attention_head(const float* q, float* out, const float* k_head, const float* v_head,
                        size_t pos, size_t head_dim, float scale, float softcap);
void orc_attention_head_debug(const float* q, float* out, const float* k_head, const float* v_head, size_t pos,
                              size_t head_dim, float scale, float* e, float* mx, float* sum);
void orc_route_experts(const float* hidden, const float* router, size_t num_experts,
                       size_t width, size_t top_k, int norm_topk, uint32_t* experts,
                       float* weights);
int orc_find_ngram_draft(const uint32_t* tokens, size_t len, size_t min_ngram,
                         size_t max_ngram, size_t max_draft, size_t* ngram, size_t* start,
                         size_t* draft_len);
size_t orc_argmax(const float* v, size_t n);

/* ---- model / decoder (rai-infer/src/model.rs, lookup.rs, kv_cache.rs) ---- */
typedef struct orc_model orc_model;
typedef struct orc_decoder orc_decoder;
orc_model* orc_model_open(const uint8_t* blob, size_t len, char* err, size_t err_len);
void orc_model_free(orc_model* m);
/* hidden, layers, heads, kv_heads, head_dim, ff, vocab, max_ctx, group, embed_group,
   num_experts, experts_per_token, tied(1/0), version */
void orc_model_config(const orc_model* m, uint32_t out[14]);
orc_decoder* orc_decoder_new(orc_model* m, size_t max_ctx, char* err, size_t err_len);
void orc_decoder_free(orc_decoder* d);
int orc_prefill(orc_decoder* d, const uint32_t* ids, size_t n, size_t* pos_out);
int orc_forward_logits(orc_decoder* d, const uint32_t* ids, size_t start_pos, size_t batch,
                       float* logits);
int orc_step_greedy(orc_decoder* d, size_t pos, const uint32_t* ctx, size_t ctx_len,
                    size_t max_draft, size_t max_ngram, size_t min_ngram, uint32_t* out_tokens,
                    size_t* n_out, size_t metrics[4]);
size_t orc_kv_filled(const orc_decoder* d, size_t layer);
void orc_kv_truncate(orc_decoder* d, size_t len);
int orc_kv_read(const orc_decoder* d, size_t layer, size_t kv_head, size_t pos, float* k,
                float* v);
size_t orc_last_error(char* buf, size_t len);

/* ---- synthetic model writing (oracle/model_writer.cpp) ---- */
/* quantize_row (rai-infer/src/convert.rs:2551-2639) over a [rows][cols]
   matrix; params rows*ceil(cols/gs)*4 bytes, codes rows*cols/2 (bits 4) or
   rows*cols (bits 8). 0 ok, -1 on bad arguments or a non-finite weight. */
int orc_rtn_quantize(const float* w, size_t rows, size_t cols, int bits, size_t gs, uint8_t* params,
                     uint8_t* codes);
/* The synthetic models' seeded N(0, stddev) source, f16-rounded. */
int orc_synth_normal_f16(uint64_t seed, uint64_t stream, size_t n, float stddev, float* out);
int orc_num_threads(void);
/* glibc expf (the reference's f32::exp) of the floats with bit patterns
   first .. first + n - 1. */
void orc_expf_range(uint32_t first, size_t n, float* out);
void orc_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
