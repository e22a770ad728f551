/* rai_gpu.h - C ABI of the B200-native prompt-lookup decode path.
 *
 * Drop-in boundary for rai-infer's prompt-lookup speculative decode step
 * (rai-infer/src/lookup.rs LookupDecoder, rai-infer/src/model.rs RaiModel,
 * rai-infer/src/kv_cache.rs KVCache). The host keeps the .raimodel loader,
 * tokenizer and sampling loop; this library uploads the model once and runs
 * draft lookup, the (k+1)-row verify forward, greedy or sampled acceptance
 * and KV rollback on the GPU with no host round-trip inside a step.
 *
 * Conventions: every function returns an int status (RAI_OK = 0, negative on
 * error) and never aborts or unwinds; rai_gpu_last_error() returns the
 * message of the calling thread's last failure. A model is shared read-only
 * by any number of decoders on its device; a decoder owns one CUDA stream, its
 * KV cache and scratch, and must not be used from two threads at once.
 * Token ids are uint32; positions and lengths are size_t.
 */
#ifndef RAI_GPU_H
#define RAI_GPU_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RAI_API __attribute__((visibility("default")))
#else
#define RAI_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  RAI_OK = 0,
  RAI_ERR_INVALID = -1,     /* bad argument / misuse (ensure! in the reference) */
  RAI_ERR_OOM = -2,         /* device or pinned-host allocation failed */
  RAI_ERR_DEVICE = -3,      /* CUDA error */
  RAI_ERR_TIMEOUT = -4,     /* a bounded device-side wait gave up */
  RAI_ERR_UNSUPPORTED = -5, /* valid model, capability this build does not run */
  RAI_ERR_FORMAT = -6       /* malformed .raimodel (format.rs validation) */
};

typedef struct rai_model rai_model;
typedef struct rai_dec rai_dec;

/* LookupConfig (rai-infer/src/lookup.rs:63-93) plus the SamplerConfig fields
 * the reference validates (lookup.rs:457-475). temperature > 1e-6 runs the
 * reference's sampled rule (accept a draft with its target probability,
 * otherwise sample the correction from the target without it; a bonus token
 * when all are accepted), with random numbers seeded by rai_gpu_set_seed.
 * temperature == 0 selects greedy acceptance, the t -> 0 limit of that rule
 * (accept a drafted token iff it is the target argmax; correction and bonus
 * are argmaxes), which the reference itself refuses. top_k must be 0, top_p
 * 1 and repetition_penalty 1, as in the reference. */
typedef struct {
  uint32_t max_draft;   /* K: tokens copied per step, >= 1 */
  uint32_t max_ngram;   /* longest suffix n-gram tried first */
  uint32_t min_ngram;   /* shortest suffix n-gram, >= 1 */
  float temperature;    /* 0 = greedy */
  uint32_t top_k;       /* must be 0 */
  float top_p;          /* must be 1 */
  float repetition_penalty; /* must be 1 */
} rai_lookup_cfg;

/* LookupMetrics (rai-infer/src/lookup.rs:111-119). matched_ngram = 0 when no
 * n-gram matched (the reference's None). */
typedef struct {
  uint32_t accepted;
  uint32_t drafted;
  uint32_t produced;
  uint32_t matched_ngram;
  float accept_rate;
} rai_lookup_metrics;

/* SpeculativeConfig (rai-infer/src/speculative.rs): draft tokens per step
 * and the SamplerConfig fields validate_speculative_config checks
 * (speculative.rs:396-407). temperature == 0 selects the greedy limit. */
typedef struct {
  uint32_t draft_k;     /* >= 1 */
  float temperature;    /* 0 = greedy, else > 1e-6 */
  uint32_t top_k;       /* must be 0 */
  float top_p;          /* must be 1 */
  float repetition_penalty; /* must be 1 */
} rai_spec_cfg;

typedef struct rai_spec rai_spec;

/* ModelConfig fields the host loop needs (rai-infer/src/format.rs:162-265). */
typedef struct {
  uint32_t hidden_size, num_layers, num_heads, num_kv_heads, head_dim;
  uint32_t intermediate_size, vocab_size, max_context;
  uint32_t group_size, embed_group_size, num_experts, experts_per_token;
  uint32_t tied_embeddings, version;
  uint64_t device_bytes; /* HBM held by the uploaded model */
} rai_model_info;

/* RaiModel::load (rai-infer/src/model.rs:97-181) from an in-memory .raimodel:
 * validates like RaiModelFile::open (format.rs:557-637), uploads the blob to
 * HBM once and repacks the weights into the device layout. */
RAI_API int rai_gpu_model_create(const uint8_t* blob, size_t len, int device, rai_model** out);
/* Refused (RAI_ERR_INVALID) while decoders created on the model are alive:
 * destroy them first. */
RAI_API int rai_gpu_model_destroy(rai_model* model);
RAI_API int rai_gpu_model_info(const rai_model* model, rai_model_info* info);

/* Tensor-parallel form of rai_gpu_model_create (no reference counterpart:
 * rai-infer runs one CPU process). One process per GPU; rank tp_rank of
 * tp_size in {2, 4, 8} uploads only its shard: every linear is split by
 * whole output rows (its query / KV heads, its ff columns, its slice of the
 * hidden rows for o / down, its vocabulary rows), so each rank computes
 * complete reference dot products and the results are identical to one GPU.
 * Ranks exchange the attention and SwiGLU outputs and the hidden rows over
 * NVLink through an exchange arena: after every rank has created its model,
 * pass each rank's 64-byte handle (rai_gpu_tp_handle, in rank order, to every
 * rank) to rai_gpu_tp_connect, and bring all ranks to a host barrier before
 * any rank creates a decoder. All ranks then make the same calls (decoder
 * create, prefill, step) with the same arguments; each returns the same
 * tokens. Mixture-of-experts models are split by experts instead (expert
 * parallel: whole experts per rank, attention and head replicated). Not on
 * multi-GPU models: rai_gpu_prefill_many; not under tensor parallelism:
 * rai_gpu_forward_logits and sampled acceptance.
 * Cross-GPU waits are bounded (about a second). When one times out (a rank
 * that stopped making the same calls) the call returns RAI_ERR_TIMEOUT and
 * the model is failed for good: every later call that would run it returns
 * RAI_ERR_TIMEOUT, because the ranks no longer agree on which exchange is
 * which. Recover by destroying and re-creating the model on every rank. */
RAI_API int rai_gpu_model_create_tp(const uint8_t* blob, size_t len, int device, int tp_rank, int tp_size,
                                    rai_model** out);
RAI_API int rai_gpu_tp_handle(rai_model* model, void* handle, size_t cap);
RAI_API int rai_gpu_tp_connect(rai_model* model, const void* handles, size_t n);

/* Which kernel the model's dense 4-bit linears run on (no reference
 * counterpart: the reference has one CPU kernel). 1 (exact, the default):
 * the bit-exact kernel everywhere. 0 (auto): forward passes of fewer than 64
 * rows run the bit-exact kernel, passes of 64 rows or more (prefill chunks,
 * many streams' verify rows) the tcgen05 kernel. 2 (tol): always the tcgen05
 * kernel. The tcgen05 kernel's int32 group dots are exact and its outputs
 * agree with the reference's to a few f32 ulps, but the reference
 * re-quantizes every linear's input to int8, which turns ulp-level
 * differences into code flips: on seeded random-weight models a 1-ulp change
 * of one constant moves the reference's own logits by up to ~18% of their
 * range, and modes 0 / 2 move them as much. They are throughput modes, not
 * parity modes. RAI_GEMM_MODE=exact|auto|tol sets the default. Multi-GPU
 * models always run exact. Set it before the model's decoders run (a step
 * graph records the mode it was built with). */
RAI_API int rai_gpu_model_set_gemm_mode(rai_model* model, int mode);
RAI_API int rai_gpu_model_gemm_mode(const rai_model* model, int* mode);

/* LookupDecoder::new (rai-infer/src/lookup.rs:192-209): context window =
 * min(max_ctx, model max_context); allocates the KV cache on the device. */
RAI_API int rai_gpu_decoder_create(rai_model* model, size_t max_ctx, rai_dec** out);
RAI_API int rai_gpu_decoder_destroy(rai_dec* dec);

/* LookupDecoder::prefill (rai-infer/src/lookup.rs:219-247): runs every prompt
 * token but the last through the model; *pos_out = n - 1. */
RAI_API int rai_gpu_prefill(rai_dec* dec, const uint32_t* ids, size_t n, size_t* pos_out);

/* rai_gpu_prefill for each of n decoders (sharing one model, empty caches),
 * with all prompts' rows batched into shared forward passes. */
RAI_API int rai_gpu_prefill_many(rai_dec* const* decs, size_t n, const uint32_t* const* ids,
                                 const size_t* lens, size_t* pos_out);

/* LookupDecoder::step (rai-infer/src/lookup.rs:260-425). `ctx` is the whole
 * token sequence; its last element lives at `pos`. Writes produced tokens to
 * out_tokens (capacity out_cap >= max_draft + 1), their count to *n_out, and
 * the step's metrics. The KV cache is rolled back to pos + produced. */
RAI_API int rai_gpu_step(rai_dec* dec, size_t pos, const uint32_t* ctx, size_t ctx_len,
                 const rai_lookup_cfg* cfg, uint32_t* out_tokens, size_t out_cap,
                 size_t* n_out, rai_lookup_metrics* metrics);

/* One token without a draft search: the no-match path of
 * LookupDecoder::step (decode_one, rai-infer/src/lookup.rs:428-454) as its
 * own call, i.e. plain autoregressive decoding. Runs `last_token` at `pos`
 * (KV stored there), then samples the next token (temperature > 1e-6, the
 * decoder's random numbers) or takes the argmax (temperature 0). The cache
 * is left filled to pos + 1. */
RAI_API int rai_gpu_decode_one(rai_dec* dec, size_t pos, uint32_t last_token, float temperature, uint32_t* token);

/* Seed of the decoder's random numbers for sampled acceptance
 * (temperature > 1e-6), standing in for the reference's `&mut impl Rng`
 * argument of LookupDecoder::step (rai-infer/src/lookup.rs:260-266); each
 * step then uses the next draws. The stream is Philox4x32-10, not the
 * reference's StdRng, so sampled outputs match the reference in
 * distribution, not token for token. Default seed 0. */
RAI_API int rai_gpu_set_seed(rai_dec* dec, uint64_t seed);

/* Draft-model speculative decoding (SpeculativeDecoder,
 * rai-infer/src/speculative.rs): a target and a smaller draft model with one
 * vocabulary on one device. create = SpeculativeDecoder::new with both KV
 * caches; prefill runs the prompt (all but the last token) through both;
 * step (speculative.rs:180-392): the draft proposes k = min(draft_k,
 * window - pos - 1) tokens one row at a time, the target verifies all k + 1
 * rows in one forward, the reference's rule accepts (greedy limit at
 * temperature 0: accept iff the target argmax; sampled: min(1, p_t / p_d),
 * correction from max(0, p_t - p_d), bonus when all accept, after which the
 * draft runs its last proposal), and both caches roll back to pos +
 * produced. metrics: accepted, drafted = k, produced (matched_ngram = 0).
 * set_seed seeds the sampled draws (Philox, distributional parity). */
RAI_API int rai_gpu_spec_create(rai_model* target, rai_model* draft, size_t max_ctx, rai_spec** out);
RAI_API int rai_gpu_spec_destroy(rai_spec* spec);
RAI_API int rai_gpu_spec_set_seed(rai_spec* spec, uint64_t seed);
RAI_API int rai_gpu_spec_prefill(rai_spec* spec, const uint32_t* ids, size_t n, size_t* pos_out);
RAI_API int rai_gpu_spec_step(rai_spec* spec, size_t pos, uint32_t last_token, const rai_spec_cfg* cfg,
                              uint32_t* out_tokens, size_t out_cap, size_t* n_out, rai_lookup_metrics* metrics);

/* One step for each of n decoders sharing one model and device, batched so
 * their verify rows share every weight read (one forward over
 * sum(k_i + 1) rows). Same semantics as n calls of rai_gpu_step.
 * out_tokens is n * out_cap. */
RAI_API int rai_gpu_step_many(rai_dec* const* decs, size_t n, const size_t* pos,
                      const uint32_t* const* ctx, const size_t* ctx_len,
                      const rai_lookup_cfg* cfg, uint32_t* out_tokens, size_t out_cap,
                      size_t* n_out, rai_lookup_metrics* metrics);

/* KVCache::filled / truncate (rai-infer/src/kv_cache.rs:289-304). */
RAI_API int rai_gpu_kv_filled(const rai_dec* dec, size_t layer, size_t* filled);
RAI_API int rai_gpu_kv_truncate(rai_dec* dec, size_t len);
/* Copy one cached (K, V) row to the host; position must be < filled. */
RAI_API int rai_gpu_kv_read(const rai_dec* dec, size_t layer, size_t kv_head, size_t pos, float* k,
                    float* v);

/* RaiModel::forward_batch + hidden_to_logits_batch
 * (rai-infer/src/model.rs:692-1033) for `batch` tokens at positions
 * start_pos.., storing their KV; logits (batch * vocab f32, host) may be
 * NULL. */
RAI_API int rai_gpu_forward_logits(rai_dec* dec, const uint32_t* ids, size_t start_pos, size_t batch,
                           float* logits);

/* Wall-clock device time (microseconds) of the decoder's last step /
 * step_many, measured with CUDA events on its stream. */
RAI_API int rai_gpu_last_step_us(const rai_dec* dec, float* us);

RAI_API size_t rai_gpu_last_error(char* buf, size_t len);

/* ---- kernel-level entry points (device pointers, caller's stream) ----
 *
 * The W4A8 linear of rai-infer/src/gemm.rs (w4a8_matmul, gemm.rs:1774-1919;
 * w4a8_matvec, gemm.rs:1336-1392): out[t * rows + r] = sum over the row's
 * groups of the int8-quantized input against 4-bit codes with f16
 * (scale, zero), bit-identical to the AVX2 kernel. Weights are first packed
 * once into the device layouts (the mma.sync kernel's 4-bit blocks, then the
 * u8 image of the opt-in tcgen05 kernel, RAI_GEMM_TC=1; the buffer is opaque
 * and rai_gpu_w4a8_packed_bytes covers both); `scratch` holds the quantized
 * activations (rai_gpu_w4a8_scratch_bytes). group_size must be 64 or 128. */
RAI_API size_t rai_gpu_w4a8_packed_bytes(size_t rows, size_t cols, size_t group_size);
RAI_API int rai_gpu_w4a8_pack(const uint8_t* nibbles, const uint8_t* params, size_t rows, size_t cols,
                      size_t group_size, void* packed, void* stream);
RAI_API size_t rai_gpu_w4a8_scratch_bytes(size_t tokens, size_t cols, size_t group_size);
RAI_API int rai_gpu_w4a8_matmul(float* out, const void* packed, const float* input, size_t rows,
                        size_t cols, size_t tokens, size_t group_size, void* scratch,
                        size_t scratch_bytes, void* stream);

/* Status of the kernel-level calls on the current device (the w4a8 GEMM
 * entries), which return as soon as their kernels are queued: synchronizes
 * `stream`, then returns RAI_ERR_TIMEOUT if one of their bounded device waits
 * gave up since the last query (that call's output is incomplete), else
 * RAI_OK. The status word is per device and cleared by the query. */
RAI_API int rai_gpu_kernel_status(void* stream);

/* The same linear on the tcgen05 tensor cores (w4a8_matmul,
 * rai-infer/src/gemm.rs:1774-1919, to the BASELINE tolerance: the int32
 * group dots are exact; per group acc += dot * (w_scale * x_scale) +
 * w_zero * x_sum in f32 fused multiply-adds, another rounding order than the
 * reference's eight lane accumulators), on activations quantized by
 * rai_gpu_w4a8_quantize. `workspace` (device, rai_gpu_w4a8_tol_workspace_bytes,
 * zeroed once before its first use; calls leave it zeroed) lets launches with
 * few row tiles split the groups over more SMs; NULL runs without the split.
 * Calls sharing a workspace must not overlap on the GPU. */
RAI_API size_t rai_gpu_w4a8_tol_workspace_bytes(void);
RAI_API int rai_gpu_w4a8_matmul_tol_prequant(float* out, const void* packed, const void* scratch, size_t rows,
                                             size_t cols, size_t tokens, size_t group_size, void* workspace,
                                             size_t workspace_bytes, void* stream);

/* rai_gpu_w4a8_matmul without a caller scratch buffer and without any
 * allocation: the quantized activations go to a 2 MiB file-scope device
 * array of the library (one per device). No reference counterpart: this
 * entry exists for callers that may not allocate device memory. Limit:
 * rai_gpu_w4a8_scratch_bytes(tokens, cols, group_size) <= 2 MiB (e.g. 64
 * tokens x 14336 columns at group 128), else RAI_ERR_INVALID. Call with the
 * stream's device current. The array's address is looked up on the first
 * call per device, so make that call before capturing a stream. The array
 * keeps the last call's contents; every byte the GEMM reads is rewritten by
 * the same call. Calls on one device share the array, so calls that overlap
 * in time (different streams or host threads) race: serialize them. */
RAI_API int rai_gpu_w4a8_matmul_static(float* out, const void* packed, const float* input, size_t rows,
                                       size_t cols, size_t tokens, size_t group_size, void* stream);

/* The two launches of rai_gpu_w4a8_matmul separately: quantize `input`
 * (tokens x cols f32) into `scratch`, then the GEMM kernel alone on an
 * already-quantized scratch (e.g. to time it). */
RAI_API int rai_gpu_w4a8_quantize(const float* input, size_t cols, size_t tokens, size_t group_size,
                                  void* scratch, size_t scratch_bytes, void* stream);
RAI_API int rai_gpu_w4a8_matmul_prequant(float* out, const void* packed, const void* scratch, size_t rows,
                                         size_t cols, size_t tokens, size_t group_size, void* stream);

/* Attention of rai-infer's attention_head_avx2 (rai-infer/src/layers.rs:
 * 1266-1380) for M query rows over one cache: q [M][nh*hd], k and v
 * [nkv][max_ctx][hd], row r attends positions 0..positions[r] (host array);
 * out [M][nh*hd]. Device pointers except `positions`. */
RAI_API int rai_gpu_attention(const float* q, const float* k, const float* v, const int* positions, size_t M,
                              size_t nh, size_t nkv, size_t hd, size_t max_ctx, float scale, float* out,
                              void* stream);

/* The sampled acceptance of one step on given verify-row logits: the loop
 * of LookupDecoder::step (rai-infer/src/lookup.rs:359-403) when
 * draft_logits is null (point-mass draft distribution), the loop of
 * SpeculativeDecoder::step (speculative.rs:300-355) with the draft model's
 * logits [n_drafted][vocab] otherwise. logits [n_drafted + 1][vocab]
 * (device), draft tokens (host), temperature > 1e-6, random numbers of
 * (seed, step) as the decoders draw them. Writes the produced tokens (host,
 * capacity n_drafted + 1), their count and the accepted count. */
RAI_API int rai_gpu_sample_accept(const float* logits, const float* draft_logits, size_t vocab,
                                  const uint32_t* draft, size_t n_drafted, float temperature, uint64_t seed,
                                  uint64_t step, uint32_t* out, size_t* n_out, size_t* accepted);

/* The library's reproduction of the host libm expf (the reference's
 * f32::exp in its softmax tails and router, rai-infer/src/layers.rs:
 * 1266-1380, 1808-1870) on the device: out[i] (device) = expf of the float
 * whose bit pattern is first_bits + i, for i < n (first_bits + n <= 2^32).
 * For checking it against the host libm over every input. */
RAI_API int rai_gpu_expf_range(uint32_t first_bits, size_t n, float* out, void* stream);

/* Number of kernels one rai_gpu_step replays (the captured CUDA graph's
 * kernel nodes for the decoder's current configuration; 0 before the first
 * step). */
RAI_API int rai_gpu_step_kernel_count(const rai_dec* dec, size_t* kernels);

/* ---- host-side .raimodel writer utilities (no device needed) ----
 *
 * The RTN quantizer of `rai convert` (quantize_row,
 * rai-infer/src/convert.rs:2551-2639), multi-threaded: per (row, group) f64
 * min/max, scale = max((max-min)/(2^bits-1), 2^-24) rounded to f16, zero =
 * f16(min), code = clamp(round_half_even((w-zero)/scale)). 4-bit codes are
 * packed low nibble = even column. */
RAI_API int rai_rtn_quantize(const float* w, size_t rows, size_t cols, int bits, size_t group_size,
                             uint8_t* params, uint8_t* codes, int threads);
/* n seeded N(0, stddev) values rounded through f16 (the checkpoint cast of
 * rai-infer/src/safetensors.rs:457-477); deterministic per (seed, stream). */
RAI_API int rai_synth_normal_f16(uint64_t seed, uint64_t stream, size_t n, float stddev, float* out,
                                 int threads);
/* binary64 -> binary16 with round-to-nearest-even. */
RAI_API int rai_f64_to_f16(const double* in, size_t n, uint16_t* out);

#ifdef __cplusplus
}
#endif
#endif /* RAI_GPU_H */
