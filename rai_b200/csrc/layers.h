// Launchers of the per-layer and speculation kernels (internal).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace rai {

constexpr int kMaxRows = 33;  // max_draft <= 32 (rai run's --lookup-k limit) + 1

// Device-resident state of one decode step. The host writes pos and ctx_len
// (and the context) before the step; the kernels fill the rest; the host
// reads it back once at the end of the step.
struct StepState {
  int pos;
  int ctx_len;
  int n_rows;    // verify rows this step: drafted + 1
  int drafted;
  int ngram;     // matched n-gram length, 0 = none
  int accepted;
  int produced;
  uint32_t err;
  uint32_t tokens[kMaxRows];  // [last, draft_0 .. draft_{k-1}]
  uint32_t out[kMaxRows];     // produced tokens
  unsigned long long amax[kMaxRows];
};

// Dynamic shared memory the attention kernel may use (the opt-in limit of
// 227 KB less its static shared memory and a margin).
constexpr size_t kAttnMaxSmem = 224 * 1024;

// Raise the dynamic shared-memory limit of the attention kernels (once per
// process, before any stream capture).
cudaError_t init_layer_attributes();

cudaError_t launch_embed(const uint32_t* ids, const int* m_dev, int M, const uint8_t* codes,
                         const uint8_t* params, int vocab, int hidden, int gs, float embed_scale,
                         float* out, uint32_t* err, cudaStream_t s);
cudaError_t launch_rmsnorm(const float* x, const float* w, int n, float eps, float* out, float* residual,
                           const int* m_dev, int M, cudaStream_t s);
cudaError_t launch_qkv_post(float* qkv, int ld, float* q_out, int nh, int nkv, int hd, const float* qn,
                            const float* kn, int qk_mode, float eps, const float* rope_cos,
                            const float* rope_sin, float* kc, float* vc, int max_ctx, const int* pos_dev,
                            int pos0, const int* m_dev, int M, cudaStream_t s);
size_t attention_smem_bytes(int hd, int hpk, int n_alloc);
cudaError_t launch_attention(const float* q, float* out, const float* kc, const float* vc, int nh, int nkv,
                             int hd, int max_ctx, const int* pos_dev, int pos0, const int* m_dev, int M,
                             float scale, float softcap, int n_alloc, const ExpfTable& et, cudaStream_t s);
cudaError_t launch_swiglu(const float* gu, int ff, float* act, const int* m_dev, int M, const ExpfTable& et,
                          cudaStream_t s);
cudaError_t launch_argmax(const float* logits, int vocab, const int* m_dev, int M, unsigned long long* best,
                          cudaStream_t s);
cudaError_t launch_ngram(const uint32_t* ctx, StepState* st, int max_draft, int max_ngram, int min_ngram,
                         int max_ctx, cudaStream_t s);
cudaError_t launch_accept(StepState* st, int* filled, int num_layers, cudaStream_t s);

}  // namespace rai
