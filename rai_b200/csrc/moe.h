// Mixture-of-experts MLP block launchers (internal).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace rai {

constexpr int kMaxMoeExperts = 256;

// Device scratch of one MoE block over up to `rows_cap` expert-sorted rows.
struct MoeBuffers {
  float* logits = nullptr;    // [M][ne] router logits, then probabilities
  int* experts = nullptr;     // [M][k] picked experts (-1 = none)
  float* weights = nullptr;   // [M][k] their weights
  int* cnt = nullptr;         // [ne] pairs per expert
  int* off = nullptr;         // [ne] first sorted row of each expert (multiple of 8)
  int* row_of_pair = nullptr; // [M * k] sorted row of (token, pick), -1 = none
  int* pair_of_row = nullptr; // [rows_cap] pair of each sorted row, -1 = padding
  int* n_rows = nullptr;      // sorted rows in use (multiple of 8)
  int rows_cap = 0;
};

// Router logits, softmax / top-k / renormalization and the expert sort for
// the *m_dev (or M) active rows of x ([M][h] normalized hidden rows).
cudaError_t moe_route(const float* x, const float* router, int h, int ne, int k, bool norm_topk, const int* m_dev,
                      int M, const ExpfTable& et, const MoeBuffers& mb, cudaStream_t s);
// Quantize x's rows into expert-sorted activation rows.
cudaError_t moe_gather_quant(const float* x, int h, int k, int gs, const MoeBuffers& mb, ActBuf act, cudaStream_t s);
// out[b] = residual[b] + sum over picks (in order) of weight * eo[row].
// Expert parallelism: with tp (world > 1) and slot >= 0, eo is first awaited
// as exchange `slot` (every rank's experts' rows).
cudaError_t moe_combine(const float* eo, int k, int h, const float* residual, float* out, const int* m_dev, int M,
                        const MoeBuffers& mb, cudaStream_t s, const TpLink* tp = nullptr, int slot = -1,
                        uint32_t* err = nullptr);
cudaError_t init_moe_attributes();

}  // namespace rai
