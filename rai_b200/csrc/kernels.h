// Host-side launch API of the sm_100a kernels (internal to librai_gpu.so).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"
#include "tp.cuh"

namespace rai {

// ---- W4A8 / W8A8 exact linear (kernels_gemm.cu) ----
constexpr int kTileRows = 64;          // weight rows per CTA tile
constexpr int kRowGroupBytes = 64;     // packed bytes per (row, group)
constexpr int kWeightStageBytes = kTileRows * kRowGroupBytes;      // 4096
constexpr int kParamStageBytes = kTileRows * 4;                    // 256
constexpr int kBlockBytes = kWeightStageBytes + kParamStageBytes;  // 4352
constexpr int kActRowBytes = 128;      // quantized activation bytes per (token, group)
constexpr int kActTokBytes = kActRowBytes + 8;  // + (scale, sum) f32 pair
// Quantized activations are stored in blocks of 8 tokens x 1 group:
// [token / 8][group] blocks of 8 x 128 code bytes then 8 (scale, sum)
// pairs, so the activations of consecutive groups of one 8-token block are
// contiguous (one bulk copy per block for several groups).
constexpr int kActBlockTok = 8;
constexpr int kActBlockBytes = kActBlockTok * kActTokBytes;  // 1088
constexpr int kTokChunk = 32;          // tokens per CTA pass

inline size_t ceil_div(size_t a, size_t b) { return (a + b - 1) / b; }
inline size_t round_up(size_t a, size_t b) { return ceil_div(a, b) * b; }

// A linear repacked for the device kernel.
struct PackedLinear {
  const uint8_t* data = nullptr;  // [tile][group] blocks of kBlockBytes
  int rows = 0, cols = 0, group_size = 0, groups = 0, tiles = 0;
  int wbits = 4;                   // 4: u4 codes (+ f16 scale/zero), 8: u8 embedding codes
  const uint8_t* tc = nullptr;     // tcgen05 weight image (4-bit linears; null: mma.sync path only)
};

inline size_t packed_linear_bytes(size_t rows, size_t cols, size_t gs) {
  return ceil_div(rows, kTileRows) * ceil_div(cols, gs) * (size_t)kBlockBytes;
}

// Weight image of the tcgen05 linear: per (128-row tile, group) the u8 codes
// in the MMA's shared-memory layout (16 KB) then the rows' f16 (scale, zero).
constexpr int kTcRows = 128;
constexpr int kTcImgBytes = kTcRows * 128;
constexpr int kTcBlockBytes = kTcImgBytes + kTcRows * 4;  // 16896
inline size_t tc_image_bytes(size_t rows, size_t cols, size_t gs) {
  return ceil_div(rows, kTcRows) * ceil_div(cols, gs) * (size_t)kTcBlockBytes;
}

// Quantized-activation staging for one linear input: per group a block of
// tok_alloc * 128 B codes then tok_alloc (scale, sum) pairs.
struct ActBuf {
  uint8_t* data = nullptr;
  int tok_alloc = 0;   // multiple of 8
  int groups = 0;
  size_t group_stride() const { return (size_t)tok_alloc * kActTokBytes; }
  static size_t bytes(int tok_alloc, int groups) { return (size_t)tok_alloc * kActTokBytes * groups; }
};

enum EpilogueMode : int { kEpiStore = 0, kEpiBias = 1, kEpiResidual = 2 };

struct GemmEpilogue {
  int mode = kEpiStore;
  const float* bias = nullptr;      // per output row
  const float* residual = nullptr;  // residual[t * ld + r]
};

// Raise the dynamic shared-memory limit of every GEMM variant (call once
// per process before capturing a graph).
cudaError_t init_gemm_attributes();

// Pack raw reference-layout weights (device pointers) into `out`.
cudaError_t pack_linear4(const uint8_t* nibbles, const uint8_t* params, int rows, int cols, int gs,
                         uint8_t* out, cudaStream_t s);
cudaError_t pack_linear8(const uint8_t* codes, const uint8_t* params, int rows, int cols, int gs,
                         uint8_t* out, cudaStream_t s);

// Quantize x[M][ldx] (f32) into `act` for a 4-bit linear (wbits = 4: per
// group of gs, +-127) or the tied 8-bit head (wbits = 8: per group of gs,
// +-63). Tokens in [M, tok_alloc) are zero-filled. `m_dev`, if non-null,
// overrides M with a device-resident active row count.
// With dst set (tensor parallelism), the codes go to every destination
// buffer at group g + dst->g_off instead of act (act gives tok_alloc).
cudaError_t quantize_act(const float* x, int ldx, int M, const int* m_dev, int K, int gs, int wbits,
                         ActBuf act, cudaStream_t s, const ActDst* dst = nullptr);

// out[t * ld_out + r] (= epilogue(dot)) for t < M, r < rows. With m_dev set,
// M is the static row budget (grid size) and *m_dev the active row count.
// RMSNorm of x (n wide; x copied to `residual` when set) quantized straight
// into `act` (one kernel).
// act.data may be null (no quantization); normed_out (optional) receives the
// normalized rows as f32.
// With tp set (world > 1) and slot >= 0, x is first awaited as exchange
// `slot` (every rank's projection rows, see tp.cuh).
cudaError_t norm_quant(const float* x, const float* w, int n, float eps, float* residual, int M,
                       const int* m_dev, int gs, int wbits, ActBuf act, cudaStream_t s,
                       float* normed_out = nullptr, const TpLink* tp = nullptr, int slot = -1,
                       uint32_t* err = nullptr);
// Grouped form of gemm_exact over ne same-shaped weight sets (expert e at
// w.data + e * w_stride): expert e multiplies activation rows off[e] ..
// off[e] + cnt[e] (device arrays; off[e] a multiple of 8) and writes the same
// output rows.
// Expert parallelism: the ne weight sets are model experts e0 .. e0 + ne
// (off / cnt indexed by model expert); with tp, result rows also go to
// tp->outs[1..n_out).
struct GemmTp;
cudaError_t gemm_grouped(const PackedLinear& w, size_t w_stride, int ne, const int* off, const int* cnt,
                         const ActBuf& act, float* out, int ld_out, uint32_t* err, cudaStream_t s, int e0 = 0,
                         const GemmTp* tp = nullptr);
// SwiGLU of gate/up rows [gate | up] (2*ff wide) quantized straight into `act`.
// Tensor parallelism: gu holds this rank's ff slice (columns col_off ..
// col_off + ff of ff_full) and the codes go to every rank through dst.
cudaError_t swiglu_quant(const float* gu, int ff, int M, const int* m_dev, int gs, const ExpfTable& et, ActBuf act,
                         cudaStream_t s, const ActDst* dst = nullptr, int col_off = 0, int ff_full = 0);

// Tensor-parallel extras of one GEMM launch: wait for exchange wait_slot
// before reading the activations; write the result also to outs[1..n_out)
// (outs[0] is `out`).
struct GemmTp {
  TpLink link;
  int wait_slot = -1;
  int n_out = 1;
  float* outs[kMaxTp] = {};
};
// Which kernel a dense 4-bit linear runs on. kGemmExact (the default): the
// bit-exact kernel. kGemmAuto: the exact kernel below kTolMinRows rows (the
// launch's static row budget), the tolerance-mode tcgen05 kernel from there
// on (prefill, many-stream verify); kGemmTol: always the tcgen05 kernel.
// Linears with a tensor-parallel exchange and the 8-bit tied head always run
// exact.
enum GemmMode : int { kGemmAuto = 0, kGemmExact = 1, kGemmTol = 2 };
constexpr int kTolMinRows = 64;
struct GemmPolicy {
  int mode = kGemmAuto;
  void* ws = nullptr;  // split-K workspace of the tcgen05 kernel (gemm_tol_workspace_bytes), may be null
  size_t ws_bytes = 0;
};
cudaError_t gemm_exact(const PackedLinear& w, const ActBuf& act, int M, float* out, int ld_out,
                       const GemmEpilogue& epi, uint32_t* err, cudaStream_t s, bool pdl = false,
                       const int* m_dev = nullptr, const GemmTp* tp = nullptr, const GemmPolicy* pol = nullptr);

// The W4A8 linear to the BASELINE tolerance on the tcgen05 tensor cores
// (kernels_gemm_tol.cu): exact int32 group dots, f32 scaling in a different
// order than the reference. `ws` (may be null: no split-K) is a per-stream
// workspace of gemm_tol_workspace_bytes() whose counters start at zero
// (cudaMemset once; the kernel leaves them at zero).
size_t gemm_tol_workspace_bytes();
cudaError_t init_gemm_tol_attributes();
cudaError_t gemm_tol(const PackedLinear& w, const ActBuf& act, int M, float* out, int ld_out,
                     const GemmEpilogue& epi, uint32_t* err, cudaStream_t s, const int* m_dev, void* ws,
                     size_t ws_bytes);

// The same linear (4-bit weights, one output buffer, no exchange) on the
// tcgen05 tensor cores; gemm_exact takes this path when RAI_GEMM_TC=1 and the
// linear has a tcgen05 weight image.
bool gemm_tc_enabled();
cudaError_t init_gemm_tc_attributes();
cudaError_t pack_linear4_tc(const uint8_t* nibbles, const uint8_t* params, int rows, int cols, int gs, uint8_t* out,
                            cudaStream_t s);
cudaError_t gemm_tc(const PackedLinear& w, const ActBuf& act, int M, float* out, int ld_out, const GemmEpilogue& epi,
                    uint32_t* err, cudaStream_t s, const int* m_dev);

}  // namespace rai
