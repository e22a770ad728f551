// Exact W4A8 (and tied W8A8 head) linear for sm_100a.
//
// Restates the arithmetic of rai-infer/src/gemm.rs bit for bit:
//   * activations quantized per (token, group): absmax -> scale = absmax/127
//     (1.0 below 1e-10) -> q = clamp(rne(x * (1/scale)), -128, 127), plus the
//     f32 group sum accumulated in 8 lanes then the fixed horizontal-sum tree
//     (quantize_input_split_avx2, gemm.rs:280-374; compute_input_sums_avx2,
//     gemm.rs:182-212). The tied head uses +-63 and the embedding group
//     (quantize_hidden_i8_avx2, gemm.rs:976-1047).
//   * per (token, row, group) the reference keeps 8 int32 lane dots: lane L
//     holds columns 8L..8L+7 of every 64-column chunk (PMADDUBSW + PMADDWD,
//     gemm.rs:455-469); each is converted to f32, multiplied by
//     (w_scale * x_scale) and added into an 8-lane f32 accumulator in group
//     order; the row result is the horizontal-sum tree plus the sequential
//     zero correction sum_g(w_zero * x_sum) (gemm.rs:599-673). For the tied
//     head lane L holds bytes 4L..4L+3 of each 32-byte chunk (gemm.rs:857-872).
//
// Device design: one CTA owns 64 weight rows and sweeps every group in order
// (the f32 lane accumulation is order-sensitive, so K is never split). A
// producer warp streams (weights + params, activation codes + scales) for
// each group through a ring of shared-memory stages with cp.async.bulk (TMA)
// and mbarriers; four consumer warps each own 16 rows. The per-lane int32
// dots run on the tensor cores: the repacked weight layout puts each
// reference lane's 16 columns into one K=16 slice, so one
// mma.m16n8k16.u8.s8 per lane yields exactly the reference's lane dot for
// 16 rows x 8 tokens. The accumulator is seeded with 0x4B400000 so the
// int32 result read as f32 is 12582912 + dot exactly; one subtraction gives
// the dot as f32 without an I2F conversion.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "quant.cuh"

namespace rai {

namespace {

// Kernel variant. Consumer warps per CTA: 4 row slabs of 16 rows, each slab
// split over LG warps by reference lane pair (lanes j and j+4 form pair j:
// they share a packed weight word and are the first two terms the
// horizontal sum adds) and over TS warps by 8-token N tiles. The lane
// accumulators are independent, so neither split changes any rounding; the
// LG warps of a slab meet once per work item to finish the horizontal sum.
// MINB: CTAs per SM the launch is sized for; UNROLL: groups unrolled in the
// consumer loop. SPLIT (for launches with fewer tiles than SMs): a 64-row
// tile is shared by LG CTAs, each owning 4 / LG slabs with 4 consumer warps,
// and a slab's LG lane groups sit on LG different warp schedulers, so each
// SM carries 64 / LG rows and the per-group chain is cut LG ways.
template <int NT_, int LG_, int TS_, int MINB_, int UNROLL_, bool SPLIT_ = false>
struct GemmCfg {
  static constexpr int NTILES = NT_, LG = LG_, TS = TS_, kMinBlocks = MINB_, kUnroll = UNROLL_;
  static constexpr bool SPLIT = SPLIT_;
  static_assert(LG == 1 || LG == 2 || LG == 4, "lane groups");
  static_assert(NTILES % TS == 0, "token split");
  static_assert(!SPLIT || TS == 1, "a split tile has no token split");
  static constexpr int kConsumerWarps = SPLIT ? 4 * TS : 4 * LG * TS;
  static constexpr int kThreads = (kConsumerWarps + 1) * 32;
  static constexpr int kTilesPerWarp = NTILES / TS;
  static constexpr int kPairs = 4 / LG;  // lane pairs per consumer warp
  // Partial horizontal sums handed to the slab's first lane group:
  // [slab][token split][LG-1][N tile][4][32] floats.
  static constexpr int kCombBytes = 4 * TS * (LG - 1) * kTilesPerWarp * 4 * 32 * 4;
};
constexpr uint32_t kMagic = 0x4B400000u;  // 12582912.0f
constexpr float kMagicF = 12582912.0f;

// ---------------------------------------------------------------------------
// Weight repack
// ---------------------------------------------------------------------------
// 4-bit block (tile, group): row r's 64 bytes are 4 slots of 16 bytes. Slot t
// (chunk c = t >> 1, column parity p = t & 1) word j, byte b holds in its low
// nibble the code of group column 64c + 8j + 2b + p (reference lane j) and
// in its high nibble column 64c + 8(j+4) + 2b + p (lane j+4): the lanes that
// the horizontal sum adds first share a word. Chunk 1 is zero when the
// group is 64 wide.
__global__ void pack4_kernel(const uint8_t* __restrict__ nib, const uint8_t* __restrict__ params,
                             int rows, int cols, int gs, int groups, uint8_t* __restrict__ out,
                             size_t total) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= total) return;
  size_t blk = i / kBlockBytes;
  int within = (int)(i % kBlockBytes);
  int g = (int)(blk % groups);
  int tile = (int)(blk / groups);
  uint8_t v = 0;
  if (within < kWeightStageBytes) {
    int r = within / kRowGroupBytes, o = within % kRowGroupBytes;
    int row = tile * kTileRows + r;
    int t = o / 16, j = (o % 16) / 4, b = o % 4;
    int c = t >> 1, p = t & 1;
    if (row < rows && 64 * c < gs) {
      size_t rowbase = (size_t)row * (cols / 2) + (size_t)g * gs / 2;
      int col0 = 64 * c + 8 * j + 2 * b;  // even column of the byte
      uint8_t lo = nib[rowbase + col0 / 2];
      uint8_t hi = nib[rowbase + (col0 + 32) / 2];
      uint8_t c0 = p ? (lo >> 4) : (lo & 0xF);
      uint8_t c1 = p ? (hi >> 4) : (hi & 0xF);
      v = (uint8_t)(c0 | (c1 << 4));
    }
  } else {
    int q = within - kWeightStageBytes;
    int r = q / 4, k = q % 4;
    int row = tile * kTileRows + r;
    if (row < rows) v = params[((size_t)row * groups + g) * 4 + k];
  }
  out[i] = v;
}

// 8-bit block (tile, group of 64): row r's 64 bytes are the group's codes in
// their original order (slot 0 = bytes 0..31, slot 1 = bytes 32..63; lane L
// of a slot = bytes 4L..4L+3).
__global__ void pack8_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ params,
                             int rows, int cols, int gs, int groups, uint8_t* __restrict__ out,
                             size_t total) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= total) return;
  size_t blk = i / kBlockBytes;
  int within = (int)(i % kBlockBytes);
  int g = (int)(blk % groups);
  int tile = (int)(blk / groups);
  uint8_t v = 0;
  if (within < kWeightStageBytes) {
    int r = within / kRowGroupBytes, o = within % kRowGroupBytes;
    int row = tile * kTileRows + r;
    if (row < rows) v = codes[(size_t)row * cols + (size_t)g * gs + o];
  } else {
    int q = within - kWeightStageBytes;
    int r = q / 4, k = q % 4;
    int row = tile * kTileRows + r;
    if (row < rows) v = params[((size_t)row * groups + g) * 4 + k];
  }
  out[i] = v;
}

// One warp per (token, group) of x.
// With several destinations (tensor parallelism) every rank's buffer gets
// the codes at group g + dst.g_off, and the stores are fenced at system
// scope before the kernel ends.
__global__ void quantize_kernel(const float* __restrict__ x, int ldx, int M, const int* m_dev,
                                int K, int gs, int wbits, ActDst dst, int tok_alloc) {
  __shared__ __align__(16) float sx[8][128];
  __shared__ uint32_t sqw[8][32];
  pdl_wait_prior();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x;
  const int mact = m_dev ? *m_dev : M;
  // The GEMM reads tokens in groups of 8: rows up to the next multiple of 8
  // past the active count are zeroed.
  const int rows = min(tok_alloc, (mact + 7) & ~7);
  const int len = min(gs, K - g * gs);
  for (int tok = blockIdx.y * 8 + warp; tok < rows; tok += gridDim.y * 8) {
    if (tok >= mact) {
      zero_group_warp(tok, dst, g);
      continue;
    }
    const float* xr = x + (size_t)tok * ldx + (size_t)g * gs;
    stage_f32(sx[warp], xr, len, lane, 32);
    cp_async_wait<0>();
    __syncwarp();
    quant_group_warp(sx[warp], len, wbits, tok, dst, g, sqw[warp]);
  }
  if (dst.n > 1) __threadfence_system();
}

// RMSNorm of rai-infer (rms_norm_with_residual_avx2 / rms_norm_avx2,
// layers.rs:433-497, 325-376) fused with the quantization of its output:
// one CTA per token. Sum of squares in two 8-lane FMA accumulators over
// 16-element strides (+ one extra 8-chunk into the first), lane-wise add,
// tree, scalar tail; inv = 1/sqrt(ss/n + eps); y = (x * inv) * w; y is then
// quantized group by group (one warp per group). With `residual` set, x is
// also copied there (the residual stream).
__global__ void __launch_bounds__(256) norm_quant_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                         int n, float eps, float* __restrict__ residual,
                                                         float* __restrict__ normed_out, const int* m_dev, int M,
                                                         int gs, int wbits, uint8_t* __restrict__ act,
                                                         int tok_alloc, TpLink tp, int slot, uint32_t* err) {
  extern __shared__ __align__(16) float sxn[];  // n floats of the row, then n of w
  float* sw = sxn + n;
  __shared__ float lanes[16];
  __shared__ float s_inv;
  __shared__ uint32_t sqw[8][32];
  // The norm weights are model constants: fetched while the previous kernel
  // (programmatic dependent launch) still runs.
  stage_f32(sw, w, n, threadIdx.x, blockDim.x);
  pdl_wait_prior();
  pdl_launch_dependents();
  // Tensor parallelism: x is assembled from every rank's projection rows.
  if (slot >= 0 && !tp_exchange(tp, slot, 0, err)) return;
  const int warp = threadIdx.x >> 5;
  const int mact = m_dev ? *m_dev : M;
  const int groups = (n + gs - 1) / gs;
  const int rows = act ? min(tok_alloc, (mact + 7) & ~7) : mact;
  for (int b = blockIdx.x; b < rows; b += gridDim.x) {
  if (b >= mact) {
    for (int g = warp; g < groups; g += 8) zero_group_warp(b, act, groups, g);
    continue;
  }
  stage_f32(sxn, x + (size_t)b * n, n, threadIdx.x, blockDim.x);
  cp_async_wait<0>();
  __syncthreads();
  if (residual)
    for (int i = threadIdx.x; i < n; i += blockDim.x) residual[(size_t)b * n + i] = sxn[i];
  const int chunks8 = n / 8, chunks16 = chunks8 / 2;
  if (threadIdx.x < 16) {
    const int j = threadIdx.x & 7, half = threadIdx.x >> 3;
    float acc = 0.f;
    int c = 0;
    for (; c + 8 <= chunks16; c += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = sxn[16 * (c + u) + 8 * half + j];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fmaf_rn(v[u], v[u], acc);
    }
    for (; c < chunks16; ++c) {
      const float v = sxn[16 * c + 8 * half + j];
      acc = __fmaf_rn(v, v, acc);
    }
    if (half == 0 && 16 * chunks16 + 8 <= n) {
      const float v = sxn[16 * chunks16 + j];
      acc = __fmaf_rn(v, v, acc);
    }
    lanes[threadIdx.x] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a[8];
    for (int j = 0; j < 8; ++j) a[j] = __fadd_rn(lanes[j], lanes[8 + j]);
    float ss = hsum8(a);
    for (int i = chunks8 * 8; i < n; ++i) ss = __fadd_rn(ss, __fmul_rn(sxn[i], sxn[i]));
    s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
  }
  __syncthreads();
  const float inv = s_inv;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float y = __fmul_rn(__fmul_rn(sxn[i], inv), sw[i]);
    sxn[i] = y;
    if (normed_out) normed_out[(size_t)b * n + i] = y;
  }
  __syncthreads();
  if (act)
    for (int g = warp; g < groups; g += 8)
      quant_group_warp(sxn + g * gs, min(gs, n - g * gs), wbits, b, act, groups, g, sqw[warp]);
  __syncthreads();  // the shared row is reused by the next row
  }
}

// SwiGLU of rai-infer (silu_mul_avx2, layers.rs:850-883) fused with the
// quantization of its output: one warp per (token, group) of the ff-wide
// activation; gate/up rows are [gate | up] of width 2*ff. Schraudolph's exp
// for the first (ff/8)*8 columns, the host-libm expf for the tail;
// y = (x / (1 + e)) * up.
// Under tensor parallelism the rows hold this rank's ff slice (columns
// col_off .. col_off + ff of the model's ff_full); the Schraudolph / expf
// split follows the model's column index.
__global__ void swiglu_quant_kernel(const float* __restrict__ gu, int ff, const int* m_dev, int M, int gs,
                                    ExpfTable et, ActDst dst, int tok_alloc, int col_off, int ff_full) {
  __shared__ __align__(16) float sx[8][128];
  __shared__ uint32_t sqw[8][32];
  pdl_wait_prior();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x;
  const int mact = m_dev ? *m_dev : M;
  const int rows = min(tok_alloc, (mact + 7) & ~7);
  const int len = min(gs, ff - g * gs);
  const int vec_end = (ff_full / 8) * 8;
  for (int tok = blockIdx.y * 8 + warp; tok < rows; tok += gridDim.y * 8) {
  if (tok >= mact) {
    zero_group_warp(tok, dst, g);
    continue;
  }
  const float* row = gu + (size_t)tok * 2 * ff;
  // len <= 128: every lane's gate and up values are loaded before the math.
  float xv[4], uv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = lane + 32 * k;
    xv[k] = i < len ? row[g * gs + i] : 0.f;
    uv[k] = i < len ? row[ff + g * gs + i] : 0.f;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = lane + 32 * k;
    if (i >= len) continue;
    const int col = g * gs + i;
    float sv;
    if (col + col_off < vec_end) {
      const float e = schraudolph(__fmul_rn(xv[k], -1.0f));
      sv = __fdiv_rn(xv[k], __fadd_rn(1.0f, e));
    } else {
      sv = __fdiv_rn(xv[k], __fadd_rn(1.0f, expf_host(-xv[k], et)));
    }
    sx[warp][i] = __fmul_rn(sv, uv[k]);
  }
  __syncwarp();
  quant_group_warp(sx[warp], len, 4, tok, dst, g, sqw[warp]);
  }
  if (dst.n > 1) __threadfence_system();
}

// ---------------------------------------------------------------------------
// The exact GEMM
// ---------------------------------------------------------------------------
struct GemmParams {
  const uint8_t* w;
  const uint8_t* act;
  float* out;
  const float* bias;
  const float* residual;
  uint32_t* err;
  const int* m_dev;  // active token count (device); overrides M when set
  int rows, groups, M, tok_alloc, ld_out, mode, stages;
  int tiles;  // work item i = (row tile i % tiles, token chunk i / tiles); tiles = 64-row tiles x split
  int split;  // CTAs per 64-row tile (1, or the lane groups of a SPLIT variant)
  // Grouped (mixture-of-experts) form, when moe_off is set: ne weight sets of
  // the same shape at w + e * w_stride; expert e's tokens are activation rows
  // moe_off[e] .. moe_off[e] + moe_cnt[e] (moe_off[e] a multiple of 8).
  const int* moe_off;
  const int* moe_cnt;
  int ne;       // weight sets (experts) of this launch: model experts moe_e0 .. moe_e0 + ne
  int moe_e0;
  size_t w_stride;
  // Tensor parallelism: the activations are complete once exchange slot
  // wait_slot (>= 0) is; the result rows also go to outs[1 .. n_out) (the
  // peers' copies of `out`).
  TpLink tp;
  int wait_slot;
  int n_out;
  float* outs[kMaxTp];
};

constexpr int kMaxExperts = 256;

// A work item: the weight set, 64-row tile (and its part `sub` of `split`)
// and token range it covers.
struct GemmItem {
  const uint8_t* w;
  int tile, t0, nt, sub;
};

// Dense form: item = (row tile item % tiles, token chunk item / tiles).
// Grouped form: items run expert by expert (cum[e] = items before expert e).
template <int NT>
__device__ __forceinline__ bool decode_item(const GemmParams& p, const int* cum, int mact, int item, GemmItem* it) {
  if (!p.moe_off) {
    const int t0 = (item / p.tiles) * kTokChunk;
    if (t0 >= mact) return false;
    const int x = item % p.tiles;
    *it = GemmItem{p.w, x / p.split, t0, min(NT, mact - t0), x % p.split};
    return true;
  }
  if (item >= cum[p.ne]) return false;
  int e = 0;
  while (cum[e + 1] <= item) ++e;
  const int local = item - cum[e], chunk = local / p.tiles;
  *it = GemmItem{p.w + (size_t)e * p.w_stride, local % p.tiles, p.moe_off[p.moe_e0 + e] + chunk * kTokChunk,
                 min(kTokChunk, p.moe_cnt[p.moe_e0 + e] - chunk * kTokChunk), 0};
  return true;
}

__device__ __forceinline__ void mma_u8s8(uint32_t a0, uint32_t a1, uint32_t b, int32_t d[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%7,%7,%7,%7};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b), "r"(kMagic));
}

// Packed pairs of f32 for the exact epilogue. mul.rn.f32x2 rounds each half
// exactly like the scalar mul.rn (checked bit for bit on the device), and
// sub.rn.f32x2 is only used for (12582912 + dot) - 12582912, which is exact
// in any rounding mode. Accumulation stays scalar __fadd_rn: a packed
// mul.rn.f32x2 -> add.rn.f32x2 chain did not reproduce the scalar rounding
// on sm_100a, so packed adds are not used.
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// acc[0..1] += exact_dot(d0, d1) * c, each term rounded as the reference.
__device__ __forceinline__ void acc_pair(float* acc, int32_t d0, int32_t d1, uint64_t c, uint64_t magic2) {
  const float2 pr = f2_unpack(mul2(sub2(f2(__int_as_float(d0), __int_as_float(d1)), magic2), c));
  acc[0] = __fadd_rn(acc[0], pr.x);
  acc[1] = __fadd_rn(acc[1], pr.y);
}

// Groups per pipeline stage: a stage carries kGPS consecutive groups of the
// tile's packed weights (one contiguous bulk copy) and the matching
// activation blocks (one copy per 8-token block), so the bulk-copy and
// mbarrier overhead is paid once per kGPS groups.
constexpr int kGPS = 4;

template <int NTILES>
struct StageCfg {
  static constexpr int kBlocks = NTILES;  // 8-token activation blocks per item
  static constexpr int kActOff = kGPS * kBlockBytes;
  static constexpr int kBytes = kGPS * kBlockBytes + kBlocks * kGPS * kActBlockBytes;
};

// Lane-pair fragments of one consumer warp: pair jj covers reference lanes
// j = j0 + jj ([0]) and j + 4 ([1]).
template <int NP>
__device__ __forceinline__ void load_words(const uint8_t* p, uint32_t (&w)[NP]) {
  if constexpr (NP == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (NP == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}

template <int WBITS, class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, Cfg::kMinBlocks) gemm_exact_kernel(GemmParams p) {
  constexpr int NTILES = Cfg::NTILES, LG = Cfg::LG;
  static_assert(WBITS == 4 || LG == 1, "the tied head runs unsplit");
  constexpr int kConsumerWarps = Cfg::kConsumerWarps;
  constexpr int NW = Cfg::kTilesPerWarp;  // N tiles per consumer warp
  constexpr int NP = Cfg::kPairs;         // lane pairs per consumer warp
  constexpr int NT = 8 * NTILES;          // token slots per work item
  constexpr int kStageBytes = StageCfg<NTILES>::kBytes;
  constexpr int kActOff = StageCfg<NTILES>::kActOff;
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * kStageBytes);
  uint64_t* empty = full + S;
  constexpr int kSlabTeams = 4 * Cfg::TS;  // (slab, token split) warp teams
  uint64_t* cfull = empty + S;            // per team: the other lane groups posted their sums
  uint64_t* cfree = cfull + kSlabTeams;   // per team: the first lane group has read them
  float* comb = reinterpret_cast<float*>(cfree + kSlabTeams);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.groups, tiles = p.tiles;
  const int nsg = (G + kGPS - 1) / kGPS;  // stages per work item
  // Persistent CTAs: each walks work items blockIdx.x, + gridDim.x, ...
  // (chunk-major, so a CTA's first item is token chunk 0 whenever
  // blockIdx.x < tiles). Chunk 0 always has work: the producer of such a
  // "lead" CTA requests its first item's weights before waiting on the
  // previous kernel (programmatic dependent launch). Other CTAs wait first
  // and exit, before touching any barrier, when they have no item. The
  // grouped form learns its items from the routing (written by earlier
  // kernels), so none of its CTAs is a lead.
  const bool lead = !p.moe_off && (int)blockIdx.x < tiles;
  __shared__ int cum[kMaxExperts + 1];
  int mact = p.M;
  if (!lead) {
    pdl_wait_prior();
    if (p.m_dev) mact = *p.m_dev;
    if (!p.moe_off && (int)(blockIdx.x / tiles) * kTokChunk >= mact) return;
    if (p.moe_off) {
      if (threadIdx.x == 0) {
        int c = 0;
        for (int e = 0; e < p.ne; ++e) {
          cum[e] = c;
          c += tiles * ((p.moe_cnt[p.moe_e0 + e] + kTokChunk - 1) / kTokChunk);
        }
        cum[p.ne] = c;
      }
      __syncthreads();
      if ((int)blockIdx.x >= cum[p.ne]) return;
    }
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int k = 0; k < kSlabTeams; ++k) {
      mbar_init(&cfull[k], LG > 1 ? LG - 1 : 1);
      mbar_init(&cfree[k], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const int pre = min(S, nsg);
      if (lead) {
        // Weights do not depend on the previous kernel: the first item's
        // first ring's worth is requested before waiting on it.
        for (int q = 0; q < pre; ++q) {
          const int g0 = q * kGPS, ng = min(kGPS, G - g0);
          mbar_expect_tx(&full[q], ng * kBlockBytes);
          bulk_g2s(smem + (size_t)q * kStageBytes, p.w + ((size_t)(blockIdx.x / p.split) * G + g0) * kBlockBytes,
                   ng * kBlockBytes, &full[q]);
        }
        pdl_wait_prior();
        if (p.m_dev) mact = *p.m_dev;
      }
      bool ok = true, first = true;
      if (p.wait_slot >= 0) {
        // The activations come from every rank: CTA 0 signals that this
        // rank's producer kernel is done, then all wait for the others. The
        // peers wrote them with generic stores; the copies below read them
        // through the async proxy.
        if (blockIdx.x == 0) tp_signal(p.tp, p.wait_slot);
        ok = tp_wait(p.tp, p.wait_slot, 0, p.err);
        asm volatile("fence.proxy.async;" ::: "memory");
      }
      int s = 0;       // ring stage of the next fill
      uint32_t n = 0;  // previous fills of stage s
      for (int item = blockIdx.x; ok; item += gridDim.x, first = false) {
        GemmItem it;
        if (!decode_item<NT>(p, cum, mact, item, &it)) break;
        const int nb = (it.nt + 7) >> 3;  // 8-token activation blocks
        const uint8_t* ab = p.act + (size_t)(it.t0 >> 3) * G * kActBlockBytes;
        for (int q = 0; q < nsg; ++q) {
          if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, p.err)) { ok = false; break; }
          const int g0 = q * kGPS, ng = min(kGPS, G - g0);
          uint8_t* st = smem + (size_t)s * kStageBytes;
          const bool prefetched = lead && first && q < pre;
          const uint32_t abytes = nb * ng * kActBlockBytes;
          mbar_arrive_expect_tx(&full[s], prefetched ? abytes : ng * kBlockBytes + abytes);
          if (!prefetched)
            bulk_g2s(st, it.w + ((size_t)it.tile * G + g0) * kBlockBytes, ng * kBlockBytes, &full[s]);
          for (int b = 0; b < nb; ++b)
            bulk_g2s(st + kActOff + b * kGPS * kActBlockBytes, ab + ((size_t)b * G + g0) * kActBlockBytes,
                     ng * kActBlockBytes, &full[s]);
          if (++s == S) {
            s = 0;
            ++n;
          }
        }
      }
      if (!ok) {
        // Gave up: wait (bounded) for this CTA's copies still in flight.
        for (int k = 0; k < S; ++k) {
          if (++s == S) {
            s = 0;
            ++n;
          }
          if (n > 0) mbar_wait(&full[s], (n - 1) & 1, nullptr);
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  if (lead) {
    pdl_wait_prior();
    if (p.m_dev) mact = *p.m_dev;
  }
  pdl_launch_dependents();
  const int gq = lane >> 2, tq = lane & 3;
  // SPLIT: warp w = (slab w / LG of the item's part, lane group w % LG).
  const int lg = Cfg::SPLIT ? warp % LG : (warp >> 2) % LG;  // lane group within the slab
  const int team = Cfg::SPLIT ? warp / LG : (warp & 3) + 4 * ((warp >> 2) / LG);  // (slab, token split)
  const int nbase = Cfg::SPLIT ? 0 : ((warp >> 2) / LG) * NW;  // this warp's first N tile
  const int j0 = lg * NP;                                      // first lane pair
  int r0 = (warp & 3) * 16 + gq;                               // tile-local rows r0 and r0 + 8
  const uint64_t magic2 = f2(kMagicF, kMagicF);
  int cs = 0;           // ring stage of the next stage to consume
  uint32_t cphase = 0;  // its fill parity
  uint32_t nitems = 0;  // items finished by this warp
  for (int item = blockIdx.x;; item += gridDim.x) {
    GemmItem it;
    if (!decode_item<NT>(p, cum, mact, item, &it)) break;
    const int tile = it.tile, t0 = it.t0;
    if constexpr (Cfg::SPLIT) r0 = (it.sub * (4 / LG) + warp / LG) * 16 + gq;
    const int nbi = (it.nt + 7) >> 3;  // 8-token blocks holding this item's tokens
    float facc[NW][NP][2][4];
    float zc[NW][4];
#pragma unroll
    for (int n = 0; n < NW; ++n) {
#pragma unroll
      for (int i = 0; i < 4; ++i) zc[n][i] = 0.f;
#pragma unroll
      for (int jj = 0; jj < NP; ++jj)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int i = 0; i < 4; ++i) facc[n][jj][h][i] = 0.f;
    }

    for (int q = 0; q < nsg; ++q) {
      const int s = cs;
      if (!mbar_wait(&full[s], cphase, p.err)) return;
      if (++cs == S) {
        cs = 0;
        cphase ^= 1u;
      }
      const uint8_t* st = smem + (size_t)s * kStageBytes;
      const int ng = min(kGPS, G - q * kGPS);
      // A warp whose N tiles all lie past the item's tokens only frees the stage.
#pragma unroll(Cfg::kUnroll)
      for (int gi = 0; gi < (nbase < nbi ? ng : 0); ++gi) {
        const uint8_t* W = st + gi * kBlockBytes;
        const uint32_t* P = reinterpret_cast<const uint32_t*>(W + kWeightStageBytes);
        const uint8_t* A = st + kActOff + gi * kActBlockBytes;  // + block * kGPS * kActBlockBytes

        uint32_t A0[NP][2], A1[NP][2];
        if constexpr (WBITS == 4) {
          // Word j of the thread's 16-byte slot: lane j (low nibbles), lane j + 4 (high).
          uint32_t wa[NP], wb[NP];
          load_words<NP>(W + r0 * kRowGroupBytes + tq * 16 + j0 * 4, wa);
          load_words<NP>(W + (r0 + 8) * kRowGroupBytes + tq * 16 + j0 * 4, wb);
#pragma unroll
          for (int jj = 0; jj < NP; ++jj) {
            A0[jj][0] = wa[jj] & 0x0F0F0F0Fu;
            A0[jj][1] = (wa[jj] >> 4) & 0x0F0F0F0Fu;
            A1[jj][0] = wb[jj] & 0x0F0F0F0Fu;
            A1[jj][1] = (wb[jj] >> 4) & 0x0F0F0F0Fu;
          }
        } else {
          // 8-bit codes: word L of the thread's 32 bytes is lane L.
          if (tq < 2) {
            const uint4* pa = reinterpret_cast<const uint4*>(W + r0 * kRowGroupBytes + tq * 32);
            const uint4* pb = reinterpret_cast<const uint4*>(W + (r0 + 8) * kRowGroupBytes + tq * 32);
            const uint4 a_lo = pa[0], a_hi = pa[1], b_lo = pb[0], b_hi = pb[1];
            const uint32_t a_[8] = {a_lo.x, a_lo.y, a_lo.z, a_lo.w, a_hi.x, a_hi.y, a_hi.z, a_hi.w};
            const uint32_t b_[8] = {b_lo.x, b_lo.y, b_lo.z, b_lo.w, b_hi.x, b_hi.y, b_hi.z, b_hi.w};
#pragma unroll
            for (int jj = 0; jj < NP; ++jj) {
              A0[jj][0] = a_[jj]; A0[jj][1] = a_[jj + 4];
              A1[jj][0] = b_[jj]; A1[jj][1] = b_[jj + 4];
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < NP; ++jj) A0[jj][0] = A0[jj][1] = A1[jj][0] = A1[jj][1] = 0u;
          }
        }
        const uint32_t p0 = P[r0], p1 = P[r0 + 8];
        const float ws0 = f16_bits_to_f32((uint16_t)(p0 & 0xFFFF));
        const float ws1 = f16_bits_to_f32((uint16_t)(p1 & 0xFFFF));

#pragma unroll
        for (int n = 0; n < NW; ++n) {
          if (nbase + n >= nbi) break;  // N tiles past the item's tokens
          // N tile (nbase + n) = activation block (nbase + n); token gq of it.
          const uint8_t* blk = A + (nbase + n) * kGPS * kActBlockBytes;
          const uint8_t* qrow = blk + gq * kActRowBytes;
          uint32_t B[NP][2];
          if constexpr (WBITS == 4) {
            // Unit 2tq holds lanes (0,4,1,5), unit 2tq+1 lanes (2,6,3,7).
            if constexpr (NP == 4) {
              const uint4 u0 = *reinterpret_cast<const uint4*>(qrow + (((2 * tq) ^ gq) << 4));
              const uint4 u1 = *reinterpret_cast<const uint4*>(qrow + (((2 * tq + 1) ^ gq) << 4));
              B[0][0] = u0.x; B[0][1] = u0.y; B[1][0] = u0.z; B[1][1] = u0.w;
              B[2][0] = u1.x; B[2][1] = u1.y; B[3][0] = u1.z; B[3][1] = u1.w;
            } else if constexpr (NP == 2) {
              const uint4 u = *reinterpret_cast<const uint4*>(qrow + (((2 * tq + lg) ^ gq) << 4));
              B[0][0] = u.x; B[0][1] = u.y; B[1][0] = u.z; B[1][1] = u.w;
            } else {
              const uint2 u =
                  *reinterpret_cast<const uint2*>(qrow + (((2 * tq + (lg >> 1)) ^ gq) << 4) + (lg & 1) * 8);
              B[0][0] = u.x; B[0][1] = u.y;
            }
          } else {
            // Tied head: unit 2tq holds lanes 0..3, unit 2tq+1 lanes 4..7.
            const uint4 u0 = *reinterpret_cast<const uint4*>(qrow + (((2 * tq) ^ gq) << 4));
            const uint4 u1 = *reinterpret_cast<const uint4*>(qrow + (((2 * tq + 1) ^ gq) << 4));
            const uint32_t x0[4] = {u0.x, u0.y, u0.z, u0.w}, x1[4] = {u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int jj = 0; jj < NP; ++jj) {
              B[jj][0] = x0[jj];
              B[jj][1] = x1[jj];
            }
          }
          const float2* XS = reinterpret_cast<const float2*>(blk + kActBlockTok * kActRowBytes);
          const float2 xa = XS[2 * tq], xb = XS[2 * tq + 1];
          // combined_scale = w_scale * x_scale (gemm.rs:606, 493)
          const uint64_t xs2 = f2(xa.x, xb.x);
          const uint64_t c0 = mul2(f2(ws0, ws0), xs2), c1 = mul2(f2(ws1, ws1), xs2);
#pragma unroll
          for (int jj = 0; jj < NP; ++jj) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              int32_t d[4];
              mma_u8s8(A0[jj][h], A1[jj][h], B[jj][h], d);
              acc_pair(&facc[n][jj][h][0], d[0], d[1], c0, magic2);
              acc_pair(&facc[n][jj][h][2], d[2], d[3], c1, magic2);
            }
          }
          if (lg == 0) {
            // zero correction: sum_g w_zero * x_sum, sequential in g (gemm.rs:666-670)
            const float wz0 = f16_bits_to_f32((uint16_t)(p0 >> 16));
            const float wz1 = f16_bits_to_f32((uint16_t)(p1 >> 16));
            zc[n][0] = __fadd_rn(zc[n][0], __fmul_rn(wz0, xa.y));
            zc[n][1] = __fadd_rn(zc[n][1], __fmul_rn(wz0, xb.y));
            zc[n][2] = __fadd_rn(zc[n][2], __fmul_rn(wz1, xa.y));
            zc[n][3] = __fadd_rn(zc[n][3], __fmul_rn(wz1, xb.y));
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // Horizontal-sum tree ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)): pair j
    // gives s_j = a_j + a_{j+4}; a warp finishes the pairs it holds.
    float part[NW][4];
#pragma unroll
    for (int n = 0; n < NW; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float sj[NP];
#pragma unroll
        for (int jj = 0; jj < NP; ++jj) sj[jj] = __fadd_rn(facc[n][jj][0][i], facc[n][jj][1][i]);
        if constexpr (NP == 4) part[n][i] = __fadd_rn(__fadd_rn(sj[0], sj[1]), __fadd_rn(sj[2], sj[3]));
        else if constexpr (NP == 2) part[n][i] = __fadd_rn(sj[0], sj[1]);
        else part[n][i] = sj[0];
      }
    if constexpr (LG > 1) {
      float* cb = comb + (size_t)team * (LG - 1) * NW * 4 * 32;
      if (lg > 0) {
        if (nitems > 0 && !mbar_wait(&cfree[team], (nitems - 1) & 1, p.err)) return;
#pragma unroll
        for (int n = 0; n < NW; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) cb[(((lg - 1) * NW + n) * 4 + i) * 32 + lane] = part[n][i];
        __syncwarp();
        if (lane == 0) mbar_arrive(&cfull[team]);
        ++nitems;
        continue;
      }
      if (!mbar_wait(&cfull[team], nitems & 1, p.err)) return;
#pragma unroll
      for (int n = 0; n < NW; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float* c = cb + (n * 4 + i) * 32 + lane;  // lane group g at c[(g - 1) * NW * 128]
          if constexpr (LG == 2) part[n][i] = __fadd_rn(part[n][i], c[0]);
          else part[n][i] = __fadd_rn(__fadd_rn(part[n][i], c[0]), __fadd_rn(c[NW * 128], c[2 * NW * 128]));
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&cfree[team]);
    }
    ++nitems;

    // Epilogue: + zero correction, then bias / residual.
#pragma unroll
    for (int n = 0; n < NW; ++n) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = tile * kTileRows + r0 + ((i & 2) ? 8 : 0);
        const int tok = t0 + (nbase + n) * 8 + 2 * tq + (i & 1);
        if (row >= p.rows || tok - t0 >= it.nt) continue;
        float v = __fadd_rn(part[n][i], zc[n][i]);
        const size_t o = (size_t)tok * p.ld_out + row;
        if (p.mode == kEpiBias) v = __fadd_rn(v, p.bias[row]);
        else if (p.mode == kEpiResidual) v = __fadd_rn(p.residual[o], v);
        p.out[o] = v;
        for (int d = 1; d < p.n_out; ++d) p.outs[d][o] = v;
      }
    }
  }
  if (p.n_out > 1) __threadfence_system();
}

int sm_count() { return device_sm_count(); }

template <class Cfg>
size_t gemm_smem_bytes(int stages) {
  return (size_t)stages * StageCfg<Cfg::NTILES>::kBytes + (2 * stages + 8 * Cfg::TS) * sizeof(uint64_t) +
         Cfg::kCombBytes;
}

// Dynamic shared memory limit raised for every variant (the static arrays
// and the per-CTA reservation stay within the SM's 228 KB).
constexpr int kGemmSmemMax = 210 * 1024;

// Ring stages that fit kMinBlocks CTAs per SM (228 KB of shared memory per
// SM, less each CTA's static arrays), at most 8 and at most the item's.
template <class Cfg>
int gemm_stages(int groups) {
  int per_cta = (228 * 1024) / Cfg::kMinBlocks - 3 * 1024;
  if (per_cta > kGemmSmemMax) per_cta = kGemmSmemMax;
  int stages = (int)((per_cta - gemm_smem_bytes<Cfg>(0)) / StageCfg<Cfg::NTILES>::kBytes);
  const int nsg = (groups + kGPS - 1) / kGPS;
  if (stages > 8) stages = 8;
  if (stages > nsg) stages = nsg;
  return stages < 2 ? 2 : stages;
}

template <int WBITS, class Cfg>
cudaError_t launch_gemm(const GemmParams& gp, int tiles, int chunks, cudaStream_t s) {
  const int stages = gemm_stages<Cfg>(gp.groups);
  GemmParams p = gp;
  p.stages = stages;
  p.split = Cfg::SPLIT ? Cfg::LG : 1;
  tiles *= p.split;
  p.tiles = tiles;
  auto kern = gemm_exact_kernel<WBITS, Cfg>;
  const size_t smem = gemm_smem_bytes<Cfg>(stages);
  // One persistent wave: as many CTAs as are resident at once, never more
  // than the work items of the static token budget. Residency is measured
  // once for the largest ring this variant uses.
  static const int resident = [] {
    int n = 0;
    const size_t full = gemm_smem_bytes<Cfg>(gemm_stages<Cfg>(1 << 20));
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemm_exact_kernel<WBITS, Cfg>, Cfg::kThreads, full) !=
            cudaSuccess || n < 1)
      n = 1;
    return n;
  }();
  const long items = (long)tiles * chunks;
  const long wave = (long)sm_count() * resident;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(items < wave ? items : wave));
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // programmatic dependent launch (see pdl_wait_prior)
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// Variants used, by N tiles per item: 4-bit linear and 8-bit tied head.
using Gemm4N1 = GemmCfg<1, 1, 1, 2, 4>;
using Gemm4N2 = GemmCfg<2, 1, 1, 2, 1>;
using Gemm4N3 = GemmCfg<3, 1, 1, 1, 1>;
using Gemm4N4 = GemmCfg<4, 1, 2, 1, 1>;
// Candidates with one 8-token N tile per consumer warp (more warps in flight,
// each with a shorter chain): 32-token items over 16 consumer warps, 16-token
// items over 8. RAI_GEMM_VARIANT=1 selects them (A/B measurement).
using Gemm4N4W = GemmCfg<4, 1, 4, 1, 1>;
using Gemm4N2W = GemmCfg<2, 1, 2, 1, 1>;
// Launches with fewer tiles than SMs: each 64-row tile split over 2 or 4
// CTAs.
using Gemm4N1S2 = GemmCfg<1, 2, 1, 2, 4, true>;
using Gemm4N1S4 = GemmCfg<1, 4, 1, 2, 4, true>;
using Gemm4N2S2 = GemmCfg<2, 2, 1, 2, 1, true>;
using Gemm4N2S4 = GemmCfg<2, 4, 1, 2, 1, true>;
using Gemm8N1 = GemmCfg<1, 1, 1, 2, 1>;
using Gemm8N2 = GemmCfg<2, 1, 1, 2, 1>;
using Gemm8N3 = GemmCfg<3, 1, 1, 1, 1>;
using Gemm8N4 = GemmCfg<4, 1, 2, 1, 1>;

// CTAs per 64-row tile for a launch of `items` (tile, token chunk) items:
// 1 when the items fill the SMs, 2 or 4 when most SMs would otherwise idle.
// RAI_GEMM_SPLIT=1|2|4 forces one.
int gemm_split(long items) {
  static const int forced = [] {
    const char* e = std::getenv("RAI_GEMM_SPLIT");
    return e ? std::atoi(e) : 0;
  }();
  if (forced == 1 || forced == 2 || forced == 4) return forced;
  const long sms = sm_count();
  return items * 4 <= sms ? 4 : items * 2 <= sms ? 2 : 1;
}

}  // namespace

cudaError_t init_gemm_attributes() {
  // Raised once per process, before any stream capture.
  const int bytes = kGemmSmemMax;
  cudaError_t e = cudaSuccess;
  auto set = [&](auto kern) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  };
  set(gemm_exact_kernel<4, Gemm4N1>); set(gemm_exact_kernel<4, Gemm4N2>);
  set(gemm_exact_kernel<4, Gemm4N3>); set(gemm_exact_kernel<4, Gemm4N4>);
  set(gemm_exact_kernel<4, Gemm4N4W>); set(gemm_exact_kernel<4, Gemm4N2W>);
  set(gemm_exact_kernel<4, Gemm4N1S2>); set(gemm_exact_kernel<4, Gemm4N1S4>);
  set(gemm_exact_kernel<4, Gemm4N2S2>); set(gemm_exact_kernel<4, Gemm4N2S4>);
  set(gemm_exact_kernel<8, Gemm8N1>); set(gemm_exact_kernel<8, Gemm8N2>);
  set(gemm_exact_kernel<8, Gemm8N3>); set(gemm_exact_kernel<8, Gemm8N4>);
  if (e == cudaSuccess) e = init_gemm_tc_attributes();
  if (e == cudaSuccess) e = init_gemm_tol_attributes();
  return e;
}

cudaError_t pack_linear4(const uint8_t* nibbles, const uint8_t* params, int rows, int cols, int gs,
                         uint8_t* out, cudaStream_t s) {
  int groups = (int)ceil_div(cols, gs);
  size_t total = packed_linear_bytes(rows, cols, gs);
  int threads = 256;
  size_t blocks = ceil_div(total, threads);
  pack4_kernel<<<(unsigned)blocks, threads, 0, s>>>(nibbles, params, rows, cols, gs, groups, out, total);
  return cudaGetLastError();
}

cudaError_t pack_linear8(const uint8_t* codes, const uint8_t* params, int rows, int cols, int gs,
                         uint8_t* out, cudaStream_t s) {
  int groups = (int)ceil_div(cols, gs);
  size_t total = packed_linear_bytes(rows, cols, gs);
  int threads = 256;
  size_t blocks = ceil_div(total, threads);
  pack8_kernel<<<(unsigned)blocks, threads, 0, s>>>(codes, params, rows, cols, gs, groups, out, total);
  return cudaGetLastError();
}

cudaError_t quantize_act(const float* x, int ldx, int M, const int* m_dev, int K, int gs, int wbits,
                         ActBuf act, cudaStream_t s, const ActDst* dst) {
  const int groups = (int)ceil_div(K, gs);  // groups this kernel quantizes
  ActDst d;
  if (dst) d = *dst;
  else { d.data[0] = act.data; d.n = 1; d.groups = act.groups; d.g_off = 0; }
  const int chunks = (int)ceil_div(act.tok_alloc, 8);
  dim3 grid((unsigned)groups, (unsigned)std::max(1, std::min(chunks, grid_cap(groups * chunks, 4) / groups)));
  return launch_pdl(quantize_kernel, grid, dim3(256), 0, s, x, ldx, M, m_dev, K, gs, wbits, d, act.tok_alloc);
}

cudaError_t norm_quant(const float* x, const float* w, int n, float eps, float* residual, int M,
                       const int* m_dev, int gs, int wbits, ActBuf act, cudaStream_t s, float* normed_out,
                       const TpLink* tp, int slot, uint32_t* err) {
  const int rows = act.data ? (int)min((size_t)act.tok_alloc, round_up((size_t)M, 8)) : M;
  TpLink link;
  if (tp && tp->world > 1 && slot >= 0) link = *tp;
  else slot = -1;
  return launch_pdl(norm_quant_kernel, dim3((unsigned)grid_cap(rows, 1)), dim3(256), 2 * (size_t)n * sizeof(float),
                    s, x, w, n, eps, residual, normed_out, m_dev, M, gs, wbits, act.data, act.tok_alloc, link, slot,
                    err);
}

cudaError_t gemm_grouped(const PackedLinear& w, size_t w_stride, int ne, const int* off, const int* cnt,
                         const ActBuf& act, float* out, int ld_out, uint32_t* err, cudaStream_t s, int e0,
                         const GemmTp* tp) {
  if (ne < 1 || ne > kMaxExperts || w.wbits != 4) return cudaErrorInvalidValue;
  GemmParams gp = {};
  gp.w = w.data;
  gp.act = act.data;
  gp.out = out;
  gp.err = err;
  gp.rows = w.rows;
  gp.groups = w.groups;
  gp.M = act.tok_alloc;
  gp.tok_alloc = act.tok_alloc;
  gp.ld_out = ld_out;
  gp.mode = kEpiStore;
  gp.moe_off = off;
  gp.moe_cnt = cnt;
  gp.ne = ne;
  gp.moe_e0 = e0;
  gp.w_stride = w_stride;
  gp.wait_slot = -1;
  gp.n_out = 1;
  if (tp && tp->link.world > 1) {
    gp.n_out = tp->n_out > 0 ? tp->n_out : 1;
    for (int d = 0; d < gp.n_out; ++d) gp.outs[d] = tp->outs[d];
  }
  // Items are known only on the device: one full persistent wave.
  return launch_gemm<4, Gemm4N4>(gp, w.tiles, 1 << 20, s);
}

cudaError_t swiglu_quant(const float* gu, int ff, int M, const int* m_dev, int gs, const ExpfTable& et, ActBuf act,
                         cudaStream_t s, const ActDst* dst, int col_off, int ff_full) {
  const int groups = (int)ceil_div(ff, gs);
  ActDst d;
  if (dst) d = *dst;
  else { d.data[0] = act.data; d.n = 1; d.groups = act.groups; d.g_off = 0; }
  const int chunks = (int)ceil_div(act.tok_alloc, 8);
  dim3 grid((unsigned)groups, (unsigned)std::max(1, std::min(chunks, grid_cap(groups * chunks, 4) / groups)));
  return launch_pdl(swiglu_quant_kernel, grid, dim3(256), 0, s, gu, ff, m_dev, M, gs, et, d, act.tok_alloc, col_off,
                    ff_full > 0 ? ff_full : ff);
}

cudaError_t gemm_exact(const PackedLinear& w, const ActBuf& act, int M, float* out, int ld_out,
                       const GemmEpilogue& epi, uint32_t* err, cudaStream_t s, bool pdl, const int* m_dev,
                       const GemmTp* tp, const GemmPolicy* pol) {
  if (M <= 0) return cudaSuccess;
  const bool exchange = tp && tp->link.world > 1;
  if (w.wbits == 4 && !exchange && pol &&
      (pol->mode == kGemmTol || (pol->mode == kGemmAuto && M >= kTolMinRows)))
    return gemm_tol(w, act, M, out, ld_out, epi, err, s, m_dev, pol->ws, pol->ws_bytes);
  if (w.wbits == 4 && w.tc && !exchange && gemm_tc_enabled())
    return gemm_tc(w, act, M, out, ld_out, epi, err, s, m_dev);
  GemmParams gp = {};
  gp.wait_slot = -1;
  gp.n_out = 1;
  if (tp && tp->link.world > 1) {
    gp.tp = tp->link;
    gp.wait_slot = tp->wait_slot;
    gp.n_out = tp->n_out > 0 ? tp->n_out : 1;
    for (int d = 0; d < gp.n_out; ++d) gp.outs[d] = tp->outs[d];
  }
  gp.m_dev = m_dev;
  gp.w = w.data;
  gp.act = act.data;
  gp.out = out;
  gp.bias = epi.bias;
  gp.residual = epi.residual;
  gp.err = err;
  gp.rows = w.rows;
  gp.groups = w.groups;
  gp.M = M;
  gp.tok_alloc = act.tok_alloc;
  gp.ld_out = ld_out;
  gp.mode = epi.mode;
  int per = M < kTokChunk ? M : kTokChunk;
  int ntiles = (per + 7) / 8;
  int chunks = (int)ceil_div(M, kTokChunk);
  (void)pdl;  // every GEMM launch uses programmatic dependent launch
  if (w.wbits == 4) {
    const int split = gemm_split(w.tiles * chunks);
    static const int variant = [] {
      const char* e = std::getenv("RAI_GEMM_VARIANT");
      return e ? std::atoi(e) : 0;
    }();
    if (variant == 1 && ntiles == 4) return launch_gemm<4, Gemm4N4W>(gp, w.tiles, chunks, s);
    if (variant == 1 && ntiles == 2 && split == 1) return launch_gemm<4, Gemm4N2W>(gp, w.tiles, chunks, s);
    switch (ntiles) {
      case 1:
        if (split == 4) return launch_gemm<4, Gemm4N1S4>(gp, w.tiles, chunks, s);
        if (split == 2) return launch_gemm<4, Gemm4N1S2>(gp, w.tiles, chunks, s);
        return launch_gemm<4, Gemm4N1>(gp, w.tiles, chunks, s);
      case 2:
        if (split == 4) return launch_gemm<4, Gemm4N2S4>(gp, w.tiles, chunks, s);
        if (split == 2) return launch_gemm<4, Gemm4N2S2>(gp, w.tiles, chunks, s);
        return launch_gemm<4, Gemm4N2>(gp, w.tiles, chunks, s);
      case 3: return launch_gemm<4, Gemm4N3>(gp, w.tiles, chunks, s);
      default: return launch_gemm<4, Gemm4N4>(gp, w.tiles, chunks, s);
    }
  }
  switch (ntiles) {
    case 1: return launch_gemm<8, Gemm8N1>(gp, w.tiles, chunks, s);
    case 2: return launch_gemm<8, Gemm8N2>(gp, w.tiles, chunks, s);
    case 3: return launch_gemm<8, Gemm8N3>(gp, w.tiles, chunks, s);
    default: return launch_gemm<8, Gemm8N4>(gp, w.tiles, chunks, s);
  }
}

}  // namespace rai
