// Per-(token, group) activation quantization shared by the kernels that feed
// the exact W4A8 GEMM (quantize_input_split_avx2 / compute_input_sums_avx2,
// rai-infer/src/gemm.rs:280-374, 182-212; the tied head's +-63 variant
// quantize_hidden_i8_avx2, gemm.rs:976-1047).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"
#include "tp.cuh"

namespace rai {

// Activation quantization of one (token, group) by one warp.
// ---------------------------------------------------------------------------
// Logical byte (slot t, lane L, elem b) of a token row is at
// t*32 + 4*pos(L) + b, with pos(L) = 2*(L & 3) + (L >> 2) for the 4-bit
// weights (lanes j and j+4 adjacent, matching the packed weight words) and
// pos(L) = L for the tied head; 16-byte unit u = offset/16 is stored at unit
// u ^ (token & 7) so the GEMM's B-fragment loads are bank-conflict free.
// xs: the group's len values in shared memory; sqw: 32 words of per-warp
// shared scratch. act: the activation buffer of `groups` groups (8-token x
// group blocks).
__device__ __forceinline__ uint8_t* act_block(uint8_t* act, int groups, int tok, int g) {
  return act + ((size_t)(tok >> 3) * groups + g) * kActBlockBytes;
}

__device__ __forceinline__ void quant_group_warp(const float* xs, int len, int wbits, int tok, const ActDst& dst,
                                                 int g, uint32_t* sqw) {
  const int lane = threadIdx.x & 31;
  float amax = 0.f;
  for (int i = lane; i < len; i += 32) amax = fmaxf(amax, fabsf(xs[i]));
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float lim = wbits == 4 ? 127.f : 63.f;
  const float lo = wbits == 4 ? -128.f : -63.f;
  const float scale = amax > 1e-10f ? __fdiv_rn(amax, lim) : 1.0f;
  const float inv = __fdiv_rn(1.0f, scale);
  uint8_t* sq = reinterpret_cast<uint8_t*>(sqw);
  sqw[lane] = 0;
  __syncwarp();
  for (int col = lane; col < len; col += 32) {
    float r = rintf(__fmul_rn(xs[col], inv));
    r = fminf(r, lim);
    r = fmaxf(r, lo);
    const int qv = (int)r;
    int off;
    if (wbits == 4) {
      const int c = col >> 6, rr = col & 63, L = rr >> 3, b = (rr & 7) >> 1, p = rr & 1;
      off = (2 * c + p) * 32 + 4 * (2 * (L & 3) + (L >> 2)) + b;
    } else {
      off = (col >> 5) * 32 + (col & 31);  // lane L = (col & 31) / 4, elem b = col % 4
    }
    sq[off] = (uint8_t)(int8_t)qv;
  }
  __syncwarp();
  // Group sum: lane j accumulates columns 8i + j in order, then the tree.
  float accj = 0.f;
  if (lane < 8) {
    // len <= 128: at most 16 chunks; all loads issued before the ordered adds.
    const int chunks8 = len / 8;
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = i < chunks8 ? xs[8 * i + lane] : 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < chunks8) accj = __fadd_rn(accj, v[i]);
  }
  float a[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = __shfl_sync(0xffffffffu, accj, j);
  float sum = hsum8(a);
  for (int i = (len / 8) * 8; i < len; ++i) sum = __fadd_rn(sum, xs[i]);
  // Swizzled store: lane writes 4 bytes of logical unit u = lane / 4, to
  // every destination (the peers' buffers under tensor parallelism).
  const int u = lane >> 2;
  const int phys = ((u ^ (tok & 7)) << 2) | (lane & 3);
  const uint32_t word = sqw[lane];
  for (int d = 0; d < dst.n; ++d) {
    uint8_t* blk = act_block(dst.data[d], dst.groups, tok, g + dst.g_off);
    reinterpret_cast<uint32_t*>(blk + (tok & 7) * kActRowBytes)[phys] = word;
    if (lane == 0) reinterpret_cast<float2*>(blk + kActBlockTok * kActRowBytes)[tok & 7] = make_float2(scale, sum);
  }
  __syncwarp();
}

__device__ __forceinline__ ActDst act_dst(uint8_t* act, int groups) {
  ActDst d;
  d.data[0] = act;
  d.n = 1;
  d.groups = groups;
  d.g_off = 0;
  return d;
}

__device__ __forceinline__ void quant_group_warp(const float* xs, int len, int wbits, int tok, uint8_t* act,
                                                 int groups, int g, uint32_t* sqw) {
  quant_group_warp(xs, len, wbits, tok, act_dst(act, groups), g, sqw);
}

// Zero codes and (scale, sum) of one (token, group): tokens past the active
// count up to the next multiple of 8 (the GEMM reads tokens in groups of 8).
__device__ __forceinline__ void zero_group_warp(int tok, const ActDst& dst, int g) {
  const int lane = threadIdx.x & 31;
  for (int d = 0; d < dst.n; ++d) {
    uint8_t* blk = act_block(dst.data[d], dst.groups, tok, g + dst.g_off);
    reinterpret_cast<uint32_t*>(blk + (tok & 7) * kActRowBytes)[lane] = 0;
    if (lane == 0) reinterpret_cast<float2*>(blk + kActBlockTok * kActRowBytes)[tok & 7] = make_float2(0.f, 0.f);
  }
}

__device__ __forceinline__ void zero_group_warp(int tok, uint8_t* act, int groups, int g) {
  zero_group_warp(tok, act_dst(act, groups), g);
}

}  // namespace rai
