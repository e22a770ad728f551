// Mixture-of-experts MLP block on the device (rai-infer/src/model.rs:208-261,
// route_experts layers.rs:1808-1870), bit for bit:
//   router logit e = sequential f32 sum over i of router[e][i] * x[i],
//     starting from -0.0 (Rust iterator sum), no FMA;
//   softmax: max, expf(v - max) (host libm), sequential sum, v / sum;
//   top-k by repeated strict '>' scans in expert order (the first maximum
//     wins); optional renormalization by the sequential sum of the picks;
//   out = 0; for each pick in order: out += weight * expert_out (mul, add);
//   hidden = residual + out.
// Each (token, pick) pair runs the expert's SwiGLU MLP through the exact
// W4A8 GEMM (per-row arithmetic does not depend on which tokens share a
// launch), grouped by expert: pairs are sorted by expert into segments that
// start at multiples of 8 rows.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "moe.h"
#include "quant.cuh"

namespace rai {

namespace {

__device__ __forceinline__ int active(const int* m_dev, int M) { return m_dev ? *m_dev : M; }

// Router logits: CTA = kRouterTok tokens x ne experts (one thread per expert);
// the tokens' normalized rows sit in shared memory. Each logit is one
// sequential chain over the hidden dimension, so what bounds the kernel is
// feeding it: the router rows stream in chunks of kRouterChunk columns
// through an NS-deep ring of coalesced 16-byte cp.async copies (rows padded
// to kRouterLd floats, so the per-thread 16-byte row reads are conflict
// free), requested before the previous kernel finishes (they are model
// constants).
constexpr int kRouterTok = 4;
constexpr int kRouterChunk = 32;
constexpr int kRouterLd = kRouterChunk + 4;
constexpr int kRouterDeep = 8;
constexpr size_t kRouterSmemMax = 200 * 1024;

template <int NS>
size_t router_smem_bytes(int h, int ne) {
  return ((size_t)kRouterTok * h + (size_t)NS * ne * kRouterLd) * sizeof(float);
}

// One full chunk of one expert's logit chains for NT tokens: the chunk's
// router values and the tokens' inputs are loaded first (16-byte shared
// loads), then each token's chain adds its products in column order.
template <int NT>
__device__ __forceinline__ void router_chunk(const float* __restrict__ rr, const float* __restrict__ sxc, int h,
                                             float (&acc)[kRouterTok]) {
  float4 rv[kRouterChunk / 4], xv[NT][kRouterChunk / 4];
#pragma unroll
  for (int q = 0; q < kRouterChunk / 4; ++q) rv[q] = *reinterpret_cast<const float4*>(rr + 4 * q);
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int q = 0; q < kRouterChunk / 4; ++q) xv[t][q] = *reinterpret_cast<const float4*>(sxc + (size_t)t * h + 4 * q);
#pragma unroll
  for (int q = 0; q < kRouterChunk / 4; ++q)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      acc[t] = __fadd_rn(acc[t], __fmul_rn(rv[q].x, xv[t][q].x));
      acc[t] = __fadd_rn(acc[t], __fmul_rn(rv[q].y, xv[t][q].y));
      acc[t] = __fadd_rn(acc[t], __fmul_rn(rv[q].z, xv[t][q].z));
      acc[t] = __fadd_rn(acc[t], __fmul_rn(rv[q].w, xv[t][q].w));
    }
}

template <int NS>
__global__ void __launch_bounds__(kMaxMoeExperts) router_kernel(const float* __restrict__ x, const float* __restrict__ router,
                                                         int h, int ne, const int* m_dev, int M,
                                                         float* __restrict__ logits) {
  extern __shared__ __align__(16) float sm[];
  float* sx = sm;                               // [kRouterTok][h]
  float* sr = sm + (size_t)kRouterTok * h;      // [NS][ne][kRouterLd]
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int nch = (h + kRouterChunk - 1) / kRouterChunk;
  auto load = [&](int c) {
    if (c < nch) {
      const int c0 = c * kRouterChunk, g4 = min(kRouterChunk, h - c0) / 4;
      float* dst = sr + (size_t)(c % NS) * ne * kRouterLd;
      if (g4 == kRouterChunk / 4) {
        constexpr int kG = kRouterChunk / 4;  // whole chunk: no division
        for (int i = tid; i < ne * kG; i += nthr) {
          const int e = i / kG, q = i % kG;
          cp_async16(dst + e * kRouterLd + 4 * q, router + (size_t)e * h + c0 + 4 * q);
        }
      } else {
        for (int i = tid; i < ne * g4; i += nthr) {
          const int e = i / g4, q = i - e * g4;
          cp_async16(dst + e * kRouterLd + 4 * q, router + (size_t)e * h + c0 + 4 * q);
        }
      }
    }
    cp_async_commit();
  };
  for (int c = 0; c < NS - 1; ++c) load(c);
  pdl_wait_prior();
  pdl_launch_dependents();
  const int b0 = blockIdx.x * kRouterTok;
  const int mact = active(m_dev, M);
  if (b0 >= mact) {
    cp_async_wait<0>();  // no copy outlives the CTA
    return;
  }
  const int nt = min(kRouterTok, mact - b0);
  stage_f32(sx, x + (size_t)b0 * h, nt * h, tid, nthr);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const int e = tid;
  float acc[kRouterTok];
#pragma unroll
  for (int t = 0; t < kRouterTok; ++t) acc[t] = -0.0f;
  for (int c = 0; c < nch; ++c) {
    load(c + NS - 1);
    cp_async_wait<NS - 1>();  // chunk c has landed (this thread's copies)
    __syncthreads();          // ... and every thread's
    const int c0 = c * kRouterChunk, cw = min(kRouterChunk, h - c0);
    const float* rr = sr + (size_t)(c % NS) * ne * kRouterLd + e * kRouterLd;
    if (e < ne && cw == kRouterChunk) {
      switch (nt) {
        case 1: router_chunk<1>(rr, sx + c0, h, acc); break;
        case 2: router_chunk<2>(rr, sx + c0, h, acc); break;
        case 3: router_chunk<3>(rr, sx + c0, h, acc); break;
        default: router_chunk<4>(rr, sx + c0, h, acc); break;
      }
    } else if (e < ne) {
      for (int i = 0; i < cw; i += 4) {
        const float4 rv = *reinterpret_cast<const float4*>(rr + i);
        const float r4[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int t = 0; t < kRouterTok; ++t) {
          if (t < nt) {
#pragma unroll
            for (int u = 0; u < 4; ++u) acc[t] = __fadd_rn(acc[t], __fmul_rn(r4[u], sx[t * h + c0 + i + u]));
          }
        }
      }
    }
    __syncthreads();  // stage c % NS is refilled by the next iteration
  }
  if (e < ne) {
#pragma unroll
    for (int t = 0; t < kRouterTok; ++t)
      if (t < nt) logits[(size_t)(b0 + t) * ne + e] = acc[t];
  }
}

// Softmax, top-k and optional renormalization: one warp per token. The max,
// the exps and the divisions run across the lanes (each element's value does
// not depend on the order); the sum runs in expert order on lane 0; each
// top-k scan takes the largest not yet taken probability, the lowest expert
// index among equals (a strict '>' scan in expert order).
constexpr int kRouteWarps = 4;

__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(float* __restrict__ logits, int ne, int k,
                                                                 int norm_topk, const int* m_dev, int M,
                                                                 int* __restrict__ experts,
                                                                 float* __restrict__ weights, ExpfTable et) {
  __shared__ float sv[kRouteWarps][kMaxMoeExperts];
  pdl_wait_prior();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * kRouteWarps + warp;
  if (b >= active(m_dev, M)) return;
  float* p = logits + (size_t)b * ne;
  float* v = sv[warp];
  float mx = -INFINITY;
  for (int e = lane; e < ne; e += 32) mx = fmaxf(mx, p[e]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  for (int e = lane; e < ne; e += 32) v[e] = expf_host(__fsub_rn(p[e], mx), et);
  __syncwarp();
  float sum = 0.0f;
  if (lane == 0)
    for (int e = 0; e < ne; ++e) sum = __fadd_rn(sum, v[e]);
  sum = __shfl_sync(0xffffffffu, sum, 0);
  for (int e = lane; e < ne; e += 32) {
    const float q = __fdiv_rn(v[e], sum);
    v[e] = q;
    p[e] = q;
  }
  __syncwarp();
  uint32_t taken = 0u;  // bit j: expert lane + 32 j (ne <= 256)
  int count = 0;
  for (int s = 0; s < k; ++s) {
    float bv = -INFINITY;
    int best = -1;
    for (int j = 0, e = lane; e < ne; ++j, e += 32)
      if (!(taken >> j & 1u) && v[e] > bv) {
        bv = v[e];
        best = e;
      }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best, o);
      if (oi >= 0 && (best < 0 || ov > bv || (ov == bv && oi < best))) {
        bv = ov;
        best = oi;
      }
    }
    if (best < 0) break;
    if ((best & 31) == lane) taken |= 1u << (best >> 5);
    if (lane == 0) {
      experts[(size_t)b * k + count] = best;
      weights[(size_t)b * k + count] = bv;
    }
    ++count;
  }
  if (lane == 0) {
    for (int s = count; s < k; ++s) {
      experts[(size_t)b * k + s] = -1;
      weights[(size_t)b * k + s] = 0.f;
    }
    if (norm_topk) {
      float total = -0.0f;
      for (int s = 0; s < count; ++s) total = __fadd_rn(total, weights[(size_t)b * k + s]);
      if (total > 0.0f)
        for (int s = 0; s < count; ++s) weights[(size_t)b * k + s] = __fdiv_rn(weights[(size_t)b * k + s], total);
    }
  }
}

// Sort the (token, pick) pairs by expert: counts, segment offsets (each
// rounded up to a multiple of 8 rows), then every pair's row. Within an
// expert's segment pairs keep their index order (a stable counting sort:
// warp match masks, per-warp counts, prefix over warps), so every rank of an
// expert-parallel group puts each pair on the same row. One CTA.
__global__ void __launch_bounds__(1024) moe_sort_kernel(const int* __restrict__ experts, int k, int ne,
                                                        const int* m_dev, int M, int* __restrict__ cnt,
                                                        int* __restrict__ off, int* __restrict__ row_of_pair,
                                                        int* __restrict__ pair_of_row, int* __restrict__ n_rows,
                                                        int rows_cap) {
  __shared__ int scnt[kMaxMoeExperts], soff[kMaxMoeExperts + 1], sfill[kMaxMoeExperts];
  __shared__ int wcnt[32][kMaxMoeExperts];  // per-warp counts, then per-warp starts
  pdl_wait_prior();
  pdl_launch_dependents();
  const int np = active(m_dev, M) * k;
  for (int e = threadIdx.x; e < ne; e += blockDim.x) {
    scnt[e] = 0;
    sfill[e] = 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < np; i += blockDim.x) {
    const int e = experts[i];
    if (e >= 0) atomicAdd(&scnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0;
    for (int e = 0; e < ne; ++e) {
      soff[e] = o;
      o += (scnt[e] + 7) & ~7;
    }
    soff[ne] = o;
    *n_rows = o;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < ne; e += blockDim.x) {
    cnt[e] = scnt[e];
    off[e] = soff[e];
  }
  // Padding rows between segments map to no pair.
  for (int r = threadIdx.x; r < soff[ne] && r < rows_cap; r += blockDim.x) pair_of_row[r] = -1;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int base = 0; base < np; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int e = i < np ? experts[i] : -1;
    for (int t = threadIdx.x; t < nw * ne; t += blockDim.x) wcnt[t / ne][t % ne] = 0;
    __syncthreads();
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int below = __popc(same & ((1u << lane) - 1u));  // same-expert pairs earlier in this warp
    if (e >= 0 && below == 0) wcnt[warp][e] = __popc(same);
    __syncthreads();
    for (int x = threadIdx.x; x < ne; x += blockDim.x) {
      int run = sfill[x];
      for (int w = 0; w < nw; ++w) {
        const int c = wcnt[w][x];
        wcnt[w][x] = run;
        run += c;
      }
      sfill[x] = run;
    }
    __syncthreads();
    if (i < np) {
      if (e < 0) {
        row_of_pair[i] = -1;
      } else {
        const int r = soff[e] + wcnt[warp][e] + below;
        row_of_pair[i] = r;
        pair_of_row[r] = i;
      }
    }
    __syncthreads();
  }
}

// Quantize the normalized rows of the pairs into expert-sorted activation
// rows (one warp per (row, group)); padding rows are zero.
__global__ void moe_gather_quant_kernel(const float* __restrict__ x, int h, int k, const int* __restrict__ pair_of_row,
                                        const int* __restrict__ n_rows, int gs, uint8_t* __restrict__ act,
                                        int tok_alloc) {
  __shared__ __align__(16) float sx[8][128];
  __shared__ uint32_t sqw[8][32];
  pdl_wait_prior();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x;
  const int r = blockIdx.y * 8 + warp;
  if (r >= *n_rows || r >= tok_alloc) return;
  const int groups = gridDim.x;
  const int pair = pair_of_row[r];
  if (pair < 0) {
    zero_group_warp(r, act, groups, g);
    return;
  }
  const float* xr = x + (size_t)(pair / k) * h + (size_t)g * gs;
  const int len = min(gs, h - g * gs);
  stage_f32(sx[warp], xr, len, lane, 32);
  cp_async_wait<0>();
  __syncwarp();
  quant_group_warp(sx[warp], len, 4, r, act, groups, g, sqw[warp]);
}

// out = residual + sum over picks (in order) of weight * expert_out.
__global__ void moe_combine_kernel(const float* __restrict__ eo, const int* __restrict__ row_of_pair,
                                   const float* __restrict__ weights, int k, int h, const float* __restrict__ residual,
                                   float* __restrict__ out, const int* m_dev, int M, TpLink tp, int slot,
                                   uint32_t* err) {
  pdl_wait_prior();
  pdl_launch_dependents();
  // Expert parallelism: eo holds every rank's experts' rows once exchange
  // `slot` completes.
  if (slot >= 0 && !tp_exchange(tp, slot, 0, err)) return;
  const int b = blockIdx.y;
  if (b >= active(m_dev, M)) return;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= h) return;
  // The picks' expert outputs are loaded before the ordered adds.
  constexpr int kBatch = 8;
  float acc = 0.0f;
  for (int s0 = 0; s0 < k; s0 += kBatch) {
    float wv[kBatch], ev[kBatch];
    bool use[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int s = s0 + u;
      const int r = s < k ? row_of_pair[(size_t)b * k + s] : -1;
      use[u] = r >= 0;
      wv[u] = use[u] ? weights[(size_t)b * k + s] : 0.f;
      ev[u] = use[u] ? eo[(size_t)r * h + i] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (use[u]) acc = __fadd_rn(acc, __fmul_rn(wv[u], ev[u]));
  }
  out[(size_t)b * h + i] = __fadd_rn(residual[(size_t)b * h + i], acc);
}

}  // namespace

cudaError_t moe_route(const float* x, const float* router, int h, int ne, int k, bool norm_topk, const int* m_dev,
                      int M, const ExpfTable& et, const MoeBuffers& mb, cudaStream_t s) {
  if (ne < 2 || ne > kMaxMoeExperts || k < 1 || k > ne || h % 4) return cudaErrorInvalidValue;
  // The deep ring for up to 64 experts, two stages beyond.
  const dim3 rg((unsigned)ceil_div(M, kRouterTok)), rb((unsigned)ne);
  cudaError_t re;
  if (ne <= 64) {
    if (router_smem_bytes<kRouterDeep>(h, ne) > kRouterSmemMax) return cudaErrorInvalidValue;
    re = launch_pdl(router_kernel<kRouterDeep>, rg, rb, router_smem_bytes<kRouterDeep>(h, ne), s, x, router, h, ne,
                    m_dev, M, mb.logits);
  } else {
    if (router_smem_bytes<2>(h, ne) > kRouterSmemMax) return cudaErrorInvalidValue;
    re = launch_pdl(router_kernel<2>, rg, rb, router_smem_bytes<2>(h, ne), s, x, router, h, ne, m_dev, M,
                    mb.logits);
  }
  if (re) return re;
  if (cudaError_t e = launch_pdl(route_kernel, dim3((unsigned)ceil_div(M, kRouteWarps)), dim3(kRouteWarps * 32), 0, s,
                                 mb.logits, ne, k, (int)norm_topk, m_dev, M, mb.experts, mb.weights, et))
    return e;
  return launch_pdl(moe_sort_kernel, dim3(1), dim3(1024), 0, s, (const int*)mb.experts, k, ne, m_dev, M, mb.cnt,
                    mb.off, mb.row_of_pair, mb.pair_of_row, mb.n_rows, mb.rows_cap);
}

cudaError_t moe_gather_quant(const float* x, int h, int k, int gs, const MoeBuffers& mb, ActBuf act, cudaStream_t s) {
  dim3 grid((unsigned)act.groups, (unsigned)ceil_div(act.tok_alloc, 8));
  return launch_pdl(moe_gather_quant_kernel, grid, dim3(256), 0, s, x, h, k, (const int*)mb.pair_of_row,
                    (const int*)mb.n_rows, gs, act.data, act.tok_alloc);
}

cudaError_t moe_combine(const float* eo, int k, int h, const float* residual, float* out, const int* m_dev, int M,
                        const MoeBuffers& mb, cudaStream_t s, const TpLink* tp, int slot, uint32_t* err) {
  dim3 grid((unsigned)ceil_div(h, 256), (unsigned)M);
  TpLink link;
  if (tp && tp->world > 1 && slot >= 0) link = *tp;
  else slot = -1;
  return launch_pdl(moe_combine_kernel, grid, dim3(256), 0, s, eo, (const int*)mb.row_of_pair,
                    (const float*)mb.weights, k, h, residual, out, m_dev, M, link, slot, err);
}

cudaError_t init_moe_attributes() {
  cudaError_t e = cudaFuncSetAttribute(router_kernel<kRouterDeep>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kRouterSmemMax);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(router_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRouterSmemMax);
  return e;
}

}  // namespace rai
