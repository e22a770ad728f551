// Per-layer and speculation kernels of the decode step (sm_100a).
//
// Each kernel restates one reference routine's floating-point order:
//   embed_kernel        embed_lookup (rai-infer/src/gemm.rs:1926-1970)
//   rmsnorm_kernel      rms_norm_avx2 / rms_norm_with_residual_avx2
//                       (rai-infer/src/layers.rs:325-376, 433-497)
//   qkv_post_kernel     QkNorm::apply -> rms_norm_heads (layers.rs:201-240,
//                       308-314), RoPETable::apply_avx2 (layers.rs:689-726),
//                       KVCache::store (rai-infer/src/kv_cache.rs:143-172)
//   attn_*_kernel       attention_head_avx2 (layers.rs:1266-1380) for every
//                       (row, head) of attend_batch (layers.rs:1675-1747):
//                       scores, then softmax, then the P.V accumulation
//   swiglu_kernel       silu_mul_avx2 (layers.rs:850-883)
//   argmax_kernel       sampler::argmax (rai-infer/src/sampler.rs:201-208)
//   ngram_kernel        find_ngram_draft (rai-infer/src/lookup.rs:131-171)
//   accept_kernel       the greedy limit of LookupDecoder::step's acceptance
//                       loop (lookup.rs:359-411)
#include <cuda_runtime.h>

#include "common.cuh"
#include "layers.h"

namespace rai {

__device__ __forceinline__ int active_rows(const int* m_dev, int M) { return m_dev ? *m_dev : M; }

// ---------------------------------------------------------------------------
__global__ void embed_kernel(const uint32_t* __restrict__ ids, const int* m_dev, int M,
                             const uint8_t* __restrict__ codes, const uint8_t* __restrict__ params,
                             int vocab, int hidden, int gs, float embed_scale, float* __restrict__ out,
                             uint32_t* err) {
  int b = blockIdx.x;
  if (b >= active_rows(m_dev, M)) return;
  uint32_t tok = ids[b];
  if (tok >= (uint32_t)vocab) {
    if (threadIdx.x == 0) atomicOr(err, kErrBadInput);
    return;
  }
  int ng = (hidden + gs - 1) / gs;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    int g = c / gs;
    const uint8_t* p = params + ((size_t)tok * ng + g) * 4;
    float scale = f16_bits_to_f32((uint16_t)(p[0] | (p[1] << 8)));
    float zero = f16_bits_to_f32((uint16_t)(p[2] | (p[3] << 8)));
    float v = __fadd_rn(__fmul_rn((float)codes[(size_t)tok * hidden + c], scale), zero);
    if (embed_scale != 1.0f) v = __fmul_rn(v, embed_scale);
    out[(size_t)b * hidden + c] = v;
  }
}

// ---------------------------------------------------------------------------
// One CTA per row. Sum of squares in two 8-lane FMA accumulators over
// 16-element strides (+ one extra 8-chunk into sq0), lane-wise add, tree,
// scalar tail; inv = 1/sqrt(ss/n + eps); out = (x * inv) * w.
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, int n,
                               float eps, float* __restrict__ out, float* __restrict__ residual,
                               const int* m_dev, int M) {
  extern __shared__ float sx[];
  __shared__ float lanes[16];
  __shared__ float s_inv;
  int b = blockIdx.x;
  if (b >= active_rows(m_dev, M)) return;
  const float* xr = x + (size_t)b * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = xr[i];
    sx[i] = v;
    if (residual) residual[(size_t)b * n + i] = v;
  }
  __syncthreads();
  int chunks8 = n / 8, chunks16 = chunks8 / 2;
  if (threadIdx.x < 16) {
    int j = threadIdx.x & 7, half = threadIdx.x >> 3;
    float acc = 0.f;
    int c = 0;
    // Loads are independent of the chain: fetch eight strides ahead.
    for (; c + 8 <= chunks16; c += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = sx[16 * (c + u) + 8 * half + j];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fmaf_rn(v[u], v[u], acc);
    }
    for (; c < chunks16; ++c) {
      float v = sx[16 * c + 8 * half + j];
      acc = __fmaf_rn(v, v, acc);
    }
    if (half == 0 && 16 * chunks16 + 8 <= n) {
      float v = sx[16 * chunks16 + j];
      acc = __fmaf_rn(v, v, acc);
    }
    lanes[threadIdx.x] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a[8];
    for (int j = 0; j < 8; ++j) a[j] = __fadd_rn(lanes[j], lanes[8 + j]);
    float ss = hsum8(a);
    for (int i = chunks8 * 8; i < n; ++i) ss = __fadd_rn(ss, __fmul_rn(sx[i], sx[i]));
    s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
  }
  __syncthreads();
  float inv = s_inv;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    out[(size_t)b * n + i] = __fmul_rn(__fmul_rn(sx[i], inv), w[i]);
}

// ---------------------------------------------------------------------------
// rms_norm_heads: sequential scalar sum of squares over `len` values.
__device__ float rms_inv_seq(const float* x, int len, float eps) {
  float ss = 0.f;
  for (int i = 0; i < len; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)len), eps)));
}

// RoPE on one head (NeoX half split): FMA form for the first (half/8)*8
// pairs, the scalar non-fused form for the tail.
__device__ __forceinline__ void rope_pair(float* h, int i, int half, int chunked, const float* c,
                                          const float* s) {
  float x0 = h[i], x1 = h[half + i];
  if (i < chunked) {
    h[i] = __fmaf_rn(x0, c[i], -__fmul_rn(x1, s[i]));
    h[half + i] = __fmaf_rn(x1, c[i], __fmul_rn(x0, s[i]));
  } else {
    h[i] = __fsub_rn(__fmul_rn(x0, c[i]), __fmul_rn(x1, s[i]));
    h[half + i] = __fadd_rn(__fmul_rn(x1, c[i]), __fmul_rn(x0, s[i]));
  }
}

// One CTA per active row: QK norm, RoPE on q and k, then store k, v into the
// row's stream cache at the row's position. qkv row layout [q | k | v].
__global__ void qkv_post_kernel(const float* __restrict__ qkv, int ld, float* __restrict__ q_out, int nh,
                                int nkv, int hd, const float* __restrict__ qn, const float* __restrict__ kn,
                                int qk_mode, float eps, const float* __restrict__ rope_cos,
                                const float* __restrict__ rope_sin, const StreamKV* __restrict__ kv, int layer,
                                const RowInfo* __restrict__ rows, const int* m_dev, int M) {
  extern __shared__ float srow[];  // q | k
  __shared__ float s_inv[2];
  int b = blockIdx.x;
  if (b >= active_rows(m_dev, M)) return;
  const RowInfo ri = rows[b];
  const StreamKV sk_ = kv[ri.stream];
  const int pos = ri.pos;
  int qd = nh * hd, kvd = nkv * hd, half = hd / 2, chunked = (half / 8) * 8;
  const float* row = qkv + (size_t)b * ld;
  for (int i = threadIdx.x; i < qd + kvd; i += blockDim.x) srow[i] = row[i];
  __syncthreads();
  float* sq = srow;
  float* sk = srow + qd;
  if (qk_mode == 2) {  // full width: one RMS over the whole projection
    if (threadIdx.x == 0) s_inv[0] = rms_inv_seq(sq, qd, eps);
    if (threadIdx.x == 32) s_inv[1] = rms_inv_seq(sk, kvd, eps);
    __syncthreads();
    for (int i = threadIdx.x; i < qd; i += blockDim.x) sq[i] = __fmul_rn(__fmul_rn(sq[i], s_inv[0]), qn[i]);
    for (int i = threadIdx.x; i < kvd; i += blockDim.x) sk[i] = __fmul_rn(__fmul_rn(sk[i], s_inv[1]), kn[i]);
    __syncthreads();
  } else if (qk_mode == 1) {  // per head, one head_dim weight shared by heads
    for (int h = threadIdx.x; h < nh + nkv; h += blockDim.x) {
      float* hp = h < nh ? sq + h * hd : sk + (h - nh) * hd;
      const float* wv = h < nh ? qn : kn;
      float inv = rms_inv_seq(hp, hd, eps);
      for (int i = 0; i < hd; ++i) hp[i] = __fmul_rn(__fmul_rn(hp[i], inv), wv[i]);
    }
    __syncthreads();
  }
  const float* c = rope_cos + (size_t)pos * half;
  const float* s = rope_sin + (size_t)pos * half;
  for (int idx = threadIdx.x; idx < (nh + nkv) * half; idx += blockDim.x) {
    int h = idx / half, i = idx % half;
    float* hp = h < nh ? sq + h * hd : sk + (h - nh) * hd;
    rope_pair(hp, i, half, chunked, c, s);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < qd; i += blockDim.x) q_out[(size_t)b * qd + i] = sq[i];
  const float* vrow = row + qd + kvd;
  const size_t lbase = (size_t)layer * nkv * sk_.max_ctx * hd;
  for (int i = threadIdx.x; i < kvd; i += blockDim.x) {
    int h = i / hd, d = i % hd;
    size_t o = lbase + ((size_t)h * sk_.max_ctx + pos) * hd + d;
    sk_.k[o] = sk[i];
    sk_.v[o] = vrow[i];
  }
}

// ---------------------------------------------------------------------------
// Attention, step 1: scores. CTA (kv head, row, chunk of kScoreChunk
// positions); thread t owns one cached position, keeps its K row in
// registers and scores it against the group's query heads: 8-lane FMA dot,
// horizontal-sum tree, times scale (then softcap).
template <int HD>
__global__ void __launch_bounds__(kScoreChunk) attn_scores_kernel(
    const float* __restrict__ q, const StreamKV* __restrict__ kv, int layer, const RowInfo* __restrict__ rows,
    const int* m_dev, int M, int nh, int nkv, float scale, float softcap, float* __restrict__ scores,
    float* __restrict__ smax, int n_alloc, int n_chunks) {
  __shared__ float sq[8 * HD];
  __shared__ float red[8][kScoreChunk / 32];
  const int kvh = blockIdx.x, j = blockIdx.y, chunk = blockIdx.z;
  if (j >= active_rows(m_dev, M)) return;
  const RowInfo ri = rows[j];
  const int n = ri.pos + 1;
  const int t0 = chunk * kScoreChunk;
  if (t0 >= n) return;
  const int hpk = nh / nkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < hpk * HD; i += blockDim.x) sq[i] = q[(size_t)j * nh * HD + (size_t)kvh * hpk * HD + i];
  __syncthreads();
  const StreamKV sk_ = kv[ri.stream];
  const int t = t0 + tid;
  // Per-thread maxima stay in registers: every loop over the (at most 8)
  // heads of the group is fully unrolled with a guard.
  float tmax[8];
#pragma unroll
  for (int h = 0; h < 8; ++h) tmax[h] = -INFINITY;
  if (t < n) {
    const float4* kp = reinterpret_cast<const float4*>(
        sk_.k + (((size_t)layer * nkv + kvh) * sk_.max_ctx + t) * HD);
    float kr[HD];
#pragma unroll
    for (int i = 0; i < HD / 4; ++i) {
      float4 v = __ldg(kp + i);
      kr[4 * i] = v.x; kr[4 * i + 1] = v.y; kr[4 * i + 2] = v.z; kr[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      if (h < hpk) {
        const float* qh = sq + h * HD;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int cc = 0; cc < HD / 8; ++cc)
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) acc[jj] = __fmaf_rn(qh[8 * cc + jj], kr[8 * cc + jj], acc[jj]);
        float sv = __fmul_rn(hsum8(acc), scale);
        if (softcap > 0.f) sv = __fmul_rn(softcap, tanhf(__fdiv_rn(sv, softcap)));
        scores[((size_t)j * nh + kvh * hpk + h) * n_alloc + t] = sv;
        tmax[h] = sv;
      }
    }
  }
#pragma unroll
  for (int h = 0; h < 8; ++h) {
    float m = tmax[h];
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[h][warp] = m;
  }
  __syncthreads();
  if (tid < hpk) {
    float m = red[tid][0];
#pragma unroll
    for (int w = 1; w < kScoreChunk / 32; ++w) m = fmaxf(m, red[tid][w]);
    smax[((size_t)j * nh + kvh * hpk + tid) * n_chunks + chunk] = m;
  }
}

// Attention, step 2: softmax of one (row, head). Schraudolph exp for the
// first (n/8)*8 scores, the host-libm expf for the tail; the sum in 8 lanes
// (lane j adds scores 8i + j in order), the tree, then the tail added in
// order; stores exp values in place and 1/sum.
__global__ void __launch_bounds__(256) attn_softmax_kernel(const RowInfo* __restrict__ rows, const int* m_dev,
                                                           int M, int nh, float* __restrict__ scores,
                                                           const float* __restrict__ smax, float* __restrict__ inv,
                                                           int n_alloc, int n_chunks, ExpfTable et) {
  extern __shared__ float se[];
  __shared__ float lanes[8];
  const int j = blockIdx.x, h = blockIdx.y;
  if (j >= active_rows(m_dev, M)) return;
  const int n = rows[j].pos + 1;
  const int nch = (n + kScoreChunk - 1) / kScoreChunk;
  const float* cm = smax + ((size_t)j * nh + h) * n_chunks;
  float m = cm[0];
  for (int c = 1; c < nch; ++c) m = fmaxf(m, cm[c]);
  float* row = scores + ((size_t)j * nh + h) * n_alloc;
  const int n8 = (n / 8) * 8;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    float x = __fsub_rn(row[t], m);
    float e = t < n8 ? schraudolph(x) : expf_host(x, et);
    row[t] = e;
    se[t] = e;
  }
  __syncthreads();
  if (threadIdx.x < 8) {
    const int jj = threadIdx.x, cnt = n8 / 8;
    float acc = 0.f;
    int i = 0;
    for (; i + 8 <= cnt; i += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = se[8 * (i + u) + jj];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, v[u]);
    }
    for (; i < cnt; ++i) acc = __fadd_rn(acc, se[8 * i + jj]);
    lanes[jj] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = hsum8(lanes);
    for (int t = n8; t < n; ++t) sum = __fadd_rn(sum, se[t]);
    inv[(size_t)j * nh + h] = __fdiv_rn(1.0f, sum);
  }
}

// Attention, step 3: out[h][d] = fma(p_t, v_t[d], out) over t in order, with
// p_t = e_t * (1/sum). CTA (kv head, row); one thread per (head, dim) chain;
// V and p tiles staged in shared memory (double-buffered V via cp.async).
template <int HD>
__global__ void __launch_bounds__(1024) attn_pv_kernel(const StreamKV* __restrict__ kv, int layer,
                                                       const RowInfo* __restrict__ rows, const int* m_dev, int M,
                                                       int nh, int nkv, const float* __restrict__ scores,
                                                       const float* __restrict__ inv, int n_alloc,
                                                       float* __restrict__ out) {
  constexpr int VT = 64;
  extern __shared__ __align__(16) float sm[];
  const int hpk = nh / nkv;
  float* vt = sm;                       // [2][VT][HD]
  float* pt = sm + 2 * VT * HD;         // [hpk][VT]
  const int kvh = blockIdx.x, j = blockIdx.y;
  if (j >= active_rows(m_dev, M)) return;
  const RowInfo ri = rows[j];
  const int n = ri.pos + 1;
  const StreamKV sk_ = kv[ri.stream];
  const float* vbase = sk_.v + ((size_t)layer * nkv + kvh) * sk_.max_ctx * HD;
  const int tid = threadIdx.x;
  const int h = tid / HD, d = tid % HD;
  const bool chain = tid < hpk * HD;
  const float* erow0 = scores + ((size_t)j * nh + kvh * hpk) * n_alloc;
  const float* invr = inv + (size_t)j * nh + kvh * hpk;
  const int ntiles = (n + VT - 1) / VT;
  auto load_v = [&](int tile, int buf) {
    int t0 = tile * VT;
    int cnt = min(VT, n - t0) * HD / 4;
    const float4* src = reinterpret_cast<const float4*>(vbase + (size_t)t0 * HD);
    float4* dst = reinterpret_cast<float4*>(vt + (size_t)buf * VT * HD);
    for (int i = tid; i < cnt; i += blockDim.x) {
      uint32_t a = smem_u32(dst + i);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(a), "l"(src + i) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float acc = 0.f;
  load_v(0, 0);
  for (int tile = 0; tile < ntiles; ++tile) {
    const int t0 = tile * VT, cnt = min(VT, n - t0);
    // p tile for this block's heads: p = e * inv (the reference's
    // `*sp *= inv_sum`).
    for (int i = tid; i < hpk * VT; i += blockDim.x) {
      int hh = i / VT, tt = i % VT;
      pt[i] = tt < cnt ? __fmul_rn(erow0[(size_t)hh * n_alloc + t0 + tt], invr[hh]) : 0.f;
    }
    if (tile + 1 < ntiles) {
      load_v(tile + 1, (tile + 1) & 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    if (chain) {
      const float* vb = vt + (size_t)(tile & 1) * VT * HD + d;
      const float* pb = pt + h * VT;
      int t = 0;
      for (; t + 8 <= cnt; t += 8) {
        float pv[8], vv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          pv[u] = pb[t + u];
          vv[u] = vb[(t + u) * HD];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) acc = __fmaf_rn(pv[u], vv[u], acc);
      }
      for (; t < cnt; ++t) acc = __fmaf_rn(pb[t], vb[t * HD], acc);
    }
    __syncthreads();
  }
  if (chain) out[(size_t)j * nh * HD + (size_t)(kvh * hpk + h) * HD + d] = acc;
}

// ---------------------------------------------------------------------------
// act[b][i] = silu(gate) * up with gate/up rows [gate | up] of width 2*ff.
__global__ void swiglu_kernel(const float* __restrict__ gu, int ff, float* __restrict__ act,
                              const int* m_dev, int M, ExpfTable et) {
  int b = blockIdx.y;
  if (b >= active_rows(m_dev, M)) return;
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ff) return;
  float x = gu[(size_t)b * 2 * ff + i], u = gu[(size_t)b * 2 * ff + ff + i];
  float s;
  if (i < (ff / 8) * 8) {
    float e = schraudolph(__fmul_rn(x, -1.0f));
    s = __fdiv_rn(x, __fadd_rn(1.0f, e));
  } else {
    s = __fdiv_rn(x, __fadd_rn(1.0f, expf_host(-x, et)));
  }
  act[(size_t)b * ff + i] = __fmul_rn(s, u);
}

// ---------------------------------------------------------------------------
// Argmax with the reference's total order (NaN -> -inf first) and ties to
// the LAST index: max over (orderable key << 32 | index).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  if (isnan(v)) v = -INFINITY;
  int32_t bits = __float_as_int(v);
  bits ^= (int32_t)(((uint32_t)(bits >> 31)) >> 1);
  uint32_t u = (uint32_t)bits ^ 0x80000000u;
  return ((unsigned long long)u << 32) | idx;
}

__global__ void argmax_kernel(const float* __restrict__ logits, int vocab, const int* m_dev, int M,
                              unsigned long long* __restrict__ best) {
  int b = blockIdx.y;
  if (b >= active_rows(m_dev, M)) return;
  unsigned long long k = 0;
  const float* row = logits + (size_t)b * vocab;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x) {
    unsigned long long c = argmax_key(row[i], (uint32_t)i);
    k = c > k ? c : k;
  }
  for (int o = 16; o; o >>= 1) {
    unsigned long long c = __shfl_xor_sync(0xffffffffu, k, o);
    k = c > k ? c : k;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(best + b, k);
}

// ---------------------------------------------------------------------------
// Draft search, one CTA per stream: for n from hi down to lo, the largest
// start s with ctx[s..s+n] == suffix (s <= len-n-1) wins; draft =
// ctx[s+n .. s+n+dl) with dl = min(max_draft, budget, len - s - n), budget =
// max_ctx - pos - 1.
__global__ void ngram_kernel(const uint32_t* __restrict__ ctx_all, int ctx_cap, StreamStep* st_all,
                             const StreamKV* __restrict__ kv, int max_draft, int max_ngram, int min_ngram) {
  __shared__ int best;
  const int sidx = blockIdx.x;
  StreamStep* st = st_all + sidx;
  const uint32_t* ctx = ctx_all + (size_t)sidx * ctx_cap;
  const int len = st->ctx_len, pos = st->pos, max_ctx = kv[sidx].max_ctx;
  const int budget = max_ctx > pos + 1 ? max_ctx - pos - 1 : 0;
  const int kcap = min(max_draft, budget);
  int found_n = 0, found_s = -1;
  if (kcap > 0 && len >= 2) {
    int hi = min(max_ngram, len - 1), lo = max(min_ngram, 1);
    for (int n = hi; n >= lo; --n) {
      if (threadIdx.x == 0) best = -1;
      __syncthreads();
      const uint32_t* suf = ctx + len - n;
      for (int s = threadIdx.x; s <= len - n - 1; s += blockDim.x) {
        bool eq = true;
        for (int i = 0; i < n && eq; ++i) eq = ctx[s + i] == suf[i];
        if (eq) atomicMax(&best, s);
      }
      __syncthreads();
      int bs = best;
      __syncthreads();
      if (bs >= 0) { found_n = n; found_s = bs; break; }
    }
  }
  if (threadIdx.x == 0) {
    st->tokens[0] = ctx[len - 1];
    if (found_s >= 0) {
      int ds = found_s + found_n;
      int dl = min(kcap, len - ds);
      for (int i = 0; i < dl; ++i) st->tokens[1 + i] = ctx[ds + i];
      st->drafted = dl;
      st->ngram = found_n;
      st->n_rows = dl + 1;
    } else {
      st->drafted = 0;
      st->ngram = 0;
      st->n_rows = 1;
    }
  }
}

// Compact every stream's verify rows into one row set (prefix sum over the
// streams), write row metadata and token ids, zero the argmax slots.
__global__ void plan_kernel(StreamStep* st, int n, RowInfo* rows, uint32_t* ids, int* m_active,
                            unsigned long long* best, int best_len) {
  if (threadIdx.x == 0) {
    int r = 0;
    for (int i = 0; i < n; ++i) {
      st[i].row0 = r;
      r += st[i].n_rows;
    }
    *m_active = r;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < best_len; i += blockDim.x) best[i] = 0ull;
  for (int i = 0; i < n; ++i) {
    const int r0 = st[i].row0, nr = st[i].n_rows, p = st[i].pos;
    for (int b = threadIdx.x; b < nr; b += blockDim.x) {
      rows[r0 + b] = RowInfo{p + b, i};
      ids[r0 + b] = st[i].tokens[b];
    }
  }
}

// Greedy acceptance per stream: accept d_i while argmax_i == d_i; the first
// mismatch is replaced by argmax_i; if all are accepted the bonus is argmax_k.
__global__ void accept_kernel(StreamStep* st_all, const unsigned long long* __restrict__ best) {
  if (threadIdx.x != 0) return;
  StreamStep* st = st_all + blockIdx.x;
  const int dl = st->drafted, r0 = st->row0;
  int produced = 0, accepted = 0;
  for (int i = 0; i < dl; ++i) {
    uint32_t target = (uint32_t)(best[r0 + i] & 0xFFFFFFFFull);
    st->out[produced++] = target;
    if (target != st->tokens[1 + i]) break;
    ++accepted;
  }
  if (accepted == dl) st->out[produced++] = (uint32_t)(best[r0 + dl] & 0xFFFFFFFFull);
  st->accepted = accepted;
  st->produced = produced;
}

// ---------------------------------------------------------------------------
// Host launchers.
cudaError_t launch_embed(const uint32_t* ids, const int* m_dev, int M, const uint8_t* codes,
                         const uint8_t* params, int vocab, int hidden, int gs, float embed_scale,
                         float* out, uint32_t* err, cudaStream_t s) {
  embed_kernel<<<M, 256, 0, s>>>(ids, m_dev, M, codes, params, vocab, hidden, gs, embed_scale, out, err);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const float* x, const float* w, int n, float eps, float* out, float* residual,
                           const int* m_dev, int M, cudaStream_t s) {
  rmsnorm_kernel<<<M, 256, n * sizeof(float), s>>>(x, w, n, eps, out, residual, m_dev, M);
  return cudaGetLastError();
}

cudaError_t launch_qkv_post(float* qkv, int ld, float* q_out, int nh, int nkv, int hd, const float* qn,
                            const float* kn, int qk_mode, float eps, const float* rope_cos,
                            const float* rope_sin, const StreamKV* kv, int layer, const RowInfo* rows,
                            const int* m_dev, int M, cudaStream_t s) {
  size_t smem = (size_t)(nh + nkv) * hd * sizeof(float);
  qkv_post_kernel<<<M, 256, smem, s>>>(qkv, ld, q_out, nh, nkv, hd, qn, kn, qk_mode, eps, rope_cos, rope_sin,
                                       kv, layer, rows, m_dev, M);
  return cudaGetLastError();
}

size_t attention_n_chunks(int n_alloc) { return (size_t)(n_alloc + kScoreChunk - 1) / kScoreChunk; }

static size_t pv_smem_bytes(int hd, int hpk) { return (size_t)(2 * 64 * hd + hpk * 64) * sizeof(float); }

cudaError_t launch_attention(const float* q, float* out, const StreamKV* kv, int layer, const RowInfo* rows,
                             const int* m_dev, int M, int nh, int nkv, int hd, float scale, float softcap,
                             float* scores, float* smax, float* inv, int n_alloc, const ExpfTable& et,
                             cudaStream_t s) {
  const int hpk = nh / nkv;
  const int nch = (int)attention_n_chunks(n_alloc);
  dim3 g1(nkv, M, nch), g2(M, nh), g3(nkv, M);
  const size_t sm2 = (size_t)n_alloc * sizeof(float);
  const size_t sm3 = pv_smem_bytes(hd, hpk);
  const int t3 = (hpk * hd + 31) / 32 * 32;
  if (sm2 > kAttnMaxSmem || sm3 > kAttnMaxSmem || hpk > 8 || t3 > 1024) return cudaErrorInvalidValue;
#define RAI_ATTN(HDV)                                                                                   \
  case HDV:                                                                                             \
    attn_scores_kernel<HDV><<<g1, kScoreChunk, 0, s>>>(q, kv, layer, rows, m_dev, M, nh, nkv, scale,    \
                                                       softcap, scores, smax, n_alloc, nch);            \
    attn_softmax_kernel<<<g2, 256, sm2, s>>>(rows, m_dev, M, nh, scores, smax, inv, n_alloc, nch, et);  \
    attn_pv_kernel<HDV><<<g3, t3, sm3, s>>>(kv, layer, rows, m_dev, M, nh, nkv, scores, inv, n_alloc,   \
                                            out);                                                       \
    break;
  switch (hd) {
    RAI_ATTN(16)
    RAI_ATTN(32)
    RAI_ATTN(64)
    RAI_ATTN(128)
    default:
      return cudaErrorInvalidValue;
  }
#undef RAI_ATTN
  return cudaGetLastError();
}

// Test diagnostics: the score pass alone (raw scores and per-chunk maxima).
cudaError_t launch_attention_scores(const float* q, const StreamKV* kv, int layer, const RowInfo* rows, int M,
                                    int nh, int nkv, int hd, float scale, float* scores, float* smax, int n_alloc,
                                    cudaStream_t s) {
  const int nch = (int)attention_n_chunks(n_alloc);
  dim3 g1(nkv, M, nch);
  switch (hd) {
    case 16: attn_scores_kernel<16><<<g1, kScoreChunk, 0, s>>>(q, kv, layer, rows, nullptr, M, nh, nkv, scale, 0.f, scores, smax, n_alloc, nch); break;
    case 32: attn_scores_kernel<32><<<g1, kScoreChunk, 0, s>>>(q, kv, layer, rows, nullptr, M, nh, nkv, scale, 0.f, scores, smax, n_alloc, nch); break;
    case 64: attn_scores_kernel<64><<<g1, kScoreChunk, 0, s>>>(q, kv, layer, rows, nullptr, M, nh, nkv, scale, 0.f, scores, smax, n_alloc, nch); break;
    case 128: attn_scores_kernel<128><<<g1, kScoreChunk, 0, s>>>(q, kv, layer, rows, nullptr, M, nh, nkv, scale, 0.f, scores, smax, n_alloc, nch); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t init_layer_attributes() {
  const int bytes = (int)kAttnMaxSmem;
  cudaError_t e = cudaFuncSetAttribute(attn_softmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_pv_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_pv_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_pv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_pv_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  return e;
}

cudaError_t launch_swiglu(const float* gu, int ff, float* act, const int* m_dev, int M, const ExpfTable& et,
                          cudaStream_t s) {
  dim3 grid((ff + 255) / 256, M);
  swiglu_kernel<<<grid, 256, 0, s>>>(gu, ff, act, m_dev, M, et);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float* logits, int vocab, const int* m_dev, int M, unsigned long long* best,
                          cudaStream_t s) {
  int blocks = (vocab + 4095) / 4096;
  if (blocks > 64) blocks = 64;
  dim3 grid(blocks, M);
  argmax_kernel<<<grid, 256, 0, s>>>(logits, vocab, m_dev, M, best);
  return cudaGetLastError();
}

cudaError_t launch_ngram(const uint32_t* ctx, int ctx_cap, StreamStep* st, const StreamKV* kv, int n,
                         int max_draft, int max_ngram, int min_ngram, cudaStream_t s) {
  ngram_kernel<<<n, 1024, 0, s>>>(ctx, ctx_cap, st, kv, max_draft, max_ngram, min_ngram);
  return cudaGetLastError();
}

cudaError_t launch_plan(StreamStep* st, int n, RowInfo* rows, uint32_t* ids, int* m_active,
                        unsigned long long* best, int best_len, cudaStream_t s) {
  plan_kernel<<<1, 256, 0, s>>>(st, n, rows, ids, m_active, best, best_len);
  return cudaGetLastError();
}

cudaError_t launch_accept(StreamStep* st, int n, const unsigned long long* best, cudaStream_t s) {
  accept_kernel<<<n, 32, 0, s>>>(st, best);
  return cudaGetLastError();
}

}  // namespace rai
