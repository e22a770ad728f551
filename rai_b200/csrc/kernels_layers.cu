// Per-layer and speculation kernels of the decode step (sm_100a).
//
// Each kernel restates one reference routine's floating-point order:
//   embed_kernel      embed_lookup (rai-infer/src/gemm.rs:1926-1970)
//   rmsnorm_kernel    rms_norm_avx2 / rms_norm_with_residual_avx2
//                     (rai-infer/src/layers.rs:325-376, 433-497)
//   qkv_post_kernel   QkNorm::apply -> rms_norm_heads (layers.rs:201-240,
//                     308-314), RoPETable::apply_avx2 (layers.rs:689-726) and
//                     KVCache::store (rai-infer/src/kv_cache.rs:143-172)
//   attention_kernel  attention_head_avx2 (layers.rs:1266-1380) for every
//                     (query row, head) of attend_batch (layers.rs:1675-1747)
//   swiglu_kernel     silu_mul_avx2 (layers.rs:850-883)
//   argmax_kernel     sampler::argmax (rai-infer/src/sampler.rs:201-208)
//   ngram_kernel      find_ngram_draft (rai-infer/src/lookup.rs:131-171)
//   accept_kernel     the greedy limit of LookupDecoder::step's acceptance
//                     loop and KV truncate (lookup.rs:359-411)
#include <cuda_runtime.h>

#include "common.cuh"
#include "layers.h"

namespace rai {

// ---------------------------------------------------------------------------
__global__ void embed_kernel(const uint32_t* __restrict__ ids, const int* m_dev, int M,
                             const uint8_t* __restrict__ codes, const uint8_t* __restrict__ params,
                             int vocab, int hidden, int gs, float embed_scale, float* __restrict__ out,
                             uint32_t* err) {
  int b = blockIdx.x;
  int mact = m_dev ? *m_dev : M;
  if (b >= mact) return;
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
  int mact = m_dev ? *m_dev : M;
  if (b >= mact) return;
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
    for (int c = 0; c < chunks16; ++c) {
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
// Sequential scalar RMS over `len` values at x (in place): rms_norm_heads.
__device__ void rms_inplace_seq(float* x, int len, const float* w, float eps, float* inv_out) {
  float ss = 0.f;
  for (int i = 0; i < len; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
  *inv_out = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)len), eps)));
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
// layer's cache at position pos + b. qkv row layout [q | k | v].
__global__ void qkv_post_kernel(float* __restrict__ qkv, int ld, float* __restrict__ q_out, int nh,
                                int nkv, int hd, const float* __restrict__ qn, const float* __restrict__ kn,
                                int qk_mode, float eps, const float* __restrict__ rope_cos,
                                const float* __restrict__ rope_sin, float* __restrict__ kc,
                                float* __restrict__ vc, int max_ctx, const int* pos_dev, int pos0,
                                const int* m_dev, int M) {
  extern __shared__ float srow[];  // q | k
  __shared__ float s_inv[2];
  int b = blockIdx.x;
  int mact = m_dev ? *m_dev : M;
  if (b >= mact) return;
  int pos = (pos_dev ? *pos_dev : pos0) + b;
  int qd = nh * hd, kvd = nkv * hd, half = hd / 2, chunked = (half / 8) * 8;
  float* row = qkv + (size_t)b * ld;
  for (int i = threadIdx.x; i < qd + kvd; i += blockDim.x) srow[i] = row[i];
  __syncthreads();
  float* sq = srow;
  float* sk = srow + qd;
  if (qk_mode == 2) {  // full-width: one RMS over the whole projection
    if (threadIdx.x == 0) rms_inplace_seq(sq, qd, qn, eps, &s_inv[0]);
    if (threadIdx.x == 32) rms_inplace_seq(sk, kvd, kn, eps, &s_inv[1]);
    __syncthreads();
    for (int i = threadIdx.x; i < qd; i += blockDim.x) sq[i] = __fmul_rn(__fmul_rn(sq[i], s_inv[0]), qn[i]);
    for (int i = threadIdx.x; i < kvd; i += blockDim.x) sk[i] = __fmul_rn(__fmul_rn(sk[i], s_inv[1]), kn[i]);
    __syncthreads();
  } else if (qk_mode == 1) {  // per head, weight of head_dim shared by heads
    for (int h = threadIdx.x; h < nh + nkv; h += blockDim.x) {
      float* hp = h < nh ? sq + h * hd : sk + (h - nh) * hd;
      const float* wv = h < nh ? qn : kn;
      float inv;
      rms_inplace_seq(hp, hd, wv, eps, &inv);
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
  for (int i = threadIdx.x; i < kvd; i += blockDim.x) {
    int h = i / hd, d = i % hd;
    size_t o = ((size_t)h * max_ctx + pos) * hd + d;
    kc[o] = sk[i];
    vc[o] = vrow[i];
  }
}

// ---------------------------------------------------------------------------
// Exact attention: CTA (kv head, query row). Scores for every cached
// position (8-lane FMA dot + tree, times scale), max, Schraudolph exp for
// the first (n/8)*8 scores and libm-accurate exp for the tail, 8-lane
// ordered sum, normalise, then out[d] = fma(p_t, v_t[d], out[d]) in
// position order. V is streamed through a double-buffered smem tile.
template <int HD>
__global__ void __launch_bounds__(256) attention_kernel(const float* __restrict__ q, float* __restrict__ out,
                                                        const float* __restrict__ kc, const float* __restrict__ vc,
                                                        int nh, int nkv, int max_ctx, const int* pos_dev, int pos0,
                                                        const int* m_dev, int M, float scale, float softcap,
                                                        int n_alloc, ExpfTable et) {
  constexpr int VT = 32;  // positions per V tile
  extern __shared__ __align__(16) float sm[];
  const int hpk = nh / nkv;
  float* sq = sm;                          // hpk * HD
  float* sc = sq + hpk * HD;               // hpk * n_alloc
  float* vt = sc + (size_t)hpk * n_alloc;  // 2 * VT * HD
  __shared__ float red[8][8];
  __shared__ float lane_part[8][8];
  __shared__ float s_max[8], s_inv[8];

  const int kvh = blockIdx.x, b = blockIdx.y;
  const int mact = m_dev ? *m_dev : M;
  if (b >= mact) return;
  const int pos = (pos_dev ? *pos_dev : pos0) + b;
  const int n = pos + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = nh * HD;
  const float* kbase = kc + (size_t)kvh * max_ctx * HD;
  const float* vbase = vc + (size_t)kvh * max_ctx * HD;

  for (int i = tid; i < hpk * HD; i += blockDim.x) sq[i] = q[(size_t)b * qd + (size_t)kvh * hpk * HD + i];
  __syncthreads();

  // Phase A: scores.
  float tmax[8];
  for (int h = 0; h < 8; ++h) tmax[h] = -INFINITY;
  for (int t = tid; t < n; t += blockDim.x) {
    float kr[HD];
    const float4* kp = reinterpret_cast<const float4*>(kbase + (size_t)t * HD);
#pragma unroll
    for (int i = 0; i < HD / 4; ++i) {
      float4 v = __ldg(kp + i);
      kr[4 * i] = v.x; kr[4 * i + 1] = v.y; kr[4 * i + 2] = v.z; kr[4 * i + 3] = v.w;
    }
    for (int h = 0; h < hpk; ++h) {
      const float* qh = sq + h * HD;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int cc = 0; cc < HD / 8; ++cc)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __fmaf_rn(qh[8 * cc + j], kr[8 * cc + j], acc[j]);
      float sv = __fmul_rn(hsum8(acc), scale);
      if (softcap > 0.f) sv = __fmul_rn(softcap, tanhf(__fdiv_rn(sv, softcap)));
      sc[(size_t)h * n_alloc + t] = sv;
      if (h < 8 && sv > tmax[h]) tmax[h] = sv;
    }
  }
  // Block max per head (hpk <= 8).
  for (int h = 0; h < hpk; ++h) {
    float m = tmax[h];
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[h][warp] = m;
  }
  __syncthreads();
  if (tid < hpk) {
    float m = red[tid][0];
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[tid][w]);
    s_max[tid] = m;
  }
  __syncthreads();
  // Phase B: exponentials.
  const int n8 = (n / 8) * 8;
  for (int idx = tid; idx < hpk * n; idx += blockDim.x) {
    int h = idx / n, t = idx % n;
    float* p = sc + (size_t)h * n_alloc + t;
    float x = __fsub_rn(*p, s_max[h]);
    *p = t < n8 ? schraudolph(x) : expf_host(x, et);
  }
  __syncthreads();
  if (tid < hpk * 8) {
    int h = tid >> 3, j = tid & 7;
    const float* p = sc + (size_t)h * n_alloc;
    float acc = 0.f;
    for (int i = 0; i < n8 / 8; ++i) acc = __fadd_rn(acc, p[8 * i + j]);
    lane_part[h][j] = acc;
  }
  __syncthreads();
  if (tid < hpk) {
    const float* p = sc + (size_t)tid * n_alloc;
    float sum = hsum8(lane_part[tid]);
    for (int t = n8; t < n; ++t) sum = __fadd_rn(sum, p[t]);
    s_inv[tid] = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  for (int idx = tid; idx < hpk * n; idx += blockDim.x) {
    int h = idx / n, t = idx % n;
    float* p = sc + (size_t)h * n_alloc + t;
    *p = __fmul_rn(*p, s_inv[h]);
  }
  // Phase C: V accumulation, chains (h, d) in position order.
  constexpr int kMaxChains = 4;
  float acc[kMaxChains];
  int ch_h[kMaxChains], ch_d[kMaxChains];
  const int chains = hpk * HD;
#pragma unroll
  for (int k = 0; k < kMaxChains; ++k) {
    int idx = tid + k * 256;
    acc[k] = 0.f;
    ch_h[k] = idx < chains ? idx / HD : 0;
    ch_d[k] = idx % HD;
  }
  const int ntiles = (n + VT - 1) / VT;
  auto load_tile = [&](int tile, int buf) {
    int t0 = tile * VT;
    int cnt = min(VT, n - t0) * HD / 4;
    const float4* src = reinterpret_cast<const float4*>(vbase + (size_t)t0 * HD);
    float4* dst = reinterpret_cast<float4*>(vt + (size_t)buf * VT * HD);
    for (int i = tid; i < cnt; i += blockDim.x) {
      uint32_t d = smem_u32(dst + i);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src + i) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_tile(0, 0);
  for (int tile = 0; tile < ntiles; ++tile) {
    if (tile + 1 < ntiles) {
      load_tile(tile + 1, (tile + 1) & 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const float* vb = vt + (size_t)(tile & 1) * VT * HD;
    const int t0 = tile * VT, cnt = min(VT, n - t0);
#pragma unroll
    for (int k = 0; k < kMaxChains; ++k) {
      if (tid + k * 256 >= chains) break;
      const float* prow = sc + (size_t)ch_h[k] * n_alloc + t0;
      float a = acc[k];
      for (int t = 0; t < cnt; ++t) a = __fmaf_rn(prow[t], vb[t * HD + ch_d[k]], a);
      acc[k] = a;
    }
    __syncthreads();
  }
#pragma unroll
  for (int k = 0; k < kMaxChains; ++k) {
    int idx = tid + k * 256;
    if (idx < chains)
      out[(size_t)b * qd + (size_t)(kvh * hpk + ch_h[k]) * HD + ch_d[k]] = acc[k];
  }
}

// ---------------------------------------------------------------------------
// act[b][i] = silu(gate) * up with gate/up rows [gate | up] of width 2*ff.
__global__ void swiglu_kernel(const float* __restrict__ gu, int ff, float* __restrict__ act,
                              const int* m_dev, int M, ExpfTable et) {
  int b = blockIdx.y;
  int mact = m_dev ? *m_dev : M;
  if (b >= mact) return;
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
  int mact = m_dev ? *m_dev : M;
  if (b >= mact) return;
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
// Draft search. One CTA: for n from hi down to lo, the largest start s with
// ctx[s..s+n] == suffix (s <= len-n-1) wins; draft = ctx[s+n .. s+n+dl).
__global__ void ngram_kernel(const uint32_t* __restrict__ ctx, StepState* st, int max_draft,
                             int max_ngram, int min_ngram, int max_ctx) {
  __shared__ int best;
  const int len = st->ctx_len, pos = st->pos;
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
    const uint32_t last = ctx[len - 1];
    st->tokens[0] = last;
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
    for (int r = 0; r < kMaxRows; ++r) st->amax[r] = 0ull;
  }
}

// Greedy acceptance: accept d_i while argmax_i == d_i; the first mismatch is
// replaced by argmax_i; if all are accepted the bonus is argmax_k. Then the
// KV watermark becomes pos + produced.
__global__ void accept_kernel(StepState* st, int* filled, int num_layers) {
  if (threadIdx.x != 0) return;
  const int dl = st->drafted;
  int produced = 0, accepted = 0;
  if (dl == 0) {
    st->out[produced++] = (uint32_t)(st->amax[0] & 0xFFFFFFFFull);
  } else {
    for (int i = 0; i < dl; ++i) {
      uint32_t target = (uint32_t)(st->amax[i] & 0xFFFFFFFFull);
      st->out[produced++] = target;
      if (target != st->tokens[1 + i]) break;
      ++accepted;
    }
    if (accepted == dl) st->out[produced++] = (uint32_t)(st->amax[dl] & 0xFFFFFFFFull);
  }
  st->accepted = accepted;
  st->produced = produced;
  // Stores reached pos + n_rows; truncate(pos + produced) leaves exactly this.
  for (int l = 0; l < num_layers; ++l) filled[l] = st->pos + produced;
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
                            const float* rope_sin, float* kc, float* vc, int max_ctx, const int* pos_dev,
                            int pos0, const int* m_dev, int M, cudaStream_t s) {
  size_t smem = (size_t)(nh + nkv) * hd * sizeof(float);
  qkv_post_kernel<<<M, 256, smem, s>>>(qkv, ld, q_out, nh, nkv, hd, qn, kn, qk_mode, eps, rope_cos, rope_sin,
                                       kc, vc, max_ctx, pos_dev, pos0, m_dev, M);
  return cudaGetLastError();
}

// n_alloc must be a multiple of 4 so the V tile behind the scores is 16-byte
// aligned for cp.async.
size_t attention_smem_bytes(int hd, int hpk, int n_alloc) {
  return ((size_t)hpk * hd + (size_t)hpk * n_alloc + 2 * 32 * (size_t)hd) * sizeof(float);
}

cudaError_t launch_attention(const float* q, float* out, const float* kc, const float* vc, int nh, int nkv,
                             int hd, int max_ctx, const int* pos_dev, int pos0, const int* m_dev, int M,
                             float scale, float softcap, int n_alloc, const ExpfTable& et, cudaStream_t s) {
  int hpk = nh / nkv;
  size_t smem = attention_smem_bytes(hd, hpk, n_alloc);
  dim3 grid(nkv, M);
  if (smem > kAttnMaxSmem) return cudaErrorInvalidValue;
#define RAI_ATTN(HDV)                                                                                  \
  case HDV:                                                                                            \
    attention_kernel<HDV><<<grid, 256, smem, s>>>(q, out, kc, vc, nh, nkv, max_ctx, pos_dev, pos0,     \
                                                  m_dev, M, scale, softcap, n_alloc, et);              \
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

cudaError_t init_layer_attributes() {
  const int bytes = (int)kAttnMaxSmem;
  cudaError_t e = cudaFuncSetAttribute(attention_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attention_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
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

cudaError_t launch_ngram(const uint32_t* ctx, StepState* st, int max_draft, int max_ngram, int min_ngram,
                         int max_ctx, cudaStream_t s) {
  ngram_kernel<<<1, 1024, 0, s>>>(ctx, st, max_draft, max_ngram, min_ngram, max_ctx);
  return cudaGetLastError();
}

cudaError_t launch_accept(StepState* st, int* filled, int num_layers, cudaStream_t s) {
  accept_kernel<<<1, 32, 0, s>>>(st, filled, num_layers);
  return cudaGetLastError();
}

}  // namespace rai
