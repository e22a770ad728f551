// Sampled (temperature > 0) acceptance of a prompt-lookup step on the device:
// the rule of LookupDecoder::step (rai-infer/src/lookup.rs:359-403) with the
// helpers of speculative.rs:414-515 and sampler.rs:47-208.
//
// For draft token d_i of a stream (its verify row i):
//   p = softmax_probabilities(logits_i, t)[d_i]   (value / t, NaN -> -inf,
//       +inf tokens share the mass, all -inf or a bad sum -> uniform);
//   the draft distribution is a point mass at d_i, so accept_prob = min(p, 1);
//   accept if u < accept_prob (u uniform f32);
//   else the correction is drawn from max(0, p_target - onehot(d_i)), i.e.
//   p_target without d_i: u64 = uniform f64 * adj_sum, the first index whose
//   cumulative f64 sum reaches u64 (index V-1 if none), and the step stops.
// If every draft is accepted, the bonus token is sample_token(logits_k, t):
// value * (1/t), the same softmax with the sum inverted once, r uniform f32,
// the first index with r < cumulative sum (argmax if none).
//
// Random numbers: Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel
// random numbers: as easy as 1, 2, 3", SC 2011), keyed by the decoder's
// 64-bit seed, counter = (step, draw). The reference draws from rand 0.8's
// StdRng, whose stream is not reproduced, so parity with the reference is
// distributional; the device sums the softmax in parallel (f32, f64 for the
// cumulative searches) instead of the reference's sequential order.
#include <cuda_runtime.h>

#include "common.cuh"
#include "layers.h"

namespace rai {

namespace {

constexpr int kSampleThreads = 1024;

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k.x += 0x9E3779B9u;
      k.y += 0xBB67AE85u;
    }
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
  }
  return c;
}

// Draw `n` of a step: uniform f32 in [0, 1) with 24 bits, f64 with 53 bits.
__device__ __forceinline__ uint4 draw_bits(const StreamStep& st, uint32_t n) {
  return philox4x32_10(make_uint4(st.rng_step_lo, st.rng_step_hi, n, 0u), make_uint2(st.rng_seed_lo, st.rng_seed_hi));
}
__device__ __forceinline__ float uniform_f32(const StreamStep& st, uint32_t n) {
  return (float)(draw_bits(st, n).x >> 8) * (1.0f / 16777216.0f);
}
__device__ __forceinline__ double uniform_f64(const StreamStep& st, uint32_t n) {
  const uint4 b = draw_bits(st, n);
  const unsigned long long v = (((unsigned long long)b.x << 32) | b.y) >> 11;
  return (double)v * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ float scale_logit(float v, float t, float inv_t, bool mul) {
  const float s = mul ? __fmul_rn(v, inv_t) : __fdiv_rn(v, t);
  return isnan(s) ? -INFINITY : s;
}

// Block reductions over kSampleThreads threads (red: 32 slots of shared memory).
template <class T, class Op>
__device__ T block_reduce(T v, Op op, T* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) v = op(v, red[w]);
  return v;
}

// Softmax of one row at temperature t: +inf count, max and the sum of
// exp(s - max) over the finite case; p(j) afterwards.
struct RowSoftmax {
  float t, inv_t;
  bool mul;  // sample_token scales by 1/t, softmax_probabilities divides by t
  int V;
  int pinf;
  float mx, sum, inv_sum;
  bool uniform;

  __device__ float p(const float* row, int j) const {
    if (uniform) return 1.0f / (float)V;
    const float s = scale_logit(row[j], t, inv_t, mul);
    if (pinf > 0) return s == INFINITY ? 1.0f / (float)pinf : 0.0f;
    const float e = expf(__fsub_rn(s, mx));
    return mul ? __fmul_rn(e, inv_sum) : __fdiv_rn(e, sum);
  }
};

__device__ RowSoftmax row_softmax(const float* row, int V, float t, bool mul, float* redf, int* redi) {
  RowSoftmax r;
  r.t = t;
  r.inv_t = __fdiv_rn(1.0f, t);
  r.mul = mul;
  r.V = V;
  int cnt = 0;
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    const float s = scale_logit(row[j], t, r.inv_t, mul);
    cnt += s == INFINITY;
    mx = fmaxf(mx, s);
  }
  r.pinf = block_reduce(cnt, [](int a, int b) { return a + b; }, redi);
  r.mx = block_reduce(mx, [](float a, float b) { return fmaxf(a, b); }, redf);
  r.sum = 0.f;
  r.uniform = false;
  if (r.pinf == 0) {
    if (r.mx == -INFINITY) {
      r.uniform = true;
    } else {
      float sum = 0.f;
      for (int j = threadIdx.x; j < V; j += blockDim.x)
        sum = __fadd_rn(sum, expf(__fsub_rn(scale_logit(row[j], t, r.inv_t, mul), r.mx)));
      r.sum = block_reduce(sum, [](float a, float b) { return __fadd_rn(a, b); }, redf);
      if (!isfinite(r.sum) || r.sum <= 0.f) r.uniform = true;
    }
  }
  r.inv_sum = r.uniform ? 0.f : __fdiv_rn(1.0f, r.sum);
  return r;
}

// Inverse-CDF search over weights q(j): the first j whose cumulative f64
// sum reaches `target` (strict: exceeds it). Each thread owns a contiguous
// chunk; chunk sums are scanned across the block. Returns -1 when no index
// qualifies (rounding at the end of the range).
template <class Q>
__device__ int cdf_search(int V, Q q, double target, bool strict, double* redd, int* res) {
  const int chunk = (V + blockDim.x - 1) / blockDim.x;
  const int j0 = min(V, (int)threadIdx.x * chunk), j1 = min(V, j0 + chunk);
  double mine = 0.0;
  for (int j = j0; j < j1; ++j) mine += (double)q(j);
  // Exclusive scan of the chunk sums in thread order.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double incl = mine;
  for (int o = 1; o < 32; o <<= 1) {
    const double u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  __syncthreads();
  if (lane == 31) redd[warp] = incl;
  if (threadIdx.x == 0) *res = 0x7fffffff;
  __syncthreads();
  double base = 0.0;
  for (int w = 0; w < warp; ++w) base += redd[w];
  double cum = base + incl - mine;  // sum of every earlier chunk
  if (j0 < j1 && (strict ? base + incl > target : base + incl >= target) && !(strict ? cum > target : cum >= target)) {
    for (int j = j0; j < j1; ++j) {
      cum += (double)q(j);
      if (strict ? cum > target : cum >= target) {
        atomicMin(res, j);  // the first chunk that qualifies holds the answer
        break;
      }
    }
  }
  __syncthreads();
  const int found = *res;
  return found == 0x7fffffff ? -1 : found;
}

// draft_logits (optional): the draft model's logits of each draft row
// (speculative decoding, speculative.rs:300-355); without them the draft
// distribution is the point mass of prompt lookup (lookup.rs:362-366).
__global__ void __launch_bounds__(kSampleThreads) sample_accept_kernel(StreamStep* st_all,
                                                                       const float* __restrict__ logits, int V,
                                                                       float t, const float* __restrict__ draft_logits) {
  pdl_wait_prior();
  pdl_launch_dependents();
  __shared__ float redf[32];
  __shared__ int redi[32];
  __shared__ double redd[32];
  __shared__ int res;
  StreamStep* st = st_all + blockIdx.x;
  const int dl = st->drafted, r0 = st->row0;
  uint32_t draw = 0;
  int produced = 0, accepted = 0;
  for (int i = 0; i < dl; ++i) {
    const float* row = logits + (size_t)(r0 + i) * V;
    const int d = (int)st->tokens[1 + i];
    const RowSoftmax sm = row_softmax(row, V, t, false, redf, redi);
    const float p_target = sm.p(row, d);
    const float* drow = draft_logits ? draft_logits + (size_t)i * V : nullptr;
    RowSoftmax dsm;
    float p_draft = 1.0f;  // point mass at d
    if (drow) {
      dsm = row_softmax(drow, V, t, false, redf, redi);
      p_draft = dsm.p(drow, d);
    }
    const float accept_prob = p_draft > 0.f ? fminf(__fdiv_rn(p_target, p_draft), 1.0f) : (p_target > 0.f ? 1.0f : 0.0f);
    const float u = uniform_f32(*st, draw++);
    if (u < accept_prob) {
      if (threadIdx.x == 0) st->out[produced] = (uint32_t)d;
      ++produced;
      ++accepted;
      continue;
    }
    // Correction from max(0, p_target - p_draft) (sample_correction).
    auto q = [&](int j) -> float {
      const float pd = drow ? dsm.p(drow, j) : (j == d ? 1.0f : 0.0f);
      return fmaxf(__fsub_rn(sm.p(row, j), pd), 0.0f);
    };
    double adj = 0.0;
    for (int j = threadIdx.x; j < V; j += blockDim.x) adj += (double)q(j);
    const double adj_sum = block_reduce(adj, [](double a, double b) { return a + b; }, redd);
    int tok;
    if (!isfinite(adj_sum) || adj_sum <= 0.0) {
      // Degenerate residual: sample_token on the target row.
      const RowSoftmax s2 = row_softmax(row, V, t, true, redf, redi);
      const float r = uniform_f32(*st, draw++);
      tok = cdf_search(V, [&](int j) { return s2.p(row, j); }, (double)r, true, redd, &res);
      if (tok < 0) tok = V - 1;
    } else {
      const double target = uniform_f64(*st, draw++) * adj_sum;
      tok = cdf_search(V, q, target, false, redd, &res);
      if (tok < 0) tok = V - 1;
    }
    if (threadIdx.x == 0) st->out[produced] = (uint32_t)tok;
    ++produced;
    break;
  }
  if (accepted == dl) {
    const float* row = logits + (size_t)(r0 + dl) * V;
    const RowSoftmax sm = row_softmax(row, V, t, true, redf, redi);
    const float r = uniform_f32(*st, draw++);
    int tok = cdf_search(V, [&](int j) { return sm.p(row, j); }, (double)r, true, redd, &res);
    if (tok < 0) {
      // Fallback of sample_token: the highest probability (last index on ties).
      float best = -1.f;
      int bi = 0;
      for (int j = 0; j < V; ++j) {
        const float pj = sm.p(row, j);
        if (pj >= best) { best = pj; bi = j; }
      }
      tok = bi;
    }
    if (threadIdx.x == 0) st->out[produced] = (uint32_t)tok;
    ++produced;
  }
  if (threadIdx.x == 0) {
    st->accepted = accepted;
    st->produced = produced;
  }
}

}  // namespace

cudaError_t launch_sample_accept(StreamStep* st, int n, const float* logits, int vocab, float temperature,
                                 cudaStream_t s, const float* draft_logits) {
  return launch_pdl(sample_accept_kernel, dim3(n), dim3(kSampleThreads), 0, s, st, logits, vocab, temperature,
                    draft_logits);
}

}  // namespace rai
