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

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "layers.h"

namespace rai {

__device__ __forceinline__ int active_rows(const int* m_dev, int M) { return m_dev ? *m_dev : M; }

constexpr int kPvMaxStages = 4;
constexpr int kPvMaxThreads = 512 + 32;  // P.V compute threads + the producer warp
constexpr int kPvMaxThreadsH2 = 256 + 32;  // ... with two heads per thread (hd <= 128, hpk <= 8)
constexpr int kPvStepHeads = 2;  // heads per P.V thread for short segments
constexpr int kPvStepRows = 4;   // ... of at most this many rows

// ---------------------------------------------------------------------------
__global__ void embed_kernel(const uint32_t* __restrict__ ids, const int* m_dev, int M,
                             const uint8_t* __restrict__ codes, const uint8_t* __restrict__ params,
                             int vocab, int hidden, int gs, float embed_scale, float* __restrict__ out,
                             uint32_t* err, uint32_t* epoch, int with_logits) {
  pdl_wait_prior();
  pdl_launch_dependents();
  // Tensor parallelism: count this forward (and whether it ends in logits)
  // for the exchange waits of the kernels after this one.
  if (epoch && blockIdx.x == 0 && threadIdx.x == 0) {
    epoch[0] += 1u;
    if (with_logits) epoch[1] += 1u;
  }
  const int mact = active_rows(m_dev, M);
  const int ng = (hidden + gs - 1) / gs;
  for (int b = blockIdx.x; b < mact; b += gridDim.x) {
    const uint32_t tok = ids[b];
    if (tok >= (uint32_t)vocab) {
      if (threadIdx.x == 0) atomicOr(err, kErrBadInput);
      continue;
    }
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
      const int g = c / gs;
      const uint8_t* p = params + ((size_t)tok * ng + g) * 4;
      const float scale = f16_bits_to_f32((uint16_t)(p[0] | (p[1] << 8)));
      const float zero = f16_bits_to_f32((uint16_t)(p[2] | (p[3] << 8)));
      float v = __fadd_rn(__fmul_rn((float)codes[(size_t)tok * hidden + c], scale), zero);
      if (embed_scale != 1.0f) v = __fmul_rn(v, embed_scale);
      out[(size_t)b * hidden + c] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// rms_norm_heads: sequential scalar sum of squares over `len` values.
// The sum of squares is one ordered chain over the row (the reference's
// scalar loop), so its loads are issued 16 elements ahead of the adds.
__device__ float rms_inv_seq(const float* x, int len, float eps) {
  float ss = 0.f;
  int i = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && len >= 16) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int n16 = len / 16;
    float4 a[4], b[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) a[u] = x4[u];
    for (int j = 0; j < n16; ++j) {
      if (j + 1 < n16) {
#pragma unroll
        for (int u = 0; u < 4; ++u) b[u] = x4[4 * (j + 1) + u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        ss = __fadd_rn(ss, __fmul_rn(a[u].x, a[u].x));
        ss = __fadd_rn(ss, __fmul_rn(a[u].y, a[u].y));
        ss = __fadd_rn(ss, __fmul_rn(a[u].z, a[u].z));
        ss = __fadd_rn(ss, __fmul_rn(a[u].w, a[u].w));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = b[u];
    }
    i = n16 * 16;
  }
  for (; i < len; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
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
  pdl_wait_prior();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float srow[];  // q | k
  __shared__ float s_inv[2];
  const int mact = active_rows(m_dev, M);
  for (int b = blockIdx.x; b < mact; b += gridDim.x) {
  const RowInfo ri = rows[b];
  const StreamKV sk_ = kv[ri.stream];
  const int pos = ri.pos;
  int qd = nh * hd, kvd = nkv * hd, half = hd / 2, chunked = (half / 8) * 8;
  const float* row = qkv + (size_t)b * ld;
  stage_f32(srow, row, qd + kvd, threadIdx.x, blockDim.x);
  cp_async_wait<0>();
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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  // Warp per head, lane per pair: no index division.
  for (int h = warp; h < nh + nkv; h += nwarps) {
    float* hp = h < nh ? sq + h * hd : sk + (h - nh) * hd;
    for (int i = lane; i < half; i += 32) rope_pair(hp, i, half, chunked, c, s);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < qd; i += blockDim.x) q_out[(size_t)b * qd + i] = sq[i];
  const float* vrow = row + qd + kvd;
  const size_t lbase = (size_t)layer * nkv * sk_.max_ctx * hd;
  // k and v go to the cache, warp per KV head; v comes from the projection
  // row, its loads issued before the stores.
  for (int h = warp; h < nkv; h += nwarps) {
    const size_t o = lbase + ((size_t)h * sk_.max_ctx + pos) * hd;
    for (int d0 = 0; d0 < hd; d0 += 128) {
      float vv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int d = d0 + lane + 32 * u;
        vv[u] = d < hd ? vrow[h * hd + d] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int d = d0 + lane + 32 * u;
        if (d < hd) {
          sk_.k[o + d] = sk[h * hd + d];
          sk_.v[o + d] = vv[u];
        }
      }
    }
  }
  __syncthreads();  // shared rows are reused by the next row
  }
}

// ---------------------------------------------------------------------------
// Attention over row segments. A segment is a run of up to kSegRows rows of
// one stream at consecutive positions pos0 .. pos0 + nrows - 1 (a stream's
// verify rows, or a slice of its prompt), so every K/V row of the stream is
// read once per segment and shared by all its rows and all query heads of
// the KV head.
//
// Step 1: scores. CTA (kv head, segment, chunk of positions); the chunk's K
// rows are staged in shared memory (coalesced 16-byte copies into rows
// padded to HD + 4 floats, so the per-thread row reads are conflict free);
// thread t owns one position, keeps its K row in registers and scores it
// against every (row, head) of the segment whose position is >= t: 8-lane
// FMA dot, horizontal-sum tree, times scale (then softcap).
template <int HD>
struct ScoreCfg {
  static constexpr int CHUNK = HD >= 128 ? 128 : 256;  // positions (= threads) per CTA
  static constexpr int LD = HD + 4;                    // padded K row stride (floats)
};

template <int HD>
__global__ void __launch_bounds__(ScoreCfg<HD>::CHUNK) attn_scores_kernel(
    const float* __restrict__ q, const StreamKV* __restrict__ kv, int layer, const AttnSeg* __restrict__ segs,
    const int* nseg_dev, int nseg_max, int nh, int nkv, float scale, float softcap, float* __restrict__ scores,
    int n_alloc) {
  pdl_wait_prior();
  pdl_launch_dependents();
  constexpr int CH = ScoreCfg<HD>::CHUNK, LD = ScoreCfg<HD>::LD;
  extern __shared__ __align__(16) float sm[];
  float* sk = sm;            // [CH][LD]
  float* sq = sm + CH * LD;  // [nrows][hpk][HD]
  const int kvh = blockIdx.x, chunk = blockIdx.z;
  const int nseg = active_rows(nseg_dev, nseg_max);
  for (int si = blockIdx.y; si < nseg; si += gridDim.y) {
  const AttnSeg sg = segs[si];
  const int n_max = sg.pos0 + sg.nrows;
  const int t0 = chunk * CH;
  if (t0 >= n_max) continue;
  const int cnt = min(CH, n_max - t0);
  const int hpk = nh / nkv;
  const int tid = threadIdx.x;
  const StreamKV sk_ = kv[sg.stream];
  const float* kb = sk_.k + (((size_t)layer * nkv + kvh) * sk_.max_ctx + t0) * HD;
  for (int i = tid; i < cnt * (HD / 4); i += CH) {
    const int row = i / (HD / 4), c4 = i - row * (HD / 4);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sk + row * LD + 4 * c4)),
                 "l"(kb + 4 * (size_t)i)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  const int per_row = hpk * HD;
  if ((reinterpret_cast<uintptr_t>(q) & 15u) == 0) {
    // The segment's q rows as 16-byte asynchronous copies beside the K
    // chunk's (row strides are multiples of 4 floats), rather than one
    // dependent global load per element before the barrier.
    const int pr4 = per_row / 4;
    for (int i = tid; i < sg.nrows * pr4; i += CH) {
      const int r = i / pr4, o4 = i - r * pr4;
      cp_async16(sq + 4 * i, q + (size_t)(sg.row0 + r) * nh * HD + (size_t)kvh * per_row + 4 * o4);
    }
    cp_async_commit();
  } else {
    for (int i = tid; i < sg.nrows * per_row; i += CH) {
      const int r = i / per_row, o = i - r * per_row;
      sq[i] = q[(size_t)(sg.row0 + r) * nh * HD + (size_t)kvh * per_row + o];
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  if (tid < cnt) {
  const int t = t0 + tid;
  float kr[HD];
  {
    const float4* kp = reinterpret_cast<const float4*>(sk + tid * LD);
#pragma unroll
    for (int i = 0; i < HD / 4; ++i) {
      float4 v = kp[i];
      kr[4 * i] = v.x; kr[4 * i + 1] = v.y; kr[4 * i + 2] = v.z; kr[4 * i + 3] = v.w;
    }
  }
  // Rows r with pos0 + r >= t see position t.
  const int r_first = max(0, t - sg.pos0);
  for (int r = r_first; r < sg.nrows; ++r) {
    float* srow = scores + ((size_t)(sg.row0 + r) * nh + (size_t)kvh * hpk) * n_alloc + t;
    for (int h = 0; h < hpk; ++h) {
      const float4* qh = reinterpret_cast<const float4*>(sq + (r * hpk + h) * HD);
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int cc = 0; cc < HD / 8; ++cc) {
        float4 a0 = qh[2 * cc], a1 = qh[2 * cc + 1];
        acc[0] = __fmaf_rn(a0.x, kr[8 * cc + 0], acc[0]);
        acc[1] = __fmaf_rn(a0.y, kr[8 * cc + 1], acc[1]);
        acc[2] = __fmaf_rn(a0.z, kr[8 * cc + 2], acc[2]);
        acc[3] = __fmaf_rn(a0.w, kr[8 * cc + 3], acc[3]);
        acc[4] = __fmaf_rn(a1.x, kr[8 * cc + 4], acc[4]);
        acc[5] = __fmaf_rn(a1.y, kr[8 * cc + 5], acc[5]);
        acc[6] = __fmaf_rn(a1.z, kr[8 * cc + 6], acc[6]);
        acc[7] = __fmaf_rn(a1.w, kr[8 * cc + 7], acc[7]);
      }
      float sv = __fmul_rn(hsum8(acc), scale);
      if (softcap > 0.f) sv = __fmul_rn(softcap, tanhf(__fdiv_rn(sv, softcap)));
      srow[(size_t)h * n_alloc] = sv;
    }
  }
  }
  __syncthreads();  // the K and q tiles are reused by the next segment
  }
}

// Step 2: softmax. CTA (row, kv head); one warp per query head of the group
// (heads processed in batches of `hb` when the context is long). The head's
// score row is brought into shared memory with one bulk copy; max;
// exp(s - max) with Schraudolph for the first (n/8)*8 positions and the
// host-libm expf for the tail; the sum in 8 lanes (lane j adds positions
// 8i + j in order), the tree, the tail in order; then p = e * (1/sum)
// written back in place.
__global__ void __launch_bounds__(256) attn_softmax_kernel(const RowInfo* __restrict__ rows, const int* m_dev,
                                                           int M, int nh, int nkv, float* __restrict__ scores,
                                                           int n_alloc, int hb, ExpfTable et, uint32_t* err) {
  pdl_wait_prior();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float se_all[];  // [hb][n_alloc]
  __shared__ __align__(8) uint64_t bars[8];
  const int kvh = blockIdx.y;
  const int mact = active_rows(m_dev, M);
  const int hpk = nh / nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    mbar_init(&bars[warp], 1);
    fence_barrier_init();
  }
  __syncwarp();
  uint32_t phase = 0;
  for (int j = blockIdx.x; j < mact; j += gridDim.x) {
  const int n = rows[j].pos + 1;
  const int n8 = (n / 8) * 8, cnt = n8 / 8;
  const uint32_t bytes = (uint32_t)((n + 3) / 4) * 16u;
  for (int hbase = 0; hbase < hpk; hbase += hb) {
    const int hh = warp;
    if (hh < hb && hbase + hh < hpk) {
      float* row = scores + ((size_t)j * nh + (size_t)kvh * hpk + hbase + hh) * n_alloc;
      float* se = se_all + (size_t)hh * n_alloc;
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[warp], bytes);
        bulk_g2s(se, row, bytes, &bars[warp]);
      }
      const bool ok = mbar_wait(&bars[warp], phase, err);
      phase ^= 1u;
      if (!__all_sync(0xffffffffu, ok)) return;
      float m = -INFINITY;
      for (int t = lane; t < n; t += 32) m = fmaxf(m, se[t]);
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      for (int t = lane; t < n; t += 32) {
        float x = __fsub_rn(se[t], m);
        se[t] = t < n8 ? schraudolph(x) : expf_host(x, et);
      }
      __syncwarp();
      float acc = 0.f;
      if (lane < 8) {
        int i = 0;
        for (; i + 8 <= cnt; i += 8) {
          float v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = se[8 * (i + u) + lane];
#pragma unroll
          for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, v[u]);
        }
        for (; i < cnt; ++i) acc = __fadd_rn(acc, se[8 * i + lane]);
      }
      float a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] = __shfl_sync(0xffffffffu, acc, u);
      float sum = hsum8(a);
      for (int t = n8; t < n; ++t) sum = __fadd_rn(sum, se[t]);
      const float inv = __fdiv_rn(1.0f, sum);
      for (int t = lane; t < n; t += 32) row[t] = __fmul_rn(se[t], inv);
      // The next bulk copy into this buffer (async proxy) follows these
      // generic reads.
      __syncwarp();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
  }
  }
}

// Step 3: out[row][h][d] = fma(p_t, v_t[d], out) over t in order. CTA
// (kv head, segment); thread (d pair, group of HPT heads) carries the 2
// chains of its dims for each of its heads and each of the segment's rows
// (RB >= nrows) in registers: one p load (4 positions) feeds 2 dims, one V
// load (2 dims) feeds RB rows x HPT heads, so the V tile is read from shared
// memory hpk / HPT times (HPT > 1 for short segments, where those V reads
// would otherwise bound the kernel); positions are taken 8 at a time with
// all loads issued before the FMAs. V and p tiles
// stream through a ring of `ns` shared-memory stages filled by bulk copies
// that complete on mbarriers ("full"). The copies are issued by a producer
// warp (the CTA's last warp), which refills a stage once every compute warp
// has released it (one "empty" mbarrier per stage), so neither the issue of
// a tile's 1 + rows x heads copies nor a CTA-wide barrier sits between the
// compute warps' tiles. Row r only takes positions t <= pos0 + r.
template <int HD>
struct PvCfg {
  static constexpr int VT = HD >= 128 ? 32 : 64;  // positions per tile
};

// The producer warp walks the CTA's segments and tiles in the compute warps'
// order. Fill f goes to stage f % ns; from the second round on it first
// waits (bounded) until the compute warps released the stage's previous
// tile. If a wait gives up it lets its fills still in flight land (bounded)
// and returns, so no copy outlives the CTA.
template <int HD>
__device__ __forceinline__ void pv_produce(const StreamKV* __restrict__ kv, int layer,
                                           const AttnSeg* __restrict__ segs, int nseg, int nh, int nkv, int hpk,
                                           int kvh, const float* __restrict__ p, int n_alloc, int rb_alloc, int ns,
                                           float* sm, uint64_t* full, uint64_t* empty, uint32_t* err) {
  constexpr int VT = PvCfg<HD>::VT;
  const int lane = threadIdx.x & 31;
  const int stage_floats = VT * HD + rb_alloc * hpk * VT;
  int st = 0;          // stage of the next fill
  uint32_t ebits = 0;  // bit s: parity of stage s's next release
  int fills = 0;
  for (int si = blockIdx.y; si < nseg; si += gridDim.y) {
    const AttnSeg sg = segs[si];
    const StreamKV sk_ = kv[sg.stream];
    const float* vbase = sk_.v + ((size_t)layer * nkv + kvh) * sk_.max_ctx * HD;
    const float* prow0 = p + ((size_t)sg.row0 * nh + (size_t)kvh * hpk) * n_alloc;
    const int nrows = sg.nrows, n_max = sg.pos0 + nrows, ntiles = (n_max + VT - 1) / VT;
    for (int tile = 0; tile < ntiles; ++tile) {
      if (fills >= ns) {
        const bool ok = mbar_wait(&empty[st], (ebits >> st) & 1u, err);
        ebits ^= 1u << st;
        if (!__all_sync(0xffffffffu, ok)) {
          if (lane == 0)
            for (int f = fills > ns ? fills - ns : 0; f < fills; ++f)
              mbar_wait(&full[f % ns], (uint32_t)(f / ns) & 1u, nullptr);
          return;
        }
      }
      const int t0 = tile * VT, cnt = min(VT, n_max - t0), c4 = (cnt + 3) / 4;
      float* sv = sm + (size_t)st * stage_floats;
      float* sp = sv + VT * HD;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[st], (uint32_t)(cnt * HD * 4 + nrows * hpk * c4 * 16));
        bulk_g2s(sv, vbase + (size_t)t0 * HD, (uint32_t)(cnt * HD * 4), &full[st]);
      }
      __syncwarp();
      for (int i = lane; i < nrows * hpk; i += 32) {
        const int r = i / hpk, hh = i - r * hpk;
        bulk_g2s(sp + i * VT, prow0 + ((size_t)r * nh + hh) * n_alloc + t0, (uint32_t)(c4 * 16), &full[st]);
      }
      ++fills;
      if (++st == ns) st = 0;
    }
  }
}

// A compute warp's tiles of one segment. The stage ring persists across the
// segments a CTA handles: `head` is the next stage to consume and bit s of
// `bits` is the parity stage s's next fill completes. Returns false (output
// not written) if a wait gave up.
template <int HD, int RB, int HPT>
__device__ __forceinline__ bool pv_consume(int nh, int hpk, int kvh, const AttnSeg& sg, int rb_alloc, int ns,
                                           float* __restrict__ out, const float* sm, uint64_t* full,
                                           uint64_t* empty, uint32_t* err, int& head, uint32_t& bits) {
  constexpr int VT = PvCfg<HD>::VT;
  constexpr int NDP = HD / 2;
  const int stage_floats = VT * HD + rb_alloc * hpk * VT;
  const int tid = threadIdx.x, lane = tid & 31;
  const int dp = tid % NDP, h0 = (tid / NDP) * HPT;
  const int d0 = 2 * dp;
  const bool active = h0 < hpk;
  bool hv[HPT];  // head h0 + j exists (hpk need not be a multiple of HPT)
#pragma unroll
  for (int j = 0; j < HPT; ++j) hv[j] = h0 + j < hpk;
  const int nrows = sg.nrows;
  const int n_max = sg.pos0 + nrows, n_all = sg.pos0 + 1;
  const int ntiles = (n_max + VT - 1) / VT;
  float acc[RB][HPT][2];
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int j = 0; j < HPT; ++j) acc[r][j][0] = acc[r][j][1] = 0.f;
  for (int tile = 0; tile < ntiles; ++tile) {
    const int st = head;
    const bool ok = mbar_wait(&full[st], (bits >> st) & 1u, err);
    bits ^= 1u << st;
    if (++head == ns) head = 0;
    if (!__all_sync(0xffffffffu, ok)) return false;
    const int t0 = tile * VT, cnt = min(VT, n_max - t0);
    const float* sv = sm + (size_t)st * stage_floats + d0;
    // p of (row r, head h0 + j) at ph + (r * hpk + j) * VT.
    const float* ph = sm + (size_t)st * stage_floats + VT * HD + (active ? h0 : 0) * VT;
    if (active) {
      if (t0 + cnt <= n_all) {
        // Every row sees the whole tile.
        int t = 0;
        for (; t + 8 <= cnt; t += 8) {
          float2 v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = *reinterpret_cast<const float2*>(sv + (t + u) * HD);
          if constexpr (HPT > 1) {
            // (row, head) chains in groups of up to 4: their p loads first,
            // then per position one FMA of each chain (independent chains
            // back to back).
            constexpr int NPR = RB * HPT, PG = NPR < 4 ? NPR : 4;
#pragma unroll
            for (int q0 = 0; q0 < NPR; q0 += PG) {
              float p8[PG][8];
              bool lv[PG];
#pragma unroll
              for (int q = 0; q < PG; ++q) {
                const int r = (q0 + q) / HPT, j = (q0 + q) % HPT;
                lv[q] = r < nrows && hv[j];
                if (lv[q]) {
                  const float* pj = ph + (r * hpk + j) * VT + t;
                  const float4 pa = *reinterpret_cast<const float4*>(pj);
                  const float4 pb = *reinterpret_cast<const float4*>(pj + 4);
                  p8[q][0] = pa.x; p8[q][1] = pa.y; p8[q][2] = pa.z; p8[q][3] = pa.w;
                  p8[q][4] = pb.x; p8[q][5] = pb.y; p8[q][6] = pb.z; p8[q][7] = pb.w;
                }
              }
#pragma unroll
              for (int u = 0; u < 8; ++u)
#pragma unroll
                for (int q = 0; q < PG; ++q) {
                  const int r = (q0 + q) / HPT, j = (q0 + q) % HPT;
                  if (lv[q]) {
                    acc[r][j][0] = __fmaf_rn(p8[q][u], v[u].x, acc[r][j][0]);
                    acc[r][j][1] = __fmaf_rn(p8[q][u], v[u].y, acc[r][j][1]);
                  }
                }
            }
          } else {
#pragma unroll
            for (int r = 0; r < RB; ++r) {
              if (r < nrows) {
                const float* pj = ph + r * hpk * VT + t;
                const float4 pa = *reinterpret_cast<const float4*>(pj);
                const float4 pb = *reinterpret_cast<const float4*>(pj + 4);
                const float p8[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  acc[r][0][0] = __fmaf_rn(p8[u], v[u].x, acc[r][0][0]);
                  acc[r][0][1] = __fmaf_rn(p8[u], v[u].y, acc[r][0][1]);
                }
              }
            }
          }
        }
        for (; t < cnt; ++t) {
          const float2 v = *reinterpret_cast<const float2*>(sv + t * HD);
#pragma unroll
          for (int r = 0; r < RB; ++r) {
#pragma unroll
            for (int j = 0; j < HPT; ++j) {
              if (r < nrows && hv[j]) {
                const float a = ph[(r * hpk + j) * VT + t];
                acc[r][j][0] = __fmaf_rn(a, v.x, acc[r][j][0]);
                acc[r][j][1] = __fmaf_rn(a, v.y, acc[r][j][1]);
              }
            }
          }
        }
      } else {
        for (int t = 0; t < cnt; ++t) {
          const float2 v = *reinterpret_cast<const float2*>(sv + t * HD);
          const int rmin = t0 + t - sg.pos0;  // rows r >= rmin see position t0 + t
#pragma unroll
          for (int r = 0; r < RB; ++r) {
#pragma unroll
            for (int j = 0; j < HPT; ++j) {
              if (r < nrows && r >= rmin && hv[j]) {
                const float a = ph[(r * hpk + j) * VT + t];
                acc[r][j][0] = __fmaf_rn(a, v.x, acc[r][j][0]);
                acc[r][j][1] = __fmaf_rn(a, v.y, acc[r][j][1]);
              }
            }
          }
        }
      }
    }
    // This warp is done with the stage.
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (active) {
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
      for (int j = 0; j < HPT; ++j)
        if (r < nrows && hv[j])
          *reinterpret_cast<float2*>(out + (size_t)(sg.row0 + r) * nh * HD + (size_t)(kvh * hpk + h0 + j) * HD +
                                     d0) = make_float2(acc[r][j][0], acc[r][j][1]);
  }
  return true;
}

// HPT > 1 serves segments of at most kPvStepRows rows (the launch
// guarantees it). Block: the compute warps plus one producer warp.
template <int HD, int HPT>
__global__ void __launch_bounds__(HPT > 1 ? kPvMaxThreadsH2 : kPvMaxThreads) attn_pv_kernel(const StreamKV* __restrict__ kv, int layer,
                                                      const AttnSeg* __restrict__ segs, const int* nseg_dev,
                                                      int nseg_max, int nh, int nkv, const float* __restrict__ p,
                                                      int n_alloc, int rb_alloc, int ns, float* __restrict__ out,
                                                      uint32_t* err) {
  pdl_wait_prior();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float sm[];
  __shared__ __align__(8) uint64_t full[kPvMaxStages], empty[kPvMaxStages];
  const int kvh = blockIdx.x;
  const int nseg = active_rows(nseg_dev, nseg_max);
  if ((int)blockIdx.y >= nseg) return;
  const int hpk = nh / nkv;
  const int ncw = (int)(blockDim.x >> 5) - 1;  // compute warps
  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], (uint32_t)ncw);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if ((int)(threadIdx.x >> 5) == ncw) {
    pv_produce<HD>(kv, layer, segs, nseg, nh, nkv, hpk, kvh, p, n_alloc, rb_alloc, ns, sm, full, empty, err);
    return;
  }
  int head = 0;
  uint32_t bits = 0;
  for (int si = blockIdx.y; si < nseg; si += gridDim.y) {
    const AttnSeg sg = segs[si];
    bool ok;
#define RAI_PV(RB) pv_consume<HD, RB, HPT>(nh, hpk, kvh, sg, rb_alloc, ns, out, sm, full, empty, err, head, bits)
    if (sg.nrows <= 1) ok = RAI_PV(1);
    else if (sg.nrows <= 2) ok = RAI_PV(2);
    else if (sg.nrows <= 4) ok = RAI_PV(4);
    else if constexpr (HPT == 1) {
      if (sg.nrows <= 8) ok = RAI_PV(8);
      else ok = RAI_PV(kSegRows);
    } else {
      ok = false;
      if (threadIdx.x == 0) atomicOr(err, kErrBadInput);
    }
#undef RAI_PV
    if (!ok) return;
  }
}

// P.V for launches with fewer (kv head, segment) pairs than SMs (one or a
// few streams). There the kernel is bound by each thread's serial chain over
// the positions, so the work is spread as thin as the exact order allows:
// the head dimension is cut into DS slices of HDS = HD / DS columns, CTA
// (kv head, segment, slice), thread (one column of the slice, head), which
// carries out[r][h][d] = fma(p_t, v_t[d], out) over t in order for each of
// the segment's rows (the chains of pv_body, so results are identical). The
// rows' FMAs are interleaved per position (independent chains back to back).
// V slices and p tiles stream through an NS-deep ring of 16-byte cp.async
// copies issued by every thread (one barrier per tile). In the tiles every
// row sees whole, a thread with one or two rows runs its chain at the FMA
// latency: the shared loads of the next 8 positions are issued before the
// FMAs of the current 8, and the copy addresses need no divisions.
constexpr int kPvsStages = 8;         // ring depth where it fits in shared memory
constexpr int kPvsShallowStages = 4;  // otherwise
constexpr int kPvsTile = 64;          // positions per tile
constexpr int kPvsMaxSlices = 16;
constexpr int kPvsMaxPairs = kSegRows * 8;  // (row, head) pairs of a segment

// Rows r0 .. r0 + RG - 1 (those < nrows) over the 8 positions t .. t + 7 of
// a full tile: p from shared memory, v[] already loaded.
template <int RG>
__device__ __forceinline__ void pvs_rows8(float* acc, const float* ph, int pstride, int r0, int nrows, int t,
                                          const float (&v)[8]) {
  float p8[RG][8];
#pragma unroll
  for (int r = 0; r < RG; ++r) {
    if (r0 + r < nrows) {
      const float4 pa = *reinterpret_cast<const float4*>(ph + (r0 + r) * pstride + t);
      const float4 pb = *reinterpret_cast<const float4*>(ph + (r0 + r) * pstride + t + 4);
      p8[r][0] = pa.x; p8[r][1] = pa.y; p8[r][2] = pa.z; p8[r][3] = pa.w;
      p8[r][4] = pb.x; p8[r][5] = pb.y; p8[r][6] = pb.z; p8[r][7] = pb.w;
    }
  }
#pragma unroll
  for (int u = 0; u < 8; ++u)
#pragma unroll
    for (int r = 0; r < RG; ++r)
      if (r0 + r < nrows) acc[r0 + r] = __fmaf_rn(p8[r][u], v[u], acc[r0 + r]);
}

// The 8 positions of chunk k of a tile (V column values and the rows' p).
template <int HDS, int RB>
__device__ __forceinline__ void pvs_chunk_load(const float* sv, const float* ph, int pstride, int nrows, int k,
                                               float (&v)[8], float (&pq)[RB][8]) {
#pragma unroll
  for (int u = 0; u < 8; ++u) v[u] = sv[(8 * k + u) * HDS];
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    if (r < nrows) {
      const float4 pa = *reinterpret_cast<const float4*>(ph + r * pstride + 8 * k);
      const float4 pb = *reinterpret_cast<const float4*>(ph + r * pstride + 8 * k + 4);
      pq[r][0] = pa.x; pq[r][1] = pa.y; pq[r][2] = pa.z; pq[r][3] = pa.w;
      pq[r][4] = pb.x; pq[r][5] = pb.y; pq[r][6] = pb.z; pq[r][7] = pb.w;
    }
  }
}

template <int HD, int DS, int RB, int NS>
__device__ __forceinline__ void pvs_body(const float* __restrict__ vbase, const float* __restrict__ p, int nh,
                                         int hpk, int kvh, const AttnSeg& sg, int n_alloc, int rb_alloc,
                                         float* __restrict__ out, float* sm, int* pofs) {
  constexpr int HDS = HD / DS, VT = kPvsTile, V4 = HDS / 4, C4 = VT / 4;
  constexpr bool kPipelined = RB <= 2;
  const int stage_floats = VT * HDS + rb_alloc * hpk * VT;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int d = tid % HDS, h = tid / HDS;
  const bool active = h < hpk;
  const int nrows = sg.nrows;
  const int n_max = sg.pos0 + nrows, n_all = sg.pos0 + 1;
  const int ntiles = (n_max + VT - 1) / VT;
  const int pstride = hpk * VT;  // p of (row r, head h) at ph + r * pstride
  const int npairs = nrows * hpk;
  const float* prow0 = p + ((size_t)sg.row0 * nh + (size_t)kvh * hpk) * n_alloc;
  const float* vsl = vbase + (size_t)blockIdx.z * HDS;
  // Offset of (row r, head hh)'s p row from prow0, pair rh = r * hpk + hh.
  for (int rh = tid; rh < npairs; rh += nthr) {
    const int r = rh / hpk, hh = rh - r * hpk;
    pofs[rh] = (r * nh + hh) * n_alloc;
  }
  __syncthreads();
  // Every thread's share of tile `tile` (none past the end: the group is
  // still committed so the wait counts stay uniform). The block is a whole
  // number of warps, so a thread copies the same V column quad vc of rows
  // vr0, vr0 + VRS, ... and the same p quad pc of pairs pr0, pr0 + PRS, ...
  // in every tile.
  const int vc = tid % V4, vr0 = tid / V4, VRS = nthr / V4;
  const int pc = tid % C4, pr0 = tid / C4, PRS = nthr / C4;
  auto load = [&](int tile) {
    if (tile < ntiles) {
      const int t0 = tile * VT, cnt = min(VT, n_max - t0);
      float* sv = sm + (size_t)(tile % NS) * stage_floats;
      float* sp = sv + VT * HDS;
      const float* vsrc = vsl + (size_t)(t0 + vr0) * HD + 4 * vc;
      float* vdst = sv + vr0 * HDS + 4 * vc;
      for (int r = vr0; r < cnt; r += VRS, vsrc += (size_t)VRS * HD, vdst += VRS * HDS) cp_async16(vdst, vsrc);
      if (4 * pc < cnt)
        for (int rh = pr0; rh < npairs; rh += PRS) cp_async16(sp + rh * VT + 4 * pc, prow0 + pofs[rh] + t0 + 4 * pc);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int j = 0; j < NS - 1; ++j) load(j);
  float acc[RB];
#pragma unroll
  for (int r = 0; r < RB; ++r) acc[r] = 0.f;
  for (int tile = 0; tile < ntiles; ++tile) {
    cp_async_wait<NS - 2>();  // this thread's copies of `tile` have landed
    __syncthreads();          // ... and everyone's; stage (tile - 1) % NS is free
    load(tile + NS - 1);
    if (!active) continue;
    const int t0 = tile * VT, cnt = min(VT, n_max - t0);
    const float* sv = sm + (size_t)(tile % NS) * stage_floats + d;
    const float* ph = sm + (size_t)(tile % NS) * stage_floats + VT * HDS + h * VT;
    if (kPipelined && t0 + VT <= n_all) {
      // Whole tile, every row: 8 chunks of 8 positions, chunk k + 1's loads
      // issued before chunk k's FMAs.
      float v[2][8], pq[2][RB][8];
      pvs_chunk_load<HDS, RB>(sv, ph, pstride, nrows, 0, v[0], pq[0]);
#pragma unroll
      for (int k = 0; k < VT / 8; ++k) {
        if (k + 1 < VT / 8) pvs_chunk_load<HDS, RB>(sv, ph, pstride, nrows, k + 1, v[(k + 1) & 1], pq[(k + 1) & 1]);
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
          for (int r = 0; r < RB; ++r)
            if (r < nrows) acc[r] = __fmaf_rn(pq[k & 1][r][u], v[k & 1][u], acc[r]);
      }
    } else if (t0 + cnt <= n_all) {
      constexpr int RG = RB < 4 ? RB : 4;  // rows per interleaved group
      int t = 0;
      for (; t + 8 <= cnt; t += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = sv[(t + u) * HDS];
#pragma unroll
        for (int r0 = 0; r0 < RB; r0 += RG) pvs_rows8<RG>(acc, ph, pstride, r0, nrows, t, v);
      }
      for (; t < cnt; ++t) {
        const float v = sv[t * HDS];
#pragma unroll
        for (int r = 0; r < RB; ++r)
          if (r < nrows) acc[r] = __fmaf_rn(ph[r * pstride + t], v, acc[r]);
      }
    } else {
      for (int t = 0; t < cnt; ++t) {
        const float v = sv[t * HDS];
        const int rmin = t0 + t - sg.pos0;  // rows r >= rmin see position t0 + t
#pragma unroll
        for (int r = 0; r < RB; ++r)
          if (r < nrows && r >= rmin) acc[r] = __fmaf_rn(ph[r * pstride + t], v, acc[r]);
      }
    }
  }
  if (active) {
#pragma unroll
    for (int r = 0; r < RB; ++r)
      if (r < nrows)
        out[(size_t)(sg.row0 + r) * nh * HD + (size_t)(kvh * hpk + h) * HD + (size_t)blockIdx.z * HDS + d] = acc[r];
  }
}

template <int HD, int DS, int NS>
__global__ void __launch_bounds__(256) attn_pv_split_kernel(const StreamKV* __restrict__ kv, int layer,
                                                            const AttnSeg* __restrict__ segs, const int* nseg_dev,
                                                            int nseg_max, int nh, int nkv,
                                                            const float* __restrict__ p, int n_alloc, int rb_alloc,
                                                            float* __restrict__ out) {
  pdl_wait_prior();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float sm[];
  __shared__ int pofs[kPvsMaxPairs];
  const int kvh = blockIdx.x;
  const int nseg = active_rows(nseg_dev, nseg_max);
  const int hpk = nh / nkv;
  for (int si = blockIdx.y; si < nseg; si += gridDim.y) {
    const AttnSeg sg = segs[si];
    const StreamKV sk_ = kv[sg.stream];
    const float* vbase = sk_.v + ((size_t)layer * nkv + kvh) * sk_.max_ctx * HD;
#define RAI_PVS(RB) pvs_body<HD, DS, RB, NS>(vbase, p, nh, hpk, kvh, sg, n_alloc, rb_alloc, out, sm, pofs)
    if (sg.nrows <= 1) RAI_PVS(1);
    else if (sg.nrows <= 2) RAI_PVS(2);
    else if (sg.nrows <= 4) RAI_PVS(4);
    else if (sg.nrows <= 8) RAI_PVS(8);
    else RAI_PVS(kSegRows);
#undef RAI_PVS
    cp_async_wait<0>();
    __syncthreads();  // the ring is refilled for the next segment
  }
}

// ---------------------------------------------------------------------------
// Fused attention for launches of many short segments (a many-stream verify
// step, each stream's rows cut into segments of at most kFusedRows). CTA
// (kv head, segment): the segment's scores and probabilities stay in shared
// memory, and the stream's K and V rows are read once each per segment,
// through a double-buffered ring of 16-byte asynchronous copies. Same
// arithmetic, in the same order, as the three kernels above:
//   scores: per (row, head, position) the 8-lane FMA dot, the horizontal-sum
//     tree, times scale (then softcap);
//   softmax: one warp per (row, head): max; Schraudolph's exp for the first
//     (n/8)*8 positions, the host-libm expf for the tail; the 8-lane ordered
//     sum, the tree, the tail in order; p = e * (1/sum);
//   P.V: out = fma(p_t, v_t[d], out) over t in order.
constexpr int kFusedRows = 2;
constexpr int kFusedThreads = 256;

template <int HD>
struct FusedCfg {
  static constexpr int CH = HD >= 128 ? 64 : 128;      // positions per K / V chunk
  static constexpr int LD = HD + 4;                    // padded row stride (floats)
  static constexpr int TPP = kFusedThreads / CH;       // score threads per position
  static constexpr int NDP = HD / 2;                   // P.V dim pairs
  static constexpr int HG = kFusedThreads / NDP;       // P.V head groups
  static constexpr int HMAX = (8 + HG - 1) / HG;       // P.V heads per thread (hpk <= 8)
};

template <int HD>
__global__ void __launch_bounds__(kFusedThreads) attn_fused_kernel(
    const float* __restrict__ q, const StreamKV* __restrict__ kv, int layer, const AttnSeg* __restrict__ segs,
    const int* nseg_dev, int nseg_max, int nh, int nkv, float scale, float softcap, int n_alloc, ExpfTable et,
    float* __restrict__ out) {
  pdl_wait_prior();
  pdl_launch_dependents();
  constexpr int CH = FusedCfg<HD>::CH, LD = FusedCfg<HD>::LD, TPP = FusedCfg<HD>::TPP;
  constexpr int NDP = FusedCfg<HD>::NDP, HG = FusedCfg<HD>::HG, HMAX = FusedCfg<HD>::HMAX;
  extern __shared__ __align__(16) float sm[];
  const int hpk = nh / nkv;
  float* kb = sm;                          // [2][CH][LD] K, then V, chunks
  float* sq = kb + 2 * CH * LD;            // [kFusedRows][hpk][HD] the segment's q rows
  float* ss = sq + kFusedRows * hpk * HD;  // [kFusedRows * hpk][n_alloc] scores, then p
  const int kvh = blockIdx.x;
  const int nseg = active_rows(nseg_dev, nseg_max);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int si = blockIdx.y; si < nseg; si += gridDim.y) {
    const AttnSeg sg = segs[si];
    const int nrows = sg.nrows;  // <= kFusedRows (the launch guarantees it)
    const int n_max = sg.pos0 + nrows;
    const int nch = (n_max + CH - 1) / CH;
    const int npairs = nrows * hpk;  // (row, head) pairs, index r * hpk + h
    const StreamKV sk_ = kv[sg.stream];
    const size_t hoff = ((size_t)layer * nkv + kvh) * sk_.max_ctx * HD;
    // Chunk c of K or V into buffer c & 1 (an empty commit past the end keeps
    // the wait counts uniform).
    auto load = [&](const float* base, int c) {
      if (c < nch) {
        const int t0 = c * CH, cnt = min(CH, n_max - t0);
        float* dst = kb + (c & 1) * CH * LD;
        for (int i = tid; i < cnt * (HD / 4); i += kFusedThreads) {
          const int row = i / (HD / 4), c4 = i - row * (HD / 4);
          cp_async16(dst + row * LD + 4 * c4, base + (size_t)(t0 + row) * HD + 4 * c4);
        }
      }
      cp_async_commit();
    };
    load(sk_.k + hoff, 0);
    {
      const int per_row = hpk * HD;
      for (int i = tid; i < nrows * per_row; i += kFusedThreads) {
        const int r = i / per_row, o = i - r * per_row;
        sq[i] = q[(size_t)(sg.row0 + r) * nh * HD + (size_t)kvh * per_row + o];
      }
    }
    // ---- scores: thread (position of the chunk, subset of the pairs) ----
    const int pl = tid % CH, part = tid / CH;
    for (int c = 0; c < nch; ++c) {
      load(sk_.k + hoff, c + 1);
      cp_async_wait<1>();  // chunk c has landed
      __syncthreads();
      const int t = c * CH + pl;
      if (t < n_max) {
        float kr[HD];
        const float4* kp = reinterpret_cast<const float4*>(kb + (c & 1) * CH * LD + pl * LD);
#pragma unroll
        for (int i = 0; i < HD / 4; ++i) {
          const float4 v = kp[i];
          kr[4 * i] = v.x; kr[4 * i + 1] = v.y; kr[4 * i + 2] = v.z; kr[4 * i + 3] = v.w;
        }
        // Rows r with pos0 + r >= t see position t.
        const int r_first = max(0, t - sg.pos0);
        for (int pi = part; pi < npairs; pi += TPP) {
          if (pi / hpk < r_first) continue;
          const float4* qh = reinterpret_cast<const float4*>(sq + pi * HD);
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int cc = 0; cc < HD / 8; ++cc) {
            const float4 a0 = qh[2 * cc], a1 = qh[2 * cc + 1];
            acc[0] = __fmaf_rn(a0.x, kr[8 * cc + 0], acc[0]);
            acc[1] = __fmaf_rn(a0.y, kr[8 * cc + 1], acc[1]);
            acc[2] = __fmaf_rn(a0.z, kr[8 * cc + 2], acc[2]);
            acc[3] = __fmaf_rn(a0.w, kr[8 * cc + 3], acc[3]);
            acc[4] = __fmaf_rn(a1.x, kr[8 * cc + 4], acc[4]);
            acc[5] = __fmaf_rn(a1.y, kr[8 * cc + 5], acc[5]);
            acc[6] = __fmaf_rn(a1.z, kr[8 * cc + 6], acc[6]);
            acc[7] = __fmaf_rn(a1.w, kr[8 * cc + 7], acc[7]);
          }
          float sv = __fmul_rn(hsum8(acc), scale);
          if (softcap > 0.f) sv = __fmul_rn(softcap, tanhf(__fdiv_rn(sv, softcap)));
          ss[(size_t)pi * n_alloc + t] = sv;
        }
      }
      __syncthreads();  // buffer c & 1 is refilled next
    }
    // V's first chunk streams in while the softmax runs.
    load(sk_.v + hoff, 0);
    // ---- softmax: one warp per (row, head) ----
    for (int pi = warp; pi < npairs; pi += kFusedThreads / 32) {
      const int n = sg.pos0 + pi / hpk + 1, n8 = (n / 8) * 8, cnt8 = n8 / 8;
      float* se = ss + (size_t)pi * n_alloc;
      float m = -INFINITY;
      for (int t = lane; t < n; t += 32) m = fmaxf(m, se[t]);
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      for (int t = lane; t < n; t += 32) {
        const float x = __fsub_rn(se[t], m);
        se[t] = t < n8 ? schraudolph(x) : expf_host(x, et);
      }
      __syncwarp();
      float acc = 0.f;
      if (lane < 8) {
        int i = 0;
        for (; i + 8 <= cnt8; i += 8) {
          float v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = se[8 * (i + u) + lane];
#pragma unroll
          for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, v[u]);
        }
        for (; i < cnt8; ++i) acc = __fadd_rn(acc, se[8 * i + lane]);
      }
      float a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] = __shfl_sync(0xffffffffu, acc, u);
      float sum = hsum8(a);
      for (int t = n8; t < n; ++t) sum = __fadd_rn(sum, se[t]);
      const float inv = __fdiv_rn(1.0f, sum);
      __syncwarp();
      for (int t = lane; t < n; t += 32) se[t] = __fmul_rn(se[t], inv);
    }
    // ---- P.V: thread (dim pair, head group), chains of its rows x heads ----
    const int dp = tid % NDP, hg = tid / NDP;
    float acc[kFusedRows][HMAX][2];
#pragma unroll
    for (int r = 0; r < kFusedRows; ++r)
#pragma unroll
      for (int j = 0; j < HMAX; ++j) acc[r][j][0] = acc[r][j][1] = 0.f;
    for (int c = 0; c < nch; ++c) {
      load(sk_.v + hoff, c + 1);
      cp_async_wait<1>();
      __syncthreads();  // chunk c of V and (first pass) every warp's p rows
      const int t0 = c * CH, cnt = min(CH, n_max - t0);
      const float* vb = kb + (c & 1) * CH * LD + 2 * dp;
      int tl = 0;
      if (t0 + cnt <= sg.pos0 + 1) {
        // Every row sees the whole chunk: 4 positions per round, loads first.
        for (; tl + 4 <= cnt; tl += 4) {
          float2 v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const float2*>(vb + (tl + u) * LD);
#pragma unroll
          for (int r = 0; r < kFusedRows; ++r) {
            if (r >= nrows) break;
#pragma unroll
            for (int j = 0; j < HMAX; ++j) {
              const int h = hg + j * HG;
              if (h >= hpk) break;
              const float4 pq = *reinterpret_cast<const float4*>(ss + (size_t)(r * hpk + h) * n_alloc + t0 + tl);
              const float p4[4] = {pq.x, pq.y, pq.z, pq.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                acc[r][j][0] = __fmaf_rn(p4[u], v[u].x, acc[r][j][0]);
                acc[r][j][1] = __fmaf_rn(p4[u], v[u].y, acc[r][j][1]);
              }
            }
          }
        }
      }
      for (; tl < cnt; ++tl) {
        const int t = t0 + tl;
        const float2 v = *reinterpret_cast<const float2*>(vb + tl * LD);
#pragma unroll
        for (int r = 0; r < kFusedRows; ++r) {
          if (r >= nrows || t > sg.pos0 + r) continue;
#pragma unroll
          for (int j = 0; j < HMAX; ++j) {
            const int h = hg + j * HG;
            if (h >= hpk) break;
            const float a = ss[(size_t)(r * hpk + h) * n_alloc + t];
            acc[r][j][0] = __fmaf_rn(a, v.x, acc[r][j][0]);
            acc[r][j][1] = __fmaf_rn(a, v.y, acc[r][j][1]);
          }
        }
      }
      __syncthreads();  // buffer c & 1 is refilled next
    }
#pragma unroll
    for (int r = 0; r < kFusedRows; ++r) {
      if (r >= nrows) break;
#pragma unroll
      for (int j = 0; j < HMAX; ++j) {
        const int h = hg + j * HG;
        if (h >= hpk) break;
        *reinterpret_cast<float2*>(out + (size_t)(sg.row0 + r) * nh * HD + (size_t)(kvh * hpk + h) * HD + 2 * dp) =
            make_float2(acc[r][j][0], acc[r][j][1]);
      }
    }
    cp_async_wait<0>();
    __syncthreads();  // shared memory is reused by the next segment
  }
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

// Tensor parallelism: logits hold vocabulary rows vocab_off .. vocab_off +
// vocab; the keys carry the model's token ids and are folded into every
// rank's best[] (dst), so all ranks end with the same argmax.
struct BestDst {
  unsigned long long* p[kMaxTp];
  int n;
};

__global__ void argmax_kernel(const float* __restrict__ logits, int vocab, const int* m_dev, int M,
                              BestDst best, int vocab_off) {
  pdl_wait_prior();
  pdl_launch_dependents();
  const int mact = active_rows(m_dev, M);
  for (int b = blockIdx.y; b < mact; b += gridDim.y) {
    unsigned long long k = 0;
    const float* row = logits + (size_t)b * vocab;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x) {
      unsigned long long c = argmax_key(row[i], (uint32_t)(i + vocab_off));
      k = c > k ? c : k;
    }
    for (int o = 16; o; o >>= 1) {
      unsigned long long c = __shfl_xor_sync(0xffffffffu, k, o);
      k = c > k ? c : k;
    }
    if ((threadIdx.x & 31) == 0)
      for (int d = 0; d < best.n; ++d) atomicMax(best.p[d] + b, k);
  }
  if (best.n > 1) __threadfence_system();
}

// ---------------------------------------------------------------------------
// Draft search, one CTA per stream: for n from hi down to lo, the largest
// start s with ctx[s..s+n] == suffix (s <= len-n-1) wins; draft =
// ctx[s+n .. s+n+dl) with dl = min(max_draft, budget, len - s - n), budget =
// max_ctx - pos - 1.
__global__ void ngram_kernel(const uint32_t* __restrict__ ctx_all, int ctx_cap, StreamStep* st_all,
                             const StreamKV* __restrict__ kv, int max_draft, int max_ngram, int min_ngram) {
  pdl_wait_prior();
  pdl_launch_dependents();
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

// Compact every stream's verify rows into one row set (block-wide prefix
// sums over the streams of rows and of attention segments), write row
// metadata, token ids and segments, zero the argmax slots.
__global__ void __launch_bounds__(1024) plan_kernel(StreamStep* st, int n, RowInfo* rows, uint32_t* ids,
                                                    int* m_active, AttnSeg* segs, int* n_segs, int seg_len,
                                                    unsigned long long* best, int best_len) {
  pdl_wait_prior();
  pdl_launch_dependents();
  __shared__ unsigned long long wsum[32];
  __shared__ unsigned long long carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry = 0ull;
  for (int i = tid; i < best_len; i += blockDim.x) best[i] = 0ull;
  __syncthreads();
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + tid;
    const int nr = i < n ? st[i].n_rows : 0;
    const int ns = (nr + seg_len - 1) / seg_len;
    // (rows << 32) | segments, inclusive scan
    unsigned long long v = ((unsigned long long)nr << 32) | (unsigned)ns;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      unsigned long long u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    if (lane == 31) wsum[warp] = v;
    __syncthreads();
    if (warp == 0) {
      const int nw = blockDim.x >> 5;
      unsigned long long w = lane < nw ? wsum[lane] : 0ull;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        unsigned long long u = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += u;
      }
      if (lane < nw) wsum[lane] = w;
    }
    __syncthreads();
    const unsigned long long before = carry + (warp ? wsum[warp - 1] : 0ull) + v -
                                      (((unsigned long long)nr << 32) | (unsigned)ns);
    if (i < n) {
      const int r0 = (int)(before >> 32), s0 = (int)(before & 0xFFFFFFFFull);
      const int p = st[i].pos;
      st[i].row0 = r0;
      for (int b = 0; b < nr; ++b) {
        rows[r0 + b] = RowInfo{p + b, i};
        ids[r0 + b] = st[i].tokens[b];
      }
      for (int k = 0; k < ns; ++k)
        segs[s0 + k] = AttnSeg{r0 + k * seg_len, min(seg_len, nr - k * seg_len), i, p + k * seg_len};
    }
    __syncthreads();
    if (tid == 0) carry += wsum[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
  if (tid == 0) {
    *m_active = (int)(carry >> 32);
    *n_segs = (int)(carry & 0xFFFFFFFFull);
  }
}

// Greedy acceptance per stream: accept d_i while argmax_i == d_i; the first
// mismatch is replaced by argmax_i; if all are accepted the bonus is argmax_k.
__global__ void accept_kernel(StreamStep* st_all, const unsigned long long* __restrict__ best, TpLink tp, int slot,
                              uint32_t* err) {
  pdl_wait_prior();
  pdl_launch_dependents();
  // Tensor parallelism: best[] holds every rank's vocabulary slice once the
  // logits exchange completes.
  if (slot >= 0 && !tp_exchange(tp, slot, 1, err)) return;
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

__global__ void expf_range_kernel(uint32_t first, size_t n, float* __restrict__ out, ExpfTable et) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = expf_host(__uint_as_float(first + (uint32_t)i), et);
}

// ---------------------------------------------------------------------------
// Host launchers.
cudaError_t launch_expf_range(uint32_t first, size_t n, float* out, const ExpfTable& et, cudaStream_t s) {
  const size_t blocks = (n + 255) / 256;
  expf_range_kernel<<<(unsigned)grid_cap((int)(blocks < (1u << 20) ? blocks : (1u << 20)), 8), 256, 0, s>>>(
      first, n, out, et);
  return cudaGetLastError();
}

cudaError_t launch_embed(const uint32_t* ids, const int* m_dev, int M, const uint8_t* codes,
                         const uint8_t* params, int vocab, int hidden, int gs, float embed_scale,
                         float* out, uint32_t* err, cudaStream_t s, uint32_t* epoch, bool with_logits) {
  return launch_pdl(embed_kernel, dim3(grid_cap(M, 1)), dim3(256), 0, s, ids, m_dev, M, codes, params, vocab, hidden, gs,
                    embed_scale, out, err, epoch, (int)with_logits);
}

cudaError_t launch_qkv_post(float* qkv, int ld, float* q_out, int nh, int nkv, int hd, const float* qn,
                            const float* kn, int qk_mode, float eps, const float* rope_cos,
                            const float* rope_sin, const StreamKV* kv, int layer, const RowInfo* rows,
                            const int* m_dev, int M, cudaStream_t s) {
  size_t smem = (size_t)(nh + nkv) * hd * sizeof(float);
  return launch_pdl(qkv_post_kernel, dim3(grid_cap(M, 1)), dim3(256), smem, s, qkv, ld, q_out, nh, nkv, hd, qn, kn, qk_mode, eps, rope_cos, rope_sin,
                                       kv, layer, rows, m_dev, M);

}

size_t attention_n_chunks(int n_alloc) { return (size_t)(n_alloc + kScoreChunk - 1) / kScoreChunk; }

namespace {
int score_chunk(int hd) { return hd >= 128 ? 128 : 256; }
size_t scores_smem_bytes(int hd, int hpk, int seg_rows) {
  return ((size_t)score_chunk(hd) * (hd + 4) + (size_t)seg_rows * hpk * hd) * sizeof(float);
}
size_t pv_stage_bytes(int hd, int hpk, int rb_alloc) {
  const int vt = hd >= 128 ? 32 : 64;
  return (size_t)(vt * hd + rb_alloc * hpk * vt) * sizeof(float);
}
// Heads per P.V thread: kPvStepHeads for short segments when there are
// enough (kv head, segment) CTAs to fill the GPU several times over (the
// shared-memory V reads then bound the kernel); one otherwise, where the
// kernel is latency bound and wants the most threads.
int pv_heads_per_thread(int hpk, int seg_rows, int nseg_max, int nkv) {
  return seg_rows <= kPvStepRows && nseg_max * nkv >= 4 * device_sm_count() ? std::min(hpk, kPvStepHeads) : 1;
}
// P.V block: the compute threads (dim pair x head group), whole warps, plus
// the producer warp.
int pv_threads(int hd, int hpk, int hpt) { return ((hd / 2) * ((hpk + hpt - 1) / hpt) + 31) / 32 * 32 + 32; }
// Head-dimension slices of the split P.V, when the (kv head, segment) pairs
// alone do not fill the SMs (1 = the pv_body path): the thinnest slices (up
// to kPvsMaxSlices, at least 4 columns each) that still give a CTA a warp of
// threads (HDS x hpk >= 32), and at least enough for a CTA of at most 256
// threads. Each thread's serial chain bounds the kernel, so the columns go
// to as many CTAs, on as many SMs, as that allows.
int pv_dim_slices(int hd, int hpk, int nseg_max, int nkv) {
  const int base = nseg_max * nkv, sms = device_sm_count();
  if (base >= sms) return 1;
  int ds = 1;
  while (ds < kPvsMaxSlices && hd / (2 * ds) >= 4 && ((hd / (2 * ds)) * hpk >= 32 || (hd / ds) * hpk > 256)) ds *= 2;
  return ds > 1 && (hd / ds) * hpk <= 256 ? ds : 1;
}
size_t fused_smem_bytes(int hd, int hpk, int n_alloc) {
  const int ch = hd >= 128 ? 64 : 128;
  return ((size_t)2 * ch * (hd + 4) + (size_t)kFusedRows * hpk * hd + (size_t)kFusedRows * hpk * n_alloc) *
         sizeof(float);
}
// The fused kernel can serve launches whose segments are all short and
// whose (kv head, segment) pairs fill the SMs (a many-stream verify step),
// when the segment's scores fit in shared memory. It is opt-in: measured on
// the 64-stream TinyLlama step it is slower than the three kernels (6.73 vs
// 4.67 ms per step): its ~160 KB of shared memory leave one CTA per SM with a
// two-deep copy ring, too few bytes in flight against the three kernels' many
// CTAs per SM. RAI_ATTN_FUSED=1 uses it where it applies, 2 for every launch
// of short segments (to test it on few streams); unset or 0: never.
bool use_fused(int hd, int hpk, int seg_rows, int nseg_max, int nkv, int n_alloc) {
  static const int mode = [] {
    const char* e = std::getenv("RAI_ATTN_FUSED");
    return e ? std::atoi(e) : 0;
  }();
  if (mode == 0 || seg_rows > kFusedRows || hpk > 8 || fused_smem_bytes(hd, hpk, n_alloc) > kAttnMaxSmem)
    return false;
  return mode == 2 || nseg_max * nkv >= device_sm_count();
}
size_t pvs_smem_bytes(int hd, int ds, int hpk, int rb_alloc, int ns) {
  return (size_t)ns * ((size_t)kPvsTile * (hd / ds) + (size_t)rb_alloc * hpk * kPvsTile) * sizeof(float);
}
// Ring depth of the split P.V: kPvsStages where it fits in shared memory.
int pvs_stages(int hd, int ds, int hpk, int rb_alloc) {
  return pvs_smem_bytes(hd, ds, hpk, rb_alloc, kPvsStages) <= kAttnMaxSmem ? kPvsStages : kPvsShallowStages;
}
}  // namespace

int build_segments(const RowInfo* rows, int M, int seg_len, AttnSeg* segs) {
  int n = 0;
  for (int i = 0; i < M;) {
    int j = i + 1;
    while (j < M && j - i < seg_len && rows[j].stream == rows[i].stream && rows[j].pos == rows[j - 1].pos + 1) ++j;
    segs[n++] = AttnSeg{i, j - i, rows[i].stream, rows[i].pos};
    i = j;
  }
  return n;
}

namespace {
template <int HD>
cudaError_t launch_pv_split(int ds, int ns, dim3 g, int threads, size_t smem, cudaStream_t s, const StreamKV* kv,
                            int layer, const AttnSeg* segs, const int* nseg_dev, int nseg_max, int nh, int nkv,
                            const float* p, int n_alloc, int rb_alloc, float* out) {
  switch (ds) {
#define RAI_PVS_CASE(DSV)                                                                                       \
  case DSV:                                                                                                     \
    if constexpr (HD / DSV >= 4) {                                                                              \
      if (ns == kPvsStages)                                                                                     \
        return launch_pdl(attn_pv_split_kernel<HD, DSV, kPvsStages>, g, dim3(threads), smem, s, kv, layer,      \
                          segs, nseg_dev, nseg_max, nh, nkv, p, n_alloc, rb_alloc, out);                        \
      return launch_pdl(attn_pv_split_kernel<HD, DSV, kPvsShallowStages>, g, dim3(threads), smem, s, kv, layer, \
                        segs, nseg_dev, nseg_max, nh, nkv, p, n_alloc, rb_alloc, out);                          \
    }                                                                                                           \
    break;
    RAI_PVS_CASE(2)
    RAI_PVS_CASE(4)
    RAI_PVS_CASE(8)
    RAI_PVS_CASE(16)
#undef RAI_PVS_CASE
  }
  return cudaErrorInvalidValue;
}
}  // namespace

cudaError_t launch_attention(const float* q, float* out, const StreamKV* kv, int layer, const RowInfo* rows,
                             const int* m_dev, int M, const AttnSeg* segs, const int* nseg_dev, int nseg_max,
                             int seg_rows, int nh, int nkv, int hd, float scale, float softcap, float* scores,
                             int n_alloc, const ExpfTable& et, uint32_t* err, cudaStream_t s) {
  const int hpk = nh / nkv;
  if (seg_rows < 1 || seg_rows > kSegRows || hpk > 8 || n_alloc % 4) return cudaErrorInvalidValue;
  const int nch = (n_alloc + score_chunk(hd) - 1) / score_chunk(hd);
  const size_t sm1 = scores_smem_bytes(hd, hpk, seg_rows);
  int hb = (int)std::min<size_t>((size_t)hpk, kAttnMaxSmem / ((size_t)n_alloc * sizeof(float)));
  const size_t stage = pv_stage_bytes(hd, hpk, seg_rows);
  // Stages: as many as fit ~72 KB (three CTAs per SM), at least 2, at most 4.
  const int ns = (int)std::max<size_t>(2, std::min<size_t>(kPvMaxStages, (72 * 1024) / stage));
  const size_t sm3 = (size_t)ns * stage;
  const int hpt = pv_heads_per_thread(hpk, seg_rows, nseg_max, nkv);
  const int t3 = pv_threads(hd, hpk, hpt);
  const int ds = pv_dim_slices(hd, hpk, nseg_max, nkv);
  const int t3s = ((hd / ds) * hpk + 31) / 32 * 32;
  const int ns_split = pvs_stages(hd, ds, hpk, seg_rows);
  const size_t sm3s = pvs_smem_bytes(hd, ds, hpk, seg_rows, ns_split);
  if (hb < 1 || sm1 > kAttnMaxSmem || sm3 > kAttnMaxSmem || t3 > (hpt > 1 ? kPvMaxThreadsH2 : kPvMaxThreads) ||
      (ds > 1 && (sm3s > kAttnMaxSmem || t3s > 256)))
    return cudaErrorInvalidValue;
  const size_t sm2 = (size_t)hb * n_alloc * sizeof(float);
  // Segment and row dimensions loop inside the kernels; the grids cover
  // about two waves.
  const int seg_grid = std::max(1, grid_cap(nseg_max * nkv * nch, 8) / (nkv * nch));
  dim3 g1(nkv, std::min(nseg_max, seg_grid), nch), g2(grid_cap(M, 1), nkv),
      g3(nkv, std::min(nseg_max, std::max(1, grid_cap(nseg_max * nkv, 3) / nkv)));
  const bool fused = use_fused(hd, hpk, seg_rows, nseg_max, nkv, n_alloc);
  const dim3 gf(nkv, std::min(nseg_max, std::max(1, grid_cap(nseg_max * nkv, 1) / nkv)));
  const size_t smf = fused_smem_bytes(hd, hpk, n_alloc);
#define RAI_ATTN(HDV)                                                                                        \
  case HDV:                                                                                                  \
    if (fused)                                                                                               \
      return launch_pdl(attn_fused_kernel<HDV>, gf, dim3(kFusedThreads), smf, s, q, kv, layer, segs,          \
                        nseg_dev, nseg_max, nh, nkv, scale, softcap, n_alloc, et, out);                      \
    if (cudaError_t e = launch_pdl(attn_scores_kernel<HDV>, g1, dim3(ScoreCfg<HDV>::CHUNK), sm1, s, q, kv,   \
                                   layer, segs, nseg_dev, nseg_max, nh, nkv, scale, softcap, scores,        \
                                   n_alloc))                                                                \
      return e;                                                                                             \
    if (cudaError_t e = launch_pdl(attn_softmax_kernel, g2, dim3(256), sm2, s, rows, m_dev, M, nh, nkv,      \
                                   scores, n_alloc, hb, et, err))                                           \
      return e;                                                                                             \
    if (ds > 1)                                                                                             \
      return launch_pv_split<HDV>(ds, ns_split, dim3(nkv, nseg_max, ds), t3s, sm3s, s, kv, layer, segs,     \
                                  nseg_dev,                                                                 \
                                  nseg_max, nh, nkv, (const float*)scores, n_alloc, seg_rows, out);         \
    return hpt > 1 ? launch_pdl(attn_pv_kernel<HDV, kPvStepHeads>, g3, dim3(t3), sm3, s, kv, layer, segs,   \
                                nseg_dev, nseg_max, nh, nkv, (const float*)scores, n_alloc, seg_rows, ns, out, \
                                err)                                                                           \
                   : launch_pdl(attn_pv_kernel<HDV, 1>, g3, dim3(t3), sm3, s, kv, layer, segs, nseg_dev,       \
                                nseg_max, nh, nkv, (const float*)scores, n_alloc, seg_rows, ns, out, err);
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

namespace {
template <int HD>
cudaError_t set_pv_split_attributes(int bytes) {
  cudaError_t e = cudaSuccess;
#define RAI_PVS_ATTR(DSV)                                                                                      \
  if constexpr (HD / DSV >= 4) {                                                                               \
    if (e == cudaSuccess)                                                                                      \
      e = cudaFuncSetAttribute(attn_pv_split_kernel<HD, DSV, kPvsStages>,                                      \
                               cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);                            \
    if (e == cudaSuccess)                                                                                      \
      e = cudaFuncSetAttribute(attn_pv_split_kernel<HD, DSV, kPvsShallowStages>,                               \
                               cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);                            \
  }
  RAI_PVS_ATTR(2)
  RAI_PVS_ATTR(4)
  RAI_PVS_ATTR(8)
  RAI_PVS_ATTR(16)
#undef RAI_PVS_ATTR
  return e;
}
}  // namespace

cudaError_t init_layer_attributes() {
  const int bytes = (int)kAttnMaxSmem;
  cudaError_t e = cudaFuncSetAttribute(attn_softmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
#define RAI_ATTR(HDV)                                                                                     \
  if (e == cudaSuccess)                                                                                   \
    e = cudaFuncSetAttribute(attn_fused_kernel<HDV>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes); \
  if (e == cudaSuccess)                                                                                   \
    e = cudaFuncSetAttribute(attn_pv_kernel<HDV, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes); \
  if (e == cudaSuccess) e = set_pv_split_attributes<HDV>(bytes);                                          \
  if (e == cudaSuccess)                                                                                   \
    e = cudaFuncSetAttribute(attn_pv_kernel<HDV, kPvStepHeads>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                             bytes);                                                                      \
  if (e == cudaSuccess)                                                                                   \
    e = cudaFuncSetAttribute(attn_scores_kernel<HDV>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  RAI_ATTR(16)
  RAI_ATTR(32)
  RAI_ATTR(64)
  RAI_ATTR(128)
#undef RAI_ATTR
  return e;
}

cudaError_t launch_argmax(const float* logits, int vocab, const int* m_dev, int M, unsigned long long* best,
                          cudaStream_t s, int vocab_off, unsigned long long* const* peers, int n_peers) {
  int blocks = (vocab + 4095) / 4096;
  if (blocks > 64) blocks = 64;
  dim3 grid(blocks, std::max(1, std::min(M, grid_cap(blocks * M, 2) / blocks)));
  BestDst d = {};
  d.p[0] = best;
  d.n = 1;
  if (peers && n_peers > 1) {
    d.n = n_peers;
    for (int i = 0; i < n_peers; ++i) d.p[i] = peers[i];
  }
  return launch_pdl(argmax_kernel, grid, dim3(256), 0, s, logits, vocab, m_dev, M, d, vocab_off);
}

cudaError_t launch_ngram(const uint32_t* ctx, int ctx_cap, StreamStep* st, const StreamKV* kv, int n,
                         int max_draft, int max_ngram, int min_ngram, cudaStream_t s) {
  return launch_pdl(ngram_kernel, dim3(n), dim3(1024), 0, s, ctx, ctx_cap, st, kv, max_draft, max_ngram, min_ngram);
}

cudaError_t launch_plan(StreamStep* st, int n, RowInfo* rows, uint32_t* ids, int* m_active, AttnSeg* segs,
                        int* n_segs, int seg_len, unsigned long long* best, int best_len, cudaStream_t s) {
  if (seg_len < 1 || seg_len > kSegRows) return cudaErrorInvalidValue;
  return launch_pdl(plan_kernel, dim3(1), dim3(1024), 0, s, st, n, rows, ids, m_active, segs, n_segs, seg_len, best,
                    best_len);
}

cudaError_t launch_accept(StreamStep* st, int n, const unsigned long long* best, cudaStream_t s, const TpLink* tp,
                          int slot, uint32_t* err) {
  TpLink link;
  if (tp && tp->world > 1 && slot >= 0) link = *tp;
  else slot = -1;
  return launch_pdl(accept_kernel, dim3(n), dim3(32), 0, s, st, (const unsigned long long*)best, link, slot, err);
}

}  // namespace rai
