// Exact W4A8 linear on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same arithmetic as gemm_exact_kernel (rai-infer/src/gemm.rs:562-674,
// 599-673): per (token, row, group) eight int32 lane dots (reference lane L
// = columns 8L..8L+7 of each 64-column chunk), each converted to f32,
// multiplied by (w_scale * x_scale) and added into lane L's f32 accumulator
// in group order; the row result is the horizontal-sum tree plus the
// sequential zero correction sum_g(w_zero * x_sum). Integer dots are exact
// in any summation order, so the tensor cores may add a lane's 16 products
// in any order; everything after the dot runs in the reference's order on
// the CUDA cores.
//
// Work item: 128 weight rows (two 64-row packed tiles) x 16 tokens, every
// group in order. Per group g one tcgen05.mma.kind::i8 per lane pair
// (2m, 2m+1), M = 128 rows, K = 32 (lane 2m's 16 codes, then lane 2m+1's),
// N = 32 = (token, lane parity): the B image holds token t's lane-2m codes in
// column t and its lane-(2m+1) codes in column 16 + t, each beside 16 zero
// bytes, so column t accumulates only lane 2m and column 16 + t only lane
// 2m+1. D (int32, TMEM) of group g holds lane L, token t of row r at lane r,
// column slot * 128 + 16 L + t. Every slot is seeded with 0x4B400000 and the
// MMAs accumulate onto it, so a lane dot read as f32 is 12582912 + dot
// exactly (one subtraction gives the dot); the epilogue re-seeds a slot as
// it reads it.
//
// Weights: a u8 image per (128-row tile, group), built once by
// pack4_tc_kernel, that is the MMA's A operand as it sits in shared memory
// (canonical K-major layout, no swizzle: lane L's 16 codes of row r at
// L * 2048 + (r / 8) * 128 + (r % 8) * 16), followed by the rows' f16
// (scale, zero) pairs; one bulk copy per group.
//
// Warps: 0 = producer (bulk copies of the weight image and the quantized
// activation blocks of each group into a ring of stages), 1 = TMEM owner
// and MMA issuer (one thread), 2-3 = converters (activation words -> the B
// image; the group's scales -> a separate ring, so a stage is free as soon
// as its MMAs complete), 4-11 = epilogue (TMEM lane quadrant warp % 4,
// tokens 8 * ((warp - 4) / 4) + 0..7).
// Every wait is bounded; on a timeout the roles stop, drain what is in
// flight and the TMEM columns are released before the CTA exits.
#include <cuda_runtime.h>

#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace rai {

namespace {

constexpr int kTcTok = 16;    // tokens per item
constexpr int kTcStages = 8;
constexpr int kTcScal = 8;  // scale ring: per group the rows' (scale, zero) and the tokens' (scale, sum)
constexpr int kTcSlots = 4;  // TMEM accumulator slots of 128 columns
constexpr int kTcCols = kTcSlots * 128;
constexpr int kTcThreads = 12 * 32;
constexpr int kTcConvThreads = 64;

// One stage = one group of one item.
constexpr int kTcAOff = 0;                                     // weight block: A image + params
constexpr int kTcParOff = kTcImgBytes;                         // (scale, zero) f16 per row
constexpr int kTcActOff = kTcBlockBytes;                       // 2 activation blocks
constexpr int kTcBOff = kTcActOff + 2 * kActBlockBytes;        // B image: 4 MMAs x 1 KB
constexpr int kTcStageBytes = kTcBOff + 4 * 1024;
static_assert(kTcAOff % 128 == 0 && kTcBOff % 128 == 0 && kTcStageBytes % 128 == 0, "stage alignment");
constexpr int kTcScalBytes = kTcRows * 4 + 2 * kActBlockTok * 8;  // 640
constexpr int kTcScalOff = kTcStages * kTcStageBytes;
constexpr int kTcBarOff = kTcScalOff + kTcScal * kTcScalBytes;
constexpr size_t kTcSmem = (size_t)kTcBarOff + 512;

constexpr uint32_t kTcMagic = 0x4B400000u;  // 12582912.0f: (magic + dot) read as f32 is exact
// Instruction descriptor: D s32 (bits 4-5 = 2), A u8 (7-9 = 0), B s8
// (10-12 = 1), both K-major, N = 32 (bits 17-22 = N >> 3), M = 128 (bits
// 24-28 = M >> 4).
constexpr uint32_t kTcIdesc = (2u << 4) | (1u << 10) | ((32u >> 3) << 17) | ((128u >> 4) << 24);

struct TcParams {
  const uint8_t* w;    // weight images ([128-row tile][group] blocks of kTcBlockBytes)
  const uint8_t* act;  // quantized activations ([8-token block][group] blocks)
  float* out;
  const float* bias;
  const float* residual;
  uint32_t* err;
  const int* m_dev;
  int rows, groups, M, ld_out, mode;
  int tiles;  // 128-row tiles; item i = (tile i % tiles, token chunk i / tiles)
  float one;   // 1.0f, opaque to the compiler: the accumulation is fma(product, one, acc)
};

// Shared-memory matrix descriptor, K-major without swizzle: 8-row x 16-byte
// core matrices, rows 16 B apart, `sbo` between 8-row blocks, `lbo` between
// the two 16-byte K chunks; version 1 (sm_100).
__device__ __forceinline__ uint64_t tc_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D += A x B (D holds the magic seed).
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t"
      "}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kTcIdesc), "r"(1u)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 8 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The magic seed into 8 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tc_seed8(uint32_t taddr) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
               "r"(kTcMagic)
               : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Packed f32 pairs (the rounding of each half equals the scalar .rn op).
__device__ __forceinline__ uint64_t tc_f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 tc_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t tc_sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t tc_mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// fma(product, one, acc) with one = 1.0 rounds once, as product + acc does;
// `one` comes from a kernel parameter so nothing is fused into it.
__device__ __forceinline__ uint64_t tc_fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Bounded wait without the suspend-time hint of mbar_wait: the pipeline's
// hand-offs are short and the hinted wait's wake-up latency dominated them.
// try_wait blocks for a hardware-defined interval per poll; the deadline
// (about a second of SM clock) bounds the whole wait.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > 2000000000ll) break;
  }
  if (err) atomicOr(err, kErrWaitTimeout);
  return false;
}

__device__ __forceinline__ bool tc_item(const TcParams& p, int mact, int item, int* tile, int* t0, int* nt) {
  const int c = item / p.tiles;
  *t0 = c * kTcTok;
  if (*t0 >= mact) return false;
  *tile = item - c * p.tiles;
  *nt = min(kTcTok, mact - *t0);
  return true;
}

__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcBarOff);  // stage loaded (bulk copies)
  uint64_t* cvt = full + kTcStages;                                 // stage images built
  uint64_t* sfree = cvt + kTcStages;                                // stage's MMAs complete
  uint64_t* qfull = sfree + kTcStages;                              // scale slot written
  uint64_t* qdone = qfull + kTcScal;                                // scale slot read by the epilogue
  uint64_t* dfull = qdone + kTcScal;                                // slot's MMAs complete
  uint64_t* dempty = dfull + kTcSlots;                              // slot read by the epilogue
  uint64_t* mdone = dempty + kTcSlots;                              // every MMA of the CTA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.groups;

  // The B images' zero halves are written once.
  for (int i = threadIdx.x; i < kTcStages * 256; i += blockDim.x)
    *reinterpret_cast<uint4*>(smem + (i >> 8) * kTcStageBytes + kTcBOff + (i & 255) * 16) = make_uint4(0, 0, 0, 0);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&cvt[s], kTcConvThreads / 32);
      mbar_init(&sfree[s], 1);
    }
    for (int r = 0; r < kTcScal; ++r) {
      mbar_init(&qfull[r], kTcConvThreads / 32);
      mbar_init(&qdone[r], 8);
    }
    for (int d = 0; d < kTcSlots; ++d) {
      mbar_init(&dfull[d], 1);
      mbar_init(&dempty[d], 8);
    }
    mbar_init(mdone, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Weights do not depend on the previous kernel: a lead CTA (its first item
  // is token chunk 0, which always exists) requests its first stages'
  // weights before waiting on it.
  const bool lead = (int)blockIdx.x < p.tiles;
  const int pre = lead ? min(kTcStages, G) : 0;
  if (warp == 0 && lane == 0) {
    for (int q = 0; q < pre; ++q) {
      mbar_expect_tx(&full[q], (uint32_t)kTcBlockBytes);
      bulk_g2s(smem + q * kTcStageBytes + kTcAOff, p.w + ((size_t)blockIdx.x * G + q) * kTcBlockBytes, kTcBlockBytes,
               &full[q]);
    }
  }
  pdl_wait_prior();
  const int mact = p.m_dev ? *p.m_dev : p.M;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      bool ok = true;
      uint32_t k = 0;
      int tile, t0, nt;
      for (int item = blockIdx.x; ok && tc_item(p, mact, item, &tile, &t0, &nt); item += gridDim.x) {
        const int nb = (nt + 7) >> 3;
        for (int g = 0; g < G; ++g, ++k) {
          const int s = k % kTcStages;
          const uint32_t n = k / kTcStages;
          if (n > 0 && !tc_wait(&sfree[s], (n - 1) & 1, p.err)) { ok = false; break; }
          uint8_t* st = smem + s * kTcStageBytes;
          const bool prefetched = (int)k < pre;
          const uint32_t abytes = (uint32_t)(nb * kActBlockBytes);
          mbar_arrive_expect_tx(&full[s], prefetched ? abytes : (uint32_t)kTcBlockBytes + abytes);
          if (!prefetched)
            bulk_g2s(st + kTcAOff, p.w + ((size_t)tile * G + g) * kTcBlockBytes, kTcBlockBytes, &full[s]);
          for (int b = 0; b < nb; ++b)
            bulk_g2s(st + kTcActOff + b * kActBlockBytes,
                     p.act + ((size_t)((t0 >> 3) + b) * G + g) * kActBlockBytes, kActBlockBytes, &full[s]);
        }
      }
      // Let every fill this CTA issued land before the CTA exits (bounded;
      // only matters after a timeout).
      for (uint32_t j = k > kTcStages ? k - kTcStages : 0; j < k; ++j)
        tc_wait(&full[j % kTcStages], (j / kTcStages) & 1, nullptr);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t sbase = smem_u32(smem);
      uint32_t k = 0;
      bool ok = true;
      int tile, t0, nt;
      for (int item = blockIdx.x; ok && tc_item(p, mact, item, &tile, &t0, &nt); item += gridDim.x) {
        for (int g = 0; g < G; ++g, ++k) {
          const int s = k % kTcStages, d = k % kTcSlots;
          const uint32_t n = k / kTcStages, u = k / kTcSlots;
          if (!tc_wait(&cvt[s], n & 1, p.err) || !tc_wait(&dempty[d], u & 1, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sbase + s * kTcStageBytes + kTcAOff, b0 = sbase + s * kTcStageBytes + kTcBOff;
#pragma unroll
          for (int m = 0; m < 4; ++m)
            tc_mma(tmem + d * 128 + m * 32, tc_desc(a0 + m * 4096, 2048, 128), tc_desc(b0 + m * 1024, 512, 128));
          tc_commit(&dfull[d]);
          tc_commit(&sfree[s]);
        }
      }
      // Drain: every MMA issued above completes before TMEM is released.
      tc_commit(mdone);
      tc_wait(mdone, 0, nullptr);
    }
  } else if (warp < 4) {
    // ---------------- converters ----------------
    const int ct = threadIdx.x - 64;
    uint32_t k = 0;
    int tile, t0, nt;
    for (int item = blockIdx.x; tc_item(p, mact, item, &tile, &t0, &nt); item += gridDim.x) {
      const int nb = (nt + 7) >> 3;
      bool ok = true;
      for (int g = 0; g < G; ++g, ++k) {
        const int s = k % kTcStages;
        const uint32_t n = k / kTcStages;
        const int r = k % kTcScal;
        const uint32_t qn = k / kTcScal;
        if (!__all_sync(0xffffffffu, tc_wait(&full[s], n & 1, p.err) &&
                                         (qn == 0 || tc_wait(&qdone[r], (qn - 1) & 1, p.err)))) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * kTcStageBytes;
        // Scales for the epilogue: rows' (scale, zero) f16 pairs, then the
        // (scale, sum) of the item's two 8-token activation blocks.
        {
          uint32_t* q = reinterpret_cast<uint32_t*>(smem + kTcScalOff + r * kTcScalBytes);
          const uint32_t* par = reinterpret_cast<const uint32_t*>(st + kTcParOff);
          q[ct] = par[ct];
          q[ct + 64] = par[ct + 64];
          if (ct < 32) {
            const int b = ct >> 4, w = ct & 15;
            q[kTcRows + ct] = b < nb ? reinterpret_cast<const uint32_t*>(st + kTcActOff + b * kActBlockBytes +
                                                                         kActBlockTok * kActRowBytes)[w]
                                     : 0u;
          }
        }
        // B image: (lane L, token t) -> 16 bytes at L * 512 + (L & 1) * 256 + 16 t.
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int pr = ct + kTcConvThreads * i;
          const int L = pr >> 4, t = pr & 15;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (t < nb * 8) {
            const uint8_t* row = st + kTcActOff + (t >> 3) * kActBlockBytes + (t & 7) * kActRowBytes;
            const int wl = 2 * (L & 3) + (L >> 2);  // lane L's word within a 32-byte slot
            uint32_t w[4];
#pragma unroll
            for (int sl = 0; sl < 4; ++sl) {
              const int off = sl * 32 + 4 * wl;
              w[sl] = *reinterpret_cast<const uint32_t*>(row + ((((off >> 4) ^ (t & 7)) << 4) | (off & 15)));
            }
            v = make_uint4(w[0], w[1], w[2], w[3]);
          }
          *reinterpret_cast<uint4*>(st + kTcBOff + L * 512 + (L & 1) * 256 + 16 * t) = v;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&cvt[s]);
          mbar_arrive(&qfull[r]);
        }
      }
      if (!ok) break;
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3, h = (warp - 4) >> 2;
    const int rl = 32 * q + lane;  // row within the item = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + 8 * h;
    const uint64_t magic2 = tc_f2(12582912.0f, 12582912.0f);
    const uint64_t one2 = tc_f2(p.one, p.one);
    // Seed this warp's columns of every slot, then release the slots for
    // their first MMAs (phase 0 of dempty).
#pragma unroll
    for (int d = 0; d < kTcSlots; ++d)
#pragma unroll
      for (int L = 0; L < 8; ++L) tc_seed8(lane_base + d * 128 + 16 * L);
    tc_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int d = 0; d < kTcSlots; ++d) mbar_arrive(&dempty[d]);
    uint32_t k = 0;
    int tile, t0, nt;
    bool ok = true;
    for (int item = blockIdx.x; ok && tc_item(p, mact, item, &tile, &t0, &nt); item += gridDim.x) {
      const int ntl = min(8, nt - 8 * h);  // this warp's tokens of the item (none if <= 0)
      uint64_t facc[4][8];  // lane L, tokens (2 tp, 2 tp + 1) as a packed pair
      float zc[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) zc[t] = 0.f;
#pragma unroll
      for (int tp = 0; tp < 4; ++tp)
#pragma unroll
        for (int L = 0; L < 8; ++L) facc[tp][L] = 0ull;
      for (int g = 0; g < G; ++g, ++k) {
        const int r = k % kTcScal, d = k % kTcSlots;
        const uint32_t qn = k / kTcScal, u = k / kTcSlots;
        if (!tc_wait(&dfull[d], u & 1, p.err) || !tc_wait(&qfull[r], qn & 1, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint8_t* sq = smem + kTcScalOff + r * kTcScalBytes;
        const uint32_t col = lane_base + d * 128;
        uint32_t v[8][8];
        if (ntl > 0) {
#pragma unroll
          for (int L = 0; L < 8; ++L) tc_ld8(col + 16 * L, v[L]);
          tc_wait_ld();
        }
        // Re-seed the slot; the stores complete while the f32 math below
        // runs, and the slot is released after it.
#pragma unroll
        for (int L = 0; L < 8; ++L) tc_seed8(col + 16 * L);
        if (ntl > 0) {
          const uint32_t pw = reinterpret_cast<const uint32_t*>(sq)[rl];
          const float ws = f16_bits_to_f32((uint16_t)(pw & 0xFFFF)), wz = f16_bits_to_f32((uint16_t)(pw >> 16));
          const float2* xsp = reinterpret_cast<const float2*>(sq + kTcRows * 4) + 8 * h;
          float2 xs[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) xs[t] = xsp[t];
          __syncwarp();
          if (lane == 0) mbar_arrive(&qdone[r]);
          const uint64_t ws2 = tc_f2(ws, ws);
#pragma unroll
          for (int tp = 0; tp < 4; ++tp) {
            if (2 * tp >= ntl) break;  // warp-uniform: no tokens left
            const int t = 2 * tp;
            // combined_scale = w_scale * x_scale (gemm.rs:606), tokens t, t + 1
            const uint64_t c2 = tc_mul2(ws2, tc_f2(xs[t].x, xs[t + 1].x));
#pragma unroll
            for (int L = 0; L < 8; ++L)
              facc[tp][L] = tc_fma2(
                  tc_mul2(tc_sub2(tc_f2(__uint_as_float(v[L][t]), __uint_as_float(v[L][t + 1])), magic2), c2),
                  one2, facc[tp][L]);
            // zero correction, sequential in g (gemm.rs:666-670)
            zc[t] = __fadd_rn(zc[t], __fmul_rn(wz, xs[t].y));
            zc[t + 1] = __fadd_rn(zc[t + 1], __fmul_rn(wz, xs[t + 1].y));
          }
        } else {
          __syncwarp();
          if (lane == 0) mbar_arrive(&qdone[r]);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dempty[d]);
      }
      if (!ok || ntl <= 0) continue;
      const int row = tile * kTcRows + rl;
      if (row >= p.rows) continue;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        if (t >= ntl) break;
        float a[8];
#pragma unroll
        for (int L = 0; L < 8; ++L) {
          const float2 pr = tc_unpack(facc[t >> 1][L]);
          a[L] = (t & 1) ? pr.y : pr.x;
        }
        // ((a0+a4) + (a1+a5)) + ((a2+a6) + (a3+a7))
        const float s0 = __fadd_rn(a[0], a[4]), s1 = __fadd_rn(a[1], a[5]);
        const float s2 = __fadd_rn(a[2], a[6]), s3 = __fadd_rn(a[3], a[7]);
        float v = __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3)), zc[t]);
        const size_t o = (size_t)(t0 + 8 * h + t) * p.ld_out + row;
        if (p.mode == kEpiBias) v = __fadd_rn(v, p.bias[row]);
        else if (p.mode == kEpiResidual) v = __fadd_rn(p.residual[o], v);
        p.out[o] = v;
      }
    }
  }

  // Teardown: every role is done with TMEM (the MMA issuer drained its
  // MMAs, the epilogue waited for its loads); release the columns.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
  }
}

// Weight image of one (128-row tile, group): byte (L, r, j) of the A image
// (j = 4 s + b, s = packed slot 2c + p) holds the code of column
// 64c + 8L + 2b + p of row r: lane L's columns in the order the activation
// blocks hold them; then (scale, zero) per row.
__global__ void pack4_tc_kernel(const uint8_t* __restrict__ nib, const uint8_t* __restrict__ params, int rows,
                                int cols, int gs, int groups, uint8_t* __restrict__ out, size_t total) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= total) return;
  const size_t blk = i / kTcBlockBytes;
  const int within = (int)(i % kTcBlockBytes);
  const int g = (int)(blk % groups), tile = (int)(blk / groups);
  uint8_t v = 0;
  if (within < kTcImgBytes) {
    const int L = within >> 11, rem = within & 2047;
    const int row = tile * kTcRows + (rem >> 7) * 8 + ((rem >> 4) & 7);
    const int j = rem & 15, sl = j >> 2, b = j & 3;
    const int col = 64 * (sl >> 1) + 8 * L + 2 * b + (sl & 1);
    if (row < rows && col < gs && g * gs + col < cols) {
      const uint8_t byte = nib[(size_t)row * (cols / 2) + ((size_t)g * gs + col) / 2];
      v = (col & 1) ? (byte >> 4) : (byte & 0xF);
    }
  } else {
    const int q = within - kTcImgBytes, r = q >> 2, k = q & 3;
    const int row = tile * kTcRows + r;
    if (row < rows) v = params[((size_t)row * groups + g) * 4 + k];
  }
  out[i] = v;
}

}  // namespace

cudaError_t pack_linear4_tc(const uint8_t* nibbles, const uint8_t* params, int rows, int cols, int gs, uint8_t* out,
                            cudaStream_t s) {
  const int groups = (int)ceil_div(cols, gs);
  const size_t total = tc_image_bytes(rows, cols, gs);
  const int threads = 256;
  pack4_tc_kernel<<<(unsigned)ceil_div(total, threads), threads, 0, s>>>(nibbles, params, rows, cols, gs, groups,
                                                                          out, total);
  return cudaGetLastError();
}

// Opt-in (RAI_GEMM_TC=1): on the B200 this kernel is bit-exact but slower
// than the mma.sync kernel at every measured shape (see the design notes).
bool gemm_tc_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("RAI_GEMM_TC");
    return e && e[0] == '1';
  }();
  return on;
}

cudaError_t init_gemm_tc_attributes() {
  return cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
}

cudaError_t gemm_tc(const PackedLinear& w, const ActBuf& act, int M, float* out, int ld_out, const GemmEpilogue& epi,
                    uint32_t* err, cudaStream_t s, const int* m_dev) {
  TcParams p = {};
  p.w = w.tc;
  p.act = act.data;
  p.out = out;
  p.bias = epi.bias;
  p.residual = epi.residual;
  p.err = err;
  p.m_dev = m_dev;
  p.rows = w.rows;
  p.groups = w.groups;
  p.M = M;
  p.ld_out = ld_out;
  p.mode = epi.mode;
  p.one = 1.0f;
  p.tiles = (int)ceil_div(w.rows, kTcRows);
  const long items = (long)p.tiles * (long)ceil_div(M, kTcTok);
  const long wave = device_sm_count();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(items < wave ? items : wave));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kTcSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel, p);
}

}  // namespace rai
