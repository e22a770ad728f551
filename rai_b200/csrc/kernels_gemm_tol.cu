// W4A8 linear on the 5th-generation tensor cores for many tokens (prefill
// and batched multi-stream verify): tcgen05.mma.kind::i8 with TMEM
// accumulators, to the BASELINE tolerance instead of bit for bit.
//
// The integer part is exact and the same as the reference's
// (rai-infer/src/gemm.rs:562-674): per (token, row, group) the dot of the
// int8-quantized activations (quantize_input_split_avx2, gemm.rs:280-374)
// with the u4 codes is an exact int32. The reference then keeps it as 8 lane
// dots, scales each in f32 and adds the lanes in a fixed tree; here the
// group's whole dot comes out of the tensor core (4 chained K = 32 MMAs into
// one TMEM column) and the f32 part is
//   acc += float(dot) * (w_scale * x_scale) + w_zero * x_sum
// per group, fused multiply-adds in group order: the same terms with a
// different rounding order, so results differ from the reference by a few
// f32 ulps of the row's terms (the tolerance the parity tests state), and an
// eighth of the exact kernel's f32 work.
//
// Work item: 128 weight rows x 128 tokens x a range of groups. Launches with
// fewer (row tile, token chunk) pairs than SMs split the groups into S
// ranges (split-K); each range's partial sums go to a workspace, and for
// each epilogue warp's slice the CTA that finishes it last adds the ranges
// in range order (deterministic).
//
// Operands per group, in shared memory:
//   * A (weights, M = 128 rows x K = 128): the two 64-row 4-bit blocks of
//     the mma.sync layout expanded to u8 by converter warps into the MMA's
//     K-major layout without swizzle (16-byte K chunk u of row r at
//     u * 2048 + (r / 8) * 128 + (r % 8) * 16);
//   * B (activations, N = 128 tokens x K = 128): the quantized-activation
//     blocks exactly as the quantize kernels wrote them. A block's 8 token
//     rows of 128 code bytes store 16-byte unit u of token t at unit
//     u ^ (t & 7): with the block at a 1024-byte aligned address that is the
//     MMA's 128-byte-swizzled K-major layout, so the bulk copies place the
//     blocks and the MMA reads them in place.
// Column k of A and of B is the same column of the group (both follow the
// activation blocks' byte order), so each MMA column is a whole group dot.
//
// Warps: 0 producer (bulk copies; lane b copies activation block b), 1 TMEM
// owner + MMA issuer (one thread), 2-3 converters (two weight rows each;
// scales for the epilogue), 4-11 epilogue (TMEM lane quadrant warp % 4, 64
// tokens each). Every wait is bounded; on a timeout the roles stop, drain
// what is in flight, and the TMEM columns are released before the CTA exits.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace rai {

namespace {

constexpr int kTolRows = 128;
constexpr int kTolTok = 128;
constexpr int kTolStages = 5;
constexpr int kTolASlots = 4;
constexpr int kTolScal = 4;
constexpr int kTolSlots = 4;  // TMEM accumulator slots of 128 columns
constexpr int kTolCols = kTolSlots * 128;
constexpr int kTolThreads = 12 * 32;
constexpr int kConvWarps = 2;
constexpr int kTolBlocks = kTolTok / kActBlockTok;  // 16 activation blocks per item

// Stage (one group of one item), 1024-byte aligned.
constexpr int kStBOff = 0;                                    // 16 x 1024 B activation codes
constexpr int kStWOff = kTolBlocks * 1024;                    // 2 x 4352 B weight blocks
constexpr int kStTOff = kStWOff + 2 * kBlockBytes;            // 16 x 64 B (scale, sum) tails
constexpr int kStBytes = ((kStTOff + kTolBlocks * 64 + 1023) / 1024) * 1024;
constexpr int kAOff = kTolStages * kStBytes;                  // A images
constexpr int kABytes = kTolRows * 128;
constexpr int kScalOff = kAOff + kTolASlots * kABytes;        // scale ring
constexpr int kScalBytes = kTolRows * 8 + kTolTok * 8;        // rows' (ws, wz), tokens' xs[], xsum[]
constexpr int kBarOff = kScalOff + kTolScal * kScalBytes;
constexpr size_t kTolSmem = (size_t)kBarOff + 512 + 1024;     // + alignment slack
static_assert(kStBytes % 1024 == 0 && kAOff % 1024 == 0, "stage alignment");

constexpr uint32_t kMagic = 0x4B400000u;  // 12582912.0f: (magic + dot) read as f32 is exact
// Instruction descriptor: D s32 (bits 4-5 = 2), A u8 (7-9 = 0), B s8
// (10-12 = 1), both K-major, N = 128 (bits 17-22 = N >> 3), M = 128
// (bits 24-28 = M >> 4).
constexpr uint32_t kIdesc = (2u << 4) | (1u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
constexpr int kMaxSplit = 8;
constexpr int kPartBytes = kTolRows * kTolTok * 4;  // one item's partial sums

struct TolParams {
  const uint8_t* w;    // mma.sync 4-bit blocks ([64-row tile][group] of kBlockBytes)
  const uint8_t* act;  // quantized activations ([8-token block][group] of kActBlockBytes)
  float* out;
  const float* bias;
  const float* residual;
  uint32_t* err;
  const int* m_dev;
  float* part;         // split-K partial sums (ws_slots x kPartBytes), may be null
  unsigned* counter;   // per (tile, chunk, epilogue warp) arrival counters (zero between launches)
  int ws_slots;
  int rows, groups, M, ld_out, mode;
  int tiles;    // 128-row tiles
  int tiles64;  // 64-row blocks of the packed weights
};

struct TolRun {
  int mact, chunks, S, per, items;
};

__device__ __forceinline__ TolRun tol_run(const TolParams& p, int mact) {
  TolRun r;
  r.mact = mact;
  r.chunks = (mact + kTolTok - 1) / kTolTok;
  const int base = p.tiles * r.chunks;
  int S = 1;
  if (base > 0 && p.part) {
    S = (int)gridDim.x / base;
    S = min(S, kMaxSplit);
    S = min(S, p.groups / 4);
    if (S < 1) S = 1;
    if (base * S > p.ws_slots) S = 1;
  }
  r.per = (p.groups + S - 1) / S;
  r.S = (p.groups + r.per - 1) / r.per;  // no empty range
  r.items = base * r.S;
  return r;
}

struct TolItem {
  int tile, chunk, split, t0, nt, g0, g1;
};

// item = ((split * chunks) + chunk) * tiles + tile: CTA b < tiles starts at
// (tile b, chunk 0, split 0), whose first groups it may prefetch.
__device__ __forceinline__ bool tol_item(const TolParams& p, const TolRun& r, int item, TolItem* it) {
  if (item >= r.items) return false;
  it->tile = item % p.tiles;
  const int rest = item / p.tiles;
  it->chunk = rest % r.chunks;
  it->split = rest / r.chunks;
  it->t0 = it->chunk * kTolTok;
  it->nt = min(kTolTok, r.mact - it->t0);
  it->g0 = it->split * r.per;
  it->g1 = min(p.groups, it->g0 + r.per);
  return true;
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major descriptor without swizzle: 8-row x 16-byte core matrices, `lbo`
// between K chunks, `sbo` between 8-row groups; version 1 (sm_100).
__device__ __forceinline__ uint64_t desc_plain(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// K-major, 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart
// (SBO), LBO unused (1), layout type 2; a K offset inside the row is added
// to the start address.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t"
      "}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(1u)
      : "memory");
}

__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tm_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tm_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The magic seed into 32 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tm_seed32(uint32_t taddr) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
      "r"(kMagic)
      : "memory");
}
__device__ __forceinline__ void tm_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint64_t pk(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 unpk(uint64_t v) {
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
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Bounded wait (about a second of SM clock), no suspend hint.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, uint32_t* err) {
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

// Expand one 16-byte slot of 4-bit words into the two 16-byte K chunks it
// covers: word j's low nibbles are columns 8j..8j+3 of the slot's 32-byte
// span in the activation order, its high nibbles 8j+4..8j+7.
__device__ __forceinline__ void expand_slot(const uint4 w, uint4& c0, uint4& c1) {
  c0 = make_uint4(w.x & 0x0F0F0F0Fu, (w.x >> 4) & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu);
  c1 = make_uint4(w.z & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu, (w.w >> 4) & 0x0F0F0F0Fu);
}

__global__ void __launch_bounds__(kTolThreads, 1) gemm_tol_kernel(TolParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);  // stage landed
  uint64_t* sfree = full + kTolStages;                             // stage consumed (converters + MMAs)
  uint64_t* cvt = sfree + kTolStages;                              // A image built
  uint64_t* afree = cvt + kTolASlots;                              // A image's MMAs complete
  uint64_t* qfull = afree + kTolASlots;                            // scale slot written
  uint64_t* qdone = qfull + kTolScal;                              // scale slot read
  uint64_t* dfull = qdone + kTolScal;                              // TMEM slot's MMAs complete
  uint64_t* dempty = dfull + kTolSlots;                            // TMEM slot read and re-seeded
  uint64_t* mdone = dempty + kTolSlots;                            // every MMA of the CTA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.groups;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTolStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&sfree[s], kConvWarps + 1);
    }
    for (int a = 0; a < kTolASlots; ++a) {
      mbar_init(&cvt[a], kConvWarps);
      mbar_init(&afree[a], 1);
    }
    for (int r = 0; r < kTolScal; ++r) {
      mbar_init(&qfull[r], kConvWarps);
      mbar_init(&qdone[r], 8);
    }
    for (int d = 0; d < kTolSlots; ++d) {
      mbar_init(&dfull[d], 1);
      mbar_init(&dempty[d], 8);
    }
    mbar_init(mdone, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTolCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  // Weights do not depend on the previous kernel: a lead CTA (its first item
  // is (tile blockIdx.x, chunk 0, split 0) whenever there is a token)
  // requests its first groups' weight blocks before waiting on it.
  const bool lead = (int)blockIdx.x < p.tiles;
  const int pre = lead ? min(min(kTolStages, G), 4) : 0;
  auto w4_bytes = [&](int tile) { return (uint32_t)kBlockBytes * (2 * tile + 1 < p.tiles64 ? 2u : 1u); };
  auto issue_w4 = [&](int tile, int g, uint8_t* st, uint64_t* bar) {
    bulk_g2s(st + kStWOff, p.w + ((size_t)(2 * tile) * G + g) * kBlockBytes, kBlockBytes, bar);
    if (2 * tile + 1 < p.tiles64)
      bulk_g2s(st + kStWOff + kBlockBytes, p.w + ((size_t)(2 * tile + 1) * G + g) * kBlockBytes, kBlockBytes, bar);
  };
  if (warp == 0 && lane == 0) {
    for (int q = 0; q < pre; ++q) {
      mbar_expect_tx(&full[q], w4_bytes(blockIdx.x));
      issue_w4(blockIdx.x, q, smem + q * kStBytes, &full[q]);
    }
  }
  pdl_wait_prior();
  const TolRun run = tol_run(p, p.m_dev ? *p.m_dev : p.M);
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- producer ----------------
    bool ok = true, first = true;
    uint32_t k = 0;
    TolItem it;
    for (int item = blockIdx.x; ok && tol_item(p, run, item, &it); item += gridDim.x, first = false) {
      const int nb = (it.nt + kActBlockTok - 1) / kActBlockTok;
      for (int g = it.g0; g < it.g1; ++g, ++k) {
        const int s = k % kTolStages;
        const uint32_t n = k / kTolStages;
        if (n > 0 && !__all_sync(0xffffffffu, wait_bar(&sfree[s], (n - 1) & 1, p.err))) { ok = false; break; }
        uint8_t* st = smem + s * kStBytes;
        const bool prefetched = first && lead && g < pre;
        if (lane == 0) {
          const uint32_t abytes = (uint32_t)nb * (1024 + 64);
          mbar_arrive_expect_tx(&full[s], prefetched ? abytes : w4_bytes(it.tile) + abytes);
          if (!prefetched) issue_w4(it.tile, g, st, &full[s]);
        }
        __syncwarp();
        const int b = lane & 15;
        if (b < nb) {
          const uint8_t* blk = p.act + ((size_t)((it.t0 >> 3) + b) * G + g) * kActBlockBytes;
          if (lane < 16) bulk_g2s(st + kStBOff + b * 1024, blk, 1024, &full[s]);
          else bulk_g2s(st + kStTOff + b * 64, blk + 1024, 64, &full[s]);
        }
      }
    }
    if (lane == 0) {
      if (k == 0) {
        // No item (no tokens): the prefetched stages still land before exit.
        for (int q = 0; q < pre; ++q) {
          mbar_arrive(&full[q]);
          wait_bar(&full[q], 0, nullptr);
        }
      } else {
        // Every fill this CTA issued lands before the CTA exits (bounded;
        // only matters after a timeout).
        for (uint32_t j = k > kTolStages ? k - kTolStages : 0; j < k; ++j)
          wait_bar(&full[j % kTolStages], (j / kTolStages) & 1, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t sbase = smem_u32(smem);
      uint32_t k = 0;
      bool ok = true;
      TolItem it;
      for (int item = blockIdx.x; ok && tol_item(p, run, item, &it); item += gridDim.x) {
        for (int g = it.g0; g < it.g1; ++g, ++k) {
          const int s = k % kTolStages, a = k % kTolASlots, d = k % kTolSlots;
          if (!wait_bar(&full[s], (k / kTolStages) & 1, p.err) || !wait_bar(&cvt[a], (k / kTolASlots) & 1, p.err) ||
              !wait_bar(&dempty[d], (k / kTolSlots) & 1, p.err)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t a0 = sbase + kAOff + a * kABytes, b0 = sbase + s * kStBytes + kStBOff;
#pragma unroll
          for (int m = 0; m < 4; ++m)
            mma_i8(tmem + d * 128, desc_plain(a0 + m * 4096, 2048, 128), desc_sw128(b0 + m * 32));
          commit(&dfull[d]);
          commit(&sfree[s]);
          commit(&afree[a]);
        }
      }
      // Drain: every MMA issued above completes before TMEM is released.
      commit(mdone);
      wait_bar(mdone, 0, nullptr);
    }
  } else if (warp < 2 + kConvWarps) {
    // ---------------- converters: two weight rows / tokens each ----------------
    const int r0 = threadIdx.x - 64;
    uint32_t k = 0;
    bool ok = true;
    TolItem it;
    for (int item = blockIdx.x; ok && tol_item(p, run, item, &it); item += gridDim.x) {
      const int nb = (it.nt + kActBlockTok - 1) / kActBlockTok;
      for (int g = it.g0; g < it.g1; ++g, ++k) {
        const int s = k % kTolStages, a = k % kTolASlots, q = k % kTolScal;
        const uint32_t an = k / kTolASlots, qn = k / kTolScal;
        if (!__all_sync(0xffffffffu, wait_bar(&full[s], (k / kTolStages) & 1, p.err) &&
                                         (an == 0 || wait_bar(&afree[a], (an - 1) & 1, p.err)) &&
                                         (qn == 0 || wait_bar(&qdone[q], (qn - 1) & 1, p.err)))) {
          ok = false;
          break;
        }
        const uint8_t* st = smem + s * kStBytes;
        uint8_t* sq = smem + kScalOff + q * kScalBytes;
#pragma unroll
        for (int rr = 0; rr < kTolRows / (32 * kConvWarps); ++rr) {
          const int r = r0 + rr * 32 * kConvWarps;
          // Weight row r: 64 bytes of 4-bit slots -> 8 K chunks of u8.
          const uint8_t* wrow = st + kStWOff + (r >> 6) * kBlockBytes + (r & 63) * kRowGroupBytes;
          uint8_t* arow = smem + kAOff + a * kABytes + (r >> 3) * 128 + (r & 7) * 16;
#pragma unroll
          for (int sl = 0; sl < 4; ++sl) {
            uint4 c0, c1;
            expand_slot(*reinterpret_cast<const uint4*>(wrow + sl * 16), c0, c1);
            *reinterpret_cast<uint4*>(arow + (2 * sl) * 2048) = c0;
            *reinterpret_cast<uint4*>(arow + (2 * sl + 1) * 2048) = c1;
          }
          // Scales: row r's (w_scale, w_zero), token r's (x_scale, x_sum).
          const uint32_t pw = *reinterpret_cast<const uint32_t*>(st + kStWOff + (r >> 6) * kBlockBytes +
                                                                kWeightStageBytes + (r & 63) * 4);
          reinterpret_cast<float2*>(sq)[r] =
              make_float2(f16_bits_to_f32((uint16_t)(pw & 0xFFFF)), f16_bits_to_f32((uint16_t)(pw >> 16)));
          float2 xs = make_float2(0.f, 0.f);
          if ((r >> 3) < nb) xs = reinterpret_cast<const float2*>(st + kStTOff + (r >> 3) * 64)[r & 7];
          reinterpret_cast<float*>(sq + kTolRows * 8)[r] = xs.x;
          reinterpret_cast<float*>(sq + kTolRows * 8 + kTolTok * 4)[r] = xs.y;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&cvt[a]);
          mbar_arrive(&qfull[q]);
          mbar_arrive(&sfree[s]);
        }
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int quad = warp & 3, h = (warp - 2 - kConvWarps) >> 2;
    const int rl = 32 * quad + lane;  // row within the tile = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(32 * quad) << 16) + 64 * h;
    const uint64_t magic2 = pk(12582912.0f, 12582912.0f);
    // Seed this warp's columns of every slot, then release the slots for
    // their first MMAs (phase 0 of dempty).
#pragma unroll
    for (int d = 0; d < kTolSlots; ++d) {
      tm_seed32(lane_base + d * 128);
      tm_seed32(lane_base + d * 128 + 32);
    }
    tm_wait_st();
    fence_before();
    __syncwarp();
    if (lane == 0)
      for (int d = 0; d < kTolSlots; ++d) mbar_arrive(&dempty[d]);
    uint32_t k = 0;
    bool ok = true;
    TolItem it;
    for (int item = blockIdx.x; ok && tol_item(p, run, item, &it); item += gridDim.x) {
      const int ntl = min(64, it.nt - 64 * h);  // this warp's tokens of the item (none if <= 0)
      uint64_t acc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = 0ull;
      for (int g = it.g0; g < it.g1; ++g, ++k) {
        const int d = k % kTolSlots, q = k % kTolScal;
        if (!wait_bar(&dfull[d], (k / kTolSlots) & 1, p.err) || !wait_bar(&qfull[q], (k / kTolScal) & 1, p.err)) {
          ok = false;
          break;
        }
        fence_after();
        const uint8_t* sq = smem + kScalOff + q * kScalBytes;
        const float2 wsz = reinterpret_cast<const float2*>(sq)[rl];
        const uint64_t ws2 = pk(wsz.x, wsz.x), wz2 = pk(wsz.y, wsz.y);
        const float* xsv = reinterpret_cast<const float*>(sq + kTolRows * 8) + 64 * h;
        const float* xsumv = reinterpret_cast<const float*>(sq + kTolRows * 8 + kTolTok * 4) + 64 * h;
        const uint32_t col = lane_base + d * 128;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t v[32];
          tm_ld32(col + 32 * half, v);
          tm_wait_ld();
          tm_seed32(col + 32 * half);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int t = 32 * half + 2 * i;
            if (t >= ntl) break;  // warp-uniform
            const float2 xs = *reinterpret_cast<const float2*>(xsv + t);
            const float2 xz = *reinterpret_cast<const float2*>(xsumv + t);
            const uint64_t dot = sub2(pk(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])), magic2);
            uint64_t a2 = fma2(dot, mul2(ws2, pk(xs.x, xs.y)), acc[16 * half + i]);
            acc[16 * half + i] = fma2(wz2, pk(xz.x, xz.y), a2);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&qdone[q]);
        tm_wait_st();
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dempty[d]);
      }
      if (!ok) break;
      const int row = it.tile * kTolRows + rl;
      if (run.S == 1) {
        if (row < p.rows) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (2 * i >= ntl) break;
            const float2 v2 = unpk(acc[i]);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              if (2 * i + e >= ntl) break;
              float v = e ? v2.y : v2.x;
              const size_t o = (size_t)(it.t0 + 64 * h + 2 * i + e) * p.ld_out + row;
              if (p.mode == kEpiBias) v += p.bias[row];
              else if (p.mode == kEpiResidual) v = p.residual[o] + v;
              p.out[o] = v;
            }
          }
        }
        continue;
      }
      // Split-K: this range's partial sums, then whichever CTA finishes a
      // warp's slice last adds the ranges in order. Each epilogue warp has
      // its own arrival counter per (tile, chunk), so no barrier spans warps.
      float* part = p.part + (size_t)item * (kPartBytes / 4) + (size_t)rl * kTolTok + 64 * h;
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        if (2 * i >= ntl) break;
        const float2 a0 = unpk(acc[i]), a1 = unpk(acc[i + 1]);
        *reinterpret_cast<float4*>(part + 2 * i) = make_float4(a0.x, a0.y, a1.x, a1.y);
      }
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        unsigned* cnt = p.counter + (size_t)(it.tile + it.chunk * p.tiles) * 8 + (warp - 2 - kConvWarps);
        last = atomicAdd(cnt, 1u) == (unsigned)(run.S - 1);
        if (last) *cnt = 0u;  // ready for the next launch
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last || ntl <= 0) continue;
      __threadfence();
      if (row >= p.rows) continue;
      for (int t = 0; t < ntl; t += 4) {
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int sp = 0; sp < run.S; ++sp) {
          const int src = ((sp * run.chunks) + it.chunk) * p.tiles + it.tile;
          const float4 v = __ldcg(reinterpret_cast<const float4*>(p.part + (size_t)src * (kPartBytes / 4) +
                                                                  (size_t)rl * kTolTok + 64 * h + t));
          sum.x += v.x;
          sum.y += v.y;
          sum.z += v.z;
          sum.w += v.w;
        }
        const float sv[4] = {sum.x, sum.y, sum.z, sum.w};
        for (int e = 0; e < 4 && t + e < ntl; ++e) {
          float v = sv[e];
          const size_t o = (size_t)(it.t0 + 64 * h + t + e) * p.ld_out + row;
          if (p.mode == kEpiBias) v += p.bias[row];
          else if (p.mode == kEpiResidual) v = p.residual[o] + v;
          p.out[o] = v;
        }
      }
    }
  }

  // Teardown: every role is done with TMEM (the MMA issuer drained its
  // MMAs, the epilogue waited for its loads and stores); release the columns.
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTolCols) : "memory");
  }
}

}  // namespace

size_t gemm_tol_workspace_bytes() {
  return (size_t)device_sm_count() * kPartBytes + (size_t)device_sm_count() * 8 * sizeof(unsigned);
}

cudaError_t init_gemm_tol_attributes() {
  return cudaFuncSetAttribute(gemm_tol_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTolSmem);
}

cudaError_t gemm_tol(const PackedLinear& w, const ActBuf& act, int M, float* out, int ld_out,
                     const GemmEpilogue& epi, uint32_t* err, cudaStream_t s, const int* m_dev, void* ws,
                     size_t ws_bytes) {
  if (w.wbits != 4 || M <= 0) return cudaErrorInvalidValue;
  TolParams p = {};
  p.w = w.data;
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
  p.tiles = (int)ceil_div(w.rows, kTolRows);
  p.tiles64 = w.tiles;
  const int sms = device_sm_count();
  if (ws && ws_bytes >= gemm_tol_workspace_bytes()) {
    p.part = static_cast<float*>(ws);
    p.counter = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + (size_t)sms * kPartBytes);
    p.ws_slots = sms;
  }
  // One persistent wave: at most one CTA per SM (the TMEM allocation takes
  // all 512 columns), never more than the static budget's items.
  const long chunks = (long)ceil_div(M, kTolTok);
  const long most = (long)p.tiles * chunks * (p.part ? kMaxSplit : 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(most < sms ? most : sms));
  cfg.blockDim = dim3(kTolThreads);
  cfg.dynamicSmemBytes = kTolSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_tol_kernel, p);
}

}  // namespace rai
