// Tensor-parallel exchange between the GPUs of one model (one process per
// GPU, NVLink peer memory mapped through CUDA IPC).
//
// The split keeps the reference's arithmetic exactly: every linear is
// column-parallel (each rank computes whole output rows over the full
// input), so no dot product or lane accumulation is ever split. Ranks swap
// what the next linear needs in full:
//   * the quantized attention output (each rank quantizes its heads' groups)
//     and the quantized SwiGLU output (each rank its ff groups), written as
//     int8 activation blocks straight into every rank's buffer;
//   * the o / down projection rows (hidden slices), written by the GEMM
//     epilogue straight into every rank's hidden state;
//   * the LM head's per-row argmax keys (atomicMax into every rank).
// Each exchange has a flag slot on every rank. Producers store to the peers
// and fence at system scope; the consumer kernel's CTA 0, once its producer
// grid has finished (griddepcontrol.wait), adds 1 to that slot on every
// rank, and every consumer CTA waits until its own slot reaches
// world x (forwards so far that used it). Slot counters only grow, so no
// reset is ever needed between steps. Waits are bounded: a rank that never
// arrives turns into a timeout status, not a hang.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace rai {

constexpr int kMaxTp = 8;

// Poll bound of a cross-GPU wait: about kTpMaxPolls x 1 us.
constexpr uint32_t kTpMaxPolls = 1u << 20;

// Exchange slots per forward: four per layer plus the logits.
enum : int { kXchActQ = 0, kXchHiddenO = 1, kXchActFF = 2, kXchHiddenDown = 3, kXchPerLayer = 4 };

struct TpLink {
  int world = 1;
  int rank = 0;
  unsigned long long* flags[kMaxTp] = {};  // every rank's slot array (same layout)
  const uint32_t* epoch = nullptr;          // this rank: [0] forwards, [1] forwards with logits
};

__device__ __forceinline__ void tp_signal(const TpLink& t, int slot) {
  __threadfence_system();
  for (int r = 0; r < t.world; ++r)
    asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(t.flags[r] + slot) : "memory");
}

__device__ __forceinline__ bool tp_wait(const TpLink& t, int slot, int which, uint32_t* err) {
  // A wait of this forward already gave up: the peers are not coming, so
  // later exchanges fail at once instead of each waiting out its bound.
  if (err && (*reinterpret_cast<volatile uint32_t*>(err) & kErrWaitTimeout)) return false;
  const unsigned long long target = (unsigned long long)t.epoch[which] * (unsigned long long)t.world;
  const unsigned long long* f = t.flags[t.rank] + slot;
  for (uint32_t i = 0; i < kTpMaxPolls; ++i) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
    if (v >= target) return true;
    __nanosleep(i < 64 ? 64 : 1000);
  }
  if (err) atomicOr(err, kErrWaitTimeout);
  return false;
}

// Consumer side of an exchange, called by every thread of a CTA after
// griddepcontrol.wait: CTA (0,0) signals, thread 0 of each CTA waits.
// Returns false (for the whole CTA) if the wait timed out.
__device__ __forceinline__ bool tp_exchange(const TpLink& t, int slot, int which, uint32_t* err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    if (blockIdx.x == 0 && blockIdx.y == 0) tp_signal(t, slot);
    s_ok = tp_wait(t, slot, which, err) ? 1 : 0;
  }
  __syncthreads();
  return s_ok != 0;
}

// Destinations of a quantized activation: the same buffer layout (groups
// per token) on every rank; this kernel's group g lands at group g + g_off.
struct ActDst {
  uint8_t* data[kMaxTp] = {};
  int n = 1;
  int groups = 0;
  int g_off = 0;
};

}  // namespace rai
