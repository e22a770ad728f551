// Shared device helpers for the sm_100a decode kernels.
//
// Numerics rule for every kernel in this library: the reference is Rust,
// which never contracts a*b+c into an FMA, while nvcc does by default. Every
// parity-critical expression is therefore written with explicit
// round-to-nearest intrinsics (__fmul_rn, __fadd_rn, __fmaf_rn, __fdiv_rn,
// __fsqrt_rn) exactly where the reference multiplies, adds, fuses, divides
// or takes a square root.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rai {

// Device-side error word (per model context): bit 0 = a bounded wait gave up.
enum : uint32_t { kErrWaitTimeout = 1u, kErrBadInput = 2u };

// A wait on an mbarrier gives up after kMaxPolls polls; each poll suspends
// the warp in hardware until the phase completes or kSuspendNs elapse, so the
// bound is ~0.5 s, after which the wait reports kErrWaitTimeout instead of
// hanging the GPU.
constexpr uint32_t kSuspendNs = 64 * 1024;
constexpr uint32_t kMaxPolls = 8192;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and sets the error word) if the phase never
// completes. Callers stop issuing work after a false return.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  for (uint32_t i = 0; i < kMaxPolls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicOr(err, kErrWaitTimeout);
  return false;
}

// TMA bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 16-byte asynchronous copy global -> shared (both addresses 16-byte
// aligned), completing with the thread's next commit group.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's commit groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Stage n floats of global memory in shared memory, cooperatively (thread
// `tid` of `nthr`): 16-byte asynchronous copies when both ends are 16-byte
// aligned and n is a multiple of 4, so every copy is in flight at once;
// otherwise plain loads, four per thread issued before their stores. The
// caller completes the staging with cp_async_wait<0>() and a barrier.
__device__ __forceinline__ void stage_f32(float* dst, const float* src, int n, int tid, int nthr) {
  if (((reinterpret_cast<uintptr_t>(src) | (uintptr_t)smem_u32(dst)) & 15u) == 0 && (n & 3) == 0) {
    for (int i = 4 * tid; i < n; i += 4 * nthr) cp_async16(dst + i, src + i);
  } else {
    for (int i = tid; i < n; i += 4 * nthr) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = i + u * nthr < n ? src[i + u * nthr] : 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i + u * nthr < n) dst[i + u * nthr] = v[u];
    }
  }
  cp_async_commit();
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous kernel's results before reading them.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// SM count of the current device (cached per device).
inline int device_sm_count() {
  static int n[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!n[dev] && cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n[dev] = 148;
  return n[dev];
}

// Grid size for kernels that loop over their (device-counted) rows or
// segments: the static budget `want`, capped at about two waves of CTAs so
// that a budget far above the active count does not launch idle CTAs.
inline int grid_cap(int want, int per_sm = 2) {
  const int cap = per_sm * device_sm_count();
  return want < cap ? (want > 0 ? want : 1) : cap;
}

// Launch with programmatic stream serialization: the kernel may be scheduled
// while the previous kernel in the stream still runs. Every kernel of this
// library therefore calls pdl_wait_prior() before reading anything an earlier
// kernel wrote (and before exiting), so results are as if serialized.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Exact IEEE half -> float (F16C _mm_cvtph_ps / half::f16::to_f32).
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// 8-lane horizontal sum of the reference (hi+lo, movehdup, add, movehl,
// add_ss): ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)).
__device__ __forceinline__ float hsum8(const float a[8]) {
  float s0 = __fadd_rn(a[0], a[4]), s1 = __fadd_rn(a[1], a[5]);
  float s2 = __fadd_rn(a[2], a[6]), s3 = __fadd_rn(a[3], a[7]);
  return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

// Schraudolph exp of silu_mul_avx2 / attention_head_avx2
// (rai-infer/src/layers.rs:862-869, 1330-1337): bits = cvt_rne(clamp(a*x+b)).
__device__ __forceinline__ float schraudolph(float x) {
  float t = __fadd_rn(__fmul_rn(12102203.0f, x), 1065353216.0f - 486411.0f);
  // _mm256_max_ps(_mm256_min_ps(t, hi), lo): NaN t yields hi then hi.
  t = (t < 2139095040.0f) ? t : 2139095040.0f;
  t = (t > 0.0f) ? t : 0.0f;
  return __int_as_float(__float2int_rn(t));
}

// Rust f32::exp resolves to the host libm's expf. The device evaluates exp in
// double and rounds once (correctly rounded), then patches the inputs where
// the host expf rounds differently, from a table generated at build time by
// running that expf over every binary32 input (csrc/gen_expf_table.c).
struct ExpfTable {
  const uint32_t* keys = nullptr;   // sorted input bit patterns
  const uint32_t* vals = nullptr;   // host expf result bits
  const uint32_t* start = nullptr;  // [kExpfBuckets + 1] key ranges by top 16 bits
  int n = 0;
};
constexpr int kExpfBuckets = 1 << 16;

__device__ __forceinline__ float expf_host(float x, const ExpfTable& t) {
  const float r = (float)exp((double)x);
  const uint32_t k = __float_as_uint(x);
  int lo = (int)__ldg(t.start + (k >> 16)), hi = (int)__ldg(t.start + (k >> 16) + 1) - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    const uint32_t v = __ldg(t.keys + mid);
    if (v == k) return __uint_as_float(__ldg(t.vals + mid));
    if (v < k) lo = mid + 1; else hi = mid - 1;
  }
  return r;
}

}  // namespace rai
