// Host-side RTN quantizer and seeded weight source for producing .raimodel
// files (the `rai convert` restatement's hot loop, rai-infer/src/convert.rs:
// 2551-2639), multi-threaded. Byte-identical to rai_b200/convert.py's numpy
// quantizer (tests/test_convert_golden.py checks both).
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/rai_gpu.h"
#include "raimodel_format.h"

namespace {

// IEEE binary64 -> binary16, round to nearest even (half::f16::from_f64,
// numpy's float64 -> float16 cast).
uint16_t f64_to_f16(double x) {
  uint64_t b;
  std::memcpy(&b, &x, 8);
  uint16_t sign = (uint16_t)((b >> 48) & 0x8000u);
  uint64_t a = b & 0x7FFFFFFFFFFFFFFFull;
  if (a >= 0x7FF0000000000000ull) return a > 0x7FF0000000000000ull ? (uint16_t)(sign | 0x7E00u) : (uint16_t)(sign | 0x7C00u);
  if ((a >> 52) == 0) return sign;  // zero or binary64 subnormal: far below half of the least f16
  int e = (int)(a >> 52) - 1023;
  uint64_t m = (a & ((1ull << 52) - 1)) | (1ull << 52);
  int shift = e >= -14 ? 42 : 42 + (-14 - e);
  if (shift > 63) return sign;
  uint64_t q = m >> shift, rem = m & ((1ull << shift) - 1), half = 1ull << (shift - 1);
  if (rem > half || (rem == half && (q & 1))) ++q;
  if (e >= -14) {
    uint32_t bits = ((uint32_t)(e + 15) << 10) + (uint32_t)(q - 1024);
    if (bits >= 0x7C00u) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | bits);
  }
  return (uint16_t)(sign | (uint16_t)q);
}

double f16_to_f64(uint16_t h) { return (double)raimodel::detail::f16_to_f32(h); }

constexpr double kMinF16Scale = 5.960464477539063e-8;  // convert.rs:44

// quantize_row: one row, all groups.
bool quantize_row(const float* row, size_t cols, size_t gs, double levels, bool packed, uint8_t* params,
                  uint8_t* codes) {
  for (size_t g0 = 0, gi = 0; g0 < cols; g0 += gs, ++gi) {
    size_t g1 = std::min(cols, g0 + gs);
    double mn = INFINITY, mx = -INFINITY;
    for (size_t c = g0; c < g1; ++c) {
      double v = row[c];
      if (!std::isfinite(v)) return false;
      if (v <= mn) mn = v;
      if (v >= mx) mx = v;
    }
    double scale = std::max((mx - mn) / levels, kMinF16Scale);
    uint16_t s16 = f64_to_f16(scale), z16 = f64_to_f16(mn);
    double s64 = f16_to_f64(s16), z64 = f16_to_f64(z16);
    if (!std::isfinite(s64) || s64 <= 0.0 || !std::isfinite(z64)) return false;
    std::memcpy(params + gi * 4, &s16, 2);
    std::memcpy(params + gi * 4 + 2, &z16, 2);
    for (size_t c = g0; c < g1; ++c) {
      double q = std::nearbyint(((double)row[c] - z64) / s64);  // ties to even (default rounding mode)
      q = std::min(std::max(q, 0.0), levels);
      uint8_t code = (uint8_t)q;
      if (packed) {
        uint8_t& byte = codes[c / 2];
        byte = (c % 2 == 0) ? (uint8_t)((byte & 0xF0) | (code & 0x0F)) : (uint8_t)((byte & 0x0F) | (code << 4));
      } else {
        codes[c] = code;
      }
    }
  }
  return true;
}

template <class F>
void parallel_for(size_t n, int threads, F f) {
  if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  if (threads == 1 || n < 2) {
    for (size_t i = 0; i < n; ++i) f(i);
    return;
  }
  std::vector<std::thread> pool;
  size_t per = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    size_t lo = t * per, hi = std::min(n, lo + per);
    if (lo >= hi) break;
    pool.emplace_back([=] { for (size_t i = lo; i < hi; ++i) f(i); });
  }
  for (auto& th : pool) th.join();
}

inline uint64_t splitmix64(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace

extern "C" {

// Quantize a [rows][cols] f32 matrix with the reference RTN rule. params gets
// rows * ceil(cols / gs) * 4 bytes; codes gets rows * cols / 2 (bits 4) or
// rows * cols (bits 8) bytes. Returns RAI_ERR_INVALID on a non-finite weight.
RAI_API int rai_rtn_quantize(const float* w, size_t rows, size_t cols, int bits, size_t gs, uint8_t* params,
                             uint8_t* codes, int threads) {
  if (!w || !params || !codes || rows == 0 || cols == 0 || gs == 0 || (bits != 4 && bits != 8)) return RAI_ERR_INVALID;
  if (bits == 4 && cols % 2) return RAI_ERR_INVALID;
  size_t ng = (cols + gs - 1) / gs;
  size_t cb = bits == 4 ? cols / 2 : cols;
  double levels = (double)((1 << bits) - 1);
  std::vector<char> ok(rows, 1);
  parallel_for(rows, threads, [&](size_t r) {
    ok[r] = quantize_row(w + r * cols, cols, gs, levels, bits == 4, params + r * ng * 4, codes + r * cb);
  });
  for (char o : ok)
    if (!o) return RAI_ERR_INVALID;
  return RAI_OK;
}

// n seeded N(0, std) values, each rounded through f16 (the checkpoint cast
// of rai-infer/src/safetensors.rs:457-477). Deterministic for a given
// (seed, stream) regardless of the thread count.
RAI_API int rai_synth_normal_f16(uint64_t seed, uint64_t stream, size_t n, float stddev, float* out, int threads) {
  if (!out) return RAI_ERR_INVALID;
  const size_t block = 1 << 16;
  size_t nb = (n + block - 1) / block;
  parallel_for(nb, threads, [&](size_t bi) {
    uint64_t s = seed * 0x9E3779B97F4A7C15ull ^ (stream + 1) * 0xD1B54A32D192ED03ull ^ (bi + 1) * 0x8CB92BA72F3D8DD7ull;
    splitmix64(s);
    size_t lo = bi * block, hi = std::min(n, lo + block);
    for (size_t i = lo; i < hi; i += 2) {
      // Box-Muller on two uniforms in (0, 1].
      double u1 = ((splitmix64(s) >> 11) + 1) * (1.0 / 9007199254740992.0);
      double u2 = (splitmix64(s) >> 11) * (1.0 / 9007199254740992.0);
      double r = std::sqrt(-2.0 * std::log(u1));
      double z0 = r * std::cos(6.283185307179586 * u2), z1 = r * std::sin(6.283185307179586 * u2);
      float v0 = (float)(z0 * stddev), v1 = (float)(z1 * stddev);
      out[i] = (float)raimodel::detail::f16_to_f32(f64_to_f16((double)v0));
      if (i + 1 < hi) out[i + 1] = (float)raimodel::detail::f16_to_f32(f64_to_f16((double)v1));
    }
  });
  return RAI_OK;
}

// binary64 -> binary16 (RNE), exported for the writer's self-test.
RAI_API int rai_f64_to_f16(const double* in, size_t n, uint16_t* out) {
  if (!in || !out) return RAI_ERR_INVALID;
  for (size_t i = 0; i < n; ++i) out[i] = f64_to_f16(in[i]);
  return RAI_OK;
}

}  // extern "C"
