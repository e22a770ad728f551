// Model-writing helpers of the oracle (TEST INFRASTRUCTURE ONLY).
//
// The reference-side arm of bench.py writes its synthetic .raimodel inputs
// with these, so that it loads no code of the product library:
//   * orc_rtn_quantize restates `rai convert`'s round-to-nearest quantizer
//     (quantize_row, rai-infer/src/convert.rs:2551-2639): per (row, group)
//     f64 min / max, scale = max((max - min) / levels, 2^-24) rounded to f16
//     (convert.rs:44 MIN_F16_SCALE), zero = f16(min), both rounded before any
//     code is derived; code = clamp(round_half_even((w - zero) / scale), 0,
//     levels); 4-bit codes packed low nibble = even column (write_matrix,
//     convert.rs:2466-2545).
//   * orc_synth_normal_f16 is the seeded N(0, std) weight source of the
//     synthetic models (splitmix64 words, Box-Muller pairs, each value rounded
//     through f16 as a checkpoint cast does, rai-infer/src/safetensors.rs:
//     457-477). It is not reference code: it only has to draw the same values
//     as the product's writer, so both bench arms see byte-identical files
//     (tests/test_bench_host.py checks the two writers against each other).
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

#include "rai_oracle.h"

namespace {

// binary64 -> binary16, round to nearest even (half::f16::from_f64).
uint16_t to_f16(double x) {
  uint64_t b;
  std::memcpy(&b, &x, 8);
  const uint16_t sign = (uint16_t)((b >> 48) & 0x8000u);
  const uint64_t mag = b & 0x7FFFFFFFFFFFFFFFull;
  if (mag >= 0x7FF0000000000000ull) return (uint16_t)(sign | (mag > 0x7FF0000000000000ull ? 0x7E00u : 0x7C00u));
  const int exp = (int)(mag >> 52) - 1023;
  if (exp < -26) return sign;  // below half of the least subnormal: rounds to zero
  const uint64_t mant = (mag & ((1ull << 52) - 1)) | (1ull << 52);
  // Keep 11 significant bits for normals, fewer for subnormals (exp < -14).
  const int drop = exp >= -14 ? 42 : 42 + (-14 - exp);
  uint64_t q = mant >> drop;
  const uint64_t rest = mant & ((1ull << drop) - 1), half = 1ull << (drop - 1);
  q += (rest > half || (rest == half && (q & 1))) ? 1 : 0;
  if (exp >= -14) {
    const uint32_t bits = ((uint32_t)(exp + 15) << 10) + (uint32_t)(q - 1024);
    return (uint16_t)(sign | (bits >= 0x7C00u ? 0x7C00u : bits));
  }
  return (uint16_t)(sign | q);  // subnormal (a carry into 0x400 is the least normal)
}

double from_f16(uint16_t h) {
  const int e = (h >> 10) & 0x1F, m = h & 0x3FF;
  double v = e == 0 ? std::ldexp((double)m, -24) : e == 31 ? (m ? NAN : INFINITY) : std::ldexp((double)(m | 0x400), e - 25);
  return (h & 0x8000) ? -v : v;
}

uint64_t mix_next(uint64_t& state) {
  uint64_t z = (state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace

extern "C" {

int orc_rtn_quantize(const float* w, size_t rows, size_t cols, int bits, size_t gs, uint8_t* params,
                     uint8_t* codes) {
  if (!w || !params || !codes || !rows || !cols || !gs || (bits != 4 && bits != 8) || (bits == 4 && cols % 2))
    return -1;
  const size_t ng = (cols + gs - 1) / gs, row_code_bytes = bits == 4 ? cols / 2 : cols;
  const double levels = (double)((1 << bits) - 1);
  int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
  for (size_t r = 0; r < rows; ++r) {
    const float* x = w + r * cols;
    uint8_t* pr = params + r * ng * 4;
    uint8_t* cr = codes + r * row_code_bytes;
    if (bits == 4) std::memset(cr, 0, row_code_bytes);
    for (size_t g = 0; g < ng && !bad; ++g) {
      const size_t c0 = g * gs, c1 = std::min(cols, c0 + gs);
      double lo = INFINITY, hi = -INFINITY;
      for (size_t c = c0; c < c1; ++c) {
        const double v = x[c];
        if (!std::isfinite(v)) { bad = 1; break; }
        lo = std::min(lo, v);
        hi = std::max(hi, v);
      }
      if (bad) break;
      const uint16_t s16 = to_f16(std::max((hi - lo) / levels, 5.960464477539063e-8));
      const uint16_t z16 = to_f16(lo);
      const double s = from_f16(s16), z = from_f16(z16);
      if (!(std::isfinite(s) && s > 0.0 && std::isfinite(z))) { bad = 1; break; }
      std::memcpy(pr + g * 4, &s16, 2);
      std::memcpy(pr + g * 4 + 2, &z16, 2);
      for (size_t c = c0; c < c1; ++c) {
        const double q = std::min(std::max(std::nearbyint(((double)x[c] - z) / s), 0.0), levels);
        const uint8_t code = (uint8_t)q;
        if (bits == 8) cr[c] = code;
        else cr[c / 2] |= (uint8_t)((c & 1) ? (code << 4) : (code & 0x0F));
      }
    }
  }
  return bad ? -1 : 0;
}

int orc_synth_normal_f16(uint64_t seed, uint64_t stream, size_t n, float stddev, float* out) {
  if (!out && n) return -1;
  const size_t block = 1 << 16, nb = (n + block - 1) / block;
#pragma omp parallel for schedule(static)
  for (size_t bi = 0; bi < nb; ++bi) {
    uint64_t st = seed * 0x9E3779B97F4A7C15ull ^ (stream + 1) * 0xD1B54A32D192ED03ull ^ (bi + 1) * 0x8CB92BA72F3D8DD7ull;
    mix_next(st);
    const size_t end = std::min(n, (bi + 1) * block);
    for (size_t i = bi * block; i < end; i += 2) {
      const double u1 = (double)((mix_next(st) >> 11) + 1) * (1.0 / 9007199254740992.0);
      const double u2 = (double)(mix_next(st) >> 11) * (1.0 / 9007199254740992.0);
      const double rad = std::sqrt(-2.0 * std::log(u1)), ang = 6.283185307179586 * u2;
      out[i] = (float)from_f16(to_f16((double)(float)(rad * std::cos(ang) * stddev)));
      if (i + 1 < end) out[i + 1] = (float)from_f16(to_f16((double)(float)(rad * std::sin(ang) * stddev)));
    }
  }
  return 0;
}

}  // extern "C"
