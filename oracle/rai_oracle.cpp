// CPU oracle (TEST INFRASTRUCTURE ONLY): intrinsic-for-intrinsic restatement
// of rai-infer's AVX2/FMA/F16C hot path. Compile with
//   -O2 -mavx2 -mfma -mf16c -ffp-contract=off -fopenmp
// (Rust never contracts a*b+c into an FMA; -ffp-contract=off keeps C++ from
// doing it either). Scalar libm calls (expf, powf, cosf, sinf) are the glibc
// functions Rust's f32 methods resolve to on Linux.
//
// rayon's row-chunk parallelism is restated with OpenMP: row chunks, heads
// and tokens are independent, so the thread split never changes a result.
#include "rai_oracle.h"

#include <immintrin.h>
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../rai_b200/csrc/raimodel_format.h"

namespace {

constexpr size_t MAX_GROUPS = 128;
thread_local std::string g_err;

inline float read_f16(const uint8_t* p) {
  uint16_t b;
  std::memcpy(&b, p, 2);
  return raimodel::detail::f16_to_f32(b);
}

// 8-lane horizontal sum used throughout the reference:
// hi+lo, movehdup, add, movehl, add_ss.
inline float hsum8(__m256 acc) {
  __m128 hi = _mm256_extractf128_ps(acc, 1);
  __m128 lo = _mm256_castps256_ps128(acc);
  __m128 s = _mm_add_ps(lo, hi);
  __m128 shuf = _mm_movehdup_ps(s);
  __m128 s2 = _mm_add_ps(s, shuf);
  __m128 hi2 = _mm_movehl_ps(s2, s2);
  return _mm_cvtss_f32(_mm_add_ss(s2, hi2));
}

// compute_input_sums_avx2 (gemm.rs:182-212).
void input_sums(const float* inp, float* sums, size_t cols, size_t gs, size_t ng) {
  for (size_t g = 0; g < ng; ++g) {
    size_t start = g * gs, end = std::min((g + 1) * gs, cols), len = end - start;
    size_t chunks8 = len / 8;
    __m256 acc = _mm256_setzero_ps();
    for (size_t i = 0; i < chunks8; ++i) acc = _mm256_add_ps(acc, _mm256_loadu_ps(inp + start + i * 8));
    float total = hsum8(acc);
    for (size_t i = chunks8 * 8; i < len; ++i) total += inp[start + i];
    sums[g] = total;
  }
}

// Rust `(x).round().max(lo).min(hi) as i8`: round half away from zero.
inline int8_t scalar_q(float v, float lo, float hi) {
  float r = std::round(v);
  r = std::max(r, lo);
  r = std::min(r, hi);
  return (int8_t)r;
}

// quantize_input_split_avx2 (gemm.rs:280-374).
void quantize_split(const float* input, int8_t* even, int8_t* odd, float* scales, size_t cols,
                    size_t gs, size_t ng) {
  const __m256 sign_mask = _mm256_castsi256_ps(_mm256_set1_epi32(0x7FFFFFFF));
  const __m128i even_shuf = _mm_setr_epi8(0, 2, 4, 6, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1);
  const __m128i odd_shuf = _mm_setr_epi8(1, 3, 5, 7, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1);
  for (size_t g = 0; g < ng; ++g) {
    size_t start = g * gs, end = std::min((g + 1) * gs, cols), len = end - start;
    const float* inp = input + start;
    size_t chunks8 = len / 8;
    __m256 vmax = _mm256_setzero_ps();
    for (size_t i = 0; i < chunks8; ++i)
      vmax = _mm256_max_ps(vmax, _mm256_and_ps(_mm256_loadu_ps(inp + i * 8), sign_mask));
    __m128 hi128 = _mm256_extractf128_ps(vmax, 1);
    __m128 lo128 = _mm256_castps256_ps128(vmax);
    __m128 m128 = _mm_max_ps(lo128, hi128);
    __m128 shuf = _mm_movehdup_ps(m128);
    __m128 m64 = _mm_max_ps(m128, shuf);
    __m128 hi64 = _mm_movehl_ps(m64, m64);
    float absmax = _mm_cvtss_f32(_mm_max_ss(m64, hi64));
    for (size_t i = chunks8 * 8; i < len; ++i) {
      float a = std::fabs(inp[i]);
      if (a > absmax) absmax = a;
    }
    float scale = absmax > 1e-10f ? absmax / 127.0f : 1.0f;
    float inv = 1.0f / scale;
    scales[g] = scale;
    __m256 inv_v = _mm256_set1_ps(inv), min_v = _mm256_set1_ps(-128.0f), max_v = _mm256_set1_ps(127.0f);
    size_t even_base = start / 2;
    for (size_t i = 0; i < chunks8; ++i) {
      __m256 v = _mm256_loadu_ps(inp + i * 8);
      __m256 scaled = _mm256_mul_ps(v, inv_v);
      __m256 rounded = _mm256_round_ps(scaled, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
      __m256 clamped = _mm256_max_ps(_mm256_min_ps(rounded, max_v), min_v);
      __m256i i32s = _mm256_cvtps_epi32(clamped);
      __m128i lo = _mm256_castsi256_si128(i32s), hi = _mm256_extracti128_si256(i32s, 1);
      __m128i p16 = _mm_packs_epi32(lo, hi);
      __m128i p8 = _mm_packs_epi16(p16, _mm_setzero_si128());
      int32_t e = _mm_cvtsi128_si32(_mm_shuffle_epi8(p8, even_shuf));
      int32_t o = _mm_cvtsi128_si32(_mm_shuffle_epi8(p8, odd_shuf));
      std::memcpy(even + even_base + i * 4, &e, 4);
      std::memcpy(odd + even_base + i * 4, &o, 4);
    }
    size_t col = start + chunks8 * 8;
    while (col + 1 < end) {
      size_t k = col / 2;
      even[k] = scalar_q(input[col] * inv, -128.f, 127.f);
      odd[k] = scalar_q(input[col + 1] * inv, -128.f, 127.f);
      col += 2;
    }
  }
}

// matmul_row_tile<T> (gemm.rs:562-674); with T = 1 it is also matvec_chunk_i8's
// per-row arithmetic (gemm.rs:401-539), which computes the same zero
// correction in the same group order.
template <int T>
void row_tile(float* output, const uint8_t* nib_row, const float* w_scales, const float* w_zeros,
              const float* input_f32, const int8_t* in_even, const int8_t* in_odd,
              const float* in_scales /*[tokens][MAX_GROUPS]*/, const float* in_sums,
              size_t t_base, size_t row, size_t rows, size_t cols, size_t gs, size_t ng) {
  const size_t half_cols = cols / 2;
  const __m256i mask_0f = _mm256_set1_epi8(0x0F);
  const __m256i ones_16 = _mm256_set1_epi16(1);
  __m256 float_acc[T];
  for (int j = 0; j < T; ++j) float_acc[j] = _mm256_setzero_ps();
  for (size_t g = 0; g < ng; ++g) {
    size_t col_start = g * gs, actual = std::min((g + 1) * gs, cols) - col_start;
    size_t nib_off = col_start / 2, chunks64 = actual / 64;
    __m256i iacc[T];
    for (int j = 0; j < T; ++j) iacc[j] = _mm256_setzero_si256();
    for (size_t c = 0; c < chunks64; ++c) {
      __m256i raw = _mm256_loadu_si256((const __m256i*)(nib_row + nib_off + c * 32));
      __m256i lo = _mm256_and_si256(raw, mask_0f);
      __m256i hi = _mm256_and_si256(_mm256_srli_epi16(raw, 4), mask_0f);
      for (int j = 0; j < T; ++j) {
        size_t base = (t_base + j) * half_cols + nib_off + c * 32;
        __m256i ie = _mm256_loadu_si256((const __m256i*)(in_even + base));
        __m256i io = _mm256_loadu_si256((const __m256i*)(in_odd + base));
        __m256i pe = _mm256_maddubs_epi16(lo, ie);
        __m256i po = _mm256_maddubs_epi16(hi, io);
        __m256i comb = _mm256_add_epi16(pe, po);
        iacc[j] = _mm256_add_epi32(iacc[j], _mm256_madd_epi16(comb, ones_16));
      }
    }
    size_t simd_done = chunks64 * 64;
    bool block32 = simd_done + 32 <= actual;
    size_t simd_done2 = simd_done + (block32 ? 32 : 0);
    for (int j = 0; j < T; ++j) {
      size_t t = t_base + j;
      float combined = w_scales[g] * in_scales[t * MAX_GROUPS + g];
      float_acc[j] = _mm256_add_ps(float_acc[j], _mm256_mul_ps(_mm256_cvtepi32_ps(iacc[j]), _mm256_set1_ps(combined)));
      if (block32) {
        const __m128i mask128 = _mm_set1_epi8(0x0F), ones128 = _mm_set1_epi16(1);
        __m128i raw = _mm_loadu_si128((const __m128i*)(nib_row + nib_off + simd_done / 2));
        __m128i lo = _mm_and_si128(raw, mask128);
        __m128i hi = _mm_and_si128(_mm_srli_epi16(raw, 4), mask128);
        size_t base = t * half_cols + nib_off + simd_done / 2;
        __m128i ie = _mm_loadu_si128((const __m128i*)(in_even + base));
        __m128i io = _mm_loadu_si128((const __m128i*)(in_odd + base));
        __m128i comb = _mm_add_epi16(_mm_maddubs_epi16(lo, ie), _mm_maddubs_epi16(hi, io));
        __m128i sums = _mm_madd_epi16(comb, ones128);
        __m128 tail_f = _mm_mul_ps(_mm_cvtepi32_ps(sums), _mm_set1_ps(combined));
        float_acc[j] = _mm256_add_ps(float_acc[j], _mm256_insertf128_ps(_mm256_setzero_ps(), tail_f, 0));
      }
      if (simd_done2 < actual) {
        const float* tok = input_f32 + t * cols;
        float tail_acc = 0.0f;
        size_t tc = simd_done2;
        while (tc + 1 < actual) {
          uint8_t b = nib_row[nib_off + tc / 2];
          float a = (float)(b & 0x0F) * tok[col_start + tc];
          float c2 = (float)(b >> 4) * tok[col_start + tc + 1];
          tail_acc += a + c2;
          tc += 2;
        }
        __m256 tail_v = _mm256_set_ps(0, 0, 0, 0, 0, 0, 0, w_scales[g] * tail_acc);
        float_acc[j] = _mm256_add_ps(float_acc[j], tail_v);
      }
    }
  }
  for (int j = 0; j < T; ++j) {
    size_t t = t_base + j;
    float dot = hsum8(float_acc[j]);
    const float* sums = in_sums + t * MAX_GROUPS;
    float zero_corr = 0.0f;
    for (size_t g = 0; g < ng; ++g) zero_corr += w_zeros[g] * sums[g];
    output[t * rows + row] = dot + zero_corr;
  }
}

inline size_t chunk_rows_for(size_t cols) {  // gemm.rs:1158-1160
  size_t c = 24576 / std::max<size_t>(cols / 2, 1);
  return std::min<size_t>(std::max<size_t>(c, 4), 64);
}

// matmul_chunk_i8 (gemm.rs:689-784), weight-stationary over 4-token tiles.
void matmul_chunk(float* out, const uint8_t* nib, const uint8_t* params, const float* in_f32,
                  const int8_t* ie, const int8_t* io, const float* iscales, const float* isums,
                  size_t start_row, size_t chunk_len, size_t rows, size_t cols, size_t gs,
                  size_t ng, size_t tokens) {
  size_t row_bytes = cols / 2;
  size_t pf_dist = row_bytes > 2048 ? 1 : 3;
  float w_scales[MAX_GROUPS], w_zeros[MAX_GROUPS];
  for (size_t local = 0; local < chunk_len; ++local) {
    size_t row = start_row + local;
    const uint8_t* nib_row = nib + row * row_bytes;
    if (local + pf_dist < chunk_len) {
      const uint8_t* pf = nib + (row + pf_dist) * row_bytes;
      for (size_t p = 0; p < row_bytes; p += 64) _mm_prefetch((const char*)(pf + p), _MM_HINT_T0);
    }
    const uint8_t* rp = params + row * ng * 4;
    for (size_t g = 0; g < ng; ++g) {
      uint32_t bits;
      std::memcpy(&bits, rp + g * 4, 4);
      __m128 f = _mm_cvtph_ps(_mm_cvtsi32_si128((int)bits));
      w_scales[g] = _mm_cvtss_f32(f);
      w_zeros[g] = _mm_cvtss_f32(_mm_shuffle_ps(f, f, 1));
    }
    size_t t = 0;
    for (; t + 4 <= tokens; t += 4)
      row_tile<4>(out, nib_row, w_scales, w_zeros, in_f32, ie, io, iscales, isums, t, row, rows, cols, gs, ng);
    for (; t < tokens; ++t)
      row_tile<1>(out, nib_row, w_scales, w_zeros, in_f32, ie, io, iscales, isums, t, row, rows, cols, gs, ng);
  }
}

// lm_head_chunk_i8 (gemm.rs:804-915).
void lm_head_chunk(float* logits, const uint8_t* embed, const uint8_t* eparams, const int8_t* hq,
                   const float* hsums, const float* hscales, size_t start, size_t chunk_len,
                   size_t hidden, size_t gs, size_t ng) {
  const __m256i ones_16 = _mm256_set1_epi16(1);
  for (size_t local = 0; local < chunk_len; ++local) {
    size_t v = start + local;
    const uint8_t* row = embed + v * hidden;
    if (local + 3 < chunk_len) {
      const uint8_t* pf = embed + (v + 3) * hidden;
      for (size_t p = 0; p < hidden; p += 64) _mm_prefetch((const char*)(pf + p), _MM_HINT_T0);
    }
    float zero_corr = 0.0f, w_scales[MAX_GROUPS];
    const uint8_t* rp = eparams + v * ng * 4;
    for (size_t g = 0; g < ng; ++g) {
      uint32_t bits;
      std::memcpy(&bits, rp + g * 4, 4);
      __m128 ff = _mm_cvtph_ps(_mm_cvtsi32_si128((int)bits));
      w_scales[g] = _mm_cvtss_f32(ff);
      zero_corr += _mm_cvtss_f32(_mm_shuffle_ps(ff, ff, 1)) * hsums[g];
    }
    __m256 float_acc = _mm256_setzero_ps();
    for (size_t g = 0; g < ng; ++g) {
      size_t cs = g * gs, actual = std::min((g + 1) * gs, hidden) - cs, chunks32 = actual / 32;
      const uint8_t* codes = row + cs;
      const int8_t* h = hq + cs;
      __m256i iacc = _mm256_setzero_si256();
      for (size_t c = 0; c < chunks32; ++c) {
        __m256i cv = _mm256_loadu_si256((const __m256i*)(codes + c * 32));
        __m256i hv = _mm256_loadu_si256((const __m256i*)(h + c * 32));
        iacc = _mm256_add_epi32(iacc, _mm256_madd_epi16(_mm256_maddubs_epi16(cv, hv), ones_16));
      }
      float combined = w_scales[g] * hscales[g];
      float_acc = _mm256_add_ps(float_acc, _mm256_mul_ps(_mm256_cvtepi32_ps(iacc), _mm256_set1_ps(combined)));
      size_t done = chunks32 * 32;
      if (done < actual) {
        float tail = 0.0f;
        for (size_t i = done; i < actual; ++i) tail += (float)codes[i] * (float)h[i];
        float tv = w_scales[g] * hscales[g] * tail;
        float_acc = _mm256_add_ps(float_acc, _mm256_set_ps(0, 0, 0, 0, 0, 0, 0, tv));
      }
    }
    logits[local] = hsum8(float_acc) + zero_corr;
  }
}

// quantize_hidden_i8_avx2 (gemm.rs:976-1047): per embed group, range +-63.
void quantize_hidden(const float* hidden, int8_t* out, float* scales, size_t n, size_t gs, size_t ng) {
  const __m256 sign_mask = _mm256_castsi256_ps(_mm256_set1_epi32(0x7FFFFFFF));
  for (size_t g = 0; g < ng; ++g) {
    size_t start = g * gs, end = std::min((g + 1) * gs, n), len = end - start;
    const float* inp = hidden + start;
    size_t chunks8 = len / 8;
    __m256 vmax = _mm256_setzero_ps();
    for (size_t i = 0; i < chunks8; ++i)
      vmax = _mm256_max_ps(vmax, _mm256_and_ps(_mm256_loadu_ps(inp + i * 8), sign_mask));
    __m128 hi128 = _mm256_extractf128_ps(vmax, 1), lo128 = _mm256_castps256_ps128(vmax);
    __m128 m128 = _mm_max_ps(lo128, hi128);
    __m128 m64 = _mm_max_ps(m128, _mm_movehdup_ps(m128));
    float absmax = _mm_cvtss_f32(_mm_max_ss(m64, _mm_movehl_ps(m64, m64)));
    for (size_t i = chunks8 * 8; i < len; ++i) {
      float a = std::fabs(inp[i]);
      if (a > absmax) absmax = a;
    }
    float scale = absmax > 1e-10f ? absmax / 63.0f : 1.0f;
    float inv = 1.0f / scale;
    scales[g] = scale;
    __m256 inv_v = _mm256_set1_ps(inv), min_v = _mm256_set1_ps(-63.f), max_v = _mm256_set1_ps(63.f);
    int8_t* op = out + start;
    for (size_t i = 0; i < chunks8; ++i) {
      __m256 v = _mm256_loadu_ps(inp + i * 8);
      __m256 r = _mm256_round_ps(_mm256_mul_ps(v, inv_v), _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
      __m256i i32s = _mm256_cvtps_epi32(_mm256_max_ps(_mm256_min_ps(r, max_v), min_v));
      __m128i p16 = _mm_packs_epi32(_mm256_castsi256_si128(i32s), _mm256_extracti128_si256(i32s, 1));
      __m128i p8 = _mm_packs_epi16(p16, _mm_setzero_si128());
      int64_t q = _mm_cvtsi128_si64(p8);
      std::memcpy(op + i * 8, &q, 8);
    }
    for (size_t i = chunks8 * 8; i < len; ++i) op[i] = scalar_q(inp[i] * inv, -63.f, 63.f);
  }
}

// Schraudolph exp used by silu_mul_avx2 and the attention softmax.
inline __m256 schraudolph(__m256 x) {
  const __m256 a = _mm256_set1_ps(12102203.0f);
  const __m256 b = _mm256_set1_ps(1065353216.0f - 486411.0f);
  __m256 t = _mm256_add_ps(_mm256_mul_ps(a, x), b);
  t = _mm256_max_ps(_mm256_min_ps(t, _mm256_set1_ps(2139095040.0f)), _mm256_set1_ps(0.0f));
  return _mm256_castsi256_ps(_mm256_cvtps_epi32(t));
}

}  // namespace

extern "C" {

void orc_quantize_input(const float* x, size_t cols, size_t gs, int8_t* even, int8_t* odd,
                        float* scales, float* sums) {
  size_t ng = (cols + gs - 1) / gs;
  input_sums(x, sums, cols, gs, ng);
  quantize_split(x, even, odd, scales, cols, gs, ng);
}

// w4a8_matmul / w4a8_matvec (gemm.rs:1774-1919, 1336-1392). Output layout
// out[t * rows + r]; each (token, row) is independent of the dispatch.
void orc_w4a8_matmul(float* out, const uint8_t* nib, const uint8_t* params, const float* input,
                     size_t rows, size_t cols, size_t tokens, size_t gs) {
  size_t ng = (cols + gs - 1) / gs, half = cols / 2;
  std::vector<int8_t> ev(tokens * half), od(tokens * half);
  std::vector<float> sc(tokens * MAX_GROUPS, 0.f), su(tokens * MAX_GROUPS, 0.f);
  for (size_t t = 0; t < tokens; ++t) {
    const float* inp = input + t * cols;
    input_sums(inp, su.data() + t * MAX_GROUPS, cols, gs, ng);
    quantize_split(inp, ev.data() + t * half, od.data() + t * half, sc.data() + t * MAX_GROUPS, cols, gs, ng);
  }
  size_t cr = chunk_rows_for(cols), nchunks = (rows + cr - 1) / cr;
  bool par = tokens > 1 || (rows >= 256 && rows * cols / 2 >= 512 * 1024);
#pragma omp parallel for schedule(dynamic) if (par)
  for (size_t ci = 0; ci < nchunks; ++ci) {
    size_t start = ci * cr, len = std::min(cr, rows - start);
    matmul_chunk(out, nib, params, input, ev.data(), od.data(), sc.data(), su.data(), start, len,
                 rows, cols, gs, ng, tokens);
  }
}

// tied_lm_head (gemm.rs:1981-2076).
void orc_tied_lm_head(float* logits, const float* hidden, const uint8_t* data, const uint8_t* params,
                      size_t vocab, size_t hidden_size, size_t gs) {
  size_t ng = (hidden_size + gs - 1) / gs;
  float sums[MAX_GROUPS], scales[MAX_GROUPS];
  input_sums(hidden, sums, hidden_size, gs, ng);
  std::vector<int8_t> hq(hidden_size);
  quantize_hidden(hidden, hq.data(), scales, hidden_size, gs, ng);
  const size_t LM_CHUNK = 512;
  size_t nchunks = (vocab + LM_CHUNK - 1) / LM_CHUNK;
#pragma omp parallel for schedule(dynamic)
  for (size_t ci = 0; ci < nchunks; ++ci) {
    size_t start = ci * LM_CHUNK, len = std::min(LM_CHUNK, vocab - start);
    lm_head_chunk(logits + start, data, params, hq.data(), sums, scales, start, len, hidden_size, gs, ng);
  }
}

// embed_lookup (gemm.rs:1926-1970): code * scale + zero, two roundings.
void orc_embed_lookup(float* out, size_t token, const uint8_t* data, const uint8_t* params,
                      size_t vocab, size_t hidden, size_t gs) {
  (void)vocab;
  size_t ng = (hidden + gs - 1) / gs;
  for (size_t g = 0; g < ng; ++g) {
    const uint8_t* p = params + (token * ng + g) * 4;
    float scale = read_f16(p), zero = read_f16(p + 2);
    for (size_t c = g * gs; c < std::min((g + 1) * gs, hidden); ++c) {
      float code = (float)data[token * hidden + c];
      float prod = code * scale;
      out[c] = prod + zero;
    }
  }
}

// rms_norm_avx2 (layers.rs:325-376).
void orc_rms_norm(float* out, const float* inp, const float* wt, size_t n, float eps) {
  size_t chunks8 = n / 8, chunks16 = chunks8 / 2, i = 0;
  __m256 sq0 = _mm256_setzero_ps(), sq1 = _mm256_setzero_ps();
  for (size_t c = 0; c < chunks16; ++c) {
    __m256 v0 = _mm256_loadu_ps(inp + i), v1 = _mm256_loadu_ps(inp + i + 8);
    sq0 = _mm256_fmadd_ps(v0, v0, sq0);
    sq1 = _mm256_fmadd_ps(v1, v1, sq1);
    i += 16;
  }
  if (i + 8 <= n) {
    __m256 v0 = _mm256_loadu_ps(inp + i);
    sq0 = _mm256_fmadd_ps(v0, v0, sq0);
    i += 8;
  }
  float sum_sq = hsum8(_mm256_add_ps(sq0, sq1));
  for (; i < n; ++i) sum_sq += inp[i] * inp[i];
  float inv_rms = 1.0f / std::sqrt(sum_sq / (float)n + eps);
  __m256 inv_v = _mm256_set1_ps(inv_rms);
  i = 0;
  for (size_t c = 0; c < chunks8; ++c) {
    _mm256_storeu_ps(out + i, _mm256_mul_ps(_mm256_mul_ps(_mm256_loadu_ps(inp + i), inv_v), _mm256_loadu_ps(wt + i)));
    i += 8;
  }
  for (; i < n; ++i) out[i] = inp[i] * inv_rms * wt[i];
}

// rms_norm_with_residual_avx2 (layers.rs:433-497): same arithmetic as
// rms_norm plus a copy of the input into `residual`.
void orc_rms_norm_with_residual(float* normed, float* residual, const float* hidden, const float* w,
                                size_t n, float eps) {
  std::memcpy(residual, hidden, n * sizeof(float));
  orc_rms_norm(normed, hidden, w, n, eps);
}

// rms_norm_heads (layers.rs:201-240): sequential scalar sum of squares.
void orc_rms_norm_heads(float* x, size_t nh, size_t hd, const float* w, float eps) {
  for (size_t h = 0; h < nh; ++h) {
    float* head = x + h * hd;
    float sum_sq = 0.0f;
    for (size_t i = 0; i < hd; ++i) sum_sq += head[i] * head[i];
    float inv = 1.0f / std::sqrt(sum_sq / (float)hd + eps);
    for (size_t i = 0; i < hd; ++i) head[i] = head[i] * inv * w[i];
  }
}

// RoPETable::with_scaling + apply_llama3_scaling (layers.rs:561-633, 760-808).
int orc_rope_table(float* cos_t, float* sin_t, size_t hd, size_t max_ctx, float theta, int rope_type,
                   float factor, float low, float high, uint32_t orig) {
  size_t half = hd / 2;
  std::vector<float> inv_freq(half);
  for (size_t i = 0; i < half; ++i) {
    float e = 2.0f * (float)i / (float)hd;
    inv_freq[i] = 1.0f / powf(theta, e);
  }
  if (rope_type == 1) {
    float old_ctx = (float)orig;
    float low_wl = old_ctx / low, high_wl = old_ctx / high;
    const float two_pi = 2.0f * 3.14159265358979323846f;
    for (size_t i = 0; i < half; ++i) {
      float value = inv_freq[i];
      float wavelen = two_pi / value;
      float banded = wavelen > low_wl ? value / factor : value;
      bool medium = wavelen >= high_wl && wavelen <= low_wl;
      if (medium) {
        float smooth = (old_ctx / wavelen - low) / (high - low);
        float a = (1.0f - smooth) * banded / factor;
        float b = smooth * banded;
        inv_freq[i] = a + b;
      } else {
        inv_freq[i] = banded;
      }
    }
  }
  for (size_t pos = 0; pos < max_ctx; ++pos)
    for (size_t i = 0; i < half; ++i) {
      float angle = (float)pos * inv_freq[i];
      cos_t[pos * half + i] = cosf(angle);
      sin_t[pos * half + i] = sinf(angle);
    }
  return 0;
}

// RoPETable::apply / apply_avx2 (layers.rs:643-726): NeoX half split.
void orc_rope_apply(float* hp, size_t nh, size_t hd, const float* cp, const float* sp) {
  size_t half = hd / 2, chunks8 = half / 8;
  for (size_t h = 0; h < nh; ++h) {
    size_t base = h * hd;
    for (size_t c = 0; c < chunks8; ++c) {
      size_t i = c * 8;
      __m256 cv = _mm256_loadu_ps(cp + i), sv = _mm256_loadu_ps(sp + i);
      __m256 x0 = _mm256_loadu_ps(hp + base + i), x1 = _mm256_loadu_ps(hp + base + half + i);
      __m256 r0 = _mm256_fmsub_ps(x0, cv, _mm256_mul_ps(x1, sv));
      __m256 r1 = _mm256_fmadd_ps(x1, cv, _mm256_mul_ps(x0, sv));
      _mm256_storeu_ps(hp + base + i, r0);
      _mm256_storeu_ps(hp + base + half + i, r1);
    }
    for (size_t i = chunks8 * 8; i < half; ++i) {
      float x0 = hp[base + i], x1 = hp[base + half + i];
      hp[base + i] = x0 * cp[i] - x1 * sp[i];
      hp[base + half + i] = x1 * cp[i] + x0 * sp[i];
    }
  }
}

// silu_mul_avx2 (layers.rs:850-883) with the libm scalar tail.
void orc_silu_mul(float* gate, const float* up, size_t n) {
  size_t chunks8 = n / 8;
  const __m256 neg_one = _mm256_set1_ps(-1.0f), one = _mm256_set1_ps(1.0f);
  for (size_t i = 0; i < chunks8; ++i) {
    __m256 x = _mm256_loadu_ps(gate + i * 8), u = _mm256_loadu_ps(up + i * 8);
    __m256 e = schraudolph(_mm256_mul_ps(x, neg_one));
    __m256 s = _mm256_div_ps(x, _mm256_add_ps(one, e));
    _mm256_storeu_ps(gate + i * 8, _mm256_mul_ps(s, u));
  }
  for (size_t i = chunks8 * 8; i < n; ++i) {
    float x = gate[i];
    float s = x / (1.0f + expf(-x));
    gate[i] = s * up[i];
  }
}

// attention_head_avx2 (layers.rs:1266-1380). K/V rows of this head at
// k_head[t * head_dim], v_head[t * head_dim].
void orc_attention_head(const float* q, float* out, const float* k_head, const float* v_head,
                        size_t pos, size_t hd, float scale, float softcap) {
  size_t chunks8 = hd / 8, n_pos = pos + 1;
  std::vector<float> scores(n_pos);
  float max_score = -INFINITY;
  for (size_t t = 0; t < n_pos; ++t) {
    const float* k = k_head + t * hd;
    __m256 acc = _mm256_setzero_ps();
    for (size_t c = 0; c < chunks8; ++c)
      acc = _mm256_fmadd_ps(_mm256_loadu_ps(q + c * 8), _mm256_loadu_ps(k + c * 8), acc);
    float dot = hsum8(acc);
    float sc = dot * scale;
    if (softcap > 0.0f) sc = softcap * tanhf(sc / softcap);
    scores[t] = sc;
    if (sc > max_score) max_score = sc;
  }
  __m256 max_v = _mm256_set1_ps(max_score);
  __m256 sum_acc = _mm256_setzero_ps();
  size_t c8 = n_pos / 8;
  for (size_t i = 0; i < c8; ++i) {
    __m256 ev = schraudolph(_mm256_sub_ps(_mm256_loadu_ps(scores.data() + i * 8), max_v));
    _mm256_storeu_ps(scores.data() + i * 8, ev);
    sum_acc = _mm256_add_ps(sum_acc, ev);
  }
  float sum_exp = hsum8(sum_acc);
  for (size_t t = c8 * 8; t < n_pos; ++t) {
    float v = expf(scores[t] - max_score);
    scores[t] = v;
    sum_exp += v;
  }
  float inv_sum = 1.0f / sum_exp;
  __m256 inv_v = _mm256_set1_ps(inv_sum);
  for (size_t i = 0; i < c8; ++i)
    _mm256_storeu_ps(scores.data() + i * 8, _mm256_mul_ps(_mm256_loadu_ps(scores.data() + i * 8), inv_v));
  for (size_t t = c8 * 8; t < n_pos; ++t) scores[t] *= inv_sum;
  for (size_t c = 0; c < chunks8; ++c) _mm256_storeu_ps(out + c * 8, _mm256_setzero_ps());
  for (size_t t = 0; t < n_pos; ++t) {
    const float* v = v_head + t * hd;
    __m256 s = _mm256_set1_ps(scores[t]);
    for (size_t c = 0; c < chunks8; ++c)
      _mm256_storeu_ps(out + c * 8, _mm256_fmadd_ps(s, _mm256_loadu_ps(v + c * 8), _mm256_loadu_ps(out + c * 8)));
  }
}

// attention_head_avx2 with its intermediates exposed (test diagnostics):
// e[t] = the exponentials before normalisation, *max and *sum.
void orc_attention_head_debug(const float* q, float* out, const float* k_head, const float* v_head, size_t pos,
                              size_t hd, float scale, float* e, float* mx, float* sum) {
  size_t chunks8 = hd / 8, n_pos = pos + 1;
  std::vector<float> scores(n_pos);
  float max_score = -INFINITY;
  for (size_t t = 0; t < n_pos; ++t) {
    const float* k = k_head + t * hd;
    __m256 acc = _mm256_setzero_ps();
    for (size_t c = 0; c < chunks8; ++c)
      acc = _mm256_fmadd_ps(_mm256_loadu_ps(q + c * 8), _mm256_loadu_ps(k + c * 8), acc);
    float sc = hsum8(acc) * scale;
    scores[t] = sc;
    if (sc > max_score) max_score = sc;
  }
  *mx = max_score;
  __m256 max_v = _mm256_set1_ps(max_score), sum_acc = _mm256_setzero_ps();
  size_t c8 = n_pos / 8;
  for (size_t i = 0; i < c8; ++i) {
    __m256 ev = schraudolph(_mm256_sub_ps(_mm256_loadu_ps(scores.data() + i * 8), max_v));
    _mm256_storeu_ps(scores.data() + i * 8, ev);
    sum_acc = _mm256_add_ps(sum_acc, ev);
  }
  float s = hsum8(sum_acc);
  for (size_t t = c8 * 8; t < n_pos; ++t) {
    float v = expf(scores[t] - max_score);
    scores[t] = v;
    s += v;
  }
  *sum = s;
  for (size_t t = 0; t < n_pos; ++t) e[t] = scores[t];
  orc_attention_head(q, out, k_head, v_head, pos, hd, scale, 0.f);
}

// route_experts (layers.rs:1808-1870) with dot_f32 (iterator sum from -0.0).
void orc_route_experts(const float* hidden, const float* router, size_t ne, size_t width, size_t k,
                       int norm_topk, uint32_t* experts, float* weights) {
  std::vector<float> probs(ne);
  for (size_t e = 0; e < ne; ++e) {
    float s = -0.0f;
    for (size_t i = 0; i < width; ++i) s += router[e * width + i] * hidden[i];
    probs[e] = s;
  }
  float mx = -INFINITY;
  for (float v : probs) mx = std::fmax(mx, v);
  float sum = 0.0f;
  for (float& v : probs) { v = expf(v - mx); sum += v; }
  for (float& v : probs) v /= sum;
  std::vector<bool> taken(ne, false);
  size_t count = 0;
  for (size_t s = 0; s < k; ++s) {
    size_t best = (size_t)-1;
    float bv = -INFINITY;
    for (size_t e = 0; e < ne; ++e)
      if (!taken[e] && probs[e] > bv) { bv = probs[e]; best = e; }
    if (best == (size_t)-1) break;
    taken[best] = true;
    experts[count] = (uint32_t)best;
    weights[count] = bv;
    ++count;
  }
  for (size_t s = count; s < k; ++s) { experts[s] = UINT32_MAX; weights[s] = 0.f; }
  if (norm_topk) {
    float total = -0.0f;
    for (size_t s = 0; s < count; ++s) total += weights[s];
    if (total > 0.0f)
      for (size_t s = 0; s < count; ++s) weights[s] /= total;
  }
}

// find_ngram_draft (lookup.rs:131-171).
int orc_find_ngram_draft(const uint32_t* tokens, size_t len, size_t min_n, size_t max_n,
                         size_t max_draft, size_t* ngram, size_t* start, size_t* dlen) {
  if (max_draft == 0 || len < 2) return 0;
  size_t hi = std::min(max_n, len - 1), lo = std::max<size_t>(min_n, 1);
  if (lo > hi) return 0;
  for (size_t n = hi; n >= lo; --n) {
    const uint32_t* suffix = tokens + len - n;
    for (size_t s = len - n; s-- > 0;) {
      if (std::memcmp(tokens + s, suffix, n * sizeof(uint32_t)) != 0) continue;
      size_t ds = s + n, dl = std::min(max_draft, len - ds);
      if (dl == 0) continue;
      *ngram = n; *start = ds; *dlen = dl;
      return 1;
    }
    if (n == lo) break;
  }
  return 0;
}

// sampler::argmax (sampler.rs:201-208) after the NaN -> -inf rewrite:
// total order, ties resolve to the LAST maximal index.
size_t orc_argmax(const float* v, size_t n) {
  auto key = [](float f) {
    if (std::isnan(f)) f = -INFINITY;
    int32_t b;
    std::memcpy(&b, &f, 4);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
    return b;
  };
  size_t best = 0;
  int32_t bk = key(v[0]);
  for (size_t i = 1; i < n; ++i) {
    int32_t k = key(v[i]);
    if (k >= bk) { bk = k; best = i; }
  }
  return best;
}

int orc_num_threads(void) { return omp_get_max_threads(); }

// f32::exp as the reference runs it (glibc expf) for the floats with bit
// patterns first .. first + n - 1.
void orc_expf_range(uint32_t first, size_t n, float* out) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; ++i) {
    const uint32_t b = first + (uint32_t)i;
    float x;
    std::memcpy(&x, &b, 4);
    out[i] = expf(x);
  }
}
void orc_set_num_threads(int n) { if (n > 0) omp_set_num_threads(n); }

size_t orc_last_error(char* buf, size_t len) {
  if (buf && len) {
    size_t n = std::min(len - 1, g_err.size());
    std::memcpy(buf, g_err.data(), n);
    buf[n] = 0;
  }
  return g_err.size();
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Model + decoder (rai-infer/src/model.rs, lookup.rs, kv_cache.rs)
// ---------------------------------------------------------------------------

struct orc_model {
  std::vector<uint8_t> blob;
  raimodel::Model m;
  std::vector<float> rope_cos, rope_sin, rope_local_cos, rope_local_sin;
  std::vector<std::vector<float>> in_norm, post_norm, q_norm, k_norm, attn_out_norm, mlp_out_norm, router;
  std::vector<std::vector<std::vector<float>>> bias;  // [layer][proj]
  std::vector<float> final_norm;
  float scale = 0.f;
  const uint8_t* p(size_t off) const { return blob.data() + off; }
};

struct orc_decoder {
  orc_model* model;
  size_t max_ctx;
  std::vector<std::vector<float>> k, v;  // [layer] -> [kv_head][max_ctx][head_dim]
  std::vector<size_t> filled;
};

namespace {

void linear_matmul(const orc_model* M, const raimodel::Linear& L, float* out, const float* in, size_t tokens) {
  orc_w4a8_matmul(out, M->p(L.nib_off), M->p(L.params_off), in, L.rows, L.cols, tokens, L.group_size);
}

void add_bias(float* x, const std::vector<float>& b) {  // add_bias (layers.rs:109-143)
  for (size_t i = 0; i < b.size(); ++i) x[i] = x[i] + b[i];
}

// KVCache::store (kv_cache.rs:143-172): gap-free watermark.
bool kv_store(orc_decoder* d, size_t layer, size_t pos, const float* kv_k, const float* kv_v) {
  const auto& c = d->model->m.cfg;
  if (pos >= d->max_ctx) { g_err = "KV cache position is out of range"; return false; }
  if (pos > d->filled[layer]) { g_err = "KV store would leave a gap"; return false; }
  size_t hd = c.head_dim;
  for (size_t h = 0; h < c.num_kv_heads; ++h) {
    std::memcpy(&d->k[layer][(h * d->max_ctx + pos) * hd], kv_k + h * hd, hd * 4);
    std::memcpy(&d->v[layer][(h * d->max_ctx + pos) * hd], kv_v + h * hd, hd * 4);
  }
  d->filled[layer] = std::max(d->filled[layer], pos + 1);
  return true;
}

void glu(const orc_model* M, float* gate, const float* up, size_t n) {
  if (M->m.cfg.activation == 0) { orc_silu_mul(gate, up, n); return; }
  // GeLU-tanh (layers.rs gelu_tanh_mul_avx2) is outside the decode path this
  // build targets; the oracle refuses such models at open.
}

// swiglu_mlp (layers.rs:1876-1910) for one token through the matvec path.
void swiglu_one(const orc_model* M, size_t li, const raimodel::Linear& g, const raimodel::Linear& u,
                const raimodel::Linear& dn, const float* in, float* out) {
  size_t ff = g.rows;
  std::vector<float> gate(ff), upv(ff);
  linear_matmul(M, g, gate.data(), in, 1);
  linear_matmul(M, u, upv.data(), in, 1);
  if (!M->bias[li][4].empty()) add_bias(gate.data(), M->bias[li][4]);
  if (!M->bias[li][5].empty()) add_bias(upv.data(), M->bias[li][5]);
  glu(M, gate.data(), upv.data(), ff);
  linear_matmul(M, dn, out, gate.data(), 1);
  if (!M->bias[li][6].empty()) add_bias(out, M->bias[li][6]);
}

const float* rope_cos_for(const orc_model* M, size_t li) {
  const auto& c = M->m.cfg;
  if (c.global_layer_stride > 0 && (li + 1) % c.global_layer_stride != 0) return M->rope_local_cos.data();
  return M->rope_cos.data();
}
const float* rope_sin_for(const orc_model* M, size_t li) {
  const auto& c = M->m.cfg;
  if (c.global_layer_stride > 0 && (li + 1) % c.global_layer_stride != 0) return M->rope_local_sin.data();
  return M->rope_sin.data();
}

void norm_block_output(const std::vector<float>& w, float* x, size_t n, float eps) {
  if (w.empty()) return;
  std::vector<float> tmp(n);
  orc_rms_norm(tmp.data(), x, w.data(), n, eps);
  std::memcpy(x, tmp.data(), n * 4);
}

// RaiModel::forward_batch (model.rs:692-963).
bool forward_batch(orc_decoder* d, float* hid, const size_t* positions, size_t batch) {
  orc_model* M = d->model;
  const auto& c = M->m.cfg;
  size_t hs = c.hidden_size, nh = c.num_heads, nkv = c.num_kv_heads, hd = c.head_dim;
  size_t ff = c.intermediate_size, qd = nh * hd, kvd = nkv * hd, half = hd / 2;
  float eps = c.norm_eps;
  for (size_t b = 0; b < batch; ++b)
    if (positions[b] >= c.max_context || positions[b] >= d->max_ctx) { g_err = "batch position exceeds model context"; return false; }
  for (size_t b = 1; b < batch; ++b)
    if (positions[b] != positions[b - 1] + 1) { g_err = "batch positions must be strictly consecutive and ascending"; return false; }
  std::vector<float> normed(batch * hs), resid(batch * hs), q(batch * qd), k(batch * kvd), v(batch * kvd);
  std::vector<float> attn(batch * qd), o(batch * hs), gate(batch * ff), up(batch * ff), mlp(batch * hs);
  for (size_t li = 0; li < c.num_layers; ++li) {
    const raimodel::Layer& L = M->m.layers[li];
    const bool post = c.post_norm;
    for (size_t b = 0; b < batch; ++b) {
      if (post) {
        std::memcpy(&normed[b * hs], &hid[b * hs], hs * 4);
        std::memcpy(&resid[b * hs], &hid[b * hs], hs * 4);
      } else {
        orc_rms_norm_with_residual(&normed[b * hs], &resid[b * hs], &hid[b * hs], M->in_norm[li].data(), hs, eps);
      }
    }
    linear_matmul(M, L.proj[0], q.data(), normed.data(), batch);
    linear_matmul(M, L.proj[1], k.data(), normed.data(), batch);
    linear_matmul(M, L.proj[2], v.data(), normed.data(), batch);
    for (size_t b = 0; b < batch; ++b) {
      if (!M->bias[li][0].empty()) add_bias(&q[b * qd], M->bias[li][0]);
      if (!M->bias[li][1].empty()) add_bias(&k[b * kvd], M->bias[li][1]);
      if (!M->bias[li][2].empty()) add_bias(&v[b * kvd], M->bias[li][2]);
    }
    if (!M->q_norm[li].empty()) {
      for (size_t b = 0; b < batch; ++b) {
        if (c.has_full_qk_norm) {
          orc_rms_norm_heads(&q[b * qd], 1, qd, M->q_norm[li].data(), eps);
          orc_rms_norm_heads(&k[b * kvd], 1, kvd, M->k_norm[li].data(), eps);
        } else {
          orc_rms_norm_heads(&q[b * qd], nh, hd, M->q_norm[li].data(), eps);
          orc_rms_norm_heads(&k[b * kvd], nkv, hd, M->k_norm[li].data(), eps);
        }
      }
    }
    const float* rc = rope_cos_for(M, li);
    const float* rs = rope_sin_for(M, li);
    for (size_t b = 0; b < batch; ++b) {
      size_t pos = positions[b];
      orc_rope_apply(&q[b * qd], nh, hd, rc + pos * half, rs + pos * half);
      orc_rope_apply(&k[b * kvd], nkv, hd, rc + pos * half, rs + pos * half);
      if (!kv_store(d, li, pos, &k[b * kvd], &v[b * kvd])) return false;
    }
    size_t hpk = nh / nkv;
    for (size_t b = 0; b < batch; ++b)
      if (positions[b] >= d->filled[li]) { g_err = "attention would read unwritten KV entries"; return false; }
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (size_t b = 0; b < batch; ++b)
      for (size_t qh = 0; qh < nh; ++qh) {
        size_t kvh = qh / hpk;
        orc_attention_head(&q[b * qd + qh * hd], &attn[b * qd + qh * hd],
                           &d->k[li][kvh * d->max_ctx * hd], &d->v[li][kvh * d->max_ctx * hd],
                           positions[b], hd, M->scale, c.attn_logit_softcap);
      }
    linear_matmul(M, L.proj[3], o.data(), attn.data(), batch);
    for (size_t b = 0; b < batch; ++b) {
      if (!M->bias[li][3].empty()) add_bias(&o[b * hs], M->bias[li][3]);
      norm_block_output(post ? M->in_norm[li] : M->attn_out_norm[li], &o[b * hs], hs, eps);
      for (size_t i = 0; i < hs; ++i) hid[b * hs + i] = resid[b * hs + i] + o[b * hs + i];
    }
    for (size_t b = 0; b < batch; ++b) {
      if (post) {
        std::memcpy(&normed[b * hs], &hid[b * hs], hs * 4);
        std::memcpy(&resid[b * hs], &hid[b * hs], hs * 4);
      } else {
        orc_rms_norm_with_residual(&normed[b * hs], &resid[b * hs], &hid[b * hs], M->post_norm[li].data(), hs, eps);
      }
    }
    if (c.num_experts > 0) {
      // mlp_block (model.rs:208-261), token by token through the matvec path.
      size_t topk = c.experts_per_token;
      std::vector<uint32_t> ex(topk);
      std::vector<float> wts(topk), eo(hs);
      for (size_t b = 0; b < batch; ++b) {
        orc_route_experts(&normed[b * hs], M->router[li].data(), c.num_experts, hs, topk, c.norm_topk_prob, ex.data(), wts.data());
        float* out = &mlp[b * hs];
        std::fill(out, out + hs, 0.0f);
        for (size_t s = 0; s < topk && ex[s] != UINT32_MAX; ++s) {
          size_t e = ex[s];
          const raimodel::Linear& g = e == 0 ? L.proj[4] : L.experts[3 * (e - 1)];
          const raimodel::Linear& u = e == 0 ? L.proj[5] : L.experts[3 * (e - 1) + 1];
          const raimodel::Linear& dn = e == 0 ? L.proj[6] : L.experts[3 * (e - 1) + 2];
          swiglu_one(M, li, g, u, dn, &normed[b * hs], eo.data());
          float w = wts[s];
          for (size_t i = 0; i < hs; ++i) out[i] = out[i] + w * eo[i];
        }
      }
    } else {
      linear_matmul(M, L.proj[4], gate.data(), normed.data(), batch);
      linear_matmul(M, L.proj[5], up.data(), normed.data(), batch);
      for (size_t b = 0; b < batch; ++b) {
        if (!M->bias[li][4].empty()) add_bias(&gate[b * ff], M->bias[li][4]);
        if (!M->bias[li][5].empty()) add_bias(&up[b * ff], M->bias[li][5]);
        glu(M, &gate[b * ff], &up[b * ff], ff);
      }
      linear_matmul(M, L.proj[6], mlp.data(), gate.data(), batch);
    }
    for (size_t b = 0; b < batch; ++b) {
      if (!M->bias[li][6].empty()) add_bias(&mlp[b * hs], M->bias[li][6]);
      norm_block_output(post ? M->post_norm[li] : M->mlp_out_norm[li], &mlp[b * hs], hs, eps);
      for (size_t i = 0; i < hs; ++i) hid[b * hs + i] = resid[b * hs + i] + mlp[b * hs + i];
    }
  }
  return true;
}

// RaiModel::hidden_to_logits_batch (model.rs:966-1033).
void hidden_to_logits(orc_decoder* d, const float* hid, size_t batch, float* logits) {
  orc_model* M = d->model;
  const auto& c = M->m.cfg;
  size_t hs = c.hidden_size, vs = c.vocab_size;
  std::vector<float> normed(batch * hs);
  for (size_t b = 0; b < batch; ++b) orc_rms_norm(&normed[b * hs], &hid[b * hs], M->final_norm.data(), hs, c.norm_eps);
  if (M->m.has_lm_head) {
    linear_matmul(M, M->m.lm_head, logits, normed.data(), batch);
  } else {
    const auto& E = M->m.embed;
    for (size_t b = 0; b < batch; ++b)
      orc_tied_lm_head(&logits[b * vs], &normed[b * hs], M->p(E.data_off), M->p(E.params_off), vs, hs, E.group_size);
  }
  if (c.final_logit_softcap > 0.f) {
    float cap = c.final_logit_softcap;
    for (size_t i = 0; i < batch * vs; ++i) logits[i] = cap * tanhf(logits[i] / cap);
  }
}

bool embed_tokens(orc_decoder* d, const uint32_t* ids, size_t n, float* out) {
  orc_model* M = d->model;
  const auto& E = M->m.embed;
  const auto& c = M->m.cfg;
  for (size_t i = 0; i < n; ++i) {
    if (ids[i] >= E.vocab) { g_err = "token id is out of model vocabulary"; return false; }
    orc_embed_lookup(out + i * E.hidden, ids[i], M->p(E.data_off), M->p(E.params_off), E.vocab, E.hidden, E.group_size);
    if (c.embed_scale != 1.0f)
      for (size_t j = 0; j < E.hidden; ++j) out[i * E.hidden + j] *= c.embed_scale;
  }
  return true;
}

}  // namespace

extern "C" {

orc_model* orc_model_open(const uint8_t* blob, size_t len, char* err, size_t err_len) {
  auto M = std::make_unique<orc_model>();
  M->blob.assign(blob, blob + len);
  std::string e;
  if (!raimodel::open(M->blob.data(), len, M->m, e)) {
    if (err && err_len) snprintf(err, err_len, "%s", e.c_str());
    g_err = e;
    return nullptr;
  }
  const auto& c = M->m.cfg;
  if (c.activation != 0) {
    g_err = "GeLU-tanh models are outside this oracle's scope";
    if (err && err_len) snprintf(err, err_len, "%s", g_err.c_str());
    return nullptr;
  }
  size_t half = c.head_dim / 2;
  M->rope_cos.resize((size_t)c.max_context * half);
  M->rope_sin.resize((size_t)c.max_context * half);
  orc_rope_table(M->rope_cos.data(), M->rope_sin.data(), c.head_dim, c.max_context, c.rope_theta,
                 c.rope_type, c.rope_factor, c.rope_low, c.rope_high, c.rope_orig_max);
  if (c.global_layer_stride > 0) {
    M->rope_local_cos.resize((size_t)c.max_context * half);
    M->rope_local_sin.resize((size_t)c.max_context * half);
    orc_rope_table(M->rope_local_cos.data(), M->rope_local_sin.data(), c.head_dim, c.max_context,
                   c.rope_local_theta, c.rope_type, c.rope_factor, c.rope_low, c.rope_high, c.rope_orig_max);
  }
  const uint8_t* b = M->blob.data();
  size_t nl = c.num_layers;
  M->in_norm.resize(nl); M->post_norm.resize(nl); M->q_norm.resize(nl); M->k_norm.resize(nl);
  M->attn_out_norm.resize(nl); M->mlp_out_norm.resize(nl); M->router.resize(nl);
  M->bias.assign(nl, std::vector<std::vector<float>>(7));
  for (size_t li = 0; li < nl; ++li) {
    const auto& L = M->m.layers[li];
    M->in_norm[li] = raimodel::read_vec(b, L.input_norm);
    M->post_norm[li] = raimodel::read_vec(b, L.post_attn_norm);
    if (L.q_norm.present) { M->q_norm[li] = raimodel::read_vec(b, L.q_norm); M->k_norm[li] = raimodel::read_vec(b, L.k_norm); }
    if (L.attn_out_norm.present) { M->attn_out_norm[li] = raimodel::read_vec(b, L.attn_out_norm); M->mlp_out_norm[li] = raimodel::read_vec(b, L.mlp_out_norm); }
    if (L.router.present) M->router[li] = raimodel::read_vec(b, L.router);
    for (int p = 0; p < 7; ++p)
      if (L.bias[p].present) M->bias[li][p] = raimodel::read_vec(b, L.bias[p]);
  }
  M->final_norm = raimodel::read_vec(b, M->m.final_norm);
  M->scale = c.attention_scale();
  return M.release();
}

void orc_model_free(orc_model* m) { delete m; }

void orc_model_config(const orc_model* M, uint32_t out[14]) {
  const auto& c = M->m.cfg;
  uint32_t v[14] = {c.hidden_size, c.num_layers, c.num_heads, c.num_kv_heads, c.head_dim,
                    c.intermediate_size, c.vocab_size, c.max_context, c.group_size,
                    c.embed_group_size, c.num_experts, c.experts_per_token,
                    (uint32_t)!M->m.has_lm_head, c.version};
  std::memcpy(out, v, sizeof(v));
}

// LookupDecoder::new (lookup.rs:192-209): context = min(max_ctx, model max).
orc_decoder* orc_decoder_new(orc_model* M, size_t max_ctx, char* err, size_t err_len) {
  const auto& c = M->m.cfg;
  size_t ctx = std::min<size_t>(max_ctx, c.max_context);
  if (ctx == 0) {
    g_err = "prompt-lookup context must be non-zero";
    if (err && err_len) snprintf(err, err_len, "%s", g_err.c_str());
    return nullptr;
  }
  auto d = std::make_unique<orc_decoder>();
  d->model = M;
  d->max_ctx = ctx;
  size_t per = (size_t)c.num_kv_heads * ctx * c.head_dim;
  d->k.assign(c.num_layers, std::vector<float>(per, 0.f));
  d->v.assign(c.num_layers, std::vector<float>(per, 0.f));
  d->filled.assign(c.num_layers, 0);
  return d.release();
}

void orc_decoder_free(orc_decoder* d) { delete d; }

// LookupDecoder::prefill (lookup.rs:219-247).
int orc_prefill(orc_decoder* d, const uint32_t* ids, size_t n, size_t* pos_out) {
  if (n == 0) { g_err = "prompt must contain at least one token"; return -1; }
  if (n > d->max_ctx) { g_err = "prompt exceeds the prompt-lookup context window"; return -1; }
  size_t m = n - 1;
  *pos_out = m;
  if (m == 0) return 0;
  size_t hs = d->model->m.cfg.hidden_size;
  std::vector<float> hid(m * hs);
  if (!embed_tokens(d, ids, m, hid.data())) return -1;
  std::vector<size_t> positions(m);
  for (size_t i = 0; i < m; ++i) positions[i] = i;
  return forward_batch(d, hid.data(), positions.data(), m) ? 0 : -1;
}

// Embed `batch` tokens at consecutive positions, run forward_batch and
// hidden_to_logits_batch; `logits` may be null.
int orc_forward_logits(orc_decoder* d, const uint32_t* ids, size_t start_pos, size_t batch, float* logits) {
  size_t hs = d->model->m.cfg.hidden_size;
  std::vector<float> hid(batch * hs);
  if (!embed_tokens(d, ids, batch, hid.data())) return -1;
  std::vector<size_t> positions(batch);
  for (size_t i = 0; i < batch; ++i) positions[i] = start_pos + i;
  if (!forward_batch(d, hid.data(), positions.data(), batch)) return -1;
  if (logits) hidden_to_logits(d, hid.data(), batch, logits);
  return 0;
}

// LookupDecoder::step (lookup.rs:260-425) with greedy acceptance: the
// temperature -> 0 limit of the exact rule (accept d_i iff argmax_i == d_i;
// the correction and the bonus are argmaxes). metrics = {accepted, drafted,
// produced, matched_ngram (0 = none)}.
int orc_step_greedy(orc_decoder* d, size_t pos, const uint32_t* ctx, size_t ctx_len, size_t max_draft,
                    size_t max_ngram, size_t min_ngram, uint32_t* out, size_t* n_out, size_t metrics[4]) {
  const auto& c = d->model->m.cfg;
  if (max_draft == 0) { g_err = "prompt-lookup max_draft must be non-zero"; return -1; }
  if (!(min_ngram >= 1 && min_ngram <= max_ngram)) { g_err = "prompt-lookup requires 1 <= min_ngram <= max_ngram"; return -1; }
  if (ctx_len == 0) { g_err = "prompt-lookup step requires a non-empty context"; return -1; }
  if (pos >= d->max_ctx) { g_err = "decode position exceeds the context window"; return -1; }
  uint32_t last = ctx[ctx_len - 1];
  size_t budget = d->max_ctx > pos + 1 ? d->max_ctx - pos - 1 : 0;
  size_t ng = 0, ds = 0, dl = 0;
  int found = budget == 0 ? 0 : orc_find_ngram_draft(ctx, ctx_len, min_ngram, max_ngram, std::min(max_draft, budget), &ng, &ds, &dl);
  size_t vs = c.vocab_size;
  if (!found) {
    std::vector<float> logits(vs);
    if (orc_forward_logits(d, &last, pos, 1, logits.data()) != 0) return -1;
    out[0] = (uint32_t)orc_argmax(logits.data(), vs);
    *n_out = 1;
    metrics[0] = 0; metrics[1] = 0; metrics[2] = 1; metrics[3] = 0;
    return 0;
  }
  for (size_t i = 0; i < dl; ++i)
    if (ctx[ds + i] >= vs) { g_err = "context contains a token outside the model vocabulary"; return -1; }
  size_t batch = dl + 1;
  std::vector<uint32_t> vt(batch);
  vt[0] = last;
  for (size_t i = 0; i < dl; ++i) vt[1 + i] = ctx[ds + i];
  std::vector<float> logits(batch * vs);
  if (orc_forward_logits(d, vt.data(), pos, batch, logits.data()) != 0) return -1;
  size_t produced = 0, accepted = 0;
  for (size_t i = 0; i < dl; ++i) {
    uint32_t target = (uint32_t)orc_argmax(&logits[i * vs], vs);
    out[produced++] = target;
    if (target != vt[1 + i]) break;
    ++accepted;
  }
  if (accepted == dl) out[produced++] = (uint32_t)orc_argmax(&logits[dl * vs], vs);
  orc_kv_truncate(d, pos + produced);
  *n_out = produced;
  metrics[0] = accepted; metrics[1] = dl; metrics[2] = produced; metrics[3] = ng;
  return 0;
}

size_t orc_kv_filled(const orc_decoder* d, size_t layer) { return d->filled[layer]; }

// KVCache::truncate (kv_cache.rs:300-304).
void orc_kv_truncate(orc_decoder* d, size_t len) {
  for (auto& f : d->filled) f = std::min(f, len);
}

int orc_kv_read(const orc_decoder* d, size_t layer, size_t kvh, size_t pos, float* k, float* v) {
  const auto& c = d->model->m.cfg;
  if (layer >= c.num_layers || kvh >= c.num_kv_heads || pos >= d->filled[layer]) return -1;
  size_t hd = c.head_dim;
  std::memcpy(k, &d->k[layer][(kvh * d->max_ctx + pos) * hd], hd * 4);
  std::memcpy(v, &d->v[layer][(kvh * d->max_ctx + pos) * hd], hd * 4);
  return 0;
}

}  // extern "C"
