// .raimodel container reader (host side, header-only C++17).
//
// Restates the validated reader of rai-infer/src/format.rs: header parse
// (format.rs:1098-1183), the v2 capability block (format.rs:1192-1365),
// config validation (format.rs:1376-1480), the section table checks of
// RaiModelFile::open (format.rs:557-637), per-layer slicing
// (RaiModelFile::layer, format.rs:826-1006), the embedding / final norm /
// lm_head sections (format.rs:801-824, 1012-1082), the expert walk of
// LayerRefs::expert (format.rs:436-477) and validate_layout
// (format.rs:686-785).
//
// Views are byte offsets into the caller's blob, so the same description
// serves the host oracle (which reads the blob in place) and the device
// loader (which uploads the blob once and repacks from device offsets).
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace raimodel {

constexpr uint32_t kFormatVersion = 2;
constexpr size_t kHeaderV1 = 64;
constexpr size_t kHeaderV2 = 128;
constexpr size_t kSectionEntry = 16;
constexpr int kNumProjections = 7;
// Kernel group capacity (rai-infer/src/gemm.rs:1167, MAX_GROUPS).
constexpr size_t kMaxGroups = 128;
// RoPE table budget (rai-infer/src/layers.rs:27, MAX_ROPE_TABLE_BYTES).
constexpr size_t kMaxRopeTableBytes = 512ull * 1024 * 1024;

constexpr uint8_t kFlagBiases = 0x01;
constexpr uint8_t kFlagQkNorm = 0x02;
constexpr uint8_t kFlagSandwich = 0x04;
constexpr uint8_t kFlagFullQkNorm = 0x08;
constexpr uint8_t kFlagPostNorm = 0x10;
constexpr uint8_t kKnownFlags = 0x1F;

enum Proj { Q = 0, K = 1, V = 2, O = 3, GATE = 4, UP = 5, DOWN = 6 };

struct Config {
  uint32_t hidden_size = 0, num_layers = 0, num_heads = 0, num_kv_heads = 0;
  uint32_t head_dim = 0, intermediate_size = 0, vocab_size = 0, max_context = 0;
  float rope_theta = 0.f, norm_eps = 0.f;
  uint8_t bits = 0, group_size = 0, embed_bits = 0, embed_group_size = 0;
  uint32_t version = 0;
  uint8_t activation = 0;  // 0 SiLU, 1 GeLU-tanh
  uint8_t rope_type = 0;   // 0 default, 1 llama3
  float rope_factor = 0.f, rope_low = 0.f, rope_high = 0.f;
  uint32_t rope_orig_max = 0;
  uint8_t bias_mask = 0;
  float embed_scale = 1.f;
  bool has_qk_norm = false, has_sandwich_norm = false, has_full_qk_norm = false;
  bool post_norm = false;
  float rope_local_theta = 0.f;
  uint8_t global_layer_stride = 0;
  uint16_t num_experts = 0;
  uint8_t experts_per_token = 0;
  bool norm_topk_prob = false;
  float attn_logit_softcap = 0.f, final_logit_softcap = 0.f, attn_scale = 0.f;

  bool has_bias(int i) const { return i < kNumProjections && (bias_mask & (1u << i)); }
  size_t q_dim() const { return (size_t)num_heads * head_dim; }
  size_t kv_dim() const { return (size_t)num_kv_heads * head_dim; }
  // ModelConfig::attention_scale (format.rs:275-281).
  float attention_scale() const {
    if (attn_scale > 0.f) return attn_scale;
    return 1.0f / std::sqrt((float)head_dim);  // f32 sqrt then f32 divide
  }
  // (rows, cols) of the seven projections, ModelConfig::projection_dims.
  void projection_dims(size_t rows[7], size_t cols[7]) const {
    size_t h = hidden_size, ff = intermediate_size, q = q_dim(), kv = kv_dim();
    size_t r[7] = {q, kv, kv, h, ff, ff, h};
    size_t c[7] = {h, h, h, q, h, h, ff};
    for (int i = 0; i < 7; ++i) { rows[i] = r[i]; cols[i] = c[i]; }
  }
};

// A quantized linear: [u32 rows][u32 cols][params rows*G*4][nibbles rows*cols/2].
struct Linear {
  size_t rows = 0, cols = 0, group_size = 0;
  size_t params_off = 0, params_len = 0;  // f16 (scale, zero) per (row, group)
  size_t nib_off = 0, nib_len = 0;        // low nibble = even column
  size_t num_groups() const { return (cols + group_size - 1) / group_size; }
};

struct Vec32 {  // raw little-endian f32 vector inside the blob
  size_t off = 0, len = 0;  // len in values
  bool present = false;
};

struct Layer {
  Linear proj[7];
  Vec32 bias[7];
  Vec32 q_norm, k_norm, attn_out_norm, mlp_out_norm, router;
  Vec32 input_norm, post_attn_norm;
  std::vector<Linear> experts;  // 3 * (num_experts - 1): gate, up, down of experts 1..
};

struct Embedding {
  size_t vocab = 0, hidden = 0, group_size = 0;
  size_t params_off = 0, data_off = 0;
};

struct Model {
  Config cfg;
  size_t num_sections = 0;
  size_t header_size = 0;
  std::vector<std::pair<uint64_t, uint64_t>> sections;
  Embedding embed;
  std::vector<Layer> layers;
  Vec32 final_norm;
  bool has_lm_head = false;
  Linear lm_head;
};

namespace detail {
inline uint32_t rd_u32(const uint8_t* p) { uint32_t v; std::memcpy(&v, p, 4); return v; }
inline uint64_t rd_u64(const uint8_t* p) { uint64_t v; std::memcpy(&v, p, 8); return v; }
inline float rd_f32(const uint8_t* p) { float v; std::memcpy(&v, p, 4); return v; }
inline uint16_t rd_u16(const uint8_t* p) { uint16_t v; std::memcpy(&v, p, 2); return v; }

// Exact IEEE half -> float (the `half` crate's f16::to_f32).
inline float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
  if (exp == 0) {
    if (man == 0) bits = sign;
    else {  // subnormal: normalise
      int e = -1;
      do { man <<= 1; ++e; } while (!(man & 0x400));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
    }
  } else if (exp == 31) bits = sign | 0x7F800000u | (man << 13);
  else bits = sign | ((exp + 112) << 23) | (man << 13);
  float f; std::memcpy(&f, &bits, 4); return f;
}

inline bool mul_ok(size_t a, size_t b, size_t* out) { return !__builtin_mul_overflow(a, b, out); }
inline bool add_ok(size_t a, size_t b, size_t* out) { return !__builtin_add_overflow(a, b, out); }
}  // namespace detail

// Parses the header; returns false with `err` set on any violation.
inline bool parse_header(const uint8_t* d, size_t n, Config& c, size_t& num_sections,
                         size_t& header_size, std::string& err) {
  using namespace detail;
  if (n < kHeaderV1) { err = "file too small for header: " + std::to_string(n) + " bytes"; return false; }
  if (std::memcmp(d, "RAIM", 4) != 0) { err = "not a .raimodel file: bad magic"; return false; }
  c.version = rd_u32(d + 4);
  if (c.version == 1) header_size = kHeaderV1;
  else if (c.version == 2) header_size = kHeaderV2;
  else { err = "unsupported format version: " + std::to_string(c.version); return false; }
  if (n < header_size) { err = "file too small for a v" + std::to_string(c.version) + " header"; return false; }
  c.hidden_size = rd_u32(d + 8); c.num_layers = rd_u32(d + 12); c.num_heads = rd_u32(d + 16);
  c.num_kv_heads = rd_u32(d + 20); c.head_dim = rd_u32(d + 24); c.intermediate_size = rd_u32(d + 28);
  c.vocab_size = rd_u32(d + 32); c.max_context = rd_u32(d + 36);
  c.rope_theta = rd_f32(d + 40); c.norm_eps = rd_f32(d + 44);
  c.bits = d[48]; c.group_size = d[49]; c.embed_bits = d[50]; c.embed_group_size = d[51];
  if (c.version >= 2) {
    for (int i = 56; i < 64; ++i) if (d[i]) { err = "header bytes 56..64 are reserved and must be zero"; return false; }
    for (size_t i = 109; i < kHeaderV2; ++i) if (d[i]) { err = "header bytes 109..128 are reserved and must be zero"; return false; }
    c.activation = d[64];
    if (c.activation > 1) { err = "unsupported activation code " + std::to_string(c.activation); return false; }
    uint8_t flags = d[65];
    if (flags & ~kKnownFlags) { err = "header flags set bits this reader does not implement"; return false; }
    uint8_t bias_mask = d[67];
    if (bias_mask & ~0x7F) { err = "bias_mask sets bits beyond the 7 projections"; return false; }
    if (((flags & kFlagBiases) != 0) != (bias_mask != 0)) { err = "header is inconsistent: bias flag disagrees with bias_mask"; return false; }
    c.bias_mask = bias_mask;
    c.has_qk_norm = flags & kFlagQkNorm; c.has_sandwich_norm = flags & kFlagSandwich;
    c.has_full_qk_norm = flags & kFlagFullQkNorm; c.post_norm = flags & kFlagPostNorm;
    if (c.has_qk_norm && c.has_full_qk_norm) { err = "header sets both per-head and full-width QK norm"; return false; }
    if (c.has_sandwich_norm && c.post_norm) { err = "header sets both sandwich norms and post-norm placement"; return false; }
    c.rope_type = d[66];
    float factor = rd_f32(d + 68), low = rd_f32(d + 72), high = rd_f32(d + 76);
    uint32_t orig = rd_u32(d + 80);
    if (c.rope_type == 0) {
      if (factor != 0.f || low != 0.f || high != 0.f || orig != 0) { err = "rope_type 0 (default) must leave the RoPE scaling parameters zero"; return false; }
    } else if (c.rope_type == 1) {
      for (float v : {factor, low, high})
        if (!std::isfinite(v) || v <= 0.f) { err = "llama3 RoPE parameters must be finite and positive"; return false; }
      if (std::fabs(high - low) == 0.f) { err = "llama3 RoPE high_freq_factor must differ from low_freq_factor"; return false; }
      if (orig == 0 || orig > 1000000u) { err = "llama3 RoPE original_max_position_embeddings out of range"; return false; }
      c.rope_factor = factor; c.rope_low = low; c.rope_high = high; c.rope_orig_max = orig;
    } else { err = "unsupported rope_type " + std::to_string(c.rope_type); return false; }
    c.embed_scale = rd_f32(d + 84);
    if (!std::isfinite(c.embed_scale) || c.embed_scale <= 0.f) { err = "embed_scale must be finite and positive"; return false; }
    auto opt_pos = [&](size_t off, const char* name, float& out) {
      float v = rd_f32(d + off);
      if (!std::isfinite(v) || v < 0.f) { err = std::string(name) + " must be finite and non-negative"; return false; }
      out = v; return true;
    };
    if (!opt_pos(88, "attn_logit_softcap", c.attn_logit_softcap)) return false;
    if (!opt_pos(92, "final_logit_softcap", c.final_logit_softcap)) return false;
    if (!opt_pos(96, "attn_scale", c.attn_scale)) return false;
    c.num_experts = rd_u16(d + 105); c.experts_per_token = d[107];
    uint8_t moe_flags = d[108];
    if (moe_flags & ~0x01) { err = "moe_flags sets bits this reader does not implement"; return false; }
    c.norm_topk_prob = moe_flags & 0x01;
    if (c.num_experts == 0) {
      if (c.experts_per_token != 0 || moe_flags != 0) { err = "header declares no experts but sets experts_per_token or moe_flags"; return false; }
    } else {
      if (c.num_experts < 2) { err = "header declares 1 expert; a dense MLP is stored with num_experts = 0"; return false; }
      if (c.experts_per_token == 0 || c.experts_per_token > c.num_experts) { err = "experts_per_token out of range"; return false; }
    }
    if (!opt_pos(100, "rope_local_theta", c.rope_local_theta)) return false;
    c.global_layer_stride = d[104];
    if ((c.rope_local_theta > 0.f) != (c.global_layer_stride > 0)) { err = "per-layer RoPE needs both rope_local_theta and global_layer_stride or neither"; return false; }
    if (c.global_layer_stride == 1) { err = "global_layer_stride of 1 makes every layer global"; return false; }
  }
  // validate_config (format.rs:1376-1480)
  struct B { const char* n; uint32_t v, m; } bounds[] = {
      {"hidden_size", c.hidden_size, 65536}, {"num_layers", c.num_layers, 1024},
      {"num_heads", c.num_heads, 1024}, {"num_kv_heads", c.num_kv_heads, 1024},
      {"head_dim", c.head_dim, 65536}, {"intermediate_size", c.intermediate_size, 1048576},
      {"vocab_size", c.vocab_size, 10000000}, {"max_context", c.max_context, 1000000}};
  for (auto& b : bounds)
    if (b.v == 0 || b.v > b.m) { err = std::string("invalid ") + b.n + ": " + std::to_string(b.v); return false; }
  if (c.bits != 4) { err = "unsupported weight bit width " + std::to_string(c.bits) + "; expected 4"; return false; }
  if (c.embed_bits != 8) { err = "unsupported embedding bit width; expected 8"; return false; }
  if (c.group_size == 0 || c.embed_group_size == 0) { err = "quantization group sizes must be non-zero"; return false; }
  if ((c.group_size & 1) || (c.embed_group_size & 1)) { err = "quantization group sizes must be even"; return false; }
  if ((c.hidden_size & 1) || (c.intermediate_size & 1)) { err = "hidden and intermediate dimensions must be even"; return false; }
  if (c.head_dim % 8) { err = "head_dim must be a multiple of 8"; return false; }
  if (c.num_heads % c.num_kv_heads) { err = "num_heads must be divisible by num_kv_heads"; return false; }
  size_t adim = c.q_dim();
  if (adim > 1048576) { err = "num_heads * head_dim exceeds the maximum"; return false; }
  if (adim & 1) { err = "num_heads * head_dim must be even"; return false; }
  size_t gs = c.group_size;
  size_t mg = (c.hidden_size + gs - 1) / gs;
  mg = std::max(mg, (c.intermediate_size + gs - 1) / gs);
  mg = std::max(mg, (adim + gs - 1) / gs);
  if (mg > kMaxGroups) { err = "model requires " + std::to_string(mg) + " quantization groups; kernel maximum is 128"; return false; }
  if ((c.hidden_size + c.embed_group_size - 1) / c.embed_group_size > kMaxGroups) { err = "embedding requires too many quantization groups"; return false; }
  if (!std::isfinite(c.rope_theta) || c.rope_theta <= 0.f) { err = "rope_theta must be finite and positive"; return false; }
  if (!std::isfinite(c.norm_eps) || c.norm_eps <= 0.f) { err = "norm_eps must be finite and positive"; return false; }
  if ((size_t)c.max_context * (c.head_dim / 2) * 2 * 4 > kMaxRopeTableBytes) { err = "RoPE table exceeds budget"; return false; }
  num_sections = rd_u32(d + 52);
  if (num_sections != c.num_layers + 2ull && num_sections != c.num_layers + 3ull) {
    err = "invalid section count " + std::to_string(num_sections); return false;
  }
  return true;
}

namespace detail {
inline bool read_linear(const uint8_t* blob, size_t sec_off, size_t sec_len, size_t& off,
                        size_t er, size_t ec, size_t gs, const std::string& label, Linear& L,
                        std::string& err) {
  size_t hdr_end;
  if (!add_ok(off, 8, &hdr_end) || hdr_end > sec_len) { err = label + ": linear header truncated"; return false; }
  size_t r = rd_u32(blob + sec_off + off), c = rd_u32(blob + sec_off + off + 4);
  if (r != er || c != ec) {
    err = label + ": linear is [" + std::to_string(r) + ", " + std::to_string(c) + "], expected [" +
          std::to_string(er) + ", " + std::to_string(ec) + "]";
    return false;
  }
  size_t ng = (c + gs - 1) / gs, plen, elems, nlen, end;
  if (!mul_ok(r, ng, &plen) || !mul_ok(plen, 4, &plen) || !mul_ok(r, c, &elems)) { err = label + ": size overflows"; return false; }
  nlen = (elems + 1) / 2;
  if (!add_ok(hdr_end, plen, &end) || !add_ok(end, nlen, &end) || end > sec_len) { err = label + ": linear data truncated"; return false; }
  L.rows = r; L.cols = c; L.group_size = gs;
  L.params_off = sec_off + hdr_end; L.params_len = plen;
  L.nib_off = sec_off + hdr_end + plen; L.nib_len = nlen;
  off = end;
  return true;
}

inline bool take_vec(size_t sec_off, size_t sec_len, size_t& off, size_t values,
                     const std::string& label, Vec32& v, std::string& err) {
  size_t bytes, end;
  if (!mul_ok(values, 4, &bytes) || !add_ok(off, bytes, &end) || end > sec_len) { err = label + " truncated"; return false; }
  v.off = sec_off + off; v.len = values; v.present = true; off = end;
  return true;
}

inline bool finite_vec(const uint8_t* blob, const Vec32& v, const std::string& label, std::string& err) {
  for (size_t i = 0; i < v.len; ++i)
    if (!std::isfinite(rd_f32(blob + v.off + 4 * i))) { err = label + " weight " + std::to_string(i) + " is non-finite"; return false; }
  return true;
}

inline bool valid_params(const uint8_t* blob, size_t off, size_t len, const std::string& label, std::string& err) {
  if (len % 4) { err = label + " quantization parameters are misaligned"; return false; }
  for (size_t i = 0; i < len / 4; ++i) {
    float s = f16_to_f32(rd_u16(blob + off + 4 * i)), z = f16_to_f32(rd_u16(blob + off + 4 * i + 2));
    if (!std::isfinite(s) || s <= 0.f || !std::isfinite(z)) {
      err = label + " quantization group " + std::to_string(i) + " contains an invalid scale or zero point";
      return false;
    }
  }
  return true;
}
}  // namespace detail

// Full open: header, section table, every section sliced and validated.
inline bool open(const uint8_t* blob, size_t n, Model& m, std::string& err) {
  using namespace detail;
  if (!parse_header(blob, n, m.cfg, m.num_sections, m.header_size, err)) return false;
  const Config& c = m.cfg;
  size_t table_end = m.header_size + m.num_sections * kSectionEntry;
  if (n < table_end) { err = "file too small for section table"; return false; }
  size_t prev = table_end;
  m.sections.clear();
  for (size_t i = 0; i < m.num_sections; ++i) {
    const uint8_t* e = blob + m.header_size + i * kSectionEntry;
    uint64_t off = rd_u64(e), sz = rd_u64(e + 8), end;
    if (sz == 0) { err = "section " + std::to_string(i) + " is empty"; return false; }
    if (off != prev) { err = "section " + std::to_string(i) + " is not contiguous"; return false; }
    if (__builtin_add_overflow(off, sz, &end) || end > n) { err = "section " + std::to_string(i) + " extends beyond file"; return false; }
    prev = end;
    m.sections.push_back({off, sz});
  }
  if (prev != n) { err = "unreferenced trailing data after the final section"; return false; }

  // Embedding (section 0).
  {
    size_t so = m.sections[0].first, sl = m.sections[0].second;
    size_t gs = c.embed_group_size, ng = (c.hidden_size + gs - 1) / gs;
    size_t plen = (size_t)c.vocab_size * ng * 4, dlen = (size_t)c.vocab_size * c.hidden_size;
    if (sl != plen + dlen) { err = "embedding section size mismatch"; return false; }
    m.embed = {c.vocab_size, c.hidden_size, gs, so, so + plen};
    if (!valid_params(blob, so, plen, "embedding", err)) return false;
  }
  size_t rows[7], cols[7];
  c.projection_dims(rows, cols);
  static const char* names[7] = {"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"};
  m.layers.assign(c.num_layers, Layer{});
  for (size_t li = 0; li < c.num_layers; ++li) {
    Layer& L = m.layers[li];
    size_t so = m.sections[1 + li].first, sl = m.sections[1 + li].second, off = 0;
    std::string lab = "layer " + std::to_string(li);
    for (int p = 0; p < 7; ++p) {
      if (!read_linear(blob, so, sl, off, rows[p], cols[p], c.group_size, lab + ": " + names[p], L.proj[p], err)) return false;
      if (!valid_params(blob, L.proj[p].params_off, L.proj[p].params_len, lab + " " + names[p], err)) return false;
    }
    for (int p = 0; p < 7; ++p) {
      if (!c.has_bias(p)) continue;
      if (!take_vec(so, sl, off, rows[p], lab + ": " + names[p] + " bias", L.bias[p], err)) return false;
      if (!finite_vec(blob, L.bias[p], lab + " " + names[p] + " bias", err)) return false;
    }
    if (c.has_qk_norm || c.has_full_qk_norm) {
      size_t qn = c.has_full_qk_norm ? c.q_dim() : c.head_dim, kn = c.has_full_qk_norm ? c.kv_dim() : c.head_dim;
      if (!take_vec(so, sl, off, qn, lab + ": q_norm", L.q_norm, err)) return false;
      if (!take_vec(so, sl, off, kn, lab + ": k_norm", L.k_norm, err)) return false;
      if (!finite_vec(blob, L.q_norm, lab + " q_norm", err) || !finite_vec(blob, L.k_norm, lab + " k_norm", err)) return false;
    }
    if (c.has_sandwich_norm) {
      if (!take_vec(so, sl, off, c.hidden_size, lab + ": attention output norm", L.attn_out_norm, err)) return false;
      if (!take_vec(so, sl, off, c.hidden_size, lab + ": MLP output norm", L.mlp_out_norm, err)) return false;
      if (!finite_vec(blob, L.attn_out_norm, lab + " attention output norm", err) ||
          !finite_vec(blob, L.mlp_out_norm, lab + " MLP output norm", err)) return false;
    }
    if (c.num_experts > 0) {
      size_t relems;
      if (!mul_ok(c.num_experts, c.hidden_size, &relems)) { err = lab + ": router size overflows"; return false; }
      if (!take_vec(so, sl, off, relems, lab + ": router", L.router, err)) return false;
      L.experts.resize(3 * (c.num_experts - 1));
      for (size_t e = 1; e < c.num_experts; ++e)
        for (int p = 0; p < 3; ++p) {
          Linear& X = L.experts[3 * (e - 1) + p];
          if (!read_linear(blob, so, sl, off, rows[4 + p], cols[4 + p], c.group_size,
                           lab + ": expert " + std::to_string(e) + " " + names[4 + p], X, err)) return false;
        }
    }
    size_t nb = (size_t)c.hidden_size * 4;
    if (off + 2 * nb != sl) { err = lab + ": section size mismatch"; return false; }
    L.input_norm = {so + off, c.hidden_size, true};
    L.post_attn_norm = {so + off + nb, c.hidden_size, true};
    if (!finite_vec(blob, L.input_norm, lab + " input norm", err) ||
        !finite_vec(blob, L.post_attn_norm, lab + " pre-MLP norm", err)) return false;
  }
  {
    size_t idx = 1 + c.num_layers;
    if (m.sections[idx].second != (size_t)c.hidden_size * 4) { err = "final norm section size mismatch"; return false; }
    m.final_norm = {m.sections[idx].first, c.hidden_size, true};
    if (!finite_vec(blob, m.final_norm, "final norm", err)) return false;
  }
  m.has_lm_head = m.num_sections == c.num_layers + 3ull;
  if (m.has_lm_head) {
    size_t so = m.sections.back().first, sl = m.sections.back().second, off = 0;
    if (!read_linear(blob, so, sl, off, c.vocab_size, c.hidden_size, c.group_size, "lm_head", m.lm_head, err)) return false;
    if (off != sl) { err = "lm_head section size mismatch"; return false; }
    if (!valid_params(blob, m.lm_head.params_off, m.lm_head.params_len, "lm_head", err)) return false;
  }
  return true;
}

inline std::vector<float> read_vec(const uint8_t* blob, const Vec32& v) {
  std::vector<float> out(v.len);
  if (v.len) std::memcpy(out.data(), blob + v.off, v.len * 4);
  return out;
}

}  // namespace raimodel
