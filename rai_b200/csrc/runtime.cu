// C ABI (include/rai_gpu.h): model upload, decoder state, the forward pass
// and the CUDA-graph decode step.
//
// The step restates LookupDecoder::step (rai-infer/src/lookup.rs:260-425)
// entirely on the device: ngram_kernel drafts from the device copy of the
// context, the verify forward runs over a fixed row budget of max_draft + 1
// with the active row count read from device memory, accept_kernel applies
// greedy acceptance and rolls the KV watermark back. The host copies the
// context in, replays one CUDA graph and reads one small struct back.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <gnu/libc-version.h>

#include <algorithm>
#include <fstream>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/rai_gpu.h"
#include "common.cuh"
#include "kernels.h"
#include "layers.h"
#include "moe.h"
#include "raimodel_format.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

// On failure the runtime's (non-sticky) last-error slot is cleared so the
// next launch check does not report this error again.
#define RAI_CUDA(call)                                                                        \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess) {                                                                  \
      (void)cudaGetLastError();                                                               \
      return fail(e_ == cudaErrorMemoryAllocation ? RAI_ERR_OOM : RAI_ERR_DEVICE,             \
                  std::string(#call) + ": " + cudaGetErrorString(e_));                        \
    }                                                                                         \
  } while (0)

using raimodel::Config;
using rai::ActBuf;
using rai::PackedLinear;

// RoPETable::with_scaling + apply_llama3_scaling (rai-infer/src/layers.rs:
// 561-633, 760-808), built on the host with the same f32 libm calls the
// reference makes, then uploaded.
void build_rope(const Config& c, float theta, std::vector<float>& cs, std::vector<float>& sn) {
  size_t hd = c.head_dim, half = hd / 2, mc = c.max_context;
  std::vector<float> inv(half);
  for (size_t i = 0; i < half; ++i) {
    float e = 2.0f * (float)i / (float)hd;
    inv[i] = 1.0f / powf(theta, e);
  }
  if (c.rope_type == 1) {
    float old_ctx = (float)c.rope_orig_max;
    float low_wl = old_ctx / c.rope_low, high_wl = old_ctx / c.rope_high;
    const float two_pi = 2.0f * 3.14159265358979323846f;
    for (size_t i = 0; i < half; ++i) {
      float v = inv[i];
      float wl = two_pi / v;
      float banded = wl > low_wl ? v / c.rope_factor : v;
      if (wl >= high_wl && wl <= low_wl) {
        float smooth = (old_ctx / wl - c.rope_low) / (c.rope_high - c.rope_low);
        float a = (1.0f - smooth) * banded;
        a = a / c.rope_factor;
        float b = smooth * banded;
        inv[i] = a + b;
      } else {
        inv[i] = banded;
      }
    }
  }
  cs.resize(mc * half);
  sn.resize(mc * half);
  for (size_t p = 0; p < mc; ++p)
    for (size_t i = 0; i < half; ++i) {
      float ang = (float)p * inv[i];
      cs[p * half + i] = cosf(ang);
      sn[p * half + i] = sinf(ang);
    }
}

}  // namespace

struct LayerDev {
  PackedLinear qkv, o, gateup, down;
  // Mixture-of-experts layers: every expert's gate|up and down packed back to
  // back (expert e at data + e * stride); router [ne][hidden] f32.
  bool moe = false;
  PackedLinear x_gateup, x_down;
  size_t x_gu_stride = 0, x_dn_stride = 0;
  float* router = nullptr;
  float* bias_qkv = nullptr;
  float* in_norm = nullptr;
  float* post_norm = nullptr;
  float* q_norm = nullptr;
  float* k_norm = nullptr;
};

struct rai_model {
  int device = 0;
  Config cfg;
  raimodel::Model layout;
  std::vector<void*> allocs;
  std::vector<LayerDev> layers;
  PackedLinear head;
  uint8_t* embed_codes = nullptr;
  uint8_t* embed_params = nullptr;
  float* final_norm = nullptr;
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  float scale = 0.f;
  int qk_mode = 0;  // 0 none, 1 per head, 2 full width
  size_t device_bytes = 0;
  uint32_t* err_dev = nullptr;
  rai::ExpfTable expf;

  // Tensor parallelism (tp_world > 1): this rank's shard of every linear
  // (whole output rows), and the exchange arena every rank maps.
  int tp_rank = 0, tp_world = 1;
  int nh_l = 0, nkv_l = 0, ff_l = 0;  // heads / ff columns this rank computes
  int h_l = 0;                         // o / down output rows per rank (hidden slice)
  int v_l = 0, v_off = 0;              // LM head rows of this rank
  // Mixture-of-experts models split by experts instead (expert parallel):
  // rank r holds experts e0 .. e0 + ne_l; attention and the head are whole.
  bool ep = false;
  int ne_l = 0, e0 = 0;
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0, arena_used = 0, flags_used = 0;
  uint8_t* peer_arena[rai::kMaxTp] = {};
  bool tp_connected = false;
  std::vector<void*> ipc_opened;
  // Set when a cross-GPU wait of this multi-GPU model timed out: the ranks'
  // exchange counters no longer agree on how many forwards ran, so a later
  // wait could pass on a peer's counts from another forward. The model
  // refuses all further work; every rank must destroy and re-create its model
  // together (fresh arenas, counters at zero).
  bool failed = false;
  // Kernel choice of the dense 4-bit linears (rai::GemmMode; RAI_GEMM_MODE
  // = exact | auto | tol sets the default, exact unless set). Multi-GPU
  // models run exact.
  int gemm_mode = rai::kGemmExact;
  // Decoders created on this model and not yet destroyed: the model refuses
  // to be destroyed under them (their teardown reads the model).
  std::atomic<int> live_decoders{0};

  template <class T>
  int alloc(T** p, size_t bytes) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
    if (e != cudaSuccess)
      return fail(RAI_ERR_OOM, "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    allocs.push_back(q);
    device_bytes += bytes;
    *p = static_cast<T*>(q);
    return RAI_OK;
  }
  ~rai_model() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    for (void* p : ipc_opened) cudaIpcCloseMemHandle(p);
    for (void* p : allocs) cudaFree(p);
    cudaSetDevice(prev);
  }
};

namespace {

// Scoped device switch for entry points.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

int upload(rai_model* M, const void* host, size_t bytes, void** dev) {
  uint8_t* p = nullptr;
  int rc = M->alloc(&p, bytes);
  if (rc) return rc;
  RAI_CUDA(cudaMemcpy(p, host, bytes, cudaMemcpyHostToDevice));
  *dev = p;
  return RAI_OK;
}

int upload_vec(rai_model* M, const uint8_t* blob, const raimodel::Vec32& v, float** dev) {
  std::vector<float> h = raimodel::read_vec(blob, v);
  return upload(M, h.data(), h.size() * 4, reinterpret_cast<void**>(dev));
}

// Rows row0 .. row0 + rows of a raw linear (all of it by default). Codes are
// [rows][cols/2] and params [rows][groups][4], so a row range is contiguous.
struct RowRange {
  const raimodel::Linear* L;
  size_t row0, rows;
};
RowRange whole(const raimodel::Linear* L) { return RowRange{L, 0, L->rows}; }

// Pack one or more raw row ranges with the same cols into one device linear
// (rows concatenated in order).
int pack_concat(rai_model* M, const uint8_t* blob_dev, const std::vector<RowRange>& parts, PackedLinear* out,
                uint8_t* dst = nullptr) {
  size_t cols = parts[0].L->cols, gs = parts[0].L->group_size, ng = parts[0].L->num_groups();
  size_t rows = 0;
  for (auto& p : parts) rows += p.rows;
  uint8_t* packed = dst;
  if (!packed)
    if (int rc = M->alloc(&packed, rai::packed_linear_bytes(rows, cols, gs))) return rc;
  const uint8_t *nib = nullptr, *par = nullptr;
  void* tmp = nullptr;
  if (parts.size() == 1) {
    nib = blob_dev + parts[0].L->nib_off + parts[0].row0 * (cols / 2);
    par = blob_dev + parts[0].L->params_off + parts[0].row0 * ng * 4;
  } else {
    size_t nb = rows * cols / 2, pb = rows * ng * 4;
    RAI_CUDA(cudaMalloc(&tmp, nb + pb));
    uint8_t* t = static_cast<uint8_t*>(tmp);
    size_t no = 0, po = 0;
    for (auto& p : parts) {
      const size_t nl = p.rows * (cols / 2), pl = p.rows * ng * 4;
      RAI_CUDA(cudaMemcpy(t + no, blob_dev + p.L->nib_off + p.row0 * (cols / 2), nl, cudaMemcpyDeviceToDevice));
      RAI_CUDA(cudaMemcpy(t + nb + po, blob_dev + p.L->params_off + p.row0 * ng * 4, pl, cudaMemcpyDeviceToDevice));
      no += nl;
      po += pl;
    }
    nib = t;
    par = t + nb;
  }
  RAI_CUDA(rai::pack_linear4(nib, par, (int)rows, (int)cols, (int)gs, packed, 0));
  // The tcgen05 weight image (dense linears; the grouped expert weights,
  // packed into a caller's buffer, keep the mma.sync path only).
  uint8_t* tc = nullptr;
  if (!dst && rai::gemm_tc_enabled()) {
    if (int rc = M->alloc(&tc, rai::tc_image_bytes(rows, cols, gs))) return rc;
    RAI_CUDA(rai::pack_linear4_tc(nib, par, (int)rows, (int)cols, (int)gs, tc, 0));
  }
  RAI_CUDA(cudaDeviceSynchronize());
  if (tmp) cudaFree(tmp);
  out->data = packed;
  out->tc = tc;
  out->rows = (int)rows;
  out->cols = (int)cols;
  out->group_size = (int)gs;
  out->groups = (int)ng;
  out->tiles = (int)rai::ceil_div(rows, rai::kTileRows);
  out->wbits = 4;
  return RAI_OK;
}

// The host-libm expf exception table written next to the library at build
// time (RAI_EXPF_TABLE overrides the path).
std::string lib_dir() {
  Dl_info info;
  if (dladdr(reinterpret_cast<void*>(&lib_dir), &info) && info.dli_fname) {
    std::string p = info.dli_fname;
    size_t k = p.rfind('/');
    return k == std::string::npos ? std::string(".") : p.substr(0, k);
  }
  return ".";
}

// One table per device, loaded on first use and kept for the process.
std::mutex g_expf_mu;
std::vector<std::pair<int, rai::ExpfTable>> g_expf;

int expf_table(rai::ExpfTable* out) {
  int dev = 0;
  RAI_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_expf_mu);
  for (auto& e : g_expf)
    if (e.first == dev) { *out = e.second; return RAI_OK; }
  const char* env = std::getenv("RAI_EXPF_TABLE");
  std::string path = env ? std::string(env) : lib_dir() + "/expf_exceptions.bin";
  std::ifstream f(path, std::ios::binary);
  if (!f) return fail(RAI_ERR_INVALID, "missing " + path + " (run rai_b200.build)");
  uint32_t hdr[2] = {0, 0};
  char ver[33] = {0};
  f.read(reinterpret_cast<char*>(hdr), 8);
  f.read(ver, 32);
  if (!f || hdr[0] != 0x32505845u) return fail(RAI_ERR_INVALID, "bad expf table " + path);
  // The table lists where this glibc's expf is not correctly rounded; the
  // reference calls the glibc of the machine it runs on, so a table made
  // with another glibc would reproduce the wrong function.
  if (std::strcmp(ver, gnu_get_libc_version()) != 0)
    return fail(RAI_ERR_UNSUPPORTED, std::string("expf table ") + path + " was made with glibc " + ver +
                                         ", this process runs glibc " + gnu_get_libc_version() +
                                         " (rebuild it: python -m rai_b200.build)");
  std::vector<uint32_t> kv(2 * (size_t)hdr[1]);
  f.read(reinterpret_cast<char*>(kv.data()), kv.size() * 4);
  if (!f) return fail(RAI_ERR_INVALID, "truncated expf table " + path);
  // Bucket index over the sorted keys: bucket b = keys whose top 16 bits are
  // b occupy [start[b], start[b + 1]).
  const size_t n = hdr[1];
  std::vector<uint32_t> start(rai::kExpfBuckets + 1, 0);
  for (size_t i = 0, b = 0; b <= (size_t)rai::kExpfBuckets; ++b) {
    while (i < n && (kv[i] >> 16) < b) ++i;
    start[b] = (uint32_t)i;
  }
  uint32_t* d = nullptr;
  RAI_CUDA(cudaMalloc(&d, (kv.size() + start.size()) * 4));
  RAI_CUDA(cudaMemcpy(d, kv.data(), kv.size() * 4, cudaMemcpyHostToDevice));
  RAI_CUDA(cudaMemcpy(d + kv.size(), start.data(), start.size() * 4, cudaMemcpyHostToDevice));
  rai::ExpfTable t;
  t.keys = d;
  t.vals = d + n;
  t.start = d + kv.size();
  t.n = (int)n;
  g_expf.emplace_back(dev, t);
  *out = t;
  return RAI_OK;
}

// RAI_GEMM_MODE = exact | auto | tol (default exact).
int default_gemm_mode() {
  const char* e = std::getenv("RAI_GEMM_MODE");
  if (!e) return rai::kGemmExact;
  if (std::strcmp(e, "auto") == 0) return rai::kGemmAuto;
  if (std::strcmp(e, "tol") == 0) return rai::kGemmTol;
  return rai::kGemmExact;
}

int check_supported(const Config& c, const raimodel::Model& L) {
  if (c.group_size != 64 && c.group_size != 128)
    return fail(RAI_ERR_UNSUPPORTED, "group_size " + std::to_string(c.group_size) + " (this build runs 64 or 128)");
  if (!L.has_lm_head && c.embed_group_size != 64)
    return fail(RAI_ERR_UNSUPPORTED, "tied head with embed_group_size != 64");
  if (c.activation != 0) return fail(RAI_ERR_UNSUPPORTED, "GeLU-tanh activation");
  if (c.has_sandwich_norm || c.post_norm) return fail(RAI_ERR_UNSUPPORTED, "sandwich / post-norm placement");
  if (c.global_layer_stride) return fail(RAI_ERR_UNSUPPORTED, "per-layer RoPE bases");
  if (c.final_logit_softcap > 0.f) return fail(RAI_ERR_UNSUPPORTED, "final logit softcap");
  if (c.num_experts > rai::kMaxMoeExperts) return fail(RAI_ERR_UNSUPPORTED, "more than 256 experts");
  if (c.num_experts && c.hidden_size % 4) return fail(RAI_ERR_UNSUPPORTED, "MoE hidden size not a multiple of 4");
  if ((c.bias_mask & 7) != 0 && (c.bias_mask & 7) != 7)
    return fail(RAI_ERR_UNSUPPORTED, "bias on only some of q/k/v");
  if (c.bias_mask & 0x78) return fail(RAI_ERR_UNSUPPORTED, "bias on o/gate/up/down projections");
  int hpk = (int)(c.num_heads / c.num_kv_heads);
  if (hpk > 8) return fail(RAI_ERR_UNSUPPORTED, "more than 8 query heads per KV head");
  if (c.head_dim != 16 && c.head_dim != 32 && c.head_dim != 64 && c.head_dim != 128)
    return fail(RAI_ERR_UNSUPPORTED, "head_dim " + std::to_string(c.head_dim));
  if (hpk * c.head_dim > 1024) return fail(RAI_ERR_UNSUPPORTED, "attention group wider than 1024");
  return RAI_OK;
}

// Tensor-parallel split (see tp.cuh): every linear column-parallel, so
// heads, ff columns and hidden rows must divide evenly, and each rank's
// attention output and ff slice must be whole activation groups.
int check_tp(const Config& c, int rank, int world) {
  if (world == 1 && rank == 0) return RAI_OK;
  if (!(world == 2 || world == 4 || world == 8)) return fail(RAI_ERR_INVALID, "tensor-parallel size must be 1, 2, 4 or 8");
  if (rank < 0 || rank >= world) return fail(RAI_ERR_INVALID, "tensor-parallel rank out of range");
  if (c.num_experts) {
    // Expert parallel: whole experts per rank.
    if (c.num_experts % world) return fail(RAI_ERR_UNSUPPORTED, "experts not divisible by the parallel size");
    return RAI_OK;
  }
  if (c.has_full_qk_norm) return fail(RAI_ERR_UNSUPPORTED, "tensor parallelism with full-width QK norm");
  if (c.num_heads % world || c.num_kv_heads % world)
    return fail(RAI_ERR_UNSUPPORTED, "heads or KV heads not divisible by the tensor-parallel size");
  if ((c.num_heads / world) * c.head_dim % c.group_size)
    return fail(RAI_ERR_UNSUPPORTED, "a rank's attention output is not whole activation groups");
  if (c.intermediate_size % (world * c.group_size))
    return fail(RAI_ERR_UNSUPPORTED, "a rank's ff slice is not whole activation groups");
  if (c.hidden_size % world) return fail(RAI_ERR_UNSUPPORTED, "hidden size not divisible by the tensor-parallel size");
  return RAI_OK;
}

// Arena layout: exchange flag slots first (never reused: slot counters only
// grow), then the batches' exchanged buffers.
constexpr size_t kArenaFlagBytes = 1u << 20;

}  // namespace

// ---------------------------------------------------------------------------
// Batch: device state for one forward / decode step over n streams that share
// a model. A decoder owns a batch of one (its own scratch); step_many builds
// (and caches in the model) a batch over the decoders it is given.
struct Batch {
  rai_model* m = nullptr;
  int n = 0;           // streams
  int R = 0;           // verify row budget per stream (max_draft + 1)
  int rows_cap = 0;    // rows the scratch holds
  int ctx_cap = 0;     // context slots per stream
  int n_alloc = 0;     // attention score row stride
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  std::vector<rai_dec*> decs;
  float *hidden = nullptr, *resid = nullptr, *normed = nullptr, *qkv = nullptr, *q = nullptr;
  float *attn = nullptr, *gu = nullptr, *ff = nullptr, *logits = nullptr;
  float* scores = nullptr;  // attention scores, then p, [rows][nh][n_alloc]
  ActBuf act_h, act_q, act_ff, act_head;
  // Mixture-of-experts scratch (models with experts only).
  rai::MoeBuffers moe;
  ActBuf moe_act_x, moe_act_f;
  float *moe_gu = nullptr, *moe_eo = nullptr;
  rai::RowInfo* rows = nullptr;
  rai::RowInfo* rows_host = nullptr;
  rai::AttnSeg* segs = nullptr;  // attention segments of the rows
  rai::AttnSeg* segs_host = nullptr;
  int* n_segs = nullptr;  // segment count written by the plan kernel
  uint32_t* ids = nullptr;
  int* m_active = nullptr;
  unsigned long long* best = nullptr;
  rai::StreamKV* kv = nullptr;
  rai::StreamStep* st = nullptr;
  rai::StreamStep* st_host = nullptr;
  uint32_t* ctx = nullptr;
  uint32_t* ctx_host = nullptr;
  // Tensor parallelism: hidden, act_q, act_ff and best live in the model's
  // exchange arena; *_peer[t] are rank t's copies (own included).
  rai::TpLink tp;
  uint32_t* epoch = nullptr;
  float* hidden_peer[rai::kMaxTp] = {};
  uint8_t* act_q_peer[rai::kMaxTp] = {};
  uint8_t* act_ff_peer[rai::kMaxTp] = {};
  unsigned long long* best_peer[rai::kMaxTp] = {};
  float* moe_eo_peer[rai::kMaxTp] = {};  // expert parallelism: rank t's expert-output rows
  // Split-K workspace of the tcgen05 linear (allocated before the first
  // forward that may use it; its counters start at zero).
  void* tol_ws = nullptr;
  size_t tol_ws_bytes = 0;
  cudaGraphExec_t graph = nullptr;
  size_t graph_kernels = 0;
  uint32_t graph_key[5] = {0, 0, 0, 0, 0};
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_us = 0.f;

  template <class T>
  int alloc(T** p, size_t bytes) {
    void* q_ = nullptr;
    cudaError_t e = cudaMalloc(&q_, bytes ? bytes : 16);
    if (e != cudaSuccess)
      return fail(RAI_ERR_OOM, "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    allocs.push_back(q_);
    *p = static_cast<T*>(q_);
    return RAI_OK;
  }
  ~Batch();
};

struct rai_dec {
  rai_model* m = nullptr;
  int max_ctx = 0;
  // Sampled acceptance: seed (rai_gpu_set_seed) and steps taken since.
  uint64_t rng_seed = 0, rng_steps = 0;
  float last_us = 0.f;
  size_t last_kernels = 0;
  float* kc = nullptr;  // [layer][kv_head][max_ctx][head_dim]
  float* vc = nullptr;
  std::vector<size_t> filled;  // per layer
  std::unique_ptr<Batch> solo;
  ~rai_dec();
};

Batch::~Batch() {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(m->device);
  if (stream) cudaStreamSynchronize(stream);
  if (graph) cudaGraphExecDestroy(graph);
  for (void* p : allocs) cudaFree(p);
  if (ctx_host) cudaFreeHost(ctx_host);
  if (st_host) cudaFreeHost(st_host);
  if (rows_host) cudaFreeHost(rows_host);
  if (segs_host) cudaFreeHost(segs_host);
  if (ev0) cudaEventDestroy(ev0);
  if (ev1) cudaEventDestroy(ev1);
  if (stream) cudaStreamDestroy(stream);
  cudaSetDevice(prev);
}

// Draft-model speculative decoder (rai-infer/src/speculative.rs): a target
// and a draft decoder on one device, plus the acceptance state.
struct rai_spec {
  rai_dec* td = nullptr;  // target
  rai_dec* dd = nullptr;  // draft
  int max_ctx = 0;
  int vocab = 0;
  float* draft_logits = nullptr;      // [kMaxRowsPerStream][vocab]
  rai::StreamStep* st = nullptr;      // one stream's step state
  unsigned long long* best = nullptr; // [kMaxRowsPerStream] argmax keys (greedy)
  rai::StreamStep* st_host = nullptr;
  uint64_t seed = 0, steps = 0;
  ~rai_spec();
};

namespace {

// Cached multi-stream batches per model (keyed by the decoder list).
std::mutex g_batch_mu;
std::vector<std::pair<rai_model*, std::unique_ptr<Batch>>> g_batches;

void drop_batches_of(rai_dec* d) {
  std::lock_guard<std::mutex> lk(g_batch_mu);
  for (size_t i = 0; i < g_batches.size();) {
    auto& b = g_batches[i].second;
    if (std::find(b->decs.begin(), b->decs.end(), d) != b->decs.end()) g_batches.erase(g_batches.begin() + i);
    else ++i;
  }
}

void drop_batches_of_model(rai_model* m) {
  std::lock_guard<std::mutex> lk(g_batch_mu);
  for (size_t i = 0; i < g_batches.size();) {
    if (g_batches[i].first == m) g_batches.erase(g_batches.begin() + i);
    else ++i;
  }
}

int alloc_act(Batch* B, ActBuf* a, int tok, int cols, int gs) {
  a->tok_alloc = (int)rai::round_up(tok, 8);
  a->groups = (int)rai::ceil_div(cols, gs);
  return B->alloc(&a->data, ActBuf::bytes(a->tok_alloc, a->groups));
}

// Exchanged buffers of a tensor-parallel batch: carved from the arena at the
// same offset on every rank (all ranks create the same batches in the same
// order), so rank t's copy is peer_arena[t] + offset. Never freed before the
// model: a peer may still write into a region this rank has left.
template <class T>
int arena_alloc(rai_model* m, size_t bytes, T** local, T** peers) {
  const size_t off = rai::round_up(m->arena_used, 256);
  if (off + bytes > m->arena_bytes)
    return fail(RAI_ERR_OOM, "tensor-parallel exchange arena exhausted (raise RAI_TP_ARENA_MB)");
  m->arena_used = off + bytes;
  *local = reinterpret_cast<T*>(m->arena + off);
  for (int t = 0; t < m->tp_world; ++t) peers[t] = reinterpret_cast<T*>(m->peer_arena[t] + off);
  return RAI_OK;
}

int create_batch(rai_model* m, const std::vector<rai_dec*>& decs, int R, int rows_cap, std::unique_ptr<Batch>* out) {
  const Config& c = m->cfg;
  auto B = std::make_unique<Batch>();
  B->m = m;
  B->n = (int)decs.size();
  B->R = R;
  B->rows_cap = rows_cap;
  B->decs = decs;
  int max_ctx = 0;
  for (auto* d : decs) max_ctx = std::max(max_ctx, d->max_ctx);
  B->ctx_cap = max_ctx;
  B->n_alloc = (int)rai::round_up(max_ctx, 4);
  RAI_CUDA(cudaStreamCreateWithFlags(&B->stream, cudaStreamNonBlocking));
  RAI_CUDA(cudaEventCreate(&B->ev0));
  RAI_CUDA(cudaEventCreate(&B->ev1));
  const size_t Rw = rows_cap, h = c.hidden_size, qd = c.q_dim(), kvd = c.kv_dim(), ff = c.intermediate_size;
  const size_t nh = c.num_heads;
  // This rank's share of the dense parts (everything unless tensor parallel).
  const bool tp = m->tp_world > 1 && !m->ep, ep = m->tp_world > 1 && m->ep;
  const size_t W = tp ? m->tp_world : 1, qd_l = qd / W, kvd_l = kvd / W, ff_l = ff / W, nh_l = nh / W;
  if ((tp || ep) && !m->tp_connected)
    return fail(RAI_ERR_INVALID, "multi-GPU model not connected (rai_gpu_tp_connect)");
  if (tp || ep) {
    const size_t slots = c.num_layers * rai::kXchPerLayer + 1;
    if (m->flags_used + slots * 8 > kArenaFlagBytes) return fail(RAI_ERR_OOM, "tensor-parallel flag slots exhausted");
    B->tp.world = m->tp_world;
    B->tp.rank = m->tp_rank;
    for (int t = 0; t < m->tp_world; ++t)
      B->tp.flags[t] = reinterpret_cast<unsigned long long*>(m->peer_arena[t] + m->flags_used);
    m->flags_used += slots * 8;
    if (int rc = B->alloc(&B->epoch, 8)) return rc;
    RAI_CUDA(cudaMemset(B->epoch, 0, 8));
    B->tp.epoch = B->epoch;
  }
  if (tp) {
    if (int rc = arena_alloc(m, Rw * h * 4, &B->hidden, B->hidden_peer)) return rc;
  } else {
    if (int rc = B->alloc(&B->hidden, Rw * h * 4)) return rc;
  }
  if (int rc = B->alloc(&B->resid, Rw * h * 4)) return rc;
  if (int rc = B->alloc(&B->normed, Rw * h * 4)) return rc;
  if (int rc = B->alloc(&B->qkv, Rw * (qd_l + 2 * kvd_l) * 4)) return rc;
  if (int rc = B->alloc(&B->q, Rw * qd_l * 4)) return rc;
  if (int rc = B->alloc(&B->attn, Rw * qd_l * 4)) return rc;
  if (int rc = B->alloc(&B->gu, Rw * 2 * ff_l * 4)) return rc;
  if (int rc = B->alloc(&B->ff, Rw * ff_l * 4)) return rc;
  const size_t lrows = std::min<size_t>(Rw, (size_t)std::max(R * B->n, (int)rai::kMaxRowsPerStream));
  if (int rc = B->alloc(&B->logits, lrows * (size_t)m->v_l * 4)) return rc;
  if (int rc = B->alloc(&B->scores, Rw * nh_l * B->n_alloc * 4)) return rc;
  if (int rc = alloc_act(B.get(), &B->act_h, (int)Rw, (int)h, c.group_size)) return rc;
  if (tp) {
    auto tp_act = [&](ActBuf* a, size_t cols, uint8_t** peers) -> int {
      a->tok_alloc = (int)rai::round_up(Rw, 8);
      a->groups = (int)rai::ceil_div(cols, c.group_size);
      return arena_alloc(m, ActBuf::bytes(a->tok_alloc, a->groups), &a->data, peers);
    };
    if (int rc = tp_act(&B->act_q, qd, B->act_q_peer)) return rc;
    if (int rc = tp_act(&B->act_ff, ff, B->act_ff_peer)) return rc;
  } else {
    if (int rc = alloc_act(B.get(), &B->act_q, (int)Rw, (int)qd, c.group_size)) return rc;
    if (int rc = alloc_act(B.get(), &B->act_ff, (int)Rw, (int)ff, c.group_size)) return rc;
  }
  int hgs = m->head.wbits == 8 ? (int)c.embed_group_size : (int)c.group_size;
  if (int rc = alloc_act(B.get(), &B->act_head, (int)lrows, (int)h, hgs)) return rc;
  if (int rc = B->alloc(&B->rows, Rw * sizeof(rai::RowInfo))) return rc;
  if (int rc = B->alloc(&B->ids, Rw * 4)) return rc;
  if (int rc = B->alloc(&B->m_active, 4)) return rc;
  if (c.num_experts) {
    const size_t ne = c.num_experts, k = c.experts_per_token, ffe = c.intermediate_size;
    rai::MoeBuffers& mb = B->moe;
    mb.rows_cap = (int)(Rw * k + 8 * ne);
    if (int rc = B->alloc(&mb.logits, Rw * ne * 4)) return rc;
    if (int rc = B->alloc(&mb.experts, Rw * k * 4)) return rc;
    if (int rc = B->alloc(&mb.weights, Rw * k * 4)) return rc;
    if (int rc = B->alloc(&mb.cnt, ne * 4)) return rc;
    if (int rc = B->alloc(&mb.off, ne * 4)) return rc;
    if (int rc = B->alloc(&mb.row_of_pair, Rw * k * 4)) return rc;
    if (int rc = B->alloc(&mb.pair_of_row, (size_t)mb.rows_cap * 4)) return rc;
    if (int rc = B->alloc(&mb.n_rows, 4)) return rc;
    if (int rc = alloc_act(B.get(), &B->moe_act_x, mb.rows_cap, (int)h, c.group_size)) return rc;
    if (int rc = alloc_act(B.get(), &B->moe_act_f, mb.rows_cap, (int)ffe, c.group_size)) return rc;
    if (int rc = B->alloc(&B->moe_gu, (size_t)mb.rows_cap * 2 * ffe * 4)) return rc;
    if (ep) {
      // Expert parallel: every rank writes its experts' rows into each copy.
      if (int rc = arena_alloc(m, (size_t)mb.rows_cap * h * 4, &B->moe_eo, B->moe_eo_peer)) return rc;
    } else {
      if (int rc = B->alloc(&B->moe_eo, (size_t)mb.rows_cap * h * 4)) return rc;
    }
  }
  if (int rc = B->alloc(&B->segs, Rw * sizeof(rai::AttnSeg))) return rc;
  if (int rc = B->alloc(&B->n_segs, 4)) return rc;
  if (tp) {
    if (int rc = arena_alloc(m, Rw * 8, &B->best, B->best_peer)) return rc;
  } else {
    if (int rc = B->alloc(&B->best, Rw * 8)) return rc;
  }
  if (int rc = B->alloc(&B->kv, B->n * sizeof(rai::StreamKV))) return rc;
  if (int rc = B->alloc(&B->st, B->n * sizeof(rai::StreamStep))) return rc;
  if (int rc = B->alloc(&B->ctx, (size_t)B->n * B->ctx_cap * 4)) return rc;
  RAI_CUDA(cudaMemset(B->st, 0, B->n * sizeof(rai::StreamStep)));
  RAI_CUDA(cudaMallocHost(&B->ctx_host, (size_t)B->n * B->ctx_cap * 4));
  RAI_CUDA(cudaMallocHost(&B->st_host, B->n * sizeof(rai::StreamStep)));
  RAI_CUDA(cudaMallocHost(&B->rows_host, Rw * sizeof(rai::RowInfo)));
  RAI_CUDA(cudaMallocHost(&B->segs_host, Rw * sizeof(rai::AttnSeg)));
  std::memset(B->st_host, 0, B->n * sizeof(rai::StreamStep));
  std::vector<rai::StreamKV> kv(B->n);
  for (int i = 0; i < B->n; ++i) kv[i] = rai::StreamKV{decs[i]->kc, decs[i]->vc, decs[i]->max_ctx, 0};
  RAI_CUDA(cudaMemcpy(B->kv, kv.data(), kv.size() * sizeof(rai::StreamKV), cudaMemcpyHostToDevice));
  if ((size_t)B->n_alloc * 4 > rai::kAttnMaxSmem)
    return fail(RAI_ERR_UNSUPPORTED, "context window too long for the attention softmax kernel");
  *out = std::move(B);
  return RAI_OK;
}

// ---------------------------------------------------------------------------
// Forward over M rows (static budget) of which *m_dev are active when m_dev
// is set; rows[] gives each row's (position, stream), ids[] its token; the
// rows' attention segments are segs[] (nseg of them, or *nseg_dev when set;
// at most seg_rows rows each).
// The kernel policy of a batch's dense linears.
rai::GemmPolicy gemm_policy(const Batch* B) {
  rai::GemmPolicy pol;
  pol.mode = B->m->tp_world > 1 ? rai::kGemmExact : B->m->gemm_mode;
  pol.ws = B->tol_ws;
  pol.ws_bytes = B->tol_ws_bytes;
  return pol;
}

// Allocate the batch's tcgen05 workspace before a forward of `rows` rows
// that may run the tcgen05 linear (never during graph capture).
int ensure_tol_ws(Batch* B, int rows) {
  const rai::GemmPolicy pol = gemm_policy(B);
  const bool may = pol.mode == rai::kGemmTol || (pol.mode == rai::kGemmAuto && rows >= rai::kTolMinRows);
  if (!may || B->tol_ws) return RAI_OK;
  const size_t bytes = rai::gemm_tol_workspace_bytes();
  if (int rc = B->alloc(&B->tol_ws, bytes)) return rc;
  RAI_CUDA(cudaMemset(B->tol_ws, 0, bytes));
  B->tol_ws_bytes = bytes;
  return RAI_OK;
}

int forward(Batch* B, int M, const int* m_dev, int nseg, const int* nseg_dev, int seg_rows, bool logits) {
  rai_model* Mo = B->m;
  const rai::GemmPolicy pol = gemm_policy(B);
  const Config& c = Mo->cfg;
  cudaStream_t s = B->stream;
  const int h = c.hidden_size, hd = c.head_dim;
  const int gs = c.group_size;
  const float eps = c.norm_eps;
  uint32_t* err = Mo->err_dev;
  // Tensor parallelism (see tp.cuh): this rank's heads / ff columns /
  // hidden rows; W == 1 is the whole model.
  const int W = Mo->tp_world, r = Mo->tp_rank;
  const bool tp = W > 1 && !Mo->ep;
  const bool ep = W > 1 && Mo->ep;  // expert parallel: only the MoE experts are split
  const int nh = Mo->nh_l, nkv = Mo->nkv_l, ffd = Mo->ff_l, h_l = Mo->h_l;
  const int qd = nh * hd, kvd = nkv * hd;
  const rai::TpLink* link = tp ? &B->tp : nullptr;
  auto slot = [&](size_t li, int k) { return (int)li * rai::kXchPerLayer + k; };
  // Destinations of the exchanged activations and hidden rows: own copy first.
  rai::ActDst dst_q, dst_ff;
  rai::GemmTp gtp;
  if (tp) {
    dst_q.n = dst_ff.n = W;
    dst_q.groups = B->act_q.groups;
    dst_ff.groups = B->act_ff.groups;
    dst_q.g_off = r * (qd / gs);
    dst_ff.g_off = r * (ffd / gs);
    gtp.link = B->tp;
    gtp.n_out = W;
    for (int t = 0, k = 0; t < W; ++t) {
      const int d = t == r ? 0 : ++k;  // slot 0 is this rank
      dst_q.data[d] = B->act_q_peer[t];
      dst_ff.data[d] = B->act_ff_peer[t];
      gtp.outs[d] = B->hidden_peer[t] + (size_t)r * h_l;
    }
  }
  float* hid_out = B->hidden + (tp ? (size_t)r * h_l : 0);  // this rank's o / down rows
  rai::GemmTp gep;  // expert parallel: the down projection's rows go to every rank
  if (ep) {
    gep.link = B->tp;
    gep.n_out = W;
    for (int t = 0, k = 0; t < W; ++t) gep.outs[t == r ? 0 : ++k] = B->moe_eo_peer[t];
  }
  RAI_CUDA(rai::launch_embed(B->ids, m_dev, M, Mo->embed_codes, Mo->embed_params, c.vocab_size, h,
                             c.embed_group_size, c.embed_scale, B->hidden, err, s, (tp || ep) ? B->epoch : nullptr,
                             logits));
  rai::GemmEpilogue e_res;
  e_res.mode = rai::kEpiResidual;
  e_res.residual = B->resid + (tp ? (size_t)r * h_l : 0);
  for (size_t li = 0; li < c.num_layers; ++li) {
    const LayerDev& L = Mo->layers[li];
    RAI_CUDA(rai::norm_quant(B->hidden, L.in_norm, h, eps, B->resid, M, m_dev, gs, 4, B->act_h, s, nullptr, link,
                             tp && li > 0 ? slot(li - 1, rai::kXchHiddenDown) : -1, err));
    rai::GemmEpilogue e_qkv;
    if (L.bias_qkv) { e_qkv.mode = rai::kEpiBias; e_qkv.bias = L.bias_qkv; }
    RAI_CUDA(rai::gemm_exact(L.qkv, B->act_h, M, B->qkv, qd + 2 * kvd, e_qkv, err, s, false, m_dev, nullptr, &pol));
    RAI_CUDA(rai::launch_qkv_post(B->qkv, qd + 2 * kvd, B->q, nh, nkv, hd, L.q_norm, L.k_norm, Mo->qk_mode, eps,
                                  Mo->rope_cos, Mo->rope_sin, B->kv, (int)li, B->rows, m_dev, M, s));
    RAI_CUDA(rai::launch_attention(B->q, B->attn, B->kv, (int)li, B->rows, m_dev, M, B->segs, nseg_dev, nseg,
                                   seg_rows, nh, nkv, hd, Mo->scale, c.attn_logit_softcap, B->scores, B->n_alloc,
                                   Mo->expf, err, s));
    RAI_CUDA(rai::quantize_act(B->attn, qd, M, m_dev, qd, gs, 4, B->act_q, s, tp ? &dst_q : nullptr));
    if (tp) gtp.wait_slot = slot(li, rai::kXchActQ);
    RAI_CUDA(rai::gemm_exact(L.o, B->act_q, M, hid_out, h, e_res, err, s, false, m_dev, tp ? &gtp : nullptr, &pol));
    if (L.moe) {
      // mlp_block (model.rs:208-261): route, expert SwiGLU MLPs grouped by
      // expert, weighted sum in pick order, residual add.
      // Expert parallel: routing and the sort run on every rank (the sort is
      // stable, so every rank assigns the same rows); each rank runs its own
      // experts and writes their rows into every rank's expert outputs; the
      // combine waits for all of them.
      const int ne = (int)c.num_experts, k = (int)c.experts_per_token;
      const rai::MoeBuffers& mb = B->moe;
      RAI_CUDA(rai::norm_quant(B->hidden, L.post_norm, h, eps, B->resid, M, m_dev, gs, 4, ActBuf{}, s, B->normed));
      RAI_CUDA(rai::moe_route(B->normed, L.router, h, ne, k, c.norm_topk_prob, m_dev, M, Mo->expf, mb, s));
      RAI_CUDA(rai::moe_gather_quant(B->normed, h, k, gs, mb, B->moe_act_x, s));
      RAI_CUDA(rai::gemm_grouped(L.x_gateup, L.x_gu_stride, Mo->ne_l, mb.off, mb.cnt, B->moe_act_x, B->moe_gu, 2 * ffd,
                                 err, s, Mo->e0));
      RAI_CUDA(rai::swiglu_quant(B->moe_gu, ffd, mb.rows_cap, mb.n_rows, gs, Mo->expf, B->moe_act_f, s));
      RAI_CUDA(rai::gemm_grouped(L.x_down, L.x_dn_stride, Mo->ne_l, mb.off, mb.cnt, B->moe_act_f, B->moe_eo, h, err, s,
                                 Mo->e0, ep ? &gep : nullptr));
      RAI_CUDA(rai::moe_combine(B->moe_eo, k, h, B->resid, B->hidden, m_dev, M, mb, s, ep ? &B->tp : nullptr,
                                ep ? slot(li, rai::kXchActFF) : -1, err));
      continue;
    }
    RAI_CUDA(rai::norm_quant(B->hidden, L.post_norm, h, eps, B->resid, M, m_dev, gs, 4, B->act_h, s, nullptr, link,
                             tp ? slot(li, rai::kXchHiddenO) : -1, err));
    RAI_CUDA(rai::gemm_exact(L.gateup, B->act_h, M, B->gu, 2 * ffd, rai::GemmEpilogue{}, err, s, false, m_dev,
                             nullptr, &pol));
    RAI_CUDA(rai::swiglu_quant(B->gu, ffd, M, m_dev, gs, Mo->expf, B->act_ff, s, tp ? &dst_ff : nullptr, r * ffd,
                               (int)c.intermediate_size));
    if (tp) gtp.wait_slot = slot(li, rai::kXchActFF);
    RAI_CUDA(rai::gemm_exact(L.down, B->act_ff, M, hid_out, h, e_res, err, s, false, m_dev, tp ? &gtp : nullptr,
                             &pol));
  }
  if (logits || tp) {
    // Under tensor parallelism the last layer's hidden exchange is awaited
    // here even without logits, so a forward always completes all its slots.
    const bool tied = Mo->head.wbits == 8;
    RAI_CUDA(rai::norm_quant(B->hidden, Mo->final_norm, h, eps, nullptr, M, m_dev, tied ? c.embed_group_size : gs,
                             tied ? 8 : 4, logits ? B->act_head : ActBuf{}, s, nullptr, link,
                             tp ? slot(c.num_layers - 1, rai::kXchHiddenDown) : -1, err));
  }
  if (logits)
    RAI_CUDA(rai::gemm_exact(Mo->head, B->act_head, M, B->logits, Mo->v_l, rai::GemmEpilogue{}, err, s, false,
                             m_dev, nullptr, &pol));
  return RAI_OK;
}

int check_err(rai_model* m, cudaStream_t s) {
  uint32_t e = 0;
  RAI_CUDA(cudaMemcpyAsync(&e, m->err_dev, 4, cudaMemcpyDeviceToHost, s));
  RAI_CUDA(cudaStreamSynchronize(s));
  if (e) {
    cudaMemsetAsync(m->err_dev, 0, 4, s);
    cudaStreamSynchronize(s);
    if ((e & rai::kErrWaitTimeout) && m->tp_world > 1) {
      m->failed = true;
      return fail(RAI_ERR_TIMEOUT, "a cross-GPU wait timed out; this multi-GPU model now refuses work until every "
                                   "rank destroys and re-creates it");
    }
    if (e & rai::kErrWaitTimeout) return fail(RAI_ERR_TIMEOUT, "a device-side wait timed out");
    return fail(RAI_ERR_INVALID, "device kernel rejected its input (token id out of range)");
  }
  return RAI_OK;
}

// Entry points that launch work on a model call this first.
int check_usable(const rai_model* m) {
  if (m->failed)
    return fail(RAI_ERR_TIMEOUT, "multi-GPU model failed after a cross-GPU wait timed out: destroy and re-create it "
                                 "on every rank");
  return RAI_OK;
}

int validate_cfg(const rai_lookup_cfg* cfg) {
  if (!cfg) return fail(RAI_ERR_INVALID, "null lookup config");
  // validate_lookup_config (rai-infer/src/lookup.rs:457-475)
  if (cfg->max_draft == 0) return fail(RAI_ERR_INVALID, "prompt-lookup max_draft must be non-zero");
  if (!(cfg->min_ngram >= 1 && cfg->min_ngram <= cfg->max_ngram))
    return fail(RAI_ERR_INVALID, "prompt-lookup requires 1 <= min_ngram <= max_ngram");
  if (!(std::isfinite(cfg->temperature) && cfg->temperature >= 0.f) || cfg->top_k != 0 || cfg->top_p != 1.0f ||
      cfg->repetition_penalty != 1.0f)
    return fail(RAI_ERR_INVALID,
                "prompt-lookup decoding requires finite temperature, top_k=0, top_p=1, and repetition_penalty=1");
  // temperature 0 is the greedy limit of the reference's rule (which refuses
  // t <= 1e-6); t > 1e-6 samples as the reference does.
  if (cfg->temperature != 0.f && !(cfg->temperature > 1e-6f))
    return fail(RAI_ERR_INVALID, "prompt-lookup decoding requires temperature 0 (greedy) or temperature > 1e-6");
  if (cfg->max_draft + 1 > (uint32_t)rai::kMaxRowsPerStream) return fail(RAI_ERR_INVALID, "max_draft exceeds 32");
  return RAI_OK;
}

int ensure_graph(Batch* B, const rai_lookup_cfg* cfg) {
  uint32_t tbits = 0;
  std::memcpy(&tbits, &cfg->temperature, 4);
  uint32_t key[5] = {cfg->max_draft, cfg->max_ngram, cfg->min_ngram, tbits, (uint32_t)B->m->gemm_mode};
  if (B->graph && std::memcmp(key, B->graph_key, sizeof(key)) == 0) return RAI_OK;
  if (B->graph) {
    cudaGraphExecDestroy(B->graph);
    B->graph = nullptr;
  }
  const int R = (int)cfg->max_draft + 1;
  const int rows = B->n * R;
  if (rows > B->rows_cap) return fail(RAI_ERR_INVALID, "batch row budget exceeded");
  if (int rc = ensure_tol_ws(B, rows)) return rc;
  cudaStream_t s = B->stream;
  cudaGraph_t g = nullptr;
  RAI_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int rc = RAI_OK;
  do {
    if (cudaSuccess != rai::launch_ngram(B->ctx, B->ctx_cap, B->st, B->kv, B->n, (int)cfg->max_draft,
                                         (int)cfg->max_ngram, (int)cfg->min_ngram, s) ||
        cudaSuccess != rai::launch_plan(B->st, B->n, B->rows, B->ids, B->m_active, B->segs, B->n_segs,
                                        std::min(R, rai::kStepSegRows), B->best, rows, s)) {
      rc = fail(RAI_ERR_DEVICE, "draft launch failed");
      break;
    }
    const int seg_rows = std::min(R, rai::kStepSegRows);
    const int nseg = B->n * ((R + seg_rows - 1) / seg_rows);
    rc = forward(B, rows, B->m_active, nseg, B->n_segs, seg_rows, true);
    if (rc) break;
    rai_model* m = B->m;
    const bool tp = m->tp_world > 1 && !m->ep;
    const int lslot = (int)m->cfg.num_layers * rai::kXchPerLayer;  // the logits exchange
    if (cfg->temperature > 0.f) {
      // Sampled acceptance (full vocabulary rows on this GPU; refused under
      // tensor parallelism before capture).
      if (cudaSuccess != rai::launch_sample_accept(B->st, B->n, B->logits, m->v_l, cfg->temperature, s)) {
        rc = fail(RAI_ERR_DEVICE, "accept launch failed");
        break;
      }
    } else if (cudaSuccess != rai::launch_argmax(B->logits, m->v_l, B->m_active, rows, B->best, s, m->v_off,
                                                 tp ? B->best_peer : nullptr, tp ? m->tp_world : 1) ||
               cudaSuccess != rai::launch_accept(B->st, B->n, B->best, s, tp ? &B->tp : nullptr, tp ? lslot : -1,
                                                 m->err_dev)) {
      rc = fail(RAI_ERR_DEVICE, "accept launch failed");
      break;
    }
  } while (0);
  cudaError_t ce = cudaStreamEndCapture(s, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    (void)cudaGetLastError();
    return rc;
  }
  if (ce != cudaSuccess) return fail(RAI_ERR_DEVICE, std::string("graph capture: ") + cudaGetErrorString(ce));
  size_t nnodes = 0;
  cudaGraphGetNodes(g, nullptr, &nnodes);
  std::vector<cudaGraphNode_t> nodes(nnodes);
  cudaGraphGetNodes(g, nodes.data(), &nnodes);
  B->graph_kernels = 0;
  for (auto nd : nodes) {
    cudaGraphNodeType ty;
    if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++B->graph_kernels;
  }
  cudaError_t ie = cudaGraphInstantiate(&B->graph, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return fail(RAI_ERR_DEVICE, std::string("graph instantiate: ") + cudaGetErrorString(ie));
  std::memcpy(B->graph_key, key, sizeof(key));
  return RAI_OK;
}

// One lookup step for every stream of the batch.
// lookup = false: no draft search (decode_one), cfg carries only the
// temperature.
int step_batch(Batch* B, const size_t* pos, const uint32_t* const* ctx, const size_t* ctx_len,
               const rai_lookup_cfg* cfg, uint32_t* out_tokens, size_t out_cap, size_t* n_out,
               rai_lookup_metrics* metrics, bool lookup = true) {
  if (int rc = check_usable(B->m)) return rc;
  if (lookup)
    if (int rc = validate_cfg(cfg)) return rc;
  if (out_cap < cfg->max_draft + 1) return fail(RAI_ERR_INVALID, "out_tokens capacity below max_draft + 1");
  if (cfg->temperature > 0.f && B->m->tp_world > 1 && !B->m->ep)
    return fail(RAI_ERR_UNSUPPORTED, "sampled acceptance on a tensor-parallel model (each rank holds a vocabulary slice)");
  const Config& c = B->m->cfg;
  for (int i = 0; i < B->n; ++i) {
    rai_dec* d = B->decs[i];
    if (!ctx[i]) return fail(RAI_ERR_INVALID, "null context");
    if (ctx_len[i] == 0) return fail(RAI_ERR_INVALID, "prompt-lookup step requires a non-empty context");
    if (pos[i] >= (size_t)d->max_ctx) return fail(RAI_ERR_INVALID, "decode position exceeds the context window");
    if (ctx_len[i] > (size_t)d->max_ctx) return fail(RAI_ERR_INVALID, "context longer than the window");
    if (pos[i] > d->filled[0]) return fail(RAI_ERR_INVALID, "KV store would leave a gap");
    // Largest id of the context (a reduction the compiler vectorizes), then
    // one comparison.
    uint32_t mx = 0;
    for (size_t t = 0; t < ctx_len[i]; ++t) mx = std::max(mx, ctx[i][t]);
    if (mx >= c.vocab_size) return fail(RAI_ERR_INVALID, "context contains a token outside the model vocabulary");
  }
  if (int rc = ensure_graph(B, cfg)) return rc;
  for (int i = 0; i < B->n; ++i) {
    std::memcpy(B->ctx_host + (size_t)i * B->ctx_cap, ctx[i], ctx_len[i] * 4);
    B->st_host[i].pos = (int)pos[i];
    B->st_host[i].ctx_len = (int)ctx_len[i];
    const rai_dec* d = B->decs[i];
    B->st_host[i].rng_seed_lo = (uint32_t)d->rng_seed;
    B->st_host[i].rng_seed_hi = (uint32_t)(d->rng_seed >> 32);
    B->st_host[i].rng_step_lo = (uint32_t)d->rng_steps;
    B->st_host[i].rng_step_hi = (uint32_t)(d->rng_steps >> 32);
  }
  cudaStream_t s = B->stream;
  size_t max_len = 0;
  for (int i = 0; i < B->n; ++i) max_len = std::max(max_len, ctx_len[i]);
  if (B->n == 1) {
    RAI_CUDA(cudaMemcpyAsync(B->ctx, B->ctx_host, ctx_len[0] * 4, cudaMemcpyHostToDevice, s));
  } else {
    RAI_CUDA(cudaMemcpyAsync(B->ctx, B->ctx_host, (size_t)B->n * B->ctx_cap * 4, cudaMemcpyHostToDevice, s));
  }
  RAI_CUDA(cudaMemcpyAsync(B->st, B->st_host, B->n * sizeof(rai::StreamStep), cudaMemcpyHostToDevice, s));
  RAI_CUDA(cudaEventRecord(B->ev0, s));
  RAI_CUDA(cudaGraphLaunch(B->graph, s));
  RAI_CUDA(cudaEventRecord(B->ev1, s));
  RAI_CUDA(cudaMemcpyAsync(B->st_host, B->st, B->n * sizeof(rai::StreamStep), cudaMemcpyDeviceToHost, s));
  if (int rc = check_err(B->m, s)) return rc;
  float ms = 0.f;
  cudaEventElapsedTime(&ms, B->ev0, B->ev1);
  B->last_us = ms * 1000.f;
  for (int i = 0; i < B->n; ++i) {
    const rai::StreamStep& st = B->st_host[i];
    n_out[i] = (size_t)st.produced;
    for (int t = 0; t < st.produced; ++t) out_tokens[i * out_cap + t] = st.out[t];
    for (auto& f : B->decs[i]->filled) f = pos[i] + st.produced;
    ++B->decs[i]->rng_steps;
    B->decs[i]->last_us = B->last_us;
    B->decs[i]->last_kernels = B->graph_kernels;
    if (metrics) {
      metrics[i].accepted = st.accepted;
      metrics[i].drafted = st.drafted;
      metrics[i].produced = st.produced;
      metrics[i].matched_ngram = st.ngram;
      metrics[i].accept_rate = st.drafted ? (float)st.accepted / (float)st.drafted : 0.f;
    }
  }
  return RAI_OK;
}

// Forward over host-described rows (B->rows_host[0..M), ids already queued):
// segments are built on the host and copied with the rows.
int forward_host_rows(Batch* B, int M, bool logits) {
  cudaStream_t s = B->stream;
  const int nseg = rai::build_segments(B->rows_host, M, rai::kSegRows, B->segs_host);
  int seg_rows = 1;
  for (int i = 0; i < nseg; ++i) seg_rows = std::max(seg_rows, B->segs_host[i].nrows);
  RAI_CUDA(cudaMemcpyAsync(B->rows, B->rows_host, M * sizeof(rai::RowInfo), cudaMemcpyHostToDevice, s));
  RAI_CUDA(cudaMemcpyAsync(B->segs, B->segs_host, nseg * sizeof(rai::AttnSeg), cudaMemcpyHostToDevice, s));
  if (int rc = ensure_tol_ws(B, M)) return rc;
  return forward(B, M, nullptr, nseg, nullptr, seg_rows, logits);
}

// Forward `rows` tokens of a single decoder at positions start.. (prefill or
// logits), through its own batch.
int forward_solo(rai_dec* d, const uint32_t* ids, size_t start, int rows, bool logits) {
  Batch* B = d->solo.get();
  for (int b = 0; b < rows; ++b) B->rows_host[b] = rai::RowInfo{(int)(start + b), 0};
  cudaStream_t s = B->stream;
  RAI_CUDA(cudaMemcpyAsync(B->ids, ids, rows * 4, cudaMemcpyHostToDevice, s));
  return forward_host_rows(B, rows, logits);
}

}  // namespace

rai_spec::~rai_spec() {
  if (td) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(td->m->device);
    if (draft_logits) cudaFree(draft_logits);
    if (st) cudaFree(st);
    if (best) cudaFree(best);
    if (st_host) cudaFreeHost(st_host);
    cudaSetDevice(prev);
  }
  delete dd;
  delete td;
}

rai_dec::~rai_dec() {
  drop_batches_of(this);
  solo.reset();
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(m->device);
  if (kc) cudaFree(kc);
  if (vc) cudaFree(vc);
  cudaSetDevice(prev);
  --m->live_decoders;
}

// ---------------------------------------------------------------------------
// Static scratch of rai_gpu_w4a8_matmul_static: the quantized activations
// live in a file-scope device array instead of caller- or library-allocated
// memory. Its device address is looked up once per device (with that device
// current) and cached.
namespace {
constexpr size_t kStaticScratchBytes = 2u << 20;  // 2 MiB per device
__device__ __align__(256) uint8_t g_w4a8_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_scratch_ptr[kMaxDevices] = {};

// Status word of the kernel-level entries (one per device): their bounded
// device waits record a timeout here; rai_gpu_kernel_status reads and
// clears it.
__device__ uint32_t g_kernel_err_word;
uint32_t* g_kernel_err_ptr[kMaxDevices] = {};

int kernel_err_word(uint32_t** out) {
  int dev = 0;
  RAI_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(RAI_ERR_UNSUPPORTED, "device ordinal beyond the status table");
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_kernel_err_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_kernel_err_word);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return fail(RAI_ERR_DEVICE, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    }
    g_kernel_err_ptr[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_kernel_err_ptr[dev];
  return RAI_OK;
}

int static_scratch(void** out) {
  int dev = 0;
  RAI_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(RAI_ERR_UNSUPPORTED, "device ordinal beyond the static scratch table");
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_w4a8_static_scratch);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return fail(RAI_ERR_DEVICE, std::string("cudaGetSymbolAddress(static scratch): ") + cudaGetErrorString(e));
    }
    g_static_scratch_ptr[dev] = p;
  }
  *out = g_static_scratch_ptr[dev];
  return RAI_OK;
}
}  // namespace

// ===========================================================================
extern "C" {

size_t rai_gpu_last_error(char* buf, size_t len) {
  if (buf && len) {
    size_t n = std::min(len - 1, g_last_error.size());
    std::memcpy(buf, g_last_error.data(), n);
    buf[n] = 0;
  }
  return g_last_error.size();
}

static int create_model(const uint8_t* blob, size_t len, int device, int tp_rank, int tp_world, rai_model** out) {
  if (!blob || !out) return fail(RAI_ERR_INVALID, "null argument");
  *out = nullptr;
  // Host-side validation first (RaiModelFile::open), so a malformed file is
  // reported as such whether or not a device is present.
  raimodel::Model layout;
  std::string err;
  if (!raimodel::open(blob, len, layout, err)) return fail(RAI_ERR_FORMAT, err);
  if (int rc = check_supported(layout.cfg, layout)) return rc;
  if (int rc = check_tp(layout.cfg, tp_rank, tp_world)) return rc;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(RAI_ERR_DEVICE, "no CUDA device");
  if (device < 0 || device >= ndev) return fail(RAI_ERR_INVALID, "device index out of range");
  DeviceGuard guard(device);
  RAI_CUDA(rai::init_gemm_attributes());
  RAI_CUDA(rai::init_layer_attributes());
  RAI_CUDA(rai::init_moe_attributes());
  auto M = std::make_unique<rai_model>();
  M->device = device;
  M->gemm_mode = default_gemm_mode();
  M->layout = std::move(layout);
  M->cfg = M->layout.cfg;
  const Config& c = M->cfg;
  M->scale = c.attention_scale();
  // This rank's shard (the whole model when tp_world == 1).
  const int r = tp_rank;
  M->tp_rank = r;
  M->tp_world = tp_world;
  M->ep = tp_world > 1 && c.num_experts > 0;
  M->ne_l = (int)c.num_experts / tp_world;
  M->e0 = r * M->ne_l;
  // Tensor-parallel split factor of the dense parts (1 under expert parallelism).
  const int W = M->ep ? 1 : tp_world;
  const int rw = M->ep ? 0 : r;
  M->nh_l = (int)c.num_heads / W;
  M->nkv_l = (int)c.num_kv_heads / W;
  M->ff_l = (int)c.intermediate_size / W;
  M->h_l = (int)c.hidden_size / W;
  M->v_l = (int)rai::ceil_div(c.vocab_size, W);
  M->v_off = rw * M->v_l;
  M->v_l = std::min<int>(M->v_l, (int)c.vocab_size - M->v_off);
  const size_t qd_l = (size_t)M->nh_l * c.head_dim, kvd_l = (size_t)M->nkv_l * c.head_dim;
  const size_t ff_l = M->ff_l, h_l = M->h_l;
  M->qk_mode = c.has_full_qk_norm ? 2 : (c.has_qk_norm ? 1 : 0);
  if (int rc = M->alloc(&M->err_dev, 4)) return rc;
  RAI_CUDA(cudaMemset(M->err_dev, 0, 4));
  if (int rc = expf_table(&M->expf)) return rc;

  // Upload the blob once; pack from the device copy, then release it.
  uint8_t* blob_dev = nullptr;
  RAI_CUDA(cudaMalloc(&blob_dev, len));
  struct Free { uint8_t* p; ~Free() { if (p) cudaFree(p); } } free_blob{blob_dev};
  RAI_CUDA(cudaMemcpy(blob_dev, blob, len, cudaMemcpyHostToDevice));

  const auto& E = M->layout.embed;
  size_t ecodes = (size_t)E.vocab * E.hidden, eparams = (size_t)E.vocab * rai::ceil_div(E.hidden, E.group_size) * 4;
  if (int rc = M->alloc(&M->embed_codes, ecodes)) return rc;
  if (int rc = M->alloc(&M->embed_params, eparams)) return rc;
  RAI_CUDA(cudaMemcpy(M->embed_codes, blob_dev + E.data_off, ecodes, cudaMemcpyDeviceToDevice));
  RAI_CUDA(cudaMemcpy(M->embed_params, blob_dev + E.params_off, eparams, cudaMemcpyDeviceToDevice));

  M->layers.resize(c.num_layers);
  for (size_t li = 0; li < c.num_layers; ++li) {
    const raimodel::Layer& L = M->layout.layers[li];
    LayerDev& D = M->layers[li];
    if (int rc = pack_concat(M.get(), blob_dev,
                             {RowRange{&L.proj[0], rw * qd_l, qd_l}, RowRange{&L.proj[1], rw * kvd_l, kvd_l},
                              RowRange{&L.proj[2], rw * kvd_l, kvd_l}},
                             &D.qkv))
      return rc;
    if (int rc = pack_concat(M.get(), blob_dev, {RowRange{&L.proj[3], rw * h_l, h_l}}, &D.o)) return rc;
    if (c.num_experts) {
      // Expert 0 is stored as the layer's gate/up/down, experts 1.. in
      // L.experts (format.rs:436-477).
      D.moe = true;
      // This rank's experts (all of them unless expert parallel).
      const size_t ne = M->ne_l, ff = L.proj[4].rows, hs = c.hidden_size, gsz = c.group_size;
      D.x_gu_stride = rai::packed_linear_bytes(2 * ff, hs, gsz);
      D.x_dn_stride = rai::packed_linear_bytes(hs, ff, gsz);
      uint8_t *gu = nullptr, *dn = nullptr;
      if (int rc = M->alloc(&gu, D.x_gu_stride * ne)) return rc;
      if (int rc = M->alloc(&dn, D.x_dn_stride * ne)) return rc;
      for (size_t j = 0; j < ne; ++j) {
        const size_t e = M->e0 + j;
        const raimodel::Linear* g = e == 0 ? &L.proj[4] : &L.experts[3 * (e - 1)];
        const raimodel::Linear* u = e == 0 ? &L.proj[5] : &L.experts[3 * (e - 1) + 1];
        const raimodel::Linear* d = e == 0 ? &L.proj[6] : &L.experts[3 * (e - 1) + 2];
        if (int rc = pack_concat(M.get(), blob_dev, {whole(g), whole(u)}, &D.x_gateup, gu + j * D.x_gu_stride))
          return rc;
        if (int rc = pack_concat(M.get(), blob_dev, {whole(d)}, &D.x_down, dn + j * D.x_dn_stride)) return rc;
      }
      D.x_gateup.data = gu;
      D.x_down.data = dn;
      if (int rc = upload_vec(M.get(), blob, L.router, &D.router)) return rc;
    } else {
      if (int rc = pack_concat(M.get(), blob_dev,
                               {RowRange{&L.proj[4], rw * ff_l, ff_l}, RowRange{&L.proj[5], rw * ff_l, ff_l}},
                               &D.gateup))
        return rc;
      if (int rc = pack_concat(M.get(), blob_dev, {RowRange{&L.proj[6], rw * h_l, h_l}}, &D.down)) return rc;
    }
    if (int rc = upload_vec(M.get(), blob, L.input_norm, &D.in_norm)) return rc;
    if (int rc = upload_vec(M.get(), blob, L.post_attn_norm, &D.post_norm)) return rc;
    if ((c.bias_mask & 7) == 7) {
      std::vector<float> b;
      for (int p = 0; p < 3; ++p) {
        auto v = raimodel::read_vec(blob, L.bias[p]);
        const size_t w = p == 0 ? qd_l : kvd_l;  // this rank's rows of q / k / v
        b.insert(b.end(), v.begin() + rw * w, v.begin() + (rw + 1) * w);
      }
      if (int rc = upload(M.get(), b.data(), b.size() * 4, reinterpret_cast<void**>(&D.bias_qkv))) return rc;
    }
    if (L.q_norm.present) {
      if (int rc = upload_vec(M.get(), blob, L.q_norm, &D.q_norm)) return rc;
      if (int rc = upload_vec(M.get(), blob, L.k_norm, &D.k_norm)) return rc;
    }
  }
  if (int rc = upload_vec(M.get(), blob, M->layout.final_norm, &M->final_norm)) return rc;
  if (M->layout.has_lm_head) {
    if (int rc = pack_concat(M.get(), blob_dev, {RowRange{&M->layout.lm_head, (size_t)M->v_off, (size_t)M->v_l}},
                             &M->head))
      return rc;
  } else {
    // Tied head: this rank's vocabulary rows of the 8-bit embedding table.
    const size_t vl = M->v_l, eng = rai::ceil_div(E.hidden, E.group_size);
    uint8_t* packed = nullptr;
    if (int rc = M->alloc(&packed, rai::packed_linear_bytes(vl, E.hidden, E.group_size))) return rc;
    RAI_CUDA(rai::pack_linear8(M->embed_codes + (size_t)M->v_off * E.hidden,
                               M->embed_params + (size_t)M->v_off * eng * 4, (int)vl, (int)E.hidden,
                               (int)E.group_size, packed, 0));
    M->head.data = packed;
    M->head.rows = (int)vl;
    M->head.cols = (int)E.hidden;
    M->head.group_size = (int)E.group_size;
    M->head.groups = (int)eng;
    M->head.tiles = (int)rai::ceil_div(vl, rai::kTileRows);
    M->head.wbits = 8;
  }
  std::vector<float> cs, sn;
  build_rope(c, c.rope_theta, cs, sn);
  if (int rc = upload(M.get(), cs.data(), cs.size() * 4, reinterpret_cast<void**>(&M->rope_cos))) return rc;
  if (int rc = upload(M.get(), sn.data(), sn.size() * 4, reinterpret_cast<void**>(&M->rope_sin))) return rc;
  if (tp_world > 1) {
    // Exchange arena: every rank maps every other rank's (rai_gpu_tp_connect).
    const char* env = std::getenv("RAI_TP_ARENA_MB");
    const size_t mb = env ? std::strtoull(env, nullptr, 10) : 1024;
    M->arena_bytes = std::max<size_t>(mb, 16) << 20;
    if (int rc = M->alloc(&M->arena, M->arena_bytes)) return rc;
    RAI_CUDA(cudaMemset(M->arena, 0, M->arena_bytes));
    M->flags_used = 0;
    M->arena_used = kArenaFlagBytes;
  }
  RAI_CUDA(cudaDeviceSynchronize());
  *out = M.release();
  return RAI_OK;
}

int rai_gpu_model_create(const uint8_t* blob, size_t len, int device, rai_model** out) {
  return create_model(blob, len, device, 0, 1, out);
}

int rai_gpu_model_create_tp(const uint8_t* blob, size_t len, int device, int tp_rank, int tp_size,
                            rai_model** out) {
  return create_model(blob, len, device, tp_rank, tp_size, out);
}

int rai_gpu_tp_handle(rai_model* m, void* handle, size_t cap) {
  if (!m || !handle) return fail(RAI_ERR_INVALID, "null argument");
  if (m->tp_world < 2) return fail(RAI_ERR_INVALID, "model is not tensor-parallel");
  if (cap < sizeof(cudaIpcMemHandle_t)) return fail(RAI_ERR_INVALID, "handle buffer below 64 bytes");
  DeviceGuard guard(m->device);
  cudaIpcMemHandle_t h;
  RAI_CUDA(cudaIpcGetMemHandle(&h, m->arena));
  std::memcpy(handle, &h, sizeof(h));
  return RAI_OK;
}

int rai_gpu_tp_connect(rai_model* m, const void* handles, size_t n) {
  if (!m || !handles) return fail(RAI_ERR_INVALID, "null argument");
  if (m->tp_world < 2) return fail(RAI_ERR_INVALID, "model is not tensor-parallel");
  if (n != (size_t)m->tp_world) return fail(RAI_ERR_INVALID, "one arena handle per rank expected");
  if (m->tp_connected) return fail(RAI_ERR_INVALID, "already connected");
  DeviceGuard guard(m->device);
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int t = 0; t < m->tp_world; ++t) {
    if (t == m->tp_rank) {
      m->peer_arena[t] = m->arena;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + (size_t)t * sizeof(h), sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return fail(RAI_ERR_DEVICE, std::string("cudaIpcOpenMemHandle(rank ") + std::to_string(t) +
                                      "): " + cudaGetErrorString(e));
    }
    m->ipc_opened.push_back(p);
    m->peer_arena[t] = static_cast<uint8_t*>(p);
  }
  m->tp_connected = true;
  return RAI_OK;
}


int rai_gpu_model_destroy(rai_model* model) {
  if (!model) return RAI_OK;
  if (const int n = model->live_decoders.load())
    return fail(RAI_ERR_INVALID, "model still has " + std::to_string(n) + " live decoder(s): destroy them first");
  drop_batches_of_model(model);
  delete model;
  return RAI_OK;
}

int rai_gpu_model_info(const rai_model* m, rai_model_info* info) {
  if (!m || !info) return fail(RAI_ERR_INVALID, "null argument");
  const Config& c = m->cfg;
  info->hidden_size = c.hidden_size;
  info->num_layers = c.num_layers;
  info->num_heads = c.num_heads;
  info->num_kv_heads = c.num_kv_heads;
  info->head_dim = c.head_dim;
  info->intermediate_size = c.intermediate_size;
  info->vocab_size = c.vocab_size;
  info->max_context = c.max_context;
  info->group_size = c.group_size;
  info->embed_group_size = c.embed_group_size;
  info->num_experts = c.num_experts;
  info->experts_per_token = c.experts_per_token;
  info->tied_embeddings = m->layout.has_lm_head ? 0 : 1;
  info->version = c.version;
  info->device_bytes = m->device_bytes;
  return RAI_OK;
}

int rai_gpu_model_set_gemm_mode(rai_model* m, int mode) {
  if (!m) return fail(RAI_ERR_INVALID, "null argument");
  if (mode != rai::kGemmAuto && mode != rai::kGemmExact && mode != rai::kGemmTol)
    return fail(RAI_ERR_INVALID, "gemm mode must be 0 (auto), 1 (exact) or 2 (tolerance)");
  m->gemm_mode = mode;
  return RAI_OK;
}

int rai_gpu_model_gemm_mode(const rai_model* m, int* mode) {
  if (!m || !mode) return fail(RAI_ERR_INVALID, "null argument");
  *mode = m->tp_world > 1 ? rai::kGemmExact : m->gemm_mode;
  return RAI_OK;
}

int rai_gpu_decoder_create(rai_model* m, size_t max_ctx, rai_dec** out) {
  if (!m || !out) return fail(RAI_ERR_INVALID, "null argument");
  *out = nullptr;
  if (int rc = check_usable(m)) return rc;
  size_t ctx = std::min<size_t>(max_ctx, m->cfg.max_context);
  if (ctx == 0) return fail(RAI_ERR_INVALID, "prompt-lookup context must be non-zero");
  DeviceGuard guard(m->device);
  const Config& c = m->cfg;
  auto d = std::make_unique<rai_dec>();
  d->m = m;
  ++m->live_decoders;  // ~rai_dec gives it back, on every path
  d->max_ctx = (int)ctx;
  // Under tensor parallelism a rank caches only its own KV heads.
  size_t kv = (size_t)c.num_layers * m->nkv_l * ctx * c.head_dim * sizeof(float);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, kv);
  if (e != cudaSuccess) return fail(RAI_ERR_OOM, "cannot allocate the KV cache");
  d->kc = static_cast<float*>(p);
  e = cudaMalloc(&p, kv);
  if (e != cudaSuccess) return fail(RAI_ERR_OOM, "cannot allocate the KV cache");
  d->vc = static_cast<float*>(p);
  RAI_CUDA(cudaMemset(d->kc, 0, kv));
  RAI_CUDA(cudaMemset(d->vc, 0, kv));
  d->filled.assign(c.num_layers, 0);
  int rows_cap = (int)std::max<size_t>(rai::kMaxRowsPerStream, std::min<size_t>(256, ctx));
  if (int rc = create_batch(m, {d.get()}, rai::kMaxRowsPerStream, rows_cap, &d->solo)) return rc;
  *out = d.release();
  return RAI_OK;
}

int rai_gpu_decoder_destroy(rai_dec* d) {
  delete d;
  return RAI_OK;
}

int rai_gpu_prefill(rai_dec* d, const uint32_t* ids, size_t n, size_t* pos_out) {
  if (!d || !pos_out || (!ids && n)) return fail(RAI_ERR_INVALID, "null argument");
  if (n == 0) return fail(RAI_ERR_INVALID, "prompt must contain at least one token");
  if (n > (size_t)d->max_ctx) return fail(RAI_ERR_INVALID, "prompt exceeds the prompt-lookup context window");
  if (int rc = check_usable(d->m)) return rc;
  const Config& c = d->m->cfg;
  for (size_t i = 0; i + 1 < n; ++i)
    if (ids[i] >= c.vocab_size) return fail(RAI_ERR_INVALID, "token id is out of model vocabulary");
  DeviceGuard guard(d->m->device);
  size_t m = n - 1;
  *pos_out = m;
  Batch* B = d->solo.get();
  for (size_t start = 0; start < m; start += B->rows_cap) {
    int rows = (int)std::min<size_t>(B->rows_cap, m - start);
    if (start > d->filled[0]) return fail(RAI_ERR_INVALID, "KV store would leave a gap");
    if (int rc = forward_solo(d, ids + start, start, rows, false)) return rc;
    if (int rc = check_err(d->m, B->stream)) return rc;
    for (auto& f : d->filled) f = std::max(f, start + rows);
  }
  return RAI_OK;
}

int rai_gpu_prefill_many(rai_dec* const* decs, size_t n, const uint32_t* const* ids, const size_t* lens,
                         size_t* pos_out) {
  if (!decs || !ids || !lens || !pos_out || n == 0) return fail(RAI_ERR_INVALID, "null argument");
  rai_model* m = decs[0]->m;
  const Config& c = m->cfg;
  if (m->tp_world > 1)
    return fail(RAI_ERR_UNSUPPORTED, "prefill_many on a tensor-parallel model (use rai_gpu_prefill per decoder)");
  for (size_t i = 0; i < n; ++i) {
    rai_dec* d = decs[i];
    if (!d || d->m != m) return fail(RAI_ERR_INVALID, "prefill_many decoders must share one model");
    for (size_t j = 0; j < i; ++j)
      if (decs[j] == d) return fail(RAI_ERR_INVALID, "prefill_many decoder listed twice");
    if (lens[i] == 0) return fail(RAI_ERR_INVALID, "prompt must contain at least one token");
    if (!ids[i]) return fail(RAI_ERR_INVALID, "null prompt");
    if (lens[i] > (size_t)d->max_ctx) return fail(RAI_ERR_INVALID, "prompt exceeds the prompt-lookup context window");
    if (d->filled[0] != 0) return fail(RAI_ERR_INVALID, "prefill_many needs empty caches");
    for (size_t t = 0; t + 1 < lens[i]; ++t)
      if (ids[i][t] >= c.vocab_size) return fail(RAI_ERR_INVALID, "token id is out of model vocabulary");
  }
  DeviceGuard guard(m->device);
  // All streams' prompt rows in order, cut into chunks of up to 2048 rows;
  // a stream's earlier positions are always in an earlier chunk or earlier
  // in the same chunk, whose K/V are stored before attention runs.
  const int chunk = 2048;
  std::unique_ptr<Batch> B;
  if (int rc = create_batch(m, std::vector<rai_dec*>(decs, decs + n), 1, chunk, &B)) return rc;
  std::vector<uint32_t> idbuf(chunk);
  int r = 0;
  auto flush = [&]() -> int {
    if (r == 0) return RAI_OK;
    cudaStream_t s = B->stream;
    RAI_CUDA(cudaMemcpyAsync(B->ids, idbuf.data(), r * 4, cudaMemcpyHostToDevice, s));
    if (int rc = forward_host_rows(B.get(), r, false)) return rc;
    if (int rc = check_err(m, s)) return rc;
    r = 0;
    return RAI_OK;
  };
  for (size_t i = 0; i < n; ++i) {
    for (size_t t = 0; t + 1 < lens[i]; ++t) {
      B->rows_host[r] = rai::RowInfo{(int)t, (int)i};
      idbuf[r] = ids[i][t];
      if (++r == chunk)
        if (int rc = flush()) return rc;
    }
  }
  if (int rc = flush()) return rc;
  for (size_t i = 0; i < n; ++i) {
    pos_out[i] = lens[i] - 1;
    for (auto& f : decs[i]->filled) f = std::max(f, lens[i] - 1);
  }
  return RAI_OK;
}

int rai_gpu_forward_logits(rai_dec* d, const uint32_t* ids, size_t start_pos, size_t batch, float* logits) {
  if (!d || !ids || batch == 0) return fail(RAI_ERR_INVALID, "bad argument");
  if (int rc = check_usable(d->m)) return rc;
  if (d->m->tp_world > 1 && !d->m->ep)
    return fail(RAI_ERR_UNSUPPORTED, "forward_logits on a tensor-parallel model (each rank holds a vocabulary slice)");
  const Config& c = d->m->cfg;
  if (batch > (size_t)rai::kMaxRowsPerStream) return fail(RAI_ERR_INVALID, "batch exceeds 33 rows");
  if (start_pos + batch > (size_t)d->max_ctx || start_pos + batch > c.max_context)
    return fail(RAI_ERR_INVALID, "batch position exceeds model context");
  if (start_pos > d->filled[0]) return fail(RAI_ERR_INVALID, "KV store would leave a gap");
  for (size_t i = 0; i < batch; ++i)
    if (ids[i] >= c.vocab_size) return fail(RAI_ERR_INVALID, "token id is out of model vocabulary");
  DeviceGuard guard(d->m->device);
  Batch* B = d->solo.get();
  if (int rc = forward_solo(d, ids, start_pos, (int)batch, true)) return rc;
  if (logits)
    RAI_CUDA(cudaMemcpyAsync(logits, B->logits, batch * c.vocab_size * 4, cudaMemcpyDeviceToHost, B->stream));
  if (int rc = check_err(d->m, B->stream)) return rc;
  for (auto& f : d->filled) f = std::max(f, start_pos + batch);
  return RAI_OK;
}

int rai_gpu_step(rai_dec* d, size_t pos, const uint32_t* ctx, size_t ctx_len, const rai_lookup_cfg* cfg,
                 uint32_t* out_tokens, size_t out_cap, size_t* n_out, rai_lookup_metrics* metrics) {
  if (!d || !ctx || !out_tokens || !n_out) return fail(RAI_ERR_INVALID, "null argument");
  DeviceGuard guard(d->m->device);
  const uint32_t* ctxs[1] = {ctx};
  return step_batch(d->solo.get(), &pos, ctxs, &ctx_len, cfg, out_tokens, out_cap, n_out, metrics);
}

int rai_gpu_step_many(rai_dec* const* decs, size_t n, const size_t* pos, const uint32_t* const* ctx,
                      const size_t* ctx_len, const rai_lookup_cfg* cfg, uint32_t* out_tokens, size_t out_cap,
                      size_t* n_out, rai_lookup_metrics* metrics) {
  if (!decs || !pos || !ctx || !ctx_len || !out_tokens || !n_out || n == 0) return fail(RAI_ERR_INVALID, "null argument");
  if (int rc = validate_cfg(cfg)) return rc;
  rai_model* m = decs[0]->m;
  for (size_t i = 0; i < n; ++i) {
    if (!decs[i] || decs[i]->m != m) return fail(RAI_ERR_INVALID, "step_many decoders must share one model");
    for (size_t j = 0; j < i; ++j)
      if (decs[j] == decs[i]) return fail(RAI_ERR_INVALID, "step_many decoder listed twice");
  }
  if (n == 1) return rai_gpu_step(decs[0], pos[0], ctx[0], ctx_len[0], cfg, out_tokens, out_cap, n_out, metrics);
  DeviceGuard guard(m->device);
  std::vector<rai_dec*> key(decs, decs + n);
  const int R = (int)cfg->max_draft + 1;
  Batch* B = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_batch_mu);
    for (auto& e : g_batches)
      if (e.first == m && e.second->decs == key && e.second->R >= R) B = e.second.get();
  }
  if (!B) {
    std::unique_ptr<Batch> nb;
    if (int rc = create_batch(m, key, R, (int)n * R, &nb)) return rc;
    B = nb.get();
    std::lock_guard<std::mutex> lk(g_batch_mu);
    g_batches.emplace_back(m, std::move(nb));
  }
  return step_batch(B, pos, ctx, ctx_len, cfg, out_tokens, out_cap, n_out, metrics);
}

int rai_gpu_spec_create(rai_model* target, rai_model* draft, size_t max_ctx, rai_spec** out) {
  if (!target || !draft || !out) return fail(RAI_ERR_INVALID, "null argument");
  *out = nullptr;
  if (target->device != draft->device) return fail(RAI_ERR_INVALID, "target and draft models must share a device");
  if (target->cfg.vocab_size != draft->cfg.vocab_size)
    return fail(RAI_ERR_INVALID, "target and draft models must share a vocabulary");
  if (target->tp_world > 1 || draft->tp_world > 1)
    return fail(RAI_ERR_UNSUPPORTED, "speculative decoding on multi-GPU models");
  auto S = std::make_unique<rai_spec>();
  if (int rc = rai_gpu_decoder_create(target, max_ctx, &S->td)) return rc;
  if (int rc = rai_gpu_decoder_create(draft, max_ctx, &S->dd)) return rc;
  S->max_ctx = std::min(S->td->max_ctx, S->dd->max_ctx);
  S->vocab = (int)target->cfg.vocab_size;
  DeviceGuard guard(target->device);
  RAI_CUDA(cudaMalloc(&S->draft_logits, (size_t)rai::kMaxRowsPerStream * S->vocab * 4));
  RAI_CUDA(cudaMalloc(&S->st, sizeof(rai::StreamStep)));
  RAI_CUDA(cudaMalloc(&S->best, rai::kMaxRowsPerStream * 8));
  RAI_CUDA(cudaMallocHost(&S->st_host, sizeof(rai::StreamStep)));
  *out = S.release();
  return RAI_OK;
}

int rai_gpu_spec_destroy(rai_spec* s) {
  delete s;
  return RAI_OK;
}

int rai_gpu_spec_set_seed(rai_spec* s, uint64_t seed) {
  if (!s) return fail(RAI_ERR_INVALID, "null argument");
  s->seed = seed;
  s->steps = 0;
  // The draft model's sampling draws from its own stream of the same seed.
  rai_gpu_set_seed(s->dd, seed ^ 0x9E3779B97F4A7C15ull);
  rai_gpu_set_seed(s->td, seed ^ 0xBB67AE8584CAA73Bull);
  return RAI_OK;
}

int rai_gpu_spec_prefill(rai_spec* s, const uint32_t* ids, size_t n, size_t* pos_out) {
  if (!s || !pos_out) return fail(RAI_ERR_INVALID, "null argument");
  size_t p2 = 0;
  if (int rc = rai_gpu_prefill(s->td, ids, n, pos_out)) return rc;
  return rai_gpu_prefill(s->dd, ids, n, &p2);
}

int rai_gpu_spec_step(rai_spec* s, size_t pos, uint32_t last_token, const rai_spec_cfg* cfg, uint32_t* out,
                      size_t out_cap, size_t* n_out, rai_lookup_metrics* metrics) {
  if (!s || !cfg || !out || !n_out) return fail(RAI_ERR_INVALID, "null argument");
  // validate_speculative_config (speculative.rs:396-407); temperature 0 is
  // the greedy limit (an extension, as for prompt lookup).
  if (cfg->draft_k == 0) return fail(RAI_ERR_INVALID, "speculative draft_k must be non-zero");
  if (cfg->draft_k + 1 > (uint32_t)rai::kMaxRowsPerStream) return fail(RAI_ERR_INVALID, "draft_k exceeds 32");
  const float t = cfg->temperature;
  if (!std::isfinite(t) || (t != 0.f && !(t > 1e-6f)))
    return fail(RAI_ERR_INVALID, "speculative decoding requires temperature 0 (greedy) or a finite temperature > 1e-6");
  if (cfg->top_k != 0 || cfg->top_p != 1.0f || cfg->repetition_penalty != 1.0f)
    return fail(RAI_ERR_INVALID, "speculative decoding requires top_k=0, top_p=1, and repetition_penalty=1");
  if (pos >= (size_t)s->max_ctx) return fail(RAI_ERR_INVALID, "decode position exceeds the speculative context window");
  if ((int)last_token >= s->vocab) return fail(RAI_ERR_INVALID, "token id is out of model vocabulary");
  if (pos > s->td->filled[0] || pos > s->dd->filled[0]) return fail(RAI_ERR_INVALID, "KV store would leave a gap");
  const size_t k = std::min<size_t>(cfg->draft_k, (size_t)s->max_ctx - pos - 1);
  if (out_cap < k + 1) return fail(RAI_ERR_INVALID, "out_tokens capacity below draft_k + 1");
  DeviceGuard guard(s->td->m->device);
  if (k == 0) {
    uint32_t tok = 0;
    if (int rc = rai_gpu_decode_one(s->td, pos, last_token, t, &tok)) return rc;
    out[0] = tok;
    *n_out = 1;
    if (metrics) *metrics = rai_lookup_metrics{0, 0, 1, 0, 0.f};
    ++s->steps;
    return RAI_OK;
  }
  // Phase 1: the draft model proposes k tokens one row at a time; each row's
  // logits are kept for the acceptance.
  Batch* DB = s->dd->solo.get();
  std::vector<uint32_t> ids(k + 1);
  ids[0] = last_token;
  uint32_t cur = last_token;
  for (size_t i = 0; i < k; ++i) {
    uint32_t next = 0;
    if (int rc = rai_gpu_decode_one(s->dd, pos + i, cur, t, &next)) return rc;
    RAI_CUDA(cudaMemcpyAsync(s->draft_logits + i * s->vocab, DB->logits, (size_t)s->vocab * 4,
                             cudaMemcpyDeviceToDevice, DB->stream));
    ids[i + 1] = next;
    cur = next;
  }
  RAI_CUDA(cudaStreamSynchronize(DB->stream));
  // Phase 2: the target verifies all k + 1 rows in one forward.
  Batch* TB = s->td->solo.get();
  if (int rc = forward_solo(s->td, ids.data(), pos, (int)k + 1, true)) return rc;
  for (auto& f : s->td->filled) f = std::max(f, pos + k + 1);
  // Phase 3: accept / reject.
  rai::StreamStep& h = *s->st_host;
  std::memset(&h, 0, sizeof(h));
  h.pos = (int)pos;
  h.drafted = (int)k;
  h.n_rows = (int)k + 1;
  h.row0 = 0;
  for (size_t i = 0; i <= k; ++i) h.tokens[i] = ids[i];
  h.rng_seed_lo = (uint32_t)s->seed;
  h.rng_seed_hi = (uint32_t)(s->seed >> 32);
  h.rng_step_lo = (uint32_t)s->steps;
  h.rng_step_hi = (uint32_t)(s->steps >> 32);
  cudaStream_t st = TB->stream;
  RAI_CUDA(cudaMemcpyAsync(s->st, &h, sizeof(h), cudaMemcpyHostToDevice, st));
  if (t > 0.f) {
    RAI_CUDA(rai::launch_sample_accept(s->st, 1, TB->logits, s->vocab, t, st, s->draft_logits));
  } else {
    RAI_CUDA(cudaMemsetAsync(s->best, 0, (k + 1) * 8, st));
    RAI_CUDA(rai::launch_argmax(TB->logits, s->vocab, nullptr, (int)k + 1, s->best, st));
    RAI_CUDA(rai::launch_accept(s->st, 1, s->best, st));
  }
  RAI_CUDA(cudaMemcpyAsync(&h, s->st, sizeof(h), cudaMemcpyDeviceToHost, st));
  if (int rc = check_err(s->td->m, st)) return rc;
  const size_t produced = (size_t)h.produced;
  if ((size_t)h.accepted == k) {
    // Every draft accepted: the draft model has not yet run its last
    // proposal; run it so its cache has no missing position.
    if (int rc = forward_solo(s->dd, &ids[k], pos + k, 1, false)) return rc;
    if (int rc = check_err(s->dd->m, DB->stream)) return rc;
  }
  // Roll both caches back to the produced frontier.
  for (auto& f : s->td->filled) f = pos + produced;
  for (auto& f : s->dd->filled) f = pos + produced;
  for (size_t i = 0; i < produced; ++i) out[i] = h.out[i];
  *n_out = produced;
  if (metrics)
    *metrics = rai_lookup_metrics{(uint32_t)h.accepted, (uint32_t)k, (uint32_t)produced, 0,
                                  (float)h.accepted / (float)k};
  ++s->steps;
  return RAI_OK;
}

int rai_gpu_decode_one(rai_dec* d, size_t pos, uint32_t last_token, float temperature, uint32_t* token) {
  if (!d || !token) return fail(RAI_ERR_INVALID, "null argument");
  if (!std::isfinite(temperature) || (temperature != 0.f && !(temperature > 1e-6f)))
    return fail(RAI_ERR_INVALID, "decoding requires temperature 0 (greedy) or temperature > 1e-6");
  if (last_token >= d->m->cfg.vocab_size) return fail(RAI_ERR_INVALID, "token id is out of model vocabulary");
  DeviceGuard guard(d->m->device);
  // The step graph with no draft search: one verify row, the bonus token.
  rai_lookup_cfg cfg = {1, 0, 1, temperature, 0, 1.0f, 1.0f};
  const uint32_t* ctxs[1] = {&last_token};
  const size_t len = 1;
  uint32_t out[2] = {0, 0};
  size_t n = 0;
  if (int rc = step_batch(d->solo.get(), &pos, ctxs, &len, &cfg, out, 2, &n, nullptr, false)) return rc;
  *token = out[0];
  return RAI_OK;
}

int rai_gpu_sample_accept(const float* logits, const float* draft_logits, size_t vocab, const uint32_t* draft,
                          size_t n_drafted, float temperature, uint64_t seed, uint64_t step, uint32_t* out,
                          size_t* n_out, size_t* accepted) {
  if (!logits || !out || !n_out || !accepted || (n_drafted && !draft) || vocab == 0)
    return fail(RAI_ERR_INVALID, "null argument");
  if (n_drafted + 1 > (size_t)rai::kMaxRowsPerStream) return fail(RAI_ERR_INVALID, "more than 32 drafts");
  if (!(std::isfinite(temperature) && temperature > 1e-6f))
    return fail(RAI_ERR_INVALID, "sampled acceptance requires a finite temperature > 1e-6");
  rai::StreamStep h = {};
  h.drafted = (int)n_drafted;
  h.n_rows = (int)n_drafted + 1;
  h.row0 = 0;
  for (size_t i = 0; i < n_drafted; ++i) h.tokens[1 + i] = draft[i];
  h.rng_seed_lo = (uint32_t)seed;
  h.rng_seed_hi = (uint32_t)(seed >> 32);
  h.rng_step_lo = (uint32_t)step;
  h.rng_step_hi = (uint32_t)(step >> 32);
  rai::StreamStep* d = nullptr;
  RAI_CUDA(cudaMalloc(&d, sizeof(h)));
  struct Free { void* p; ~Free() { cudaFree(p); } } fr{d};
  RAI_CUDA(cudaMemcpy(d, &h, sizeof(h), cudaMemcpyHostToDevice));
  RAI_CUDA(rai::launch_sample_accept(d, 1, logits, (int)vocab, temperature, 0, draft_logits));
  RAI_CUDA(cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost));
  *n_out = (size_t)h.produced;
  *accepted = (size_t)h.accepted;
  for (int i = 0; i < h.produced; ++i) out[i] = h.out[i];
  return RAI_OK;
}

int rai_gpu_set_seed(rai_dec* d, uint64_t seed) {
  if (!d) return fail(RAI_ERR_INVALID, "null argument");
  d->rng_seed = seed;
  d->rng_steps = 0;
  return RAI_OK;
}

int rai_gpu_kv_filled(const rai_dec* d, size_t layer, size_t* filled) {
  if (!d || !filled) return fail(RAI_ERR_INVALID, "null argument");
  if (layer >= d->filled.size()) return fail(RAI_ERR_INVALID, "layer index out of range");
  *filled = d->filled[layer];
  return RAI_OK;
}

int rai_gpu_kv_truncate(rai_dec* d, size_t len) {
  if (!d) return fail(RAI_ERR_INVALID, "null argument");
  for (auto& f : d->filled) f = std::min(f, len);
  return RAI_OK;
}

int rai_gpu_kv_read(const rai_dec* d, size_t layer, size_t kvh, size_t pos, float* k, float* v) {
  if (!d || !k || !v) return fail(RAI_ERR_INVALID, "null argument");
  const Config& c = d->m->cfg;
  const size_t nkv = (size_t)d->m->nkv_l;  // this rank's KV heads under tensor parallelism
  if (layer >= c.num_layers || kvh >= nkv) return fail(RAI_ERR_INVALID, "KV cache head is out of range");
  if (pos >= d->filled[layer]) return fail(RAI_ERR_INVALID, "KV read at unwritten position");
  DeviceGuard guard(d->m->device);
  size_t off = ((layer * nkv + kvh) * (size_t)d->max_ctx + pos) * c.head_dim;
  RAI_CUDA(cudaMemcpy(k, d->kc + off, c.head_dim * 4, cudaMemcpyDeviceToHost));
  RAI_CUDA(cudaMemcpy(v, d->vc + off, c.head_dim * 4, cudaMemcpyDeviceToHost));
  return RAI_OK;
}

int rai_gpu_step_kernel_count(const rai_dec* d, size_t* kernels) {
  if (!d || !kernels) return fail(RAI_ERR_INVALID, "null argument");
  *kernels = d->last_kernels;
  return RAI_OK;
}

int rai_gpu_last_step_us(const rai_dec* d, float* us) {
  if (!d || !us) return fail(RAI_ERR_INVALID, "null argument");
  *us = d->last_us;
  return RAI_OK;
}

// ---- kernel-level entry points ----
// A packed buffer holds the mma.sync blocks, then (at tc_offset) the
// tcgen05 weight image.
namespace {
size_t tc_offset(size_t rows, size_t cols, size_t gs) {
  return rai::round_up(rai::packed_linear_bytes(rows, cols, gs), 256);
}
PackedLinear packed_view(const void* packed, size_t rows, size_t cols, size_t gs) {
  PackedLinear w;
  w.data = static_cast<const uint8_t*>(packed);
  w.tc = w.data + tc_offset(rows, cols, gs);
  w.rows = (int)rows;
  w.cols = (int)cols;
  w.group_size = (int)gs;
  w.groups = (int)rai::ceil_div(cols, gs);
  w.tiles = (int)rai::ceil_div(rows, rai::kTileRows);
  w.wbits = 4;
  return w;
}
}  // namespace

namespace {
// Sizes the kernel-level linear accepts: counts stay far inside the int
// ranges the kernels index with (rows and columns below 2^30, tokens below
// 2^24, the group count within the kernels' limit), checked before any
// narrowing.
constexpr size_t kMaxLinearDim = (size_t)1 << 30, kMaxLinearTokens = (size_t)1 << 24;
int check_linear(size_t rows, size_t cols, size_t tokens, size_t gs) {
  if (gs != 64 && gs != 128) return fail(RAI_ERR_UNSUPPORTED, "group_size must be 64 or 128");
  if (tokens == 0 || rows == 0 || cols == 0 || cols % 2) return fail(RAI_ERR_INVALID, "bad dimensions");
  if (rows > kMaxLinearDim || cols > kMaxLinearDim || tokens > kMaxLinearTokens)
    return fail(RAI_ERR_INVALID, "rows / cols above 2^30 or tokens above 2^24");
  if (rai::ceil_div(cols, gs) > raimodel::kMaxGroups)
    return fail(RAI_ERR_INVALID, "quantization group count exceeds kernel capacity");
  return RAI_OK;
}
}  // namespace

size_t rai_gpu_w4a8_packed_bytes(size_t rows, size_t cols, size_t gs) {
  return tc_offset(rows, cols, gs) + rai::tc_image_bytes(rows, cols, gs);
}

int rai_gpu_w4a8_pack(const uint8_t* nibbles, const uint8_t* params, size_t rows, size_t cols, size_t gs,
                      void* packed, void* stream) {
  if (!nibbles || !params || !packed) return fail(RAI_ERR_INVALID, "null argument");
  if (int rc = check_linear(rows, cols, 1, gs)) return rc;
  RAI_CUDA(rai::pack_linear4(nibbles, params, (int)rows, (int)cols, (int)gs, static_cast<uint8_t*>(packed),
                             static_cast<cudaStream_t>(stream)));
  RAI_CUDA(rai::pack_linear4_tc(nibbles, params, (int)rows, (int)cols, (int)gs,
                                static_cast<uint8_t*>(packed) + tc_offset(rows, cols, gs),
                                static_cast<cudaStream_t>(stream)));
  return RAI_OK;
}

size_t rai_gpu_w4a8_scratch_bytes(size_t tokens, size_t cols, size_t gs) {
  if (tokens > kMaxLinearTokens || gs == 0) return SIZE_MAX;  // rejected by every entry that takes a scratch
  return rai::round_up(tokens, 8) * rai::kActTokBytes * rai::ceil_div(cols, gs);
}

int rai_gpu_w4a8_matmul(float* out, const void* packed, const float* input, size_t rows, size_t cols, size_t tokens,
                        size_t gs, void* scratch, size_t scratch_bytes, void* stream) {
  if (!out || !packed || !input || !scratch) return fail(RAI_ERR_INVALID, "null argument");
  if (int rc = check_linear(rows, cols, tokens, gs)) return rc;
  if (scratch_bytes < rai_gpu_w4a8_scratch_bytes(tokens, cols, gs)) return fail(RAI_ERR_INVALID, "scratch buffer is too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  RAI_CUDA(rai::init_gemm_attributes());
  ActBuf a;
  a.data = static_cast<uint8_t*>(scratch);
  a.tok_alloc = (int)rai::round_up(tokens, 8);
  a.groups = (int)rai::ceil_div(cols, gs);
  uint32_t* err = nullptr;
  if (int rc = kernel_err_word(&err)) return rc;
  RAI_CUDA(rai::quantize_act(input, (int)cols, (int)tokens, nullptr, (int)cols, (int)gs, 4, a, s));
  const PackedLinear w = packed_view(packed, rows, cols, gs);
  RAI_CUDA(rai::gemm_exact(w, a, (int)tokens, out, (int)rows, rai::GemmEpilogue{}, err, s));
  return RAI_OK;
}

int rai_gpu_attention(const float* q, const float* k, const float* v, const int* positions, size_t M, size_t nh,
                      size_t nkv, size_t hd, size_t max_ctx, float scale, float* out, void* stream) {
  if (!q || !k || !v || !positions || !out || M == 0) return fail(RAI_ERR_INVALID, "null argument");
  if (nh % nkv || nh / nkv > 8 || (hd != 16 && hd != 32 && hd != 64 && hd != 128))
    return fail(RAI_ERR_UNSUPPORTED, "attention shape");
  for (size_t i = 0; i < M; ++i)
    if (positions[i] < 0 || (size_t)positions[i] >= max_ctx) return fail(RAI_ERR_INVALID, "position out of range");
  rai::ExpfTable et;
  if (int rc = expf_table(&et)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  RAI_CUDA(rai::init_layer_attributes());
  int n_alloc = (int)rai::round_up(max_ctx, 4);
  std::vector<rai::RowInfo> rows(M);
  for (size_t i = 0; i < M; ++i) rows[i] = rai::RowInfo{positions[i], 0};
  std::vector<rai::AttnSeg> segs(M);
  const int nseg = rai::build_segments(rows.data(), (int)M, rai::kSegRows, segs.data());
  int seg_rows = 1;
  for (int i = 0; i < nseg; ++i) seg_rows = std::max(seg_rows, segs[i].nrows);
  rai::StreamKV kv{const_cast<float*>(k), const_cast<float*>(v), (int)max_ctx, 0};
  char* buf = nullptr;
  const size_t off_seg = rai::round_up(M * sizeof(rai::RowInfo), 16);
  const size_t off_kv = off_seg + rai::round_up(nseg * sizeof(rai::AttnSeg), 16);
  const size_t off_err = rai::round_up(off_kv + sizeof(kv), 16);
  const size_t off_sc = off_err + 16;
  const size_t need = off_sc + M * nh * n_alloc * 4;
  RAI_CUDA(cudaMalloc(&buf, need));
  struct Free { char* p; ~Free() { cudaFree(p); } } fr{buf};
  rai::RowInfo* rows_d = reinterpret_cast<rai::RowInfo*>(buf);
  rai::AttnSeg* segs_d = reinterpret_cast<rai::AttnSeg*>(buf + off_seg);
  rai::StreamKV* kv_d = reinterpret_cast<rai::StreamKV*>(buf + off_kv);
  float* scores = reinterpret_cast<float*>(buf + off_sc);
  uint32_t* err_d = reinterpret_cast<uint32_t*>(buf + off_err);
  RAI_CUDA(cudaMemsetAsync(err_d, 0, 4, s));
  RAI_CUDA(cudaMemcpyAsync(rows_d, rows.data(), M * sizeof(rai::RowInfo), cudaMemcpyHostToDevice, s));
  RAI_CUDA(cudaMemcpyAsync(segs_d, segs.data(), nseg * sizeof(rai::AttnSeg), cudaMemcpyHostToDevice, s));
  RAI_CUDA(cudaMemcpyAsync(kv_d, &kv, sizeof(kv), cudaMemcpyHostToDevice, s));
  RAI_CUDA(rai::launch_attention(q, out, kv_d, 0, rows_d, nullptr, (int)M, segs_d, nullptr, nseg, seg_rows, (int)nh,
                                 (int)nkv, (int)hd, scale, 0.f, scores, n_alloc, et, err_d, s));
  uint32_t e = 0;
  RAI_CUDA(cudaMemcpyAsync(&e, err_d, 4, cudaMemcpyDeviceToHost, s));
  RAI_CUDA(cudaStreamSynchronize(s));
  if (e) return fail(RAI_ERR_TIMEOUT, "a device-side wait timed out");
  return RAI_OK;
}

int rai_gpu_kernel_status(void* stream) {
  uint32_t* err = nullptr;
  if (int rc = kernel_err_word(&err)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t e = 0;
  RAI_CUDA(cudaMemcpyAsync(&e, err, 4, cudaMemcpyDeviceToHost, s));
  RAI_CUDA(cudaStreamSynchronize(s));
  if (e) {
    RAI_CUDA(cudaMemsetAsync(err, 0, 4, s));
    RAI_CUDA(cudaStreamSynchronize(s));
    return fail(RAI_ERR_TIMEOUT, "a device-side wait of a kernel-level call timed out (its output is incomplete)");
  }
  return RAI_OK;
}

int rai_gpu_expf_range(uint32_t first_bits, size_t n, float* out, void* stream) {
  if (!out && n) return fail(RAI_ERR_INVALID, "null argument");
  if (n > ((size_t)1 << 32) - first_bits) return fail(RAI_ERR_INVALID, "range passes 2^32");
  rai::ExpfTable et;
  if (int rc = expf_table(&et)) return rc;
  if (n) RAI_CUDA(rai::launch_expf_range(first_bits, n, out, et, static_cast<cudaStream_t>(stream)));
  return RAI_OK;
}

int rai_gpu_w4a8_quantize(const float* input, size_t cols, size_t tokens, size_t gs, void* scratch,
                          size_t scratch_bytes, void* stream) {
  if (!input || !scratch) return fail(RAI_ERR_INVALID, "null argument");
  if (int rc = check_linear(1, cols, tokens, gs)) return rc;
  if (scratch_bytes < rai_gpu_w4a8_scratch_bytes(tokens, cols, gs)) return fail(RAI_ERR_INVALID, "scratch buffer is too small");
  ActBuf a;
  a.data = static_cast<uint8_t*>(scratch);
  a.tok_alloc = (int)rai::round_up(tokens, 8);
  a.groups = (int)rai::ceil_div(cols, gs);
  RAI_CUDA(rai::quantize_act(input, (int)cols, (int)tokens, nullptr, (int)cols, (int)gs, 4, a,
                             static_cast<cudaStream_t>(stream)));
  return RAI_OK;
}

int rai_gpu_w4a8_matmul_prequant(float* out, const void* packed, const void* scratch, size_t rows, size_t cols,
                                 size_t tokens, size_t gs, void* stream) {
  if (!out || !packed || !scratch) return fail(RAI_ERR_INVALID, "null argument");
  if (int rc = check_linear(rows, cols, tokens, gs)) return rc;
  RAI_CUDA(rai::init_gemm_attributes());
  ActBuf a;
  a.data = static_cast<uint8_t*>(const_cast<void*>(scratch));
  a.tok_alloc = (int)rai::round_up(tokens, 8);
  a.groups = (int)rai::ceil_div(cols, gs);
  const PackedLinear w = packed_view(packed, rows, cols, gs);
  uint32_t* err = nullptr;
  if (int rc = kernel_err_word(&err)) return rc;
  RAI_CUDA(rai::gemm_exact(w, a, (int)tokens, out, (int)rows, rai::GemmEpilogue{}, err,
                           static_cast<cudaStream_t>(stream)));
  return RAI_OK;
}

size_t rai_gpu_w4a8_tol_workspace_bytes(void) { return rai::gemm_tol_workspace_bytes(); }

int rai_gpu_w4a8_matmul_tol_prequant(float* out, const void* packed, const void* scratch, size_t rows, size_t cols,
                                     size_t tokens, size_t gs, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  if (!out || !packed || !scratch) return fail(RAI_ERR_INVALID, "null argument");
  if (int rc = check_linear(rows, cols, tokens, gs)) return rc;
  if (workspace && workspace_bytes < rai::gemm_tol_workspace_bytes())
    return fail(RAI_ERR_INVALID, "workspace smaller than rai_gpu_w4a8_tol_workspace_bytes()");
  RAI_CUDA(rai::init_gemm_attributes());
  ActBuf a;
  a.data = static_cast<uint8_t*>(const_cast<void*>(scratch));
  a.tok_alloc = (int)rai::round_up(tokens, 8);
  a.groups = (int)rai::ceil_div(cols, gs);
  const PackedLinear w = packed_view(packed, rows, cols, gs);
  uint32_t* err = nullptr;
  if (int rc = kernel_err_word(&err)) return rc;
  RAI_CUDA(rai::gemm_tol(w, a, (int)tokens, out, (int)rows, rai::GemmEpilogue{}, err, static_cast<cudaStream_t>(stream),
                         nullptr, workspace, workspace_bytes));
  return RAI_OK;
}

int rai_gpu_w4a8_matmul_static(float* out, const void* packed, const float* input, size_t rows, size_t cols,
                               size_t tokens, size_t gs, void* stream) {
  if (!out || !packed || !input) return fail(RAI_ERR_INVALID, "null argument");
  if (int rc = check_linear(rows, cols, tokens, gs)) return rc;
  const size_t need = rai_gpu_w4a8_scratch_bytes(tokens, cols, gs);
  if (need > kStaticScratchBytes)
    return fail(RAI_ERR_INVALID, "tokens x groups exceed the 2 MiB static scratch (136 B per token per group, "
                                 "tokens rounded up to 8)");
  void* scratch = nullptr;
  if (int rc = static_scratch(&scratch)) return rc;
  return rai_gpu_w4a8_matmul(out, packed, input, rows, cols, tokens, gs, scratch, need, stream);
}

}  // extern "C"
