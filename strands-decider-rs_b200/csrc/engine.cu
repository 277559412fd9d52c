// The torso engine behind the C ABI (include/sd_b200.h): model loading, the per-layer launch
// sequence, snapshots, and the pointer head. It replaces the reference's `Engine`
// (src/engine.rs:104-662) and `Head` (src/head.rs).
//
// Device layout: the weight shard is uploaded as is (norm weights, conv taps and gate constants are
// read from it in place); every int4 matmul weight is repacked once into the GEMM's tile layout
// (gate_up with gate and up rows interleaved, for the SwiGLU epilogue); the embedding table keeps
// the reference's packed rows. Per gated-delta layer: state [16][128][128] f32 and conv history
// [3][6144] f16; per attention layer: K and V caches [2][4096][256] f16. Activations live in a pool
// sized for the longest forward so far.
#include <immintrin.h>
#include <sys/stat.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/sd_b200.h"
#include "json.h"
#include "sd_internal.h"

using sd::QWeight;

struct sd_engine;

namespace {
thread_local std::string g_last_error;
void set_global_error(const std::string& s) { g_last_error = s; }
}  // namespace

namespace sd {
void set_last_error(const std::string& s) { set_global_error(s); }
}  // namespace sd

namespace {

struct LayerW {
  int kind = 0;  // 0 linear_attention, 1 full_attention, 2 adapter
  int slot = -1;
  const float* in_norm = nullptr;
  const float* post_norm = nullptr;
  QWeight in_proj, out_proj, qkv, o_proj, gate_up, down, proj;
  const float *conv = nullptr, *neg_a = nullptr, *dt_bias = nullptr, *gnorm = nullptr;
  const float *q_norm = nullptr, *k_norm = nullptr, *bias = nullptr;
};

bool file_exists(const std::string& path) {
  struct stat st;
  return stat(path.c_str(), &st) == 0;
}

bool read_file(const std::string& path, std::string& out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  std::ostringstream ss;
  ss << f.rdbuf();
  out = ss.str();
  return true;
}

}  // namespace

// A snapshot is one stream-ordered allocation: [n_lin state][n_lin hist][n_full K][n_full V], K and
// V compact as [hk][len][hd]. It is freed on its engine's stream, after any work that reads it.
struct sd_snapshot {
  int len = 0;
  int device = 0;
  sd_engine* owner = nullptr;
  uint8_t* base = nullptr;
  std::vector<float*> state;
  std::vector<__half*> hist, k, v;
  ~sd_snapshot();
};

struct sd_qweight {
  QWeight w;
  int device = 0;
};

struct sd_head {
  std::vector<float> nw, nb, qw, qb, kw, kb;
  int dim = 0, d = 0;
  // the weights on each device that ran the head there ([qw | kw | nw | nb | qb | kb] f32), uploaded
  // on first use
  mutable std::mutex mu;
  mutable float* dev[sd::kMaxDevices] = {};
};

struct sd_engine {
  int device = 0;
  int num_sms = 148;
  // which scan the gated-delta layers take: 0 the faster by gdn_pick's estimate, 1 always the fused
  // tcgen05 scan (gdn_tc.cu), 2 always the mma.sync scans (single-pass and two-phase); set once at
  // engine creation from SD_GDN_KERNEL (unset, "tc" or "legacy"), for comparisons
  int gdn_mode = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  sd::Dims dm;
  int vocab = 0, n_layers = 0, embed_bits = 4;
  double rope_theta = 1e7;
  std::vector<double> unrotate;
  std::vector<uint8_t*> shards;
  std::vector<std::pair<uint64_t, uint64_t>> shard_ranges;
  uint8_t* embed_q = nullptr;
  __half* embed_s = nullptr;
  const float* final_norm = nullptr;
  std::vector<LayerW> layers;
  std::vector<float*> state;
  std::vector<__half*> hist, kc, vc;
  float* rope = nullptr;
  int n_lin = 0, n_full = 0;
  int in_n = 0, qkv_n = 0;
  // activation pool
  int cap = 0;
  uint32_t* d_ids = nullptr;
  int* d_rows = nullptr;
  float *x = nullptr, *of = nullptr, *beta = nullptr, *decay = nullptr, *out = nullptr, *ws = nullptr;
  float* trace_dev = nullptr;
  size_t ws_bytes = 0;
  void* gdn_scratch = nullptr;  // per-chunk records of the two-phase scan
  size_t gdn_scratch_bytes = 0;
  __half *h = nullptr, *big = nullptr, *mid = nullptr, *o = nullptr, *y = nullptr, *q = nullptr, *qkvc = nullptr;
  int* d_err = nullptr;
  // snapshots: stream-ordered allocations from the engine's own pool, which keeps freed memory
  // (release threshold unlimited), so a snapshot after a synchronisation does not map memory anew
  cudaMemPool_t snap_pool = nullptr;
  // batched fork: per-token / per-sequence index arrays and the packed tokens' K and V (one attention
  // layer at a time), grown as needed
  int* fk_meta = nullptr;
  size_t fk_meta_ints = 0;
  __half* fk_kv = nullptr;
  size_t fk_kv_halves = 0;
  // continuations' keys and values gathered per sequence (prefix then own rows) for the tcgen05
  // attention: [2][hk][ktot][hd], grown as needed
  __half* fk_gather = nullptr;
  size_t fk_gather_halves = 0;
  // pinned staging of fk_meta: a ring of slots, each reused once the copy out of it (event) is done
  static constexpr int kForkSlots = 4;
  int* fk_pin[kForkSlots] = {};
  size_t fk_pin_ints[kForkSlots] = {};
  cudaEvent_t fk_ev[kForkSlots] = {};
  int fk_next = 0;
  // pinned staging
  uint32_t* p_ids = nullptr;
  int* p_rows = nullptr;
  float* p_out = nullptr;
  int p_cap = 0;      // tokens of p_ids
  int p_row_cap = 0;  // rows of p_rows and p_out
  float* trace_host = nullptr;
  size_t trace_floats = 0;
  // the pointer head on the device: question table, xn, proj and probabilities (grown as needed),
  // the rotated torso's per-channel factors, and pinned staging of the probabilities
  void* hd_buf = nullptr;
  size_t hd_bytes = 0;
  double* d_unrot = nullptr;
  double* hd_pin = nullptr;
  size_t hd_pin_doubles = 0;
  std::string err;
  // launches of this library's kernels since creation
  long long launches = 0;
  // profiling (the reference's `Engine::profile`, src/engine.rs:665-711): events around each launch
  bool prof_on = false;
  std::vector<cudaEvent_t> prof_events;
  size_t prof_used = 0;
  std::vector<std::pair<int, double>> prof_pending;  // (kind, algorithmic units) per event pair
  double prof_ms[SD_PROF_KINDS] = {}, prof_units[SD_PROF_KINDS] = {};
  long long prof_count[SD_PROF_KINDS] = {};
  std::vector<sd_snapshot*> live;

  int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    err = buf;
    set_global_error(err);
    return code;
  }
};

sd_snapshot::~sd_snapshot() {
  if (!base) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  if (owner) {
    cudaFreeAsync(base, owner->stream);  // after any queued work that reads it
    auto& v = owner->live;
    v.erase(std::remove(v.begin(), v.end(), this), v.end());
  } else {
    cudaFree(base);
  }
  cudaSetDevice(prev);
}

#define CK(call)                                                                                    \
  do {                                                                                              \
    cudaError_t _e = (call);                                                                        \
    if (_e != cudaSuccess) return e->fail(SD_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(_e)); \
  } while (0)

namespace {

void free_pool(sd_engine* e) {
  cudaFree(e->d_ids); cudaFree(e->d_rows); cudaFree(e->x); cudaFree(e->qkvc); cudaFree(e->of); cudaFree(e->beta);
  cudaFree(e->decay); cudaFree(e->out); cudaFree(e->ws); cudaFree(e->h); cudaFree(e->big); cudaFree(e->mid);
  cudaFree(e->o); cudaFree(e->y); cudaFree(e->q); cudaFree(e->trace_dev); cudaFree(e->gdn_scratch);
  e->gdn_scratch = nullptr;
  e->d_ids = nullptr; e->d_rows = nullptr; e->x = e->of = e->beta = e->decay = e->out = e->ws = nullptr;
  e->qkvc = nullptr;
  e->trace_dev = nullptr;
  e->h = e->big = e->mid = e->o = e->y = e->q = nullptr;
  e->cap = 0;
}

// Activation buffers for `l` tokens, grown to 128 or the next power of two as the reference does
// (src/engine.rs:364-393).
int ensure_pool(sd_engine* e, int l) {
  int cap = l <= 128 ? 128 : 1;
  while (cap < l) cap <<= 1;
  if (e->cap >= cap && (!e->trace_host || e->trace_dev)) return SD_OK;
  free_pool(e);
  const sd::Dims& d = e->dm;
  const size_t maxn = std::max({(size_t)2 * d.inter, (size_t)e->in_n, (size_t)e->qkv_n});
  CK(cudaMalloc(&e->d_ids, cap * sizeof(uint32_t)));
  CK(cudaMalloc(&e->d_rows, cap * sizeof(int)));
  CK(cudaMalloc(&e->x, (size_t)cap * d.d * 4));
  CK(cudaMalloc(&e->h, (size_t)cap * d.d * 2));
  CK(cudaMalloc(&e->big, (size_t)cap * maxn * 2));
  CK(cudaMalloc(&e->mid, (size_t)cap * d.inter * 2));
  CK(cudaMalloc(&e->qkvc, (size_t)cap * d.C() * 2));
  CK(cudaMalloc(&e->of, (size_t)cap * d.h * d.dv * 4));
  CK(cudaMalloc(&e->o, (size_t)cap * std::max(d.hq * d.hd, d.h * d.dv) * 2));
  CK(cudaMalloc(&e->y, (size_t)cap * d.d * 2));
  CK(cudaMalloc(&e->q, (size_t)d.hq * cap * d.hd * 2));
  CK(cudaMalloc(&e->beta, (size_t)cap * d.h * 4));
  CK(cudaMalloc(&e->decay, (size_t)cap * d.h * 4));
  CK(cudaMalloc(&e->out, (size_t)cap * d.d * 4));
  // split-K workspace (one f32 slice per split): the planner splits K only when the grid is short,
  // i.e. for small M; 64 MiB covers 32 splits of 64 x 8256 or 16 of 64 x 12288
  e->ws_bytes = (size_t)64 << 20;
  CK(cudaMalloc(&e->ws, e->ws_bytes));
  e->gdn_scratch_bytes = sd::gdn_two_phase_scratch(cap, d.h);
  CK(cudaMalloc(&e->gdn_scratch, e->gdn_scratch_bytes));
  if (e->trace_host) CK(cudaMalloc(&e->trace_dev, (size_t)e->n_layers * cap * d.d * 4));
  e->cap = cap;
  return SD_OK;
}

// Pinned staging: ids for l tokens, rows and output rows for nrows rows (grown as needed).
int ensure_pinned(sd_engine* e, int l, int nrows) {
  if (e->p_cap < l) {
    cudaFreeHost(e->p_ids);
    e->p_ids = nullptr, e->p_cap = 0;
    const int cap = std::max(l, 256);
    CK(cudaMallocHost(&e->p_ids, cap * sizeof(uint32_t)));
    e->p_cap = cap;
  }
  if (e->p_row_cap < nrows) {
    cudaFreeHost(e->p_rows);
    cudaFreeHost(e->p_out);
    e->p_rows = nullptr, e->p_out = nullptr, e->p_row_cap = 0;
    const int cap = std::max(nrows, 64);
    CK(cudaMallocHost(&e->p_rows, cap * sizeof(int)));
    CK(cudaMallocHost(&e->p_out, (size_t)cap * e->dm.d * sizeof(float)));
    e->p_row_cap = cap;
  }
  return SD_OK;
}

// In-place fast Walsh-Hadamard transform, Sylvester order, unnormalised (src/engine.rs:713-727).
void fwht(float* x, int n) {
  for (int h = 1; h < n; h *= 2)
    for (int i = 0; i < n; i += 2 * h)
      for (int j = i; j < i + h; j++) {
        float a = x[j], b = x[j + h];
        x[j] = a + b;
        x[j + h] = a - b;
      }
}

int load_engine(sd_engine* e, const std::string& dir) {
  std::string text;
  if (!read_file(dir + "/manifest.json", text)) return e->fail(SD_ERR_IO, "%s/manifest.json: cannot read", dir.c_str());
  sd::json::Value m;
  try {
    m = sd::json::parse(text);
  } catch (const std::exception& ex) {
    return e->fail(SD_ERR_FORMAT, "manifest.json: %s", ex.what());
  }
  try {
    const auto& c = m.at("config");
    sd::Dims& d = e->dm;
    d.d = (int)c.at("hidden_size").integer();
    d.inter = (int)c.at("intermediate_size").integer();
    d.hq = (int)c.at("num_attention_heads").integer();
    d.hk = (int)c.at("num_key_value_heads").integer();
    d.hd = (int)c.at("head_dim").integer();
    d.h = (int)c.at("linear_num_key_heads").integer();
    d.dk = (int)c.at("linear_key_head_dim").integer();
    d.dv = (int)c.at("linear_value_head_dim").integer();
    d.rd = (int)c.at("rotary_dim").integer();
    e->rope_theta = c.at("rope_theta").number();
    if (const auto* u = c.get("unrotate"); u && u->kind == sd::json::Value::Array)
      for (auto& x : u->arr) e->unrotate.push_back(x.number());
    // The GEMM's K tile (64) and the row-wise norms (one CTA per row, up to 8192 in registers) bound
    // the hidden size; the attention and scan tiles fix the head sizes.
    if (d.d <= 0 || d.d % 64 || d.d > 8192 || d.hd != 256 || d.dk != 128 || d.dv != 128 || d.hq <= 0 || d.hk <= 0 ||
        d.h <= 0 || d.hq % d.hk || d.rd > d.hd || d.rd % 2 || d.inter <= 0 || d.inter % 128)
      return e->fail(SD_ERR_FORMAT,
                     "unsupported dims (hidden size a multiple of 64 up to 8192, intermediate a multiple of 128, "
                     "HD=256, DK=DV=128)");
    if (!e->unrotate.empty() && ((int)e->unrotate.size() != d.d || (d.d & (d.d - 1))))
      return e->fail(SD_ERR_FORMAT, "unrotate needs %d factors and a power-of-two hidden size", d.d);
    const auto& types = c.at("layer_types").arr;
    e->n_layers = (int)types.size();
    e->layers.resize(e->n_layers);
    for (int i = 0; i < e->n_layers; i++) {
      const std::string& k = types[i].str;
      if (k == "linear_attention") e->layers[i].kind = 0, e->layers[i].slot = e->n_lin++;
      else if (k == "full_attention") e->layers[i].kind = 1, e->layers[i].slot = e->n_full++;
      else if (k == "adapter") e->layers[i].kind = 2;
      else return e->fail(SD_ERR_FORMAT, "unsupported layer type %s", k.c_str());
    }
  } catch (const std::exception& ex) {
    return e->fail(SD_ERR_FORMAT, "manifest.json config: %s", ex.what());
  }
  const auto& tensors = m.at("tensors");
  for (auto& kv : tensors.obj)
    if (const auto* hd = kv.second.get("had"); hd && !hd->is_null())
      return e->fail(SD_ERR_FORMAT, "%s: online Hadamard rotation is not supported", kv.first.c_str());

  // shards, uploaded as is in 64 MiB chunks through pinned memory (src/engine.rs:215-229)
  const auto& shards = m.at("shards").arr;
  uint8_t* pinned = nullptr;
  const size_t chunk = 64ull << 20;
  CK(cudaMallocHost(&pinned, chunk));
  std::unique_ptr<uint8_t, void (*)(uint8_t*)> pin_guard(pinned, [](uint8_t* p) { cudaFreeHost(p); });
  // Reads `bytes` bytes of `path` into device memory at `dev` through the pinned chunk; `jmax_at`
  // (optional): per chunk, the largest u16 at row offsets of `row_bytes` + `jmax_off` (the embedding
  // rows' scale-code headers) is folded into *jmax.
  auto upload = [&](const std::string& path, FILE* f, uint8_t* dev, uint64_t bytes, size_t row_bytes, size_t jmax_off,
                    int* jmax) -> int {
    const size_t step = row_bytes ? chunk / row_bytes * row_bytes : chunk;
    for (uint64_t off = 0; off < bytes; off += step) {
      const size_t n = (size_t)std::min<uint64_t>(step, bytes - off);
      if (fread(pinned, 1, n, f) != n)
        return e->fail(SD_ERR_IO, "%s: %llu bytes, expected %llu", path.c_str(), (unsigned long long)off,
                       (unsigned long long)bytes);
      if (jmax)
        for (size_t r = 0; r + row_bytes <= n; r += row_bytes)
          *jmax = std::max(*jmax, (int)(pinned[r + jmax_off + 2] | (pinned[r + jmax_off + 3] << 8)));
      CK(cudaMemcpy(dev + off, pinned, n, cudaMemcpyHostToDevice));
    }
    return SD_OK;
  };
  for (size_t i = 0; i < shards.size(); i++) {
    const uint64_t start = (uint64_t)shards[i].at("start").integer(), bytes = (uint64_t)shards[i].at("bytes").integer();
    std::string path = dir + "/weights." + std::to_string(i) + ".bin";
    const auto* wire = shards[i].get("wire");
    const bool packed = wire && !wire->is_null() && !file_exists(path);
    if (packed) path = dir + "/" + shards[i].at("path").str;
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return e->fail(SD_ERR_IO, "%s: cannot open", path.c_str());
    std::unique_ptr<FILE, int (*)(FILE*)> f_guard(f, fclose);
    uint8_t* dev = nullptr;
    cudaError_t ce = cudaMalloc(&dev, std::max<uint64_t>(bytes, 16));
    if (ce != cudaSuccess) return e->fail(SD_ERR_CUDA, "shard %zu: %s", i, cudaGetErrorString(ce));
    e->shards.push_back(dev);
    e->shard_ranges.push_back({start, bytes});
    if (!packed) {
      int rc = upload(path, f, dev, bytes, 0, 0, nullptr);
      if (rc != SD_OK) return rc;
      continue;
    }
    // a packed shard (`unpack_shard`, src/model.rs:239-258): its tensors back to back, scales as 8-bit
    // codes; uploaded as is, then each tensor goes to its offset, the codes decoded on the device
    const uint64_t wbytes = (uint64_t)wire->integer();
    if (path.size() > 3 && path.compare(path.size() - 3, 3, ".gz") == 0)
      return e->fail(SD_ERR_FORMAT, "%s: a compressed shard (decompress it first)", path.c_str());
    uint8_t* wdev = nullptr;
    CK(cudaMalloc(&wdev, std::max<uint64_t>(wbytes, 16)));
    std::unique_ptr<uint8_t, cudaError_t (*)(void*)> w_guard(wdev, cudaFree);
    int rc = upload(path, f, wdev, wbytes, 0, 0, nullptr);
    if (rc != SD_OK) return rc;
    CK(cudaMemset(dev, 0, bytes));
    for (const auto& kv : tensors.obj) {
      const auto& t = kv.second;
      const auto* tw = t.get("wire");
      if (!tw || tw->is_null()) continue;
      const uint64_t off = t.get("offset") ? (uint64_t)t.at("offset").integer() : 0;
      const uint64_t tb = t.get("bytes") ? (uint64_t)t.at("bytes").integer() : 0;
      if (off < start || off >= start + bytes) continue;
      if (off + tb > start + bytes) return e->fail(SD_ERR_FORMAT, "packed shard: %s out of range", kv.first.c_str());
      const uint64_t w = (uint64_t)tw->integer();
      const bool u8 = t.get("u8") && t.at("u8").boolean();
      uint8_t* dst = dev + (off - start);
      if (u8) {
        const auto& shape = t.at("shape").arr;
        if (shape.size() != 2) return e->fail(SD_ERR_FORMAT, "packed shard: %s: 8-bit scales need a 2-D shape", kv.first.c_str());
        const uint64_t n = (uint64_t)shape[0].integer(), g = (uint64_t)shape[1].integer();
        if (w + 4 * n + n * g > wbytes || 2 * n * g > tb)
          return e->fail(SD_ERR_FORMAT, "packed shard: %s out of range", kv.first.c_str());
        // the rows' largest j bounds the power table (headers: m, j as u16 each)
        std::vector<uint8_t> hdr(4 * n);
        CK(cudaMemcpy(hdr.data(), wdev + w, hdr.size(), cudaMemcpyDeviceToHost));
        int jmax = 0;
        for (uint64_t r = 0; r < n; r++) jmax = std::max(jmax, (int)(hdr[4 * r + 2] | (hdr[4 * r + 3] << 8)));
        CK(sd::decode_scales_dev(wdev + w, 4, wdev + w + 4 * n, g, (long long)n, (int)g, jmax, (uint16_t*)dst, g, e->stream));
      } else {
        if (w + tb > wbytes) return e->fail(SD_ERR_FORMAT, "packed shard: %s out of range", kv.first.c_str());
        CK(cudaMemcpyAsync(dst, wdev + w, tb, cudaMemcpyDeviceToDevice, e->stream));
      }
    }
    CK(cudaStreamSynchronize(e->stream));
  }
  auto tensor_ptr = [&](const std::string& name, const sd::json::Value** meta) -> const uint8_t* {
    const auto* t = tensors.get(name);
    if (!t) return nullptr;
    if (meta) *meta = t;
    const uint64_t off = (uint64_t)t->at("offset").integer();
    for (size_t i = 0; i < e->shards.size(); i++)
      if (off >= e->shard_ranges[i].first && off < e->shard_ranges[i].first + e->shard_ranges[i].second)
        return e->shards[i] + (off - e->shard_ranges[i].first);
    return nullptr;
  };
  std::string missing;
  auto f32 = [&](const std::string& name) -> const float* {
    const float* p = reinterpret_cast<const float*>(tensor_ptr(name, nullptr));
    if (!p && missing.empty()) missing = name;
    return p;
  };
  int rc = SD_OK;
  auto mat = [&](const std::string& name, bool interleave, QWeight* w) {
    const sd::json::Value* t = nullptr;
    const uint8_t* q = tensor_ptr(name + ".q", &t);
    const uint8_t* s = tensor_ptr(name + ".s", nullptr);
    if (!q || !s) {
      if (missing.empty()) missing = name;
      return;
    }
    const int bits = (int)(t->get("bits") ? t->at("bits").integer() : 4);
    const int group = (int)(t->get("group") ? t->at("group").integer() : 32);
    const bool asym = t->get("asym") ? t->at("asym").boolean() : false;
    const int n = (int)t->at("N").integer(), k = (int)t->at("K").integer();
    if (bits < 2 || bits > 4 || group < 32 || group % 32 || k % 64 || (interleave && n % 2)) {
      if (rc == SD_OK)
        rc = e->fail(SD_ERR_FORMAT,
                     "%s: matmul weights must be int2, int3 or int4 with groups of a multiple of 32 and K a multiple of 64",
                     name.c_str());
      return;
    }
    const uint8_t* b = asym ? tensor_ptr(name + ".b", nullptr) : nullptr;  // the per-group f16 biases
    if (asym && !b) {
      if (missing.empty()) missing = name + ".b";
      return;
    }
    cudaError_t ce = sd::repack_weight(q, reinterpret_cast<const __half*>(s), n, k, interleave, w, e->stream, bits, group,
                                       reinterpret_cast<const __half*>(b));
    if (ce != cudaSuccess && rc == SD_OK) rc = e->fail(SD_ERR_CUDA, "%s: %s", name.c_str(), cudaGetErrorString(ce));
  };
  for (int i = 0; i < e->n_layers; i++) {
    LayerW& L = e->layers[i];
    const std::string pre = "layers." + std::to_string(i) + ".";
    L.in_norm = f32(pre + "in_norm");
    if (L.kind == 0) {
      mat(pre + "in_proj", false, &L.in_proj);
      mat(pre + "out_proj", false, &L.out_proj);
      L.conv = f32(pre + "conv");
      L.neg_a = f32(pre + "neg_exp_A");
      L.dt_bias = f32(pre + "dt_bias");
      L.gnorm = f32(pre + "gnorm");
      e->in_n = std::max(e->in_n, L.in_proj.n);
    } else if (L.kind == 1) {
      mat(pre + "qkv", false, &L.qkv);
      mat(pre + "o_proj", false, &L.o_proj);
      L.q_norm = f32(pre + "q_norm");
      L.k_norm = f32(pre + "k_norm");
      e->qkv_n = std::max(e->qkv_n, L.qkv.n);
    } else {
      mat(pre + "proj", false, &L.proj);
      L.bias = f32(pre + "bias");
    }
    if (L.kind != 2) {
      L.post_norm = f32(pre + "post_norm");
      mat(pre + "gate_up", true, &L.gate_up);
      mat(pre + "down", false, &L.down);
    }
    if (rc != SD_OK) return rc;
  }
  e->final_norm = f32("final_norm");
  if (!missing.empty()) return e->fail(SD_ERR_FORMAT, "no tensor %s", missing.c_str());
  const sd::Dims& d = e->dm;
  for (auto& L : e->layers) {
    if (L.kind == 0 && L.in_proj.n < d.C() + d.h * d.dv + 2 * d.h)
      return e->fail(SD_ERR_FORMAT, "in_proj has %d rows, fewer than q,k,v,z,a,b need", L.in_proj.n);
    if (L.kind == 1 && L.qkv.n < d.hq * d.hd * 2 + 2 * d.hk * d.hd)
      return e->fail(SD_ERR_FORMAT, "qkv has %d rows, fewer than q,gate,k,v need", L.qkv.n);
  }

  // embedding parts (src/model.rs:260-283)
  const auto* emb = m.get("embed");
  if (!emb || emb->is_null()) return e->fail(SD_ERR_FORMAT, "manifest has no embed");
  {
    const sd::json::Value* et = tensors.get("embed.q");
    e->embed_bits = et && et->get("bits") ? (int)et->at("bits").integer() : 4;
    const int egroup = et && et->get("group") ? (int)et->at("group").integer() : 32;
    const bool easym = et && et->get("asym") ? et->at("asym").boolean() : false;
    if (easym || egroup != 32 || e->embed_bits < 2 || e->embed_bits > 4)
      return e->fail(SD_ERR_FORMAT, "embedding format not supported (symmetric int2/3/4, group 32)");
    e->vocab = (int)emb->at("vocab").integer();
    const auto& parts = emb->at("parts").arr;
    if (parts.size() != 2 || parts[0].arr[0].str != "embed.q" || parts[1].arr[0].str != "embed.s")
      return e->fail(SD_ERR_FORMAT, "embed parts must be [embed.q, embed.s]");
    const size_t qb = (size_t)parts[0].arr[1].integer(), sb = (size_t)parts[1].arr[1].integer();
    const bool u8 = emb->get("u8") ? emb->at("u8").boolean() : false;
    const auto* wrb = emb->get("wire_row_bytes");
    const size_t rb = (wrb && !wrb->is_null()) ? (size_t)wrb->integer() : (size_t)emb->at("row_bytes").integer();
    if (qb != (size_t)d.d / 32 * 4 * e->embed_bits || sb != (size_t)d.d / 32 * 2)
      return e->fail(SD_ERR_FORMAT, "embed part sizes do not match the hidden size");
    if (rb < qb + (u8 ? 4 + sb / 2 : sb)) return e->fail(SD_ERR_FORMAT, "embedding rows of %zu bytes are shorter than their parts", rb);
    std::string path = dir + "/" + emb->at("rows").str;
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return e->fail(SD_ERR_IO, "%s: cannot open", path.c_str());
    std::unique_ptr<FILE, int (*)(FILE*)> f_guard(f, fclose);
    struct stat stbuf;
    if (fstat(fileno(f), &stbuf) != 0 || (size_t)stbuf.st_size != (size_t)e->vocab * rb)
      return e->fail(SD_ERR_IO, "%s: %lld bytes, expected %d rows of %zu", path.c_str(), (long long)stbuf.st_size, e->vocab, rb);
    // the rows file goes up as is; the parts are split out (and 8-bit scale codes decoded,
    // `decode_scales`, src/model.rs:219-236) on the device
    uint8_t* raw = nullptr;
    CK(cudaMalloc(&raw, (size_t)e->vocab * rb));
    std::unique_ptr<uint8_t, cudaError_t (*)(void*)> raw_guard(raw, cudaFree);
    int jmax = 0;
    int rc = upload(path, f, raw, (uint64_t)e->vocab * rb, rb, qb, u8 ? &jmax : nullptr);
    if (rc != SD_OK) return rc;
    CK(cudaMalloc(&e->embed_q, (size_t)e->vocab * qb));
    CK(cudaMalloc(&e->embed_s, (size_t)e->vocab * sb));
    CK(sd::split_rows_dev(raw, rb, 0, qb, e->vocab, e->embed_q, e->stream));
    if (u8)
      CK(sd::decode_scales_dev(raw + qb, rb, raw + qb + 4, rb, e->vocab, (int)sb / 2, jmax,
                               reinterpret_cast<uint16_t*>(e->embed_s), sb / 2, e->stream));
    else
      CK(sd::split_rows_dev(raw, rb, qb, sb, e->vocab, reinterpret_cast<uint8_t*>(e->embed_s), e->stream));
    CK(cudaStreamSynchronize(e->stream));
  }

  // recurrent state, conv history, K/V caches (src/engine.rs:251-257), RoPE table (:259-269)
  for (int i = 0; i < e->n_lin; i++) {
    float* s = nullptr;
    __half* h = nullptr;
    CK(cudaMalloc(&s, (size_t)d.h * d.dk * d.dv * 4));
    CK(cudaMalloc(&h, (size_t)3 * d.C() * 2));
    CK(cudaMemset(s, 0, (size_t)d.h * d.dk * d.dv * 4));
    CK(cudaMemset(h, 0, (size_t)3 * d.C() * 2));
    e->state.push_back(s);
    e->hist.push_back(h);
  }
  for (int i = 0; i < e->n_full; i++) {
    __half *k = nullptr, *v = nullptr;
    CK(cudaMalloc(&k, (size_t)d.hk * SD_CONTEXT * d.hd * 2));
    CK(cudaMalloc(&v, (size_t)d.hk * SD_CONTEXT * d.hd * 2));
    CK(cudaMemset(k, 0, (size_t)d.hk * SD_CONTEXT * d.hd * 2));
    CK(cudaMemset(v, 0, (size_t)d.hk * SD_CONTEXT * d.hd * 2));
    e->kc.push_back(k);
    e->vc.push_back(v);
  }
  std::vector<float> table((size_t)SD_CONTEXT * d.rd);
  for (int t = 0; t < SD_CONTEXT; t++)
    for (int i = 0; i < d.rd / 2; i++) {
      const double a = (double)t / std::pow(e->rope_theta, (double)(2 * i) / (double)d.rd);
      table[(size_t)t * d.rd + 2 * i] = (float)std::cos(a);
      table[(size_t)t * d.rd + 2 * i + 1] = (float)std::sin(a);
    }
  CK(cudaMalloc(&e->rope, table.size() * 4));
  CK(cudaMemcpy(e->rope, table.data(), table.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMalloc(&e->d_err, sizeof(int)));
  CK(cudaMemset(e->d_err, 0, sizeof(int)));
  CK(cudaStreamSynchronize(e->stream));
  return SD_OK;
}

// Waits for the stream, folds profiled event pairs into the totals, and turns a launch failure or a
// kernel error word into the call's error.
int sync_engine(sd_engine* e) {
  cudaError_t ce = cudaStreamSynchronize(e->stream);
  if (ce != cudaSuccess) return e->fail(SD_ERR_CUDA, "forward: %s", cudaGetErrorString(ce));
  for (size_t i = 0; i < e->prof_pending.size(); i++) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->prof_events[2 * i], e->prof_events[2 * i + 1]);
    const int kind = e->prof_pending[i].first;
    e->prof_ms[kind] += ms;
    e->prof_units[kind] += e->prof_pending[i].second;
    e->prof_count[kind] += 1;
  }
  e->prof_pending.clear();
  e->prof_used = 0;
  int herr = 0;
  CK(cudaMemcpy(&herr, e->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (herr != 0) {
    cudaMemset(e->d_err, 0, sizeof(int));
    return e->fail(SD_ERR_KERNEL, "a kernel reported error %d (%s)", herr,
                   herr == sd::kErrBadShape ? "token id or row out of range" : "a bounded wait ran out");
  }
  return SD_OK;
}

cudaEvent_t prof_event(sd_engine* e) {
  if (e->prof_used >= e->prof_events.size()) {
    cudaEvent_t ev;
    cudaEventCreate(&ev);
    e->prof_events.push_back(ev);
  }
  return e->prof_events[e->prof_used++];
}

// Runs `launch` (which returns a cudaError_t and adds its kernel count to *n), bracketed by
// profiling events when profiling is on.
template <class F>
cudaError_t launch(sd_engine* e, int kind, double units, F&& fn) {
  cudaEvent_t a = nullptr;
  if (e->prof_on) {
    a = prof_event(e);
    cudaEventRecord(a, e->stream);
  }
  int n = 1;
  cudaError_t ce = fn(&n);
  e->launches += n;
  if (e->prof_on) {
    cudaEvent_t b = prof_event(e);
    cudaEventRecord(b, e->stream);
    e->prof_pending.push_back({kind, units});
  }
  return ce;
}

#define LK(kind, units, call)                                                                            \
  do {                                                                                                   \
    cudaError_t _e = launch(e, kind, units, [&](int* nl) -> cudaError_t { (void)nl; return (call); });   \
    if (_e != cudaSuccess) return e->fail(SD_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(_e));      \
  } while (0)

// A packed pass (sd_forward_batch and the batched forks built on it): several sequences back to back,
// sequence b continuing snapshot b (the same one for every question of one request, one per request
// when several requests run together, or none: a fresh sequence), whose states, conv histories and
// prefix K/V are read in place and never written; with `keep`, each sequence's new state, history
// and K/V go to a new snapshot of its own. In a tree pass a sequence may instead continue an earlier
// sequence of the same pass (a request's questions after its state): the parent's new snapshot is
// written layer by layer before the children read it. Device arrays: per-layer tables of each sequence's
// snapshot buffers (null entries: no source snapshot); tpos (position of each packed token), tstart
// (first token of each token's sequence), tseq (its sequence); seq_off / seq_len / plen (prefix
// length) per sequence; blk (sequence, first query) per 64-query attention block; for the two-phase
// scan of long sequences, chunk_tab (first token, tokens) per 64-token chunk, chunk0 (first chunk)
// per sequence and order (sequences, longest first).
struct Fork {
  const uint32_t* ids;  // [l] token ids
  const int* rows;      // output rows (indices into the packed tokens)
  const float* const* states;   // [n_lin][nseq] GDN states
  const __half* const* hists;   // [n_lin][nseq] conv histories
  const __half* const* kp;      // [n_full][nseq] prefix keys ([hk][plen][hd])
  const __half* const* vp;      // [n_full][nseq] prefix values
  // keep: the new snapshots' buffers, [n_lin][nseq] / [n_full][nseq] (null: nothing kept)
  float* const* s_out = nullptr;
  __half* const* h_out = nullptr;
  __half* const* k_out = nullptr;
  __half* const* v_out = nullptr;
  const int *tpos, *tstart, *tseq, *seq_off, *seq_len, *plen, *blk;
  const int *chunk_tab = nullptr, *chunk0 = nullptr, *order = nullptr;
  const int* blk128 = nullptr;  // (sequence, first query) per 128-query block, most keys first (the tcgen05 kernel)
  const int* gofs = nullptr;    // first row of each sequence in the gathered keys (prefix + own rows)
  int ktot = 0;                 // rows per head of the gathered keys
  int nseq, nblk, max_len, max_p, max_rows, chunks = 0, nblk128 = 0;
  bool two_phase = false;
  // a tree pass: sequences nroot .. of gorder continue sequences of the same pass (their parents, in
  // gorder's first nroot entries), reading the parents' new snapshot buffers of each layer
  bool tree = false;
  const int* gorder = nullptr;  // [nseq]: the roots, then the children, each longest first
  int nroot = 0;
  double pairs;       // causal (query, key) pairs of every sequence: len p + len (len + 1) / 2
  __half *kt, *vt;    // [hk][l][hd] K and V of the packed tokens
};

// Whether a gated-delta layer over `walks` (sequence, head) walks, the longest of max_chunks 64-token
// chunks and chunks x heads chunk records in all, takes the fused tcgen05 scan rather than the
// two-phase one. Estimates from B200 timings: the fused scan walks about 6 us per chunk (config 3,
// B = 16, L = 1024: 204 us for two waves of 16 chunks), one CTA per walk and SM, so a wave lasts its
// longest walk; the two-phase scan's preparation does about two
// chunk records per SM each 21 us, then its walk takes about 4 us per chunk of the longest sequence.
static bool gdn_pick_tc(const sd_engine* e, long long walks, long long max_chunks, long long records, bool two_phase_ok) {
  if (e->gdn_mode) return e->gdn_mode == 1;
  if (!two_phase_ok) return true;
  const long long sms = std::max(1, e->num_sms);
  const double fused = (double)((walks + sms - 1) / sms) * max_chunks * 6.0;
  const double two_phase = (double)((records + 2 * sms - 1) / (2 * sms)) * 21.0 + max_chunks * 4.0;
  return fused <= two_phase;
}

// The layer loop (src/engine.rs:446-522), launched on the engine's stream. With `fk`, the l tokens are
// a batched fork's packed sequences (each at position p + its index within its sequence).
int run_layers(sd_engine* e, int l, int p, bool has_cache, int nrows, const Fork* fk = nullptr) {
  const sd::Dims& d = e->dm;
  cudaStream_t st = e->stream;
  const int C = d.C();
  const double L = l;
  auto mm = [&](const QWeight& w, const __half* a, int lda, __half* y, int ldy, bool silu) -> int {
    const double flops = 2.0 * L * w.n * w.k;
    LK(SD_PROF_GEMM, flops, sd::gemm_q4(w, a, l, lda, y, ldy, silu, e->ws, e->ws_bytes, e->d_err, e->num_sms, st, nl));
    return SD_OK;
  };
  // x += f16(a W^T): the layer's output matmuls add into the residual stream in their epilogue
  auto mm_add = [&](const QWeight& w, const __half* a, int lda) -> int {
    const double flops = 2.0 * L * w.n * w.k;
    LK(SD_PROF_GEMM, flops,
       sd::gemm_q4(w, a, l, lda, nullptr, d.d, false, e->ws, e->ws_bytes, e->d_err, e->num_sms, st, nl, e->x));
    return SD_OK;
  };
  int rc;
#define MM(...)                          \
  do {                                   \
    if ((rc = mm(__VA_ARGS__)) != SD_OK) \
      return rc;                         \
  } while (0)
#define MM_ADD(...)                          \
  do {                                       \
    if ((rc = mm_add(__VA_ARGS__)) != SD_OK) \
      return rc;                             \
  } while (0)
  // whether y holds a layer output not yet added into x (an adapter's projection: its bias is added
  // to the f16 output first, as the reference does)
  bool pending = false;
  const double row_bytes = (double)d.d * (4 + 2);
  LK(SD_PROF_OTHER, L * (d.d / 32 * (4.0 * e->embed_bits + 2) + row_bytes),
     sd::launch_embed_norm(fk ? fk->ids : e->d_ids, l, e->embed_q, e->embed_s, e->embed_bits, d.d, e->vocab, e->layers[0].in_norm, e->x,
                           e->h, e->d_err, st));
  for (int i = 0; i < e->n_layers; i++) {
    const LayerW& Lw = e->layers[i];
    if (i > 0)
      LK(SD_PROF_OTHER, L * d.d * (pending ? 12.0 : 6.0), sd::launch_add_norm(e->x, e->y, Lw.in_norm, l, d.d, pending, e->h, st));
    pending = false;
    if (Lw.kind == 2) {
      MM(Lw.proj, e->h, d.d, e->y, d.d, false);
      LK(SD_PROF_OTHER, L * d.d * 4.0, sd::launch_add_bias(e->y, Lw.bias, l, d.d, st));
      pending = true;
    } else {
      if (Lw.kind == 0) {
        const int N = Lw.in_proj.n;
        __half* hist = fk ? nullptr : e->hist[Lw.slot];
        MM(Lw.in_proj, e->h, d.d, e->big, N, false);
        // the new snapshots' conv histories; in a tree pass before the conv, whose children read
        // their parents' (only parents have new snapshots there)
        auto pack_hist = [&]() -> int {
          LK(SD_PROF_OTHER, fk->nseq * C * 12.0,
             sd::launch_hist_pack(e->big, N, C, fk->seq_off, fk->seq_len, fk->hists + (size_t)Lw.slot * fk->nseq,
                                  fk->h_out + (size_t)Lw.slot * fk->nseq, fk->nseq, st));
          return SD_OK;
        };
        if (fk && fk->tree && (rc = pack_hist()) != SD_OK) return rc;
        LK(SD_PROF_OTHER, L * C * 4.0,
           sd::launch_conv(e->big, N, Lw.conv, hist, l, C, e->qkvc, fk ? fk->tstart : nullptr,
                           fk ? fk->hists + (size_t)Lw.slot * fk->nseq : nullptr, fk ? fk->tseq : nullptr, st));
        if (!fk) LK(SD_PROF_OTHER, C * 12.0, sd::launch_hist_update(e->big, N, hist, l, C, st));
        else if (fk->h_out && !fk->tree && (rc = pack_hist()) != SD_OK) return rc;
        const int aoff = C + d.h * d.dv, boff = aoff + d.h;
        LK(SD_PROF_OTHER, L * d.h * 12.0,
           sd::launch_gdn_gates(e->big, N, aoff, boff, Lw.neg_a, Lw.dt_bias, l, d.h, e->beta, e->decay, st));
        const double gdn_bytes = L * (C * 2.0 + d.h * 8.0 + d.h * d.dv * 4.0) + 2.0 * d.h * d.dk * d.dv * 4.0;
        // one chunk: the single-pass scan; longer: the two-phase scan (chunks in parallel, then the state walk);
        // packed sequences, each from its snapshot's state (or zeros): short ones with the single-pass
        // scan, long ones with the two-phase scan
        const long long max_chunks = fk ? (fk->max_len + 63) / 64 : (l + 63) / 64;
        const bool use_tc = fk ? fk->tree || gdn_pick_tc(e, (long long)fk->nseq * d.h, max_chunks, (long long)fk->chunks * d.h,
                                                         fk->two_phase)
                               : gdn_pick_tc(e, d.h, max_chunks, max_chunks * d.h, l > 64);
        if (fk && fk->tree) {  // the fused scan over the roots, then over the children from the roots' new states
          sd::GdnTcArgs ga;
          ga.beta = e->beta, ga.g = e->decay, ga.o = e->of, ga.h = d.h, ga.err = e->d_err;
          ga.seq_off = fk->seq_off, ga.seq_len = fk->seq_len;
          ga.s_in = fk->states + (size_t)Lw.slot * fk->nseq;
          ga.s_out = fk->s_out + (size_t)Lw.slot * fk->nseq;
          ga.order = fk->gorder;
          LK(SD_PROF_GDN, gdn_bytes,
             sd::launch_gdn_tc(e->qkvc, e->qkvc + d.h * d.dk, C, e->qkvc + 2 * d.h * d.dk, C, (long long)l * C,
                               (long long)l * C, l, ga, fk->nroot * d.h, st));
          ga.order = fk->gorder + fk->nroot;
          LK(SD_PROF_GDN, 0.0,
             sd::launch_gdn_tc(e->qkvc, e->qkvc + d.h * d.dk, C, e->qkvc + 2 * d.h * d.dk, C, (long long)l * C,
                               (long long)l * C, l, ga, (fk->nseq - fk->nroot) * d.h, st));
        } else if (use_tc) {  // the fused tcgen05 scan: one CTA per (sequence, head)
          sd::GdnTcArgs ga;
          ga.beta = e->beta, ga.g = e->decay, ga.o = e->of, ga.h = d.h, ga.err = e->d_err;
          int walks = d.h;
          if (fk) {
            ga.seq_off = fk->seq_off, ga.seq_len = fk->seq_len, ga.order = fk->order;
            ga.s_in = fk->states + (size_t)Lw.slot * fk->nseq;
            ga.s_out = fk->s_out ? fk->s_out + (size_t)Lw.slot * fk->nseq : nullptr;
            walks = fk->nseq * d.h;
          } else {
            ga.l = l, ga.state = e->state[Lw.slot], ga.load_state = has_cache, ga.store_state = 1;
          }
          LK(SD_PROF_GDN, gdn_bytes,
             sd::launch_gdn_tc(e->qkvc, e->qkvc + d.h * d.dk, C, e->qkvc + 2 * d.h * d.dk, C, (long long)l * C,
                               (long long)l * C, l, ga, walks, st));
        } else if (fk && fk->two_phase)
          LK(SD_PROF_GDN, gdn_bytes,
             (*nl = 2, sd::launch_gdn_two_phase_packed(
                           e->qkvc, e->qkvc + d.h * d.dk, C, e->qkvc + 2 * d.h * d.dk, C, e->beta, e->decay,
                           fk->states + (size_t)Lw.slot * fk->nseq, fk->s_out ? fk->s_out + (size_t)Lw.slot * fk->nseq : nullptr,
                           e->of, fk->seq_off, fk->seq_len, fk->chunk0, fk->order, fk->chunk_tab, fk->nseq, fk->chunks, d.h,
                           e->gdn_scratch, e->gdn_scratch_bytes, e->num_sms, st)));
        else if (fk)
          LK(SD_PROF_GDN, gdn_bytes,
             sd::launch_gdn_chunked_packed(e->qkvc, e->qkvc + d.h * d.dk, C, e->qkvc + 2 * d.h * d.dk, C, e->beta,
                                           e->decay, fk->states + (size_t)Lw.slot * fk->nseq,
                                           fk->s_out ? fk->s_out + (size_t)Lw.slot * fk->nseq : nullptr, e->of, fk->seq_off,
                                           fk->seq_len, fk->nseq, d.h, st));
        else if (l <= 64)
          LK(SD_PROF_GDN, gdn_bytes,
             sd::launch_gdn_chunked(e->qkvc, e->qkvc + d.h * d.dk, C, e->qkvc + 2 * d.h * d.dk, C, 0, 0, true, e->beta,
                                    e->decay, e->state[Lw.slot], has_cache, e->of, l, d.h, 1, st));
        else
          LK(SD_PROF_GDN, gdn_bytes,
             (*nl = 2, sd::launch_gdn_two_phase(e->qkvc, e->qkvc + d.h * d.dk, C, e->qkvc + 2 * d.h * d.dk, C, e->beta,
                                                e->decay, e->state[Lw.slot], has_cache, e->of, l, d.h, e->gdn_scratch,
                                                e->gdn_scratch_bytes, st)));
        LK(SD_PROF_OTHER, L * d.h * d.dv * 8.0, sd::launch_gnorm(e->of, e->big, N, C, Lw.gnorm, l, d.h, e->o, st));
        MM_ADD(Lw.out_proj, e->o, d.h * d.dv);
      } else {
        const int N = Lw.qkv.n;
        MM(Lw.qkv, e->h, d.d, e->big, N, false);
        if (fk) {
          LK(SD_PROF_OTHER, L * (N * 2.0 + (d.hq + 2.0 * d.hk) * d.hd * 2.0),
             sd::launch_qk_prep(e->big, N, Lw.q_norm, Lw.k_norm, e->rope, l, p, l, d, fk->tpos, e->q, fk->kt, fk->vt, st));
          sd::AttnPacked pk;
          pk.blk = fk->blk, pk.seq_off = fk->seq_off, pk.seq_len = fk->seq_len, pk.kt = fk->kt, pk.vt = fk->vt, pk.T = l;
          pk.kp = fk->kp + (size_t)Lw.slot * fk->nseq, pk.vp = fk->vp + (size_t)Lw.slot * fk->nseq, pk.plen = fk->plen;
          // the sequences' keys and values (prefix and own) into their new snapshots; in a tree pass
          // first, since the children's prefixes are their parents' new snapshots
          auto pack_kv = [&]() -> int {
            LK(SD_PROF_OTHER, 8.0 * d.hk * d.hd * (L + fk->max_p),
               sd::launch_kv_pack(fk->kt, fk->vt, l, d.hk, d.hd, fk->seq_off, fk->seq_len, fk->plen,
                                  fk->kp + (size_t)Lw.slot * fk->nseq, fk->vp + (size_t)Lw.slot * fk->nseq,
                                  fk->k_out + (size_t)Lw.slot * fk->nseq, fk->v_out + (size_t)Lw.slot * fk->nseq, fk->nseq,
                                  fk->max_rows, st));
            return SD_OK;
          };
          if (fk->tree && (rc = pack_kv()) != SD_OK) return rc;
          if (fk->max_p == 0 && fk->max_len >= 128 && d.hd == 256) {
            // fresh sequences (prefills): the tcgen05 kernel over 128-query blocks
            sd::AttnTcArgs ta;
            ta.blk = fk->blk128, ta.seq_off = fk->seq_off, ta.seq_len = fk->seq_len, ta.hq = d.hq, ta.hk = d.hk;
            ta.gate = e->big, ta.gstride = N, ta.goff = d.hd, ta.gstep = 2 * d.hd, ta.out = e->o, ta.err = e->d_err;
            LK(SD_PROF_ATTN, 4.0 * d.hd * d.hq * fk->pairs,
               sd::launch_attention_tc(e->q, l, fk->kt, fk->vt, l, l, ta, fk->nblk128, st));
          } else if (fk->max_p > 0 && d.hd == 256 && fk->ktot > 0) {
            // continuations (questions over snapshots): each sequence's prefix and own keys gathered into
            // one tensor, then the tcgen05 kernel with per-sequence key rows and prefix lengths
            __half* gk = e->fk_gather;
            __half* gv = gk + (size_t)d.hk * fk->ktot * d.hd;
            LK(SD_PROF_OTHER, 8.0 * d.hk * d.hd * (double)fk->ktot,
               sd::launch_kv_gather(fk->kt, fk->vt, l, d.hk, d.hd, fk->seq_off, fk->seq_len, fk->plen,
                                    fk->kp + (size_t)Lw.slot * fk->nseq, fk->vp + (size_t)Lw.slot * fk->nseq, fk->gofs,
                                    fk->ktot, gk, gv, fk->nseq, fk->max_rows, st));
            sd::AttnTcArgs ta;
            ta.blk = fk->blk128, ta.seq_off = fk->seq_off, ta.seq_len = fk->seq_len, ta.hq = d.hq, ta.hk = d.hk;
            ta.kbase_tab = fk->gofs, ta.plen = fk->plen;
            ta.gate = e->big, ta.gstride = N, ta.goff = d.hd, ta.gstep = 2 * d.hd, ta.out = e->o, ta.err = e->d_err;
            LK(SD_PROF_ATTN, 4.0 * d.hd * d.hq * fk->pairs,
               sd::launch_attention_tc(e->q, l, gk, gv, fk->ktot, fk->ktot, ta, fk->nblk128, st));
          } else {
            int splits = sd::attention_splits_packed(fk->nblk, fk->max_p, fk->max_len, d.hq, e->num_sms);
            while (splits > 1 && sd::attention_split_bytes(l, d.hq, splits) > e->ws_bytes) splits--;
            LK(SD_PROF_ATTN, 4.0 * d.hd * d.hq * fk->pairs,
               (*nl = splits > 1 ? 2 : 1,
                sd::launch_attention_packed(e->q, nullptr, nullptr, e->big, N, d.hd, 2 * d.hd, e->o, l, fk->max_p, fk->max_p,
                                            d.hq, d.hk, d.hd, pk, fk->nblk, splits, e->ws, e->ws_bytes, st)));
          }
          if (fk->k_out && !fk->tree && (rc = pack_kv()) != SD_OK) return rc;
          MM_ADD(Lw.o_proj, e->o, d.hq * d.hd);
        } else {
        LK(SD_PROF_OTHER, L * (N * 2.0 + (d.hq + 2.0 * d.hk) * d.hd * 2.0),
           sd::launch_qk_prep(e->big, N, Lw.q_norm, Lw.k_norm, e->rope, l, p, SD_CONTEXT, d, nullptr, e->q, e->kc[Lw.slot],
                              e->vc[Lw.slot], st));
        const double pairs = L * p + L * (L + 1) / 2;  // causal (query, key) pairs
        if (l >= 128 && d.hd == 256) {  // query blocks of 128: the tcgen05 kernel
          sd::AttnTcArgs ta;
          ta.l = l, ta.p = p, ta.hq = d.hq, ta.hk = d.hk;
          ta.gate = e->big, ta.gstride = N, ta.goff = d.hd, ta.gstep = 2 * d.hd, ta.out = e->o, ta.err = e->d_err;
          LK(SD_PROF_ATTN, 4.0 * d.hd * d.hq * pairs,
             sd::launch_attention_tc(e->q, l, e->kc[Lw.slot], e->vc[Lw.slot], SD_CONTEXT, p + l, ta, (l + 127) / 128, st));
        } else {
          int splits = sd::attention_splits(l, p, d.hq, e->num_sms);  // keys split for short continuations
          while (splits > 1 && sd::attention_split_bytes(l, d.hq, splits) > e->ws_bytes) splits--;
          LK(SD_PROF_ATTN, 4.0 * d.hd * d.hq * pairs,
             (*nl = splits > 1 ? 2 : 1,  // with split keys, a second kernel merges the splits
              sd::launch_attention(e->q, e->kc[Lw.slot], e->vc[Lw.slot], e->big, N, d.hd, 2 * d.hd, e->o, l, p, SD_CONTEXT,
                                   d.hq, d.hk, d.hd, splits, e->ws, e->ws_bytes, st)));
        }
        MM_ADD(Lw.o_proj, e->o, d.hq * d.hd);
        }
      }
    }
    if (Lw.kind != 2) {
      LK(SD_PROF_OTHER, L * d.d * 6.0, sd::launch_add_norm(e->x, nullptr, Lw.post_norm, l, d.d, false, e->h, st));
      MM(Lw.gate_up, e->h, d.d, e->mid, d.inter, true);
      MM_ADD(Lw.down, e->mid, d.inter);
    }
    if (e->trace_dev)
      LK(SD_PROF_OTHER, L * d.d * 10.0,
         sd::launch_trace(e->x, pending ? e->y : nullptr, l * d.d, e->trace_dev + (size_t)i * l * d.d, st));
  }
  if (nrows > 0)
    LK(SD_PROF_OTHER, nrows * d.d * 14.0,
       sd::launch_final_norm(e->x, pending ? e->y : nullptr, e->final_norm, fk ? fk->rows : e->d_rows, nrows, l, d.d, e->out,
                             e->d_err, st));
#undef MM
#undef MM_ADD
  return SD_OK;
}

// A new snapshot of T tokens (uninitialised), one stream-ordered allocation from the engine's pool.
int alloc_snapshot(sd_engine* e, int T, std::unique_ptr<sd_snapshot>* out) {
  const sd::Dims& d = e->dm;
  const size_t state_bytes = (size_t)d.h * d.dk * d.dv * 4, hist_bytes = (size_t)3 * d.C() * 2;
  const size_t kv_bytes = (size_t)d.hk * T * d.hd * 2;
  const size_t total = e->n_lin * (state_bytes + hist_bytes) + 2 * e->n_full * kv_bytes;
  std::unique_ptr<sd_snapshot> snap(new sd_snapshot());
  snap->device = e->device;
  snap->len = T;
  CK(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&snap->base), std::max<size_t>(total, 256), e->snap_pool, e->stream));
  snap->owner = e;
  uint8_t* q = snap->base;
  for (int i = 0; i < e->n_lin; i++, q += state_bytes) snap->state.push_back(reinterpret_cast<float*>(q));
  for (int i = 0; i < e->n_lin; i++, q += hist_bytes) snap->hist.push_back(reinterpret_cast<__half*>(q));
  for (int i = 0; i < e->n_full; i++, q += kv_bytes) snap->k.push_back(reinterpret_cast<__half*>(q));
  for (int i = 0; i < e->n_full; i++, q += kv_bytes) snap->v.push_back(reinterpret_cast<__half*>(q));
  *out = std::move(snap);
  return SD_OK;
}

// Restores the prefix or clears the conv history (src/engine.rs:552-571), runs the layers and, with
// `keep`, copies the state into a new snapshot (src/engine.rs:592-614). Everything is enqueued on the
// engine's stream; e->d_ids and e->d_rows hold this call's inputs.
int forward_core(sd_engine* e, int l, const sd_snapshot* cache, int nrows, bool keep, sd_snapshot** snapshot_out) {
  const sd::Dims& d = e->dm;
  cudaStream_t st = e->stream;
  const int p = cache ? cache->len : 0;
  const size_t state_bytes = (size_t)d.h * d.dk * d.dv * 4, hist_bytes = (size_t)3 * d.C() * 2;
  const size_t row_bytes = (size_t)d.hd * 2;
  if (cache) {
    for (int i = 0; i < e->n_lin; i++) {
      CK(cudaMemcpyAsync(e->state[i], cache->state[i], state_bytes, cudaMemcpyDeviceToDevice, st));
      CK(cudaMemcpyAsync(e->hist[i], cache->hist[i], hist_bytes, cudaMemcpyDeviceToDevice, st));
    }
    for (int i = 0; i < e->n_full && p > 0; i++) {
      CK(cudaMemcpy2DAsync(e->kc[i], SD_CONTEXT * row_bytes, cache->k[i], (size_t)p * row_bytes, (size_t)p * row_bytes, d.hk,
                           cudaMemcpyDeviceToDevice, st));
      CK(cudaMemcpy2DAsync(e->vc[i], SD_CONTEXT * row_bytes, cache->v[i], (size_t)p * row_bytes, (size_t)p * row_bytes, d.hk,
                           cudaMemcpyDeviceToDevice, st));
    }
  } else {
    for (int i = 0; i < e->n_lin; i++) CK(cudaMemsetAsync(e->hist[i], 0, hist_bytes, st));
  }
  int rc = run_layers(e, l, p, cache != nullptr, nrows);
  if (rc != SD_OK) return rc;
  if (keep) {
    const int T = p + l;
    std::unique_ptr<sd_snapshot> snap;
    if ((rc = alloc_snapshot(e, T, &snap)) != SD_OK) return rc;
    for (int i = 0; i < e->n_lin; i++) {
      CK(cudaMemcpyAsync(snap->state[i], e->state[i], state_bytes, cudaMemcpyDeviceToDevice, st));
      CK(cudaMemcpyAsync(snap->hist[i], e->hist[i], hist_bytes, cudaMemcpyDeviceToDevice, st));
    }
    for (int i = 0; i < e->n_full; i++) {
      CK(cudaMemcpy2DAsync(snap->k[i], (size_t)T * row_bytes, e->kc[i], SD_CONTEXT * row_bytes, (size_t)T * row_bytes, d.hk,
                           cudaMemcpyDeviceToDevice, st));
      CK(cudaMemcpy2DAsync(snap->v[i], (size_t)T * row_bytes, e->vc[i], SD_CONTEXT * row_bytes, (size_t)T * row_bytes, d.hk,
                           cudaMemcpyDeviceToDevice, st));
    }
    e->live.push_back(snap.get());
    *snapshot_out = snap.release();
  }
  return SD_OK;
}

int check_forward_args(sd_engine* e, int l, int nrows, const sd_snapshot* cache, int keep, sd_snapshot** snapshot_out) {
  const int p = cache ? cache->len : 0;
  if (l <= 0 || p + l > SD_CONTEXT) return e->fail(SD_ERR_INVALID, "context of %d tokens: must be 1 to %d", p + l, SD_CONTEXT);
  if (nrows < 0) return e->fail(SD_ERR_INVALID, "negative row count");
  if (cache && cache->owner != e) return e->fail(SD_ERR_INVALID, "snapshot belongs to another engine");
  if (keep && !snapshot_out) return e->fail(SD_ERR_INVALID, "keep without a snapshot output");
  if (e->trace_host && e->trace_floats < (size_t)e->n_layers * l * e->dm.d)
    return e->fail(SD_ERR_INVALID, "trace buffer too small");
  return SD_OK;
}

// Staged ints of a packed pass (pointer tables as two ints a pointer, index arrays, rows, the two-phase
// scan's tables when chunks >= 0, host ids).
size_t packed_ints(const sd_engine* e, long long T, long long nq, long long nblk, long long R, bool keep, long long chunks,
                   bool host_ids) {
  const size_t per_set = (size_t)(2 * e->n_lin + 2 * e->n_full) * nq;
  return 2 * per_set * (keep ? 2 : 1) + 3 * (size_t)T + 4 * (size_t)nq + 2 * (size_t)nblk + (size_t)R +
         (chunks >= 0 ? 2 * (size_t)chunks + 2 * (size_t)nq : 0) + (host_ids ? (size_t)T : 0);
}

// Grows the packed pass's device buffers (staged index arrays, the packed tokens' K/V, the two-phase
// scan's records) to hold a pass of T tokens, `ints` staged ints and `chunks` records per head, by at
// least a quarter at a time. A resize first waits for the queued work that may use the old buffers.
int ensure_packed(sd_engine* e, long long T, size_t ints, long long chunks) {
  const sd::Dims& d = e->dm;
  cudaStream_t st = e->stream;
  if (chunks > 0 && e->gdn_scratch_bytes < sd::gdn_two_phase_packed_scratch((int)chunks, d.h)) {
    CK(cudaStreamSynchronize(st));
    cudaFree(e->gdn_scratch);
    const size_t bytes = std::max(sd::gdn_two_phase_packed_scratch((int)chunks, d.h), e->gdn_scratch_bytes * 5 / 4);
    e->gdn_scratch = nullptr, e->gdn_scratch_bytes = 0;
    CK(cudaMalloc(&e->gdn_scratch, bytes));
    e->gdn_scratch_bytes = bytes;
  }
  if (e->fk_meta_ints < ints) {
    CK(cudaStreamSynchronize(st));
    cudaFree(e->fk_meta);
    const size_t cap = std::max<size_t>({ints, e->fk_meta_ints * 5 / 4, 32768});
    e->fk_meta = nullptr, e->fk_meta_ints = 0;
    CK(cudaMalloc(&e->fk_meta, cap * sizeof(int)));
    e->fk_meta_ints = cap;
  }
  const size_t kv = 2 * (size_t)d.hk * T * d.hd;
  if (e->fk_kv_halves < kv) {
    CK(cudaStreamSynchronize(st));
    cudaFree(e->fk_kv);
    const size_t cap = std::max<size_t>({kv, e->fk_kv_halves * 5 / 4, (size_t)2 * d.hk * 1024 * d.hd});
    e->fk_kv = nullptr, e->fk_kv_halves = 0;
    CK(cudaMalloc(&e->fk_kv, cap * sizeof(__half)));
    e->fk_kv_halves = cap;
  }
  return SD_OK;
}

// Grows the gathered keys of continuations (sd_forward_fork and friends) to `ktot` rows per head, by at
// least a quarter at a time, after the queued work that may use the old buffer.
int ensure_gather(sd_engine* e, long long ktot) {
  const size_t need = 2 * (size_t)e->dm.hk * ktot * e->dm.hd;
  if (ktot <= 0 || e->fk_gather_halves >= need) return SD_OK;
  CK(cudaStreamSynchronize(e->stream));
  cudaFree(e->fk_gather);
  const size_t cap = std::max(need, e->fk_gather_halves * 5 / 4);
  e->fk_gather = nullptr, e->fk_gather_halves = 0;
  CK(cudaMalloc(&e->fk_gather, cap * sizeof(__half)));
  e->fk_gather_halves = cap;
  return SD_OK;
}

// Grows pinned staging slot `slot` to `ints` ints, after its previous upload (event) is done.
int ensure_pin_slot(sd_engine* e, int slot, size_t ints) {
  if (e->fk_ev[slot]) CK(cudaEventSynchronize(e->fk_ev[slot]));
  else CK(cudaEventCreateWithFlags(&e->fk_ev[slot], cudaEventDisableTiming));
  if (e->fk_pin_ints[slot] < ints) {
    cudaFreeHost(e->fk_pin[slot]);
    const size_t cap = std::max<size_t>({ints, e->fk_pin_ints[slot] * 5 / 4, 32768});
    e->fk_pin[slot] = nullptr, e->fk_pin_ints[slot] = 0;
    CK(cudaMallocHost(&e->fk_pin[slot], cap * sizeof(int)));
    e->fk_pin_ints[slot] = cap;
  }
  return SD_OK;
}

// Validates a packed pass and enqueues it on the engine's stream: one upload (through a pinned ring
// slot) carries the per-layer tables of each sequence's snapshot buffers (and of its new snapshot,
// with `keep`), the index arrays, the global rows and, from the host, the ids; ids already on the
// device are read in place. Then the layers. caches: one per sequence, entries may be null (a fresh
// sequence; the whole array may be null); `fork` names the call in errors and requires every
// sequence to continue a snapshot. `timed` brackets the layers with the engine's events. *R_out: rows;
// snaps_out (with keep): the new snapshots. parent (may be null): per sequence -1, or the index of an
// earlier sequence without a parent that this one continues (no snapshot of its own then; no keep).
int packed_enqueue(sd_engine* e, const char* fn, const sd_snapshot* const* caches, bool fork, const uint32_t* ids_host,
                   const uint32_t* ids_dev, const int32_t* lens, int32_t nq, const int32_t* rows, const int32_t* nrows,
                   bool keep, sd_snapshot** snaps_out, bool has_out, bool timed, long long* R_out,
                   const int32_t* parent = nullptr) {
  if (nq <= 0 || (!ids_host && !ids_dev) || !lens || !nrows) return e->fail(SD_ERR_INVALID, "%s: no sequences", fn);
  if (nq > 4096) return e->fail(SD_ERR_INVALID, "%s: %d sequences in one call (at most 4096)", fn, nq);
  if (e->trace_host) return e->fail(SD_ERR_INVALID, "%s: per-layer tracing is for sd_forward only", fn);
  if (keep && !snaps_out) return e->fail(SD_ERR_INVALID, "%s: keep without a snapshot output", fn);
  long long T = 0, R = 0;
  int max_len = 0, max_p = 0, max_rows = 0, nblk = 0, nblk128 = 0, chunks = 0, max_chunks = 0;
  double pairs = 0;
  std::vector<int> pl(nq, 0);   // prefix length of each sequence
  std::vector<char> has_child(nq, 0);
  bool tree = false;
  int nroot = 0;
  for (int b = 0; b < nq; b++) {
    const int par = parent ? parent[b] : -1;
    if (par < -1 || par >= b || (par >= 0 && parent[par] >= 0))
      return e->fail(SD_ERR_INVALID, "%s: sequence %d: parent %d (an earlier sequence without a parent, or -1)", fn, b, par);
    if (par >= 0 && caches && caches[b])
      return e->fail(SD_ERR_INVALID, "%s: sequence %d continues both a snapshot and sequence %d", fn, b, par);
    if (par >= 0) tree = true, has_child[par] = 1;
    else nroot++;
    const sd_snapshot* c = par < 0 && caches ? caches[b] : nullptr;
    if (!c && par < 0 && fork) return e->fail(SD_ERR_INVALID, "%s: question %d has no snapshot (the questions continue one)", fn, b);
    if (c && c->owner != e) return e->fail(SD_ERR_INVALID, "snapshot belongs to another engine");
    const int p = par >= 0 ? pl[par] + lens[par] : (c ? c->len : 0);
    pl[b] = p;
    if (lens[b] <= 0 || p + lens[b] > SD_CONTEXT)
      return e->fail(SD_ERR_INVALID, "sequence %d: context of %d tokens: must be %d to %d", b, p + lens[b], p + 1, SD_CONTEXT);
    if (nrows[b] < 0) return e->fail(SD_ERR_INVALID, "sequence %d: negative row count", b);
    T += lens[b];
    R += nrows[b];
    max_len = std::max(max_len, (int)lens[b]);
    max_p = std::max(max_p, p);
    max_rows = std::max(max_rows, p + (int)lens[b]);
    pairs += (double)lens[b] * p + (double)lens[b] * (lens[b] + 1) / 2;
    nblk += (lens[b] + 63) / 64;
    nblk128 += (lens[b] + 127) / 128;
    chunks += (lens[b] + 63) / 64;
    max_chunks = std::max(max_chunks, ((int)lens[b] + 63) / 64);
  }
  if (T > (1 << 16)) return e->fail(SD_ERR_INVALID, "%s: %lld tokens in one call (at most 65536)", fn, T);
  if (tree && keep) return e->fail(SD_ERR_INVALID, "%s: keep with parents in the pass", fn);
  long long ktot_ll = 0;  // rows of the gathered keys (continuations: every prefix with its own rows)
  if (max_p > 0)
    for (int b = 0; b < nq; b++) ktot_ll += pl[b] + lens[b];
  if (ktot_ll > (1 << 24)) return e->fail(SD_ERR_INVALID, "%s: %lld key rows in one call", fn, ktot_ll);
  const int ktot = (int)ktot_ll;
  if (R > 0 && (!rows || !has_out)) return e->fail(SD_ERR_INVALID, "rows given without an output buffer");
  if (ids_host)
    for (long long i = 0; i < T; i++)
      if (ids_host[i] >= (uint32_t)e->vocab)
        return e->fail(SD_ERR_INVALID, "token id %u out of range (vocab %d)", ids_host[i], e->vocab);
  // long sequences (more than two 64-token chunks): the two-phase scan (a tree pass: the fused scan,
  // roots then children)
  const bool two_phase = !tree && max_chunks > 2;
  const bool outs = keep || tree;  // tables of new snapshots (a tree: the parents', written in the pass)
  // staged layout: pointer tables (8-byte words): states[n_lin][nq], hists[n_lin][nq], k[n_full][nq],
  // v[n_full][nq], with keep the same four for the new snapshots; then ints: tpos[T], tstart[T],
  // tseq[T], seq_off[nq], seq_len[nq], plen[nq], blk[2 nblk], rows[R], with the two-phase scan
  // chunk_tab[2 chunks], chunk0[nq], order[nq]; then ids[T] (host ids)
  const size_t per_set = (size_t)(2 * e->n_lin + 2 * e->n_full) * nq;
  const size_t i0 = 2 * per_set * (outs ? 2 : 1);  // ints before the index arrays
  const size_t n_idx = i0 + 3 * (size_t)T + 4 * (size_t)nq + 2 * (size_t)nblk + 2 * (size_t)nblk128;
  const size_t n_gdn = two_phase ? 2 * (size_t)chunks + 2 * (size_t)nq : 0;
  const size_t n_base = packed_ints(e, T, nq, nblk + nblk128, R, outs, two_phase ? chunks : -1, ids_host != nullptr);
  const size_t n_all = n_base + (tree ? (size_t)nq : 0);  // a tree: gorder last
  {  // rows in range
    long long r = 0;
    for (int b = 0; b < nq; b++)
      for (int j = 0; j < nrows[b]; j++, r++)
        if (rows[r] < 0 || rows[r] >= lens[b])
          return e->fail(SD_ERR_INVALID, "sequence %d: row %d out of range for %d tokens", b, rows[r], lens[b]);
  }
  cudaSetDevice(e->device);
  int rc;
  if ((rc = ensure_pool(e, (int)T)) != SD_OK || (rc = ensure_packed(e, T, n_all, two_phase ? chunks : 0)) != SD_OK ||
      (rc = ensure_gather(e, ktot)) != SD_OK)
    return rc;
  const sd::Dims& d = e->dm;
  cudaStream_t st = e->stream;
  // the new snapshots (stream-ordered allocations, before the upload that names them)
  // (a tree: the parents' new snapshots, freed after the pass in stream order)
  std::vector<std::unique_ptr<sd_snapshot>> fresh;
  if (outs) {
    fresh.resize(nq);
    for (int b = 0; b < nq; b++)
      if (keep || has_child[b])
        if ((rc = alloc_snapshot(e, pl[b] + lens[b], &fresh[b])) != SD_OK) return rc;
  }
  const int slot = e->fk_next;
  e->fk_next = (slot + 1) % sd_engine::kForkSlots;
  if ((rc = ensure_pin_slot(e, slot, n_all)) != SD_OK) return rc;
  {
    const void** pt = reinterpret_cast<const void**>(e->fk_pin[slot]);
    const size_t kb = (size_t)2 * e->n_lin * nq, vb = kb + (size_t)e->n_full * nq;
    for (int b = 0; b < nq; b++) {
      const int par = parent ? parent[b] : -1;
      // a child reads its parent's new snapshot (written earlier in each layer)
      const sd_snapshot* c = par >= 0 ? fresh[par].get() : (caches ? caches[b] : nullptr);
      for (int i = 0; i < e->n_lin; i++) {
        pt[(size_t)i * nq + b] = c ? c->state[i] : nullptr;
        pt[(size_t)(e->n_lin + i) * nq + b] = c ? c->hist[i] : nullptr;
      }
      for (int i = 0; i < e->n_full; i++) {
        pt[kb + (size_t)i * nq + b] = c ? c->k[i] : nullptr;
        pt[vb + (size_t)i * nq + b] = c ? c->v[i] : nullptr;
      }
      if (outs) {
        const sd_snapshot* o = fresh[b].get();  // null: nothing written for this sequence
        for (int i = 0; i < e->n_lin; i++) {
          pt[per_set + (size_t)i * nq + b] = o ? o->state[i] : nullptr;
          pt[per_set + (size_t)(e->n_lin + i) * nq + b] = o ? o->hist[i] : nullptr;
        }
        for (int i = 0; i < e->n_full; i++) {
          pt[per_set + kb + (size_t)i * nq + b] = o ? o->k[i] : nullptr;
          pt[per_set + vb + (size_t)i * nq + b] = o ? o->v[i] : nullptr;
        }
      }
    }
  }
  int* tpos = e->fk_pin[slot] + i0;
  int* tstart = tpos + T;
  int* tseq = tstart + T;
  int* soff = tseq + T;
  int* slen = soff + nq;
  int* plen = slen + nq;
  int* blk = plen + nq;
  int* blk128 = blk + 2 * (size_t)nblk;
  int* gofs = blk128 + 2 * (size_t)nblk128;
  int* grows = e->fk_pin[slot] + n_idx;
  int* ctab = grows + R;
  int* c0 = ctab + 2 * (size_t)chunks;
  int* order = c0 + nq;
  {
    int t = 0, k = 0, ch = 0;
    long long r = 0;
    for (int b = 0; b < nq; b++) {
      const int p = pl[b];
      soff[b] = t, slen[b] = lens[b], plen[b] = p;
      for (int j = 0; j < lens[b]; j++) tpos[t + j] = p + j, tstart[t + j] = t, tseq[t + j] = b;
      for (int q0 = 0; q0 < lens[b]; q0 += 64, k++) blk[2 * k] = b, blk[2 * k + 1] = q0;
      for (int j = 0; j < nrows[b]; j++, r++) grows[r] = t + rows[r];
      if (two_phase) {
        c0[b] = ch;
        for (int q0 = 0; q0 < lens[b]; q0 += 64, ch++) ctab[2 * ch] = t + q0, ctab[2 * ch + 1] = std::min(64, (int)lens[b] - q0);
        order[b] = b;
      }
      t += lens[b];
    }
    if (two_phase) std::stable_sort(order, order + nq, [&](int a, int b) { return lens[a] > lens[b]; });
    // 128-query blocks, those with the most keys (latest queries, longest prefixes) first
    int k2 = 0;
    for (int b = 0; b < nq; b++)
      for (int q0 = 0; q0 < lens[b]; q0 += 128, k2++) blk128[2 * k2] = b, blk128[2 * k2 + 1] = q0;
    std::vector<std::pair<int, int>> bl(nblk128);
    for (int i = 0; i < nblk128; i++) bl[i] = {blk128[2 * i], blk128[2 * i + 1]};
    auto keys = [&](const std::pair<int, int>& x) { return plen[x.first] + std::min(x.second + 128, (int)lens[x.first]); };
    std::stable_sort(bl.begin(), bl.end(),
                     [&](const std::pair<int, int>& x, const std::pair<int, int>& y) { return keys(x) > keys(y); });
    for (int i = 0; i < nblk128; i++) blk128[2 * i] = bl[i].first, blk128[2 * i + 1] = bl[i].second;
    // the gathered keys: sequence b at rows gofs[b] .. + plen[b] + lens[b]
    long long g = 0;
    for (int b = 0; b < nq; b++) gofs[b] = (int)g, g += plen[b] + lens[b];
  }
  if (ids_host) memcpy(e->fk_pin[slot] + n_idx + R + n_gdn, ids_host, T * sizeof(uint32_t));
  if (tree) {  // the scan's walk order: the roots, then the children, each longest first
    int* go = e->fk_pin[slot] + n_base;
    int k = 0;
    for (int b = 0; b < nq; b++)
      if (parent[b] < 0) go[k++] = b;
    for (int b = 0; b < nq; b++)
      if (parent[b] >= 0) go[k++] = b;
    auto longer = [&](int a, int b) { return lens[a] > lens[b]; };
    std::stable_sort(go, go + nroot, longer);
    std::stable_sort(go + nroot, go + nq, longer);
  }
  CK(cudaMemcpyAsync(e->fk_meta, e->fk_pin[slot], n_all * sizeof(int), cudaMemcpyHostToDevice, st));
  CK(cudaEventRecord(e->fk_ev[slot], st));
  if (timed) CK(cudaEventRecord(e->ev0, st));
  const int* dm = e->fk_meta;
  const void* const* dp = reinterpret_cast<const void* const*>(dm);
  const int* di = dm + i0;
  const uint32_t* ids = ids_host ? reinterpret_cast<const uint32_t*>(dm + n_idx + R + n_gdn) : ids_dev;
  Fork fk;
  fk.ids = ids;
  fk.rows = dm + n_idx;
  fk.states = reinterpret_cast<const float* const*>(dp);
  fk.hists = reinterpret_cast<const __half* const*>(dp + (size_t)e->n_lin * nq);
  fk.kp = reinterpret_cast<const __half* const*>(dp + (size_t)2 * e->n_lin * nq);
  fk.vp = reinterpret_cast<const __half* const*>(dp + (size_t)(2 * e->n_lin + e->n_full) * nq);
  if (outs) {
    void* const* op = const_cast<void* const*>(dp + per_set);
    fk.s_out = reinterpret_cast<float* const*>(op);
    fk.h_out = reinterpret_cast<__half* const*>(op + (size_t)e->n_lin * nq);
    fk.k_out = reinterpret_cast<__half* const*>(op + (size_t)2 * e->n_lin * nq);
    fk.v_out = reinterpret_cast<__half* const*>(op + (size_t)(2 * e->n_lin + e->n_full) * nq);
  }
  fk.tpos = di, fk.tstart = di + T, fk.tseq = di + 2 * T;
  fk.seq_off = di + 3 * T, fk.seq_len = fk.seq_off + nq, fk.plen = fk.seq_len + nq, fk.blk = fk.plen + nq;
  fk.blk128 = fk.blk + 2 * (size_t)nblk, fk.nblk128 = nblk128;
  fk.gofs = fk.blk128 + 2 * (size_t)nblk128, fk.ktot = ktot;
  if (two_phase) {
    fk.chunk_tab = dm + n_idx + R;
    fk.chunk0 = fk.chunk_tab + 2 * (size_t)chunks;
    fk.order = fk.chunk0 + nq;
    fk.chunks = chunks;
    fk.two_phase = true;
  }
  if (tree) fk.tree = true, fk.gorder = dm + n_base, fk.nroot = nroot;
  fk.nseq = nq, fk.nblk = nblk, fk.max_len = max_len, fk.max_p = max_p, fk.max_rows = max_rows, fk.pairs = pairs;
  fk.kt = e->fk_kv, fk.vt = e->fk_kv + (size_t)d.hk * T * d.hd;
  rc = run_layers(e, (int)T, max_p, true, (int)R, &fk);
  if (rc != SD_OK) {
    cudaStreamSynchronize(st);
    return rc;  // the new snapshots are freed with `fresh`
  }
  if (timed) CK(cudaEventRecord(e->ev1, st));
  if (keep)
    for (int b = 0; b < nq; b++) {
      e->live.push_back(fresh[b].get());
      snaps_out[b] = fresh[b].release();
    }
  *R_out = R;
  return SD_OK;
}

// A packed pass with host buffers: enqueue, copy the rows out, wait, and un-rotate the rows of a
// rotated torso (src/engine.rs:652-660). On a failure after the enqueue the new snapshots are freed.
int batch_host(sd_engine* e, const char* fn, const sd_snapshot* const* caches, bool fork, const uint32_t* ids,
               const int32_t* lens, int32_t nq, const int32_t* rows, const int32_t* nrows, bool keep, float* hidden_out,
               sd_snapshot** snaps_out, double* gpu_ms_out, const int32_t* parent = nullptr) {
  if (!ids) return e->fail(SD_ERR_INVALID, "%s: no token ids", fn);
  long long R = 0;
  int rc = packed_enqueue(e, fn, caches, fork, ids, nullptr, lens, nq, rows, nrows, keep, snaps_out, hidden_out != nullptr,
                          true, &R, parent);
  if (rc != SD_OK) return rc;
  const sd::Dims& d = e->dm;
  cudaStream_t st = e->stream;
  auto drop = [&]() {
    if (keep)
      for (int b = 0; b < nq; b++) {
        delete snaps_out[b];
        snaps_out[b] = nullptr;
      }
  };
  if ((rc = ensure_pinned(e, 1, (int)R)) != SD_OK) {
    drop();
    return rc;
  }
  if (R > 0 && cudaMemcpyAsync(e->p_out, e->out, (size_t)R * d.d * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) {
    drop();
    return e->fail(SD_ERR_CUDA, "%s: copying the rows out", fn);
  }
  if ((rc = sync_engine(e)) != SD_OK) {
    drop();
    return rc;
  }
  if (gpu_ms_out) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev0, e->ev1);
    *gpu_ms_out = ms;
  }
  if (R > 0) {
    memcpy(hidden_out, e->p_out, (size_t)R * d.d * 4);
    if ((int)e->unrotate.size() == d.d)
      for (long long r = 0; r < R; r++) {
        float* row = hidden_out + (size_t)r * d.d;
        fwht(row, d.d);
        for (int c = 0; c < d.d; c++) row[c] = (float)((double)row[c] * e->unrotate[c]);
      }
  }
  return SD_OK;
}

// The head's weights on the engine's device, uploaded on first use.
int head_weights(sd_engine* e, const sd_head* h, sd::HeadWeights* hw) {
  std::lock_guard<std::mutex> lock(h->mu);
  float*& p = h->dev[e->device];
  const size_t w = (size_t)h->dim * h->d;
  if (!p) {
    std::vector<float> all;
    all.reserve(2 * w + 2 * (size_t)h->d + 2 * (size_t)h->dim);
    for (const auto* v : {&h->qw, &h->kw, &h->nw, &h->nb, &h->qb, &h->kb}) all.insert(all.end(), v->begin(), v->end());
    float* dp = nullptr;
    CK(cudaMalloc(&dp, all.size() * sizeof(float)));
    if (cudaMemcpy(dp, all.data(), all.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaFree(dp);
      return e->fail(SD_ERR_CUDA, "uploading the head");
    }
    p = dp;
  }
  hw->qw = p, hw->kw = p + w, hw->nw = p + 2 * w, hw->nb = hw->nw + h->d, hw->qb = hw->nb + h->d, hw->kb = hw->qb + h->dim;
  return SD_OK;
}

// Queues the pointer head over the hidden rows at `hidden` (question after question, nrows[i] rows
// each: options, then the answer) on the engine's stream; the probabilities go to probs_dev, or to
// the engine's own buffer when probs_dev is null (*probs_at, *n_probs either way).
int enqueue_head(sd_engine* e, const char* fn, const sd_head* h, const float* hidden, const int32_t* nrows, int nq,
                 const double* temps, double* probs_dev, double** probs_at, long long* n_probs) {
  if (!h || !nrows || !temps || nq <= 0) return e->fail(SD_ERR_INVALID, "%s: bad arguments", fn);
  if (nq > 65535) return e->fail(SD_ERR_INVALID, "%s: %d questions in one call (at most 65535)", fn, nq);
  if (h->d != e->dm.d) return e->fail(SD_ERR_INVALID, "%s: head of width %d on a torso of %d", fn, h->d, e->dm.d);
  std::vector<sd::HeadQuestion> qs(nq);
  long long R = 0, P = 0;
  for (int i = 0; i < nq; i++) {
    if (nrows[i] < 2) return e->fail(SD_ERR_INVALID, "%s: question %d has %d rows (options and the answer: 2 or more)", fn, i, nrows[i]);
    qs[i].row0 = (int)R, qs[i].nrows = nrows[i], qs[i].prob0 = (int)P, qs[i].pad = 0;
    qs[i].scale = std::pow((double)h->dim, -0.5) / std::max(temps[i], 1e-6);
    R += nrows[i];
    P += nrows[i] - 1;
  }
  if (R > (1 << 24)) return e->fail(SD_ERR_INVALID, "%s: %lld rows", fn, R);
  cudaSetDevice(e->device);
  sd::HeadWeights hw;
  int rc = head_weights(e, h, &hw);
  if (rc != SD_OK) return rc;
  if (!e->unrotate.empty() && !e->d_unrot) {
    CK(cudaMalloc(&e->d_unrot, e->unrotate.size() * sizeof(double)));
    CK(cudaMemcpy(e->d_unrot, e->unrotate.data(), e->unrotate.size() * sizeof(double), cudaMemcpyHostToDevice));
  }
  auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
  const size_t tb = up((size_t)nq * sizeof(sd::HeadQuestion)), xb = up((size_t)R * h->d * 8), pb = up((size_t)R * h->dim * 8),
               ob = up((size_t)P * 8);
  if (e->hd_bytes < tb + xb + pb + ob) {
    CK(cudaStreamSynchronize(e->stream));
    cudaFree(e->hd_buf);
    e->hd_buf = nullptr, e->hd_bytes = 0;
    const size_t want = std::max<size_t>(tb + xb + pb + ob, (size_t)4 << 20);
    CK(cudaMalloc(&e->hd_buf, want));
    e->hd_bytes = want;
  }
  char* base = (char*)e->hd_buf;
  auto* dq = (sd::HeadQuestion*)base;
  auto* xn = (double*)(base + tb);
  auto* proj = (double*)(base + tb + xb);
  double* probs = probs_dev ? probs_dev : (double*)(base + tb + xb + pb);
  // a pageable source: staged before the call returns, so `qs` may go
  CK(cudaMemcpyAsync(dq, qs.data(), (size_t)nq * sizeof(sd::HeadQuestion), cudaMemcpyHostToDevice, e->stream));
  const double* unrot = (int)e->unrotate.size() == h->d ? e->d_unrot : nullptr;
  const double bytes = (double)R * h->d * 4 + 2.0 * h->dim * h->d * 4 + (double)P * 8;
  cudaError_t ce = launch(e, SD_PROF_OTHER, bytes, [&](int* nl) -> cudaError_t {
    *nl = 3;
    return sd::launch_head(hidden, (int)R, dq, nq, h->d, h->dim, unrot, hw, xn, proj, probs, e->stream);
  });
  if (ce != cudaSuccess) return e->fail(SD_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(ce));
  if (probs_at) *probs_at = probs;
  if (n_probs) *n_probs = P;
  return SD_OK;
}

}  // namespace

extern "C" {

const char* sd_last_error(void) { return g_last_error.c_str(); }

int sd_engine_create(const char* model_dir, int device, sd_engine** out) {
  if (!model_dir || !out) {
    set_global_error("sd_engine_create: null argument");
    return SD_ERR_INVALID;
  }
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev || device >= sd::kMaxDevices) {
    set_global_error("sd_engine_create: no CUDA device " + std::to_string(device));
    return SD_ERR_CUDA;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) {
    set_global_error("sd_engine_create: device " + std::to_string(device) + " is not an sm_100 (B200) GPU");
    return SD_ERR_CUDA;
  }
  auto* e = new sd_engine();
  e->device = device;
  e->num_sms = prop.multiProcessorCount;
  if (const char* k = getenv("SD_GDN_KERNEL")) e->gdn_mode = strcmp(k, "tc") == 0 ? 1 : strcmp(k, "legacy") == 0 ? 2 : 0;
  cudaSetDevice(device);
  if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess || cudaEventCreate(&e->ev0) != cudaSuccess ||
      cudaEventCreate(&e->ev1) != cudaSuccess) {
    set_global_error("sd_engine_create: cannot create a stream");
    sd_engine_destroy(e);
    return SD_ERR_CUDA;
  }
  {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    uint64_t keep_all = UINT64_MAX;
    if (cudaMemPoolCreate(&e->snap_pool, &props) != cudaSuccess ||
        cudaMemPoolSetAttribute(e->snap_pool, cudaMemPoolAttrReleaseThreshold, &keep_all) != cudaSuccess) {
      set_global_error("sd_engine_create: cannot create the snapshot memory pool");
      sd_engine_destroy(e);
      return SD_ERR_CUDA;
    }
  }
  int rc = load_engine(e, model_dir);
  if (rc != SD_OK) {
    set_global_error(e->err);
    sd_engine_destroy(e);
    return rc;
  }
  cudaError_t ce;
  if ((ce = sd::preload_gemm()) != cudaSuccess || (ce = sd::preload_attention()) != cudaSuccess ||
      (ce = sd::preload_attention_tc()) != cudaSuccess ||
      (ce = sd::preload_gdn()) != cudaSuccess || (ce = sd::preload_gdn_tc()) != cudaSuccess ||
      (ce = sd::preload_kernels()) != cudaSuccess ||
      (ce = sd::preload_head()) != cudaSuccess) {
    set_global_error(std::string("sd_engine_create: loading the kernels: ") + cudaGetErrorString(ce));
    sd_engine_destroy(e);
    return SD_ERR_CUDA;
  }
  // pinned staging for the largest context up front (a resize inside a timed forward would cost a
  // pinned allocation)
  if ((rc = ensure_pinned(e, SD_CONTEXT, 64)) != SD_OK) {
    set_global_error(e->err);
    sd_engine_destroy(e);
    return rc;
  }
  *out = e;
  return SD_OK;
}

void sd_engine_destroy(sd_engine* e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (auto* snap : e->live) snap->owner = nullptr;  // freed synchronously later
  for (auto ev : e->prof_events) cudaEventDestroy(ev);
  free_pool(e);
  for (auto p : e->shards) cudaFree(p);
  for (auto& L : e->layers)
    for (QWeight* w : {&L.in_proj, &L.out_proj, &L.qkv, &L.o_proj, &L.gate_up, &L.down, &L.proj}) cudaFree(w->tiles);
  for (auto p : e->state) cudaFree(p);
  for (auto p : e->hist) cudaFree(p);
  for (auto p : e->kc) cudaFree(p);
  for (auto p : e->vc) cudaFree(p);
  cudaFree(e->embed_q);
  cudaFree(e->embed_s);
  cudaFree(e->rope);
  cudaFree(e->d_err);
  cudaFreeHost(e->p_ids);
  cudaFreeHost(e->p_rows);
  cudaFreeHost(e->p_out);
  cudaFree(e->fk_meta);
  cudaFree(e->fk_kv);
  cudaFree(e->fk_gather);
  cudaFree(e->hd_buf);
  cudaFree(e->d_unrot);
  cudaFreeHost(e->hd_pin);
  for (int i = 0; i < sd_engine::kForkSlots; i++) {
    cudaFreeHost(e->fk_pin[i]);
    if (e->fk_ev[i]) cudaEventDestroy(e->fk_ev[i]);
  }
  if (e->ev0) cudaEventDestroy(e->ev0);
  if (e->ev1) cudaEventDestroy(e->ev1);
  if (e->snap_pool) cudaMemPoolDestroy(e->snap_pool);  // deferred while snapshots still hold memory
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

int sd_engine_reserve(sd_engine* e, int32_t max_tokens, int32_t max_seqs, int32_t max_rows) {
  if (!e) return SD_ERR_INVALID;
  if (max_tokens <= 0 || max_tokens > (1 << 16) || max_seqs <= 0 || max_seqs > 4096 || max_rows < 0)
    return e->fail(SD_ERR_INVALID, "sd_engine_reserve: tokens 1..65536, sequences 1..4096, rows >= 0");
  cudaSetDevice(e->device);
  const long long T = max_tokens, nq = max_seqs, chunks = T / 64 + nq;
  const size_t ints = packed_ints(e, T, nq, 2 * chunks, max_rows, true, chunks, true);  // 64- and 128-query blocks
  int rc;
  if ((rc = ensure_pool(e, max_tokens)) != SD_OK || (rc = ensure_packed(e, T, ints, chunks)) != SD_OK ||
      (rc = ensure_pinned(e, max_tokens, max_rows)) != SD_OK)
    return rc;
  for (int s = 0; s < sd_engine::kForkSlots; s++)
    if ((rc = ensure_pin_slot(e, s, ints)) != SD_OK) return rc;
  // continuations' gathered keys: every sequence a whole context at most (capped at 2^20 rows a head)
  if ((rc = ensure_gather(e, std::min<long long>((long long)max_seqs * SD_CONTEXT, 1 << 20))) != SD_OK) return rc;
  // the snapshots of such a pass (kept by the pool once freed): max_seqs states and histories, and
  // K/V for max_tokens rows
  const sd::Dims& d = e->dm;
  const size_t snap_bytes = (size_t)max_seqs * e->n_lin * ((size_t)d.h * d.dk * d.dv * 4 + (size_t)3 * d.C() * 2) +
                            (size_t)2 * e->n_full * d.hk * max_tokens * d.hd * 2;
  void* prime = nullptr;
  CK(cudaMallocFromPoolAsync(&prime, snap_bytes, e->snap_pool, e->stream));
  CK(cudaFreeAsync(prime, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  return SD_OK;
}

int sd_engine_hidden_size(const sd_engine* e) { return e ? e->dm.d : 0; }
int sd_engine_num_layers(const sd_engine* e) { return e ? e->n_layers : 0; }
const char* sd_engine_last_error(const sd_engine* e) { return e ? e->err.c_str() : g_last_error.c_str(); }

int sd_engine_set_trace(sd_engine* e, float* host_buf, size_t floats) {
  if (!e) return SD_ERR_INVALID;
  cudaSetDevice(e->device);
  e->trace_host = host_buf;
  e->trace_floats = host_buf ? floats : 0;
  if (!host_buf) {
    cudaFree(e->trace_dev);
    e->trace_dev = nullptr;
  } else if (e->cap > 0 && !e->trace_dev) {
    CK(cudaMalloc(&e->trace_dev, (size_t)e->n_layers * e->cap * e->dm.d * 4));
  }
  return SD_OK;
}

int sd_forward(sd_engine* e, const uint32_t* ids, int32_t l, const int32_t* rows, int32_t nrows, const sd_snapshot* cache,
               int32_t keep, float* hidden_out, sd_snapshot** snapshot_out, double* gpu_ms_out) {
  if (!e) return SD_ERR_INVALID;
  int rc = check_forward_args(e, l, nrows, cache, keep, snapshot_out);
  if (rc != SD_OK) return rc;
  if (!ids) return e->fail(SD_ERR_INVALID, "no token ids");
  if (nrows > 0 && (!rows || !hidden_out)) return e->fail(SD_ERR_INVALID, "rows given without an output buffer");
  for (int i = 0; i < nrows; i++)
    if (rows[i] < 0 || rows[i] >= l) return e->fail(SD_ERR_INVALID, "row %d out of range for %d tokens", rows[i], l);
  for (int i = 0; i < l; i++)
    if (ids[i] >= (uint32_t)e->vocab) return e->fail(SD_ERR_INVALID, "token id %u out of range (vocab %d)", ids[i], e->vocab);
  cudaSetDevice(e->device);
  if ((rc = ensure_pool(e, l)) != SD_OK || (rc = ensure_pinned(e, l, nrows)) != SD_OK) return rc;
  const sd::Dims& d = e->dm;
  cudaStream_t st = e->stream;
  memcpy(e->p_ids, ids, l * sizeof(uint32_t));
  CK(cudaMemcpyAsync(e->d_ids, e->p_ids, l * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
  if (nrows > 0) {
    memcpy(e->p_rows, rows, nrows * sizeof(int));
    CK(cudaMemcpyAsync(e->d_rows, e->p_rows, nrows * sizeof(int), cudaMemcpyHostToDevice, st));
  }
  CK(cudaEventRecord(e->ev0, st));
  sd_snapshot* snap = nullptr;
  rc = forward_core(e, l, cache, nrows, keep != 0, &snap);
  if (rc != SD_OK) {
    cudaStreamSynchronize(st);
    return rc;
  }
  CK(cudaEventRecord(e->ev1, st));
  if (nrows > 0) CK(cudaMemcpyAsync(e->p_out, e->out, (size_t)nrows * d.d * 4, cudaMemcpyDeviceToHost, st));
  if (e->trace_dev)
    CK(cudaMemcpyAsync(e->trace_host, e->trace_dev, (size_t)e->n_layers * l * d.d * 4, cudaMemcpyDeviceToHost, st));
  rc = sync_engine(e);
  if (rc != SD_OK) {
    delete snap;
    return rc;
  }
  if (gpu_ms_out) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev0, e->ev1);
    *gpu_ms_out = ms;
  }
  if (nrows > 0) {
    memcpy(hidden_out, e->p_out, (size_t)nrows * d.d * 4);
    // a rotated torso: the head's basis is unrotate * FWHT(row) (src/engine.rs:652-660)
    if ((int)e->unrotate.size() == d.d)
      for (int r = 0; r < nrows; r++) {
        float* row = hidden_out + (size_t)r * d.d;
        fwht(row, d.d);
        for (int c = 0; c < d.d; c++) row[c] = (float)((double)row[c] * e->unrotate[c]);
      }
  }
  if (keep) *snapshot_out = snap;
  return SD_OK;
}

int sd_forward_fork(sd_engine* e, const sd_snapshot* cache, const uint32_t* ids, const int32_t* lens, int32_t nq,
                    const int32_t* rows, const int32_t* nrows, float* hidden_out, double* gpu_ms_out) {
  if (!e) return SD_ERR_INVALID;
  if (!cache) return e->fail(SD_ERR_INVALID, "sd_forward_fork: no snapshot (the questions continue one)");
  if (nq <= 0 || nq > 4096) return e->fail(SD_ERR_INVALID, "sd_forward_fork: %d questions (1 to 4096)", nq);
  const std::vector<const sd_snapshot*> caches(nq, cache);
  return sd_forward_fork_multi(e, caches.data(), ids, lens, nq, rows, nrows, hidden_out, gpu_ms_out);
}

int sd_forward_fork_multi(sd_engine* e, const sd_snapshot* const* caches, const uint32_t* ids, const int32_t* lens,
                          int32_t nq, const int32_t* rows, const int32_t* nrows, float* hidden_out, double* gpu_ms_out) {
  if (!e) return SD_ERR_INVALID;
  if (!caches) return e->fail(SD_ERR_INVALID, "sd_forward_fork: no snapshots (the questions continue one)");
  return batch_host(e, "sd_forward_fork", caches, true, ids, lens, nq, rows, nrows, false, hidden_out, nullptr, gpu_ms_out);
}

int sd_forward_batch(sd_engine* e, const sd_snapshot* const* caches, const uint32_t* ids, const int32_t* lens, int32_t nseq,
                     const int32_t* rows, const int32_t* nrows, int32_t keep, float* hidden_out, sd_snapshot** snapshots_out,
                     double* gpu_ms_out) {
  if (!e) return SD_ERR_INVALID;
  return batch_host(e, "sd_forward_batch", caches, false, ids, lens, nseq, rows, nrows, keep != 0, hidden_out, snapshots_out,
                    gpu_ms_out);
}

int sd_forward_fork_dev(sd_engine* e, const sd_snapshot* cache, const uint32_t* ids_dev, const int32_t* lens, int32_t nq,
                        const int32_t* rows, const int32_t* nrows, float* hidden_dev) {
  if (!e) return SD_ERR_INVALID;
  if (!cache) return e->fail(SD_ERR_INVALID, "sd_forward_fork: no snapshot (the questions continue one)");
  if (nq <= 0 || nq > 4096) return e->fail(SD_ERR_INVALID, "sd_forward_fork: %d questions (1 to 4096)", nq);
  const std::vector<const sd_snapshot*> caches(nq, cache);
  return sd_forward_fork_multi_dev(e, caches.data(), ids_dev, lens, nq, rows, nrows, hidden_dev);
}

int sd_forward_fork_multi_dev(sd_engine* e, const sd_snapshot* const* caches, const uint32_t* ids_dev, const int32_t* lens,
                              int32_t nq, const int32_t* rows, const int32_t* nrows, float* hidden_dev) {
  if (!e) return SD_ERR_INVALID;
  if (!caches) return e->fail(SD_ERR_INVALID, "sd_forward_fork: no snapshots (the questions continue one)");
  long long R = 0;
  int rc = packed_enqueue(e, "sd_forward_fork", caches, true, nullptr, ids_dev, lens, nq, rows, nrows, false, nullptr,
                          hidden_dev != nullptr, false, &R);
  if (rc != SD_OK) return rc;
  if (R > 0) CK(cudaMemcpyAsync(hidden_dev, e->out, (size_t)R * e->dm.d * 4, cudaMemcpyDeviceToDevice, e->stream));
  return SD_OK;
}

int sd_forward_batch_dev(sd_engine* e, const sd_snapshot* const* caches, const uint32_t* ids_dev, const int32_t* lens,
                         int32_t nseq, const int32_t* rows, const int32_t* nrows, int32_t keep, float* hidden_dev,
                         sd_snapshot** snapshots_out) {
  if (!e) return SD_ERR_INVALID;
  long long R = 0;
  int rc = packed_enqueue(e, "sd_forward_batch", caches, false, nullptr, ids_dev, lens, nseq, rows, nrows, keep != 0,
                          snapshots_out, hidden_dev != nullptr, false, &R);
  if (rc != SD_OK) return rc;
  if (R > 0) CK(cudaMemcpyAsync(hidden_dev, e->out, (size_t)R * e->dm.d * 4, cudaMemcpyDeviceToDevice, e->stream));
  return SD_OK;
}

int sd_forward_tree_dev(sd_engine* e, const sd_snapshot* const* caches, const int32_t* parent, const uint32_t* ids_dev,
                        const int32_t* lens, int32_t nseq, const int32_t* rows, const int32_t* nrows, float* hidden_dev) {
  if (!e) return SD_ERR_INVALID;
  if (!parent) return e->fail(SD_ERR_INVALID, "sd_forward_tree: no parent table");
  long long R = 0;
  int rc = packed_enqueue(e, "sd_forward_tree", caches, false, nullptr, ids_dev, lens, nseq, rows, nrows, false, nullptr,
                          hidden_dev != nullptr, false, &R, parent);
  if (rc != SD_OK) return rc;
  if (R > 0) CK(cudaMemcpyAsync(hidden_dev, e->out, (size_t)R * e->dm.d * 4, cudaMemcpyDeviceToDevice, e->stream));
  return SD_OK;
}

int sd_forward_dev(sd_engine* e, const uint32_t* ids_dev, int32_t l, const int32_t* rows_dev, int32_t nrows,
                   const sd_snapshot* cache, int32_t keep, float* hidden_dev, sd_snapshot** snapshot_out) {
  if (!e) return SD_ERR_INVALID;
  int rc = check_forward_args(e, l, nrows, cache, keep, snapshot_out);
  if (rc != SD_OK) return rc;
  if (!ids_dev || (nrows > 0 && (!rows_dev || !hidden_dev)))
    return e->fail(SD_ERR_INVALID, "null device buffer");
  if (e->trace_host) return e->fail(SD_ERR_INVALID, "tracing needs sd_forward");
  cudaSetDevice(e->device);
  if ((rc = ensure_pool(e, l)) != SD_OK) return rc;
  cudaStream_t st = e->stream;
  CK(cudaMemcpyAsync(e->d_ids, ids_dev, l * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
  if (nrows > 0) CK(cudaMemcpyAsync(e->d_rows, rows_dev, nrows * sizeof(int), cudaMemcpyDeviceToDevice, st));
  sd_snapshot* snap = nullptr;
  rc = forward_core(e, l, cache, nrows, keep != 0, &snap);
  if (rc != SD_OK) return rc;
  if (nrows > 0) CK(cudaMemcpyAsync(hidden_dev, e->out, (size_t)nrows * e->dm.d * 4, cudaMemcpyDeviceToDevice, st));
  if (keep) *snapshot_out = snap;
  return SD_OK;
}

int sd_engine_synchronize(sd_engine* e) {
  if (!e) return SD_ERR_INVALID;
  cudaSetDevice(e->device);
  return sync_engine(e);
}

int sd_engine_selftest_wait(sd_engine* e, int32_t limit_us) {
  if (!e) return SD_ERR_INVALID;
  if (limit_us < 1 || limit_us > 1000000) return e->fail(SD_ERR_INVALID, "selftest: limit_us must be 1..1000000");
  cudaSetDevice(e->device);
  int rc = sync_engine(e);  // earlier work first, so that its errors stay its own
  if (rc != SD_OK) return rc;
  const cudaError_t ce = sd::launch_wait_probe(e->d_err, (unsigned long long)limit_us * 1000ull, e->stream);
  if (ce != cudaSuccess) return e->fail(SD_ERR_CUDA, "selftest: %s", cudaGetErrorString(ce));
  return sync_engine(e);
}

void* sd_engine_stream(const sd_engine* e) { return e ? (void*)e->stream : nullptr; }
int64_t sd_engine_launches(const sd_engine* e) { return e ? e->launches : 0; }

int sd_engine_profile(sd_engine* e, int32_t enable) {
  if (!e) return SD_ERR_INVALID;
  cudaSetDevice(e->device);
  int rc = sync_engine(e);
  e->prof_on = enable != 0;
  for (int k = 0; k < SD_PROF_KINDS; k++) e->prof_ms[k] = e->prof_units[k] = 0.0, e->prof_count[k] = 0;
  return rc;
}

int sd_engine_profile_get(sd_engine* e, int32_t kind, double* ms, int64_t* launches, double* work) {
  if (!e || kind < 0 || kind >= SD_PROF_KINDS) return SD_ERR_INVALID;
  cudaSetDevice(e->device);
  int rc = sync_engine(e);
  if (ms) *ms = e->prof_ms[kind];
  if (launches) *launches = e->prof_count[kind];
  if (work) *work = e->prof_units[kind];
  return rc;
}

int32_t sd_snapshot_len(const sd_snapshot* s) { return s ? s->len : 0; }
void sd_snapshot_free(sd_snapshot* s) { delete s; }

// ---------------------------------------------------------------------------------------------
// Pointer head (src/head.rs): LayerNorm (eps 1e-5), q/k projections, scaled dot, softmax; f64.
// ---------------------------------------------------------------------------------------------
int sd_head_load(const char* path, sd_head** out) {
  if (!path || !out) return SD_ERR_INVALID;
  std::string bytes;
  if (!read_file(path, bytes)) {
    set_global_error(std::string(path) + ": cannot read");
    return SD_ERR_IO;
  }
  auto bad = [](const char* why) {
    set_global_error(std::string("head.safetensors: ") + why);
    return SD_ERR_FORMAT;
  };
  if (bytes.size() < 8) return bad("malformed");
  uint64_t n = 0;
  memcpy(&n, bytes.data(), 8);
  if (8 + n > bytes.size()) return bad("malformed");
  sd::json::Value hdr;
  try {
    hdr = sd::json::parse(bytes.substr(8, n));
  } catch (...) {
    return bad("malformed");
  }
  auto h = std::make_unique<sd_head>();
  const char* names[6] = {"norm.weight", "norm.bias", "q.weight", "q.bias", "k.weight", "k.bias"};
  std::vector<float>* dst[6] = {&h->nw, &h->nb, &h->qw, &h->qb, &h->kw, &h->kb};
  for (int i = 0; i < 6; i++) {
    const auto* t = hdr.get(names[i]);
    if (!t) {
      set_global_error(std::string("head.safetensors: no ") + names[i]);
      return SD_ERR_FORMAT;
    }
    if (t->at("dtype").str != "F32") return bad("tensors must be F32");
    const auto& off = t->at("data_offsets").arr;
    const size_t a = (size_t)off[0].integer(), b = (size_t)off[1].integer();
    if (b < a || 8 + n + b > bytes.size() || (b - a) % 4) return bad("malformed");
    dst[i]->resize((b - a) / 4);
    memcpy(dst[i]->data(), bytes.data() + 8 + n + a, b - a);
    if (i == 2) h->dim = (int)t->at("shape").arr[0].integer();
  }
  h->d = (int)h->nw.size();
  if (h->dim <= 0 || h->qw.size() != (size_t)h->dim * h->d || h->kw.size() != h->qw.size()) return bad("shapes");
  *out = h.release();
  return SD_OK;
}

void sd_head_free(sd_head* h) {
  if (!h) return;
  for (int dv = 0; dv < sd::kMaxDevices; dv++)
    if (h->dev[dv]) {
      cudaSetDevice(dv);
      cudaFree(h->dev[dv]);
    }
  delete h;
}

int sd_head_probs(const sd_head* h, const float* hidden, int32_t nrows, int32_t d, double temperature, double* probs) {
  if (!h || !hidden || !probs || nrows < 2 || d != h->d) {
    set_global_error("sd_head_probs: bad arguments");
    return SD_ERR_INVALID;
  }
  // LayerNorm (eps 1e-5) then the q or k projection, in f64 (src/head.rs:55-66): xn = (x - mean) r
  // norm.weight + norm.bias, out[o] = bias[o] + sum_j w[o][j] xn[j] with the f32 weights promoted; all
  // `n` rows at once, so each weight row is read once for all of them
  auto project = [&](const float* x, int n, const std::vector<float>& w, const std::vector<float>& b,
                     std::vector<double>& outv) {
    std::vector<double> xn((size_t)n * d);
    for (int i = 0; i < n; i++) {
      const float* xi = x + (size_t)i * d;
      double mean = 0.0, var = 0.0;
      for (int j = 0; j < d; j++) mean += (double)xi[j];
      mean /= d;
      for (int j = 0; j < d; j++) var += ((double)xi[j] - mean) * ((double)xi[j] - mean);
      var /= d;
      const double r = 1.0 / std::sqrt(var + 1e-5);
      for (int j = 0; j < d; j++) xn[(size_t)i * d + j] = ((double)xi[j] - mean) * r * (double)h->nw[j] + (double)h->nb[j];
    }
    outv.assign((size_t)n * h->dim, 0.0);
    for (int o = 0; o < h->dim; o++) {
      const float* wp = w.data() + (size_t)o * d;
      for (int i = 0; i < n; i++) {
        const double* xp = xn.data() + (size_t)i * d;
        // four 4-wide f64 partial sums over j (AVX2 + FMA); the tail in scalar
        __m256d a0 = _mm256_setzero_pd(), a1 = a0, a2 = a0, a3 = a0;
        int j = 0;
        for (; j + 16 <= d; j += 16) {
          a0 = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm_loadu_ps(wp + j)), _mm256_loadu_pd(xp + j), a0);
          a1 = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm_loadu_ps(wp + j + 4)), _mm256_loadu_pd(xp + j + 4), a1);
          a2 = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm_loadu_ps(wp + j + 8)), _mm256_loadu_pd(xp + j + 8), a2);
          a3 = _mm256_fmadd_pd(_mm256_cvtps_pd(_mm_loadu_ps(wp + j + 12)), _mm256_loadu_pd(xp + j + 12), a3);
        }
        double part[4];
        _mm256_storeu_pd(part, _mm256_add_pd(_mm256_add_pd(a0, a1), _mm256_add_pd(a2, a3)));
        double sum = (part[0] + part[1]) + (part[2] + part[3]);
        for (; j < d; j++) sum += (double)wp[j] * xp[j];
        outv[(size_t)i * h->dim + o] = (double)b[o] + sum;
      }
    }
  };
  std::vector<double> q, k;
  const int nopt = nrows - 1;
  project(hidden + (size_t)nopt * d, 1, h->qw, h->qb, q);
  project(hidden, nopt, h->kw, h->kb, k);
  const double scale = std::pow((double)h->dim, -0.5) / std::max(temperature, 1e-6);
  double mx = -1.79769313486231570e308;
  for (int i = 0; i < nopt; i++) {
    double s = 0.0;
    for (int o = 0; o < h->dim; o++) s += k[(size_t)i * h->dim + o] * q[o];
    probs[i] = s * scale;
    mx = std::max(mx, probs[i]);
  }
  double z = 0.0;
  for (int i = 0; i < nopt; i++) {
    probs[i] = std::exp(probs[i] - mx);
    z += probs[i];
  }
  for (int i = 0; i < nopt; i++) probs[i] /= z;
  return SD_OK;
}

int sd_head_probs_dev(sd_engine* e, const sd_head* h, const float* hidden_dev, const int32_t* nrows, int32_t nq,
                      const double* temperatures, double* probs_dev) {
  if (!e) return SD_ERR_INVALID;
  if (!hidden_dev || !probs_dev) return e->fail(SD_ERR_INVALID, "sd_head_probs_dev: null device buffer");
  return enqueue_head(e, "sd_head_probs_dev", h, hidden_dev, nrows, nq, temperatures, probs_dev, nullptr, nullptr);
}

int sd_forward_fork_multi_probs(sd_engine* e, const sd_snapshot* const* caches, const uint32_t* ids, const int32_t* lens,
                                int32_t nq, const int32_t* rows, const int32_t* nrows, const sd_head* h,
                                const double* temperatures, double* probs_out) {
  if (!e) return SD_ERR_INVALID;
  const char* fn = "sd_forward_fork_multi_probs";
  if (!caches) return e->fail(SD_ERR_INVALID, "%s: no snapshots (the questions continue one)", fn);
  if (!ids || !probs_out || !rows || !nrows) return e->fail(SD_ERR_INVALID, "%s: null argument", fn);
  if (!h || !temperatures) return e->fail(SD_ERR_INVALID, "%s: no head", fn);
  if (h->d != e->dm.d) return e->fail(SD_ERR_INVALID, "%s: head of width %d on a torso of %d", fn, h->d, e->dm.d);
  for (int i = 0; i < nq; i++)
    if (nrows[i] < 2) return e->fail(SD_ERR_INVALID, "%s: question %d has %d rows (options and the answer: 2 or more)", fn, i, nrows[i]);
  long long R = 0;
  int rc = packed_enqueue(e, fn, caches, true, ids, nullptr, lens, nq, rows, nrows, false, nullptr, true, true, &R);
  if (rc != SD_OK) return rc;
  double* probs = nullptr;
  long long P = 0;
  if ((rc = enqueue_head(e, fn, h, e->out, nrows, nq, temperatures, nullptr, &probs, &P)) != SD_OK) return rc;
  if (e->hd_pin_doubles < (size_t)P) {
    CK(cudaStreamSynchronize(e->stream));
    cudaFreeHost(e->hd_pin);
    e->hd_pin = nullptr, e->hd_pin_doubles = 0;
    const size_t cap = std::max<size_t>((size_t)P, 4096);
    CK(cudaMallocHost(&e->hd_pin, cap * sizeof(double)));
    e->hd_pin_doubles = cap;
  }
  CK(cudaMemcpyAsync(e->hd_pin, probs, (size_t)P * sizeof(double), cudaMemcpyDeviceToHost, e->stream));
  if ((rc = sync_engine(e)) != SD_OK) return rc;
  memcpy(probs_out, e->hd_pin, (size_t)P * sizeof(double));
  return SD_OK;
}

int sd_forward_tree(sd_engine* e, const sd_snapshot* const* caches, const int32_t* parent, const uint32_t* ids,
                    const int32_t* lens, int32_t nseq, const int32_t* rows, const int32_t* nrows, float* hidden_out) {
  if (!e) return SD_ERR_INVALID;
  if (!parent) return e->fail(SD_ERR_INVALID, "sd_forward_tree: no parent table");
  return batch_host(e, "sd_forward_tree", caches, false, ids, lens, nseq, rows, nrows, false, hidden_out, nullptr, nullptr,
                    parent);
}

int sd_forward_tree_probs(sd_engine* e, const sd_snapshot* const* caches, const int32_t* parent, const uint32_t* ids,
                          const int32_t* lens, int32_t nseq, const int32_t* rows, const int32_t* nrows, const sd_head* h,
                          const double* temperatures, double* probs_out) {
  if (!e) return SD_ERR_INVALID;
  const char* fn = "sd_forward_tree_probs";
  if (!parent || !ids || !lens || !nrows || !probs_out) return e->fail(SD_ERR_INVALID, "%s: null argument", fn);
  if (!h || !temperatures) return e->fail(SD_ERR_INVALID, "%s: no head", fn);
  if (h->d != e->dm.d) return e->fail(SD_ERR_INVALID, "%s: head of width %d on a torso of %d", fn, h->d, e->dm.d);
  if (nseq <= 0 || nseq > 4096) return e->fail(SD_ERR_INVALID, "%s: %d sequences", fn, nseq);
  // the head runs over the sequences with rows (their options and the answer row), in order
  std::vector<int32_t> hn;
  std::vector<double> ht;
  for (int i = 0; i < nseq; i++) {
    if (nrows[i] == 0) continue;
    if (nrows[i] < 2) return e->fail(SD_ERR_INVALID, "%s: sequence %d has %d rows (none, or options and the answer)", fn, i, nrows[i]);
    hn.push_back(nrows[i]);
    ht.push_back(temperatures[i]);
  }
  if (hn.empty()) return e->fail(SD_ERR_INVALID, "%s: no sequence has rows", fn);
  if (!rows) return e->fail(SD_ERR_INVALID, "%s: null argument", fn);
  long long R = 0;
  int rc = packed_enqueue(e, fn, caches, false, ids, nullptr, lens, nseq, rows, nrows, false, nullptr, true, true, &R, parent);
  if (rc != SD_OK) return rc;
  double* probs = nullptr;
  long long P = 0;
  if ((rc = enqueue_head(e, fn, h, e->out, hn.data(), (int32_t)hn.size(), ht.data(), nullptr, &probs, &P)) != SD_OK) return rc;
  if (e->hd_pin_doubles < (size_t)P) {
    CK(cudaStreamSynchronize(e->stream));
    cudaFreeHost(e->hd_pin);
    e->hd_pin = nullptr, e->hd_pin_doubles = 0;
    const size_t cap = std::max<size_t>((size_t)P, 4096);
    CK(cudaMallocHost(&e->hd_pin, cap * sizeof(double)));
    e->hd_pin_doubles = cap;
  }
  CK(cudaMemcpyAsync(e->hd_pin, probs, (size_t)P * sizeof(double), cudaMemcpyDeviceToHost, e->stream));
  if ((rc = sync_engine(e)) != SD_OK) return rc;
  memcpy(probs_out, e->hd_pin, (size_t)P * sizeof(double));
  return SD_OK;
}

// ---------------------------------------------------------------------------------------------
// Kernel-level entry points
// ---------------------------------------------------------------------------------------------
static int op_result(cudaError_t ce, const char* what) {
  if (ce == cudaSuccess) return SD_OK;
  set_global_error(std::string(what) + ": " + cudaGetErrorString(ce));
  return ce == cudaErrorInvalidValue ? SD_ERR_INVALID : SD_ERR_CUDA;
}

int sd_decode_scales(const void* src_dev, int32_t n, int32_t g, void* dst_dev, void* stream) {
  if (!src_dev || !dst_dev || n < 0 || g <= 0 || g > (1 << 20)) {
    set_global_error("sd_decode_scales: bad arguments");
    return SD_ERR_INVALID;
  }
  if (n == 0) return SD_OK;
  const uint8_t* src = (const uint8_t*)src_dev;
  std::vector<uint8_t> hdr((size_t)4 * n);
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t ce = cudaMemcpyAsync(hdr.data(), src, hdr.size(), cudaMemcpyDeviceToHost, st);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
  if (ce != cudaSuccess) return op_result(ce, "sd_decode_scales");
  int jmax = 0;
  for (int32_t r = 0; r < n; r++) jmax = std::max(jmax, (int)(hdr[4 * (size_t)r + 2] | (hdr[4 * (size_t)r + 3] << 8)));
  return op_result(sd::decode_scales_dev(src, 4, src + 4 * (size_t)n, g, n, g, jmax, (uint16_t*)dst_dev, g, st),
                   "sd_decode_scales");
}

int sd_attention(const void* q, const void* k, const void* v, const void* gate, int32_t gstride, int32_t goff, int32_t gstep,
                 void* out, int32_t l, int32_t p, int32_t lt, int32_t hq, int32_t hk, int32_t hd, void* stream) {
  if (!q || !k || !v || !out || l <= 0 || p < 0 || p + l > lt || hk <= 0 || hq % hk) {
    set_global_error("sd_attention: bad arguments");
    return SD_ERR_INVALID;
  }
  if (l >= 128 && hd == 256) {  // query blocks of 128: the tcgen05 kernel
    sd::AttnTcArgs ta;
    ta.l = l, ta.p = p, ta.hq = hq, ta.hk = hk, ta.gate = (const __half*)gate, ta.gstride = gstride, ta.goff = goff,
    ta.gstep = gstep, ta.out = (__half*)out;
    return op_result(sd::launch_attention_tc((const __half*)q, l, (const __half*)k, (const __half*)v, lt, p + l, ta,
                                             (l + 127) / 128, (cudaStream_t)stream),
                     "sd_attention");
  }
  return op_result(sd::launch_attention((const __half*)q, (const __half*)k, (const __half*)v, (const __half*)gate, gstride, goff,
                                        gstep, (__half*)out, l, p, lt, hq, hk, hd, 1, nullptr, 0, (cudaStream_t)stream),
                   "sd_attention");
}

int sd_attention_batch(const void* q, const void* k, const void* v, const void* gate, int32_t gstride, int32_t goff,
                       int32_t gstep, void* out, int32_t batch, int32_t l, int32_t p, int32_t lt, int32_t hq, int32_t hk,
                       int32_t hd, void* stream) {
  if (!q || !k || !v || !out || batch < 1 || l <= 0 || p < 0 || p + l > lt || hk <= 0 || hq % hk) {
    set_global_error("sd_attention_batch: bad arguments");
    return SD_ERR_INVALID;
  }
  if (l < 128 || hd != 256) {  // the mma.sync kernel, one sequence at a time
    for (int b = 0; b < batch; b++) {
      const size_t qo = (size_t)b * hq * l * hd, ko = (size_t)b * hk * lt * hd, go = (size_t)b * l * gstride,
                   oo = (size_t)b * l * hq * hd;
      const int rc = op_result(sd::launch_attention((const __half*)q + qo, (const __half*)k + ko, (const __half*)v + ko,
                                                    gate ? (const __half*)gate + go : nullptr, gstride, goff, gstep,
                                                    (__half*)out + oo, l, p, lt, hq, hk, hd, 1, nullptr, 0, (cudaStream_t)stream),
                               "sd_attention_batch");
      if (rc != SD_OK) return rc;
    }
    return SD_OK;
  }
  sd::AttnTcArgs ta;
  ta.l = l, ta.p = p, ta.hq = hq, ta.hk = hk, ta.batch = batch, ta.gate = (const __half*)gate, ta.gstride = gstride,
  ta.goff = goff, ta.gstep = gstep, ta.out = (__half*)out;
  return op_result(sd::launch_attention_tc((const __half*)q, l, (const __half*)k, (const __half*)v, lt, p + l, ta,
                                           (l + 127) / 128, (cudaStream_t)stream),
                   "sd_attention_batch");
}

int sd_attention_split(const void* q, const void* k, const void* v, const void* gate, int32_t gstride, int32_t goff,
                       int32_t gstep, void* out, int32_t l, int32_t p, int32_t lt, int32_t hq, int32_t hk, int32_t hd,
                       int32_t splits, void* ws, size_t ws_bytes, void* stream) {
  if (!q || !k || !v || !out || l <= 0 || p < 0 || p + l > lt || hk <= 0 || hq % hk || splits < 0 || (size_t)ws % 16) {
    set_global_error("sd_attention_split: bad arguments");
    return SD_ERR_INVALID;
  }
  if (splits == 0) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    splits = sd::attention_splits(l, p, hq, sms);
  }
  if (splits > 1 && (!ws || ws_bytes < sd::attention_split_bytes(l, hq, splits))) {
    char msg[160];
    snprintf(msg, sizeof msg, "sd_attention_split: the workspace needs %zu bytes for %d splits",
             sd::attention_split_bytes(l, hq, splits), (int)splits);
    set_global_error(msg);
    return SD_ERR_INVALID;
  }
  return op_result(sd::launch_attention((const __half*)q, (const __half*)k, (const __half*)v, (const __half*)gate, gstride, goff,
                                        gstep, (__half*)out, l, p, lt, hq, hk, hd, splits, (float*)ws, ws_bytes,
                                        (cudaStream_t)stream),
                   "sd_attention_split");
}

int sd_gdn(const void* q, const void* k, int32_t qk_stride, const void* v, int32_t v_stride, const void* beta,
           const void* g, void* state, int32_t load_state, void* o, int32_t l, int32_t h, int32_t batch, int64_t seq_qk,
           int64_t seq_v, int32_t in_f16, int32_t algo, void* scratch, size_t scratch_bytes, void* stream) {
  const size_t align = in_f16 ? 8 : 16;
  if (!q || !k || !v || !beta || !g || !state || !o || l <= 0 || h <= 0 || batch <= 0 || qk_stride % 4 ||
      (size_t)q % align || (size_t)k % align || algo < 0 || algo > 3 || (algo == 1 && (in_f16 || batch != 1)) ||
      (algo == 2 && (!in_f16 || batch != 1 || !scratch || scratch_bytes < sd::gdn_two_phase_scratch(l, h))) ||
      (algo == 3 && !in_f16)) {
    set_global_error("sd_gdn: bad arguments");
    return SD_ERR_INVALID;
  }
  cudaStream_t st = (cudaStream_t)stream;
  if (algo == 0 && in_f16) {
    // the fused tcgen05 scan: its TMA reads need 16-byte aligned rows and sequences
    if ((size_t)v % 16 || (size_t)q % 16 || (size_t)k % 16 || (size_t)o % 16 || qk_stride % 8 || v_stride % 8 || seq_qk % 8 ||
        seq_v % 8 || (batch > 1 && (seq_qk < (int64_t)l * qk_stride || seq_v < (int64_t)l * v_stride))) {
      set_global_error("sd_gdn: the tcgen05 scan needs 16-byte aligned q/k/v/o, strides that are multiples of 8 elements "
                       "and sequences that do not overlap");
      return SD_ERR_INVALID;
    }
    sd::GdnTcArgs a;
    a.beta = (const float*)beta, a.g = (const float*)g, a.o = (float*)o, a.h = h, a.l = l;
    a.state = (float*)state, a.load_state = load_state != 0, a.store_state = 1;
    return op_result(sd::launch_gdn_tc((const __half*)q, (const __half*)k, qk_stride, (const __half*)v, v_stride,
                                       batch > 1 ? seq_qk : (int64_t)l * qk_stride, batch > 1 ? seq_v : (int64_t)l * v_stride,
                                       l, a, batch * h, st),
                     "sd_gdn");
  }
  if (algo == 1)
    return op_result(sd::launch_gdn_recurrent((const float*)q, (const float*)k, qk_stride, (const float*)v, v_stride,
                                              (const float*)beta, (const float*)g, (float*)state, load_state != 0, (float*)o,
                                              l, h, st),
                     "sd_gdn");
  if (algo == 2)
    return op_result(sd::launch_gdn_two_phase((const __half*)q, (const __half*)k, qk_stride, (const __half*)v, v_stride,
                                              (const float*)beta, (const float*)g, (float*)state, load_state != 0, (float*)o,
                                              l, h, scratch, scratch_bytes, st),
                     "sd_gdn");
  return op_result(sd::launch_gdn_chunked(q, k, qk_stride, v, v_stride, seq_qk, seq_v, in_f16 != 0, (const float*)beta,
                                          (const float*)g, (float*)state, load_state != 0, (float*)o, l, h, batch, st),
                   "sd_gdn");
}

size_t sd_gdn_scratch_bytes(int32_t l, int32_t h) { return l > 0 && h > 0 ? sd::gdn_two_phase_scratch(l, h) : 0; }

int sd_qweight_create(const void* q, const void* s, int32_t n, int32_t k, int32_t interleave, sd_qweight** out) {
  return sd_qweight_create_format(q, s, nullptr, n, k, 4, 32, interleave, out);
}

int sd_qweight_create_format(const void* q, const void* s, const void* b, int32_t n, int32_t k, int32_t bits, int32_t group,
                             int32_t interleave, sd_qweight** out) {
  if (!q || !s || !out || n <= 0 || k <= 0 || k % 64 || (interleave && n % 2) || bits < 2 || bits > 4 || group < 32 ||
      group % 32) {
    set_global_error("sd_qweight_create: bad arguments (k a multiple of 64; bits 2, 3 or 4; group a multiple of 32)");
    return SD_ERR_INVALID;
  }
  auto w = std::make_unique<sd_qweight>();
  cudaGetDevice(&w->device);
  cudaError_t ce = sd::repack_weight((const uint8_t*)q, (const __half*)s, n, k, interleave != 0, &w->w, nullptr, bits, group,
                                     (const __half*)b);
  if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
  if (ce != cudaSuccess) return op_result(ce, "sd_qweight_create");
  *out = w.release();
  return SD_OK;
}

void sd_qweight_free(sd_qweight* w) {
  if (!w) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(w->device);
  cudaFree(w->w.tiles);
  cudaSetDevice(prev);
  delete w;
}

// sd_matmul's error word on device `dev` (allocated by the first sd_matmul there, `create`; never
// freed: one int per device)
static int* matmul_err_word(int dev, bool create) {
  static int* word[sd::kMaxDevices] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  if (create && !word[dev] && cudaMalloc(&word[dev], sizeof(int)) == cudaSuccess) cudaMemset(word[dev], 0, sizeof(int));
  return word[dev];
}

int sd_matmul_ex(const sd_qweight* w, const void* act, int32_t m, void* y, int32_t ldy, int32_t silu, void* x, void* ws,
                 size_t ws_bytes, int32_t algo, void* stream) {
  if (!w || !act || (!y && !x) || m <= 0 || (silu && !w->w.interleaved) || (x && silu) || algo < 0 || algo > 2) {
    set_global_error("sd_matmul: bad arguments");
    return SD_ERR_INVALID;
  }
  // the epilogue stores 16-byte vectors: 16-byte aligned buffers, rows of whole vectors
  const int nout = silu ? w->w.n / 2 : w->w.n;
  if (ldy < nout || ldy % 8 || w->w.n % 8 || (silu && w->w.n % 32) || ((uintptr_t)act | (uintptr_t)y | (uintptr_t)x) % 16 ||
      (uintptr_t)ws % 16) {
    set_global_error("sd_matmul: ldy must be >= the output width and a multiple of 8, n a multiple of 8 (32 with "
                     "silu), and act, y, x and ws 16-byte aligned");
    return SD_ERR_INVALID;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= sd::kMaxDevices) return op_result(cudaErrorInvalidDevice, "sd_matmul");
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (algo == 2) {
    int nt, sp, kts;
    if (!sd::gemm_small_plan(w->w, m, sms, &nt, &sp, &kts)) {
      set_global_error("sd_matmul: the small-M kernel takes up to 256 tokens and k a multiple of 128");
      return SD_ERR_INVALID;
    }
  }
  int* err_word = matmul_err_word(dev, true);
  if (!err_word) return op_result(cudaErrorMemoryAllocation, "sd_matmul");
  return op_result(sd::gemm_q4(w->w, (const __half*)act, m, w->w.k, (__half*)y, ldy, silu != 0, (float*)ws, ws_bytes,
                               err_word, sms, (cudaStream_t)stream, nullptr, (float*)x, algo),
                   "sd_matmul");
}

int sd_matmul(const sd_qweight* w, const void* act, int32_t m, void* y, int32_t ldy, int32_t silu, void* ws, size_t ws_bytes,
              void* stream) {
  if (!y) {
    set_global_error("sd_matmul: bad arguments");
    return SD_ERR_INVALID;
  }
  return sd_matmul_ex(w, act, m, y, ldy, silu, nullptr, ws, ws_bytes, 0, stream);
}

int sd_op_status(void* stream) {
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return op_result(e, "sd_op_status");
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return op_result(e, "sd_op_status");
  int codes[3] = {0, 0, 0};
  const char* names[3] = {"sd_gdn (tcgen05 scan)", "sd_attention (tcgen05)", "sd_matmul"};
  if ((e = sd::take_gdn_tc_err(&codes[0])) != cudaSuccess || (e = sd::take_attn_tc_err(&codes[1])) != cudaSuccess)
    return op_result(e, "sd_op_status");
  if (int* w = dev >= 0 && dev < sd::kMaxDevices ? matmul_err_word(dev, false) : nullptr) {
    if ((e = cudaMemcpy(&codes[2], w, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess) return op_result(e, "sd_op_status");
    if (codes[2] != 0 && (e = cudaMemset(w, 0, sizeof(int))) != cudaSuccess) return op_result(e, "sd_op_status");
  }
  for (int i = 0; i < 3; i++)
    if (codes[i] != 0) {
      char msg[256];
      snprintf(msg, sizeof(msg), "%s: a kernel reported error %d (%s)", names[i], codes[i],
               codes[i] == sd::kErrBadShape ? "token id or row out of range" : "a bounded wait ran out");
      set_global_error(msg);
      return SD_ERR_KERNEL;
    }
  return SD_OK;
}

}  // extern "C"
