// Engram runtime: GGUF metadata, hashing, token histories and the CPU (fp32) injection.
//
// GGUF layout (kept identical to the reference's llama_cpp/gguf_add_engram.py:85-101, :152-176
// so one file serves both): arrays micro_engram.{layers, table_size, table_rows, dim, n_tables,
// gate, pad_id, table_orders, mults, canon} and the scalar micro_engram.max_order; tensors
// blk.L.engram_kv.mengram_{tables, key, value, down, up} and blk.L.engram_gate.mengram_{q,k}_scale.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "engram_runtime.h"
#include "runtime.h"

using me::Engram;
using me::GType;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

constexpr uint64_t kPrime = 2147483647ull;  // 2^31 - 1
constexpr float kRmsEps = 1.1920928955078125e-07f;  // torch's default rms_norm eps for fp32

// The metadata arrays of every engram, from a GGUF file or from a caller (me_rt_create).
struct Desc {
  std::vector<uint32_t> layers, table_size, dim, n_tables, gate, orders, table_rows;
  std::vector<int32_t> pad_id;
  std::vector<uint64_t> mults;
  bool has_rows = false;
};

int read_file_desc(me_rt* rt, Desc* d) {
  const me::Gguf& f = rt->file;
  std::string err;
  if (!f.array("micro_engram.layers", GType::U32, &d->layers, &err, false) || d->layers.empty())
    return fail(ME_RT_ERR_FORMAT, "no micro_engram metadata in this GGUF");
  if (!f.array("micro_engram.table_size", GType::U32, &d->table_size, &err) ||
      !f.array("micro_engram.dim", GType::U32, &d->dim, &err) ||
      !f.array("micro_engram.n_tables", GType::U32, &d->n_tables, &err) ||
      !f.array("micro_engram.gate", GType::U32, &d->gate, &err) ||
      !f.array("micro_engram.pad_id", GType::I32, &d->pad_id, &err) ||
      !f.array("micro_engram.table_orders", GType::U32, &d->orders, &err) ||
      !f.array("micro_engram.mults", GType::U64, &d->mults, &err) ||
      !f.array("micro_engram.canon", GType::I32, &rt->canon, &err))
    return fail(ME_RT_ERR_FORMAT, "micro_engram: " + err);
  d->has_rows = f.array("micro_engram.table_rows", GType::U32, &d->table_rows, &err, false);
  if (!f.u32("micro_engram.max_order", &rt->max_order))
    return fail(ME_RT_ERR_FORMAT, "micro_engram: missing key micro_engram.max_order");
  return ME_RT_OK;
}

// Validate the metadata and build the engrams (tensors not attached yet).
int build_engrams(me_rt* rt, const Desc& D, int32_t n_layer) {
  const size_t ne = D.layers.size();
  if (ne == 0) return fail(ME_RT_ERR_FORMAT, "no engrams");
  if (D.table_size.size() != ne || D.dim.size() != ne || D.n_tables.size() != ne || D.gate.size() != ne ||
      D.pad_id.size() != ne || rt->canon.empty() || rt->max_order < 1)
    return fail(ME_RT_ERR_FORMAT, "micro_engram metadata is inconsistent");
  for (int32_t c : rt->canon)
    if (c < 0) return fail(ME_RT_ERR_FORMAT, "micro_engram: negative id in the token-merge map");
  size_t t0 = 0;
  for (size_t i = 0; i < ne; ++i) {
    Engram e;
    e.layer = (int32_t)D.layers[i];
    e.table_size = D.table_size[i];
    e.dim = D.dim[i];
    e.n_tables = D.n_tables[i];
    e.gate = (int32_t)D.gate[i];
    e.pad_id = D.pad_id[i];
    const std::string L = "micro_engram layer " + std::to_string(D.layers[i]);
    if (n_layer >= 0 && D.layers[i] >= (uint32_t)n_layer) return fail(ME_RT_ERR_FORMAT, L + " is out of range");
    if (i > 0 && D.layers[i] <= D.layers[i - 1]) return fail(ME_RT_ERR_FORMAT, L + " is out of order");
    if ((!D.has_rows && e.table_size == 0) || e.dim == 0 || e.n_tables == 0 || D.gate[i] > ME_RT_GATE_PLE)
      return fail(ME_RT_ERR_FORMAT, L + ": bad table settings");
    if (D.orders.size() < t0 + e.n_tables || D.mults.size() < (t0 + e.n_tables) * rt->max_order ||
        (D.has_rows && D.table_rows.size() < t0 + e.n_tables))
      return fail(ME_RT_ERR_FORMAT, "micro_engram metadata is inconsistent");
    for (uint32_t k = 0; k < e.n_tables; ++k) {
      const uint32_t r = D.has_rows ? D.table_rows[t0 + k] : e.table_size;
      if (r == 0) return fail(ME_RT_ERR_FORMAT, L + ": table " + std::to_string(k) + " has no rows");
      e.rows.push_back(r);
      e.offs.push_back(e.total_rows);
      e.total_rows += r;
    }
    if (e.total_rows > (uint64_t)INT32_MAX) return fail(ME_RT_ERR_FORMAT, L + ": too many table rows");
    e.orders.assign(D.orders.begin() + t0, D.orders.begin() + t0 + e.n_tables);
    e.mults.assign(D.mults.begin() + t0 * rt->max_order, D.mults.begin() + (t0 + e.n_tables) * rt->max_order);
    for (uint32_t n : e.orders)
      if (n < 1 || n > rt->max_order) return fail(ME_RT_ERR_FORMAT, L + ": bad n-gram order " + std::to_string(n));
    t0 += e.n_tables;
    rt->engrams.push_back(std::move(e));
  }
  return ME_RT_OK;
}

// The expected shape (ne, innermost first) of one engram tensor, or empty if the gate has none.
std::vector<int64_t> expected_shape(const Engram& e, int64_t d, const std::string& which) {
  const int64_t md = e.mem_dim();
  if (which == "tables") return {(int64_t)e.dim, (int64_t)e.total_rows};
  if (e.gate == ME_RT_GATE_PLE) {
    if (which == "down") return {d, md};
    if (which == "up") return {md, d};
    return {};
  }
  if (which == "key" || which == "value") return {md, d};
  if (e.gate == ME_RT_GATE_SCALAR_SQRT && (which == "q_scale" || which == "k_scale")) return {d};
  return {};
}

const me::Tensor** slot(Engram& e, const std::string& which) {
  if (which == "tables") return &e.tables;
  if (which == "key") return &e.key;
  if (which == "value") return &e.value;
  if (which == "down") return &e.down;
  if (which == "up") return &e.up;
  if (which == "q_scale") return &e.q_scale;
  if (which == "k_scale") return &e.k_scale;
  return nullptr;
}

const char* kTensorNames[] = {"tables", "key", "value", "down", "up", "q_scale", "k_scale"};

int check_tensor(const Engram& e, int64_t d, const std::string& which, const me::Tensor* t) {
  const std::string L = "micro_engram layer " + std::to_string(e.layer);
  const auto want = expected_shape(e, d, which);
  if (want.empty()) return ME_RT_OK;
  if (!t || t->ne != want) return fail(ME_RT_ERR_FORMAT, L + ": tensor " + which + " missing or of the wrong shape");
  if (!t->nbytes) return fail(ME_RT_ERR_FORMAT, L + ": tensor " + which + " is not F32/F16/BF16");
  return ME_RT_OK;
}

int attach_file_tensors(me_rt* rt) {
  for (Engram& e : rt->engrams) {
    const std::string kv = "blk." + std::to_string(e.layer) + ".engram_kv.mengram_";
    const std::string gv = "blk." + std::to_string(e.layer) + ".engram_gate.mengram_";
    for (const char* w : kTensorNames) {
      if (expected_shape(e, rt->n_embd, w).empty()) continue;
      const bool vec = std::string(w) == "q_scale" || std::string(w) == "k_scale";
      const me::Tensor* t = rt->file.tensor((vec ? gv : kv) + w);
      if (int rc = check_tensor(e, rt->n_embd, w, t)) return rc;
      *slot(e, w) = t;
    }
  }
  return ME_RT_OK;
}

bool tensors_ready(const Engram& e, int64_t d) {
  for (const char* w : kTensorNames) {
    if (expected_shape(e, d, w).empty()) continue;
    if (!*slot(const_cast<Engram&>(e), w)) return false;
  }
  return true;
}

void gather_row(const Engram& e, int64_t row, float* out) {
  const me::Tensor* t = e.tables;
  if (t->type == me::GGML_F32) {
    std::memcpy(out, reinterpret_cast<const float*>(t->data) + row * e.dim, e.dim * 4);
    return;
  }
  if (t->type == me::GGML_BF16) {  // bf16 is the top half of an fp32
    const uint16_t* src = reinterpret_cast<const uint16_t*>(t->data) + row * e.dim;
    for (uint32_t i = 0; i < e.dim; ++i) {
      const uint32_t bits = (uint32_t)src[i] << 16;
      std::memcpy(out + i, &bits, 4);
    }
    return;
  }
  me::Tensor v = *t;
  v.data = t->data + (size_t)row * e.dim * 2;
  v.ne = {(int64_t)e.dim};
  std::vector<float> tmp;
  me::tensor_to_f32(v, &tmp);
  std::memcpy(out, tmp.data(), e.dim * 4);
}

void ensure_f32(const me::Tensor* t, std::vector<float>* out) {
  if (t && out->empty()) me::tensor_to_f32(*t, out);
}

// y[r] = sum_i W[r, i] x[i] with W row-major [rows, cols]
void matvec(const std::vector<float>& W, int64_t rows, int64_t cols, const float* x, float* y) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* w = W.data() + r * cols;
    double acc = 0;
    for (int64_t i = 0; i < cols; ++i) acc += (double)w[i] * x[i];
    y[r] = (float)acc;
  }
}

void rms(const float* x, int64_t n, float* y) {
  double ss = 0;
  for (int64_t i = 0; i < n; ++i) ss += (double)x[i] * x[i];
  const float r = 1.0f / std::sqrt((float)(ss / n) + kRmsEps);
  for (int64_t i = 0; i < n; ++i) y[i] = x[i] * r;
}

}  // namespace

extern "C" {

const char* me_rt_last_error(void) { return g_err.c_str(); }

int me_rt_open(const char* path, int32_t n_layer_hint, me_rt** out) {
  if (!path || !out) return fail(ME_RT_ERR_ARG, "null argument");
  auto rt = std::make_unique<me_rt>();
  std::string err;
  if (!rt->file.open(path, &err)) return fail(ME_RT_ERR_IO, err);
  std::string arch;
  if (const me::KV* a = rt->file.find("general.architecture"); a && a->type == GType::STR) arch = a->strs[0];
  uint32_t v = 0;
  if (!rt->file.u32(arch + ".embedding_length", &v) || v == 0)
    return fail(ME_RT_ERR_FORMAT, "missing " + arch + ".embedding_length");
  rt->n_embd = v;
  int32_t n_layer = n_layer_hint;
  if (n_layer < 0 && rt->file.u32(arch + ".block_count", &v)) n_layer = (int32_t)v;
  Desc desc;
  if (int rc = read_file_desc(rt.get(), &desc)) return rc;
  if (int rc = build_engrams(rt.get(), desc, n_layer)) return rc;
  if (int rc = attach_file_tensors(rt.get())) return rc;
  *out = rt.release();
  return ME_RT_OK;
}

int me_rt_create(const me_rt_desc* desc, me_rt** out) {
  if (!desc || !out || desc->n_engrams <= 0 || desc->n_embd <= 0) return fail(ME_RT_ERR_ARG, "bad runtime description");
  auto rt = std::make_unique<me_rt>();
  const size_t n = (size_t)desc->n_engrams;
  auto take = [](auto* p, size_t k, auto* v) {
    if (p) v->assign(p, p + k);
  };
  Desc D;
  take(desc->layers, n, &D.layers);
  take(desc->table_size, n, &D.table_size);
  take(desc->dim, n, &D.dim);
  take(desc->n_tables, n, &D.n_tables);
  take(desc->gate, n, &D.gate);
  take(desc->pad_id, n, &D.pad_id);
  take(desc->table_orders, (size_t)std::max<int64_t>(desc->n_table_orders, 0), &D.orders);
  take(desc->mults, (size_t)std::max<int64_t>(desc->n_mults, 0), &D.mults);
  D.has_rows = desc->table_rows != nullptr;
  take(desc->table_rows, (size_t)std::max<int64_t>(desc->n_table_rows, 0), &D.table_rows);
  take(desc->canon, (size_t)std::max<int64_t>(desc->n_canon, 0), &rt->canon);
  rt->max_order = desc->max_order;
  rt->n_embd = desc->n_embd;
  if (int rc = build_engrams(rt.get(), D, desc->n_layer)) return rc;
  *out = rt.release();
  return ME_RT_OK;
}

int me_rt_bind_tensor(me_rt* rt, int32_t ei, const char* which, const void* data, uint32_t ggml_type,
                      const int64_t* ne, int32_t n_dims) {
  if (!rt || ei < 0 || ei >= (int32_t)rt->engrams.size() || !which || !data || !ne || n_dims < 1 || n_dims > 4)
    return fail(ME_RT_ERR_ARG, "bad bind arguments");
  Engram& e = rt->engrams[ei];
  const me::Tensor** dst = slot(e, which);
  if (!dst) return fail(ME_RT_ERR_ARG, std::string("unknown engram tensor ") + which);
  me::Tensor t;
  t.name = which;
  t.ne.assign(ne, ne + n_dims);
  while (t.ne.size() > 1 && t.ne.back() == 1) t.ne.pop_back();  // ggml pads shapes with 1s
  t.type = ggml_type;
  t.data = static_cast<const uint8_t*>(data);
  int64_t numel = 1;
  for (int64_t v : t.ne) numel *= v;
  const uint64_t es = ggml_type == me::GGML_F32 ? 4 : (ggml_type == me::GGML_F16 || ggml_type == me::GGML_BF16) ? 2 : 0;
  t.nbytes = es * (uint64_t)numel;
  if (int rc = check_tensor(e, rt->n_embd, which, &t)) return rc;
  rt->bound.push_back(std::move(t));
  *dst = &rt->bound.back();
  // a re-bound tensor invalidates the fp32 copies and the device upload
  e.key_f.clear(); e.value_f.clear(); e.down_f.clear(); e.up_f.clear(); e.qs_f.clear(); e.ks_f.clear();
  me::cuda_release(e);
  return ME_RT_OK;
}

void me_rt_close(me_rt* rt) {
  if (!rt) return;
  for (auto& e : rt->engrams) me::cuda_release(e);
  delete rt;
}

int32_t me_rt_n_engrams(const me_rt* rt) { return rt ? (int32_t)rt->engrams.size() : 0; }
int32_t me_rt_max_order(const me_rt* rt) { return rt ? (int32_t)rt->max_order : 0; }
int64_t me_rt_n_embd(const me_rt* rt) { return rt ? rt->n_embd : 0; }

int me_rt_engram_info(const me_rt* rt, int32_t e, int32_t* layer, int32_t* gate, int32_t* n_tables, int32_t* dim,
                      int64_t* total_rows) {
  if (!rt || e < 0 || e >= (int32_t)rt->engrams.size()) return fail(ME_RT_ERR_ARG, "no such engram");
  const Engram& g = rt->engrams[e];
  if (layer) *layer = g.layer;
  if (gate) *gate = g.gate;
  if (n_tables) *n_tables = (int32_t)g.n_tables;
  if (dim) *dim = (int32_t)g.dim;
  if (total_rows) *total_rows = (int64_t)g.total_rows;
  return ME_RT_OK;
}

int32_t me_rt_engram_at_layer(const me_rt* rt, int32_t layer) {
  if (!rt) return -1;
  for (size_t i = 0; i < rt->engrams.size(); ++i)
    if (rt->engrams[i].layer == layer) return (int32_t)i;
  return -1;
}

int me_rt_hash(const me_rt* rt, int32_t ei, const int32_t* tokens, const int32_t* prev, int64_t n, int32_t* rows) {
  if (!rt || ei < 0 || ei >= (int32_t)rt->engrams.size() || (n > 0 && (!tokens || !rows)) ||
      (n > 0 && rt->max_order > 1 && !prev))
    return fail(ME_RT_ERR_ARG, "bad hash arguments");
  const Engram& e = rt->engrams[ei];
  const int64_t nc = (int64_t)rt->canon.size();
  const uint32_t np = rt->max_order - 1;
  auto canon_of = [&](int64_t t) -> uint64_t { return (uint64_t)rt->canon[std::clamp<int64_t>(t, 0, nc - 1)]; };
  std::vector<uint64_t> toks(rt->max_order);
  for (int64_t i = 0; i < n; ++i) {
    toks[0] = tokens[i] < 0 ? (uint64_t)e.pad_id : canon_of(tokens[i]);
    for (uint32_t s = 1; s < rt->max_order; ++s) {
      const int32_t t = prev[(size_t)i * np + (np - s)];
      toks[s] = t < 0 ? (uint64_t)e.pad_id : canon_of(t);
    }
    for (uint32_t k = 0; k < e.n_tables; ++k) {
      uint64_t x = 0;  // ids and multipliers are below 2^31: every term and the sum fit in 64 bits
      for (uint32_t s = 0; s < e.orders[k]; ++s) x += toks[s] * e.mults[(size_t)k * rt->max_order + s];
      rows[i * e.n_tables + k] = (int32_t)(e.offs[k] + (x % kPrime) % e.rows[k]);
    }
  }
  return ME_RT_OK;
}

// ------------------------------------------------------------------ histories
int me_rt_hist_new(me_rt_hist** out) {
  if (!out) return fail(ME_RT_ERR_ARG, "null argument");
  *out = new me_rt_hist();
  return ME_RT_OK;
}

void me_rt_hist_free(me_rt_hist* h) { delete h; }

int me_rt_hist_set(me_rt_hist* h, int32_t seq, int64_t pos, int32_t tok) {
  if (!h || pos < 0) return fail(ME_RT_ERR_ARG, "bad history position");
  auto& v = h->seqs[seq];
  if ((int64_t)v.size() <= pos) v.resize((size_t)pos + 1, -1);
  v[(size_t)pos] = tok;
  return ME_RT_OK;
}

int me_rt_hist_remove(me_rt_hist* h, int32_t seq, int64_t p0, int64_t p1) {
  if (!h) return fail(ME_RT_ERR_ARG, "null history");
  auto cut = [&](std::vector<int32_t>& v) {
    const int64_t a = std::max<int64_t>(p0, 0);
    const int64_t b = p1 < 0 ? (int64_t)v.size() : std::min<int64_t>(p1, (int64_t)v.size());
    for (int64_t p = a; p < b; ++p) v[(size_t)p] = -1;
    while (!v.empty() && v.back() < 0) v.pop_back();
  };
  if (seq < 0) {
    for (auto& kv : h->seqs) cut(kv.second);
  } else if (auto it = h->seqs.find(seq); it != h->seqs.end()) {
    cut(it->second);
  }
  return ME_RT_OK;
}

int me_rt_hist_copy(me_rt_hist* h, int32_t src, int32_t dst) {
  if (!h) return fail(ME_RT_ERR_ARG, "null history");
  auto it = h->seqs.find(src);
  h->seqs[dst] = it == h->seqs.end() ? std::vector<int32_t>() : it->second;
  return ME_RT_OK;
}

int me_rt_hist_prev(const me_rt_hist* h, const int32_t* seq, const int64_t* pos, int64_t n, int32_t n_prev,
                    int32_t* prev) {
  if (!h || n_prev < 0 || (n > 0 && n_prev > 0 && (!seq || !pos || !prev))) return fail(ME_RT_ERR_ARG, "bad args");
  for (int64_t i = 0; i < n; ++i) {
    auto it = h->seqs.find(seq[i]);
    for (int32_t s = 1; s <= n_prev; ++s) {
      const int64_t p = pos[i] - s;
      int32_t t = -1;
      if (it != h->seqs.end() && p >= 0 && p < (int64_t)it->second.size()) t = it->second[(size_t)p];
      prev[(size_t)i * n_prev + (n_prev - s)] = t;
    }
  }
  return ME_RT_OK;
}

int me_rt_hist_save(const me_rt_hist* h, int32_t seq, void* buf, size_t* size) {
  if (!h || !size) return fail(ME_RT_ERR_ARG, "null argument");
  auto it = h->seqs.find(seq);
  const uint64_t n = it == h->seqs.end() ? 0 : it->second.size();
  const size_t need = 16 + n * 4;
  if (!buf) {
    *size = need;
    return ME_RT_OK;
  }
  if (*size < need) return fail(ME_RT_ERR_ARG, "buffer too small");
  uint8_t* p = static_cast<uint8_t*>(buf);
  const uint32_t magic = 0x5348454du, version = 1;  // "MEHS"
  std::memcpy(p, &magic, 4);
  std::memcpy(p + 4, &version, 4);
  std::memcpy(p + 8, &n, 8);
  if (n) std::memcpy(p + 16, it->second.data(), n * 4);
  *size = need;
  return ME_RT_OK;
}

int me_rt_hist_load(me_rt_hist* h, int32_t seq, const void* buf, size_t size) {
  if (!h || !buf || size < 16) return fail(ME_RT_ERR_STATE, "history state too short");
  const uint8_t* p = static_cast<const uint8_t*>(buf);
  uint32_t magic, version;
  uint64_t n;
  std::memcpy(&magic, p, 4);
  std::memcpy(&version, p + 4, 4);
  std::memcpy(&n, p + 8, 8);
  if (magic != 0x5348454du || version != 1 || size != 16 + n * 4)
    return fail(ME_RT_ERR_STATE, "not an engram history state");
  auto& v = h->seqs[seq];
  v.resize((size_t)n);
  if (n) std::memcpy(v.data(), p + 16, n * 4);
  return ME_RT_OK;
}

// ------------------------------------------------------------------ injection (CPU, fp32)
}  // extern "C"

namespace {

// One position: gather its rows, then the gate and the residual add into x (fp32 weights, double
// accumulation). Positions are independent, so any split over threads gives the same bits.
void inject_position(const Engram& e, int64_t d, const int32_t* rows, float* x, float kp, std::vector<float>& mem,
                     std::vector<float>& h, std::vector<float>& a, std::vector<float>& b) {
  const int64_t md = e.mem_dim();
  for (uint32_t k = 0; k < e.n_tables; ++k) gather_row(e, rows[k], mem.data() + (size_t)k * e.dim);
  rms(x, d, h.data());
  if (e.gate == ME_RT_GATE_PLE) {
    matvec(e.down_f, md, d, h.data(), a.data());  // down: [mem_dim, d]
    for (int64_t i = 0; i < md; ++i) {
      const float z = a[i];
      const float g = 0.5f * z * (1.0f + std::tanh(0.7978845608028654f * (z + 0.044715f * z * z * z)));
      a[i] = g * mem[i];
    }
    matvec(e.up_f, d, md, a.data(), b.data());  // up: [d, mem_dim]
    for (int64_t j = 0; j < d; ++j) x[j] += b[j] * kp;
    return;
  }
  matvec(e.key_f, d, md, mem.data(), a.data());
  rms(a.data(), d, a.data());
  double s = 0;
  for (int64_t j = 0; j < d; ++j) {
    const double qh = e.qs_f.empty() ? h[j] : h[j] * e.qs_f[j];
    const double kk = e.ks_f.empty() ? a[j] : a[j] * e.ks_f[j];
    s += qh * kk;
  }
  float sc = (float)(s / std::sqrt((double)d));
  if (e.gate == ME_RT_GATE_SCALAR_SQRT) {
    const float sg = sc > 0 ? 1.f : (sc < 0 ? -1.f : 0.f);
    sc = sg * std::sqrt(std::max(std::fabs(sc), 1e-6f));
  }
  const float alpha = 1.0f / (1.0f + std::exp(-sc));
  matvec(e.value_f, d, md, mem.data(), b.data());
  for (int64_t j = 0; j < d; ++j) x[j] += alpha * b[j] * kp;
}

// Worker threads for n positions: ME_RT_THREADS, else the machine's hardware threads, with at
// least 4 positions per thread (a decode step of one token stays on the calling thread).
int64_t worker_count(int64_t n) {
  int64_t want = 0;
  if (const char* env = std::getenv("ME_RT_THREADS")) want = std::atoll(env);
  if (want <= 0) want = std::max(1u, std::thread::hardware_concurrency());
  return std::max<int64_t>(1, std::min<int64_t>(want, n / 4));
}

}  // namespace

extern "C" {

int me_rt_inject_cpu(const me_rt* crt, int32_t ei, float* hidden, const int32_t* rows, const float* keep, int64_t n) {
  me_rt* rt = const_cast<me_rt*>(crt);  // lazily made fp32 copies only
  if (!rt || ei < 0 || ei >= (int32_t)rt->engrams.size() || (n > 0 && (!hidden || !rows)))
    return fail(ME_RT_ERR_ARG, "bad inject arguments");
  Engram& e = rt->engrams[ei];
  if (!tensors_ready(e, rt->n_embd)) return fail(ME_RT_ERR_STATE, "engram tensors are not bound");
  const int64_t d = rt->n_embd, md = e.mem_dim();
  if (e.gate == ME_RT_GATE_PLE) {
    ensure_f32(e.down, &e.down_f);
    ensure_f32(e.up, &e.up_f);
  } else {
    ensure_f32(e.key, &e.key_f);
    ensure_f32(e.value, &e.value_f);
    ensure_f32(e.q_scale, &e.qs_f);
    ensure_f32(e.k_scale, &e.ks_f);
  }
  for (int64_t i = 0; i < n * (int64_t)e.n_tables; ++i)  // checked up front: the workers cannot fail
    if (rows[i] < 0 || (uint64_t)rows[i] >= e.total_rows) return fail(ME_RT_ERR_ARG, "row index out of range");
  auto run = [&](int64_t t0, int64_t t1) {
    std::vector<float> mem(md), h(d), a(std::max(d, md)), b(std::max(d, md));
    for (int64_t t = t0; t < t1; ++t)
      inject_position(e, d, rows + t * e.n_tables, hidden + t * d, keep ? keep[t] : 1.0f, mem, h, a, b);
  };
  const int64_t workers = worker_count(n);
  if (workers == 1) {
    run(0, n);
    return ME_RT_OK;
  }
  std::vector<std::thread> pool;
  const int64_t per = (n + workers - 1) / workers;
  for (int64_t t0 = per; t0 < n; t0 += per) pool.emplace_back(run, t0, std::min(n, t0 + per));
  run(0, std::min(n, per));
  for (auto& th : pool) th.join();
  return ME_RT_OK;
}

// ------------------------------------------------------------------ GPU entry points
int me_rt_cuda_available(void) { return me::cuda_available(); }

int me_rt_cuda_upload(me_rt* rt, int32_t ei, int32_t device) {
  if (!rt || ei < 0 || ei >= (int32_t)rt->engrams.size()) return fail(ME_RT_ERR_ARG, "no such engram");
  if (!tensors_ready(rt->engrams[ei], rt->n_embd)) return fail(ME_RT_ERR_STATE, "engram tensors are not bound");
  std::string err;
  const int rc = me::cuda_upload(rt->engrams[ei], rt->n_embd, device, &err);
  return rc == ME_RT_OK ? rc : fail(rc, err);
}

int me_rt_cuda_inject(me_rt* rt, int32_t ei, float* d_hidden, const int32_t* d_rows, const float* d_keep, int64_t n,
                      void* stream) {
  if (!rt || ei < 0 || ei >= (int32_t)rt->engrams.size()) return fail(ME_RT_ERR_ARG, "no such engram");
  std::string err;
  const int rc = me::cuda_inject(rt->engrams[ei], rt->n_embd, d_hidden, d_rows, d_keep, n, stream, &err);
  return rc == ME_RT_OK ? rc : fail(rc, err);
}

}  // extern "C"
