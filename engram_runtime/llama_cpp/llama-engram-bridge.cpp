// llama.cpp <-> engram runtime bridge; see llama-engram-bridge.h for the hook points.
#include "llama-engram-bridge.h"

#include "llama-batch.h"
#include "llama-graph.h"
#include "llama-impl.h"
#include "llama-kv-cache.h"
#include "llama-kv-cache-iswa.h"

#include "ggml.h"
#include "ggml-backend.h"
#include "gguf.h"

#include <cstring>
#include <stdexcept>
#include <string>

namespace {

template <typename T>
bool gguf_array(const gguf_context* meta, const char* key, gguf_type type, std::vector<T>& out, bool required) {
  const int64_t id = gguf_find_key(meta, key);
  if (id < 0) {
    if (required) throw std::runtime_error(std::string("micro_engram: missing key ") + key);
    return false;
  }
  if (gguf_get_kv_type(meta, id) != GGUF_TYPE_ARRAY || gguf_get_arr_type(meta, id) != type)
    throw std::runtime_error(std::string("micro_engram: key ") + key + " has the wrong type");
  const T* p = static_cast<const T*>(gguf_get_arr_data(meta, id));
  out.assign(p, p + gguf_get_arr_n(meta, id));
  return true;
}

const llama_kv_cache_context* kv_base(const llama_memory_context_i* m) {
  if (auto* c = dynamic_cast<const llama_kv_cache_iswa_context*>(m)) return c->get_base();
  return dynamic_cast<const llama_kv_cache_context*>(m);
}

}  // namespace

llama_engram_bridge::~llama_engram_bridge() {
  if (rt) me_rt_close(rt);
}

bool llama_engram_bridge::load(const gguf_context* meta, int64_t n_embd, int32_t n_layer) {
  std::vector<uint32_t> layers;
  if (!gguf_array(meta, "micro_engram.layers", GGUF_TYPE_UINT32, layers, false) || layers.empty()) return false;
  std::vector<uint32_t> table_size, dim, n_tables, gate, orders, rows;
  std::vector<int32_t> pad_id, canon;
  std::vector<uint64_t> mults;
  gguf_array(meta, "micro_engram.table_size", GGUF_TYPE_UINT32, table_size, true);
  gguf_array(meta, "micro_engram.dim", GGUF_TYPE_UINT32, dim, true);
  gguf_array(meta, "micro_engram.n_tables", GGUF_TYPE_UINT32, n_tables, true);
  gguf_array(meta, "micro_engram.gate", GGUF_TYPE_UINT32, gate, true);
  gguf_array(meta, "micro_engram.pad_id", GGUF_TYPE_INT32, pad_id, true);
  gguf_array(meta, "micro_engram.table_orders", GGUF_TYPE_UINT32, orders, true);
  gguf_array(meta, "micro_engram.mults", GGUF_TYPE_UINT64, mults, true);
  gguf_array(meta, "micro_engram.canon", GGUF_TYPE_INT32, canon, true);
  const bool has_rows = gguf_array(meta, "micro_engram.table_rows", GGUF_TYPE_UINT32, rows, false);
  const int64_t id = gguf_find_key(meta, "micro_engram.max_order");
  if (id < 0 || gguf_get_kv_type(meta, id) != GGUF_TYPE_UINT32)
    throw std::runtime_error("micro_engram: missing key micro_engram.max_order");
  me_rt_desc d{};
  d.n_engrams = (int32_t)layers.size();
  d.layers = layers.data();
  d.table_size = table_size.size() == layers.size() ? table_size.data() : nullptr;
  d.dim = dim.data();
  d.n_tables = n_tables.data();
  d.gate = gate.data();
  d.pad_id = pad_id.data();
  d.table_orders = orders.data();
  d.n_table_orders = (int64_t)orders.size();
  d.mults = mults.data();
  d.n_mults = (int64_t)mults.size();
  d.table_rows = has_rows ? rows.data() : nullptr;
  d.n_table_rows = (int64_t)rows.size();
  d.canon = canon.data();
  d.n_canon = (int64_t)canon.size();
  d.max_order = gguf_get_val_u32(meta, id);
  d.n_embd = n_embd;
  d.n_layer = n_layer;
  if (dim.size() != layers.size() || n_tables.size() != layers.size() || gate.size() != layers.size() ||
      pad_id.size() != layers.size() || !d.table_size)
    throw std::runtime_error("micro_engram metadata is inconsistent");
  if (me_rt_create(&d, &rt) != ME_RT_OK) throw std::runtime_error(me_rt_last_error());
  max_order = (int32_t)d.max_order;
  LLAMA_LOG_INFO("%s: micro_engram: %zu engram(s), max order %u\n", __func__, layers.size(), d.max_order);
  return true;
}

void llama_engram_bridge::add_tensor(int32_t e, const char* which, ggml_tensor* t) {
  if (t) tensors.push_back({e, which, t});
}

void llama_engram_bridge::bind_all() const {
  if (bound || !rt) return;
  for (const pending& p : tensors) {
    if (!p.t->buffer || !ggml_backend_buffer_is_host(p.t->buffer))
      throw std::runtime_error(std::string("micro_engram: tensor ") + ggml_get_name(p.t) +
                               " is not in host memory; keep the engram tensors on the CPU (-ot \"mengram=CPU\")");
    const int64_t ne[4] = {p.t->ne[0], p.t->ne[1], p.t->ne[2], p.t->ne[3]};
    if (me_rt_bind_tensor(rt, p.e, p.which, p.t->data, (uint32_t)p.t->type, ne, 4) != ME_RT_OK)
      throw std::runtime_error(me_rt_last_error());
  }
  bound = true;
}

struct llama_engram_graph::state {
  const llama_engram_bridge* br = nullptr;
  const llama_memory_context_i* mctx = nullptr;
  int64_t n_tokens = 0;
  bool active = false;
  std::vector<std::vector<int32_t>> rows;  // per engram, [n_tokens * n_tables]

  void fill(const llama_ubatch& ub) {
    active = ub.token != nullptr;
    n_tokens = ub.n_tokens;
    if (!active) return;
    const llama_kv_cache_context* kv = kv_base(mctx);
    GGML_ASSERT(kv != nullptr && "micro_engram needs the KV cache's token history");
    std::vector<llama_token> prev;
    kv->get_prev_tokens(ub, br->max_order - 1, prev);
    std::vector<int32_t> toks(ub.token, ub.token + ub.n_tokens);
    rows.resize(me_rt_n_engrams(br->rt));
    for (int32_t e = 0; e < (int32_t)rows.size(); ++e) {
      int32_t nt = 0;
      me_rt_engram_info(br->rt, e, nullptr, nullptr, &nt, nullptr, nullptr);
      rows[e].resize((size_t)ub.n_tokens * nt);
      if (me_rt_hash(br->rt, e, toks.data(), prev.data(), ub.n_tokens, rows[e].data()) != ME_RT_OK)
        throw std::runtime_error(me_rt_last_error());
    }
  }
};

namespace {

class graph_input_engram : public llm_graph_input_i {
 public:
  explicit graph_input_engram(std::shared_ptr<llama_engram_graph::state> s) : st(std::move(s)) {}
  void set_input(const llama_ubatch* ub) override { st->fill(*ub); }
  std::shared_ptr<llama_engram_graph::state> st;
};

struct op_data {
  std::shared_ptr<llama_engram_graph::state> st;
  int32_t e;
};

// dst = a + engram(a); b (optional): ids of the ubatch tokens the rows of `a` are
void engram_op(ggml_tensor* dst, const ggml_tensor* a, const ggml_tensor* b, int ith, int, void* ud) {
  if (ith != 0) return;
  const op_data* od = static_cast<const op_data*>(ud);
  const int64_t d = a->ne[0], n = a->ne[1];
  std::memcpy(dst->data, a->data, (size_t)n * d * sizeof(float));
  if (!od->st->active) return;
  const auto& all = od->st->rows[od->e];
  const int64_t nt = (int64_t)all.size() / std::max<int64_t>(od->st->n_tokens, 1);
  std::vector<int32_t> rows((size_t)n * nt);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t tok = b ? static_cast<const int32_t*>(b->data)[i] : i;
    std::memcpy(rows.data() + i * nt, all.data() + tok * nt, nt * sizeof(int32_t));
  }
  if (me_rt_inject_cpu(od->st->br->rt, od->e, static_cast<float*>(dst->data), rows.data(), nullptr, n) != ME_RT_OK)
    GGML_ABORT("micro_engram: %s", me_rt_last_error());
}

void op1(ggml_tensor* dst, const ggml_tensor* a, int ith, int nth, void* ud) { engram_op(dst, a, nullptr, ith, nth, ud); }
void op2(ggml_tensor* dst, const ggml_tensor* a, const ggml_tensor* b, int ith, int nth, void* ud) {
  engram_op(dst, a, b, ith, nth, ud);
}

}  // namespace

llama_engram_graph::llama_engram_graph(llm_graph_context& g, const llama_engram_bridge& br) : g(g), br(br) {
  if (!br.enabled()) return;
  br.bind_all();
  st = std::make_shared<state>();
  st->br = &br;
  st->mctx = g.mctx;
  g.res->add_input(std::make_unique<graph_input_engram>(st));
}

ggml_tensor* llama_engram_graph::inject(ggml_tensor* cur, int il, ggml_tensor* out_ids) {
  const int32_t e = br.engram_at(il);
  if (e < 0 || !st) return cur;
  auto* od = new op_data{st, e};  // owned by the graph's lifetime: freed with the graph result below
  struct holder : llm_graph_input_i {
    std::unique_ptr<op_data> p;
    void set_input(const llama_ubatch*) override {}
  };
  auto h = std::make_unique<holder>();
  h->p.reset(od);
  g.res->add_input(std::move(h));
  ggml_tensor* out = cur->ne[1] == g.n_tokens ? ggml_map_custom1(g.ctx0, cur, op1, 1, od)
                                               : ggml_map_custom2(g.ctx0, cur, out_ids, op2, 1, od);
  g.cb(out, "engram_out", il);
  return out;
}
