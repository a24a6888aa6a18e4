// llama.cpp <-> engram runtime bridge (compiled inside llama.cpp's src/ by apply.py).
//
// Hook points in a Gemma 4 model, the same places an engram must sit in any integration:
//   1. load_arch_hparams: the micro_engram.* metadata (read with llama.cpp's gguf API) becomes a
//      runtime (me_rt_create); the KV cache is told to keep token ids (has_cell_ext), which is
//      where the n-gram history comes from, including after seq_rm / seq_cp / state restore.
//   2. load_arch_tensors: the engram tensors are created by llama.cpp's loader under the GGUF
//      names, and bound to the runtime once their data is in host memory.
//   3. graph build, after each layer's scaled output: one custom op adds the engram memory. Its
//      graph input hashes the ubatch's tokens (runtime me_rt_hash on the KV cache's previous
//      tokens) in set_input; the op itself calls me_rt_inject_cpu on the rows it is given.
// The custom op runs on the CPU backend (ggml schedules it there; with GPU offload the layer
// output crosses to host memory and back for the engram layers only).
#pragma once

#include <cstdint>
#include <memory>
#include <vector>

#include "engram_runtime.h"

struct ggml_context;
struct ggml_tensor;
struct gguf_context;
struct llama_ubatch;
struct llm_graph_context;

struct llama_engram_bridge {
  me_rt* rt = nullptr;
  int32_t max_order = 0;
  ~llama_engram_bridge();

  // metadata -> runtime; false when the file has no engram
  bool load(const gguf_context* meta, int64_t n_embd, int32_t n_layer);
  bool enabled() const { return rt != nullptr; }
  int32_t engram_at(int il) const { return rt ? me_rt_engram_at_layer(rt, il) : -1; }
  // remember a tensor created by llama.cpp's loader; its data is bound on first use
  void add_tensor(int32_t e, const char* which, ggml_tensor* t);
  // bind every remembered tensor (needs the weights loaded, in host memory)
  void bind_all() const;

 private:
  struct pending {
    int32_t e;
    const char* which;
    ggml_tensor* t;
  };
  std::vector<pending> tensors;
  mutable bool bound = false;
};

// per-graph part: the rows of every engram for the current ubatch
struct llama_engram_graph {
  llama_engram_graph(llm_graph_context& g, const llama_engram_bridge& br);
  ggml_tensor* inject(ggml_tensor* cur, int il, ggml_tensor* out_ids);

 private:
  llm_graph_context& g;
  const llama_engram_bridge& br;
  struct state;
  std::shared_ptr<state> st;  // shared with the graph input and the custom ops
};
