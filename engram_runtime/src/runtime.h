// Internal types of the engram runtime (the C API is in include/engram_runtime.h).
#pragma once

#include <cstdint>
#include <deque>
#include <string>
#include <unordered_map>
#include <vector>

#include "gguf.h"

namespace me {

struct GpuEngram;  // device copies and scratch (engram_cuda.cu)

struct Engram {
  int32_t layer = -1;
  uint32_t table_size = 0, dim = 0, n_tables = 0;
  int32_t gate = 0;
  int64_t pad_id = 0;
  std::vector<uint32_t> orders;   // [n_tables]
  std::vector<uint64_t> mults;    // [n_tables * max_order]
  std::vector<uint32_t> rows;     // [n_tables]
  std::vector<uint64_t> offs;     // [n_tables] first row of each table in the concatenated tables
  uint64_t total_rows = 0;
  const Tensor* tables = nullptr;  // ne [dim, total_rows]
  const Tensor *key = nullptr, *value = nullptr, *down = nullptr, *up = nullptr;
  const Tensor *q_scale = nullptr, *k_scale = nullptr;
  // fp32 copies of the projections for the CPU path, made on first use
  std::vector<float> key_f, value_f, down_f, up_f, qs_f, ks_f;
  GpuEngram* gpu = nullptr;
  int64_t mem_dim() const { return (int64_t)n_tables * dim; }
};

// CUDA side (engram_cuda.cu); both return an ME_RT_* code
int cuda_available();
int cuda_upload(Engram& e, int64_t n_embd, int device, std::string* err);
int cuda_inject(Engram& e, int64_t n_embd, float* d_hidden, const int32_t* d_rows, const float* d_keep, int64_t n,
                void* stream, std::string* err);
void cuda_release(Engram& e);

}  // namespace me

struct me_rt {
  me::Gguf file;
  std::vector<me::Engram> engrams;
  std::vector<int32_t> canon;
  uint32_t max_order = 0;
  int64_t n_embd = 0;
  std::deque<me::Tensor> bound;  // tensors bound by the caller (me_rt_bind_tensor); stable addresses
};

struct me_rt_hist {
  std::unordered_map<int32_t, std::vector<int32_t>> seqs;  // token by position, -1 = unknown
};
