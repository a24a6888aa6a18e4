// engram_runtime: a standalone C++ runtime for micro-engrams stored in a GGUF file, for
// GGUF/llama.cpp-style serving (no PyTorch). It reads and validates the `micro_engram.*`
// metadata and tensors, hashes token histories exactly like the training hash
// (micro_engram/module.py:183-226 of the reference; its llama.cpp port is
// llama_cpp/src/llama-micro-engram.cpp:150-176), keeps per-sequence token histories
// (the KV cache's token ids: append, rewind, copy, save/restore), and adds the gated memory
// to a layer's hidden states, on the CPU (fp32 oracle) or on an sm_100a GPU (fused kernels).
//
// The C API below is what integrations (the llama.cpp patch, the logit driver, the Python
// tests through ctypes) call. All functions return 0 on success or a negative error code;
// me_rt_last_error() describes the last failure of the calling thread.
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct me_rt me_rt;  // one loaded GGUF: every engram it holds

enum {
  ME_RT_OK = 0,
  ME_RT_ERR_IO = -1,        // file missing / unreadable / not a GGUF
  ME_RT_ERR_FORMAT = -2,    // micro_engram metadata missing or inconsistent
  ME_RT_ERR_ARG = -3,       // bad argument (index, size, null pointer)
  ME_RT_ERR_CUDA = -4,      // a CUDA call failed, or the GPU path is not built
  ME_RT_ERR_STATE = -5,     // history state blob does not match
};

enum { ME_RT_GATE_SCALAR = 0, ME_RT_GATE_SCALAR_SQRT = 1, ME_RT_GATE_PLE = 2 };

// ---------------------------------------------------------------- loading and metadata
int me_rt_open(const char* gguf_path, int32_t n_layer_hint, me_rt** out);  // hint < 0: use <arch>.block_count
void me_rt_close(me_rt* rt);
const char* me_rt_last_error(void);

// A runtime from metadata the caller already parsed (e.g. llama.cpp's own GGUF reader), with
// the tensors bound afterwards from the caller's memory. Arrays follow the GGUF layout above;
// table_rows may be NULL (then table_size rows per table).
typedef struct {
  int32_t n_engrams;
  const uint32_t* layers;
  const uint32_t* table_size;
  const uint32_t* dim;
  const uint32_t* n_tables;
  const uint32_t* gate;
  const int32_t* pad_id;
  const uint32_t* table_orders;
  int64_t n_table_orders;
  const uint64_t* mults;
  int64_t n_mults;
  const uint32_t* table_rows;
  int64_t n_table_rows;
  const int32_t* canon;
  int64_t n_canon;
  uint32_t max_order;
  int64_t n_embd;
  int32_t n_layer;  // < 0: not checked
} me_rt_desc;
int me_rt_create(const me_rt_desc* desc, me_rt** out);
// Bind tensor `which` ("tables", "key", "value", "down", "up", "q_scale", "k_scale") of engram e
// to host memory the caller keeps alive: ggml type F32 (0), F16 (1) or BF16 (30), ne innermost first.
int me_rt_bind_tensor(me_rt* rt, int32_t e, const char* which, const void* data, uint32_t ggml_type,
                      const int64_t* ne, int32_t n_dims);

int32_t me_rt_n_engrams(const me_rt* rt);
int32_t me_rt_max_order(const me_rt* rt);
int64_t me_rt_n_embd(const me_rt* rt);
// layer, gate, n_tables, dim and total table rows of engram e
int me_rt_engram_info(const me_rt* rt, int32_t e, int32_t* layer, int32_t* gate, int32_t* n_tables, int32_t* dim,
                      int64_t* total_rows);
int32_t me_rt_engram_at_layer(const me_rt* rt, int32_t layer);  // engram index, or -1

// ---------------------------------------------------------------- hashing
// Rows to gather for n tokens: rows[i*n_tables + k] = offset of table k + its hashed row.
// tokens[i] is token i (a negative token = an embedding row: hashed as pad_id);
// prev[i*(max_order-1) + (max_order-2-j)] is the token j+1 places before token i (-1 = none),
// i.e. the oldest first, as llama.cpp's get_prev_tokens lays them out.
int me_rt_hash(const me_rt* rt, int32_t e, const int32_t* tokens, const int32_t* prev, int64_t n, int32_t* rows);

// ---------------------------------------------------------------- token histories
typedef struct me_rt_hist me_rt_hist;  // token ids per sequence, by position
int me_rt_hist_new(me_rt_hist** out);
void me_rt_hist_free(me_rt_hist* h);
// token `tok` at position `pos` of sequence `seq` (positions may arrive out of order)
int me_rt_hist_set(me_rt_hist* h, int32_t seq, int64_t pos, int32_t tok);
// forget positions [p0, p1) of a sequence (p1 < 0: to the end); seq < 0: every sequence
int me_rt_hist_remove(me_rt_hist* h, int32_t seq, int64_t p0, int64_t p1);
int me_rt_hist_copy(me_rt_hist* h, int32_t src, int32_t dst);
// previous tokens of n (seq, pos) pairs, laid out for me_rt_hash (-1 where there is none)
int me_rt_hist_prev(const me_rt_hist* h, const int32_t* seq, const int64_t* pos, int64_t n, int32_t n_prev,
                    int32_t* prev);
// serialise one sequence (size query with buf == NULL), and restore it into `seq`
int me_rt_hist_save(const me_rt_hist* h, int32_t seq, void* buf, size_t* size);
int me_rt_hist_load(me_rt_hist* h, int32_t seq, const void* buf, size_t size);

// ---------------------------------------------------------------- injection
// hidden [n, n_embd] fp32 in place: hidden += gated memory of `rows` (from me_rt_hash).
// keep (optional, [n]): 0 = no memory for that row (embedding rows of a mixed batch).
int me_rt_inject_cpu(const me_rt* rt, int32_t e, float* hidden, const int32_t* rows, const float* keep, int64_t n);

// GPU: upload engram e's tensors once (bf16) to `device`, then inject on device memory.
int me_rt_cuda_available(void);
int me_rt_cuda_upload(me_rt* rt, int32_t e, int32_t device);
// d_hidden [n, n_embd] fp32 device memory (in place); d_rows [n*n_tables] int32 device memory;
// d_keep optional [n] fp32 device memory; stream: a cudaStream_t (NULL = default stream).
int me_rt_cuda_inject(me_rt* rt, int32_t e, float* d_hidden, const int32_t* d_rows, const float* d_keep, int64_t n,
                      void* stream);

#ifdef __cplusplus
}
#endif
