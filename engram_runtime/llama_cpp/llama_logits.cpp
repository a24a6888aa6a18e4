// Logits of every position of one token sequence through llama.cpp's public API (llama.h), for
// the parity test of the engram bridge (tests/test_llama_cpp.py):
//
//   llama_logits MODEL.gguf TOKENS.i32 N OUT.f32 [UBATCH]
//
// Decodes the N tokens as sequence 0 in ubatches of UBATCH (default N) and writes N x n_vocab
// fp32 logits. Build against a llama.cpp checkout with the bridge applied:
//   g++ -O2 -std=c++17 -I$L/include -I$L/ggml/include llama_logits.cpp \
//       -L$L/build/bin -lllama -lggml -lggml-base -Wl,-rpath,$L/build/bin -o llama_logits
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "llama.h"

static int fail(const char* what) {
  std::fprintf(stderr, "llama_logits: %s\n", what);
  return 1;
}

int main(int argc, char** argv) {
  if (argc < 5) return fail("usage: llama_logits MODEL.gguf TOKENS.i32 N OUT.f32 [UBATCH]");
  const int n = std::atoi(argv[3]);
  const int ub = argc > 5 ? std::atoi(argv[5]) : n;
  if (n <= 0 || ub <= 0) return fail("N and UBATCH must be positive");
  std::vector<llama_token> toks(n);
  FILE* f = std::fopen(argv[2], "rb");
  if (!f || std::fread(toks.data(), sizeof(llama_token), n, f) != (size_t)n) return fail("cannot read the tokens");
  std::fclose(f);

  llama_backend_init();
  llama_model* model = llama_model_load_from_file(argv[1], llama_model_default_params());
  if (!model) return fail("cannot load the model");
  llama_context_params cp = llama_context_default_params();
  cp.n_ctx = n;
  cp.n_batch = n;
  cp.n_ubatch = ub;
  llama_context* ctx = llama_init_from_model(model, cp);
  if (!ctx) return fail("cannot create a context");
  const int n_vocab = llama_vocab_n_tokens(llama_model_get_vocab(model));

  std::vector<float> out((size_t)n * n_vocab);
  for (int a = 0; a < n; a += ub) {
    const int m = a + ub <= n ? ub : n - a;
    llama_batch b = llama_batch_init(m, 0, 1);
    for (int i = 0; i < m; ++i) {
      b.token[i] = toks[a + i];
      b.pos[i] = a + i;
      b.n_seq_id[i] = 1;
      b.seq_id[i][0] = 0;
      b.logits[i] = 1;
    }
    b.n_tokens = m;
    if (llama_decode(ctx, b) != 0) return fail("llama_decode failed");
    for (int i = 0; i < m; ++i) {
      const float* l = llama_get_logits_ith(ctx, i);
      for (int v = 0; v < n_vocab; ++v) out[(size_t)(a + i) * n_vocab + v] = l[v];
    }
    llama_batch_free(b);
  }
  f = std::fopen(argv[4], "wb");
  if (!f || std::fwrite(out.data(), sizeof(float), out.size(), f) != out.size()) return fail("cannot write");
  std::fclose(f);
  llama_free(ctx);
  llama_model_free(model);
  llama_backend_free();
  return 0;
}
