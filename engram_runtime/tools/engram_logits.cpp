// Engram output driver for the runtime (the reference's counterpart is
// llama_cpp/test/engram_logits.cpp, which dumps llama.cpp logits; without llama.cpp here the
// driver runs the engram stage itself): it feeds token sequences through the runtime's
// history -> hash -> inject pipeline the way a server would, in one of four modes, and writes
// the injected hidden states for comparison with the PyTorch oracle.
//
//   engram_logits --gguf F --engram E --n-seq S --n-tok T --tokens tok.i32 --hidden h.f32
//                 --mode full|decode|two|state [--ubatch U] [--gpu] --out out.f32
//
// tokens: int32 [S, T]; hidden: fp32 [S, T, n_embd] (the layer's output before the engram);
// out: the same shape after the engram.
//   full    each sequence in ubatches of U tokens (default: all at once)
//   decode  the first token alone, then one token per step
//   two     sequences 0 and 1 interleaved: step i holds token i of both (two sequence ids)
//   state   sequence 0 decoded up to T/2, its history saved, cleared, restored as sequence 7,
//           and the rest decoded there
// ENGRAM_DUMP=1 prints the norm of every injected row (a debugging aid).
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#ifndef ME_RT_NO_CUDA
#include <cuda_runtime.h>
#endif

#include "engram_runtime.h"

namespace {

struct Run {
  me_rt* rt = nullptr;
  me_rt_hist* hist = nullptr;
  int e = 0;
  int64_t d = 0;
  int nt = 0, n_prev = 0;
  bool gpu = false;
  float* d_hidden = nullptr;
  int32_t* d_rows = nullptr;
  int64_t d_cap = 0;
};

void die(const char* what) {
  std::fprintf(stderr, "engram_logits: %s: %s\n", what, me_rt_last_error());
  std::exit(1);
}

// one ubatch: tokens (seq, pos, tok) with their hidden rows, injected in place
void ubatch(Run& r, const std::vector<int32_t>& seq, const std::vector<int64_t>& pos, const std::vector<int32_t>& tok,
            std::vector<float*>& rows_h) {
  const int64_t n = (int64_t)tok.size();
  for (int64_t i = 0; i < n; ++i)
    if (me_rt_hist_set(r.hist, seq[i], pos[i], tok[i])) die("hist_set");
  std::vector<int32_t> prev((size_t)n * r.n_prev), rows((size_t)n * r.nt);
  if (me_rt_hist_prev(r.hist, seq.data(), pos.data(), n, r.n_prev, prev.data())) die("hist_prev");
  if (me_rt_hash(r.rt, r.e, tok.data(), prev.data(), n, rows.data())) die("hash");
  std::vector<float> h((size_t)n * r.d);
  for (int64_t i = 0; i < n; ++i) std::memcpy(h.data() + i * r.d, rows_h[i], r.d * 4);
#ifndef ME_RT_NO_CUDA
  if (r.gpu) {
    if (r.d_cap < n) {
      cudaFree(r.d_hidden);
      cudaFree(r.d_rows);
      if (cudaMalloc(&r.d_hidden, n * r.d * 4) || cudaMalloc(&r.d_rows, n * r.nt * 4)) die("cudaMalloc");
      r.d_cap = n;
    }
    cudaMemcpy(r.d_hidden, h.data(), n * r.d * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(r.d_rows, rows.data(), n * r.nt * 4, cudaMemcpyHostToDevice);
    if (me_rt_cuda_inject(r.rt, r.e, r.d_hidden, r.d_rows, nullptr, n, nullptr)) die("cuda_inject");
    cudaMemcpy(h.data(), r.d_hidden, n * r.d * 4, cudaMemcpyDeviceToHost);
  } else
#endif
  if (me_rt_inject_cpu(r.rt, r.e, h.data(), rows.data(), nullptr, n)) {
    die("inject_cpu");
  }
  const bool dump = std::getenv("ENGRAM_DUMP") != nullptr;
  for (int64_t i = 0; i < n; ++i) {
    std::memcpy(rows_h[i], h.data() + i * r.d, r.d * 4);
    if (dump) {
      double s = 0;
      for (int64_t j = 0; j < r.d; ++j) s += (double)h[i * r.d + j] * h[i * r.d + j];
      std::fprintf(stderr, "seq %d pos %lld |h| %.6f\n", seq[i], (long long)pos[i], std::sqrt(s));
    }
  }
}

template <typename T>
std::vector<T> read_file(const char* path, size_t count) {
  std::vector<T> v(count);
  FILE* f = std::fopen(path, "rb");
  if (!f || std::fread(v.data(), sizeof(T), count, f) != count) {
    std::fprintf(stderr, "engram_logits: cannot read %zu values from %s\n", count, path);
    std::exit(1);
  }
  std::fclose(f);
  return v;
}

}  // namespace

int main(int argc, char** argv) {
  std::string gguf, tokens_path, hidden_path, out_path, mode = "full";
  int e = 0, S = 1, T = 0, U = 0;
  bool gpu = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto next = [&]() -> const char* {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "engram_logits: %s needs a value\n", a.c_str());
        std::exit(2);
      }
      return argv[++i];
    };
    if (a == "--gguf") gguf = next();
    else if (a == "--engram") e = std::atoi(next());
    else if (a == "--n-seq") S = std::atoi(next());
    else if (a == "--n-tok") T = std::atoi(next());
    else if (a == "--tokens") tokens_path = next();
    else if (a == "--hidden") hidden_path = next();
    else if (a == "--mode") mode = next();
    else if (a == "--ubatch") U = std::atoi(next());
    else if (a == "--gpu") gpu = true;
    else if (a == "--out") out_path = next();
    else {
      std::fprintf(stderr, "engram_logits: unknown argument %s\n", a.c_str());
      return 2;
    }
  }
  if (gguf.empty() || tokens_path.empty() || hidden_path.empty() || out_path.empty() || T <= 0 || S <= 0) {
    std::fprintf(stderr, "usage: engram_logits --gguf F --n-seq S --n-tok T --tokens t.i32 --hidden h.f32 "
                         "--mode full|decode|two|state [--engram E] [--ubatch U] [--gpu] --out o.f32\n");
    return 2;
  }
  Run r;
  r.e = e;
  r.gpu = gpu;
  if (me_rt_open(gguf.c_str(), -1, &r.rt)) die("open");
  r.d = me_rt_n_embd(r.rt);
  r.n_prev = me_rt_max_order(r.rt) - 1;
  if (me_rt_engram_info(r.rt, e, nullptr, nullptr, &r.nt, nullptr, nullptr)) die("engram_info");
#ifdef ME_RT_NO_CUDA
  if (gpu) {
    std::fprintf(stderr, "engram_logits: --gpu needs the CUDA build (make, not make cpu)\n");
    return 2;
  }
#endif
  if (gpu && me_rt_cuda_upload(r.rt, e, 0)) die("cuda_upload");
  if (me_rt_hist_new(&r.hist)) die("hist_new");
  auto tok = read_file<int32_t>(tokens_path.c_str(), (size_t)S * T);
  auto hid = read_file<float>(hidden_path.c_str(), (size_t)S * T * r.d);
  auto H = [&](int s, int t) { return hid.data() + ((size_t)s * T + t) * r.d; };
  auto run_range = [&](int s, int seq_id, int t0, int t1, int step) {
    for (int a = t0; a < t1; a += step) {
      std::vector<int32_t> sq, tk;
      std::vector<int64_t> ps;
      std::vector<float*> hr;
      for (int t = a; t < std::min(t1, a + step); ++t) {
        sq.push_back(seq_id);
        ps.push_back(t);
        tk.push_back(tok[(size_t)s * T + t]);
        hr.push_back(H(s, t));
      }
      ubatch(r, sq, ps, tk, hr);
    }
  };
  if (mode == "full") {
    for (int s = 0; s < S; ++s) run_range(s, s, 0, T, U > 0 ? U : T);
  } else if (mode == "decode") {
    for (int s = 0; s < S; ++s) {
      run_range(s, s, 0, 1, 1);
      run_range(s, s, 1, T, 1);
    }
  } else if (mode == "two") {
    if (S < 2) die("mode two needs two sequences");
    for (int t = 0; t < T; ++t) {
      std::vector<int32_t> sq = {0, 1}, tk = {tok[t], tok[(size_t)T + t]};
      std::vector<int64_t> ps = {t, t};
      std::vector<float*> hr = {H(0, t), H(1, t)};
      ubatch(r, sq, ps, tk, hr);
    }
  } else if (mode == "state") {
    const int half = T / 2;
    run_range(0, 0, 0, half, 1);
    size_t size = 0;
    if (me_rt_hist_save(r.hist, 0, nullptr, &size)) die("hist_save");
    std::vector<uint8_t> blob(size);
    if (me_rt_hist_save(r.hist, 0, blob.data(), &size)) die("hist_save");
    if (me_rt_hist_remove(r.hist, -1, 0, -1)) die("hist_remove");
    if (me_rt_hist_load(r.hist, 7, blob.data(), blob.size())) die("hist_load");
    run_range(0, 7, half, T, 1);
  } else {
    std::fprintf(stderr, "engram_logits: unknown mode %s\n", mode.c_str());
    return 2;
  }
  FILE* f = std::fopen(out_path.c_str(), "wb");
  if (!f || std::fwrite(hid.data(), 4, hid.size(), f) != hid.size()) {
    std::fprintf(stderr, "engram_logits: cannot write %s\n", out_path.c_str());
    return 1;
  }
  std::fclose(f);
#ifndef ME_RT_NO_CUDA
  if (gpu) {
    cudaFree(r.d_hidden);
    cudaFree(r.d_rows);
  }
#endif
  me_rt_hist_free(r.hist);
  me_rt_close(r.rt);
  return 0;
}
