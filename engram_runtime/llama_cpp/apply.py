"""Add micro-engram support to a llama.cpp checkout (Gemma 4) through the engram runtime.

    make -C engram_runtime
    python engram_runtime/llama_cpp/apply.py /path/to/llama.cpp
    cmake -B build && cmake --build build -j --target llama-server

Copies llama-engram-bridge.{h,cpp} into llama.cpp's src/ and makes five anchored edits: the
bridge source and the runtime library in src/CMakeLists.txt, an hparams flag that makes the KV
cache keep token ids (has_cell_ext), the bridge member of the Gemma 4 model, its metadata and
tensors at load time, and the engram after each layer's scaled output. Every anchor is checked
before anything is written; a checkout whose code moved reports which anchor is missing. The
engram tensors are created by llama.cpp's loader under the GGUF names and must stay in host
memory (the engram runs as a CPU custom op).
"""
import os
import re
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
RUNTIME = os.path.dirname(HERE)
MARK = "llama-engram-bridge"

LOAD_HPARAMS = """
    engram = std::make_shared<llama_engram_bridge>();
    hparams.micro_engram = engram->load(ml.metadata, hparams.n_embd, (int32_t) hparams.n_layer());
"""
LOAD_TENSORS = """
    if (engram && engram->enabled()) {
        for (int32_t e = 0; e < me_rt_n_engrams(engram->rt); ++e) {
            int32_t il = 0, gate = 0, nt = 0, dim = 0;
            int64_t rows = 0;
            me_rt_engram_info(engram->rt, e, &il, &gate, &nt, &dim, &rows);
            const int64_t md = (int64_t) nt * dim;
            auto kv = [&](const char * s, std::initializer_list<int64_t> ne) {
                return create_tensor(tn(LLM_TENSOR_ENGRAM_KV, s, il), ne, 0);
            };
            engram->add_tensor(e, "tables", kv("mengram_tables", {dim, rows}));
            if (gate == ME_RT_GATE_PLE) {
                engram->add_tensor(e, "down", kv("mengram_down", {n_embd, md}));
                engram->add_tensor(e, "up", kv("mengram_up", {md, n_embd}));
            } else {
                engram->add_tensor(e, "key", kv("mengram_key", {md, n_embd}));
                engram->add_tensor(e, "value", kv("mengram_value", {md, n_embd}));
                if (gate == ME_RT_GATE_SCALAR_SQRT) {
                    engram->add_tensor(e, "q_scale", create_tensor(tn(LLM_TENSOR_ENGRAM_GATE, "mengram_q_scale", il), {n_embd}, 0));
                    engram->add_tensor(e, "k_scale", create_tensor(tn(LLM_TENSOR_ENGRAM_GATE, "mengram_k_scale", il), {n_embd}, 0));
                }
            }
        }
    }
"""
GRAPH_SETUP = """    static const llama_engram_bridge engram_none;
    const auto & engram_b = static_cast<const llama_model_gemma4 &>(model).engram;
    llama_engram_graph engram_g(*this, engram_b ? *engram_b : engram_none);

"""


def _func_end(src, signature):
    """Index of the closing brace of the function whose definition starts with `signature`."""
    i = src.index(signature)
    depth, j = 0, src.index("{", i)
    while True:
        if src[j] == "{":
            depth += 1
        elif src[j] == "}":
            depth -= 1
            if depth == 0:
                return j
        j += 1


def plan(root):
    """[(path, new text)] for every edit; raises SystemExit naming a missing anchor."""
    def read(rel):
        with open(os.path.join(root, rel)) as f:
            return f.read()

    def need(text, anchor, rel):
        if anchor not in text:
            raise SystemExit(f"{rel}: anchor not found: {anchor!r} (this llama.cpp moved; edit by hand)")

    edits = []
    rel = "src/CMakeLists.txt"
    s = read(rel)
    need(s, "llama-model-saver.cpp", rel)
    s = s.replace("    llama-model-saver.cpp\n", "    llama-model-saver.cpp\n    llama-engram-bridge.cpp\n", 1)
    s += (f"\n# micro_engram: the engram runtime ({RUNTIME})\n"
          f"set(MICRO_ENGRAM_RUNTIME_DIR \"{RUNTIME}\" CACHE PATH \"engram runtime folder\")\n"
          "target_include_directories(llama PRIVATE ${MICRO_ENGRAM_RUNTIME_DIR}/include)\n"
          "target_link_libraries(llama PRIVATE ${MICRO_ENGRAM_RUNTIME_DIR}/build/libengram_runtime.so)\n")
    edits.append((rel, s))
    rel = "src/llama-hparams.h"
    s = read(rel)
    need(s, "struct llama_hparams {", rel)
    s = s.replace("struct llama_hparams {\n", "struct llama_hparams {\n    bool micro_engram = false; // engram n-gram memory: the KV cache keeps token ids\n", 1)
    edits.append((rel, s))
    rel = "src/llama-kv-cache.cpp"
    s = read(rel)
    sig = "bool llama_kv_cache::has_cell_ext() const {"
    need(s, sig, rel)
    a, b = s.index(sig), _func_end(s, sig)
    body = re.sub(r"return (.*?);", r"return (\1) || hparams.micro_engram;", s[a:b], count=1)
    edits.append((rel, s[:a] + body + s[b:]))
    rel = "src/models/models.h"
    s = read(rel)
    anchor = "struct llama_model_gemma4 : public llama_model_base {"
    need(s, anchor, rel)
    s = s.replace(anchor + "\n", anchor + "\n    std::shared_ptr<struct llama_engram_bridge> engram;\n", 1)
    edits.append((rel, s))
    rel = "src/models/gemma4.cpp"
    s = read(rel)
    for anchor in ("void llama_model_gemma4::load_arch_hparams(llama_model_loader & ml) {",
                   "void llama_model_gemma4::load_arch_tensors(", "for (int il = 0; il < n_layer; ++il) {",
                   "cur = build_cvec(cur, il);"):
        need(s, anchor, rel)
    s = '#include "llama-engram-bridge.h"\n' + s
    end = _func_end(s, "void llama_model_gemma4::load_arch_hparams(llama_model_loader & ml) {")
    s = s[:end] + LOAD_HPARAMS + s[end:]
    end = _func_end(s, "void llama_model_gemma4::load_arch_tensors(")
    s = s[:end] + LOAD_TENSORS + s[end:]
    i = s.index("for (int il = 0; il < n_layer; ++il) {")
    line0 = s.rfind("\n", 0, i) + 1
    s = s[:line0] + GRAPH_SETUP + s[line0:]
    i = s.index("cur = build_cvec(cur, il);")
    line0 = s.rfind("\n", 0, i) + 1
    s = s[:line0] + "        cur = engram_g.inject(cur, il, inp_out_ids);\n\n" + s[line0:]
    edits.append((rel, s))
    return edits


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 1:
        raise SystemExit("usage: apply.py /path/to/llama.cpp")
    root = os.path.abspath(argv[0])
    if not os.path.isfile(os.path.join(root, "src/models/gemma4.cpp")):
        raise SystemExit(f"not a llama.cpp checkout with Gemma 4 (no src/models/gemma4.cpp): {root}")
    with open(os.path.join(root, "src/CMakeLists.txt")) as f:
        if MARK in f.read():
            print(f"micro_engram is already applied to {root}")
            return
    if not os.path.isfile(os.path.join(RUNTIME, "build", "libengram_runtime.so")):
        raise SystemExit(f"build the runtime first: make -C {RUNTIME}")
    edits = plan(root)  # every anchor checked before anything is written
    for rel, text in edits:
        with open(os.path.join(root, rel), "w") as f:
            f.write(text)
    for name in ("llama-engram-bridge.h", "llama-engram-bridge.cpp"):
        shutil.copy(os.path.join(HERE, name), os.path.join(root, "src", name))
    print(f"micro_engram applied to {root}; build as usual, e.g. cmake -B build -DGGML_CUDA=ON && "
          f"cmake --build build -j --target llama-server")


if __name__ == "__main__":
    main()
