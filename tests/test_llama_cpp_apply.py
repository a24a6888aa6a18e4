"""The llama.cpp integration script (engram_runtime/llama_cpp/apply.py) on a stand-in checkout:
every anchored edit lands once, a second run is a no-op, and a checkout whose code moved is
refused before anything is written. (llama.cpp itself is not on this machine: the bridge is
exercised through the runtime's C API by test_engram_runtime.py.)"""
import importlib.util
import os

import pytest

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FILES = {
    "src/CMakeLists.txt": "set(LLAMA_CORE_SOURCES\n    llama-mmap.cpp\n    llama-model-saver.cpp\n    llama-model.cpp\n)\n",
    "src/llama-hparams.h": "struct llama_hparams {\n    uint32_t n_embd;\n};\n",
    "src/llama-kv-cache.cpp": ("bool llama_kv_cache::has_cell_ext() const {\n"
                               "    return hparams.n_pos_per_embd() > 1 || hparams.ple_n_heads > 0;\n}\n"),
    "src/models/models.h": "struct llama_model_gemma4 : public llama_model_base {\n    void f();\n};\n",
    "src/models/gemma4.cpp": (
        '#include "models.h"\n\nvoid llama_model_gemma4::load_arch_hparams(llama_model_loader & ml) {\n'
        "    if (x) { y(); }\n}\n\nvoid llama_model_gemma4::load_arch_tensors(llama_model_loader &) {\n"
        "    z();\n}\n\nllama_model_gemma4::graph::graph(const llama_model & model) {\n"
        "    for (int il = 0; il < n_layer; ++il) {\n        cur = f(cur);\n"
        '        cur = build_cvec(cur, il);\n        cb(cur, "l_out", il);\n    }\n}\n'),
}


def _apply_module():
    spec = importlib.util.spec_from_file_location("apply", os.path.join(HERE, "engram_runtime", "llama_cpp", "apply.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _tree(root, files=FILES):
    for rel, text in files.items():
        os.makedirs(os.path.dirname(os.path.join(root, rel)), exist_ok=True)
        with open(os.path.join(root, rel), "w") as f:
            f.write(text)


def test_apply_edits(tmp_path, monkeypatch):
    m = _apply_module()
    _tree(str(tmp_path))
    lib = os.path.join(m.RUNTIME, "build", "libengram_runtime.so")
    monkeypatch.setattr(os.path, "isfile", lambda p: True if p == lib else os.path.exists(p) and not os.path.isdir(p))
    m.main([str(tmp_path)])
    read = lambda rel: open(os.path.join(tmp_path, rel)).read()  # noqa: E731
    assert "llama-engram-bridge.cpp" in read("src/CMakeLists.txt") and "libengram_runtime.so" in read("src/CMakeLists.txt")
    assert "bool micro_engram = false;" in read("src/llama-hparams.h")
    assert "|| hparams.micro_engram;" in read("src/llama-kv-cache.cpp")
    assert "std::shared_ptr<struct llama_engram_bridge> engram;" in read("src/models/models.h")
    g = read("src/models/gemma4.cpp")
    assert g.startswith('#include "llama-engram-bridge.h"')
    assert g.index("engram->load(ml.metadata") < g.index("void llama_model_gemma4::load_arch_tensors")
    assert g.index("engram->add_tensor(e, \"tables\"") < g.index("llama_model_gemma4::graph::graph")
    assert g.index("llama_engram_graph engram_g") < g.index("for (int il = 0")
    assert g.index("cur = engram_g.inject(cur, il, inp_out_ids);") < g.index("cur = build_cvec(cur, il);")
    assert os.path.isfile(os.path.join(tmp_path, "src", "llama-engram-bridge.cpp"))
    before = read("src/models/gemma4.cpp")
    m.main([str(tmp_path)])  # already applied: nothing changes
    assert read("src/models/gemma4.cpp") == before


def test_apply_refuses_moved_code(tmp_path):
    m = _apply_module()
    files = dict(FILES)
    files["src/models/gemma4.cpp"] = files["src/models/gemma4.cpp"].replace("build_cvec", "build_control_vector")
    _tree(str(tmp_path), files)
    with pytest.raises(SystemExit, match="anchor not found"):
        m.plan(str(tmp_path))
    assert "engram" not in open(os.path.join(tmp_path, "src/models/gemma4.cpp")).read()
