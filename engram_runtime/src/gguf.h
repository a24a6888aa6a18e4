// Minimal read-only GGUF (v2/v3) parser: the key/value metadata and the tensor directory of a
// memory-mapped file. Only what the engram runtime needs: typed scalar / array lookups and
// pointers to F32 / F16 / BF16 tensor data. The file format is the public GGUF
// specification (ggml's docs/gguf.md): little-endian header "GGUF", version, tensor and
// key counts, key/value records, tensor infos, then the aligned data section.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace me {

enum class GType : uint32_t {
  U8 = 0, I8 = 1, U16 = 2, I16 = 3, U32 = 4, I32 = 5, F32 = 6, BOOL = 7, STR = 8, ARR = 9, U64 = 10, I64 = 11,
  F64 = 12,
};

// ggml tensor element types used by the engram tensors
enum : uint32_t { GGML_F32 = 0, GGML_F16 = 1, GGML_BF16 = 30 };

struct KV {
  GType type = GType::U8;
  GType arr_type = GType::U8;  // element type when type == ARR
  uint64_t n = 0;              // array length (1 for scalars)
  const uint8_t* data = nullptr;  // first element (not for string arrays)
  std::vector<std::string> strs;  // string scalar / string array
};

struct Tensor {
  std::string name;
  std::vector<int64_t> ne;  // ne[0] = innermost (contiguous) dimension
  uint32_t type = 0;
  const uint8_t* data = nullptr;
  uint64_t nbytes = 0;  // 0 when the type's size is not known here (quantized base tensors)
};

class Gguf {
 public:
  ~Gguf();
  bool open(const std::string& path, std::string* err);
  const KV* find(const std::string& key) const;
  const Tensor* tensor(const std::string& name) const;
  uint32_t version() const { return version_; }

  template <typename T>
  bool array(const std::string& key, GType want, std::vector<T>* out, std::string* err, bool required = true) const;
  bool u32(const std::string& key, uint32_t* out) const;

 private:
  void* map_ = nullptr;
  size_t size_ = 0;
  uint32_t version_ = 0;
  std::map<std::string, KV> kv_;
  std::map<std::string, Tensor> tensors_;
};

template <typename T>
bool Gguf::array(const std::string& key, GType want, std::vector<T>* out, std::string* err, bool required) const {
  const KV* kv = find(key);
  if (!kv) {
    if (required && err) *err = "missing key " + key;
    return false;
  }
  if (kv->type != GType::ARR || kv->arr_type != want) {
    if (err) *err = "key " + key + " has the wrong type";
    return false;
  }
  const T* p = reinterpret_cast<const T*>(kv->data);
  out->assign(p, p + kv->n);
  return true;
}

// fp32 copy of an F32 / F16 / BF16 tensor (false for other types)
bool tensor_to_f32(const Tensor& t, std::vector<float>* out);
// bf16 bits of an F32 / F16 / BF16 tensor (round to nearest even)
bool tensor_to_bf16(const Tensor& t, std::vector<uint16_t>* out);

}  // namespace me
