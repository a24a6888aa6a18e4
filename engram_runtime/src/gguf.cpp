#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace me {

namespace {

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;

  template <typename T>
  T get() {
    T v{};
    if (p + sizeof(T) > end) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > (uint64_t)(end - p)) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
  void skip(uint64_t n) {
    if (n > (uint64_t)(end - p)) ok = false;
    else p += n;
  }
};

size_t scalar_size(GType t) {
  switch (t) {
    case GType::U8: case GType::I8: case GType::BOOL: return 1;
    case GType::U16: case GType::I16: return 2;
    case GType::U32: case GType::I32: case GType::F32: return 4;
    case GType::U64: case GType::I64: case GType::F64: return 8;
    default: return 0;
  }
}

float half_to_float(uint16_t h) {  // IEEE 754 binary16 -> binary32
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0x1f) {
    bits = sign | 0x7f800000u | (man << 13);
  } else if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while (!(man & 0x400));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
    }
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t float_to_bf16(float f) {  // round to nearest even; NaN stays NaN
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

}  // namespace

Gguf::~Gguf() {
  if (map_) munmap(map_, size_);
}

bool Gguf::open(const std::string& path, std::string* err) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) {
    *err = "cannot open " + path;
    return false;
  }
  struct stat st {};
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    ::close(fd);
    *err = path + " is not a GGUF file";
    return false;
  }
  size_ = (size_t)st.st_size;
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    *err = "cannot map " + path;
    return false;
  }
  const uint8_t* base = static_cast<const uint8_t*>(map_);
  Cursor c{base, base + size_};
  if (c.get<uint32_t>() != 0x46554747u) {  // "GGUF" little-endian
    *err = path + " is not a GGUF file (bad magic)";
    return false;
  }
  version_ = c.get<uint32_t>();
  if (version_ < 2 || version_ > 3) {
    *err = "unsupported GGUF version " + std::to_string(version_);
    return false;
  }
  const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
  for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
    std::string key = c.str();
    KV kv;
    kv.type = static_cast<GType>(c.get<uint32_t>());
    if (kv.type == GType::STR) {
      kv.n = 1;
      kv.strs.push_back(c.str());
    } else if (kv.type == GType::ARR) {
      kv.arr_type = static_cast<GType>(c.get<uint32_t>());
      kv.n = c.get<uint64_t>();
      if (kv.arr_type == GType::STR) {
        for (uint64_t j = 0; j < kv.n && c.ok; ++j) kv.strs.push_back(c.str());
      } else {
        const size_t es = scalar_size(kv.arr_type);
        if (es == 0) {
          *err = "key " + key + ": nested or unknown array type";
          return false;
        }
        kv.data = c.p;
        c.skip(kv.n * es);
      }
    } else {
      const size_t es = scalar_size(kv.type);
      if (es == 0) {
        *err = "key " + key + ": unknown value type";
        return false;
      }
      kv.n = 1;
      kv.data = c.p;
      c.skip(es);
    }
    kv_[key] = std::move(kv);
  }
  std::vector<std::pair<Tensor, uint64_t>> infos;
  for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
    Tensor t;
    t.name = c.str();
    const uint32_t nd = c.get<uint32_t>();
    if (nd > 4) {
      *err = "tensor " + t.name + " has " + std::to_string(nd) + " dimensions";
      return false;
    }
    for (uint32_t d = 0; d < nd; ++d) t.ne.push_back((int64_t)c.get<uint64_t>());
    t.type = c.get<uint32_t>();
    infos.emplace_back(std::move(t), c.get<uint64_t>());
  }
  if (!c.ok) {
    *err = path + ": truncated GGUF header";
    return false;
  }
  uint32_t align = 32;
  u32("general.alignment", &align);
  if (align == 0) align = 32;
  const uint64_t header = (uint64_t)(c.p - base);
  const uint64_t data0 = (header + align - 1) / align * align;
  for (auto& [t, off] : infos) {
    int64_t numel = 1;
    for (int64_t v : t.ne) numel *= v;
    const uint64_t es = t.type == GGML_F32 ? 4 : (t.type == GGML_F16 || t.type == GGML_BF16) ? 2 : 0;
    t.nbytes = es * (uint64_t)numel;
    if (data0 + off > size_ || (es && data0 + off + t.nbytes > size_)) {
      *err = "tensor " + t.name + " lies outside the file";
      return false;
    }
    t.data = base + data0 + off;
    tensors_[t.name] = std::move(t);
  }
  return true;
}

const KV* Gguf::find(const std::string& key) const {
  auto it = kv_.find(key);
  return it == kv_.end() ? nullptr : &it->second;
}

const Tensor* Gguf::tensor(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

bool Gguf::u32(const std::string& key, uint32_t* out) const {
  const KV* kv = find(key);
  if (!kv || kv->type != GType::U32) return false;
  std::memcpy(out, kv->data, 4);
  return true;
}

bool tensor_to_f32(const Tensor& t, std::vector<float>* out) {
  int64_t n = 1;
  for (int64_t v : t.ne) n *= v;
  out->resize((size_t)n);
  if (t.type == GGML_F32) {
    std::memcpy(out->data(), t.data, (size_t)n * 4);
  } else if (t.type == GGML_F16 || t.type == GGML_BF16) {
    const uint16_t* s = reinterpret_cast<const uint16_t*>(t.data);
    for (int64_t i = 0; i < n; ++i) {
      if (t.type == GGML_F16) {
        (*out)[i] = half_to_float(s[i]);
      } else {
        const uint32_t b = (uint32_t)s[i] << 16;
        std::memcpy(&(*out)[i], &b, 4);
      }
    }
  } else {
    return false;
  }
  return true;
}

bool tensor_to_bf16(const Tensor& t, std::vector<uint16_t>* out) {
  int64_t n = 1;
  for (int64_t v : t.ne) n *= v;
  if (t.type == GGML_BF16) {
    const uint16_t* s = reinterpret_cast<const uint16_t*>(t.data);
    out->assign(s, s + n);
    return true;
  }
  std::vector<float> f;
  if (!tensor_to_f32(t, &f)) return false;
  out->resize((size_t)n);
  for (int64_t i = 0; i < n; ++i) (*out)[i] = float_to_bf16(f[i]);
  return true;
}

}  // namespace me
