// The GPU entry points of the engram runtime for a build without CUDA (`make cpu`): every call
// reports that the GPU path is not built, so callers fall back to the CPU injection.
#include <string>

#include "engram_runtime.h"
#include "runtime.h"

namespace me {

int cuda_available() { return 0; }

int cuda_upload(Engram&, int64_t, int, std::string* err) {
  if (err) *err = "engram runtime built without CUDA (make cpu)";
  return ME_RT_ERR_CUDA;
}

int cuda_inject(Engram&, int64_t, float*, const int32_t*, const float*, int64_t, void*, std::string* err) {
  if (err) *err = "engram runtime built without CUDA (make cpu)";
  return ME_RT_ERR_CUDA;
}

void cuda_release(Engram&) {}

}  // namespace me
