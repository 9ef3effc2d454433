// Library-wide C ABI helpers: version, thread-local last error, kernel attribute cache.
#include <mutex>
#include <string>
#include <unordered_set>

#include "sva_internal.h"

namespace sva {

static thread_local std::string g_last_error;

int set_error(int code, const char* msg) {
  g_last_error = msg ? msg : "";
  return code;
}

int ensure_smem_attr(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::unordered_set<unsigned long long> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  const unsigned long long key = (reinterpret_cast<unsigned long long>(kernel) << 6) ^ static_cast<unsigned long long>(dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (done.count(key)) return SVA_OK;
  }
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  done.insert(key);
  return SVA_OK;
}

}  // namespace sva

extern "C" const char* sva_version(void) { return "sva_b200 0.1.0 (sm_100a)"; }

extern "C" const char* sva_last_error(void) { return sva::g_last_error.c_str(); }
