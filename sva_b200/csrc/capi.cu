// Library-wide C ABI helpers: version, thread-local last error, kernel attribute cache.
#include <mutex>
#include <string>
#include <unordered_map>
#include <unordered_set>

#include "sva_internal.h"

namespace sva {

static thread_local std::string g_last_error;

int set_error(int code, const char* msg) {
  g_last_error = msg ? msg : "";
  return code;
}

int ensure_smem_attr(const void* kernel, int bytes) {
  // (kernel, device) -> the limit set so far; a call asking for more raises it again
  static std::mutex mu;
  static std::unordered_map<unsigned long long, int> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  }
  const unsigned long long key = (reinterpret_cast<unsigned long long>(kernel) << 6) ^ static_cast<unsigned long long>(dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return SVA_OK;
  }
  // The dynamic limit may not exceed the opt-in maximum minus the kernel's static shared memory.
  cudaFuncAttributes fa;
  int optin = 0;
  int set = bytes;
  e = cudaFuncGetAttributes(&fa, kernel);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e == cudaSuccess) {
    const int room = optin - static_cast<int>(fa.sharedSizeBytes);
    set = bytes < room ? bytes : room;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, set);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();  // do not leave the error for the next runtime call
    return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  }
  std::lock_guard<std::mutex> lock(mu);
  int& v = done[key];
  if (set > v) v = set;
  return SVA_OK;
}

static thread_local void* const* g_prof_events = nullptr;
static thread_local int g_prof_n = 0;

void profile_mark(int i, cudaStream_t stream) {
  if (!g_prof_events || i >= g_prof_n || !g_prof_events[i]) return;
  // External event records are only valid while the stream is being captured into a graph.
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &status) != cudaSuccess) status = cudaStreamCaptureStatusNone;
  const cudaEvent_t ev = static_cast<cudaEvent_t>(g_prof_events[i]);
  const cudaError_t e = (status == cudaStreamCaptureStatusActive)
                            ? cudaEventRecordWithFlags(ev, stream, cudaEventRecordExternal)
                            : cudaEventRecord(ev, stream);
  if (e != cudaSuccess) cudaGetLastError();  // timing is best effort; never fail the launch
}

static thread_local void* g_debug_ts = nullptr;

void* debug_timestamps() { return g_debug_ts; }

}  // namespace sva

extern "C" int sva_debug_timestamps(void* device_buffer) {
  sva::g_debug_ts = device_buffer;
  return SVA_OK;
}

extern "C" int sva_profile_events(void* const* events, int32_t n) {
  sva::g_prof_events = (n > 0) ? events : nullptr;
  sva::g_prof_n = (n > 0) ? n : 0;
  return SVA_OK;
}

extern "C" int sva_host_buffer_device_accessible(const void* p) {
  if (!p) return 0;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return (attr.type == cudaMemoryTypeHost && attr.devicePointer == p) ? 1 : 0;
}

extern "C" const char* sva_version(void) { return "sva_b200 0.1.0 (sm_100a)"; }

extern "C" const char* sva_last_error(void) { return sva::g_last_error.c_str(); }
