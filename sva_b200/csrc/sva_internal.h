// Host-side helpers shared by the translation units of libsva_b200.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/sva_b200.h"

namespace sva {

constexpr int kMaxDynSmem = 227 * 1024;

// Records a one-line message for sva_last_error() and returns `code`.
int set_error(int code, const char* msg);

// Raises a kernel's dynamic shared-memory limit once per (kernel, device).
int ensure_smem_attr(const void* kernel, int bytes);

// Device buffer for phase timestamps set by sva_debug_timestamps (measurement only), or NULL.
void* debug_timestamps();

// Records the calling thread's i-th profiling event (sva_profile_events) on `stream`, if set.
void profile_mark(int i, cudaStream_t stream);

}  // namespace sva
