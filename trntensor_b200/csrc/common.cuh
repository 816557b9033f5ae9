// Host-side helpers shared by the C-ABI translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/trntensor_b200.h"

namespace tt {

// Last CUDA error text per host thread (reported by tt_last_cuda_error).
extern thread_local char g_last_cuda_error[256];

inline int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return TT_OK;
  std::strncpy(g_last_cuda_error, cudaGetErrorString(e), sizeof(g_last_cuda_error) - 1);
  return TT_ERR_CUDA;
}
#define TT_CUDA(call)                          \
  do {                                         \
    int _s = ::tt::cuda_status((call));        \
    if (_s != TT_OK) return _s;                \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device capability check, cached per device.
int check_device(int* device_out);

// Encode a row-major fp32 tensor map of rank 2 or 3 (dims innermost first).
int encode_tmap(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                const uint64_t* strides_bytes /* rank-1 entries */, const uint32_t* box,
                CUtensorMapSwizzle swizzle, CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_FLOAT32);

// Run `fn` once per device (e.g. raising the dynamic shared-memory limit).
template <typename F>
int once_per_device(std::once_flag* flags, int* results, int device, F fn) {
  std::call_once(flags[device], [&] { results[device] = fn(); });
  return results[device];
}
constexpr int kMaxDevices = 64;

}  // namespace tt
