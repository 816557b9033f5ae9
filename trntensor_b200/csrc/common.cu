// Device checks, tensor-map encoding and status strings for the C ABI.
#include "common.cuh"
#include "ptx.cuh"

namespace tt {

thread_local char g_last_cuda_error[256] = {0};

namespace {
std::once_flag g_dev_flags[kMaxDevices];
int g_dev_ok[kMaxDevices];

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::once_flag g_encode_flag;
EncodeTiledFn g_encode = nullptr;
}  // namespace

int check_device(int* device_out) {
  int dev = 0;
  TT_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return TT_ERR_DEVICE;
  if (device_out) *device_out = dev;
  return once_per_device(g_dev_flags, g_dev_ok, dev, [dev]() -> int {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return TT_ERR_CUDA;
    if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return TT_ERR_CUDA;
    return (major == 10 && minor == 0) ? TT_OK : TT_ERR_DEVICE;
  });
}

int encode_tmap(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle,
                CUtensorMapDataType dtype) {
  std::call_once(g_encode_flag, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  });
  if (g_encode == nullptr) return TT_ERR_TMA;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5], es[5];
  for (int r = 0; r < rank; ++r) {
    d[r] = dims[r];
    bx[r] = box[r];
    es[r] = 1;
  }
  for (int r = 0; r + 1 < rank; ++r) st[r] = strides_bytes[r];
  CUresult res = g_encode(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return res == CUDA_SUCCESS ? TT_OK : TT_ERR_TMA;
}

// One thread waits, with the library's bounded mbarrier wait, on a phase
// that nothing completes; the wait gives up after `budget` cycles and
// records kDevTimeoutFull in *status, as every kernel's waits do.
__global__ void wait_timeout_kernel(int* status, long long budget, long long* cycles) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  const long long t0 = clock64();
  mbar_wait_budget(&bar, 0, status, kDevTimeoutFull, budget);
  *cycles = clock64() - t0;
}

}  // namespace tt

extern "C" {

int tt_debug_wait_timeout(int* dev_status, long long budget_cycles, long long* dev_cycles,
                          void* stream) {
  if (!dev_status || !dev_cycles) return TT_ERR_NULL;
  if (budget_cycles < 0 || budget_cycles > tt::kWaitBudgetCycles) return TT_ERR_SHAPE;
  int st = tt::check_device(nullptr);
  if (st != TT_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  TT_CUDA(cudaMemsetAsync(dev_status, 0, sizeof(int), s));
  tt::wait_timeout_kernel<<<1, 32, 0, s>>>(dev_status, budget_cycles, dev_cycles);
  return tt::cuda_status(cudaGetLastError());
}

const char* tt_status_string(int status) {
  switch (status) {
    case TT_OK: return "ok";
    case TT_ERR_NULL: return "a required pointer is NULL";
    case TT_ERR_SHAPE: return "a size argument is out of range";
    case TT_ERR_ALIGN: return "a pointer is not 16-byte aligned";
    case TT_ERR_WORKSPACE: return "workspace too small";
    case TT_ERR_DEVICE: return "current CUDA device is not an sm_100 (B200-class) GPU";
    case TT_ERR_CUDA: return "CUDA runtime or launch error";
    case TT_ERR_TMA: return "tensor-map encoding failed";
    default: return "unknown status";
  }
}

int tt_version(void) { return 100; }

int tt_device_check(void) { return tt::check_device(nullptr); }

const char* tt_last_cuda_error(void) { return tt::g_last_cuda_error; }

}  // extern "C"
