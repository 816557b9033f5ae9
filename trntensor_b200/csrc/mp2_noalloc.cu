// DF-MP2 energy without any device allocation.
//
// Some callers cannot allocate device memory at all: a host program that
// has already carved the whole HBM budget into its own pools (large
// quantum-chemistry codes commonly do this) and refuses foreign allocations,
// a latency-sensitive pipeline for which cudaMalloc/cudaFree's implicit
// device-wide synchronisation would stall other streams, or an FFI caller
// that has no allocator to hand. tt_mp2_energy_f32 needs a caller-provided
// workspace for the int8 slices of B; this variant instead uses a fixed
// scratch array that lives in the library's own device image.
//
// The scratch is a file-scope __device__ array of TT_MP2_NOALLOC_SCRATCH_BYTES
// bytes. Every GPU that loads the library keeps it until the process exits.
// Its host-side name is only a stand-in: the device address is looked up
// once per device with cudaGetSymbolAddress (the first call on a device does
// that set-up, so make that first call before any stream capture).
#include "common.cuh"

static __device__ __align__(256) unsigned char g_mp2_scratch[TT_MP2_NOALLOC_SCRATCH_BYTES];

namespace {

std::once_flag g_scratch_flags[tt::kMaxDevices];
int g_scratch_status[tt::kMaxDevices];
void* g_scratch_ptr[tt::kMaxDevices];

// Device address of g_mp2_scratch on the current device (looked up once).
int scratch_address(int dev, void** out) {
  const int st = tt::once_per_device(g_scratch_flags, g_scratch_status, dev, [dev]() -> int {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_mp2_scratch);
    if (e != cudaSuccess) return tt::cuda_status(e);
    g_scratch_ptr[dev] = p;
    return TT_OK;
  });
  *out = g_scratch_ptr[dev];
  return st;
}

}  // namespace

extern "C" int tt_mp2_energy_f32_noalloc(const float* B, const float* eps_occ,
                                         const float* eps_vir, int nocc, int nvir, int naux,
                                         double* energy, double* pair_partials, int* dev_status,
                                         void* stream) {
  if (!B || !eps_occ || !eps_vir || !energy || !dev_status) return TT_ERR_NULL;
  if (nocc <= 0 || nvir <= 0 || naux <= 0) return TT_ERR_SHAPE;
  const size_t need = tt_mp2_workspace_bytes(nocc, nvir, naux);
  if (need == 0 || need > (size_t)TT_MP2_NOALLOC_SCRATCH_BYTES) return TT_ERR_WORKSPACE;
  int dev = 0;
  int st = tt::check_device(&dev);
  if (st != TT_OK) return st;
  void* scratch = nullptr;
  st = scratch_address(dev, &scratch);
  if (st != TT_OK) return st;
  // The split kernel rewrites every byte of the slices and scales it uses,
  // so nothing left in the scratch by an earlier call needs clearing.
  return tt_mp2_energy_f32(B, eps_occ, eps_vir, nocc, nvir, naux, 0,
                           tt_mp2_num_pairs(nocc), scratch, need, energy, pair_partials,
                           dev_status, stream);
}
