// C-ABI entry points for the AO->MO transform (two-step form).
#include "ao2mo_simt.cuh"
#include "common.cuh"

namespace tt {
namespace {

std::once_flag g_flags[kMaxDevices];
int g_ok[kMaxDevices];
int g_sms[kMaxDevices];

int setup(int dev) {
  return once_per_device(g_flags, g_ok, dev, [dev]() -> int {
    if (cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return TT_ERR_CUDA;
    return TT_OK;
  });
}

template <typename T>
int launch_gemm(const ao2mo::GemmParams<T>& p, cudaStream_t s, int sms) {
  constexpr int BM = sizeof(T) == 4 ? 128 : 64;
  constexpr int BN = sizeof(T) == 4 ? 128 : 64;
  constexpr int TM = sizeof(T) == 4 ? 8 : 4;
  constexpr int TN = sizeof(T) == 4 ? 8 : 4;
  constexpr int BK = 16;
  const long long tiles =
      (long long)((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN) * (long long)p.batch;
  if (tiles == 0) return TT_OK;
  const long long cap = (long long)sms * 4;
  const int grid = (int)(tiles < cap ? tiles : cap);
  ao2mo::gemm_at_b<T, BM, BN, BK, TM, TN><<<grid, (BM / TM) * (BN / TN), 0, s>>>(p);
  return cuda_status(cudaGetLastError());
}

template <typename T>
int ao2mo_simt(const T* eri, const T* C_occ, const T* C_vir, int nbf, int nocc, int nvir,
               int naux, void* workspace, size_t workspace_bytes, T* B_out, void* stream) {
  if (!eri || !C_occ || !C_vir || !workspace || !B_out) return TT_ERR_NULL;
  if (nbf <= 0 || nocc <= 0 || nvir <= 0 || naux <= 0) return TT_ERR_SHAPE;
  const size_t need = (size_t)nocc * nbf * naux * sizeof(T);
  if (workspace_bytes < need) return TT_ERR_WORKSPACE;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = setup(dev);
  if (st != TT_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  T* inter = static_cast<T*>(workspace);
  // step 1: inter (nocc, nbf*naux) = C_occ^T (nocc x nbf) . eri (nbf x nbf*naux)
  ao2mo::GemmParams<T> p1{C_occ, eri, inter, nocc, (long long)nbf * naux, (long long)nbf * naux,
                          0, 0, 0, nocc, nbf * naux, nbf, 1};
  st = launch_gemm<T>(p1, s, g_sms[dev]);
  if (st != TT_OK) return st;
  // step 2: B_out[i] (nvir, naux) = C_vir^T (nvir x nbf) . inter[i] (nbf x naux)
  ao2mo::GemmParams<T> p2{C_vir, inter, B_out, nvir, naux, naux,
                          0, (long long)nbf * naux, (long long)nvir * naux,
                          nvir, naux, nbf, nocc};
  return launch_gemm<T>(p2, s, g_sms[dev]);
}

}  // namespace
}  // namespace tt

extern "C" {

size_t tt_ao2mo_workspace_bytes(int nbf, int nocc, int nvir, int naux, int elem_bytes) {
  if (nbf <= 0 || nocc <= 0 || nvir <= 0 || naux <= 0) return 0;
  if (elem_bytes != 4 && elem_bytes != 8) return 0;
  return (size_t)nocc * nbf * naux * (size_t)elem_bytes;
}

int tt_ao2mo_f32(const float* eri, const float* C_occ, const float* C_vir, int nbf, int nocc,
                 int nvir, int naux, void* workspace, size_t workspace_bytes, float* B_out,
                 void* stream) {
  return tt::ao2mo_simt<float>(eri, C_occ, C_vir, nbf, nocc, nvir, naux, workspace,
                               workspace_bytes, B_out, stream);
}

int tt_ao2mo_f64(const double* eri, const double* C_occ, const double* C_vir, int nbf,
                 int nocc, int nvir, int naux, void* workspace, size_t workspace_bytes,
                 double* B_out, void* stream) {
  return tt::ao2mo_simt<double>(eri, C_occ, C_vir, nbf, nocc, nvir, naux, workspace,
                                workspace_bytes, B_out, stream);
}

}  // extern "C"
