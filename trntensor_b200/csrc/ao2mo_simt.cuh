// AO->MO transform on CUDA cores: a batched "A^T B" GEMM used for both steps
// of the two-step form (trntensor tests/test_quantum.py:73-74):
//   step 1: inter[i, (n,P)] = sum_m C_occ[m, i] eri[m, (n,P)]
//           A = C_occ (K=nbf, M=nocc), B = eri (K=nbf, N=nbf*naux)
//   step 2: B_out[i][a, P] = sum_n C_vir[n, a] inter[i][n, P]   (batch i)
//           A = C_vir (K=nbf, M=nvir), B_i = inter[i] (K=nbf, N=naux)
// Both operands are "K rows, M/N contiguous", C is row-major (M, N).
// Templated on the arithmetic type: double serves precision="kahan" and
// float64 inputs; float is the fp32 CUDA-core path.
#pragma once
#include <cstdint>

namespace tt {
namespace ao2mo {

template <typename T>
struct GemmParams {
  const T* A;  // (K, M) row-major, lda between k rows
  const T* B;  // (K, N) row-major, ldb
  T* C;        // (M, N) row-major, ldc
  long long lda, ldb, ldc;
  long long strideA, strideB, strideC;  // per batch (elements)
  int M, N, K, batch;
};

template <typename T, int BM, int BN, int BK, int TM, int TN>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    gemm_at_b(GemmParams<T> p) {
  constexpr int NT = (BM / TM) * (BN / TN);
  __shared__ T As[BK][BM];
  __shared__ T Bs[BK][BN];
  const int tiles_m = (p.M + BM - 1) / BM, tiles_n = (p.N + BN - 1) / BN;
  const long long tiles = (long long)tiles_m * tiles_n * p.batch;
  const int tx = threadIdx.x % (BN / TN), ty = threadIdx.x / (BN / TN);
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int b = (int)(t / ((long long)tiles_m * tiles_n));
    const int rem = (int)(t % ((long long)tiles_m * tiles_n));
    const int m0 = (rem / tiles_n) * BM, n0 = (rem % tiles_n) * BN;
    const T* A = p.A + b * p.strideA;
    const T* B = p.B + b * p.strideB;
    T acc[TM][TN];
#pragma unroll
    for (int u = 0; u < TM; ++u)
#pragma unroll
      for (int v = 0; v < TN; ++v) acc[u][v] = T(0);
    for (int k0 = 0; k0 < p.K; k0 += BK) {
      __syncthreads();
      for (int e = threadIdx.x; e < BK * BM; e += NT) {
        const int k = e / BM, m = e % BM;
        As[k][m] = (k0 + k < p.K && m0 + m < p.M) ? A[(long long)(k0 + k) * p.lda + m0 + m] : T(0);
      }
      for (int e = threadIdx.x; e < BK * BN; e += NT) {
        const int k = e / BN, n = e % BN;
        Bs[k][n] = (k0 + k < p.K && n0 + n < p.N) ? B[(long long)(k0 + k) * p.ldb + n0 + n] : T(0);
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < BK; ++k) {
        T a[TM], bb[TN];
#pragma unroll
        for (int u = 0; u < TM; ++u) a[u] = As[k][ty * TM + u];
#pragma unroll
        for (int v = 0; v < TN; ++v) bb[v] = Bs[k][tx + v * (BN / TN)];
#pragma unroll
        for (int u = 0; u < TM; ++u)
#pragma unroll
          for (int v = 0; v < TN; ++v) acc[u][v] = fma(a[u], bb[v], acc[u][v]);
      }
    }
    T* C = p.C + b * p.strideC;
#pragma unroll
    for (int u = 0; u < TM; ++u) {
      const int m = m0 + ty * TM + u;
      if (m >= p.M) continue;
#pragma unroll
      for (int v = 0; v < TN; ++v) {
        const int n = n0 + tx + v * (BN / TN);
        if (n < p.N) C[(long long)m * p.ldc + n] = acc[u][v];
      }
    }
  }
}

}  // namespace ao2mo
}  // namespace tt
