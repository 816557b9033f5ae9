// DF-MP2 pair energy on CUDA cores, templated on the arithmetic type.
//   double: the fp64 path (precision="kahan" and float64 inputs);
//   float : an independent on-device cross-check of the tensor-core kernel.
// Same sum and the same (i <= j, upper-triangle) decomposition as the tcgen05
// kernel, with 64 x 64 square blocks (A <= B) and both T_ab and T_ba held in
// registers: acc0 = B_i[A] B_j[B]^T, acc1 = B_j[A] B_i[B]^T.
#pragma once
#include <cstdint>

namespace tt {
namespace mp2s {

constexpr int kT = 64;      // block edge
constexpr int kKC = 16;     // aux chunk
constexpr int kThreads = 256;  // 16 x 16, 4 x 4 outputs each

__host__ __device__ inline long long pair_offset(long long i, long long n) {
  return i * n - i * (i - 1) / 2;
}

template <typename T>
struct Params {
  const T* B;  // (nocc, nvir, naux) row-major
  const T* eps_occ;
  const T* eps_vir;
  int nocc, nvir, naux;
  long long pair_begin, pair_end;
  int nblk;  // ceil(nvir / 64)
  double* energy;
  double* pair_partials;
};

template <typename T>
__global__ void __launch_bounds__(kThreads) energy_kernel(Params<T> p) {
  __shared__ T s[4][kKC][kT + 1];  // B_i[A], B_j[B], B_j[A], B_i[B], k-major
  __shared__ double red[kThreads / 32];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const long long npairs = p.pair_end - p.pair_begin;
  const int nbp = p.nblk * (p.nblk + 1) / 2;  // A <= B block pairs
  const long long n_items = npairs * nbp;
  double my = 0.0;

  for (long long w = blockIdx.x; w < n_items; w += gridDim.x) {
    const long long pr = p.pair_begin + w / nbp;
    int bp = (int)(w % nbp);
    // pair decode
    int i = 0;
    while (i + 1 < p.nocc && pair_offset(i + 1, p.nocc) <= pr) ++i;
    const int j = (int)(i + (pr - pair_offset(i, p.nocc)));
    int A = 0;
    while (bp >= p.nblk - A) {
      bp -= p.nblk - A;
      ++A;
    }
    const int Bb = A + bp;
    const int a0 = A * kT, b0 = Bb * kT;

    T acc0[4][4], acc1[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int v = 0; v < 4; ++v) acc0[u][v] = acc1[u][v] = T(0);

    for (int k0 = 0; k0 < p.naux; k0 += kKC) {
      __syncthreads();
      for (int e = threadIdx.x; e < 4 * kT * kKC; e += kThreads) {
        const int which = e / (kT * kKC);
        const int r = (e / kKC) % kT;
        const int k = e % kKC;
        const int occ = (which == 0 || which == 3) ? i : j;
        const int vr = ((which == 0 || which == 2) ? a0 : b0) + r;
        T val = T(0);
        if (vr < p.nvir && k0 + k < p.naux)
          val = p.B[((long long)occ * p.nvir + vr) * p.naux + k0 + k];
        s[which][k][r] = val;
      }
      __syncthreads();
#pragma unroll 4
      for (int k = 0; k < kKC; ++k) {
        T xa0[4], xb0[4], xa1[4], xb1[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          xa0[u] = s[0][k][ty * 4 + u];
          xa1[u] = s[2][k][ty * 4 + u];
          xb0[u] = s[1][k][tx * 4 + u];
          xb1[u] = s[3][k][tx * 4 + u];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            acc0[u][v] += xa0[u] * xb0[v];
            acc1[u][v] += xa1[u] * xb1[v];
          }
      }
    }
    const T eij = p.eps_occ[i] + p.eps_occ[j];
    double part = 0.0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int a = a0 + ty * 4 + u;
      if (a >= p.nvir) continue;
      const T eija = eij - p.eps_vir[a];
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int b = b0 + tx * 4 + v;
        if (b >= p.nvir || a > b) continue;
        const T x = acc0[u][v], y = acc1[u][v];
        T val = T(2) * (x * x - x * y + y * y) / (eija - p.eps_vir[b]);
        if (a == b) val *= T(0.5);
        part += (double)val;
      }
    }
    const double wgt = (i == j) ? 1.0 : 2.0;
    my += wgt * part;
    if (p.pair_partials != nullptr) {
      double t = part;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if ((threadIdx.x & 31) == 0) {
        atomicAdd(p.pair_partials + (long long)i * p.nocc + j, t);
        if (i != j) atomicAdd(p.pair_partials + (long long)j * p.nocc + i, t);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) my += __shfl_xor_sync(0xffffffffu, my, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = my;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int k = 0; k < kThreads / 32; ++k) t += red[k];
    if (t != 0.0) atomicAdd(p.energy, t);
  }
}

}  // namespace mp2s
}  // namespace tt
