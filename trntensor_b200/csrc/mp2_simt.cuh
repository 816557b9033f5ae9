// DF-MP2 pair energy on CUDA cores, templated on the arithmetic type.
//   double: the fp64 path (precision="kahan" and float64 inputs);
//   float : an independent on-device cross-check of the tensor-core kernel.
// Same sum and decomposition as the tensor-core kernel (unordered pairs
// i <= j, 128 x 128 blocks A <= B of the virtual pair matrix):
//   pass x: x = B_i[A] B_j[B]^T  (8 x 8 outputs per thread, kept in shared memory)
//   pass y: y = B_j[A] B_i[B]^T, or y = x for i == j, or y = x^T for A == B,
// then the (a,b)+(b,a) energy terms with weights 1 / 1/2 / 0 for a < b / = / >.
#pragma once
#include <cstdint>

namespace tt {
namespace mp2s {

constexpr int kT = 128;        // block edge
constexpr int kKC = 16;        // aux chunk
constexpr int kThreads = 256;  // 16 x 16 threads, 8 x 8 outputs each
constexpr int kLd = kT + 1;    // padded shared-memory row

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
  int nblk;  // ceil(nvir / 128)
  double* energy;
  double* pair_partials;
};

template <typename T>
constexpr int smem_bytes() {
  return (2 * 2 * kKC * kLd + kT * kLd) * (int)sizeof(T);
}

// acc[u][v] = sum_k B[occA][a0 + ty + 16u][k] * B[occB][b0 + tx + 16v][k]
template <typename T>
__device__ __forceinline__ void block_gemm(const Params<T>& p, int occA, int a0, int occB, int b0,
                                           T* As, T* Bs, T (&acc)[8][8]) {
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
#pragma unroll
  for (int u = 0; u < 8; ++u)
#pragma unroll
    for (int v = 0; v < 8; ++v) acc[u][v] = T(0);
  // loader mapping: 16 consecutive threads read one row's 16 k values
  const int lk = threadIdx.x & 15, lr = threadIdx.x >> 4;
  const T* rowA = p.B + (long long)occA * p.nvir * p.naux;
  const T* rowB = p.B + (long long)occB * p.nvir * p.naux;
  T ra[8], rb[8];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int row = lr + 16 * r, k = k0 + lk;
      const bool kin = k < p.naux;
      ra[r] = (kin && a0 + row < p.nvir) ? rowA[(long long)(a0 + row) * p.naux + k] : T(0);
      rb[r] = (kin && b0 + row < p.nvir) ? rowB[(long long)(b0 + row) * p.naux + k] : T(0);
    }
  };
  auto stash = [&](int buf) {
    T* as = As + buf * kKC * kLd;
    T* bs = Bs + buf * kKC * kLd;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      as[lk * kLd + lr + 16 * r] = ra[r];
      bs[lk * kLd + lr + 16 * r] = rb[r];
    }
  };
  const int nk = (p.naux + kKC - 1) / kKC;
  fetch(0);
  __syncthreads();  // previous users of As/Bs are done
  stash(0);
  __syncthreads();
  for (int c = 0; c < nk; ++c) {
    const int buf = c & 1;
    if (c + 1 < nk) fetch((c + 1) * kKC);
    const T* as = As + buf * kKC * kLd;
    const T* bs = Bs + buf * kKC * kLd;
#pragma unroll 4
    for (int k = 0; k < kKC; ++k) {
      T a[8], b[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] = as[k * kLd + ty + 16 * u];
#pragma unroll
      for (int v = 0; v < 8; ++v) b[v] = bs[k * kLd + tx + 16 * v];
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int v = 0; v < 8; ++v) acc[u][v] = fma(a[u], b[v], acc[u][v]);
    }
    if (c + 1 < nk) stash(buf ^ 1);
    __syncthreads();
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) energy_kernel(Params<T> p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* As = reinterpret_cast<T*>(smem_raw);
  T* Bs = As + 2 * kKC * kLd;
  T* Xs = Bs + 2 * kKC * kLd;  // kT x kLd: x of the current block
  __shared__ double red[kThreads / 32];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const long long npairs = p.pair_end - p.pair_begin;
  const int nbp = p.nblk * (p.nblk + 1) / 2;
  const long long n_items = npairs * nbp;
  double my = 0.0;

  for (long long w = blockIdx.x; w < n_items; w += gridDim.x) {
    const long long pr = p.pair_begin + w / nbp;
    int bp = (int)(w % nbp);
    int i = 0;
    while (i + 1 < p.nocc && pair_offset(i + 1, p.nocc) <= pr) ++i;
    const int j = (int)(i + (pr - pair_offset(i, p.nocc)));
    int A = 0;
    while (bp >= p.nblk - A) {
      bp -= p.nblk - A;
      ++A;
    }
    const int a0 = A * kT, b0 = (A + bp) * kT;
    const bool diag = bp == 0;

    T acc[8][8];
    block_gemm(p, i, a0, j, b0, As, Bs, acc);  // x
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
      for (int v = 0; v < 8; ++v) Xs[(ty + 16 * u) * kLd + tx + 16 * v] = acc[u][v];
    if (i != j && !diag) {
      block_gemm(p, j, a0, i, b0, As, Bs, acc);  // y
    } else {
      __syncthreads();  // Xs complete
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const int r = ty + 16 * u, c = tx + 16 * v;
          acc[u][v] = (i == j) ? Xs[r * kLd + c] : Xs[c * kLd + r];
        }
    }
    const T eij = p.eps_occ[i] + p.eps_occ[j];
    double part = 0.0;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int a = a0 + ty + 16 * u;
      if (a >= p.nvir) continue;
      const T eija = eij - p.eps_vir[a];
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const int b = b0 + tx + 16 * v;
        if (b >= p.nvir || a > b) continue;
        const T x = Xs[(ty + 16 * u) * kLd + tx + 16 * v], y = acc[u][v];
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
    __syncthreads();  // Xs is rewritten by the next item
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
