// precision="dd": double-double arithmetic on CUDA cores.
//
// A double-double value is an unevaluated sum hi + lo of two doubles with
// |lo| <= ulp(hi) / 2, about 106 significant bits. The building blocks are
// the classic error-free transformations, written here from their published
// definitions:
//   two_sum (Knuth, TAOCP vol. 2, 4.2.2): s + e == a + b exactly;
//   two_prod (with a fused multiply-add, as in Ogita, Rump & Oishi,
//     "Accurate sum and dot product", SIAM J. Sci. Comput. 26, 2005):
//     p + e == a * b exactly;
// dot products accumulate as that paper's Dot2 (sum in two_sum, the rounding
// errors of both the products and the sums collected in a second double),
// and the energy terms use double-double add / multiply / divide in the
// style of Hida, Li & Bailey's double-double library (2001).
//
// Kernels:
//   mp2dd::energy_kernel  DF-MP2 pair energies, one block per unordered pair
//                         at a time (both T_ab and T_ba dot products, the
//                         reference's own formulation), dd per-pair partials,
//                         dd per-block totals;
//   mp2dd::reduce_kernel  the per-block totals summed in a fixed order;
//   gdd::gemm_kernel      batched C = A B with optional lo parts on A and B
//                         (double-double inputs) and hi / lo outputs; serves
//                         the AO->MO transform and einsum contractions.
#include "common.cuh"

namespace tt {
namespace dd {

struct ddv {
  double hi, lo;
};

__device__ __forceinline__ ddv two_sum(double a, double b) {
  const double s = a + b;
  const double bb = s - a;
  return {s, (a - (s - bb)) + (b - bb)};
}
// |a| >= |b| (or a == 0)
__device__ __forceinline__ ddv quick_two_sum(double a, double b) {
  const double s = a + b;
  return {s, b - (s - a)};
}
__device__ __forceinline__ ddv two_prod(double a, double b) {
  const double p = a * b;
  return {p, fma(a, b, -p)};
}
__device__ __forceinline__ ddv add(ddv x, ddv y) {
  ddv s = two_sum(x.hi, y.hi);
  const ddv t = two_sum(x.lo, y.lo);
  s.lo += t.hi;
  s = quick_two_sum(s.hi, s.lo);
  s.lo += t.lo;
  return quick_two_sum(s.hi, s.lo);
}
__device__ __forceinline__ ddv neg(ddv x) { return {-x.hi, -x.lo}; }
__device__ __forceinline__ ddv sub(ddv x, ddv y) { return add(x, neg(y)); }
__device__ __forceinline__ ddv mul(ddv x, ddv y) {
  ddv p = two_prod(x.hi, y.hi);
  p.lo += x.hi * y.lo + x.lo * y.hi;
  return quick_two_sum(p.hi, p.lo);
}
__device__ __forceinline__ ddv mul_d(ddv x, double b) {
  ddv p = two_prod(x.hi, b);
  p.lo += x.lo * b;
  return quick_two_sum(p.hi, p.lo);
}
// x / y: three quotient digits, each from the running remainder.
__device__ __forceinline__ ddv div(ddv x, ddv y) {
  const double q1 = x.hi / y.hi;
  ddv r = sub(x, mul_d(y, q1));
  const double q2 = r.hi / y.hi;
  r = sub(r, mul_d(y, q2));
  const double q3 = r.hi / y.hi;
  const ddv q = quick_two_sum(q1, q2);
  return add(q, ddv{q3, 0.0});
}

// Dot2 accumulator: s + c carries the running sum; c collects the rounding
// errors of every product and every addition.
struct Dot2 {
  double s = 0.0, c = 0.0;
  __device__ __forceinline__ void add_prod(double a, double b) {
    const ddv p = two_prod(a, b);
    const ddv t = two_sum(s, p.hi);
    s = t.hi;
    c += t.lo + p.lo;
  }
  // (a_hi + a_lo)(b_hi + b_lo) with the lo x lo term dropped (2^-106 relative)
  __device__ __forceinline__ void add_prod_dd(double ah, double al, double bh, double bl) {
    const ddv p = two_prod(ah, bh);
    const ddv t = two_sum(s, p.hi);
    s = t.hi;
    c += t.lo + (p.lo + (ah * bl + al * bh));
  }
  __device__ __forceinline__ ddv value() const { return quick_two_sum(s, c); }
};

// Block-wide sum of one ddv per thread (blockDim.x == kThreads) in a fixed
// tree order; the result is valid in thread 0.
template <int kThreads>
__device__ ddv block_sum(ddv v, ddv* sh) {
  sh[threadIdx.x] = v;
  __syncthreads();
#pragma unroll
  for (int w = kThreads / 2; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) sh[threadIdx.x] = add(sh[threadIdx.x], sh[threadIdx.x + w]);
    __syncthreads();
  }
  const ddv r = sh[0];
  __syncthreads();
  return r;
}

}  // namespace dd

namespace mp2dd {

using dd::ddv;
constexpr int kE = 32;         // edge of the (a, b) tile
constexpr int kPC = 32;        // aux chunk
constexpr int kThreads = 256;  // 16 x 16 threads, 2 x 2 elements each
constexpr int kLd = kPC + 1;

__host__ __device__ inline long long pair_offset(long long i, long long n) {
  return i * n - i * (i - 1) / 2;
}

struct Params {
  const double* B;  // (nocc, nvir, naux)
  const double* eps_occ;
  const double* eps_vir;
  int nocc, nvir, naux;
  long long pair_begin, pair_end;
  double* block_totals;   // [gridDim.x][2]
  double* pair_partials;  // nullable, (nocc, nocc, 2): E_ij as hi, lo
};

// E_ij = sum_ab T_ab (2 T_ab - T_ba) / (e_i + e_j - e_a - e_b) for one
// unordered pair per iteration (weight 2 for i < j into the block total).
__global__ void __launch_bounds__(kThreads) energy_kernel(Params p) {
  __shared__ double tIa[kE][kLd], tJb[kE][kLd], tIb[kE][kLd], tJa[kE][kLd];
  __shared__ ddv red[kThreads];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  ddv total{0.0, 0.0};
  for (long long pid = p.pair_begin + blockIdx.x; pid < p.pair_end; pid += gridDim.x) {
    // pair (i, j), i <= j, from its row-major id
    long long lo = 0, hi = p.nocc - 1;
    while (lo < hi) {
      const long long mid = (lo + hi + 1) / 2;
      if (pair_offset(mid, p.nocc) <= pid) lo = mid; else hi = mid - 1;
    }
    const int i = (int)lo, j = (int)(i + (pid - pair_offset(i, p.nocc)));
    const double* Bi = p.B + (size_t)i * p.nvir * p.naux;
    const double* Bj = p.B + (size_t)j * p.nvir * p.naux;
    const ddv eij = dd::two_sum(p.eps_occ[i], p.eps_occ[j]);
    ddv acc{0.0, 0.0};
    for (int a0 = 0; a0 < p.nvir; a0 += kE) {
      for (int b0 = 0; b0 < p.nvir; b0 += kE) {
        dd::Dot2 tab[2][2], tba[2][2];
        for (int p0 = 0; p0 < p.naux; p0 += kPC) {
          for (int e = threadIdx.x; e < kE * kPC; e += kThreads) {
            const int r = e / kPC, c = e % kPC;
            const bool pc = p0 + c < p.naux;
            const bool ra = a0 + r < p.nvir, rb = b0 + r < p.nvir;
            const size_t oa = (size_t)(a0 + r) * p.naux + p0 + c;
            const size_t ob = (size_t)(b0 + r) * p.naux + p0 + c;
            tIa[r][c] = (pc && ra) ? Bi[oa] : 0.0;
            tJa[r][c] = (pc && ra) ? Bj[oa] : 0.0;
            tJb[r][c] = (pc && rb) ? Bj[ob] : 0.0;
            tIb[r][c] = (pc && rb) ? Bi[ob] : 0.0;
          }
          __syncthreads();
#pragma unroll 4
          for (int c = 0; c < kPC; ++c) {
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
              for (int v = 0; v < 2; ++v) {
                const int ra = 2 * ty + u, rb = 2 * tx + v;
                tab[u][v].add_prod(tIa[ra][c], tJb[rb][c]);  // T_ab = B_i[a] . B_j[b]
                tba[u][v].add_prod(tIb[rb][c], tJa[ra][c]);  // T_ba = B_i[b] . B_j[a]
              }
          }
          __syncthreads();
        }
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int v = 0; v < 2; ++v) {
            const int a = a0 + 2 * ty + u, b = b0 + 2 * tx + v;
            if (a >= p.nvir || b >= p.nvir) continue;
            const ddv t = tab[u][v].value(), tt = tba[u][v].value();
            const ddv ev = dd::two_sum(p.eps_vir[a], p.eps_vir[b]);
            const ddv den = dd::sub(eij, ev);
            const ddv num = dd::mul(t, dd::sub(dd::mul_d(t, 2.0), tt));
            acc = dd::add(acc, dd::div(num, den));
          }
      }
    }
    const ddv eij_sum = dd::block_sum<kThreads>(acc, red);
    if (threadIdx.x == 0) {
      if (p.pair_partials) {
        double* pp = p.pair_partials;
        pp[((size_t)i * p.nocc + j) * 2] = eij_sum.hi;
        pp[((size_t)i * p.nocc + j) * 2 + 1] = eij_sum.lo;
        pp[((size_t)j * p.nocc + i) * 2] = eij_sum.hi;
        pp[((size_t)j * p.nocc + i) * 2 + 1] = eij_sum.lo;
      }
      total = dd::add(total, i < j ? ddv{2.0 * eij_sum.hi, 2.0 * eij_sum.lo} : eij_sum);
    }
  }
  if (threadIdx.x == 0) {
    p.block_totals[2 * blockIdx.x] = total.hi;
    p.block_totals[2 * blockIdx.x + 1] = total.lo;
  }
}

// energy[0..1] = sum of the n block totals, in a fixed order.
__global__ void __launch_bounds__(kThreads) reduce_kernel(const double* totals, int n,
                                                          double* energy) {
  __shared__ ddv red[kThreads];
  ddv acc{0.0, 0.0};
  for (int k = threadIdx.x; k < n; k += kThreads)
    acc = dd::add(acc, ddv{totals[2 * k], totals[2 * k + 1]});
  const ddv s = dd::block_sum<kThreads>(acc, red);
  if (threadIdx.x == 0) {
    energy[0] = s.hi;
    energy[1] = s.lo;
  }
}

}  // namespace mp2dd

namespace gdd {

using dd::ddv;
constexpr int kT = 16;  // 16 x 16 outputs per block, one per thread
constexpr int kKC = 16;

struct Params {
  const double *Ah, *Al, *Bh, *Bl;
  int a_kmajor, b_kmajor;
  long long sA, sB, sC;
  double *Ch, *Cl;
  int M, N, K;
};

__device__ __forceinline__ double ld(const double* X, size_t off, bool ok) {
  return (X != nullptr && ok) ? X[off] : 0.0;
}

__global__ void __launch_bounds__(kT* kT) gemm_kernel(Params p) {
  __shared__ double ah[kT][kKC + 1], al[kT][kKC + 1], bh[kKC][kT + 1], bl[kKC][kT + 1];
  const int tx = threadIdx.x % kT, ty = threadIdx.x / kT;
  const int m0 = blockIdx.y * kT, n0 = blockIdx.x * kT;
  const long long bt = blockIdx.z;
  const double* Ah = p.Ah + bt * p.sA;
  const double* Al = p.Al ? p.Al + bt * p.sA : nullptr;
  const double* Bh = p.Bh + bt * p.sB;
  const double* Bl = p.Bl ? p.Bl + bt * p.sB : nullptr;
  dd::Dot2 acc;
  for (int k0 = 0; k0 < p.K; k0 += kKC) {
    {
      // A tile: rows m0.., columns k0.. ; B tile: rows k0.., columns n0..
      const int r = threadIdx.x / kKC, c = threadIdx.x % kKC;
      const int m = m0 + r, k = k0 + c;
      const bool okA = m < p.M && k < p.K;
      const size_t oA = p.a_kmajor ? (size_t)m * p.K + k : (size_t)k * p.M + m;
      ah[r][c] = ld(Ah, oA, okA);
      al[r][c] = ld(Al, oA, okA);
      const int kb = k0 + r, n = n0 + c;
      const bool okB = kb < p.K && n < p.N;
      const size_t oB = p.b_kmajor ? (size_t)n * p.K + kb : (size_t)kb * p.N + n;
      bh[r][c] = ld(Bh, oB, okB);
      bl[r][c] = ld(Bl, oB, okB);
    }
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < kKC; ++c) acc.add_prod_dd(ah[ty][c], al[ty][c], bh[c][tx], bl[c][tx]);
    __syncthreads();
  }
  const int m = m0 + ty, n = n0 + tx;
  if (m < p.M && n < p.N) {
    const ddv v = acc.value();
    const size_t o = bt * p.sC + (size_t)m * p.N + n;
    p.Ch[o] = v.hi;
    if (p.Cl) p.Cl[o] = v.lo;
  }
}

}  // namespace gdd
}  // namespace tt

using namespace tt;

extern "C" {

size_t tt_mp2_dd_workspace_bytes(int nocc, int nvir, int naux) {
  if (nocc <= 0 || nvir <= 0 || naux <= 0) return 0;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (size_t)4 * sms * 2 * sizeof(double);
}

int tt_mp2_energy_dd(const double* B, const double* eps_occ, const double* eps_vir, int nocc,
                     int nvir, int naux, long long pair_begin, long long pair_end,
                     void* workspace, size_t workspace_bytes, double* energy,
                     double* pair_partials, void* stream) {
  if (!B || !eps_occ || !eps_vir || !workspace || !energy) return TT_ERR_NULL;
  if (nocc <= 0 || nvir <= 0 || naux <= 0) return TT_ERR_SHAPE;
  const long long np = (long long)nocc * (nocc + 1) / 2;
  if (pair_begin < 0 || pair_end < pair_begin || pair_end > np) return TT_ERR_SHAPE;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  int sms = 0;
  TT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = 4 * sms;
  if (workspace_bytes < (size_t)grid * 2 * sizeof(double)) return TT_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  if (pair_partials)
    TT_CUDA(cudaMemsetAsync(pair_partials, 0, (size_t)nocc * nocc * 2 * sizeof(double), s));
  mp2dd::Params p{B, eps_occ, eps_vir, nocc, nvir, naux, pair_begin, pair_end,
                  static_cast<double*>(workspace), pair_partials};
  mp2dd::energy_kernel<<<grid, mp2dd::kThreads, 0, s>>>(p);
  TT_CUDA(cudaGetLastError());
  mp2dd::reduce_kernel<<<1, mp2dd::kThreads, 0, s>>>(static_cast<double*>(workspace), grid,
                                                     energy);
  return cuda_status(cudaGetLastError());
}

int tt_gemm_dd(const double* A_hi, const double* A_lo, int a_kmajor, long long strideA,
               const double* B_hi, const double* B_lo, int b_kmajor, long long strideB,
               double* C_hi, double* C_lo, long long strideC, int M, int N, int K, int batch,
               void* stream) {
  if (!A_hi || !B_hi || !C_hi) return TT_ERR_NULL;
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || batch > 65535) return TT_ERR_SHAPE;
  if (strideC < (long long)M * N) return TT_ERR_SHAPE;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  gdd::Params p{A_hi, A_lo, B_hi, B_lo, a_kmajor, b_kmajor, strideA, strideB, strideC,
                C_hi, C_lo, M, N, K};
  const dim3 grid((N + gdd::kT - 1) / gdd::kT, (M + gdd::kT - 1) / gdd::kT, batch);
  if (grid.y > 65535) return TT_ERR_SHAPE;
  gdd::gemm_kernel<<<grid, gdd::kT * gdd::kT, 0, (cudaStream_t)stream>>>(p);
  return cuda_status(cudaGetLastError());
}

}  // extern "C"
