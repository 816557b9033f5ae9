// DF-MP2 pair-energy contraction on tcgen05 tensor cores, 3xTF32.
//
// Math (the reference's trntensor/quantum.py:87-100 and the device kernel
// trntensor/nki/_kernels.py:119-207 compute the same sum):
//   E = sum_{i,j} sum_{a,b} T_ab (2 T_ab - T_ba) / (e_i + e_j - e_a - e_b),
//   T = B_i . B_j^T  (B_i = B[i] is nvir x naux, row-major, aux fastest).
//
// Work decomposition (B200-specific, not the reference's):
//  * only unordered occupied pairs i <= j are visited (E_ij == E_ji, so an
//    i < j pair is weighted 2);
//  * the nvir x nvir pair matrix is covered by rectangles of 128 rows (block
//    A) x 256 columns (block B) that cover its upper triangle a <= b;
//  * one CTA computes, for a rectangle, two accumulators in TMEM:
//        acc0[a][b] = sum_P B_i[a,P] B_j[b,P] = T_ab
//        acc1[a][b] = sum_P B_j[a,P] B_i[b,P] = T_ba
//    so T_ab and its exchange partner T_ba sit in the same TMEM lane and
//    column; the epilogue adds the (a,b) and (b,a) terms together:
//        x(2x-y) + y(2y-x) = 2(x^2 - xy + y^2)
//    with weight 1 for a < b, 1/2 for a == b and 0 for a > b;
//  * each fp32 operand is pre-split into hi = tf32(x) and lo = tf32(x - hi);
//    acc += hi.hi + hi.lo + lo.hi (3xTF32) restores fp32-level accuracy.
//
// Roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer, warps 2..5 = epilogue (TMEM lane quarter = warp % 4).
#pragma once
#include "ptx.cuh"

namespace tt {
namespace mp2tf {

constexpr int kM = 128;               // rows per rectangle (block A)
constexpr int kN = 256;               // columns per rectangle (block B)
constexpr int kKC = 16;               // aux elements per pipeline stage (64 B)
constexpr int kStages = 4;
constexpr int kTileA = kM * kKC * 4;  // 8 KB
constexpr int kTileB = kN * kKC * 4;  // 16 KB
constexpr int kStageBytes = 2 * kTileA + 2 * kTileB;  // hi + lo of A and B: 48 KB
constexpr int kThreads = 192;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;

struct Params {
  const float* eps_occ;
  const float* eps_vir;
  int nocc, nvir, naux_pad;
  long long pair_begin, pair_end;  // half-open range of linear i<=j pair ids
  int n_rects;                     // rectangles per pair
  double* energy;                  // += sum of all contributions
  double* pair_partials;           // optional (nocc, nocc), += E_ij and E_ji
  int* err;
};

// Linear id of the unordered pair (i, j), i <= j, row-major over i.
__host__ __device__ inline long long pair_offset(long long i, long long n) {
  return i * n - i * (i - 1) / 2;
}
__device__ inline void pair_decode(long long p, int n, int& i, int& j) {
  double nn = 2.0 * n + 1.0;
  long long ii = (long long)((nn - sqrt(nn * nn - 8.0 * (double)p)) * 0.5);
  if (ii < 0) ii = 0;
  if (ii > n - 1) ii = n - 1;
  while (ii > 0 && pair_offset(ii, n) > p) --ii;
  while (ii + 1 < n && pair_offset(ii + 1, n) <= p) ++ii;
  i = (int)ii;
  j = (int)(ii + (p - pair_offset(ii, n)));
}
// Rectangle r of the upper-triangle cover: row block A (128 rows starting at
// a0 = 128*A), columns [b0, b0 + 256) with b0 = a0 + 256*t.
__host__ __device__ inline int rects_in_row(int A, int nvir) {
  int span = nvir - kM * A;
  return (span + kN - 1) / kN;
}
__host__ __device__ inline int rect_count(int nvir) {
  int nA = (nvir + kM - 1) / kM, c = 0;
  for (int A = 0; A < nA; ++A) c += rects_in_row(A, nvir);
  return c;
}
__device__ inline void rect_decode(int r, int nvir, int& a0, int& b0) {
  int A = 0;
  while (true) {
    int c = rects_in_row(A, nvir);
    if (r < c) break;
    r -= c;
    ++A;
  }
  a0 = kM * A;
  b0 = a0 + kN * r;
}

struct Item {
  int i, j, a0, b0;
};
__device__ inline Item item_decode(long long w, const Params& p) {
  Item it;
  long long pr = p.pair_begin + w / p.n_rects;
  pair_decode(pr, p.nocc, it.i, it.j);
  rect_decode((int)(w % p.n_rects), p.nvir, it.a0, it.b0);
  return it;
}

static __global__ void __launch_bounds__(kThreads, 1)
    energy_kernel(const __grid_constant__ CUtensorMap mapA_hi,
                  const __grid_constant__ CUtensorMap mapA_lo,
                  const __grid_constant__ CUtensorMap mapB_hi,
                  const __grid_constant__ CUtensorMap mapB_lo, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* final_bar = acc_empty + 1;
  uint32_t* tmem_slot = (uint32_t*)(final_bar + 1);
  double* red = (double*)(tmem_slot + 2);  // 4 doubles (8-byte aligned)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long n_items = (p.pair_end - p.pair_begin) * (long long)p.n_rects;
  const int nkc = p.naux_pad / kKC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 128);
    mbar_init(final_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&mapA_hi);
    tma_prefetch_desc(&mapA_lo);
    tma_prefetch_desc(&mapB_hi);
    tma_prefetch_desc(&mapB_lo);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  double my_energy = 0.0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (long long w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
        Item t = item_decode(w, p);
        for (int kc = 0; kc < nkc && ok; ++kc) {
          for (int g = 0; g < 2; ++g, ++it) {
            const int s = it % kStages;
            const uint32_t ph = (it / kStages) & 1u;
            if (!mbar_wait(&empty[s], ph ^ 1u, p.err, kDevTimeoutEmpty)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + s * kStageBytes;
            const int occA = g == 0 ? t.i : t.j;
            const int occB = g == 0 ? t.j : t.i;
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            tma_load_3d(st, &mapA_hi, &full[s], kc * kKC, t.a0, occA);
            tma_load_3d(st + kTileA, &mapA_lo, &full[s], kc * kKC, t.a0, occA);
            tma_load_3d(st + 2 * kTileA, &mapB_hi, &full[s], kc * kKC, t.b0, occB);
            tma_load_3d(st + 2 * kTileA + kTileB, &mapB_lo, &full[s], kc * kKC, t.b0, occB);
          }
        }
      }
      // Drain: wait until every issued stage has landed so that no bulk copy
      // is still writing into shared memory when the CTA exits.
      const uint32_t issued = it;
      for (uint32_t k = (issued > kStages ? issued - kStages : 0); k < issued; ++k) {
        mbar_wait_drain(&full[k % kStages], (k / kStages) & 1u);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kM, kN, 0, 0);
      uint32_t it = 0, titem = 0;
      bool ok = true;
      for (long long w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++titem) {
        if (!mbar_wait(acc_empty, (titem & 1u) ^ 1u, p.err, kDevTimeoutAccFree)) break;
        tc_fence_after();
        for (int kc = 0; kc < nkc && ok; ++kc) {
          for (int g = 0; g < 2; ++g, ++it) {
            const int s = it % kStages;
            const uint32_t ph = (it / kStages) & 1u;
            if (!mbar_wait(&full[s], ph, p.err, kDevTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + s * kStageBytes);
            const uint32_t d = tmem + g * kN;
#pragma unroll
            for (int ks = 0; ks < kKC / 8; ++ks) {
              const uint64_t ahi = smem_desc(sa + ks * 32, 16, 512, 4);
              const uint64_t alo = smem_desc(sa + kTileA + ks * 32, 16, 512, 4);
              const uint64_t bhi = smem_desc(sa + 2 * kTileA + ks * 32, 16, 512, 4);
              const uint64_t blo = smem_desc(sa + 2 * kTileA + kTileB + ks * 32, 16, 512, 4);
              mma_tf32(d, ahi, bhi, idesc, (kc | ks) != 0);
              mma_tf32(d, ahi, blo, idesc, 1);
              mma_tf32(d, alo, bhi, idesc, 1);
            }
            mma_commit(&empty[s]);
          }
        }
        if (ok) mma_commit(acc_full);
      }
      // All MMAs issued by this thread must finish before TMEM is freed.
      mma_commit(final_bar);
      mbar_wait_drain(final_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    uint32_t titem = 0;
    for (long long w = blockIdx.x; w < n_items; w += gridDim.x, ++titem) {
      if (!mbar_wait(acc_full, titem & 1u, p.err, kDevTimeoutAcc)) break;
      tc_fence_after();
      const Item t = item_decode(w, p);
      const int a = t.a0 + row;
      const bool arow = a < p.nvir;
      const float eij = __ldg(p.eps_occ + t.i) + __ldg(p.eps_occ + t.j);
      const float ea = arow ? __ldg(p.eps_vir + a) : 0.f;
      const float eija = eij - ea;
      double acc = 0.0;
      const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
      for (int c = 0; c < kN; c += 16) {
        float x[16], y[16];
        tmem_ld16(lane_base + c, x);
        tmem_ld16(lane_base + kN + c, y);
        tmem_ld_wait();
        float part = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int b = t.b0 + c + k;
          if (arow && b < p.nvir && a <= b) {
            const float den = eija - __ldg(p.eps_vir + b);
            float v = 2.f * (x[k] * x[k] - x[k] * y[k] + y[k] * y[k]) / den;
            if (a == b) v *= 0.5f;
            part += v;
          }
        }
        acc += (double)part;
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
      const double wgt = (t.i == t.j) ? 1.0 : 2.0;
      my_energy += wgt * acc;
      if (p.pair_partials != nullptr) {
        double s = acc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) {
          atomicAdd(p.pair_partials + (long long)t.i * p.nocc + t.j, s);
          if (t.i != t.j) atomicAdd(p.pair_partials + (long long)t.j * p.nocc + t.i, s);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) my_energy += __shfl_xor_sync(0xffffffffu, my_energy, o);
    if (lane == 0) red[warp - 2] = my_energy;
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    const double tot = red[0] + red[1] + red[2] + red[3];
    if (tot != 0.0) atomicAdd(p.energy, tot);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace mp2tf
}  // namespace tt
