// DF-MP2 pair-energy contraction on tcgen05 int8 tensor cores (Ozaki scheme).
//
// Math (the reference's trntensor/quantum.py:87-100; device kernel
// trntensor/nki/_kernels.py:119-207):
//   E = sum_{i,j} sum_{a,b} T_ab (2 T_ab - T_ba) / (e_i + e_j - e_a - e_b),
//   T = B_i . B_j^T   (B_i = B[i], nvir x naux, aux fastest).
//
// Why int8: tcgen05's fp32 accumulation of tf32 products rounds toward
// zero, so a K = 6144 contraction in 3xTF32 comes out biased by ~1e-4
// (measured), far outside the 1e-6 energy tolerance. Integer MMAs
// accumulate exactly. Each B row r = (i, a) is written as
//     B[r, P] = s_r * (q1 + q2 / 2^8 + q3 / 2^16)[r, P] + O(s_r 2^-17),
// s_r a power of two, q_t int8 ("slices", Ozaki et al. error-free
// splitting with a per-row exponent; format in ozaki_digits.cuh), and
//     T_ab = s_a s_b (L2 + L3 / 2^8 + L4 / 2^16),
//     L2 = Q1.Q1^T, L3 = Q1.Q2^T + Q2.Q1^T, L4 = Q1.Q3^T + Q2.Q2^T + Q3.Q1^T
// are six exact int8 GEMMs accumulated in int32 TMEM columns (one column
// block per level). Dropped terms are O(2^-23) relative and unbiased.
//
// Work decomposition: unordered occupied pairs i <= j (E_ij == E_ji, weight
// 2 for i < j), square 128 x 128 virtual blocks A <= B covering the upper
// triangle a <= b. Per (pair, block) a CTA runs two phases over the full aux
// range: x = T[A,B] (operands B_i[A], B_j[B]), whose fp32 value is parked in
// TMEM columns 384..511, then y = (T[B,A])^T (operands B_j[A], B_i[B]), so
// that T_ab and its exchange partner T_ba share a TMEM lane and column. The
// epilogue adds the (a,b) and (b,a) terms: x(2x-y) + y(2y-x), weight 1 for
// a < b, 1/2 for a == b, 0 for a > b.
//
// Roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer, warps 2..9 = epilogue (lane quarter = warp % 4, column half =
// (warp - 2) / 4).
#pragma once
#include "ozaki_digits.cuh"
#include "ptx.cuh"

namespace tt {
namespace mp2 {

constexpr int kBlk = 128;                 // virtual block edge (M = N = 128)
constexpr int kKC = 64;                   // aux elements (bytes) per stage
constexpr int kSlices = 3;
constexpr int kStages = 4;
constexpr int kSliceTile = kBlk * kKC;    // 8 KB
constexpr int kOperandBytes = kSlices * kSliceTile;  // 24 KB
constexpr int kStageBytes = 2 * kOperandBytes;       // A and B: 48 KB
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
// Diagonal blocks (A == B) of an i != j pair need y = x^T: x is exchanged
// through a padded shared-memory half-tile (64 rows x 129 floats) in two rounds.
constexpr int kTLd = kBlk + 1;
constexpr int kTBytes = (kBlk / 2) * kTLd * 4;
constexpr int kSmemBytes = kStages * kStageBytes + kTBytes + 1024 + 256;
constexpr int kColStash = 3 * kBlk;       // TMEM column of the parked x

struct Params {
  const float* scale;    // (nocc, nvir) power-of-two row scales s_r
  const float* eps_occ;
  const float* eps_vir;
  int nocc, nvir, naux_pad;
  long long pair_begin, pair_end;
  int nblk;              // ceil(nvir / 128)
  // Which (pair, block) items this launch runs (pairs in [pair_begin, pair_end)):
  //   0: all of them;
  //   1: the two-phase items only, i < j and A < B (strict pair q_begin on);
  //   2: the one-phase items only: A == B for every pair, then A < B for the
  //      i == j pairs, whose rows are diag_lo, diag_lo + 1, ...
  // Launches of one kind run items of equal length, so the CTAs stay in step
  // and read the same operand rows at the same time.
  int mode;
  long long q_begin;
  int diag_lo;
  long long n_items;
  double* energy;
  double* pair_partials;
  int* err;
  long long* prof;  // optional per-CTA wait-cycle counters (TT_MP2_PROFILE builds)
};

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

struct Item {
  int i, j, a0, b0;
  // One accumulation phase is enough when y follows from x: i == j gives
  // T symmetric (y = x), a diagonal block gives y = x^T.
  __device__ bool single() const { return i == j || a0 == b0; }
};
// A < B from its row-major index among the nblk (nblk - 1) / 2 off-diagonal blocks
__device__ inline void offdiag_decode(int r, int nblk, int& A, int& B) {
  A = 0;
  while (r >= nblk - 1 - A) {
    r -= nblk - 1 - A;
    ++A;
  }
  B = A + 1 + r;
}
__device__ inline Item item_decode(long long w, const Params& p) {
  Item it;
  int A = 0, B = 0;
  if (p.mode == 1) {
    const int nodp = p.nblk * (p.nblk - 1) / 2;
    // strict pairs i < j of n rows enumerate like pairs i <= j' of n - 1 rows
    int jj;
    pair_decode(p.q_begin + w / nodp, p.nocc - 1, it.i, jj);
    it.j = jj + 1;
    offdiag_decode((int)(w % nodp), p.nblk, A, B);
  } else if (p.mode == 2) {
    const long long nd = (p.pair_end - p.pair_begin) * p.nblk;
    if (w < nd) {
      pair_decode(p.pair_begin + w / p.nblk, p.nocc, it.i, it.j);
      A = B = (int)(w % p.nblk);
    } else {
      const int nodp = p.nblk * (p.nblk - 1) / 2;
      w -= nd;
      it.i = it.j = p.diag_lo + (int)(w / nodp);
      offdiag_decode((int)(w % nodp), p.nblk, A, B);
    }
  } else {
    const int nbp = p.nblk * (p.nblk + 1) / 2;
    pair_decode(p.pair_begin + w / nbp, p.nocc, it.i, it.j);
    int r = (int)(w % nbp);
    while (r >= p.nblk - A) {
      r -= p.nblk - A;
      ++A;
    }
    B = A + r;
  }
  it.a0 = A * kBlk;
  it.b0 = B * kBlk;
  return it;
}

using ozd::level_combine;

static __global__ void __launch_bounds__(kThreads, 1)
    energy_kernel(const __grid_constant__ CUtensorMap mapQ, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* tbuf = (float*)(smem + kStages * kStageBytes);
  uint64_t* full = (uint64_t*)(smem + kStages * kStageBytes + kTBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* final_bar = acc_empty + 1;
  uint32_t* tmem_slot = (uint32_t*)(final_bar + 1);
  double* red = (double*)(tmem_slot + 2);  // kEpiWarps doubles

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long n_items = p.n_items;
  const int nkc = p.naux_pad / kKC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 32 * kEpiWarps);
    mbar_init(final_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&mapQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (long long w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
        const Item t = item_decode(w, p);
        const int nph = t.single() ? 1 : 2;
        for (int ph = 0; ph < nph && ok; ++ph) {
          const int occA = ph == 0 ? t.i : t.j;
          const int occB = ph == 0 ? t.j : t.i;
          for (int kc = 0; kc < nkc; ++kc, ++it) {
            const int s = it % kStages;
            if (!mbar_wait(&empty[s], ((it / kStages) & 1u) ^ 1u, p.err, kDevTimeoutEmpty)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + s * kStageBytes;
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            tma_load_4d(st, &mapQ, &full[s], kc * kKC, t.a0, occA, 0);
            tma_load_4d(st + kOperandBytes, &mapQ, &full[s], kc * kKC, t.b0, occB, 0);
          }
        }
      }
      const uint32_t issued = it;
      for (uint32_t k = (issued > kStages ? issued - kStages : 0); k < issued; ++k)
        mbar_wait_drain(&full[k % kStages], (k / kStages) & 1u);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8(kBlk, kBlk, 0, 0);
      uint32_t it = 0, round = 0;
#ifdef TT_MP2_PROFILE
      long long wait_acc = 0, wait_full = 0;
      const long long t_begin = clock64();
#endif
      bool ok = true;
      for (long long w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
        const int nph = item_decode(w, p).single() ? 1 : 2;
        for (int ph = 0; ph < nph && ok; ++ph, ++round) {
#ifdef TT_MP2_PROFILE
          long long t0 = clock64();
#endif
          if (!mbar_wait(acc_empty, (round & 1u) ^ 1u, p.err, kDevTimeoutAccFree)) {
            ok = false;
            break;
          }
#ifdef TT_MP2_PROFILE
          wait_acc += clock64() - t0;
#endif
          tc_fence_after();
          for (int kc = 0; kc < nkc; ++kc, ++it) {
            const int s = it % kStages;
#ifdef TT_MP2_PROFILE
            long long t1 = clock64();
#endif
            if (!mbar_wait(&full[s], (it / kStages) & 1u, p.err, kDevTimeoutFull)) {
              ok = false;
              break;
            }
#ifdef TT_MP2_PROFILE
            wait_full += clock64() - t1;
#endif
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + s * kStageBytes);
            const uint32_t sb = sa + kOperandBytes;
#pragma unroll
            for (int ks = 0; ks < kKC / 32; ++ks) {
              uint64_t a[3], b[3];
#pragma unroll
              for (int t = 0; t < 3; ++t) {
                a[t] = smem_desc(sa + t * kSliceTile + ks * 32, 16, 512, 4);
                b[t] = smem_desc(sb + t * kSliceTile + ks * 32, 16, 512, 4);
              }
              const uint32_t first = (kc | ks) != 0;
              // Grouped by A slice so that each A slice is read from shared
              // memory once per 32-wide k-step (collector buffer reuse).
#ifndef TT_MP2_NO_COLLECTOR
              mma_i8_fill(tmem + 0 * kBlk, a[0], b[0], idesc, first);
              mma_i8_use(tmem + 1 * kBlk, a[0], b[1], idesc, first);
              mma_i8_lastuse(tmem + 2 * kBlk, a[0], b[2], idesc, first);
              mma_i8_fill(tmem + 1 * kBlk, a[1], b[0], idesc, 1);
              mma_i8_lastuse(tmem + 2 * kBlk, a[1], b[1], idesc, 1);
#else
              mma_i8(tmem + 0 * kBlk, a[0], b[0], idesc, first);
              mma_i8(tmem + 1 * kBlk, a[0], b[1], idesc, first);
              mma_i8(tmem + 2 * kBlk, a[0], b[2], idesc, first);
              mma_i8(tmem + 1 * kBlk, a[1], b[0], idesc, 1);
              mma_i8(tmem + 2 * kBlk, a[1], b[1], idesc, 1);
#endif
              mma_i8(tmem + 2 * kBlk, a[2], b[0], idesc, 1);
            }
            mma_commit(&empty[s]);
          }
          if (ok) mma_commit(acc_full);
        }
      }
      mma_commit(final_bar);
      mbar_wait_drain(final_bar, 0);
#ifdef TT_MP2_PROFILE
      if (p.prof) {
        p.prof[blockIdx.x * 4 + 0] = clock64() - t_begin;
        p.prof[blockIdx.x * 4 + 1] = wait_full;
        p.prof[blockIdx.x * 4 + 2] = wait_acc;
      }
#endif
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int q = warp & 3;            // TMEM lane quarter
    const int c0 = (ew >> 2) * (kBlk / 2);  // this warp's 64-column half
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    double my_energy = 0.0;
    uint32_t round = 0;
    for (long long w = blockIdx.x; w < n_items; w += gridDim.x) {
      const Item t = item_decode(w, p);
      const int a = t.a0 + row;
      const bool arow = a < p.nvir;
      // ---- phase x: park s_ia s_jb (L2 + L3/2^8 + L4/2^16) in the stash columns
      if (!group_all<32 * kEpiWarps>(mbar_wait(acc_full, round & 1u, p.err, kDevTimeoutAcc)))
        break;
      tc_fence_after();
      {
        const float sa = arow ? __ldg(p.scale + (long long)t.i * p.nvir + a) : 0.f;
        for (int c = c0; c < c0 + kBlk / 2; c += 16) {
          int l2[16], l3[16], l4[16];
          tmem_ld16i(lane_base + 0 * kBlk + c, l2);
          tmem_ld16i(lane_base + 1 * kBlk + c, l3);
          tmem_ld16i(lane_base + 2 * kBlk + c, l4);
          tmem_ld_wait();
          float x[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int b = t.b0 + c + k;
            const float sb = b < p.nvir ? __ldg(p.scale + (long long)t.j * p.nvir + b) : 0.f;
            x[k] = level_combine(l2[k], l3[k], l4[k]) * (sa * sb);
          }
          tmem_st16(lane_base + kColStash + c, x);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
      ++round;
      double acc = 0.0;
      const float eija = arow ? (__ldg(p.eps_occ + t.i) + __ldg(p.eps_occ + t.j)) -
                                    __ldg(p.eps_vir + a)
                              : 0.f;
      // sum over this thread's 16 columns starting at c of the (a,b)+(b,a) terms
      auto chunk_energy = [&](int c, const float (&x)[16], const float (&y)[16]) {
        float part = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int b = t.b0 + c + k;
          if (arow && b < p.nvir && a <= b) {
            // 1/den by the hardware reciprocal (relative error ~1e-7,
            // unbiased at the level the energy tolerance cares about)
            const float inv = __frcp_rn(eija - __ldg(p.eps_vir + b));
            float v = 2.f * (x[k] * x[k] - x[k] * y[k] + y[k] * y[k]) * inv;
            if (a == b) v *= 0.5f;
            part += v;
          }
        }
        return (double)part;
      };
      if (t.i == t.j) {
        // ---- T_ii is symmetric: y = x
        for (int c = c0; c < c0 + kBlk / 2; c += 16) {
          float x[16];
          tmem_ld16(lane_base + kColStash + c, x);
          tmem_ld_wait();
          acc += chunk_energy(c, x, x);
        }
      } else if (t.a0 == t.b0) {
        // ---- diagonal block: y[a][b] = x[b][a], exchanged through shared memory.
        // Round r: the warps holding rows [64r, 64r+64) publish them; the warps
        // whose columns are [64r, 64r+64) read their transposed values.
        for (int r = 0; r < 2; ++r) {
          asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps));
          if ((q >> 1) == r) {
            for (int c = c0; c < c0 + kBlk / 2; c += 16) {
              float x[16];
              tmem_ld16(lane_base + kColStash + c, x);
              tmem_ld_wait();
#pragma unroll
              for (int k = 0; k < 16; ++k) tbuf[(row - 64 * r) * kTLd + c + k] = x[k];
            }
          }
          asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps));
          if ((c0 >> 6) == r) {
            for (int c = c0; c < c0 + kBlk / 2; c += 16) {
              float x[16], y[16];
              tmem_ld16(lane_base + kColStash + c, x);
              tmem_ld_wait();
#pragma unroll
              for (int k = 0; k < 16; ++k) y[k] = tbuf[(c + k - 64 * r) * kTLd + row];
              acc += chunk_energy(c, x, y);
            }
          }
        }
      } else {
        // ---- phase y: combine with the parked x and reduce the energy
        if (!group_all<32 * kEpiWarps>(mbar_wait(acc_full, round & 1u, p.err, kDevTimeoutAcc)))
          break;
        tc_fence_after();
        const float sa = arow ? __ldg(p.scale + (long long)t.j * p.nvir + a) : 0.f;
        // Combine all of this thread's y values into registers first so the
        // accumulator goes back to the MMA warp before the energy is summed.
        float y[kBlk / 2];
#pragma unroll
        for (int cc = 0; cc < kBlk / 32; ++cc) {
          const int c = c0 + 16 * cc;
          int l2[16], l3[16], l4[16];
          tmem_ld16i(lane_base + 0 * kBlk + c, l2);
          tmem_ld16i(lane_base + 1 * kBlk + c, l3);
          tmem_ld16i(lane_base + 2 * kBlk + c, l4);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int b = t.b0 + c + k;
            const float sb = b < p.nvir ? __ldg(p.scale + (long long)t.i * p.nvir + b) : 0.f;
            y[16 * cc + k] = level_combine(l2[k], l3[k], l4[k]) * (sa * sb);
          }
        }
        tc_fence_before();
        mbar_arrive(acc_empty);
        ++round;
#pragma unroll
        for (int cc = 0; cc < kBlk / 32; ++cc) {
          const int c = c0 + 16 * cc;
          float x[16];
          tmem_ld16(lane_base + kColStash + c, x);
          tmem_ld_wait();
          acc += chunk_energy(c, x, *reinterpret_cast<const float(*)[16]>(y + 16 * cc));
        }
      }
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
    if (lane == 0) red[ew] = my_energy;
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int k = 0; k < kEpiWarps; ++k) tot += red[k];
    if (tot != 0.0) atomicAdd(p.energy, tot);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Ozaki split of one row per warp into the slice format of ozaki_digits.cuh
// (row scale s, three int8 slice planes).
// `plane` is the distance in bytes between the three slice planes (rows of
// a larger matrix can be split piecewise into one set of planes).
static __global__ void split_kernel(const float* __restrict__ x, int8_t* __restrict__ q,
                             float* __restrict__ scale, long long rows, int cols, int cols_pad,
                             long long plane) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += warps) {
    const float* xr = x + r * cols;
    float m = 0.f;
    for (int c = lane; c < cols; c += 32) m = ozd::absmax(m, __ldg(xr + c));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = ozd::scale_for_max(m);
    const float inv1 = ozd::inv_scale(s);
    if (lane == 0) scale[r] = s;
    int8_t* q1 = q + r * cols_pad;
    int8_t* q2 = q1 + plane;
    int8_t* q3 = q2 + plane;
    const float inv[4] = {inv1, inv1, inv1, inv1};
    for (int c = lane * 4; c < cols_pad; c += 128) {
      float v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = (c + k < cols) ? __ldg(xr + c + k) : 0.f;
      uint32_t w1, w2, w3;
      ozd::split4(v, inv, w1, w2, w3);
      *reinterpret_cast<uint32_t*>(q1 + c) = w1;
      *reinterpret_cast<uint32_t*>(q2 + c) = w2;
      *reinterpret_cast<uint32_t*>(q3 + c) = w3;
    }
  }
}

// Statistics of the three-digit format over rows of x (one warp per row),
// accumulated into acc[0..2] (fp64 atomics, one per block and value):
//   acc[0] += sum_r n_r s_r^2 u2_r,  acc[1] += sum_r n_r s_r^2 u3_r,
//   acc[2] += sum_r n_r,
// n_r = sum_P x_rP^2, s_r the row scale and u2_r, u3_r the sums of squares of
// the row's second and third digits. The digit products q2 q3' + q3 q2' are
// the largest terms the energy kernel drops; these sums give the size of
// that error relative to the energy when the rows' inner products behave
// like random sums (the host turns them into an estimate). The digits are
// computed exactly as split_kernel computes them.
static __global__ void range_stats_kernel(const float* __restrict__ x, long long rows, int cols,
                                          double* __restrict__ acc) {
  __shared__ double part[3][8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  double a2 = 0.0, a3 = 0.0, an = 0.0;
  for (long long r = blockIdx.x * (long long)(blockDim.x >> 5) + warp; r < rows; r += warps) {
    const float* xr = x + r * cols;
    float m = 0.f;
    for (int c = lane; c < cols; c += 32) m = ozd::absmax(m, __ldg(xr + c));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = ozd::scale_for_max(m);
    const float inv = ozd::inv_scale(s);
    double n = 0.0, u2 = 0.0, u3 = 0.0;
    for (int c = lane; c < cols; c += 32) {
      const float v = __ldg(xr + c);
      const int z = ozd::digit_word(v, inv);
      const int q2 = ((z >> 8) & 0xFF) - 128, q3 = (z & 0xFF) - 128;
      n += (double)v * v;
      u2 += (double)(q2 * q2);
      u3 += (double)(q3 * q3);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      n += __shfl_xor_sync(0xffffffffu, n, o);
      u2 += __shfl_xor_sync(0xffffffffu, u2, o);
      u3 += __shfl_xor_sync(0xffffffffu, u3, o);
    }
    const double w = n * (double)s * (double)s;
    a2 += w * u2;
    a3 += w * u3;
    an += n;
  }
  if (lane == 0) {
    part[0][warp] = a2;
    part[1][warp] = a3;
    part[2][warp] = an;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[threadIdx.x][w];
    atomicAdd(acc + threadIdx.x, t);
  }
}

}  // namespace mp2
}  // namespace tt
