// fp64 GEMM on int8 tensor cores (six-digit Ozaki scheme), for operands
// stored "K rows, M/N contiguous" (MN-major), batched:
//   C[b][m][n] = sum_k A[bA][k][m] B[b][k][n]        (fp64 in and out)
// Used for both steps of the fp64 AO->MO transform (precision="kahan").
//
// Each operand column (fixed m or n, all k) gets a power-of-two scale
// s = 2^(e-6) with max_k |X[k][c]| < 2^e and six int8 digits of
// Y = rint(X 2^40 / s) (|Y| < 2^46): the digit format of csrc/mp2_i8x5.cuh,
// one digit longer, per column instead of per row. C = sA_m sB_n
// sum_{l=0..5} L_l 2^-8l, where L_l collects the digit products q_a q'_b with
// a + b = l + 2 (21 exact int8 GEMMs, int32 sums exact while K <= 26214).
// Unlike the MP2 energy, whose sum averages the per-element errors, a GEMM
// output carries them directly: five digits left 5e-12 of max|C| in the
// AO->MO transform (measured against the fp64 CUDA-core path), six digits
// bound the representation error by 2^-47 and the dropped levels
// (a + b >= 8) by ~2^-46 of s_a s_b. Levels L0..L2 and L3..L5 are
// accumulated in two sweeps over K because six 128-column levels exceed
// TMEM's 512 columns; the epilogue writes sweep 0's fp64 partial into C and
// adds sweep 1's levels to it (each thread re-reads only what it wrote).
//
// Tile M = N = 128 (MN-major, 128B swizzle: the layout of ozaki_gemm.cuh),
// 4 stages of 48 KB: one 32-wide k-step of six digits of A and B (sweep 1)
// or two k-steps of three digits (sweep 0, k-step 1 at +3 slices), so both
// sweeps give the ring the same MMA work per stage.
// Roles: warp 0 TMA, warp 1 TMEM + MMA, warps 2..9 epilogue.
#pragma once
#include "ozaki_digits.cuh"
#include "ptx.cuh"

namespace tt {
namespace oz64 {

constexpr int kTile = 128;
constexpr int kKC = 32;
constexpr int kDigits = 6;
constexpr int kStages = 4;
constexpr int kSliceTile = kTile * kKC;             // 4 KB
constexpr int kOperandBytes = kDigits * kSliceTile;  // 24 KB
constexpr int kStageBytes = 2 * kOperandBytes;       // 48 KB
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
constexpr int kMaxK = 26214;  // K (2 * 64 * 128 + 4 * 128 * 128) < 2^31

__host__ __device__ constexpr int sweep_digits(int s) { return s == 0 ? 3 : kDigits; }

struct Params {
  const double* sA;  // [batchA][ldsA] column scales of A
  const double* sB;  // [batch][ldsB]
  long long ldsA, ldsB;
  double* C;
  long long ldc, strideC;
  int M, N, K, batch;
  int shared_A;  // 1: every batch uses A batch 0
  int tiles_m, tiles_n;
  int* err;
};

struct Tile {
  int b, m0, n0;
};
__device__ inline Tile tile_decode(long long w, const Params& p) {
  Tile t;
  const long long per_b = (long long)p.tiles_m * p.tiles_n;
  t.b = (int)(w / per_b);
  const int r = (int)(w % per_b);
  t.n0 = (r / p.tiles_m) * kTile;
  t.m0 = (r % p.tiles_m) * kTile;
  return t;
}

// a3/b3: tensor maps whose box holds digits 0..2 (sweep 0); a5/b5: all six.
static __global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap a3, const __grid_constant__ CUtensorMap a5,
                const __grid_constant__ CUtensorMap b3, const __grid_constant__ CUtensorMap b5,
                Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* final_bar = acc_empty + 1;
  uint32_t* tmem_slot = (uint32_t*)(final_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long n_tiles = (long long)p.tiles_m * p.tiles_n * p.batch;
  const int nkc = (p.K + kKC - 1) / kKC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 32 * kEpiWarps);
    mbar_init(final_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&a3);
    tma_prefetch_desc(&a5);
    tma_prefetch_desc(&b3);
    tma_prefetch_desc(&b5);
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
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (long long w = blockIdx.x; w < n_tiles && ok; w += gridDim.x) {
        const Tile t = tile_decode(w, p);
        const int bA = p.shared_A ? 0 : t.b;
        for (int sweep = 0; sweep < 2 && ok; ++sweep) {
          const CUtensorMap* ma = sweep ? &a5 : &a3;
          const CUtensorMap* mb = sweep ? &b5 : &b3;
          const int ksteps = sweep ? 1 : 2;  // k-steps per stage
          for (int kc = 0; kc < nkc; kc += ksteps, ++it) {
            const int s = it % kStages;
            if (!mbar_wait(&empty[s], ((it / kStages) & 1u) ^ 1u, p.err, kDevTimeoutEmpty)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + s * kStageBytes;
            const int nks = kc + ksteps <= nkc ? ksteps : nkc - kc;
            mbar_arrive_expect_tx(&full[s], 2u * nks * sweep_digits(sweep) * kSliceTile);
            for (int ks = 0; ks < nks; ++ks) {
              const int off = ks * 3 * kSliceTile;
              tma_load_4d(st + off, ma, &full[s], t.m0, (kc + ks) * kKC, bA, 0);
              tma_load_4d(st + kOperandBytes + off, mb, &full[s], t.n0, (kc + ks) * kKC, t.b, 0);
            }
          }
        }
      }
      const uint32_t issued = it;
      for (uint32_t k = (issued > kStages ? issued - kStages : 0); k < issued; ++k)
        mbar_wait_drain(&full[k % kStages], (k / kStages) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8(kTile, kTile, 1, 1);
      uint32_t it = 0, round = 0;
      bool ok = true;
      for (long long w = blockIdx.x; w < n_tiles && ok; w += gridDim.x) {
        for (int sweep = 0; sweep < 2 && ok; ++sweep, ++round) {
          if (!mbar_wait(acc_empty, (round & 1u) ^ 1u, p.err, kDevTimeoutAccFree)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int ksteps = sweep ? 1 : 2;
          for (int kc = 0; kc < nkc; kc += ksteps, ++it) {
            const int s = it % kStages;
            if (!mbar_wait(&full[s], (it / kStages) & 1u, p.err, kDevTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + s * kStageBytes);
            const uint32_t sb = sa + kOperandBytes;
            // MN-major SW128: 8 k-rows of 128 B per 1 KB atom, 32 k = 4 atoms
            if (sweep == 0) {
              const int nks = kc + 2 <= nkc ? 2 : nkc - kc;
              for (int ks = 0; ks < nks; ++ks) {
                uint64_t a[3], b[3];
#pragma unroll
                for (int d = 0; d < 3; ++d) {
                  a[d] = smem_desc(sa + (3 * ks + d) * kSliceTile, 8192, 1024, 2);
                  b[d] = smem_desc(sb + (3 * ks + d) * kSliceTile, 8192, 1024, 2);
                }
                const uint32_t acc = (kc | ks) != 0;
                mma_i8_fill(tmem + 0 * kTile, a[0], b[0], idesc, acc);
                mma_i8_use(tmem + 1 * kTile, a[0], b[1], idesc, acc);
                mma_i8_lastuse(tmem + 2 * kTile, a[0], b[2], idesc, acc);
                mma_i8_fill(tmem + 1 * kTile, a[1], b[0], idesc, 1);
                mma_i8_lastuse(tmem + 2 * kTile, a[1], b[1], idesc, 1);
                mma_i8(tmem + 2 * kTile, a[2], b[0], idesc, 1);
              }
            } else {
              uint64_t a[kDigits], b[kDigits];
#pragma unroll
              for (int d = 0; d < kDigits; ++d) {
                a[d] = smem_desc(sa + d * kSliceTile, 8192, 1024, 2);
                b[d] = smem_desc(sb + d * kSliceTile, 8192, 1024, 2);
              }
              const uint32_t acc = kc != 0;
              // L3 at column 0, L4 at 128, L5 at 256
              mma_i8_fill(tmem + 0 * kTile, a[0], b[3], idesc, acc);
              mma_i8_use(tmem + 1 * kTile, a[0], b[4], idesc, acc);
              mma_i8_lastuse(tmem + 2 * kTile, a[0], b[5], idesc, acc);
              mma_i8_fill(tmem + 0 * kTile, a[1], b[2], idesc, 1);
              mma_i8_use(tmem + 1 * kTile, a[1], b[3], idesc, 1);
              mma_i8_lastuse(tmem + 2 * kTile, a[1], b[4], idesc, 1);
              mma_i8_fill(tmem + 0 * kTile, a[2], b[1], idesc, 1);
              mma_i8_use(tmem + 1 * kTile, a[2], b[2], idesc, 1);
              mma_i8_lastuse(tmem + 2 * kTile, a[2], b[3], idesc, 1);
              mma_i8_fill(tmem + 0 * kTile, a[3], b[0], idesc, 1);
              mma_i8_use(tmem + 1 * kTile, a[3], b[1], idesc, 1);
              mma_i8_lastuse(tmem + 2 * kTile, a[3], b[2], idesc, 1);
              mma_i8_fill(tmem + 1 * kTile, a[4], b[0], idesc, 1);
              mma_i8_lastuse(tmem + 2 * kTile, a[4], b[1], idesc, 1);
              mma_i8(tmem + 2 * kTile, a[5], b[0], idesc, 1);
            }
            mma_commit(&empty[s]);
          }
          if (ok) mma_commit(acc_full);
        }
      }
      mma_commit(final_bar);
      mbar_wait_drain(final_bar, 0);
    }
  } else {
    // Each thread owns one row (its TMEM lane) and 64 columns of the tile in
    // both sweeps: sweep 0 writes the partial into C, sweep 1 completes it.
    const int ew = warp - 2;
    const int q = warp & 3;
    const int c0 = (ew >> 2) * (kTile / 2);
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const bool vec = (p.ldc % 2 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                     (p.strideC % 2 == 0);
    uint32_t round = 0;
    for (long long w = blockIdx.x; w < n_tiles; w += gridDim.x) {
      const Tile t = tile_decode(w, p);
      const int bA = p.shared_A ? 0 : t.b;
      const int m = t.m0 + row;
      const bool mrow = m < p.M;
      const double sa = mrow ? __ldg(p.sA + bA * p.ldsA + m) : 0.0;
      const double* sbp = p.sB + t.b * p.ldsB;
      double* crow = p.C + t.b * p.strideC + (long long)(mrow ? m : 0) * p.ldc + t.n0;
      bool ok = true;
      for (int sweep = 0; sweep < 2; ++sweep, ++round) {
        if (!group_all<32 * kEpiWarps>(mbar_wait(acc_full, round & 1u, p.err, kDevTimeoutAcc))) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int c = c0; c < c0 + kTile / 2; c += 16) {
          double v[16];
          if (sweep == 0) {
            int l0[16], l1[16], l2[16];
            tmem_ld16i(lane_base + 0 * kTile + c, l0);
            tmem_ld16i(lane_base + 1 * kTile + c, l1);
            tmem_ld16i(lane_base + 2 * kTile + c, l2);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 16; ++k)
              v[k] = ((double)l2[k] * (1.0 / 256.0) + (double)l1[k]) * (1.0 / 256.0) + (double)l0[k];
          } else {
            int l3[16], l4[16], l5[16];
            tmem_ld16i(lane_base + 0 * kTile + c, l3);
            tmem_ld16i(lane_base + 1 * kTile + c, l4);
            tmem_ld16i(lane_base + 2 * kTile + c, l5);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 16; ++k)
              v[k] = (((double)l5[k] * (1.0 / 256.0) + (double)l4[k]) * (1.0 / 256.0) +
                      (double)l3[k]) * (1.0 / 16777216.0);
          }
          if (!mrow) continue;
          const int nvalid = p.N - (t.n0 + c);
          if (vec && nvalid >= 16) {
            double2* d2 = reinterpret_cast<double2*>(crow + c);
#pragma unroll
            for (int k = 0; k < 16; k += 2) {
              const double s0 = sa * __ldg(sbp + t.n0 + c + k);
              const double s1 = sa * __ldg(sbp + t.n0 + c + k + 1);
              double2 o = make_double2(v[k] * s0, v[k + 1] * s1);
              if (sweep) {
                const double2 prev = d2[k / 2];
                o = make_double2(prev.x + o.x, prev.y + o.y);
              }
              d2[k / 2] = o;
            }
          } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              if (k < nvalid) {
                const double o = v[k] * (sa * __ldg(sbp + t.n0 + c + k));
                crow[c + k] = sweep ? crow[c + k] + o : o;
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(acc_empty);
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Column-scaled six-digit split of X[b][k][n] (fp64), in two streaming
// passes like the fp32 split of ozaki_gemm.cuh:
//   colmax_kernel: S[b][n] = power-of-two scale of column n (max over k);
//                  NaN for a column holding inf or NaN, 0 for a zero column;
//   slice_kernel : Q[d][b][k][n] int8 digits (row length npad, zero padding).
// A block covers 128 columns (4 per lane) and all k; its 8 warps take every
// 8th row.
constexpr int kSplitThreads = 256;
constexpr int kSplitCols = 128;

__device__ __forceinline__ void load4d(const double* xc, int nvalid, double (&v)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = j < nvalid ? __ldg(xc + j) : 0.0;
}

static __global__ void __launch_bounds__(kSplitThreads)
    colmax_kernel(const double* __restrict__ X, long long ldx, long long bsx, int batch, int K,
                  int N, int npad, double* __restrict__ S) {
  __shared__ double red[kSplitThreads / 32][kSplitCols];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int ncb = (npad + kSplitCols - 1) / kSplitCols;
  for (long long blk = blockIdx.x; blk < (long long)batch * ncb; blk += gridDim.x) {
    const int b = (int)(blk / ncb);
    const int n = (int)(blk % ncb) * kSplitCols + lane * 4;
    const int nvalid = N - n;
    const double* xc = X + b * bsx + n;
    double mx[4] = {0.0, 0.0, 0.0, 0.0};
    if (nvalid > 0) {
#pragma unroll 4
      for (int k = wp; k < K; k += kSplitThreads / 32) {
        double v[4];
        load4d(xc + (long long)k * ldx, nvalid, v);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mx[j] = fmax(mx[j], v[j] == v[j] ? fabs(v[j]) : __longlong_as_double(0x7ff0000000000000LL));
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) red[wp][lane * 4 + j] = mx[j];
    __syncthreads();
    if (threadIdx.x < kSplitCols) {
      double m = 0.0;
#pragma unroll
      for (int w = 0; w < kSplitThreads / 32; ++w) m = fmax(m, red[w][threadIdx.x]);
      const int nn = (int)(blk % ncb) * kSplitCols + threadIdx.x;
      double s = 0.0;
      if (!(m <= 1.7976931348623157e308))
        s = __longlong_as_double(0x7ff8000000000000LL);
      else if (m > 1.0e-290)
        s = ldexp(1.0, ilogb(m) + 1 - 6);  // m < 2^(ilogb + 1): |x / s| < 64
      if (nn < npad) S[(long long)b * npad + nn] = nn < N ? s : 0.0;
    }
    __syncthreads();
  }
}

static __global__ void __launch_bounds__(kSplitThreads)
    slice_kernel(const double* __restrict__ X, long long ldx, long long bsx, int batch, int K,
                 int N, int npad, const double* __restrict__ S, int8_t* __restrict__ Q) {
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  constexpr int kWarps = kSplitThreads / 32;
  const int ncb = (npad + kSplitCols - 1) / kSplitCols;
  const long long plane = (long long)batch * K * npad;
  for (long long blk = blockIdx.x; blk < (long long)batch * ncb; blk += gridDim.x) {
    const int b = (int)(blk / ncb);
    const int n = (int)(blk % ncb) * kSplitCols + lane * 4;
    if (n >= npad) continue;
    const int nvalid = N - n;
    const double* xc = X + b * bsx + n;
    double inv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const double sc = S[(long long)b * npad + n + j];
      inv[j] = sc > 0.0 ? ldexp(1.0, 40 - ilogb(sc)) : 0.0;  // 2^40 / s, exact
    }
    int8_t* q1 = Q + (long long)b * K * npad + n;
    for (int k = wp; k < K; k += kWarps) {
      double v[4];
      if (nvalid > 0) load4d(xc + (long long)k * ldx, nvalid, v);
      else v[0] = v[1] = v[2] = v[3] = 0.0;
      uint32_t word[kDigits] = {0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // Y = rint(v 2^40 / s), |Y| < 2^46; digits 2..6 are the low five bytes
        // of Y + 0x8080808080 minus 128 each, digit 1 the rest
        const long long z = __double2ll_rn(v[j] * inv[j]) + 0x8080808080LL;
        word[0] |= ((uint32_t)(z >> 40) & 0xffu) << (8 * j);
#pragma unroll
        for (int d = 1; d < kDigits; ++d)
          word[d] |= ((uint32_t)((z >> (8 * (kDigits - 1 - d))) & 0xff) ^ 0x80u) << (8 * j);
      }
      const long long o = (long long)k * npad;
#pragma unroll
      for (int d = 0; d < kDigits; ++d) *reinterpret_cast<uint32_t*>(q1 + o + d * plane) = word[d];
    }
  }
}

}  // namespace oz64
}  // namespace tt
