// DF-MP2 pair energy for fp64 inputs (precision="kahan") on tcgen05 int8
// tensor cores: the Ozaki scheme of mp2_i8.cuh carried to five digits.
//
// Math (the reference's trntensor/quantum.py:87-100 run on fp64-promoted
// inputs, which is what precision="kahan" means in trntensor/einsum.py:108-111):
//   E = sum_{i,j} sum_{a,b} T_ab (2 T_ab - T_ba) / (e_i + e_j - e_a - e_b),
//   T = B_i . B_j^T.
//
// Digits. Each row r = (i, a) of B gets s_r = 2^(e-6) with max_P |B[r,P]| <
// 2^e, and Y = rint(B 2^32 / s_r) (|Y| < 2^38, exact in fp64 and int64) is
// written as Y = q1 2^32 + q2 2^24 + q3 2^16 + q4 2^8 + q5 with q2..q5 in
// [-128, 127] (the bytes of Y + 0x80808080, each minus 128) and q1 in
// [-64, 64]: B = s (q1 + q2 2^-8 + ... + q5 2^-32) + O(s 2^-33).
// A product of two rows keeps the levels L0..L5 (level l collects the digit
// products q_a q'_b with a + b = l + 2, weight 2^-8l): 1 + 2 + 3 + 4 + 5 + 4
// = 19 int8 GEMMs accumulated exactly in int32 while K (2 * 64 * 128 +
// 3 * 128^2) < 2^31, i.e. K <= 32767. The dropped levels start at a + b = 8
// (2^-48 of s_a s_b per term). A CPU emulation of exactly this arithmetic
// gives |dE|/|E| <= 5e-14 on the reference's known-answer cases (naux 5 to
// 128); stopping at L4 (15 GEMMs) gave 1.8e-12 at naux = 6, where nothing
// averages the dropped terms, and four digits (10 GEMMs) leave a biased
// q3 q3 term on T's diagonal (1e-8).
//
// TMEM holds 512 int32 columns, fewer than the 6 x 128 that six levels of a
// 128 x 128 block need, so each accumulation phase runs as two sweeps over
// the aux range: sweep 0 accumulates L0, L1, L2 (digits q1..q3, 6 MMAs per
// k-step) and sweep 1 accumulates L3, L4, L5 (digits q1..q5, 13 MMAs per
// k-step).
// The epilogue turns sweep 0's levels into an fp64 partial and parks it in a
// per-CTA fp64 scratch tile in global memory (each thread writes and later
// reads back only its own row segment; the tile stays in L2), then adds
// sweep 1's levels to it.
//
// Work decomposition, phases and weights as in mp2_i8.cuh: unordered pairs
// i <= j, 128 x 128 blocks A <= B, phase x = T[A,B], phase y = (T[B,A])^T,
// y = x for i == j and y = x^T for a diagonal block (exchanged through the
// scratch tile). The energy terms are formed and summed in fp64.
//
// Roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer, warps 2..9 = epilogue (lane quarter = warp % 4, column half =
// (warp - 2) / 4). Ten warps put three on some of the SM's four register-file
// quarters (16384 registers each), so a thread can have at most 168.
#pragma once
#include "mp2_i8.cuh"
#include "ptx.cuh"

namespace tt {
namespace mp2d {

constexpr int kBlk = 128;
constexpr int kKC = 32;                        // aux elements (bytes) per stage = one k-step
constexpr int kDigits = 5;
constexpr int kStages = 4;
constexpr int kSliceTile = kBlk * kKC;         // 4 KB, 32B swizzle
// A stage holds two k-steps of sweep 0 (3 digits each) or one of sweep 1
// (5 digits): A at offset 0, B at kOperandBytes, k-step 1 of sweep 0 at
// +3 slices. Sweep 0 then has as much MMA work per stage as sweep 1, so
// that the same ring depth covers the load latency in both sweeps.
constexpr int kOperandBytes = 6 * kSliceTile;  // 24 KB
constexpr int kStageBytes = 2 * kOperandBytes; // 48 KB
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
constexpr int kMaxK = 32767;                   // int32-exact contraction length
constexpr int kMaxGrid = 256;                  // scratch tiles in the workspace
constexpr long long kScratchDoubles = 2LL * kBlk * kBlk;  // x tile + partial tile per CTA

// digits of sweep s: 3 then 5
__host__ __device__ constexpr int sweep_digits(int s) { return s == 0 ? 3 : 5; }

struct Params {
  mp2::Params base;    // sizes, pair range, launch mode, energy outputs (base.scale unused)
  const double* scale;  // (nocc, nvir) power-of-two row scales
  const double* eps_occ;
  const double* eps_vir;
  double* scratch;     // kMaxGrid x kScratchDoubles
};

// L0 + L1 2^-8 + L2 2^-16, exact in fp64 (|L| < 2^31)
__device__ __forceinline__ double level_sum012(int l0, int l1, int l2) {
  return ((double)l2 * (1.0 / 256.0) + (double)l1) * (1.0 / 256.0) + (double)l0;
}

// 1 / d in fp64: the fp32 reciprocal refined by two Newton-Raphson steps
// r <- r (2 - d r) (relative error 2^-23 -> 2^-46 -> fp64 rounding). Valid
// for |d| within the fp32 normal range, which orbital-energy gaps are.
__device__ __forceinline__ double recip_f64(double d) {
  double r = (double)__frcp_rn((float)d);
  r = r * fma(-d, r, 2.0);
  return r * fma(-d, r, 2.0);
}

static __global__ void __launch_bounds__(kThreads, 1)
    energy_kernel(const __grid_constant__ CUtensorMap map3, const __grid_constant__ CUtensorMap map5,
                  Params P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* final_bar = acc_empty + 1;
  uint32_t* tmem_slot = (uint32_t*)(final_bar + 1);
  double* red = (double*)(tmem_slot + 2);  // kEpiWarps doubles

  const mp2::Params& p = P.base;
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
    tma_prefetch_desc(&map3);
    tma_prefetch_desc(&map5);
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
        const mp2::Item t = mp2::item_decode(w, p);
        const int nrounds = t.single() ? 2 : 4;
        for (int r = 0; r < nrounds && ok; ++r) {
          const int sweep = r & 1;
          const int occA = r < 2 ? t.i : t.j;
          const int occB = r < 2 ? t.j : t.i;
          const CUtensorMap* map = sweep ? &map5 : &map3;
          const int ksteps = sweep ? 1 : 2;  // k-steps per stage
          const uint32_t bytes = 2u * ksteps * sweep_digits(sweep) * kSliceTile;
          for (int kc = 0; kc < nkc; kc += ksteps, ++it) {
            const int s = it % kStages;
            if (!mbar_wait(&empty[s], ((it / kStages) & 1u) ^ 1u, p.err, kDevTimeoutEmpty)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + s * kStageBytes;
            mbar_arrive_expect_tx(&full[s], bytes);
            for (int ks = 0; ks < ksteps; ++ks) {
              const int off = ks * 3 * kSliceTile;
              tma_load_4d(st + off, map, &full[s], (kc + ks) * kKC, t.a0, occA, 0);
              tma_load_4d(st + kOperandBytes + off, map, &full[s], (kc + ks) * kKC, t.b0, occB, 0);
            }
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
      bool ok = true;
      for (long long w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
        const int nrounds = mp2::item_decode(w, p).single() ? 2 : 4;
        for (int r = 0; r < nrounds && ok; ++r, ++round) {
          const int sweep = r & 1;
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
            // Grouped by A digit (collector buffer: each A digit is read from
            // shared memory once per k-step). Level l sits at column 128 l
            // (sweep 0: L0..L2) or 128 (l - 3) (sweep 1: L3..L5).
            if (sweep == 0) {
#pragma unroll
              for (int ks = 0; ks < 2; ++ks) {
                uint64_t a[3], b[3];
#pragma unroll
                for (int d = 0; d < 3; ++d) {
                  a[d] = smem_desc(sa + (3 * ks + d) * kSliceTile, 16, 256, 6);
                  b[d] = smem_desc(sb + (3 * ks + d) * kSliceTile, 16, 256, 6);
                }
                const uint32_t acc = (kc | ks) != 0;
                mma_i8_fill(tmem + 0 * kBlk, a[0], b[0], idesc, acc);
                mma_i8_use(tmem + 1 * kBlk, a[0], b[1], idesc, acc);
                mma_i8_lastuse(tmem + 2 * kBlk, a[0], b[2], idesc, acc);
                mma_i8_fill(tmem + 1 * kBlk, a[1], b[0], idesc, 1);
                mma_i8_lastuse(tmem + 2 * kBlk, a[1], b[1], idesc, 1);
                mma_i8(tmem + 2 * kBlk, a[2], b[0], idesc, 1);
              }
            } else {
              uint64_t a[kDigits], b[kDigits];
#pragma unroll
              for (int d = 0; d < kDigits; ++d) {
                a[d] = smem_desc(sa + d * kSliceTile, 16, 256, 6);
                b[d] = smem_desc(sb + d * kSliceTile, 16, 256, 6);
              }
              const uint32_t acc = kc != 0;
              mma_i8_fill(tmem + 0 * kBlk, a[0], b[3], idesc, acc);
              mma_i8_lastuse(tmem + 1 * kBlk, a[0], b[4], idesc, acc);
              mma_i8_fill(tmem + 0 * kBlk, a[1], b[2], idesc, 1);
              mma_i8_use(tmem + 1 * kBlk, a[1], b[3], idesc, 1);
              mma_i8_lastuse(tmem + 2 * kBlk, a[1], b[4], idesc, acc);
              mma_i8_fill(tmem + 0 * kBlk, a[2], b[1], idesc, 1);
              mma_i8_use(tmem + 1 * kBlk, a[2], b[2], idesc, 1);
              mma_i8_lastuse(tmem + 2 * kBlk, a[2], b[3], idesc, 1);
              mma_i8_fill(tmem + 0 * kBlk, a[3], b[0], idesc, 1);
              mma_i8_use(tmem + 1 * kBlk, a[3], b[1], idesc, 1);
              mma_i8_lastuse(tmem + 2 * kBlk, a[3], b[2], idesc, 1);
              mma_i8_fill(tmem + 1 * kBlk, a[4], b[0], idesc, 1);
              mma_i8_lastuse(tmem + 2 * kBlk, a[4], b[1], idesc, 1);
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
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int q = warp & 3;                  // TMEM lane quarter
    const int c0 = (ew >> 2) * (kBlk / 2);   // this warp's 64-column half
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    // scratch tiles of this CTA: X (x, or its sweep-0 partial) and Yp (y's partial)
    double* const xs = P.scratch + (long long)blockIdx.x * kScratchDoubles;
    double* const yp = xs + kBlk * kBlk;
    double my_energy = 0.0;
    uint32_t round = 0;
    bool ok = true;

    // Sweep 0 of a phase: L0 + L1 2^-8 + L2 2^-16 -> dst[row][c0 .. c0 + 64).
    auto drain_sweep0 = [&](double* dst) -> bool {
      if (!group_all<32 * kEpiWarps>(mbar_wait(acc_full, round & 1u, p.err, kDevTimeoutAcc)))
        return false;
      tc_fence_after();
      for (int c = c0; c < c0 + kBlk / 2; c += 16) {
        int l0[16], l1[16], l2[16];
        tmem_ld16i(lane_base + 0 * kBlk + c, l0);
        tmem_ld16i(lane_base + 1 * kBlk + c, l1);
        tmem_ld16i(lane_base + 2 * kBlk + c, l2);
        tmem_ld_wait();
        double2* d2 = reinterpret_cast<double2*>(dst + row * kBlk + c);
#pragma unroll
        for (int k = 0; k < 16; k += 2)
          d2[k / 2] = make_double2(level_sum012(l0[k], l1[k], l2[k]),
                                   level_sum012(l0[k + 1], l1[k + 1], l2[k + 1]));
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
      ++round;
      return true;
    };
    // Sweep 1 of a phase, 16 columns at c: part[] (sweep 0's partial) plus
    // L3 2^-24 + L4 2^-32 + L5 2^-40, scaled by s_row s_col -> v[].
    auto sweep1_chunk = [&](int c, const double* part, double srow, int occ_col, int b0,
                            double (&v)[16]) {
      // L5 and L4 first (combined into t), then L3, so that only two int
      // column blocks are live at a time
      double t[16];
      {
        int l4[16], l5[16];
        tmem_ld16i(lane_base + 2 * kBlk + c, l5);
        tmem_ld16i(lane_base + 1 * kBlk + c, l4);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 16; ++k) t[k] = (double)l5[k] * (1.0 / 256.0) + (double)l4[k];
      }
      int l3[16];
      tmem_ld16i(lane_base + 0 * kBlk + c, l3);
      tmem_ld_wait();
      const double2* p2 = reinterpret_cast<const double2*>(part + row * kBlk + c);
#pragma unroll
      for (int k = 0; k < 16; k += 2) {
        const double2 pp = p2[k / 2];
        const double pk[2] = {pp.x, pp.y};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int b = b0 + c + k + h;
          const double sb = b < p.nvir ? __ldg(P.scale + (long long)occ_col * p.nvir + b) : 0.0;
          const double hi = (t[k + h] * (1.0 / 256.0) + (double)l3[k + h]) * (1.0 / 16777216.0);
          v[k + h] = (pk[h] + hi) * (srow * sb);
        }
      }
    };

    for (long long w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const mp2::Item t = mp2::item_decode(w, p);
      const int a = t.a0 + row;
      const bool arow = a < p.nvir;
      const double eija =
          arow ? (__ldg(P.eps_occ + t.i) + __ldg(P.eps_occ + t.j)) - __ldg(P.eps_vir + a) : 0.0;
      // sum of the (a,b) + (b,a) terms over 16 columns starting at c; x may
      // point into registers or into this thread's own scratch row
      auto chunk_energy = [&](int c, const double* x, const double* y) {
        double part = 0.0;
#pragma unroll 4
        for (int k = 0; k < 16; ++k) {
          const int b = t.b0 + c + k;
          if (arow && b < p.nvir && a <= b) {
            double v = 2.0 * (x[k] * x[k] - x[k] * y[k] + y[k] * y[k]) *
                       recip_f64(eija - __ldg(P.eps_vir + b));
            if (a == b) v *= 0.5;
            part += v;
          }
        }
        return part;
      };
      double acc = 0.0;
      // ---- phase x
      const double sa_x = arow ? __ldg(P.scale + (long long)t.i * p.nvir + a) : 0.0;
      if (!drain_sweep0(xs)) { ok = false; break; }
      if (!group_all<32 * kEpiWarps>(mbar_wait(acc_full, round & 1u, p.err, kDevTimeoutAcc))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // Values are completed into the scratch tile and the accumulator is
      // released before the fp64 energy terms are formed, so that the next
      // sweep's MMAs do not wait for them.
      auto finish_into = [&](double* dst, double srow, int occ_col) {
        for (int c = c0; c < c0 + kBlk / 2; c += 16) {
          double v[16];
          sweep1_chunk(c, dst, srow, occ_col, t.b0, v);
          double2* d2 = reinterpret_cast<double2*>(dst + row * kBlk + c);
#pragma unroll
          for (int k = 0; k < 16; k += 2) d2[k / 2] = make_double2(v[k], v[k + 1]);
        }
        tc_fence_before();
        mbar_arrive(acc_empty);
        ++round;
      };
      if (t.i == t.j) {
        // T_ii symmetric: y = x
        finish_into(xs, sa_x, t.j);
        for (int c = c0; c < c0 + kBlk / 2; c += 16)
          acc += chunk_energy(c, xs + row * kBlk + c, xs + row * kBlk + c);
      } else {
        finish_into(xs, sa_x, t.j);  // complete x into the X tile
        if (t.a0 == t.b0) {
          // diagonal block: y[a][b] = x[b][a], read back transposed from X
          group_sync<32 * kEpiWarps, 1>();
          // (gathered into this thread's row of the Yp tile first)
          for (int c = c0; c < c0 + kBlk / 2; ++c) yp[row * kBlk + c] = xs[c * kBlk + row];
          group_sync<32 * kEpiWarps, 1>();  // X free for the next item
          for (int c = c0; c < c0 + kBlk / 2; c += 16)
            acc += chunk_energy(c, xs + row * kBlk + c, yp + row * kBlk + c);
        } else {
          // ---- phase y: operands B_j[A], B_i[B]
          const double sa_y = arow ? __ldg(P.scale + (long long)t.j * p.nvir + a) : 0.0;
          if (!drain_sweep0(yp)) { ok = false; break; }
          if (!group_all<32 * kEpiWarps>(mbar_wait(acc_full, round & 1u, p.err, kDevTimeoutAcc))) {
            ok = false;
            break;
          }
          tc_fence_after();
          finish_into(yp, sa_y, t.i);
          for (int c = c0; c < c0 + kBlk / 2; c += 16)
            acc += chunk_energy(c, xs + row * kBlk + c, yp + row * kBlk + c);
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

// Five-digit split of fp64 rows, one row per warp: scale[r] = s_r and the
// digit planes q_t[r][c] (planes `plane` bytes apart, rows cols_pad long,
// zero padded). A row holding inf or NaN gets a NaN scale.
static __global__ void split_kernel(const double* __restrict__ x, int8_t* __restrict__ q,
                                    double* __restrict__ scale, long long rows, int cols,
                                    int cols_pad, long long plane) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += warps) {
    const double* xr = x + r * cols;
    double m = 0.0;
    for (int c = lane; c < cols; c += 32) {
      const double v = __ldg(xr + c);
      m = fmax(m, v == v ? fabs(v) : __longlong_as_double(0x7ff0000000000000LL));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    double s, inv;
    if (!(m <= 1.7976931348623157e308)) {
      s = __longlong_as_double(0x7ff8000000000000LL);
      inv = 0.0;
    } else if (!(m > 1.0e-290)) {
      s = 0.0;
      inv = 0.0;
    } else {
      const int e = ilogb(m) + 1;      // m < 2^e
      s = ldexp(1.0, e - 6);           // |x / s| < 64
      inv = ldexp(1.0, 32 - (e - 6));  // 2^32 / s, exact
    }
    if (lane == 0) scale[r] = s;
    int8_t* qr = q + r * cols_pad;
    for (int c = lane * 4; c < cols_pad; c += 128) {
      uint32_t word[kDigits] = {0, 0, 0, 0, 0};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const double v = (c + k < cols) ? __ldg(xr + c + k) : 0.0;
        // Y = rint(v 2^32 / s), |Y| < 2^38; bytes of Y + 0x80808080
        const long long z = __double2ll_rn(v * inv) + 0x80808080LL;
        const uint32_t lo = (uint32_t)z;
        word[0] |= ((uint32_t)(z >> 32) & 0xffu) << (8 * k);                 // q1 (two's complement)
        word[1] |= (((lo >> 24) & 0xffu) ^ 0x80u) << (8 * k);               // q2 + 128 -> q2
        word[2] |= (((lo >> 16) & 0xffu) ^ 0x80u) << (8 * k);
        word[3] |= (((lo >> 8) & 0xffu) ^ 0x80u) << (8 * k);
        word[4] |= ((lo & 0xffu) ^ 0x80u) << (8 * k);
      }
#pragma unroll
      for (int d = 0; d < kDigits; ++d) *reinterpret_cast<uint32_t*>(qr + d * plane + c) = word[d];
    }
  }
}

}  // namespace mp2d
}  // namespace tt
