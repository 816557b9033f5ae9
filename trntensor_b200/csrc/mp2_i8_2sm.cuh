// DF-MP2 pair energy on pairs of SMs (tcgen05 cta_group::2), int8 Ozaki.
//
// Same mathematics as csrc/mp2_i8.cuh (one-SM kernel): three int8 slices
// per B row, six exact int32 slice GEMMs per block, x = T[A,B] parked in
// TMEM, y = (T[B,A])^T, energy terms added in the epilogue. What changes is
// the tile: a cluster of two CTAs computes a 256 x 128 strip with one paired
// MMA stream (M = 256, N = 128, K = 32 per instruction):
//   CTA r (r = 0 leader, 1 peer) holds the 128 A rows 256*R + 128*r and the
//   64 B rows 128*C + 64*r of every stage; each CTA's TMEM holds its 128
//   output rows x all 128 columns.
// Sharing B between the two SMs cuts the operand bytes every SM streams
// from L2 per MAC by a quarter. Measured on B200 it is nonetheless slower
// than the one-SM kernel (289 vs 316 TFLOP/s at config 4): with three int32
// accumulator levels TMEM caps the paired tile at N = 128, where the paired
// MMA stream reaches 0.72 of the int8 peak per clock against 0.86 for
// one-SM 128 x 128 MMAs, and the strip cover adds 7 % of below-diagonal
// blocks. It is therefore opt-in (TRNTENSOR_B200_MP2_2SM=1).
//
// Work item (per cluster): (unordered pair i <= j, strip R, column block C)
// with C >= 2R. The strip's two 128-row blocks are 2R + r. Phases:
//   i == j            : one phase, y = x (T_ii symmetric);
//   i != j, C == 2R   : one phase; block (2R, 2R) is diagonal (y = x^T via
//                       shared memory), block (2R+1, 2R) lies below the
//                       diagonal and contributes nothing;
//   otherwise         : two phases (x, then y by MMA).
//
// Synchronisation: both CTAs' TMA loads complete on the leader's full[s]
// (tx bytes of both halves); the leader's MMA thread commits to empty[s] and
// acc_full of both CTAs; all 16 epilogue warps arrive on the leader's
// acc_empty. Every wait is bounded; a timeout records an error code and the
// kernel unwinds. Roles per CTA as in the one-SM kernel (warp 0 TMA, warp 1
// TMEM + MMA, warps 2..9 epilogue).
#pragma once
#include "mp2_i8.cuh"
#include "ptx2sm.cuh"

namespace tt {
namespace mp2x2 {

using mp2::kBlk;      // 128
using mp2::kKC;       // 64 aux bytes per stage
using mp2::kEpiWarps; // 8
using mp2::kThreads;  // 320
using mp2::level_combine;
using mp2::pair_decode;
using mp2::Params;

constexpr int kStages = 5;
constexpr int kATile = kBlk * kKC;             // 8 KB per slice
constexpr int kBTile = (kBlk / 2) * kKC;       // 4 KB per slice
constexpr int kAOperand = 3 * kATile;          // 24 KB
constexpr int kBOperand = 3 * kBTile;          // 12 KB
constexpr int kStageBytes = kAOperand + kBOperand;  // 36 KB per CTA
constexpr int kTLd = kBlk + 1;
constexpr int kTBytes = (kBlk / 2) * kTLd * 4;
constexpr int kSmemBytes = kStages * kStageBytes + kTBytes + 1024 + 256;
constexpr int kColStash = 3 * kBlk;

struct Item {
  int i, j, a0, b0;  // a0: this CTA's first row; b0: the strip's first column
  int nph;           // accumulation phases
  int mode;          // 0: two-phase, 1: y = x, 2: y = x^T (diagonal), 3: contributes nothing
};

__host__ __device__ inline int items_per_pair(int nblk) {
  const int nR = (nblk + 1) / 2;
  int c = 0;
  for (int R = 0; R < nR; ++R) c += nblk - 2 * R;
  return c;
}

__device__ inline Item item_decode(long long w, const Params& p, int ipp, uint32_t rank) {
  Item t;
  pair_decode(p.pair_begin + w / ipp, p.nocc, t.i, t.j);
  int r = (int)(w % ipp), R = 0;
  while (r >= p.nblk - 2 * R) {
    r -= p.nblk - 2 * R;
    ++R;
  }
  const int C = 2 * R + r;
  t.a0 = (2 * R + (int)rank) * kBlk;
  t.b0 = C * kBlk;
  if (t.i == t.j) {
    t.nph = 1;
    t.mode = 1;
  } else if (C == 2 * R) {
    t.nph = 1;
    t.mode = rank == 0 ? 2 : 3;
  } else {
    t.nph = 2;
    t.mode = 0;
  }
  return t;
}

static __global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    energy_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                  Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  float* tbuf = (float*)(smem + kStages * kStageBytes);
  uint64_t* full = (uint64_t*)(smem + kStages * kStageBytes + kTBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* final_bar = acc_empty + 1;
  uint32_t* tmem_slot = (uint32_t*)(final_bar + 1);
  double* red = (double*)(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const long long cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  const int ipp = items_per_pair(p.nblk);
  const long long n_items = (p.pair_end - p.pair_begin) * (long long)ipp;
  const int nkc = p.naux_pad / kKC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * kEpiWarps);
    mbar_init(final_bar, 1);
    tmem_slot[1] = 0;  // stages issued by this CTA's producer (read by the drain)
    fence_mbar_init();
    tma_prefetch_desc(&mapA);
    tma_prefetch_desc(&mapB);
  }
  if (warp == 1) {
    tmem_alloc2(tmem_slot, 512);
    tmem_relinquish2();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // shared::cluster addresses of the barriers the pair shares
  const uint32_t full0 = mapa(smem_u32(full), 0);
  const uint32_t acc_empty0 = mapa(smem_u32(acc_empty), 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      uint32_t* issued_out = reinterpret_cast<uint32_t*>(tmem_slot + 1);
      bool ok = true;
      for (long long w = cid; w < n_items && ok; w += ncl) {
        const Item t = item_decode(w, p, ipp, rank);
        for (int ph = 0; ph < t.nph && ok; ++ph) {
          const int occA = ph == 0 ? t.i : t.j;
          const int occB = ph == 0 ? t.j : t.i;
          for (int kc = 0; kc < nkc; ++kc, ++it) {
            const int s = it % kStages;
            if (!mbar_wait(&empty[s], ((it / kStages) & 1u) ^ 1u, p.err, kDevTimeoutEmpty)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + s * kStageBytes;
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * kStageBytes);
            const uint32_t bar = full0 + (uint32_t)(s * sizeof(uint64_t));
            tma2_load_4d(st, &mapA, bar, kc * kKC, t.a0, occA, 0);
            tma2_load_4d(st + kAOperand, &mapB, bar, kc * kKC, t.b0 + (int)rank * (kBlk / 2),
                         occB, 0);
          }
        }
      }
      *issued_out = it;
    }
  } else if (warp == 1) {
    // ------------------------------------------ MMA issuer (pair leader only)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_s8(2 * kBlk, kBlk, 0, 0);
      const uint32_t empty_l = mapa(smem_u32(empty), 0), empty_p = mapa(smem_u32(empty), 1);
      const uint32_t accf_l = mapa(smem_u32(acc_full), 0), accf_p = mapa(smem_u32(acc_full), 1);
      uint32_t it = 0, round = 0;
      bool ok = true;
#ifdef TT_MP2_PROFILE
      long long wait_acc = 0, wait_full = 0;
      const long long t_begin = clock64();
#endif
      for (long long w = cid; w < n_items && ok; w += ncl) {
        const int nph = item_decode(w, p, ipp, 0).nph;
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
            const uint32_t sb = sa + kAOperand;
#pragma unroll
            for (int ks = 0; ks < kKC / 32; ++ks) {
              uint64_t a[3], b[3];
#pragma unroll
              for (int q = 0; q < 3; ++q) {
                a[q] = smem_desc(sa + q * kATile + ks * 32, 16, 512, 4);
                b[q] = smem_desc(sb + q * kBTile + ks * 32, 16, 512, 4);
              }
              const uint32_t first = (kc | ks) != 0;
              mma2_i8(tmem + 0 * kBlk, a[0], b[0], idesc, first);
              mma2_i8(tmem + 1 * kBlk, a[0], b[1], idesc, first);
              mma2_i8(tmem + 2 * kBlk, a[0], b[2], idesc, first);
              mma2_i8(tmem + 1 * kBlk, a[1], b[0], idesc, 1);
              mma2_i8(tmem + 2 * kBlk, a[1], b[1], idesc, 1);
              mma2_i8(tmem + 2 * kBlk, a[2], b[0], idesc, 1);
            }
            const uint32_t off = (uint32_t)(s * sizeof(uint64_t));
            mma2_commit(empty_l + off);
            mma2_commit(empty_p + off);
          }
          if (ok) {
            mma2_commit(accf_l);
            mma2_commit(accf_p);
          }
        }
      }
      mma2_commit(smem_u32(final_bar));
      mbar_wait_drain(final_bar, 0);
#ifdef TT_MP2_PROFILE
      if (p.prof) {
        p.prof[cid * 4 + 0] = clock64() - t_begin;
        p.prof[cid * 4 + 1] = wait_full;
        p.prof[cid * 4 + 2] = wait_acc;
      }
#endif
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int q = warp & 3;
    const int c0 = (ew >> 2) * (kBlk / 2);
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    double my_energy = 0.0;
    uint32_t round = 0;
    // Every epilogue warp of both CTAs signals the leader's acc_empty once
    // its TMEM reads of the round are complete.
    auto release_acc = [&]() {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0);
    };
    for (long long w = cid; w < n_items; w += ncl) {
      const Item t = item_decode(w, p, ipp, rank);
      const int a = t.a0 + row;
      const bool arow = a < p.nvir;
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
      release_acc();
      ++round;
      double acc = 0.0;
      const float eija = arow ? (__ldg(p.eps_occ + t.i) + __ldg(p.eps_occ + t.j)) -
                                    __ldg(p.eps_vir + a)
                              : 0.f;
      auto chunk_energy = [&](int c, const float (&x)[16], const float (&y)[16]) {
        float part = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int b = t.b0 + c + k;
          if (arow && b < p.nvir && a <= b) {
            const float inv = __frcp_rn(eija - __ldg(p.eps_vir + b));
            float v = 2.f * (x[k] * x[k] - x[k] * y[k] + y[k] * y[k]) * inv;
            if (a == b) v *= 0.5f;
            part += v;
          }
        }
        return (double)part;
      };
      if (t.mode == 1) {
        for (int c = c0; c < c0 + kBlk / 2; c += 16) {
          float x[16];
          tmem_ld16(lane_base + kColStash + c, x);
          tmem_ld_wait();
          acc += chunk_energy(c, x, x);
        }
      } else if (t.mode == 2) {
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
      } else if (t.mode == 0) {
        if (!group_all<32 * kEpiWarps>(mbar_wait(acc_full, round & 1u, p.err, kDevTimeoutAcc)))
          break;
        tc_fence_after();
        const float sa = arow ? __ldg(p.scale + (long long)t.j * p.nvir + a) : 0.f;
        for (int c = c0; c < c0 + kBlk / 2; c += 16) {
          int l2[16], l3[16], l4[16];
          float x[16], y[16];
          tmem_ld16i(lane_base + 0 * kBlk + c, l2);
          tmem_ld16i(lane_base + 1 * kBlk + c, l3);
          tmem_ld16i(lane_base + 2 * kBlk + c, l4);
          tmem_ld16(lane_base + kColStash + c, x);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int b = t.b0 + c + k;
            const float sb = b < p.nvir ? __ldg(p.scale + (long long)t.i * p.nvir + b) : 0.f;
            y[k] = level_combine(l2[k], l3[k], l4[k]) * (sa * sb);
          }
          acc += chunk_energy(c, x, y);
        }
        release_acc();
        ++round;
      }
      // mode 3: the block lies below the diagonal and adds nothing
      const double wgt = (t.i == t.j) ? 1.0 : 2.0;
      my_energy += wgt * acc;
      if (p.pair_partials != nullptr) {
        double s = acc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0 && s != 0.0) {
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
  // Drain (matters only after a timeout): the leader waits until the last
  // stages it issued have fully landed, which needs both CTAs' bytes, so no
  // bulk copy is still writing shared memory when the pair exits.
  if (rank == 0 && threadIdx.x == 0) {
    const uint32_t issued = *reinterpret_cast<uint32_t*>(tmem_slot + 1);
    for (uint32_t k = (issued > kStages ? issued - kStages : 0); k < issued; ++k)
      mbar_wait_drain(&full[k % kStages], (k / kStages) & 1u);
  }
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int k = 0; k < kEpiWarps; ++k) tot += red[k];
    if (tot != 0.0) atomicAdd(p.energy, tot);
  }
  cluster_sync();  // the leader's MMAs are complete before either CTA frees TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem, 512);
  }
}

}  // namespace mp2x2
}  // namespace tt
