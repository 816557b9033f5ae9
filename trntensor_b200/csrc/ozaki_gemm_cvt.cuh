// Step 1 of the AO->MO transform with the B operand converted on chip:
//   C[m][n] = sum_k A[k][m] X[k][n]
// A: int8 Ozaki slices of C_occ (MN-major, as in ozaki_gemm.cuh), kARep
//    identical copies;
// X: fp32 rows (eri viewed as nbf x nbf*naux), read by TMA in 64 x 128
//    tiles and split in shared memory. The column scales s_n (max over all k)
//    come either from colmax_kernel (kFuse = false) or from the kernel itself
//    (kFuse = true): each CTA streams the whole K x 128 strip of its NEXT
//    tile through the fp32 ring once for the column maxima while it converts
//    its current tile, whose strip it read the same way one tile earlier and
//    now re-reads from L2 (148 CTAs x 512 KB strips at nbf = 1024, well
//    inside the 126 MB L2). eri then crosses HBM once instead of twice.
// This removes the separate slice pass and its 3 bytes/element round trip
// through HBM. Two rings in shared memory:
//   fp32 landing ring (3 x 32 KB): one producer warp's TMA fills X tiles;
//     converter warps read their rows (lane l: one float4 of a row, a warp
//     reads a whole row) and release the slot at once, so the ring only has
//     to cover HBM latency;
//   int8 ring (2 x 48 KB): a second producer warp's TMA brings the A slice
//     tiles; converter warps write the three B slice tiles in the MN-major
//     128B-swizzled layout the MMA descriptors expect (one 32-bit store per
//     lane and slice, a warp writes a whole 128-byte row), fence the async
//     proxy and arrive on conv; the MMA thread waits on fullA and conv.
//     The A loads have their own warp so that they run ahead of the MMA
//     independently of the fp32 stream.
// Epilogue: the three level accumulators (TMEM columns 0..383) are combined
// into fp32 and parked in columns 384..511, which releases the accumulator
// to the next tile's MMAs at once; the parked tile then leaves through a
// 16-column shared-memory stage as coalesced row segments.
// Roles: warp 0 fp32 TMA, warp 1 TMEM + MMA, warps 2..9 epilogue, 10..17
// convert, warp 18 A-slice TMA (a separate warp, so that neither producer's
// barrier wait holds up the other).
#pragma once
#include "ozaki_gemm.cuh"
#include "ptx2sm.cuh"

namespace tt {
namespace ozc {

using oz::kTile;  // 128
using oz::kKC;    // 64
using oz::level_combine;

// Ring depths (template parameters of the kernel): kFStages fp32 landing
// slots (TMA -> converters) and kIStages int8 slots (A by TMA, B by the
// converters -> MMA). 3 + 2 and 2 + 3 (a deeper int8 ring in the same shared
// memory) are both built; TRNTENSOR_B200_AO2MO_RING=23 selects the latter.
// The fused column scales need more k-chunks per CTA than int8 slots (the
// scale double buffer is rewritten only after the MMA has started the next
// tile, which a converter can only know from an int8 slot of that tile):
// nkl >= kIStages + 1, which the host checks before choosing kFuse / kSplit.
constexpr int kFStagesDefault = 3;
constexpr int kIStagesDefault = 2;
constexpr int kFBytes = kTile * kKC * 4;      // 32 KB fp32 tile
constexpr int kARegion = 3 * kTile * kKC;     // 24 KB of A slices
constexpr int kIBytes = 2 * kARegion;         // A and B slices: 48 KB
#ifndef TT_OZC_EPI_WARPS
#define TT_OZC_EPI_WARPS 8
#endif
#ifndef TT_OZC_CVT_WARPS
#define TT_OZC_CVT_WARPS 8
#endif
constexpr int kEpiWarps = TT_OZC_EPI_WARPS;  // 4 or 8: each lane quarter's columns split evenly
constexpr int kCvtWarps = TT_OZC_CVT_WARPS;  // 8 or 16: divides the 64 rows of a chunk
constexpr int kEpiCols = kTile * 4 / kEpiWarps;  // columns of one epilogue warp
constexpr int kAWarp = 2 + kEpiWarps + kCvtWarps;  // A-slice producer (its own warp)
constexpr int kThreads = 32 * (kAWarp + 1);
// kGMax: the column maxima of the next tile come from kMaxWarps extra warps
// that read the strip with plain global loads into registers, so that it
// passes through neither the TMA landing ring nor shared memory, and the
// converters only convert. The landing ring then carries each chunk once.
#ifndef TT_OZC_MAX_WARPS
#define TT_OZC_MAX_WARPS 8
#endif
#ifndef TT_OZC_MAX_UNROLL
#define TT_OZC_MAX_UNROLL 8
#endif
constexpr int kMaxWarps = TT_OZC_MAX_WARPS;
constexpr int kMaxUnroll = TT_OZC_MAX_UNROLL;  // rows in flight per lane of a max warp
constexpr int kThreadsG = kThreads + 32 * kMaxWarps;
constexpr int kMaxBar = 3;     // named barrier of the max warps
constexpr int kQCols = 16;                    // output staged 16 columns at a time
constexpr int kQLd = kQCols + 4;
constexpr int kColPark = 3 * kTile;           // TMEM columns of the parked fp32 tile
constexpr int kARep = 8;                      // copies of the A slices (CTA b reads copy b % kARep)
constexpr int kOutBytes = kTile * kQLd * 4;
constexpr int kCMaxBytes = kCvtWarps * kTile * 4;  // per-warp column maxima (fused scales)
constexpr int kGMaxBytes = kMaxWarps * kTile * 4 + 2 * kTile * 4;  // kGMax: per-warp maxima, inv x 2
constexpr int smem_bytes(int fstages, int istages, bool gmax = false) {
  return fstages * kFBytes + istages * kIBytes + kOutBytes + 2 * kTile * 4 + kCMaxBytes +
         2 * kTile * 4 + (gmax ? kGMaxBytes : 0) + 1024 + 256;
}
constexpr int kSmemBytes = smem_bytes(kFStagesDefault, kIStagesDefault);
static_assert(smem_bytes(2, 3) <= 232448, "2 + 3 ring exceeds shared memory");
static_assert(smem_bytes(3, 2, true) <= 232448, "max-warp buffers exceed shared memory");
constexpr int kCvtBar = 2;  // named barrier of the converter warps
constexpr int kProfSlots = 12;  // per-CTA counters of TT_OZC_PROFILE builds

struct Params {
  const float* sA;    // column scales of A (per m)
  const float* sX;    // column scales of X (per n), from colmax_kernel; unused when kFuse
  float* C;
  long long ldc;
  int M, N, K;
  int tiles_m, tiles_n;
  int* err;
  long long* prof;  // optional per-CTA wait-cycle counters (TT_OZC_PROFILE builds)
  int l2hint;       // kFuse: keep max-pass lines in L2 (evict_last) for the conversion
                    // re-read, which marks them evict_first; output stores streaming
  // P-slab mode (slab_p > 0, kFuse only): X is a strided (m, n, P) view with
  // slab_p aux columns per n row, read through a 3-D tensor map; a column
  // tile is 128 aux columns of one n (tiles_p per n row). The output stays
  // compact: column n * slab_p + P.
  int slab_p;
  int tiles_p;
  // kGMax: X itself for the max warps' loads. Element (k, column n0 + c) of
  // a tile is X[k * ldx_m + col_off(n0) + c], col_off(n0) = n0 (dense) or
  // (n0 / slab_p) * ldx_n + n0 % slab_p (P-slab).
  const float* X;
  long long ldx_m;
  long long ldx_n;
};

// 16-byte read-only global load with an L2 eviction-priority policy, not
// allocated in L1 (each line is read once per pass).
__device__ __forceinline__ float4 ldg_nc_hint_v4(const float* src, uint64_t policy) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(src), "l"(policy));
  return v;
}

// 16-byte store to a shared::cluster address (another CTA's shared memory).
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, const float (&v)[4]) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v[0]),
               "f"(v[1]), "f"(v[2]), "f"(v[3])
               : "memory");
}
// red.add of four floats at a 16-byte aligned global address.
__device__ __forceinline__ void red_add_v4(float* dst, float4 v) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
// Wait on a local mbarrier that the peer CTA of the cluster arrives on
// (acquire at cluster scope, so that what the peer wrote before arriving is
// visible), bounded like mbar_wait.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err, int code) {
  const long long t0 = clock64();
  uint32_t n = 0;
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if ((++n & 1023u) == 0) {
      if (*(volatile int*)err != 0) return false;
      if (clock64() - t0 > kWaitBudgetCycles) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

// kSplit (with kFuse): a cluster of two CTAs shares each tile and splits its
// K range in halves, so that each CTA keeps only half a strip (256 KB at
// nbf = 1024) between its two reads of eri. The column maxima of the halves
// are exchanged through distributed shared memory (pmax, pfull); rank 0
// stores its partial tile, then rank 1 adds its own with red.global.add
// (out_ready / out_done order the two and keep the barriers' phases apart).
// C = (rank 0 partial) + (rank 1 partial): one fp32 rounding, deterministic.
template <bool kFuse, bool kSplit, bool kGMax, int kFStages, int kIStages>
__device__ __forceinline__ void gemm_cvt_body(const CUtensorMap& mapA, const CUtensorMap& mapX,
                                              const Params& p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* fring = smem;
  uint8_t* iring = smem + kFStages * kFBytes;
  float* ostage = (float*)(iring + kIStages * kIBytes);
  float* escale = (float*)((uint8_t*)ostage + kOutBytes);  // column scales, [2][kTile]
  float* cmax = escale + 2 * kTile;                         // [kCvtWarps][kTile] (kFuse)
  float* pmax = cmax + kCvtWarps * kTile;                    // [2][kTile] kSplit: the peer's maxima
  uint64_t* fullF = (uint64_t*)(pmax + 2 * kTile);
  uint64_t* freeF = fullF + kFStages;
  uint64_t* fullA = freeF + kFStages;
  uint64_t* conv = fullA + kIStages;
  uint64_t* emptyI = conv + kIStages;
  uint64_t* acc_full = emptyI + kIStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* final_bar = acc_empty + 1;
  uint64_t* scale_full = final_bar + 1;  // [2]: tile scales ready (kFuse), by tile parity
  uint64_t* pfull = scale_full + 2;      // [2] kSplit: the peer's column maxima have landed
  uint64_t* out_ready = pfull + 2;       // kSplit, rank 1: rank 0 has stored the tile
  uint64_t* out_done = out_ready + 1;    // kSplit, rank 0: rank 1 has added its partial
  uint64_t* scale_free = out_done + 1;   // [2] kGMax: scales of a tile read by epilogue + converters
  uint64_t* cvt_took = scale_free + 2;   // [2] kGMax: the converters have taken a tile's scales
  uint32_t* tmem_slot = (uint32_t*)(cvt_took + 2);
  // kGMax: per-warp column maxima of the max warps, [kMaxWarps][kTile], and
  // the converters' 2^16 / s_n, [2][kTile] (after the barriers' 256 bytes)
  float* gcmax = (float*)(smem + kFStages * kFBytes + kIStages * kIBytes + kOutBytes +
                          2 * kTile * 4 + kCMaxBytes + 2 * kTile * 4 + 256);
  float* einv = gcmax + kMaxWarps * kTile;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long n_tiles = (long long)p.tiles_m * p.tiles_n;
  const int nkc = (p.K + kKC - 1) / kKC;
  const uint32_t rank = kSplit ? cluster_ctarank() : 0u;
  const uint32_t peer = rank ^ 1u;
  // tiles of this CTA (of this cluster when kSplit) and its k-chunk range
  const long long w0 = kSplit ? blockIdx.x / 2 : blockIdx.x;
  const long long wstep = kSplit ? gridDim.x / 2 : gridDim.x;
  const int k_lo = kSplit && rank ? (nkc + 1) / 2 : 0;
  const int k_hi = kSplit && !rank ? (nkc + 1) / 2 : nkc;
  const int nkl = k_hi - k_lo;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFStages; ++s) {
      mbar_init(&fullF[s], 1);
      mbar_init(&freeF[s], 32 * kCvtWarps);
    }
    for (int s = 0; s < kIStages; ++s) {
      mbar_init(&fullA[s], 1);
      mbar_init(&conv[s], 32 * kCvtWarps);
      mbar_init(&emptyI[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 32 * kEpiWarps);
    mbar_init(final_bar, 1);
    mbar_init(&scale_full[0], 32);
    mbar_init(&scale_full[1], 32);
    mbar_init(&pfull[0], 32);
    mbar_init(&pfull[1], 32);
    mbar_init(out_ready, 32 * kEpiWarps);
    mbar_init(out_done, 32 * kEpiWarps);
    mbar_init(&scale_free[0], 32 * (kEpiWarps + kCvtWarps));
    mbar_init(&scale_free[1], 32 * (kEpiWarps + kCvtWarps));
    mbar_init(&cvt_took[0], 32 * kCvtWarps);
    mbar_init(&cvt_took[1], 32 * kCvtWarps);
    fence_mbar_init();
    tma_prefetch_desc(&mapA);
    tma_prefetch_desc(&mapX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  if (kSplit) cluster_sync();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Output column base n0 of tile w (and its row tile m0). Consecutive tiles
  // share the X columns.
  auto tile_of = [&](long long w, int& m0, int& n0) {
    const long long ct = w / p.tiles_m;
    m0 = (int)(w % p.tiles_m) * kTile;
    if (p.slab_p)
      n0 = (int)((ct / p.tiles_p) * p.slab_p + (ct % p.tiles_p) * kTile);
    else
      n0 = (int)ct * kTile;
  };
  // Valid output columns of the tile at column base n0.
  auto cols_of = [&](int n0) -> int {
    const int left = p.slab_p ? p.slab_p - n0 % p.slab_p : p.N - n0;
    return left < kTile ? left : kTile;
  };

  if (warp == 0 || warp == kAWarp) {
    // ------------------------------------------------ producers (one lane each)
    // warp 0: fp32 X tiles into the landing ring; warp kAWarp: A slice tiles
    // into the int8 ring as soon as the MMA has released a slot.
    if (lane == 0) {
      const bool fp32 = warp == 0;
      const int nst = fp32 ? kFStages : kIStages;
      uint64_t* wait_bar = fp32 ? freeF : emptyI;
      uint64_t* fill_bar = fp32 ? fullF : fullA;
      uint32_t it = 0;
      bool ok = true;
#ifdef TT_OZC_PROFILE
      long long w_prod = 0;
#endif
      const uint64_t keep = l2_policy_evict_last(), drop = l2_policy_evict_first();
      // one ring slot: wait for it, then fill it with chunk kc of tile w
      // (max_pass: the first of the strip's two reads)
      auto issue = [&](long long w, int kc, bool max_pass) {
        if (!ok) return;
        int m0, n0;
        tile_of(w, m0, n0);
        const int s = it % nst;
#ifdef TT_OZC_PROFILE
        const long long tw = clock64();
#endif
        if (!mbar_wait(&wait_bar[s], ((it / nst) & 1u) ^ 1u, p.err, kDevTimeoutEmpty)) {
          ok = false;
          return;
        }
#ifdef TT_OZC_PROFILE
        w_prod += clock64() - tw;
#endif
        if (fp32) {
          mbar_arrive_expect_tx(&fill_bar[s], kFBytes);
          if (p.slab_p) {  // box {128 P, 1 n, 64 m} of the strided slab
            const int n = n0 / p.slab_p, p0 = n0 % p.slab_p;
            if (kFuse && p.l2hint)
              tma_load_3d_hint(fring + s * kFBytes, &mapX, &fill_bar[s], p0, n, kc * kKC,
                               max_pass ? keep : drop);
            else
              tma_load_3d(fring + s * kFBytes, &mapX, &fill_bar[s], p0, n, kc * kKC);
          } else if (kFuse && p.l2hint)
            tma_load_2d_hint(fring + s * kFBytes, &mapX, &fill_bar[s], n0, kc * kKC,
                             max_pass ? keep : drop);
          else
            tma_load_2d(fring + s * kFBytes, &mapX, &fill_bar[s], n0, kc * kKC);
        } else {
          mbar_arrive_expect_tx(&fill_bar[s], kARegion);
          tma_load_4d(iring + s * kIBytes, &mapA, &fill_bar[s], m0, kc * kKC, blockIdx.x % kARep, 0);
        }
        ++it;
      };
      // fused scales: the fp32 stream is the first tile's strip (maxima), then
      // per tile the chunks of the next tile's strip (maxima) interleaved with
      // the current tile's (conversion), in the order the converters take them
      // (kGMax: the max warps read the strips themselves; the ring carries
      // only the conversion chunks)
      if (kFuse && !kGMax && fp32 && w0 < n_tiles)
        for (int kc = k_lo; kc < k_hi; ++kc) issue(w0, kc, true);
      for (long long w = w0; w < n_tiles && ok; w += wstep) {
        const long long nxt = w + wstep;
        for (int kc = k_lo; kc < k_hi; ++kc) {
          issue(w, kc, false);
          if (kFuse && !kGMax && fp32 && nxt < n_tiles) issue(nxt, kc, true);
        }
      }
      const uint32_t issued = it;
      for (uint32_t k = (issued > (uint32_t)nst ? issued - nst : 0); k < issued; ++k)
        mbar_wait_drain(&fill_bar[k % nst], (k / nst) & 1u);
#ifdef TT_OZC_PROFILE
      if (p.prof) p.prof[blockIdx.x * kProfSlots + (fp32 ? 6 : 7)] = w_prod;
#endif
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8(kTile, kTile, 1, 1);
      uint32_t it = 0, round = 0;
      bool ok = true;
#ifdef TT_OZC_PROFILE
      long long w_acc = 0, w_a = 0, w_c = 0;
      const long long t_begin = clock64();
#endif
      for (long long w = w0; w < n_tiles && ok; w += wstep, ++round) {
#ifdef TT_OZC_PROFILE
        long long t0 = clock64();
#endif
        if (!mbar_wait(acc_empty, (round & 1u) ^ 1u, p.err, kDevTimeoutAccFree)) break;
#ifdef TT_OZC_PROFILE
        w_acc += clock64() - t0;
#endif
        tc_fence_after();
        for (int kc = k_lo; kc < k_hi; ++kc, ++it) {
          const int s = it % kIStages;
          const uint32_t ph = (it / kIStages) & 1u;
#ifdef TT_OZC_PROFILE
          long long t1 = clock64();
#endif
          if (!mbar_wait(&fullA[s], ph, p.err, kDevTimeoutFull)) {
            ok = false;
            break;
          }
#ifdef TT_OZC_PROFILE
          long long t2 = clock64();
          w_a += t2 - t1;
#endif
          if (!mbar_wait(&conv[s], ph, p.err, kDevTimeoutFull)) {
            ok = false;
            break;
          }
#ifdef TT_OZC_PROFILE
          w_c += clock64() - t2;
#endif
          tc_fence_after();
          const uint32_t sa = smem_u32(iring + s * kIBytes);
          const uint32_t sb = sa + kARegion;
#pragma unroll
          for (int ks = 0; ks < kKC / 32; ++ks) {
            uint64_t a[3], b[3];
#pragma unroll
            for (int t = 0; t < 3; ++t) {
              a[t] = smem_desc(sa + t * oz::kSliceTile + ks * 4096, 8192, 1024, 2);
              b[t] = smem_desc(sb + t * oz::kSliceTile + ks * 4096, 8192, 1024, 2);
            }
            const uint32_t first = ((kc - k_lo) | ks) != 0;
            mma_i8_fill(tmem + 0 * kTile, a[0], b[0], idesc, first);
            mma_i8_use(tmem + 1 * kTile, a[0], b[1], idesc, first);
            mma_i8_lastuse(tmem + 2 * kTile, a[0], b[2], idesc, first);
            mma_i8_fill(tmem + 1 * kTile, a[1], b[0], idesc, 1);
            mma_i8_lastuse(tmem + 2 * kTile, a[1], b[1], idesc, 1);
            mma_i8(tmem + 2 * kTile, a[2], b[0], idesc, 1);
          }
          mma_commit(&emptyI[s]);
        }
        if (ok) mma_commit(acc_full);
      }
      mma_commit(final_bar);
      mbar_wait_drain(final_bar, 0);
#ifdef TT_OZC_PROFILE
      if (p.prof) {
        p.prof[blockIdx.x * kProfSlots + 0] = clock64() - t_begin;
        p.prof[blockIdx.x * kProfSlots + 1] = w_acc;
        p.prof[blockIdx.x * kProfSlots + 2] = w_a;
        p.prof[blockIdx.x * kProfSlots + 3] = w_c;
      }
#endif
    }
  } else if (warp < 2 + kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int q = warp & 3;
    const int half = ew >> 2;  // this warp's block of kEpiCols columns
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const bool vec = (p.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                     (p.slab_p % 4 == 0);
    uint32_t round = 0;
    for (long long w = w0; w < n_tiles; w += wstep, ++round) {
      int m0, n0;
      tile_of(w, m0, n0);
      // stage the tile's column scales while the MMAs run (kFuse: the
      // converters computed them into escale[round & 1])
      const float* esc = escale + (kFuse ? (round & 1u) * kTile : 0);
      if (!kFuse && ew < 4) {
        const int n = n0 + ew * 32 + lane;
        escale[ew * 32 + lane] = n < p.N ? __ldg(p.sX + n) : 0.f;
      }
      bool got = mbar_wait(acc_full, round & 1u, p.err, kDevTimeoutAcc);
      if (kFuse && got)
        got = mbar_wait(&scale_full[round & 1u], (round >> 1) & 1u, p.err, kDevTimeoutFull);
      if (!group_all<32 * kEpiWarps, 1>(got)) break;
      tc_fence_after();
      const int m = m0 + row;
      const float sa = m < p.M ? __ldg(p.sA + m) : 0.f;
      const int nn = cols_of(n0);
      // combine this thread's 64 columns and park them as fp32
#pragma unroll
      for (int c = half * kEpiCols; c < (half + 1) * kEpiCols; c += 16) {
        int l2[16], l3[16], l4[16];
        tmem_ld16i(lane_base + 0 * kTile + c, l2);
        tmem_ld16i(lane_base + 1 * kTile + c, l3);
        tmem_ld16i(lane_base + 2 * kTile + c, l4);
        tmem_ld_wait();
        float v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = level_combine(l2[k], l3[k], l4[k]) * (sa * esc[c + k]);
        tmem_st16(lane_base + kColPark + c, v);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(acc_empty);  // levels drained: the next tile's MMAs may start
      if (kGMax) mbar_arrive(&scale_free[round & 1u]);  // esc read
      // kSplit, rank 1: add onto rank 0's stored partial, so wait for it
      const bool adder = kSplit && rank == 1;
      if (adder && !group_all<32 * kEpiWarps, 1>(
                       mbar_wait_cluster(out_ready, round & 1u, p.err, kDevTimeoutAcc)))
        break;
      // Eight rounds through the 16-column stage: the warps owning columns
      // [16h, 16h+16) copy them out of TMEM, then all eight warps store
      // 128 rows x 16 columns (4 lanes x float4 per row).
      for (int h = 0; h < kTile / kQCols; ++h) {
        const int c0 = h * kQCols;
        if (half == c0 / kEpiCols) {
          float v[16];
          tmem_ld16(lane_base + kColPark + c0, v);
          tmem_ld_wait();
          float4* dst = reinterpret_cast<float4*>(ostage + row * kQLd);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            dst[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
        }
        group_sync<32 * kEpiWarps, 1>();
        const int ncols = nn - c0;
        const int l4 = lane & 3;
        for (int r = ew * 8 + (lane >> 2); r < kTile; r += 8 * kEpiWarps) {
          const int mm = m0 + r;
          if (mm >= p.M || ncols <= 0) continue;
          float* crow = p.C + (long long)mm * p.ldc + n0 + c0;
          const float* srow = ostage + r * kQLd;
          if (vec && ncols >= kQCols) {
            const float4 v = reinterpret_cast<const float4*>(srow)[l4];
            if (adder)
              red_add_v4(crow + 4 * l4, v);
            else if (kFuse && !kSplit && p.l2hint)  // (kSplit: rank 1 adds to these lines)
              __stcs(reinterpret_cast<float4*>(crow) + l4, v);
            else
              reinterpret_cast<float4*>(crow)[l4] = v;
          } else {
            for (int c = l4; c < ncols && c < kQCols; c += 4) {
              if (adder)
                atomicAdd(crow + c, srow[c]);
              else
                crow[c] = srow[c];
            }
          }
        }
        group_sync<32 * kEpiWarps, 1>();  // stage free for the next round
      }
      if (kSplit) {
        if (rank == 0) {
          // Tell rank 1 that this tile is stored; first make sure rank 1 has
          // taken the previous one, so that out_ready never runs two phases ahead.
          bool ok0 = round == 0 ||
                     mbar_wait_cluster(out_done, (round - 1) & 1u, p.err, kDevTimeoutAcc);
          if (!group_all<32 * kEpiWarps, 1>(ok0)) break;
          mbar_arrive_cluster(mapa(smem_u32(out_ready), peer));
        } else {
          mbar_arrive_cluster(mapa(smem_u32(out_done), peer));
        }
      }
    }
  } else if (kGMax && warp > kAWarp) {
    // ------------------------------------------------------------ max warps
    // Per tile of this CTA, in order: the column maxima of its K range (each
    // lane owns four columns; warp mw reads rows mw, mw + kMaxWarps, ... with
    // kMaxUnroll rows in flight), then the tile's scales. They run at most
    // two tiles ahead of the converters and the epilogue (scale_free).
    const int mw = warp - kAWarp - 1;
    const uint64_t pol = p.l2hint ? l2_policy_evict_last() : l2_policy_evict_first();
    const int kb = k_lo * kKC, ke = (k_hi * kKC < p.K) ? k_hi * kKC : p.K;
    uint32_t round = 0;
    bool ok = true;
#ifdef TT_OZC_PROFILE
    long long w_load = 0, w_free = 0, w_lead = 0;
#endif
    for (long long w = w0; w < n_tiles && ok; w += wstep, ++round) {
      int m0, n0;
      tile_of(w, m0, n0);
      const uint32_t par = round & 1u;
      const int nn = cols_of(n0);
      const int c0 = 4 * lane;
      const long long coff =
          p.slab_p ? (long long)(n0 / p.slab_p) * p.ldx_n + n0 % p.slab_p : (long long)n0;
      const float* col = p.X + coff + c0;
      float mx[4] = {0.f, 0.f, 0.f, 0.f};
      // Read tile r's strip only once the converters have begun tile r - 1,
      // so that a CTA keeps about one strip between its two reads of it and
      // the conversion's re-read still finds it in L2.
#ifdef TT_OZC_PROFILE
      const long long tt0 = clock64();
#endif
      if (round > 0 && !mbar_wait(&cvt_took[par ^ 1u], ((round - 1) >> 1) & 1u, p.err, kDevTimeoutFull))
        ok = false;
      if (!group_all<32 * kMaxWarps, kMaxBar>(ok)) break;
#ifdef TT_OZC_PROFILE
      w_lead += clock64() - tt0;
      const long long tl = clock64();
#endif
      if (c0 + 3 < nn) {
        int k = kb + mw;
        for (; k + (kMaxUnroll - 1) * kMaxWarps < ke; k += kMaxUnroll * kMaxWarps) {
          float4 v[kMaxUnroll];
#pragma unroll
          for (int u = 0; u < kMaxUnroll; ++u)
            v[u] = ldg_nc_hint_v4(col + (long long)(k + u * kMaxWarps) * p.ldx_m, pol);
#pragma unroll
          for (int u = 0; u < kMaxUnroll; ++u) {
            mx[0] = ozd::absmax(mx[0], v[u].x);
            mx[1] = ozd::absmax(mx[1], v[u].y);
            mx[2] = ozd::absmax(mx[2], v[u].z);
            mx[3] = ozd::absmax(mx[3], v[u].w);
          }
        }
        for (; k < ke; k += kMaxWarps) {
          const float4 v = ldg_nc_hint_v4(col + (long long)k * p.ldx_m, pol);
          mx[0] = ozd::absmax(mx[0], v.x);
          mx[1] = ozd::absmax(mx[1], v.y);
          mx[2] = ozd::absmax(mx[2], v.z);
          mx[3] = ozd::absmax(mx[3], v.w);
        }
      } else {
        // ragged last columns (the TMA tile reads zeros there)
        for (int k = kb + mw; k < ke; k += kMaxWarps)
          for (int j = 0; j < 4; ++j)
            if (c0 + j < nn) mx[j] = ozd::absmax(mx[j], __ldg(col + (long long)k * p.ldx_m + j));
      }
#ifdef TT_OZC_PROFILE
      w_load += clock64() - tl;
#endif
      reinterpret_cast<float4*>(gcmax)[mw * 32 + lane] = make_float4(mx[0], mx[1], mx[2], mx[3]);
      group_sync<32 * kMaxWarps, kMaxBar>();
      if (mw == 0) {
        float mm[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          mm[k] = 0.f;
#pragma unroll
          for (int v = 0; v < kMaxWarps; ++v) mm[k] = fmaxf(mm[k], gcmax[v * kTile + c0 + k]);
        }
        if (kSplit) {
          // Same exchange as the ring form: this warp alone reads pmax, in
          // program order before it arrives on the peer's pfull for the next
          // tile, so the peer's write of pmax[par] two tiles later cannot
          // overtake these reads.
          st_cluster_v4(mapa(smem_u32(pmax + par * kTile + c0), peer), mm);
          mbar_arrive_cluster(mapa(smem_u32(&pfull[par]), peer));
          ok = mbar_wait_cluster(&pfull[par], (round >> 1) & 1u, p.err, kDevTimeoutFull);
#pragma unroll
          for (int k = 0; k < 4; ++k) mm[k] = fmaxf(mm[k], pmax[par * kTile + c0 + k]);
        }
        // the epilogue and the converters are done with the scales of the
        // tile two rounds back, which used this buffer
#ifdef TT_OZC_PROFILE
        const long long tf = clock64();
#endif
        if (ok) ok = mbar_wait(&scale_free[par], ((round >> 1) & 1u) ^ 1u, p.err, kDevTimeoutEmpty);
#ifdef TT_OZC_PROFILE
        w_free += clock64() - tf;
#endif
        if (ok) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float sc = ozd::scale_for_max(mm[k]);
            escale[par * kTile + c0 + k] = sc;
            einv[par * kTile + c0 + k] = ozd::inv_scale(sc);
          }
          mbar_arrive(&scale_full[par]);
        }
      }
      // (the next tile's gcmax writes wait here until warp 0 has read it)
      if (!group_all<32 * kMaxWarps, kMaxBar>(ok)) break;
    }
#ifdef TT_OZC_PROFILE
    if (p.prof && mw == 0 && lane == 0) {
      p.prof[blockIdx.x * kProfSlots + 8] = w_load;
      p.prof[blockIdx.x * kProfSlots + 9] = w_free;
      p.prof[blockIdx.x * kProfSlots + 11] = w_lead;
    }
#endif
  } else if (warp < kAWarp) {
    // ----------------------------------------------------------- converters
    const int cw = warp - (2 + kEpiWarps);
    constexpr int kRows = kKC / kCvtWarps;  // rows per warp and stage
    uint32_t itF = 0, itI = 0;  // fp32 ring and int8 ring positions
    bool ok = true;
#ifdef TT_OZC_PROFILE
    long long w_f = 0, w_e = 0, w_s = 0;
#endif
    float inv[4];  // 2^16 / s_n of this lane's four columns of the current tile
    float mx[4];   // running |max| of the same columns of the next tile (kFuse)
    // Wait for the next fp32 slot; false (and nothing to read) after an error.
    auto wait_f = [&]() -> bool {
#ifdef TT_OZC_PROFILE
      const long long t0 = clock64();
#endif
      if (ok && !mbar_wait(&fullF[itF % kFStages], (itF / kFStages) & 1u, p.err, kDevTimeoutFull))
        ok = false;
#ifdef TT_OZC_PROFILE
      w_f += clock64() - t0;
#endif
      return ok;
    };
    // Releasing a landing slot is a write-after-read hand-off across proxies:
    // the converters read the slot with generic shared-memory loads, and the
    // producer's next TMA (the async proxy) rewrites it. An mbarrier
    // release/acquire chain orders generic accesses only, so every converter
    // thread first fences its own reads against the async proxy
    // (fence.proxy.async) and then arrives itself. Without the fence, about
    // one transform in 300 read a slot that the next TMA had already begun
    // to overwrite: the column maxima of a few columns (scales off by a power
    // of two, results off in the last bits) or the digits of an 8-column
    // group came from the following chunk.
    auto release_f = [&]() {
      fence_proxy_async_smem();
      mbar_arrive(&freeF[itF % kFStages]);
      ++itF;
    };
    // One fp32 chunk of the next tile's strip folded into the column maxima.
    auto max_chunk = [&]() {
      if (!wait_f()) return;
      const float4* src = reinterpret_cast<const float4*>(fring + (itF % kFStages) * kFBytes);
#pragma unroll
      for (int j = 0; j < kRows; ++j) {
        const float4 v = src[(cw + kCvtWarps * j) * (kTile / 4) + lane];
        mx[0] = ozd::absmax(mx[0], v.x);
        mx[1] = ozd::absmax(mx[1], v.y);
        mx[2] = ozd::absmax(mx[2], v.z);
        mx[3] = ozd::absmax(mx[3], v.w);
      }
      release_f();
    };
    // Column maxima of all converter warps (and, kSplit, of the peer CTA's
    // half of K) -> scales of this CTA's tile number tr: inv for the
    // converters, escale[tr & 1] + scale_full[tr & 1] for the epilogue. Every
    // converter thread calls this (it holds named barriers).
    auto finish_scales = [&](uint32_t tr) -> bool {
      const uint32_t par = tr & 1u;
      reinterpret_cast<float4*>(cmax)[cw * 32 + lane] = make_float4(mx[0], mx[1], mx[2], mx[3]);
      if (!group_all<32 * kCvtWarps, kCvtBar>(ok)) return false;
      float mm[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        mm[k] = 0.f;
#pragma unroll
        for (int v = 0; v < kCvtWarps; ++v) mm[k] = fmaxf(mm[k], cmax[v * kTile + 4 * lane + k]);
      }
      if (kSplit) {
        // Publish this half's maxima in the peer's pmax[par] and take the
        // peer's. The peer overwrites pmax[par] only for tile tr + 2, after
        // it has waited on pfull for tile tr + 1, which this CTA arrives on
        // after the group_sync below, i.e. after every read of pmax[par].
        if (cw == 0) {
          st_cluster_v4(mapa(smem_u32(pmax + par * kTile + 4 * lane), peer), mm);
          mbar_arrive_cluster(mapa(smem_u32(&pfull[par]), peer));
        }
        const bool got = mbar_wait_cluster(&pfull[par], (tr >> 1) & 1u, p.err, kDevTimeoutFull);
        if (!group_all<32 * kCvtWarps, kCvtBar>(got)) return false;
#pragma unroll
        for (int k = 0; k < 4; ++k) mm[k] = fmaxf(mm[k], pmax[par * kTile + 4 * lane + k]);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float sc = ozd::scale_for_max(mm[k]);
        inv[k] = ozd::inv_scale(sc);
        if (cw == 0) escale[par * kTile + 4 * lane + k] = sc;
      }
      if (cw == 0) mbar_arrive(&scale_full[par]);
      group_sync<32 * kCvtWarps, kCvtBar>();  // cmax free for the next tile
      return true;
    };
    // kFuse requires nkl > kIStages: then a converter that finishes tile r + 1
    // (and writes the scales of tile r + 2 into escale[r & 1]) has waited for
    // an int8 slot that the MMA freed inside tile r + 1, so the epilogue has
    // already read escale[r & 1] and waited on scale_full[r & 1] for tile r.
    if (kFuse && !kGMax && w0 < n_tiles) {
      mx[0] = mx[1] = mx[2] = mx[3] = 0.f;
      for (int kc = 0; kc < nkl; ++kc) max_chunk();
      if (!finish_scales(0)) ok = false;
    }
    uint32_t round = 0;
    for (long long w = w0; w < n_tiles && ok; w += wstep, ++round) {
      int m0, n0;
      tile_of(w, m0, n0);
      const bool next = kFuse && !kGMax && w + wstep < n_tiles;
      if (kGMax) {
        const uint32_t par = round & 1u;
#ifdef TT_OZC_PROFILE
        const long long ts = clock64();
#endif
        if (!mbar_wait(&scale_full[par], (round >> 1) & 1u, p.err, kDevTimeoutFull)) {
          ok = false;
          break;
        }
#ifdef TT_OZC_PROFILE
        w_s += clock64() - ts;
#endif
#pragma unroll
        for (int k = 0; k < 4; ++k) inv[k] = einv[par * kTile + 4 * lane + k];
        mbar_arrive(&scale_free[par]);
        mbar_arrive(&cvt_took[par]);
      } else if (!kFuse) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int n = n0 + 4 * lane + k;
          const float sc = n < p.N ? __ldg(p.sX + n) : 0.f;
          inv[k] = ozd::inv_scale(sc);
        }
      }
      mx[0] = mx[1] = mx[2] = mx[3] = 0.f;
      for (int kc = 0; kc < nkl; ++kc) {
        const int s = itI % kIStages;
        const uint32_t ph = (itI / kIStages) & 1u;
        ++itI;
        if (!wait_f()) continue;  // error: run on without waiting, to the next group_all
        const float4* src = reinterpret_cast<const float4*>(fring + (itF % kFStages) * kFBytes);
        // Split this warp's rows into registers first, then release the
        // slot (each thread fences and arrives for its own loads), so that
        // the producer can refill it while the digits wait for an int8 slot.
        uint32_t q[kRows][3];
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
          const float4 v = src[(cw + kCvtWarps * j) * (kTile / 4) + lane];
          const float x4[4] = {v.x, v.y, v.z, v.w};
          ozd::split4(x4, inv, q[j][0], q[j][1], q[j][2]);  // one FMA per value
        }
        release_f();  // this warp's rows are consumed
#ifdef TT_OZC_PROFILE
        long long t2 = clock64();
#endif
        if (!mbar_wait(&emptyI[s], ph ^ 1u, p.err, kDevTimeoutEmpty)) {
          ok = false;
          continue;
        }
#ifdef TT_OZC_PROFILE
        w_e += clock64() - t2;
#endif
        uint8_t* tile = iring + s * kIBytes + kARegion;
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
          const int r = cw + kCvtWarps * j;
          // MN-major SW128 atom: 8 k-rows x 128 bytes; the 16-byte chunk
          // index (lane / 4) is XORed with (row mod 8).
          const int off = (r >> 3) * 1024 + (r & 7) * 128 + ((((lane >> 2) ^ (r & 7))) << 4) +
                          (lane & 3) * 4;
          *reinterpret_cast<uint32_t*>(tile + 0 * oz::kSliceTile + off) = q[j][0];
          *reinterpret_cast<uint32_t*>(tile + 1 * oz::kSliceTile + off) = q[j][1];
          *reinterpret_cast<uint32_t*>(tile + 2 * oz::kSliceTile + off) = q[j][2];
        }
        // each thread makes its own slice writes visible to the tensor cores
        // and arrives (conv counts every converter thread)
        fence_proxy_async_smem();
        mbar_arrive(&conv[s]);
        if (next) max_chunk();  // the producer queued it right after this chunk
      }
      if (next && !finish_scales(round + 1)) ok = false;
    }
#ifdef TT_OZC_PROFILE
    if (p.prof && cw == 0 && lane == 0) {
      p.prof[blockIdx.x * kProfSlots + 4] = w_f;
      p.prof[blockIdx.x * kProfSlots + 5] = w_e;
      p.prof[blockIdx.x * kProfSlots + 10] = w_s;
    }
#endif
  }

  tc_fence_before();
  __syncthreads();
  if (kSplit) cluster_sync();  // no remote access to this CTA's shared memory is left
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool kFuse, int kFStages = kFStagesDefault, int kIStages = kIStagesDefault>
static __global__ void __launch_bounds__(kThreads, 1)
    gemm_cvt_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapX,
                    Params p) {
  gemm_cvt_body<kFuse, false, false, kFStages, kIStages>(mapA, mapX, p);
}

template <int kFStages = kFStagesDefault, int kIStages = kIStagesDefault>
static __global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_cvt_split_kernel(const __grid_constant__ CUtensorMap mapA,
                          const __grid_constant__ CUtensorMap mapX, Params p) {
  gemm_cvt_body<true, true, false, kFStages, kIStages>(mapA, mapX, p);
}

// Fused scales from the max warps (kGMax): one CTA per tile, or split K over
// a cluster of two CTAs (the pair exchanges maxima and partial tiles through
// distributed shared memory, so that form needs the cluster launch).
template <int kFStages, int kIStages>
static __global__ void __launch_bounds__(kThreadsG, 1)
    gemm_cvt_gmax_kernel(const __grid_constant__ CUtensorMap mapA,
                         const __grid_constant__ CUtensorMap mapX, Params p) {
  gemm_cvt_body<true, false, true, kFStages, kIStages>(mapA, mapX, p);
}
template <int kFStages, int kIStages>
static __global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreadsG, 1)
    gemm_cvt_gmax_split_kernel(const __grid_constant__ CUtensorMap mapA,
                               const __grid_constant__ CUtensorMap mapX, Params p) {
  gemm_cvt_body<true, true, true, kFStages, kIStages>(mapA, mapX, p);
}

}  // namespace ozc
}  // namespace tt
