// C-ABI entry points for the AO->MO transform (two-step form).
#include "ao2mo_simt.cuh"
#include "common.cuh"
#include "ozaki_gemm.cuh"
#include "ozaki_gemm_cvt.cuh"
#include "ozaki_gemm64.cuh"

#include <cstdlib>

namespace tt {
namespace {

std::once_flag g_flags[kMaxDevices];
int g_ok[kMaxDevices];
int g_sms[kMaxDevices];
int g_split_clusters[kMaxDevices];  // co-resident 2-CTA clusters of gemm_cvt_split_kernel
int g_gmax_clusters[kMaxDevices];   // the same for gemm_cvt_gmax_split_kernel

int setup(int dev) {
  return once_per_device(g_flags, g_ok, dev, [dev]() -> int {
    if (cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return TT_ERR_CUDA;
    const int sm32 = ozc::smem_bytes(3, 2), sm23 = ozc::smem_bytes(2, 3);
    if (cudaFuncSetAttribute(ozc::gemm_cvt_kernel<false, 3, 2>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, sm32) != cudaSuccess ||
        cudaFuncSetAttribute(ozc::gemm_cvt_kernel<true, 3, 2>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, sm32) != cudaSuccess ||
        cudaFuncSetAttribute(ozc::gemm_cvt_split_kernel<3, 2>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, sm32) != cudaSuccess ||
        cudaFuncSetAttribute(ozc::gemm_cvt_kernel<false, 2, 3>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, sm23) != cudaSuccess ||
        cudaFuncSetAttribute(ozc::gemm_cvt_kernel<true, 2, 3>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, sm23) != cudaSuccess ||
        cudaFuncSetAttribute(ozc::gemm_cvt_split_kernel<2, 3>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, sm23) != cudaSuccess)
      return TT_ERR_CUDA;
    {
      // A persistent grid of more clusters than fit at once would leave a
      // tail of clusters running alone: size the grid to what is co-resident.
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(2 * 1024, 1, 1);
      cfg.blockDim = dim3(ozc::kThreads, 1, 1);
      cfg.dynamicSmemBytes = sm32;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0, n23 = 0;
      if (cudaOccupancyMaxActiveClusters(&n, ozc::gemm_cvt_split_kernel<3, 2>, &cfg) !=
          cudaSuccess)
        return TT_ERR_CUDA;
      cfg.dynamicSmemBytes = sm23;
      if (cudaOccupancyMaxActiveClusters(&n23, ozc::gemm_cvt_split_kernel<2, 3>, &cfg) !=
          cudaSuccess)
        return TT_ERR_CUDA;
      g_split_clusters[dev] = n < n23 ? n : n23;
      const int smg = ozc::smem_bytes(3, 2, true);
      if (cudaFuncSetAttribute(ozc::gemm_cvt_gmax_split_kernel<3, 2>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, smg) != cudaSuccess ||
          cudaFuncSetAttribute(ozc::gemm_cvt_gmax_kernel<3, 2>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, smg) != cudaSuccess)
        return TT_ERR_CUDA;
      cfg.blockDim = dim3(ozc::kThreadsG, 1, 1);
      cfg.dynamicSmemBytes = smg;
      int ng = 0;
      if (cudaOccupancyMaxActiveClusters(&ng, ozc::gemm_cvt_gmax_split_kernel<3, 2>, &cfg) !=
          cudaSuccess)
        return TT_ERR_CUDA;
      g_gmax_clusters[dev] = ng;
    }
    if (cudaFuncSetAttribute(oz64::gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             oz64::kSmemBytes) != cudaSuccess)
      return TT_ERR_CUDA;
    if (cudaFuncSetAttribute(oz::gemm_kernel<false, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             oz::kSmemBytes) != cudaSuccess)
      return TT_ERR_CUDA;
    return TT_OK;
  });
}

inline size_t pad16(size_t x) { return (x + 15) / 16 * 16; }
inline size_t al256(size_t x) { return (x + 255) / 256 * 256; }

// Layout of the tensor-core workspace (all offsets 256-byte aligned).
struct OzLayout {
  size_t qo, so, qv, sv, qe, se, inter, qi, si, total;
  OzLayout(size_t nbf, size_t nocc, size_t nvir, size_t naux) {
    size_t o = 0;
    auto take = [&o](size_t bytes) { size_t r = o; o += al256(bytes); return r; };
    qo = take(3 * nbf * pad16(nocc) * ozc::kARep);  // replicated for the on-chip path
    so = take(4 * pad16(nocc) * ozc::kARep);
    qv = take(3 * nbf * pad16(nvir));
    sv = take(4 * pad16(nvir));
    qe = take(3 * nbf * pad16(nbf * naux));
    se = take(4 * pad16(nbf * naux));
    inter = take(4 * nocc * nbf * naux);
    qi = take(3 * nocc * nbf * pad16(naux));
    si = take(4 * nocc * pad16(naux));
    total = o;
  }
};

int split_cols(const float* X, long long ldx, long long bsx, int batch, int K, int N, int npad,
               int8_t* Q, float* S, cudaStream_t s, int sms) {
  const long long nblk = (long long)batch * ((npad + oz::kSplitCols - 1) / oz::kSplitCols);
  const long long cap = (long long)sms * 8;
  const int grid = (int)(nblk < cap ? nblk : cap);
  // One read of X (colmax_slice_kernel) unless TRNTENSOR_B200_SPLIT_TWOPASS=1.
  const char* tp = std::getenv("TRNTENSOR_B200_SPLIT_TWOPASS");
  if (tp != nullptr && tp[0] == '1') {
    oz::colmax_kernel<<<grid, oz::kSplitThreads, 0, s>>>(X, ldx, bsx, batch, K, N, npad, S);
    oz::slice_kernel<<<grid, oz::kSplitThreads, 0, s>>>(X, ldx, bsx, batch, K, N, npad, S, Q);
  } else {
    const int g1 = (int)(nblk < sms ? nblk : sms);
    oz::colmax_slice_kernel<<<g1, oz::kFusedThreads, 0, s>>>(X, ldx, bsx, batch, K, N, npad, S, Q);
  }
  return cuda_status(cudaGetLastError());
}

// Tensor map over slice planes Q[3][batch][K][npad] (bytes), box 128 x 64 x 1 x 3.
int slice_map(CUtensorMap* m, const int8_t* Q, int npad, int K, int batch) {
  const uint64_t dims[4] = {(uint64_t)npad, (uint64_t)K, (uint64_t)batch, 3};
  const uint64_t strides[3] = {(uint64_t)npad, (uint64_t)npad * K, (uint64_t)npad * K * batch};
  const uint32_t box[4] = {(uint32_t)oz::kTile, (uint32_t)oz::kKC, 1, 3};
  return encode_tmap(m, Q, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_DATA_TYPE_UINT8);
}

int oz_gemm(const int8_t* QA, const float* SA, int mpad, int batchA, const int8_t* QB,
            const float* SB, int npad, int batch, int M, int N, int K, float* C, long long ldc,
            long long strideC, int* err, cudaStream_t s, int sms) {
  CUtensorMap ma, mb;
  if (slice_map(&ma, QA, mpad, K, batchA) || slice_map(&mb, QB, npad, K, batch)) return TT_ERR_TMA;
  oz::Params p;
  p.sA = SA;
  p.sB = SB;
  p.ldsA = mpad;
  p.ldsB = npad;
  p.C = C;
  p.ldc = ldc;
  p.strideC = strideC;
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = batch;
  p.shared_A = batchA == 1 && batch > 1;
  p.tiles_m = (M + oz::kTile - 1) / oz::kTile;
  p.tiles_n = (N + oz::kTile - 1) / oz::kTile;
  p.err = err;
  const long long tiles = (long long)p.tiles_m * p.tiles_n * batch;
  const int grid = (int)(tiles < sms ? tiles : sms);
  oz::gemm_kernel<false, false><<<grid, oz::kThreads, oz::kSmemBytes, s>>>(ma, mb, p);
  return cuda_status(cudaGetLastError());
}

// fp64 tensor-core workspace: six digit planes per operand, fp64 scales.
struct OzLayout64 {
  size_t qo, so, qv, sv, qe, se, inter, qi, si, total;
  OzLayout64(size_t nbf, size_t nocc, size_t nvir, size_t naux) {
    size_t o = 0;
    auto take = [&o](size_t bytes) { size_t r = o; o += al256(bytes); return r; };
    constexpr size_t D = oz64::kDigits;
    qo = take(D * nbf * pad16(nocc));
    so = take(8 * pad16(nocc));
    qv = take(D * nbf * pad16(nvir));
    sv = take(8 * pad16(nvir));
    qe = take(D * nbf * pad16(nbf * naux));
    se = take(8 * pad16(nbf * naux));
    inter = take(8 * nocc * nbf * naux);
    qi = take(D * nocc * nbf * pad16(naux));
    si = take(8 * nocc * pad16(naux));
    total = o;
  }
};

int split_cols64(const double* X, long long ldx, long long bsx, int batch, int K, int N, int npad,
                 int8_t* Q, double* S, cudaStream_t s, int sms) {
  const long long nblk = (long long)batch * ((npad + oz64::kSplitCols - 1) / oz64::kSplitCols);
  const long long cap = (long long)sms * 8;
  const int grid = (int)(nblk < cap ? nblk : cap);
  oz64::colmax_kernel<<<grid, oz64::kSplitThreads, 0, s>>>(X, ldx, bsx, batch, K, N, npad, S);
  oz64::slice_kernel<<<grid, oz64::kSplitThreads, 0, s>>>(X, ldx, bsx, batch, K, N, npad, S, Q);
  return cuda_status(cudaGetLastError());
}

// Tensor map over digit planes Q[6][batch][K][npad], box 128 x 32 x 1 x nd.
int slice_map64(CUtensorMap* m, const int8_t* Q, int npad, int K, int batch, int nd) {
  const uint64_t dims[4] = {(uint64_t)npad, (uint64_t)K, (uint64_t)batch,
                            (uint64_t)oz64::kDigits};
  const uint64_t strides[3] = {(uint64_t)npad, (uint64_t)npad * K, (uint64_t)npad * K * batch};
  const uint32_t box[4] = {(uint32_t)oz64::kTile, (uint32_t)oz64::kKC, 1, (uint32_t)nd};
  return encode_tmap(m, Q, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_DATA_TYPE_UINT8);
}

int oz_gemm64(const int8_t* QA, const double* SA, int mpad, int batchA, const int8_t* QB,
              const double* SB, int npad, int batch, int M, int N, int K, double* C,
              long long ldc, long long strideC, int* err, cudaStream_t s, int sms) {
  CUtensorMap a3, a5, b3, b5;
  if (slice_map64(&a3, QA, mpad, K, batchA, 3) ||
      slice_map64(&a5, QA, mpad, K, batchA, oz64::kDigits) ||
      slice_map64(&b3, QB, npad, K, batch, 3) ||
      slice_map64(&b5, QB, npad, K, batch, oz64::kDigits))
    return TT_ERR_TMA;
  oz64::Params p;
  p.sA = SA;
  p.sB = SB;
  p.ldsA = mpad;
  p.ldsB = npad;
  p.C = C;
  p.ldc = ldc;
  p.strideC = strideC;
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = batch;
  p.shared_A = batchA == 1 && batch > 1;
  p.tiles_m = (M + oz64::kTile - 1) / oz64::kTile;
  p.tiles_n = (N + oz64::kTile - 1) / oz64::kTile;
  p.err = err;
  const long long tiles = (long long)p.tiles_m * p.tiles_n * batch;
  const int grid = (int)(tiles < sms ? tiles : sms);
  oz64::gemm_kernel<<<grid, oz64::kThreads, oz64::kSmemBytes, s>>>(a3, a5, b3, b5, p);
  return cuda_status(cudaGetLastError());
}

template <typename T>
int launch_gemm(const ao2mo::GemmParams<T>& p, cudaStream_t s, int sms) {
  constexpr int BM = sizeof(T) == 4 ? 128 : 64;
  constexpr int BN = sizeof(T) == 4 ? 128 : 64;
  constexpr int TM = sizeof(T) == 4 ? 8 : 4;
  constexpr int TN = sizeof(T) == 4 ? 8 : 4;
  constexpr int BK = 16;
  const long long tiles =
      (long long)((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN) * (long long)p.batch;
  if (tiles == 0) return TT_OK;
  const long long cap = (long long)sms * 4;
  const int grid = (int)(tiles < cap ? tiles : cap);
  ao2mo::gemm_at_b<T, BM, BN, BK, TM, TN><<<grid, (BM / TM) * (BN / TN), 0, s>>>(p);
  return cuda_status(cudaGetLastError());
}

template <typename T>
int ao2mo_simt(const T* eri, const T* C_occ, const T* C_vir, int nbf, int nocc, int nvir,
               int naux, void* workspace, size_t workspace_bytes, T* B_out, void* stream) {
  if (!eri || !C_occ || !C_vir || !workspace || !B_out) return TT_ERR_NULL;
  if (nbf <= 0 || nocc <= 0 || nvir <= 0 || naux <= 0) return TT_ERR_SHAPE;
  const size_t need = (size_t)nocc * nbf * naux * sizeof(T);
  if (workspace_bytes < need) return TT_ERR_WORKSPACE;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = setup(dev);
  if (st != TT_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  T* inter = static_cast<T*>(workspace);
  // step 1: inter (nocc, nbf*naux) = C_occ^T (nocc x nbf) . eri (nbf x nbf*naux)
  ao2mo::GemmParams<T> p1{C_occ, eri, inter, nocc, (long long)nbf * naux, (long long)nbf * naux,
                          0, 0, 0, nocc, nbf * naux, nbf, 1};
  st = launch_gemm<T>(p1, s, g_sms[dev]);
  if (st != TT_OK) return st;
  // step 2: B_out[i] (nvir, naux) = C_vir^T (nvir x nbf) . inter[i] (nbf x naux)
  ao2mo::GemmParams<T> p2{C_vir, inter, B_out, nvir, naux, naux,
                          0, (long long)nbf * naux, (long long)nvir * naux,
                          nvir, naux, nbf, nocc};
  return launch_gemm<T>(p2, s, g_sms[dev]);
}

}  // namespace
}  // namespace tt

// Per-CTA wait-cycle counters exist only in TT_OZC_PROFILE builds (a
// measurement build, never the shipped library).
#ifdef TT_OZC_PROFILE
static long long* g_ozc_prof = nullptr;
extern "C" void tt_debug_set_ao2mo_profile_buffer(long long* buf) { g_ozc_prof = buf; }
#endif

extern "C" {

size_t tt_ao2mo_workspace_bytes(int nbf, int nocc, int nvir, int naux, int elem_bytes) {
  if (nbf <= 0 || nocc <= 0 || nvir <= 0 || naux <= 0) return 0;
  if (elem_bytes == 4) return tt::OzLayout(nbf, nocc, nvir, naux).total;
  if (elem_bytes == 8) return (size_t)nocc * nbf * naux * 8;
  return 0;
}

// ld_m / ld_n: eri strides (elements) of its m and n indices; a contiguous
// eri has ld_n = naux, ld_m = nbf * naux. slab: eri is a strided P-slab
// (ld_n > naux possible), read through a 3-D tensor map by the fused step 1.
static int ao2mo_f32_impl(const float* eri, long long ld_m, long long ld_n, bool slab,
                          const float* C_occ, const float* C_vir, int nbf, int nocc, int nvir,
                          int naux, void* workspace, size_t workspace_bytes, float* B_out,
                          int* dev_status, void* stream) {
  using namespace tt;
  if (!eri || !C_occ || !C_vir || !workspace || !B_out || !dev_status) return TT_ERR_NULL;
  if (nbf <= 0 || nocc <= 0 || nvir <= 0 || naux <= 0) return TT_ERR_SHAPE;
  if ((long long)nbf * naux > 0x7fffffffLL) return TT_ERR_SHAPE;
  if (nbf > ozd::kMaxK) return TT_ERR_SHAPE;  // int32 slice sums exact up to this K
  const OzLayout L(nbf, nocc, nvir, naux);
  if (workspace_bytes < L.total) return TT_ERR_WORKSPACE;
  if (!aligned16(workspace)) return TT_ERR_ALIGN;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = setup(dev);
  if (st != TT_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  TT_CUDA(cudaMemsetAsync(dev_status, 0, sizeof(int), s));
  char* w = static_cast<char*>(workspace);
  int8_t* qo = (int8_t*)(w + L.qo);
  float* so = (float*)(w + L.so);
  int8_t* qv = (int8_t*)(w + L.qv);
  float* sv = (float*)(w + L.sv);
  int8_t* qe = (int8_t*)(w + L.qe);
  float* se = (float*)(w + L.se);
  float* inter = (float*)(w + L.inter);
  int8_t* qi = (int8_t*)(w + L.qi);
  float* si = (float*)(w + L.si);
  const int sms = g_sms[dev];
  const int po = (int)pad16(nocc), pv = (int)pad16(nvir), pe = (int)pad16((size_t)nbf * naux),
            pa = (int)pad16(naux);
  const long long ncol = (long long)nbf * naux;
  const char* pre = std::getenv("TRNTENSOR_B200_AO2MO_PRESLICE");
  const bool preslice =
      !slab && ((pre != nullptr && pre[0] == '1') || (ncol % 4 != 0) || !aligned16(eri));
  if (slab) {
    // the fused on-chip split (its own column scales) is the only slab reader
    const int istages = 2;
    if ((nbf + ozc::kKC - 1) / ozc::kKC < istages + 1) return TT_ERR_SHAPE;
    if (!aligned16(eri) || ld_n % 4 != 0 || ld_m % 4 != 0) return TT_ERR_ALIGN;
    if (ld_n < naux || ld_m < ld_n * nbf) return TT_ERR_SHAPE;
  }
  // Column-scaled int8 slices of C_occ and C_vir. For the on-chip path C_occ's
  // slices are written kARep times (batch stride 0 on the source): every CTA
  // re-reads them for each tile, and spreading those reads over several copies
  // keeps them off a few hot L2 lines.
  if ((st = split_cols(C_occ, nocc, 0, preslice ? 1 : ozc::kARep, nbf, nocc, po, qo, so, s, sms)))
    return st;
  if ((st = split_cols(C_vir, nvir, 0, 1, nbf, nvir, pv, qv, sv, s, sms))) return st;
  if (preslice) {
    // eri split into int8 slices in HBM, then the generic slice GEMM
    if ((st = split_cols(eri, ncol, 0, 1, nbf, nbf * naux, pe, qe, se, s, sms))) return st;
    // step 1: inter[i][(n,P)] = sum_m C_occ[m][i] eri[m][(n,P)]
    if ((st = oz_gemm(qo, so, po, 1, qe, se, pe, 1, nocc, nbf * naux, nbf, inter, ncol, 0,
                      dev_status, s, sms)))
      return st;
  } else {
    // The GEMM splits fp32 eri tiles on chip. Its column scales come from the
    // GEMM itself (one HBM read of eri) when the contraction has more than two
    // 64-row chunks, else from a separate column-max pass.
    // TRNTENSOR_B200_AO2MO_RING=23: 2 fp32 + 3 int8 ring slots instead of 3 + 2.
    const char* rg = std::getenv("TRNTENSOR_B200_AO2MO_RING");
    const bool ring23 = rg != nullptr && rg[0] == '2' && rg[1] == '3';
    const int istages = ring23 ? 3 : 2;
    // The fused column scales need more k-chunks than int8 slots per CTA
    // (ozaki_gemm_cvt.cuh); with fewer, a separate column-max pass runs.
    const char* cm = std::getenv("TRNTENSOR_B200_AO2MO_COLMAX");
    const int nkc = (nbf + ozc::kKC - 1) / ozc::kKC;
    const bool fuse = slab || (nkc >= istages + 1 && !(cm != nullptr && cm[0] == '1'));
    if (slab && nkc < istages + 1) return TT_ERR_SHAPE;
    // Split-K over CTA pairs: each half needs as many k-chunks.
    const char* sk = std::getenv("TRNTENSOR_B200_AO2MO_SPLITK");
    const bool split = fuse && nkc / 2 >= istages + 1 && g_split_clusters[dev] > 0 &&
                       !(sk != nullptr && sk[0] == '0');
    if (!fuse) {
      const long long nblk = (pe + oz::kSplitCols - 1) / oz::kSplitCols;
      const int g = (int)(nblk < (long long)sms * 8 ? nblk : (long long)sms * 8);
      oz::colmax_kernel<<<g, oz::kSplitThreads, 0, s>>>(eri, ncol, 0, 1, nbf, nbf * naux, pe, se);
      if ((st = cuda_status(cudaGetLastError()))) return st;
    }
    CUtensorMap ma, mx;
    const uint64_t xd[2] = {(uint64_t)ncol, (uint64_t)nbf};
    const uint64_t xs[1] = {(uint64_t)ncol * 4};
    const uint32_t xb[2] = {(uint32_t)ozc::kTile, (uint32_t)ozc::kKC};
    if (slice_map(&ma, qo, po, nbf, ozc::kARep)) return TT_ERR_TMA;
    if (slab) {
      // (P, n, m) with strides ld_n, ld_m; box 128 P x 1 n x 64 m
      const uint64_t sd[3] = {(uint64_t)naux, (uint64_t)nbf, (uint64_t)nbf};
      const uint64_t ss[2] = {(uint64_t)ld_n * 4, (uint64_t)ld_m * 4};
      const uint32_t sb[3] = {(uint32_t)ozc::kTile, 1u, (uint32_t)ozc::kKC};
      if (encode_tmap(&mx, eri, 3, sd, ss, sb, CU_TENSOR_MAP_SWIZZLE_NONE)) return TT_ERR_TMA;
    } else if (encode_tmap(&mx, eri, 2, xd, xs, xb, CU_TENSOR_MAP_SWIZZLE_NONE)) {
      return TT_ERR_TMA;
    }
    ozc::Params pc;
    pc.sA = so;
    pc.sX = se;
    pc.C = inter;
    pc.ldc = ncol;
    pc.M = nocc;
    pc.N = nbf * naux;
    pc.K = nbf;
    pc.tiles_m = (nocc + ozc::kTile - 1) / ozc::kTile;
    pc.slab_p = slab ? naux : 0;
    pc.tiles_p = (naux + ozc::kTile - 1) / ozc::kTile;
    pc.tiles_n = slab ? nbf * pc.tiles_p : (int)((ncol + ozc::kTile - 1) / ozc::kTile);
    pc.err = dev_status;
#ifdef TT_OZC_PROFILE
    pc.prof = g_ozc_prof;
#else
    pc.prof = nullptr;
#endif
    const char* hint = std::getenv("TRNTENSOR_B200_AO2MO_L2HINT");
    pc.l2hint = !(hint != nullptr && hint[0] == '0');  // on unless set to 0
    pc.X = eri;
    pc.ldx_m = slab ? ld_m : ncol;
    pc.ldx_n = slab ? ld_n : 0;
    // Column maxima from the max warps' global loads (default; 3 + 2 ring,
    // one CTA per tile unless TRNTENSOR_B200_AO2MO_SPLITK=1) or through the
    // landing ring (TRNTENSOR_B200_AO2MO_GMAX=0).
    const char* gm = std::getenv("TRNTENSOR_B200_AO2MO_GMAX");
    const bool gmax = fuse && !ring23 && !(gm != nullptr && gm[0] == '0');
    const bool gsplit = gmax && split && sk != nullptr && sk[0] == '1' && g_gmax_clusters[dev] > 0;
    const long long tiles = (long long)pc.tiles_m * pc.tiles_n;
    const int grid = (int)(tiles < sms ? tiles : sms);
    const int smem = ozc::smem_bytes(ring23 ? 2 : 3, istages);
    const long long cl = tiles < g_split_clusters[dev] ? tiles : g_split_clusters[dev];
    if (gmax) {
      const int smg = ozc::smem_bytes(3, 2, true);
      const long long cg = tiles < g_gmax_clusters[dev] ? tiles : g_gmax_clusters[dev];
      if (gsplit)
        ozc::gemm_cvt_gmax_split_kernel<3, 2><<<(int)(2 * cg), ozc::kThreadsG, smg, s>>>(ma, mx, pc);
      else
        ozc::gemm_cvt_gmax_kernel<3, 2><<<grid, ozc::kThreadsG, smg, s>>>(ma, mx, pc);
    } else if (ring23) {
      if (split)
        ozc::gemm_cvt_split_kernel<2, 3><<<(int)(2 * cl), ozc::kThreads, smem, s>>>(ma, mx, pc);
      else if (fuse)
        ozc::gemm_cvt_kernel<true, 2, 3><<<grid, ozc::kThreads, smem, s>>>(ma, mx, pc);
      else
        ozc::gemm_cvt_kernel<false, 2, 3><<<grid, ozc::kThreads, smem, s>>>(ma, mx, pc);
    } else {
      if (split)
        ozc::gemm_cvt_split_kernel<3, 2><<<(int)(2 * cl), ozc::kThreads, smem, s>>>(ma, mx, pc);
      else if (fuse)
        ozc::gemm_cvt_kernel<true, 3, 2><<<grid, ozc::kThreads, smem, s>>>(ma, mx, pc);
      else
        ozc::gemm_cvt_kernel<false, 3, 2><<<grid, ozc::kThreads, smem, s>>>(ma, mx, pc);
    }
    if ((st = cuda_status(cudaGetLastError()))) return st;
  }
  // slices of inter[i] (K = n, N = P), scales per (i, P)
  if ((st = split_cols(inter, naux, (long long)nbf * naux, nocc, nbf, naux, pa, qi, si, s, sms)))
    return st;
  // step 2: B_out[i][a][P] = sum_n C_vir[n][a] inter[i][n][P]
  return oz_gemm(qv, sv, pv, 1, qi, si, pa, nocc, nvir, naux, nbf, B_out, naux,
                 (long long)nvir * naux, dev_status, s, sms);
}

int tt_ao2mo_f32(const float* eri, const float* C_occ, const float* C_vir, int nbf, int nocc,
                 int nvir, int naux, void* workspace, size_t workspace_bytes, float* B_out,
                 int* dev_status, void* stream) {
  return ao2mo_f32_impl(eri, (long long)nbf * naux, naux, false, C_occ, C_vir, nbf, nocc, nvir,
                        naux, workspace, workspace_bytes, B_out, dev_status, stream);
}

int tt_ao2mo_f32_slab(const float* eri, long long ld_m, long long ld_n, const float* C_occ,
                      const float* C_vir, int nbf, int nocc, int nvir, int naux_local,
                      void* workspace, size_t workspace_bytes, float* B_out, int* dev_status,
                      void* stream) {
  return ao2mo_f32_impl(eri, ld_m, ld_n, true, C_occ, C_vir, nbf, nocc, nvir, naux_local,
                        workspace, workspace_bytes, B_out, dev_status, stream);
}

size_t tt_ao2mo_f64_workspace_bytes(int nbf, int nocc, int nvir, int naux) {
  if (nbf <= 0 || nocc <= 0 || nvir <= 0 || naux <= 0) return 0;
  return tt::OzLayout64(nbf, nocc, nvir, naux).total;
}

int tt_ao2mo_f64_tc(const double* eri, const double* C_occ, const double* C_vir, int nbf,
                    int nocc, int nvir, int naux, void* workspace, size_t workspace_bytes,
                    double* B_out, int* dev_status, void* stream) {
  using namespace tt;
  if (!eri || !C_occ || !C_vir || !workspace || !B_out || !dev_status) return TT_ERR_NULL;
  if (nbf <= 0 || nocc <= 0 || nvir <= 0 || naux <= 0) return TT_ERR_SHAPE;
  if ((long long)nbf * naux > 0x7fffffffLL) return TT_ERR_SHAPE;
  if (nbf > oz64::kMaxK) return TT_ERR_SHAPE;  // int32 digit sums exact up to this K
  const OzLayout64 L(nbf, nocc, nvir, naux);
  if (workspace_bytes < L.total) return TT_ERR_WORKSPACE;
  if (!aligned16(workspace)) return TT_ERR_ALIGN;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = setup(dev);
  if (st != TT_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  TT_CUDA(cudaMemsetAsync(dev_status, 0, sizeof(int), s));
  char* w = static_cast<char*>(workspace);
  int8_t* qo = (int8_t*)(w + L.qo);
  double* so = (double*)(w + L.so);
  int8_t* qv = (int8_t*)(w + L.qv);
  double* sv = (double*)(w + L.sv);
  int8_t* qe = (int8_t*)(w + L.qe);
  double* se = (double*)(w + L.se);
  double* inter = (double*)(w + L.inter);
  int8_t* qi = (int8_t*)(w + L.qi);
  double* si = (double*)(w + L.si);
  const int sms = g_sms[dev];
  const int po = (int)pad16(nocc), pv = (int)pad16(nvir), pe = (int)pad16((size_t)nbf * naux),
            pa = (int)pad16(naux);
  const long long ncol = (long long)nbf * naux;
  if ((st = split_cols64(C_occ, nocc, 0, 1, nbf, nocc, po, qo, so, s, sms))) return st;
  if ((st = split_cols64(C_vir, nvir, 0, 1, nbf, nvir, pv, qv, sv, s, sms))) return st;
  if ((st = split_cols64(eri, ncol, 0, 1, nbf, nbf * naux, pe, qe, se, s, sms))) return st;
  // step 1: inter[i][(n,P)] = sum_m C_occ[m][i] eri[m][(n,P)]
  if ((st = oz_gemm64(qo, so, po, 1, qe, se, pe, 1, nocc, nbf * naux, nbf, inter, ncol, 0,
                      dev_status, s, sms)))
    return st;
  // digits of inter[i] (K = n, N = P), scales per (i, P)
  if ((st = split_cols64(inter, naux, (long long)nbf * naux, nocc, nbf, naux, pa, qi, si, s, sms)))
    return st;
  // step 2: B_out[i][a][P] = sum_n C_vir[n][a] inter[i][n][P]
  return oz_gemm64(qv, sv, pv, 1, qi, si, pa, nocc, nvir, naux, nbf, B_out, naux,
                   (long long)nvir * naux, dev_status, s, sms);
}

int tt_ao2mo_simt_f32(const float* eri, const float* C_occ, const float* C_vir, int nbf, int nocc,
                 int nvir, int naux, void* workspace, size_t workspace_bytes, float* B_out,
                 void* stream) {
  return tt::ao2mo_simt<float>(eri, C_occ, C_vir, nbf, nocc, nvir, naux, workspace,
                               workspace_bytes, B_out, stream);
}

int tt_ao2mo_f64(const double* eri, const double* C_occ, const double* C_vir, int nbf,
                 int nocc, int nvir, int naux, void* workspace, size_t workspace_bytes,
                 double* B_out, void* stream) {
  return tt::ao2mo_simt<double>(eri, C_occ, C_vir, nbf, nocc, nvir, naux, workspace,
                                workspace_bytes, B_out, stream);
}

}  // extern "C"
