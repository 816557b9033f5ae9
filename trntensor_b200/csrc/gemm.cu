// fp32-accurate (batched) GEMM on int8 tensor cores for einsum's matmul /
// bmm strategies: C[b] = A[b] (M x K) . B[b] (K x N), fp32 in and out.
// Each operand may be given K-major (rows of k contiguous) or MN-major
// (rows of m / n contiguous); it is split into three int8 slices with a
// power-of-two scale per m (resp. n) along k (Ozaki scheme), and the six
// slice GEMMs accumulate exactly in int32 TMEM (csrc/ozaki_gemm.cuh).
#include "common.cuh"
#include "mp2_i8.cuh"
#include "ozaki_gemm.cuh"

namespace tt {
namespace {

std::once_flag g_flags[kMaxDevices];
int g_ok[kMaxDevices];
int g_sms[kMaxDevices];

template <bool AK, bool BK>
int set_attr() {
  return cudaFuncSetAttribute(oz::gemm_kernel<AK, BK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              oz::kSmemBytes) == cudaSuccess
             ? TT_OK
             : TT_ERR_CUDA;
}

int setup(int dev) {
  return once_per_device(g_flags, g_ok, dev, [dev]() -> int {
    if (cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return TT_ERR_CUDA;
    int st = set_attr<false, false>();
    if (st == TT_OK) st = set_attr<false, true>();
    if (st == TT_OK) st = set_attr<true, false>();
    if (st == TT_OK) st = set_attr<true, true>();
    return st;
  });
}

inline size_t pad16(size_t x) { return (x + 15) / 16 * 16; }
inline size_t pad64(size_t x) { return (x + 63) / 64 * 64; }
inline size_t al256(size_t x) { return (x + 255) / 256 * 256; }

// Slice storage of one operand: (3, batch, mn, kpad) if K-major,
// (3, batch, K, mnpad) if MN-major; plus batch * mn(pad) fp32 scales.
struct Operand {
  bool kmajor;
  size_t inner, outer;  // elements per stored row, rows per batch
  size_t qbytes, sbytes;
  Operand(bool km, size_t mn, size_t K, size_t batch) : kmajor(km) {
    inner = km ? pad64(K) : pad16(mn);
    outer = km ? mn : K;
    qbytes = al256(3 * batch * outer * inner);
    sbytes = al256(4 * batch * (km ? mn : pad16(mn)));
  }
};

int split_operand(const float* X, const Operand& o, size_t mn, size_t K, int batch,
                  long long stride, int8_t* Q, float* S, cudaStream_t s, int sms) {
  if (o.kmajor) {
    // rows = batch * mn, each row K contiguous (row stride K, batch stride mn*K)
    if (stride != (long long)(mn * K)) return TT_ERR_SHAPE;
    long long rows = (long long)batch * mn;
    long long blocks = (rows + 7) / 8;
    const long long cap = (long long)sms * 16;
    if (blocks > cap) blocks = cap;
    if (rows == 0) return TT_OK;
    mp2::split_kernel<<<(unsigned)blocks, 256, 0, s>>>(X, Q, S, rows, (int)K, (int)o.inner,
                                                     rows * (long long)o.inner);
  } else {
    const long long nblk = (long long)batch * ((o.inner + oz::kSplitCols - 1) / oz::kSplitCols);
    const long long cap = (long long)sms * 8;
    const int grid = (int)(nblk < cap ? nblk : cap);
    oz::colmax_kernel<<<grid, oz::kSplitThreads, 0, s>>>(X, mn, stride, batch, (int)K, (int)mn,
                                                         (int)o.inner, S);
    oz::slice_kernel<<<grid, oz::kSplitThreads, 0, s>>>(X, mn, stride, batch, (int)K, (int)mn,
                                                        (int)o.inner, S, Q);
  }
  return cuda_status(cudaGetLastError());
}

int operand_map(CUtensorMap* m, const int8_t* Q, const Operand& o, int batch) {
  const uint64_t dims[4] = {(uint64_t)o.inner, (uint64_t)o.outer, (uint64_t)batch, 3};
  const uint64_t strides[3] = {(uint64_t)o.inner, (uint64_t)o.inner * o.outer,
                               (uint64_t)o.inner * o.outer * batch};
  const uint32_t box[4] = {o.kmajor ? (uint32_t)oz::kKC : (uint32_t)oz::kTile,
                           o.kmajor ? (uint32_t)oz::kTile : (uint32_t)oz::kKC, 1, 3};
  return encode_tmap(m, Q, 4, dims, strides, box,
                     o.kmajor ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_DATA_TYPE_UINT8);
}

}  // namespace
}  // namespace tt

extern "C" {

size_t tt_gemm_workspace_bytes(int M, int N, int K, int batch, int a_kmajor, int b_kmajor) {
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) return 0;
  const tt::Operand a(a_kmajor != 0, M, K, batch), b(b_kmajor != 0, N, K, batch);
  return a.qbytes + a.sbytes + b.qbytes + b.sbytes;
}

int tt_gemm_f32(const float* A, int a_kmajor, long long strideA, const float* B, int b_kmajor,
                long long strideB, float* C, long long strideC, int M, int N, int K, int batch,
                void* workspace, size_t workspace_bytes, int* dev_status, void* stream) {
  using namespace tt;
  if (!A || !B || !C || !workspace || !dev_status) return TT_ERR_NULL;
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) return TT_ERR_SHAPE;
  if (K > ozd::kMaxK) return TT_ERR_SHAPE;  // int32 slice sums exact up to this K
  const Operand oa(a_kmajor != 0, M, K, batch), ob(b_kmajor != 0, N, K, batch);
  if (workspace_bytes < oa.qbytes + oa.sbytes + ob.qbytes + ob.sbytes) return TT_ERR_WORKSPACE;
  if (!aligned16(workspace)) return TT_ERR_ALIGN;
  if (strideC < (long long)M * N) return TT_ERR_SHAPE;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = setup(dev);
  if (st != TT_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  TT_CUDA(cudaMemsetAsync(dev_status, 0, sizeof(int), s));
  char* w = static_cast<char*>(workspace);
  int8_t* qa = (int8_t*)w;
  float* sa = (float*)(w + oa.qbytes);
  int8_t* qb = (int8_t*)(w + oa.qbytes + oa.sbytes);
  float* sb = (float*)(w + oa.qbytes + oa.sbytes + ob.qbytes);
  if ((st = split_operand(A, oa, M, K, batch, strideA, qa, sa, s, g_sms[dev]))) return st;
  if ((st = split_operand(B, ob, N, K, batch, strideB, qb, sb, s, g_sms[dev]))) return st;
  CUtensorMap ma, mb;
  if (operand_map(&ma, qa, oa, batch) || operand_map(&mb, qb, ob, batch)) return TT_ERR_TMA;
  oz::Params p;
  p.sA = sa;
  p.sB = sb;
  p.ldsA = oa.kmajor ? M : pad16(M);
  p.ldsB = ob.kmajor ? N : pad16(N);
  p.C = C;
  p.ldc = N;
  p.strideC = strideC;
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = batch;
  p.shared_A = 0;
  p.tiles_m = (M + oz::kTile - 1) / oz::kTile;
  p.tiles_n = (N + oz::kTile - 1) / oz::kTile;
  p.err = dev_status;
  const long long tiles = (long long)p.tiles_m * p.tiles_n * batch;
  const int grid = (int)(tiles < g_sms[dev] ? tiles : g_sms[dev]);
  const dim3 blk(oz::kThreads);
  if (oa.kmajor && ob.kmajor)
    oz::gemm_kernel<true, true><<<grid, blk, oz::kSmemBytes, s>>>(ma, mb, p);
  else if (oa.kmajor)
    oz::gemm_kernel<true, false><<<grid, blk, oz::kSmemBytes, s>>>(ma, mb, p);
  else if (ob.kmajor)
    oz::gemm_kernel<false, true><<<grid, blk, oz::kSmemBytes, s>>>(ma, mb, p);
  else
    oz::gemm_kernel<false, false><<<grid, blk, oz::kSmemBytes, s>>>(ma, mb, p);
  return cuda_status(cudaGetLastError());
}

}  // extern "C"
