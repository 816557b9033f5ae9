// C-ABI entry points for the DF-MP2 energy: int8 Ozaki tensor-core kernel
// (the fp32 path), the 3xTF32 tensor-core kernel (kept as a diagnostic),
// fp64 and fp32 CUDA-core kernels, and the operand splits they consume.
#include "common.cuh"

#include <cstdlib>
#include "mp2_i8.cuh"
#include "mp2_i8_2sm.cuh"
#include "mp2_i8x5.cuh"
#include "mp2_simt.cuh"
#include "mp2_tf32.cuh"

namespace tt {

__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi = tf32(x), lo = tf32(x - hi); rows x cols -> rows x cols_pad, zero pad.
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                  float* __restrict__ lo, long long rows, int cols,
                                  int cols_pad) {
  const long long nvec = rows * (long long)(cols_pad / 4);
  for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < nvec;
       v += (long long)gridDim.x * blockDim.x) {
    const long long r = v / (cols_pad / 4);
    const int c = (int)(v % (cols_pad / 4)) * 4;
    float in[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) in[k] = (c + k < cols) ? __ldg(x + r * cols + c + k) : 0.f;
    float4 h, l;
    h.x = to_tf32(in[0]); l.x = to_tf32(in[0] - h.x);
    h.y = to_tf32(in[1]); l.y = to_tf32(in[1] - h.y);
    h.z = to_tf32(in[2]); l.z = to_tf32(in[2] - h.z);
    h.w = to_tf32(in[3]); l.w = to_tf32(in[3] - h.w);
    reinterpret_cast<float4*>(hi + r * cols_pad)[c / 4] = h;
    reinterpret_cast<float4*>(lo + r * cols_pad)[c / 4] = l;
  }
}

namespace {
std::once_flag g_mp2_attr_flags[kMaxDevices];
int g_mp2_attr_ok[kMaxDevices];
int g_num_sms[kMaxDevices];

int mp2_setup(int dev) {
  return once_per_device(g_mp2_attr_flags, g_mp2_attr_ok, dev, [dev]() -> int {
    if (cudaFuncSetAttribute(mp2::energy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             mp2::kSmemBytes) != cudaSuccess)
      return TT_ERR_CUDA;
    if (cudaFuncSetAttribute(mp2d::energy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             mp2d::kSmemBytes) != cudaSuccess)
      return TT_ERR_CUDA;
    if (cudaFuncSetAttribute(mp2x2::energy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             mp2x2::kSmemBytes) != cudaSuccess)
      return TT_ERR_CUDA;
    if (cudaFuncSetAttribute(mp2tf::energy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             mp2tf::kSmemBytes) != cudaSuccess)
      return TT_ERR_CUDA;
    if (cudaFuncSetAttribute(mp2s::energy_kernel<double>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             mp2s::smem_bytes<double>()) != cudaSuccess ||
        cudaFuncSetAttribute(mp2s::energy_kernel<float>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             mp2s::smem_bytes<float>()) != cudaSuccess)
      return TT_ERR_CUDA;
    if (cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev) !=
        cudaSuccess)
      return TT_ERR_CUDA;
    return TT_OK;
  });
}

// TRNTENSOR_B200_MP2_2SM=1 selects the paired-SM (cta_group::2) kernel;
// the one-SM kernel is the default (faster on B200, see mp2_i8_2sm.cuh).
// Read on every call so that callers and tests can switch between them.
bool use_paired_kernel() {
  const char* e = std::getenv("TRNTENSOR_B200_MP2_2SM");
  return e != nullptr && e[0] == '1';
}

inline int naux_padded(int naux) { return (naux + 15) / 16 * 16; }     // tf32 split
inline int naux_padded_i8(int naux) { return (naux + 63) / 64 * 64; }  // int8 slices
inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

int check_pairs(int nocc, long long pb, long long pe) {
  const long long np = (long long)nocc * (nocc + 1) / 2;
  if (pb < 0 || pe < pb || pe > np) return TT_ERR_SHAPE;
  return TT_OK;
}
}  // namespace

int launch_split(const float* x, float* hi, float* lo, long long rows, int cols, int cols_pad,
                 cudaStream_t s, int num_sms) {
  const long long nvec = rows * (long long)(cols_pad / 4);
  if (nvec == 0) return TT_OK;
  long long blocks = (nvec + 255) / 256;
  const long long cap = (long long)num_sms * 16;
  if (blocks > cap) blocks = cap;
  split_tf32_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, hi, lo, rows, cols, cols_pad);
  return cuda_status(cudaGetLastError());
}

}  // namespace tt

using namespace tt;

// Number of diagonal pairs (i, i) whose id is below pair id p: the rows i
// with pair_offset(i) < p (row-major enumeration of i <= j).
static long long diag_pairs_before(long long p, int n) {
  long long lo = 0, hi = n;  // smallest i in [0, n] with pair_offset(i) >= p
  while (lo < hi) {
    const long long mid = (lo + hi) / 2;
    if (mp2::pair_offset(mid, n) >= p) hi = mid; else lo = mid + 1;
  }
  return lo;
}

// Issues the pair range [pair_begin, pair_end) as consecutive launches of
// per_launch pairs. With split_modes each chunk is one launch of its
// two-phase items (mode 1) and one of its one-phase items (mode 2), so that
// every item of a launch has the same length; else one launch of all of
// them (mode 0). launch(n_items) runs the kernel on p as set here.
template <class Launch>
static int launch_chunks(mp2::Params& p, long long pair_begin, long long pair_end,
                         long long per_launch, long long ipp, bool split_modes, Launch&& launch) {
  const long long nodp = (long long)p.nblk * (p.nblk - 1) / 2;
  int st = TT_OK;
  for (long long lo = pair_begin; lo < pair_end; lo += per_launch) {
    const long long hi = lo + per_launch < pair_end ? lo + per_launch : pair_end;
    p.pair_begin = lo;
    p.pair_end = hi;
    if (!split_modes) {
      p.mode = 0;
      if ((st = launch((hi - lo) * ipp)) != TT_OK) return st;
      continue;
    }
    // diagonal pairs (i, i) below a pair id = rows whose first pair precedes it
    const long long d_lo = diag_pairs_before(lo, p.nocc), d_hi = diag_pairs_before(hi, p.nocc);
    p.mode = 1;
    p.q_begin = lo - d_lo;
    if ((st = launch(((hi - d_hi) - (lo - d_lo)) * nodp)) != TT_OK) return st;
    p.mode = 2;
    p.diag_lo = (int)d_lo;
    if ((st = launch((hi - lo) * p.nblk + (d_hi - d_lo) * nodp)) != TT_OK) return st;
  }
  return TT_OK;
}

// Per-CTA wait-cycle counters exist only in TT_MP2_PROFILE builds (a
// measurement build, never the shipped library): there the buffer is set
// once by tt_debug_set_profile_buffer before any launch.
#ifdef TT_MP2_PROFILE
static long long* g_mp2_prof = nullptr;
extern "C" void tt_debug_set_profile_buffer(long long* buf) { g_mp2_prof = buf; }
#endif

extern "C" {

long long tt_mp2_num_pairs(int nocc) {
  return nocc > 0 ? (long long)nocc * (nocc + 1) / 2 : 0;
}

size_t tt_mp2_workspace_bytes(int nocc, int nvir, int naux) {
  if (nocc <= 0 || nvir <= 0 || naux <= 0) return 0;
  const size_t rows = (size_t)nocc * (size_t)nvir;
  return align256(3ull * rows * (size_t)naux_padded_i8(naux)) + align256(rows * sizeof(float));
}

size_t tt_mp2_tf32_workspace_bytes(int nocc, int nvir, int naux) {
  if (nocc <= 0 || nvir <= 0 || naux <= 0) return 0;
  return 2ull * (size_t)nocc * (size_t)nvir * (size_t)naux_padded(naux) * sizeof(float);
}

int tt_split_i8_rows(const float* x, signed char* q, float* scale, long long row_begin,
                     long long row_count, long long total_rows, int cols, int cols_pad,
                     void* stream) {
  if (!x || !q || !scale) return TT_ERR_NULL;
  if (row_begin < 0 || row_count < 0 || row_begin + row_count > total_rows || cols <= 0 ||
      cols_pad < cols || cols_pad % 64 != 0)
    return TT_ERR_SHAPE;
  if (!aligned16(q)) return TT_ERR_ALIGN;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = mp2_setup(dev);
  if (st != TT_OK) return st;
  if (row_count == 0) return TT_OK;
  long long blocks = (row_count + 7) / 8;
  const long long cap = (long long)g_num_sms[dev] * 16;
  if (blocks > cap) blocks = cap;
  mp2::split_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      x + row_begin * cols, reinterpret_cast<int8_t*>(q) + row_begin * cols_pad,
      scale + row_begin, row_count, cols, cols_pad, total_rows * (long long)cols_pad);
  return cuda_status(cudaGetLastError());
}

int tt_mp2_range_stats_f32(const float* x, long long rows, int cols, double* stats,
                           void* stream) {
  if (!x || !stats) return TT_ERR_NULL;
  if (rows < 0 || cols <= 0) return TT_ERR_SHAPE;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = mp2_setup(dev);
  if (st != TT_OK) return st;
  if (rows == 0) return TT_OK;
  long long blocks = (rows + 7) / 8;
  const long long cap = (long long)g_num_sms[dev] * 16;
  if (blocks > cap) blocks = cap;
  mp2::range_stats_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(x, rows, cols,
                                                                             stats);
  return cuda_status(cudaGetLastError());
}

int tt_split_i8(const float* x, signed char* q, float* scale, long long rows, int cols,
                int cols_pad, void* stream) {
  return tt_split_i8_rows(x, q, scale, 0, rows, rows, cols, cols_pad, stream);
}

int tt_mp2_energy_presplit_i8(const signed char* Q, const float* scale, int naux_pad,
                              const float* eps_occ, const float* eps_vir, int nocc, int nvir,
                              long long pair_begin, long long pair_end, double* energy,
                              double* pair_partials, int* dev_status, void* stream) {
  if (!Q || !scale || !eps_occ || !eps_vir || !energy || !dev_status) return TT_ERR_NULL;
  if (nocc <= 0 || nvir <= 0 || naux_pad <= 0 || naux_pad % 64 != 0) return TT_ERR_SHAPE;
  if (nocc > 65535 || nvir > 65535 || naux_pad > ozd::kMaxK) return TT_ERR_SHAPE;
  if (check_pairs(nocc, pair_begin, pair_end) != TT_OK) return TT_ERR_SHAPE;
  if (!aligned16(Q)) return TT_ERR_ALIGN;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = mp2_setup(dev);
  if (st != TT_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  TT_CUDA(cudaMemsetAsync(energy, 0, sizeof(double), s));
  TT_CUDA(cudaMemsetAsync(dev_status, 0, sizeof(int), s));
  if (pair_partials)
    TT_CUDA(cudaMemsetAsync(pair_partials, 0, sizeof(double) * (size_t)nocc * nocc, s));
  if (pair_end == pair_begin) return TT_OK;
  // Slices as a 4-D byte tensor (aux, vir, occ, slice), innermost first;
  // one box = 64 aux x 128 rows (64 for the paired kernel's B half) x all 3
  // slices, 64B swizzle.
  CUtensorMap mq, mq_half;
  const uint64_t rows = (uint64_t)nocc * nvir;
  const uint64_t dims[4] = {(uint64_t)naux_pad, (uint64_t)nvir, (uint64_t)nocc, 3};
  const uint64_t strides[3] = {(uint64_t)naux_pad, (uint64_t)naux_pad * nvir,
                               (uint64_t)naux_pad * rows};
  const uint32_t box[4] = {(uint32_t)mp2::kKC, (uint32_t)mp2::kBlk, 1, 3};
  const uint32_t box_half[4] = {(uint32_t)mp2::kKC, (uint32_t)mp2::kBlk / 2, 1, 3};
  if (encode_tmap(&mq, Q, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_DATA_TYPE_UINT8) ||
      encode_tmap(&mq_half, Q, 4, dims, strides, box_half, CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_DATA_TYPE_UINT8))
    return TT_ERR_TMA;
  mp2::Params p{};
  p.scale = scale;
  p.eps_occ = eps_occ;
  p.eps_vir = eps_vir;
  p.nocc = nocc;
  p.nvir = nvir;
  p.naux_pad = naux_pad;
  p.pair_begin = pair_begin;
  p.pair_end = pair_end;
  p.nblk = (nvir + mp2::kBlk - 1) / mp2::kBlk;
  p.energy = energy;
  p.pair_partials = pair_partials;
  p.err = dev_status;
#ifdef TT_MP2_PROFILE
  p.prof = g_mp2_prof;
#else
  p.prof = nullptr;
#endif
  // The pair range is issued as consecutive launches of about kWavesPerLaunch
  // waves each, accumulating into the same energy. A single persistent launch
  // lets CTAs drift apart over thousands of items (one- and two-phase items
  // differ in length); concurrently running items then stop sharing B rows
  // in L2 and the extra HBM traffic costs power and clock. Re-aligning every
  // ~48 waves measured +27-32 % at config 4 (same energy to the last digit).
  // Each chunk is further issued as one launch of its two-phase items and one
  // of its one-phase items (p.mode), so that within a launch every item has
  // the same length.
  constexpr long long kWavesPerLaunch = 48;
  const bool paired = use_paired_kernel();
  const long long ipp = paired ? mp2x2::items_per_pair(p.nblk) : (long long)(p.nblk * (p.nblk + 1) / 2);
  const long long slots = paired ? g_num_sms[dev] / 2 : g_num_sms[dev];
  long long per_launch = slots * kWavesPerLaunch / ipp;
  if (per_launch < 1) per_launch = 1;
  const char* sp = std::getenv("TRNTENSOR_B200_MP2_SPLIT_MODES");
  const bool split_modes = !paired && !(sp != nullptr && sp[0] == '0');
  auto launch = [&](long long n_items) -> int {
    if (n_items <= 0) return TT_OK;
    p.n_items = n_items;
    const int grid = (int)(n_items < slots ? n_items : slots);
    if (paired)
      mp2x2::energy_kernel<<<2 * grid, mp2x2::kThreads, mp2x2::kSmemBytes, s>>>(mq, mq_half, p);
    else
      mp2::energy_kernel<<<grid, mp2::kThreads, mp2::kSmemBytes, s>>>(mq, p);
    return cuda_status(cudaGetLastError());
  };
  return launch_chunks(p, pair_begin, pair_end, per_launch, ipp, split_modes, launch);
}

int tt_split_tf32(const float* x, float* hi, float* lo, long long rows, int cols, int cols_pad,
                  void* stream) {
  if (!x || !hi || !lo) return TT_ERR_NULL;
  if (rows < 0 || cols <= 0 || cols_pad < cols || cols_pad % 4 != 0) return TT_ERR_SHAPE;
  if (!aligned16(hi) || !aligned16(lo)) return TT_ERR_ALIGN;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = mp2_setup(dev);
  if (st != TT_OK) return st;
  return launch_split(x, hi, lo, rows, cols, cols_pad, (cudaStream_t)stream, g_num_sms[dev]);
}

int tt_mp2_energy_tf32x3(const float* B_hi, const float* B_lo, int naux_pad,
                               const float* eps_occ, const float* eps_vir, int nocc, int nvir,
                               long long pair_begin, long long pair_end, double* energy,
                               double* pair_partials, int* dev_status, void* stream) {
  if (!B_hi || !B_lo || !eps_occ || !eps_vir || !energy || !dev_status) return TT_ERR_NULL;
  if (nocc <= 0 || nvir <= 0 || naux_pad <= 0 || naux_pad % 16 != 0) return TT_ERR_SHAPE;
  if (nocc > 65535 || nvir > 65535) return TT_ERR_SHAPE;
  if (check_pairs(nocc, pair_begin, pair_end) != TT_OK) return TT_ERR_SHAPE;
  if (!aligned16(B_hi) || !aligned16(B_lo)) return TT_ERR_ALIGN;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = mp2_setup(dev);
  if (st != TT_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  TT_CUDA(cudaMemsetAsync(energy, 0, sizeof(double), s));
  TT_CUDA(cudaMemsetAsync(dev_status, 0, sizeof(int), s));
  if (pair_partials)
    TT_CUDA(cudaMemsetAsync(pair_partials, 0, sizeof(double) * (size_t)nocc * nocc, s));
  if (pair_end == pair_begin) return TT_OK;

  // Tensor maps over (naux_pad, nvir, nocc), innermost first; 64-byte rows
  // with 64B swizzle, boxes of 128 (A operand) and 256 (B operand) rows.
  CUtensorMap mA_hi, mA_lo, mB_hi, mB_lo;
  const uint64_t dims[3] = {(uint64_t)naux_pad, (uint64_t)nvir, (uint64_t)nocc};
  const uint64_t strides[2] = {(uint64_t)naux_pad * 4, (uint64_t)naux_pad * 4 * nvir};
  const uint32_t boxA[3] = {(uint32_t)mp2tf::kKC, (uint32_t)mp2tf::kM, 1};
  const uint32_t boxB[3] = {(uint32_t)mp2tf::kKC, (uint32_t)mp2tf::kN, 1};
  if (encode_tmap(&mA_hi, B_hi, 3, dims, strides, boxA, CU_TENSOR_MAP_SWIZZLE_64B) ||
      encode_tmap(&mA_lo, B_lo, 3, dims, strides, boxA, CU_TENSOR_MAP_SWIZZLE_64B) ||
      encode_tmap(&mB_hi, B_hi, 3, dims, strides, boxB, CU_TENSOR_MAP_SWIZZLE_64B) ||
      encode_tmap(&mB_lo, B_lo, 3, dims, strides, boxB, CU_TENSOR_MAP_SWIZZLE_64B))
    return TT_ERR_TMA;

  mp2tf::Params p;
  p.eps_occ = eps_occ;
  p.eps_vir = eps_vir;
  p.nocc = nocc;
  p.nvir = nvir;
  p.naux_pad = naux_pad;
  p.pair_begin = pair_begin;
  p.pair_end = pair_end;
  p.n_rects = mp2tf::rect_count(nvir);
  p.energy = energy;
  p.pair_partials = pair_partials;
  p.err = dev_status;
  const long long n_items = (pair_end - pair_begin) * (long long)p.n_rects;
  const int grid = (int)(n_items < g_num_sms[dev] ? n_items : g_num_sms[dev]);
  mp2tf::energy_kernel<<<grid, mp2tf::kThreads, mp2tf::kSmemBytes, s>>>(mA_hi, mA_lo, mB_hi, mB_lo, p);
  return cuda_status(cudaGetLastError());
}

int tt_mp2_energy_f32(const float* B, const float* eps_occ, const float* eps_vir, int nocc,
                      int nvir, int naux, long long pair_begin, long long pair_end,
                      void* workspace, size_t workspace_bytes, double* energy,
                      double* pair_partials, int* dev_status, void* stream) {
  if (!B || !workspace || !eps_occ || !eps_vir || !energy || !dev_status) return TT_ERR_NULL;
  if (nocc <= 0 || nvir <= 0 || naux <= 0) return TT_ERR_SHAPE;
  if (nocc > 65535 || nvir > 65535) return TT_ERR_SHAPE;
  if (check_pairs(nocc, pair_begin, pair_end) != TT_OK) return TT_ERR_SHAPE;
  const size_t need = tt_mp2_workspace_bytes(nocc, nvir, naux);
  if (workspace_bytes < need) return TT_ERR_WORKSPACE;
  if (!aligned16(workspace)) return TT_ERR_ALIGN;
  const int naux_pad = naux_padded_i8(naux);
  const size_t rows = (size_t)nocc * nvir;
  signed char* q = static_cast<signed char*>(workspace);
  float* scale = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                          align256(3ull * rows * (size_t)naux_pad));
  int st = tt_split_i8(B, q, scale, (long long)rows, naux, naux_pad, stream);
  if (st != TT_OK) return st;
  return tt_mp2_energy_presplit_i8(q, scale, naux_pad, eps_occ, eps_vir, nocc, nvir, pair_begin,
                                   pair_end, energy, pair_partials, dev_status, stream);
}

size_t tt_mp2_f64_workspace_bytes(int nocc, int nvir, int naux) {
  if (nocc <= 0 || nvir <= 0 || naux <= 0) return 0;
  const size_t rows = (size_t)nocc * (size_t)nvir;
  return align256((size_t)mp2d::kDigits * rows * (size_t)naux_padded_i8(naux)) +
         align256(rows * sizeof(double)) +
         (size_t)mp2d::kMaxGrid * (size_t)mp2d::kScratchDoubles * sizeof(double);
}

int tt_mp2_energy_f64_tc(const double* B, const double* eps_occ, const double* eps_vir, int nocc,
                         int nvir, int naux, long long pair_begin, long long pair_end,
                         void* workspace, size_t workspace_bytes, double* energy,
                         double* pair_partials, int* dev_status, void* stream) {
  if (!B || !workspace || !eps_occ || !eps_vir || !energy || !dev_status) return TT_ERR_NULL;
  if (nocc <= 0 || nvir <= 0 || naux <= 0) return TT_ERR_SHAPE;
  if (nocc > 65535 || nvir > 65535 || naux_padded_i8(naux) > mp2d::kMaxK) return TT_ERR_SHAPE;
  if (check_pairs(nocc, pair_begin, pair_end) != TT_OK) return TT_ERR_SHAPE;
  if (workspace_bytes < tt_mp2_f64_workspace_bytes(nocc, nvir, naux)) return TT_ERR_WORKSPACE;
  if (!aligned16(workspace)) return TT_ERR_ALIGN;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = mp2_setup(dev);
  if (st != TT_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  const int naux_pad = naux_padded_i8(naux);
  const size_t rows = (size_t)nocc * nvir;
  const size_t plane = rows * (size_t)naux_pad;
  int8_t* q = static_cast<int8_t*>(workspace);
  double* scale = reinterpret_cast<double*>(static_cast<char*>(workspace) +
                                            align256((size_t)mp2d::kDigits * plane));
  double* scratch = reinterpret_cast<double*>(reinterpret_cast<char*>(scale) +
                                              align256(rows * sizeof(double)));
  TT_CUDA(cudaMemsetAsync(energy, 0, sizeof(double), s));
  TT_CUDA(cudaMemsetAsync(dev_status, 0, sizeof(int), s));
  if (pair_partials)
    TT_CUDA(cudaMemsetAsync(pair_partials, 0, sizeof(double) * (size_t)nocc * nocc, s));
  if (pair_end == pair_begin) return TT_OK;
  {
    long long blocks = ((long long)rows + 7) / 8;
    const long long cap = (long long)g_num_sms[dev] * 16;
    if (blocks > cap) blocks = cap;
    mp2d::split_kernel<<<(unsigned)blocks, 256, 0, s>>>(B, q, scale, (long long)rows, naux,
                                                        naux_pad, (long long)plane);
    if ((st = cuda_status(cudaGetLastError())) != TT_OK) return st;
  }
  // Digit planes as a 4-D byte tensor (aux, vir, occ, digit), innermost
  // first; a box is 32 aux x 128 rows x the first 3 (sweep 0) or all 5
  // (sweep 1) digits, 32B swizzle.
  CUtensorMap m3, m5;
  const uint64_t dims[4] = {(uint64_t)naux_pad, (uint64_t)nvir, (uint64_t)nocc,
                            (uint64_t)mp2d::kDigits};
  const uint64_t strides[3] = {(uint64_t)naux_pad, (uint64_t)naux_pad * nvir, (uint64_t)plane};
  const uint32_t box3[4] = {(uint32_t)mp2d::kKC, (uint32_t)mp2d::kBlk, 1, 3};
  const uint32_t box5[4] = {(uint32_t)mp2d::kKC, (uint32_t)mp2d::kBlk, 1, 5};
  if (encode_tmap(&m3, q, 4, dims, strides, box3, CU_TENSOR_MAP_SWIZZLE_32B,
                  CU_TENSOR_MAP_DATA_TYPE_UINT8) ||
      encode_tmap(&m5, q, 4, dims, strides, box5, CU_TENSOR_MAP_SWIZZLE_32B,
                  CU_TENSOR_MAP_DATA_TYPE_UINT8))
    return TT_ERR_TMA;
  mp2d::Params P{};
  mp2::Params& p = P.base;
  p.nocc = nocc;
  p.nvir = nvir;
  p.naux_pad = naux_pad;
  p.nblk = (nvir + mp2d::kBlk - 1) / mp2d::kBlk;
  p.energy = energy;
  p.pair_partials = pair_partials;
  p.err = dev_status;
  P.scale = scale;
  P.eps_occ = eps_occ;
  P.eps_vir = eps_vir;
  P.scratch = scratch;
  const long long ipp = (long long)p.nblk * (p.nblk + 1) / 2;
  const long long slots =
      g_num_sms[dev] < mp2d::kMaxGrid ? (long long)g_num_sms[dev] : (long long)mp2d::kMaxGrid;
  // chunks of ~16 waves: an fp64 item issues ~3x the MMAs of an fp32 one,
  // whose launches are ~48 waves long
  long long per_launch = slots * 16 / ipp;
  if (per_launch < 1) per_launch = 1;
  auto launch = [&](long long n_items) -> int {
    if (n_items <= 0) return TT_OK;
    p.n_items = n_items;
    const int grid = (int)(n_items < slots ? n_items : slots);
    mp2d::energy_kernel<<<grid, mp2d::kThreads, mp2d::kSmemBytes, s>>>(m3, m5, P);
    return cuda_status(cudaGetLastError());
  };
  return launch_chunks(p, pair_begin, pair_end, per_launch, ipp, true, launch);
}

}  // extern "C"

namespace {
template <typename T>
int launch_simt(const T* B, const T* eps_occ, const T* eps_vir, int nocc, int nvir, int naux,
                long long pair_begin, long long pair_end, double* energy, double* pair_partials,
                void* stream) {
  if (!B || !eps_occ || !eps_vir || !energy) return TT_ERR_NULL;
  if (nocc <= 0 || nvir <= 0 || naux <= 0) return TT_ERR_SHAPE;
  if (check_pairs(nocc, pair_begin, pair_end) != TT_OK) return TT_ERR_SHAPE;
  int dev = 0;
  int st = check_device(&dev);
  if (st != TT_OK) return st;
  st = mp2_setup(dev);
  if (st != TT_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  TT_CUDA(cudaMemsetAsync(energy, 0, sizeof(double), s));
  if (pair_partials)
    TT_CUDA(cudaMemsetAsync(pair_partials, 0, sizeof(double) * (size_t)nocc * nocc, s));
  if (pair_end == pair_begin) return TT_OK;
  mp2s::Params<T> p;
  p.B = B;
  p.eps_occ = eps_occ;
  p.eps_vir = eps_vir;
  p.nocc = nocc;
  p.nvir = nvir;
  p.naux = naux;
  p.pair_begin = pair_begin;
  p.pair_end = pair_end;
  p.nblk = (nvir + mp2s::kT - 1) / mp2s::kT;
  p.energy = energy;
  p.pair_partials = pair_partials;
  const long long n_items = (pair_end - pair_begin) * (long long)(p.nblk * (p.nblk + 1) / 2);
  const long long cap = (long long)g_num_sms[dev];
  const int grid = (int)(n_items < cap ? n_items : cap);
  mp2s::energy_kernel<T><<<grid, mp2s::kThreads, mp2s::smem_bytes<T>(), s>>>(p);
  return cuda_status(cudaGetLastError());
}
}  // namespace

extern "C" {
int tt_mp2_energy_f64(const double* B, const double* eps_occ, const double* eps_vir, int nocc,
                      int nvir, int naux, long long pair_begin, long long pair_end,
                      double* energy, double* pair_partials, void* stream) {
  return launch_simt<double>(B, eps_occ, eps_vir, nocc, nvir, naux, pair_begin, pair_end, energy,
                             pair_partials, stream);
}
int tt_mp2_energy_simt_f32(const float* B, const float* eps_occ, const float* eps_vir, int nocc,
                           int nvir, int naux, long long pair_begin, long long pair_end,
                           double* energy, double* pair_partials, void* stream) {
  return launch_simt<float>(B, eps_occ, eps_vir, nocc, nvir, naux, pair_begin, pair_end, energy,
                            pair_partials, stream);
}
}  // extern "C"
