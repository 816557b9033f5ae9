/*
 * trntensor_b200 C ABI.
 *
 * Drop-in device boundary for the trntensor DF-MP2 / AO->MO hot path on
 * NVIDIA B200 (sm_100a). Every entry point:
 *   - takes plain device pointers, sizes and a CUDA stream (cudaStream_t
 *     passed as void*; NULL = legacy default stream);
 *   - enqueues work asynchronously on that stream and returns a status code
 *     (TT_OK == 0) describing argument checks and launch errors only;
 *   - allocates no memory: outputs and workspaces are owned by the caller,
 *     whose sizes the *_workspace_bytes queries give;
 *   - never falls back to another implementation.
 * Device-side waits are bounded; a wait that runs out writes a nonzero code
 * into the caller's int `dev_status` (device memory), which the caller reads
 * after synchronising.
 *
 * Layouts are those of the reference's torch tensors (row-major, contiguous):
 *   B       (nocc, nvir, naux)      eri (nbf, nbf, naux)
 *   C_occ   (nbf, nocc)             C_vir (nbf, nvir)
 */
#ifndef TRNTENSOR_B200_H_
#define TRNTENSOR_B200_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TT_OK 0
#define TT_ERR_NULL 1        /* a required pointer is NULL */
#define TT_ERR_SHAPE 2       /* a size is out of range */
#define TT_ERR_ALIGN 3       /* a pointer is not 16-byte aligned */
#define TT_ERR_WORKSPACE 4   /* workspace too small */
#define TT_ERR_DEVICE 5      /* current device is not sm_100 */
#define TT_ERR_CUDA 6        /* CUDA runtime / launch error */
#define TT_ERR_TMA 7         /* tensor-map encoding failed */

/* Human-readable text for a status code. */
const char* tt_status_string(int status);
/* Library ABI version (major * 10000 + minor * 100 + patch). */
int tt_version(void);
/* TT_OK when the current CUDA device can run this library (sm_100). */
int tt_device_check(void);
/* Text of the last CUDA error seen by this thread's calls ("" if none). */
const char* tt_last_cuda_error(void);

/* Number of unordered occupied pairs i <= j: nocc * (nocc + 1) / 2. */
long long tt_mp2_num_pairs(int nocc);

/* Workspace bytes tt_mp2_energy_f32 needs: three int8 slices of B (naux
 * padded to a multiple of 64) plus one fp32 scale per (i, a) row. */
size_t tt_mp2_workspace_bytes(int nocc, int nvir, int naux);

/*
 * DF-MP2 correlation energy for fp32 inputs on int8 tensor cores (Ozaki
 * scheme: each B row = power-of-two scale x three int8 slices; six exact
 * int32-accumulated slice GEMMs per block; energy reduced in the epilogue).
 *   *energy = sum over the unordered pairs [pair_begin, pair_end) (linear
 *             id of (i, j), i <= j, row-major; the full sum is
 *             [0, tt_mp2_num_pairs(nocc))) of w_ij * E_ij, w = 2 for i < j,
 *             1 for i == j, E_ij = sum_ab T_ab (2T_ab - T_ba) / D_ijab.
 *   pair_partials (nullable, nocc*nocc doubles): E_ij written at [i][j] and
 *             [j][i] for the visited pairs, zero elsewhere.
 * energy, pair_partials and dev_status are zeroed by the call.
 * Replaces trntensor/nki/dispatch.py:240-283 (_nki_mp2_energy) and the
 * device kernel trntensor/nki/_kernels.py:119-207 (mp2_energy_kernel).
 */
int tt_mp2_energy_f32(const float* B, const float* eps_occ, const float* eps_vir, int nocc,
                      int nvir, int naux, long long pair_begin, long long pair_end,
                      void* workspace, size_t workspace_bytes, double* energy,
                      double* pair_partials, int* dev_status, void* stream);

/* Ozaki split of x (rows x cols, row-major fp32): per row a power-of-two
 * scale[r] and three int8 slice planes q[t][r][0..cols_pad) (zero padded,
 * cols_pad % 64 == 0) with x = scale * (q1 + q2/2^8 + q3/2^16) + r, |r| <= scale/2^17,
 * scale = 2^(e-6) with max|x| < 2^e (NaN for a row holding inf or NaN). */
int tt_split_i8(const float* x, signed char* q, float* scale, long long rows, int cols,
                int cols_pad, void* stream);

/* Accuracy statistics of the three-digit format of tt_split_i8 over rows x
 * cols (row-major fp32), ADDED into stats[0..2] (device fp64; the caller
 * zeroes them, so that a matrix can be summed piecewise):
 *   stats[0] += sum_r n_r s_r^2 u2_r,  stats[1] += sum_r n_r s_r^2 u3_r,
 *   stats[2] += sum_r n_r,
 * n_r = sum of squares of row r, s_r its scale, u2_r / u3_r the sums of
 * squares of its second / third digits. With K = cols,
 *   est = 2 sqrt(2^-47 stats[0] stats[1] / K) / (stats[2]^2 / K)
 * estimates the relative energy error tt_mp2_energy_f32 makes by dropping
 * the q2 q3 digit products (an over-estimate by 10-100x on the cases
 * measured). Rows whose entries span many decades, or hold a few entries far
 * above the rest, raise it; Gaussian rows give ~2e-7 or less. The Python
 * layer computes the energy with the five-digit kernel when est > 1e-6.
 * No counterpart in the reference (its fp32 GEMM rounds per element). */
int tt_mp2_range_stats_f32(const float* x, long long rows, int cols, double* stats, void* stream);

/* tt_split_i8 for rows [row_begin, row_begin + row_count) of a total_rows x
 * cols matrix, written into the slice planes of the whole matrix (plane
 * stride total_rows * cols_pad). Lets a caller split B as its rows arrive
 * (e.g. while copying it from host memory in chunks). */
int tt_split_i8_rows(const float* x, signed char* q, float* scale, long long row_begin,
                     long long row_count, long long total_rows, int cols, int cols_pad,
                     void* stream);

/* tt_mp2_energy_f32 on operands already split by tt_split_i8 with rows =
 * nocc * nvir and cols_pad = naux_pad (lets callers reuse one split). */
int tt_mp2_energy_presplit_i8(const signed char* Q, const float* scale, int naux_pad,
                              const float* eps_occ, const float* eps_vir, int nocc, int nvir,
                              long long pair_begin, long long pair_end, double* energy,
                              double* pair_partials, int* dev_status, void* stream);

/* Split x (rows x cols, row-major) into hi = tf32(x), lo = tf32(x - hi),
 * written as rows x cols_pad with zero padding (cols_pad >= cols, % 4 == 0). */
int tt_split_tf32(const float* x, float* hi, float* lo, long long rows, int cols, int cols_pad,
                  void* stream);

/* Bytes of hi + lo for tt_mp2_energy_tf32x3 (naux padded to 16). */
size_t tt_mp2_tf32_workspace_bytes(int nocc, int nvir, int naux);

/* Diagnostic: the same energy with 3xTF32 tcgen05 MMAs on tt_split_tf32
 * operands (naux_pad % 16 == 0). The tensor core's fp32 accumulation rounds
 * toward zero, so this variant is biased by ~2.4e-8 relative per 8 aux
 * elements; it is kept to document that, not as a production path. */
int tt_mp2_energy_tf32x3(const float* B_hi, const float* B_lo, int naux_pad,
                         const float* eps_occ, const float* eps_vir, int nocc, int nvir,
                         long long pair_begin, long long pair_end, double* energy,
                         double* pair_partials, int* dev_status, void* stream);

/* Scratch size of tt_mp2_energy_f32_noalloc (64 MiB of device memory that
 * every GPU using the library keeps until the process exits). */
#define TT_MP2_NOALLOC_SCRATCH_BYTES (64u * 1024u * 1024u)

/*
 * tt_mp2_energy_f32 for callers that cannot allocate device memory (host
 * programs that own the whole HBM budget, pipelines that cannot afford
 * cudaMalloc's device-wide synchronisation, FFI callers with no allocator).
 * No counterpart in the reference. Computes the full energy (all pairs)
 * using a fixed scratch array inside the library instead of a workspace:
 * problems with tt_mp2_workspace_bytes(nocc, nvir, naux) >
 * TT_MP2_NOALLOC_SCRATCH_BYTES are rejected with TT_ERR_WORKSPACE, and, as
 * for tt_mp2_energy_f32, naux padded to 64 must not exceed 65535
 * (TT_ERR_SHAPE even when the slices would fit the scratch). Calls no
 * allocation routine. All calls share the one scratch array: calls that
 * overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller. The first call on a device looks up the
 * scratch's device address; make it before any stream capture.
 */
int tt_mp2_energy_f32_noalloc(const float* B, const float* eps_occ, const float* eps_vir,
                              int nocc, int nvir, int naux, double* energy,
                              double* pair_partials, int* dev_status, void* stream);

/* Workspace of tt_mp2_energy_f64_tc: five int8 digit planes
 * (5, nocc*nvir, naux padded to 64), fp64 row scales and the per-CTA fp64
 * scratch tiles of the energy kernel. */
size_t tt_mp2_f64_workspace_bytes(int nocc, int nvir, int naux);

/* DF-MP2 energy of fp64 inputs on int8 tensor cores (precision="kahan":
 * trntensor/einsum.py:108-111 applied to trntensor/quantum.py:87-100; replaces
 * the fp64 route through trntensor/nki/dispatch.py:240-283). Five-digit Ozaki
 * split of B's rows, 19 exact int8 GEMMs per pair block, energy terms in fp64;
 * |dE|/|E| ~ 1e-14. naux padded to 64 must be <= 32767 (TT_ERR_SHAPE
 * otherwise). Same pair-range, energy, partials and dev_status contract as
 * tt_mp2_energy_f32. */
int tt_mp2_energy_f64_tc(const double* B, const double* eps_occ, const double* eps_vir,
                         int nocc, int nvir, int naux, long long pair_begin, long long pair_end,
                         void* workspace, size_t workspace_bytes, double* energy,
                         double* pair_partials, int* dev_status, void* stream);

/* DF-MP2 energy in fp64 throughout on CUDA cores (precision="kahan"
 * semantics of trntensor/einsum.py:108-111 applied to
 * trntensor/quantum.py:87-100); the fp64 path for naux beyond the limit of
 * tt_mp2_energy_f64_tc and an independent check of it. */
int tt_mp2_energy_f64(const double* B, const double* eps_occ, const double* eps_vir, int nocc,
                      int nvir, int naux, long long pair_begin, long long pair_end,
                      double* energy, double* pair_partials, void* stream);

/* Same sum on CUDA cores in plain fp32 FMA; an independent on-device check
 * of tt_mp2_energy_f32, not a production path. */
int tt_mp2_energy_simt_f32(const float* B, const float* eps_occ, const float* eps_vir, int nocc,
                           int nvir, int naux, long long pair_begin, long long pair_end,
                           double* energy, double* pair_partials, void* stream);

/* ------------------------------------------------------------ AO -> MO */

/* Workspace bytes for tt_ao2mo_f32 (elem_bytes 4: int8 slices of every
 * operand, the fp32 intermediate and its slices) or tt_ao2mo_f64 /
 * tt_ao2mo_simt_f32 (elem_bytes 8 / 4 are enough: the (nocc, nbf, naux)
 * intermediate). */
size_t tt_ao2mo_workspace_bytes(int nbf, int nocc, int nvir, int naux, int elem_bytes);

/*
 * B[i,a,P] = sum_{m,n} C_occ[m,i] C_vir[n,a] eri[m,n,P] on int8 tensor cores
 * (Ozaki splitting with per-column scales along each contraction index; six
 * exact int32-accumulated slice GEMMs per step), in two steps with the
 * (i, n, P) intermediate in the caller's workspace:
 *   inter = einsum("mi,mnP->inP"), B = einsum("na,inP->iaP").
 * eri (nbf, nbf, naux), C_occ (nbf, nocc), C_vir (nbf, nvir), B_out
 * (nocc, nvir, naux), all contiguous row-major. For a P-sharded run pass the
 * rank's contiguous (nbf, nbf, naux_local) slab. dev_status (device int) is
 * zeroed and receives a nonzero code if a device wait ran out.
 * Replaces trntensor/nki/dispatch.py:286-336 (_nki_ao_to_mo_transform) and
 * trntensor/nki/_kernels.py:209-296 (ao_to_mo_transform_kernel); the math is
 * trntensor/quantum.py:188-194.
 */
int tt_ao2mo_f32(const float* eri, const float* C_occ, const float* C_vir, int nbf, int nocc,
                 int nvir, int naux, void* workspace, size_t workspace_bytes, float* B_out,
                 int* dev_status, void* stream);

/*
 * tt_ao2mo_f32 on a strided P-slab of a larger eri, without copying it: the
 * rank's aux columns [p0, p0 + naux_local) of an (nbf, nbf, naux_total)
 * tensor are passed as eri = base + p0 with ld_n = naux_total and
 * ld_m = nbf * naux_total (elements); step 1 reads the slab through a 3-D
 * tensor map. B_out is the compact (nocc, nvir, naux_local) block and the
 * workspace is tt_ao2mo_workspace_bytes(nbf, nocc, nvir, naux_local, 4).
 * Needs eri 16-byte aligned, ld_n and ld_m multiples of 4 (TT_ERR_ALIGN)
 * and nbf > 128 (TT_ERR_SHAPE; the caller copies the slab then).
 * The interface the multi-GPU aux split needs (each rank reads its P range
 * in place); replaces the pad-and-copy at trntensor/nki/dispatch.py:286-336.
 */
int tt_ao2mo_f32_slab(const float* eri, long long ld_m, long long ld_n, const float* C_occ,
                      const float* C_vir, int nbf, int nocc, int nvir, int naux_local,
                      void* workspace, size_t workspace_bytes, float* B_out, int* dev_status,
                      void* stream);

/* Diagnostic: the same transform in plain fp32 on CUDA cores. */
int tt_ao2mo_simt_f32(const float* eri, const float* C_occ, const float* C_vir, int nbf,
                      int nocc, int nvir, int naux, void* workspace, size_t workspace_bytes,
                      float* B_out, void* stream);

/* Workspace of tt_ao2mo_f64_tc: six int8 digit planes of C_occ, C_vir, eri
 * and the intermediate, fp64 column scales, and the fp64 intermediate. */
size_t tt_ao2mo_f64_workspace_bytes(int nbf, int nocc, int nvir, int naux);

/* AO->MO transform of fp64 inputs on int8 tensor cores (precision="kahan":
 * trntensor/einsum.py:108-111 applied to the two-step form of
 * trntensor/quantum.py:188-194; replaces the fp64 route through
 * trntensor/nki/dispatch.py:286-336): six-digit column-scaled Ozaki split,
 * 21 exact int8 GEMMs per tile, fp64 output; max|dB|/max|B| ~ 1e-14.
 * nbf <= 26214 (TT_ERR_SHAPE otherwise). dev_status as for tt_ao2mo_f32. */
int tt_ao2mo_f64_tc(const double* eri, const double* C_occ, const double* C_vir, int nbf,
                    int nocc, int nvir, int naux, void* workspace, size_t workspace_bytes,
                    double* B_out, int* dev_status, void* stream);

/* The same in fp64 on CUDA cores (precision="kahan" and float64 inputs):
 * the path for nbf beyond tt_ao2mo_f64_tc's limit, and its cross-check. */
int tt_ao2mo_f64(const double* eri, const double* C_occ, const double* C_vir, int nbf,
                 int nocc, int nvir, int naux, void* workspace, size_t workspace_bytes,
                 double* B_out, void* stream);

/* --------------------------------------------------------------- GEMM */

/* Workspace bytes for tt_gemm_f32 (int8 slices + scales of both operands). */
size_t tt_gemm_workspace_bytes(int M, int N, int K, int batch, int a_kmajor, int b_kmajor);

/*
 * C[b] = A[b] . B[b] for b < batch, fp32 in and out, on int8 tensor cores
 * (Ozaki splitting: per-row / per-column power-of-two scales along K, three
 * int8 slices, six exact int32-accumulated slice GEMMs; accuracy at the fp32
 * level, error ~1e-7 relative to the operands' magnitudes).
 * A is M x K: a_kmajor = 1 -> stored (M, K) row-major, 0 -> stored (K, M).
 * B is K x N: b_kmajor = 1 -> stored (N, K) row-major, 0 -> stored (K, N).
 * strideA/B/C: elements between batches (A/B stride must equal the operand
 * size; C stride >= M*N). C is (M, N) row-major per batch.
 * Serves einsum's matmul / bmm strategies (trntensor/einsum.py:129-148,
 * trntensor/nki/dispatch.py:187-237 nki_matmul and 339-387
 * nki_batched_matmul).
 */
int tt_gemm_f32(const float* A, int a_kmajor, long long strideA, const float* B, int b_kmajor,
                long long strideB, float* C, long long strideC, int M, int N, int K, int batch,
                void* workspace, size_t workspace_bytes, int* dev_status, void* stream);

/* ------------------------------------------------- double-double (dd) */

/* Workspace of tt_mp2_energy_dd (per-block partial sums on this device). */
size_t tt_mp2_dd_workspace_bytes(int nocc, int nvir, int naux);

/*
 * DF-MP2 energy in double-double arithmetic on CUDA cores
 * (precision="dd": trntensor/einsum.py:112-116 names it, the reference
 * raises NotImplementedError). fp64 inputs; every T_ab and T_ba is a Dot2
 * dot product (sum and product errors collected, ~2^-106 relative for
 * well-conditioned sums), energy terms in double-double add / multiply /
 * divide, sums over (a, b), pairs and blocks in double-double, in a fixed
 * order (deterministic). energy[0..1] = (hi, lo) of the sum over the
 * unordered pairs [pair_begin, pair_end) with the weights of
 * tt_mp2_energy_f32; pair_partials (nullable, nocc*nocc*2 doubles) receives
 * each visited E_ij as (hi, lo) at [i][j] and [j][i], zero elsewhere.
 * A correctness mode: about 20x the fp64 CUDA-core kernel's time.
 */
int tt_mp2_energy_dd(const double* B, const double* eps_occ, const double* eps_vir, int nocc,
                     int nvir, int naux, long long pair_begin, long long pair_end,
                     void* workspace, size_t workspace_bytes, double* energy,
                     double* pair_partials, void* stream);

/*
 * Batched C[b] = A[b] . B[b] in double-double on CUDA cores: A and B given
 * as hi parts plus optional (nullable) lo parts, so that double-double
 * intermediates chain; C returned as hi and (nullable) lo. Layouts as in
 * tt_gemm_f32 (a_kmajor / b_kmajor; C (M, N) row-major per batch, batch
 * strides in elements). Serves precision="dd" for einsum contractions
 * (trntensor/einsum.py:112-116) and the two AO->MO steps.
 */
int tt_gemm_dd(const double* A_hi, const double* A_lo, int a_kmajor, long long strideA,
               const double* B_hi, const double* B_lo, int b_kmajor, long long strideB,
               double* C_hi, double* C_lo, long long strideC, int M, int N, int K, int batch,
               void* stream);

/* Failure-detection check (no counterpart in the reference): one thread waits,
 * through the same bounded mbarrier wait every kernel here uses, on a phase
 * that nothing completes. After budget_cycles (at most the kernels' own
 * budget, about 2 s) the wait gives up, *dev_status becomes 0x101 (a stage
 * never arrived) and *dev_cycles the cycles waited; the context stays usable.
 * Lets a caller test its handling of a device timeout without a GPU fault. */
int tt_debug_wait_timeout(int* dev_status, long long budget_cycles, long long* dev_cycles,
                          void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TRNTENSOR_B200_H_ */
