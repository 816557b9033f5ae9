// Ozaki slice format shared by every int8 tensor-core path (MP2 rows,
// AO->MO columns, the einsum GEMM):
//
//   x = s (q1 + q2 / 2^8 + q3 / 2^16) + r,   |r| <= s / 2^17,
//
// s = 2^(e-6) one power of two per row (or column) with max|x| < 2^e, so
// |x / s| < 64; q1 in [-64, 64], q2 and q3 in [-128, 127]. The digits are the
// balanced base-256 digits of Y = rint(x 2^16 / s): every digit is rounded to
// nearest, so the error of the terms a product drops (q2 q3 and below, 2^-24
// of s_x s_y) has zero mean. A product of two split values is
//
//   x y = s_x s_y (L2 + L3 / 2^8 + L4 / 2^16) + O(2^-23 s_x s_y),
//   L2 = q1 q1',  L3 = q1 q2' + q2 q1',  L4 = q1 q3' + q2 q2' + q3 q1',
//
// and a K-long dot product of such terms is exact in int32 while
// K (64*128 + 128*128 + 128*64) < 2^31, i.e. K <= 65535.
//
// Digit extraction without integer division: Y + 1.5 * 2^23 held as a float
// keeps Y in its low mantissa bits while |Y| <= 2^22, so one fused
// multiply-add rounds x 2^16 / s to Y, and with a bias of 128 + 128 * 256
// the three bytes of Z = Y + bias are q3 + 128, q2 + 128 and q1.
#pragma once
#include <cstdint>

namespace tt {
namespace ozd {

constexpr int kMaxK = 65535;

__device__ __forceinline__ float pow2f(int k) { return __int_as_float((k + 127) << 23); }

// |x| folded into a running maximum; NaN counts as +inf so that a non-finite
// input poisons its row or column scale instead of vanishing from the max.
__device__ __forceinline__ float absmax(float m, float v) {
  return fmaxf(m, v == v ? fabsf(v) : __int_as_float(0x7f800000));
}

// Power-of-two scale for a row/column whose largest magnitude is mx:
// 0 for (near-)zero data, NaN for non-finite data (the NaN then reaches every
// output that uses this row or column).
__device__ __forceinline__ float scale_for_max(float mx) {
  if (!(mx <= 3.4028234e38f)) return __int_as_float(0x7fc00000);
  if (!(mx > 1.0e-30f)) return 0.f;
  return pow2f(ilogbf(mx) + 1 - 6);  // mx < 2^(ilogb + 1)
}

// 2^16 / s (exact: s is a power of two); 0 and NaN pass through.
__device__ __forceinline__ float inv_scale(float s) { return s > 0.f ? 65536.0f / s : s; }

constexpr int kBias = 128 + 128 * 256;
constexpr int kMagicBits = 0x4B400000;  // bit pattern of 1.5 * 2^23

// Z = rint(x * inv) + kBias, for |x * inv| <= 2^22.
__device__ __forceinline__ int digit_word(float x, float inv) {
  return __float_as_int(__fmaf_rn(x, inv, 12582912.0f)) - (kMagicBits - kBias);
}

// Four digit words -> the three slices as packed int8 (byte j = value j).
__device__ __forceinline__ void pack_digits(const int (&z)[4], uint32_t& w1, uint32_t& w2,
                                            uint32_t& w3) {
  const uint32_t h1 = __byte_perm(z[0], z[1], 0x0062), l1 = __byte_perm(z[2], z[3], 0x0062);
  const uint32_t h2 = __byte_perm(z[0], z[1], 0x0051), l2 = __byte_perm(z[2], z[3], 0x0051);
  const uint32_t h3 = __byte_perm(z[0], z[1], 0x0040), l3 = __byte_perm(z[2], z[3], 0x0040);
  w1 = __byte_perm(h1, l1, 0x5410);
  w2 = __byte_perm(h2, l2, 0x5410) ^ 0x80808080u;
  w3 = __byte_perm(h3, l3, 0x5410) ^ 0x80808080u;
}

__device__ __forceinline__ void split4(const float (&v)[4], const float (&inv)[4], uint32_t& w1,
                                       uint32_t& w2, uint32_t& w3) {
  const int z[4] = {digit_word(v[0], inv[0]), digit_word(v[1], inv[1]),
                    digit_word(v[2], inv[2]), digit_word(v[3], inv[3])};
  pack_digits(z, w1, w2, w3);
}

__device__ __forceinline__ float level_combine(int l2, int l3, int l4) {
  return (float)l2 + (float)l3 * (1.0f / 256.0f) + (float)l4 * (1.0f / 65536.0f);
}

}  // namespace ozd
}  // namespace tt
