// Exact arithmetic of the ConvRot-256 rotation (y = x @ H, H = H4^(x)4 / 16 the
// normalised regular Hadamard matrix, tensor/int8_utils.py:11-74), shared by the
// rotation kernel (convrot.cu) and usable on the host.
//
// Fast path. Each bf16 value is converted to a double exactly. The 256-point
// transform is four radix-4 stages; every intermediate is a signed subset sum
// of the group's inputs (times a power of two), a multiple of the smallest
// input's last bit and below 256 times the largest input. When the exponent
// fields of the group's nonzero inputs span at most 37 (and |x| < 2^124, no inf
// or NaN) each such sum needs at most 53 bits, so every double operation is
// exact and the results are the exact rotation. The last stage also scales by
// 2^-896 (exact: the results stay multiples of 2^-1034, above the double
// subnormal unit), so a result's double exponent field is its fp32 one and the
// fp32 pattern rounded to odd comes from the high word by integer operations;
// rounding that to bf16 (nearest even) is the correctly rounded bf16 of the
// exact value.
//
// Slow path (any group that fails the test): each output is summed exactly in
// an integer accumulator of nine 32-bit digits held in 64-bit words (2^-138
// times the group's smallest input granule per unit; 256 terms of at most 2^40
// cannot overflow a word), then rounded to bf16 once; inf and NaN follow IEEE
// rules (NaN anywhere: NaN; +inf and -inf terms: NaN; else the infinity).
#pragma once

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define CV_HD __host__ __device__ __forceinline__
#else
#define CV_HD inline
#endif

namespace h3 {
namespace cv {

CV_HD double make_double(uint32_t hi, uint32_t lo) {
#if defined(__CUDA_ARCH__)
  return __hiloint2double((int)hi, (int)lo);
#else
  const uint64_t b = ((uint64_t)hi << 32) | lo;
  double d;
  memcpy(&d, &b, 8);
  return d;
#endif
}
CV_HD void split_double(double d, uint32_t& hi, uint32_t& lo) {
#if defined(__CUDA_ARCH__)
  hi = (uint32_t)__double2hiint(d);
  lo = (uint32_t)__double2loint(d);
#else
  uint64_t b;
  memcpy(&b, &d, 8);
  hi = (uint32_t)(b >> 32);
  lo = (uint32_t)b;
#endif
}
CV_HD float bits_float(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

// The bf16 in the low 16 bits of v as a double (exact; the hardware fp32 -> fp64
// conversion of its fp32 pattern).
CV_HD double bf16_double(uint32_t v) { return (double)bits_float(v << 16); }

// y_j = sum_i x_i H4[i][j] with H4[i][j] = -1 iff i + j == 3: y_j = s - 2 x_(3-j),
// s = x0 + x1 + x2 + x3. LAST folds the 1/16 normalisation and the 2^-896 scaling
// of the result in (both exact: see the header): y_j = s 2^-900 - x_(3-j) 2^-899.
template <bool LAST>
CV_HD void h4(double& a, double& b, double& c, double& d) {
  const double k = LAST ? 0x1p-900 : 1.0;
  const double m = LAST ? -0x1p-899 : -2.0;
#if defined(__CUDA_ARCH__)
  double s = __dadd_rn(__dadd_rn(a, b), __dadd_rn(c, d));
  if (LAST) s = __dmul_rn(s, k);
  const double y0 = __fma_rn(m, d, s), y1 = __fma_rn(m, c, s), y2 = __fma_rn(m, b, s), y3 = __fma_rn(m, a, s);
#else
  double s = (a + b) + (c + d);
  if (LAST) s = s * k;
  const double y0 = m * d + s, y1 = m * c + s, y2 = m * b + s, y3 = m * a + s;  // exact products: no fma needed
#endif
  a = y0;
  b = y1;
  c = y2;
  d = y3;
}

// |y| as an fp32 pattern rounded to odd at 21 significant bits, from the scaled
// double y * 2^-896 (|y| < 2^128): the high word shifted left by 3 (its exponent
// field is the fp32 one; the sign drops out) plus a sticky last bit when the low
// word is not zero. 21 bits exceed 8 + 1, so rounding this to bf16 (nearest
// even) gives the correctly rounded bf16 of |y|; the sign is put back on the
// bf16 pair (bf16_pair_signs).
CV_HD uint32_t rto21_abs_bits(double ys) {
  uint32_t hi, lo;
  split_double(ys, hi, lo);
  return (hi << 3) + (lo != 0u ? 1u : 0u);
}
// The same pattern with the sign of y: (hi * 8 + sticky) keeps the exponent field
// (its top bit, hi's bit 28, is zero for |y| < 2^128) and 20 mantissa bits; the sticky
// bit is min(lo, 1). Rounding it to bf16 (nearest even) gives the correctly rounded bf16 of y.
CV_HD uint32_t rto21_signed_bits(double ys) {
  uint32_t hi, lo;
  split_double(ys, hi, lo);
  return (hi * 8u + (lo < 1u ? lo : 1u)) | (hi & 0x80000000u);
}
// sign bits of two scaled doubles (high words hi0, hi1) at bits 15 and 31
CV_HD uint32_t bf16_pair_signs(uint32_t hi0, uint32_t hi1) {
#if defined(__CUDA_ARCH__)
  return __byte_perm(hi0, hi1, 0x7030) & 0x80008000u;
#else
  return ((hi0 >> 16) & 0x8000u) | (hi1 & 0x80000000u);
#endif
}
CV_HD uint32_t double_hi(double d) {
  uint32_t hi, lo;
  split_double(d, hi, lo);
  return hi;
}

// H[i][o] < 0: an odd number of base-4 digits d with i_d + o_d == 3 (i_d ^ o_d == 3)
CV_HD uint32_t h_negative(uint32_t i, uint32_t o) {
  const uint32_t t = i ^ o;
#if defined(__CUDA_ARCH__)
  return (uint32_t)__popc(t & (t >> 1) & 0x55u) & 1u;
#else
  return (uint32_t)__builtin_popcount(t & (t >> 1) & 0x55u) & 1u;
#endif
}

// Exponent-field statistics of a group: the largest |x| bits and the smallest
// effective field (max(field, 1)) of its nonzero finite inputs.
CV_HD bool fast_path_ok(uint32_t max_abs_bits, uint32_t min_abs_minus1) {
  // min_abs_minus1: min over inputs of (|x| bits - 1) as unsigned (zero -> 0xFFFFFFFF)
  if (max_abs_bits >= 0x7D80u) return false;  // |x| >= 2^124, inf or NaN
  const int fmax = (int)(max_abs_bits >> 7);
  if (min_abs_minus1 == 0xFFFFFFFFu) return true;  // all zero
  int fmin = (int)((min_abs_minus1 + 1u) >> 7);
  fmin = fmin < 1 ? 1 : fmin;
  return fmax - fmin <= 37;
}

// bits [lo, lo + n) of the 288-bit magnitude dig (n <= 9); lo may be negative (zeros below)
CV_HD uint32_t acc_bits(const uint32_t (&dig)[9], int lo, int n) {
  uint64_t window;
  if (lo >= 0) {
    const int w = lo >> 5, sh = lo & 31;
    const uint64_t a = w < 9 ? dig[w] : 0u, b = w + 1 < 9 ? dig[w + 1] : 0u;
    window = ((b << 32) | a) >> sh;
  } else {
    window = (uint64_t)dig[0] << (-lo);  // only reached when the value fits in a few bits
  }
  return (uint32_t)(window & ((1ull << n) - 1ull));
}
CV_HD bool acc_any_below(const uint32_t (&dig)[9], int pos) {  // any bit in [0, pos)
  if (pos <= 0) return false;
  const int w = pos >> 5, sh = pos & 31;
  for (int i = 0; i < w && i < 9; ++i)
    if (dig[i]) return true;
  return w < 9 && sh && (dig[w] & ((1u << sh) - 1u));
}

// Correctly rounded bf16 of V * 2^(fmin - 138), V = sum_w acc[w] * 2^(32 w) (signed)
CV_HD uint32_t acc_to_bf16(const long long (&acc)[9], int fmin) {
  uint32_t dig[9];
  long long c = 0;
  for (int w = 0; w < 9; ++w) {
    const long long t = acc[w] + c;
    dig[w] = (uint32_t)t;
    c = t >> 32;
  }
  uint32_t sign = 0u;
  if (c < 0) {  // negative: two's complement over the 288 bits
    sign = 0x8000u;
    uint64_t carry = 1u;
    for (int w = 0; w < 9; ++w) {
      const uint64_t t = (uint64_t)(~dig[w]) + carry;
      dig[w] = (uint32_t)t;
      carry = t >> 32;
    }
  }
  int top = -1;
  for (int w = 8; w >= 0 && top < 0; --w)
    if (dig[w]) {
      int b = 31;
      while (!((dig[w] >> b) & 1u)) --b;
      top = 32 * w + b;
    }
  if (top < 0) return 0u;  // exact zero
  const int e_top = top + fmin - 138;
  const bool normal = e_top >= -126;
  const int lsb = normal ? top - 7 : 5 - fmin;  // position of the last kept bit (weight 2^(e_top-7) or 2^-133)
  const int n = top - lsb + 1;                  // kept bits (<= 8)
  uint32_t kept = n > 0 ? acc_bits(dig, lsb, n) : 0u;
  const bool rb = lsb >= 1 && n >= 0 && ((acc_bits(dig, lsb - 1, 1)) != 0u);
  const bool st = lsb >= 2 && acc_any_below(dig, lsb - 1);
  if (rb && (st || (kept & 1u))) ++kept;
  if (normal) {
    int e = e_top;
    if (kept == 256u) {
      kept = 128u;
      ++e;
    }
    if (e > 127) return sign | 0x7F80u;
    return sign | ((uint32_t)(e + 127) << 7) | (kept & 0x7Fu);
  }
  return sign | kept;  // units of 2^-133; 128 is the smallest normal
}

// One output of the exact rotation of a group given as 256 bf16 patterns (low 16 bits).
// has_nan / fmin: group facts (fmin = smallest effective exponent field of the nonzero
// finite inputs, 1..254).
template <typename Load>
CV_HD uint32_t slow_output(const Load& load, uint32_t o, bool has_nan, int fmin) {
  if (has_nan) return 0x7FC0u;
  bool pinf = false, ninf = false;
  long long acc[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
  for (uint32_t i = 0; i < 256u; ++i) {
    const uint32_t b = load(i);
    const uint32_t a = b & 0x7FFFu;
    if (a == 0u) continue;
    const uint32_t neg = ((b >> 15) ^ h_negative(i, o)) & 1u;
    if (a == 0x7F80u) {
      if (neg) ninf = true;
      else pinf = true;
      continue;
    }
    const int f = (int)(a >> 7);
    const long long mant = (long long)((a & 0x7Fu) | (f ? 0x80u : 0u));
    const int pos = (f < 1 ? 1 : f) - fmin;
    const long long term = mant << (pos & 31);
    acc[pos >> 5] += neg ? -term : term;
  }
  if (pinf || ninf) return (pinf && ninf) ? 0x7FC0u : (pinf ? 0x7F80u : 0xFF80u);
  return acc_to_bf16(acc, fmin);
}

// Exchange tile of a half-warp: 16 x 16 doubles in rows padded to 144 bytes,
// element (r, c) at byte r * 144 + 8 c. Sixteen lanes writing column c of one
// row fill 128 consecutive bytes (every bank once); eight lanes reading 16 bytes
// at the same column of rows r..r+7 start 144 = 128 + 16 bytes apart, on eight
// different 16-byte bank groups. Both address forms are a per-lane base plus a
// constant, so no per-element address arithmetic is needed.
constexpr int kXRow = 144;
CV_HD int xtile_off(int r, int c) { return r * kXRow + (c << 3); }
CV_HD int xtile_pair_off(int r, int k) { return r * kXRow + (k << 4); }

}  // namespace cv
}  // namespace h3
