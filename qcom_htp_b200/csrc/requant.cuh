// Exact requantization of an integer accumulator to an output code.
//
// The real value of an output element is  z* = T * mul * mA * 2^e2 / (mO * 2^eO) + zp_out, where
//   T    : int64 accumulator (q-plane x m_q + e'-plane + effective bias; see the prepare kernel),
//   mul  : extra integer factor (1, or the f32 weight-scale mantissa in exact-dequant mode),
//   mA   : 53-bit integer mantissa of the activation scale, e2 the combined binary exponent,
//   mO,eO: 53-bit mantissa / exponent of the output scale.
// The output code is clip(round_half_even(z*), 0, qmax), the rounding of the reference oracle
// (generate_qnn_matmul_python_cases.py:217 np.rint, :474-481).
//
// Fast path: z = double(T) * c + zp_out with c = double(mul*mA*2^e2/(mO*2^eO)); its absolute error
// is below 6e-11 for |z| < 2^17.  Whenever z lies within kTieEps of a .5 boundary the decision is
// redone exactly with 128-bit integer arithmetic.
#pragma once
#include <cmath>
#include <cstdint>

#ifdef __CUDACC__
#define QHTP_HD __host__ __device__ __forceinline__
#else
#define QHTP_HD inline
#endif

namespace qhtp {

constexpr double kTieEps = 1e-9;

struct U128 {
  uint64_t lo, hi;
};

QHTP_HD U128 mul_64x64(uint64_t a, uint64_t b) {
#ifdef __CUDA_ARCH__
  return U128{a * b, __umul64hi(a, b)};
#else
  unsigned __int128 p = static_cast<unsigned __int128>(a) * b;
  return U128{static_cast<uint64_t>(p), static_cast<uint64_t>(p >> 64)};
#endif
}

// (a * b) mod 2^128; exact when the true product is below 2^128.
QHTP_HD U128 mul_128x64(U128 a, uint64_t b) {
  U128 r = mul_64x64(a.lo, b);
  r.hi += a.hi * b;
  return r;
}

QHTP_HD int bitlen64(uint64_t x) {
#ifdef __CUDA_ARCH__
  return 64 - __clzll(static_cast<long long>(x));
#else
  return x ? 64 - __builtin_clzll(x) : 0;
#endif
}

QHTP_HD int bitlen128(U128 x) { return x.hi ? 64 + bitlen64(x.hi) : bitlen64(x.lo); }

QHTP_HD U128 shl128(U128 x, int s) {  // 0 <= s < 128
  if (s == 0) return x;
  if (s >= 64) return U128{0, x.lo << (s - 64)};
  return U128{x.lo << s, (x.hi << s) | (x.lo >> (64 - s))};
}

QHTP_HD int cmp128(U128 a, U128 b) {
  if (a.hi != b.hi) return a.hi < b.hi ? -1 : 1;
  if (a.lo != b.lo) return a.lo < b.lo ? -1 : 1;
  return 0;
}

// Compare X * 2^ex with Y * 2^ey for nonnegative X, Y (bit lengths <= 128).
QHTP_HD int cmp_scaled(U128 X, int ex, U128 Y, int ey) {
  const int bx = bitlen128(X), by = bitlen128(Y);
  if (bx == 0 || by == 0) return (bx == 0 && by == 0) ? 0 : (bx == 0 ? -1 : 1);
  const int d = ex - ey;
  const int lx = bx + d;  // bit length of X*2^d
  if (lx > by) return 1;
  if (lx < by) return -1;
  // equal bit lengths (<= 128 on both sides): align exactly
  if (d >= 0) return cmp128(shl128(X, d), Y);
  return cmp128(X, shl128(Y, -d));
}

// Exact decision between floor(z) and floor(z)+1 for a z within 1e-9 of a .5 boundary.
// |T| * mul must stay below 2^75 (so that |T|*mul*mA < 2^128): guaranteed by the K limit.
QHTP_HD int64_t exact_round_near_tie(int64_t T, uint32_t mul, uint64_t mA, int e2, uint64_t mO, int eO,
                                     int64_t zp_out, double z) {
  const int64_t r0 = static_cast<int64_t>(floor(z));
  const int64_t hn = 2 * (r0 - zp_out) + 1;  // boundary = hn/2 (odd numerator, never 0)
  const uint64_t absT = T < 0 ? static_cast<uint64_t>(-(T + 1)) + 1u : static_cast<uint64_t>(T);
  const U128 L = mul_128x64(mul_64x64(absT, mul), mA);
  const uint64_t absH = hn < 0 ? static_cast<uint64_t>(-hn) : static_cast<uint64_t>(hn);
  const U128 R = mul_64x64(absH, mO);
  const int sL = (T > 0) - (T < 0);
  const int sR = hn > 0 ? 1 : -1;
  int c;  // sign(value - boundary)
  if (sL == 0) {
    c = -sR;
  } else if (sL != sR) {
    c = sL;
  } else {
    c = cmp_scaled(L, e2, R, eO - 1) * sL;
  }
  if (c > 0) return r0 + 1;
  if (c < 0) return r0;
  return (r0 % 2 == 0) ? r0 : r0 + 1;  // exact tie: half to even
}

#ifdef __CUDA_ARCH__
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double i2d(int64_t v) { return __ll2double_rn(v); }
#else
inline double dmul(double a, double b) { return a * b; }
inline double dadd(double a, double b) { return a + b; }
inline double i2d(int64_t v) { return static_cast<double>(v); }
#endif

// Full requant of one element: returns the clipped output code.
QHTP_HD int32_t requant_code(int64_t T, double c, uint32_t mul, int e2, uint64_t mA, uint64_t mO, int eO,
                             int32_t zp_out, int32_t qmax) {
  const double z = dadd(dmul(i2d(T), c), static_cast<double>(zp_out));
  if (!(z > -1.0)) return 0;                                       // also catches NaN
  if (!(z < static_cast<double>(qmax) + 1.0)) return qmax;
  int64_t r;
  const double f = z - floor(z);
  if (fabs(f - 0.5) <= kTieEps) {
    r = exact_round_near_tie(T, mul, mA, e2, mO, eO, zp_out, z);
  } else {
    r = static_cast<int64_t>(rint(z));
  }
  if (r < 0) r = 0;
  if (r > qmax) r = qmax;
  return static_cast<int32_t>(r);
}

}  // namespace qhtp
