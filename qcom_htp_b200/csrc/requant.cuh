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
// Fast path, pure integer: with the float64 multiplier c = cm * 2^-s (cm its 53-bit mantissa),
// T*cm is formed exactly in 128 bits and split into integer part and s-bit fraction.  c carries a
// relative error <= 2^-52, i.e. <= 2^-35 absolute for |z - zp| < 2^17, so the rounding is decided
// there unless the fraction lies within 2^-30 of one half; those elements are redone exactly with
// 128-bit integer arithmetic on the unrounded scales.
#pragma once
#include <cstdint>

#ifdef __CUDACC__
#define QHTP_HD __host__ __device__ __forceinline__
#define QHTP_HD_NOINLINE static __host__ __device__ __noinline__
#else
#define QHTP_HD inline
#define QHTP_HD_NOINLINE static
#endif

namespace qhtp {

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

QHTP_HD U128 shr128(U128 x, int s) {  // 0 <= s < 128
  if (s == 0) return x;
  if (s >= 64) return U128{x.hi >> (s - 64), 0};
  return U128{(x.lo >> s) | (x.hi << (64 - s)), x.hi >> s};
}

QHTP_HD U128 low_bits(U128 x, int s) {  // x mod 2^s, 1 <= s < 128
  if (s >= 64) return U128{x.lo, s == 64 ? 0 : (x.hi & ((1ull << (s - 64)) - 1))};
  return U128{x.lo & ((1ull << s) - 1), 0};
}

QHTP_HD U128 sub128(U128 a, U128 b) {  // a - b, a >= b
  U128 r{a.lo - b.lo, a.hi - b.hi};
  if (a.lo < b.lo) r.hi -= 1;
  return r;
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
  if (d >= 0) return cmp128(shl128(X, d), Y);  // equal bit lengths (<= 128): align exactly
  return cmp128(X, shl128(Y, -d));
}

// Exact decision between r0 and r0 + 1, where r0 = floor(z*) for a z* within 1e-9 of r0 + 1/2.
// |T| * mul must stay below 2^75 (so that |T|*mul*mA < 2^128): guaranteed by the K limit.
QHTP_HD_NOINLINE int64_t exact_round_near_tie(int64_t T, uint32_t mul, uint64_t mA, int e2, uint64_t mO, int eO,
                                              int64_t zp_out, int64_t r0) {
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

// Branch-free fast path for the epilogue.  c = cm * 2^-s with 31 <= s <= 127 (checked at prepare).
// Returns the clipped code computed as round_half_up(T*c) + zp, and sets *near when the fraction of
// T*c lies within 2^-30 of one half (then the caller must use requant_code, which breaks the tie
// exactly); away from ties round-half-up equals round-half-even.
QHTP_HD int32_t requant_fast(int64_t T, uint64_t cm, int s, int32_t zp_out, int32_t qmax, bool* near) {
  const bool neg = T < 0;
  const uint64_t a = neg ? static_cast<uint64_t>(-(T + 1)) + 1u : static_cast<uint64_t>(T);
  uint64_t lo = a * cm;
#ifdef __CUDA_ARCH__
  uint64_t hi = __umul64hi(a, cm);
#else
  uint64_t hi = static_cast<uint64_t>((static_cast<unsigned __int128>(a) * cm) >> 64);
#endif
  // |T*c| >= 2^20, i.e. P >> (s + 20) != 0, lies far outside [0, qmax] (zp < 2^16): saturate.
  // Branches on s are uniform across a warp (one channel per step).
  bool big;
  if (s >= 108) {
    big = false;  // P < 2^117 < 2^(s+20)
  } else if (s >= 44) {
    big = (hi >> (s - 44)) != 0;
  } else {
    big = hi != 0 || (lo >> (s + 20)) != 0;
  }
  // add one half at the binary point (bit s-1), then keep 30 fraction bits: W = (P + half) >> (s-30)
  if (s - 1 >= 64) {
    hi += 1ull << (s - 65);
  } else {
    const uint64_t lo2 = lo + (1ull << (s - 1));
    hi += lo2 < lo ? 1ull : 0ull;
    lo = lo2;
  }
  const int sh = s - 30;  // 1 <= sh <= 97
  const uint64_t W = sh >= 64 ? (hi >> (sh - 64)) : ((lo >> sh) | (hi << (64 - sh)));
  const uint32_t win = static_cast<uint32_t>(W) & 0x3FFFFFFFu;
  *near = !big && ((win == 0u) | (win == 0x3FFFFFFFu));
  const int64_t mag = static_cast<int64_t>(W >> 30);
  int64_t r = (neg ? -mag : mag) + zp_out;
  if (big) r = neg ? 0 : qmax;
  r = r < 0 ? 0 : r;
  r = r > qmax ? qmax : r;
  return static_cast<int32_t>(r);
}

// Per-channel constants of the epilogue fast path: the float64 multiplier c = cm * 2^-cshift
// (cm its 53-bit mantissa) is applied as  V = (|T| << tn) * cmn * 2^-96, i.e. tn = 96 - cshift and
// cmn = cm, so the binary point of the 128-bit product sits at bit 96 for every channel.  Channels
// with c < 2^-44 (cshift > 96) use tn = 0 and cmn = cm * 2^(96-cshift) rounded half up.
// Requires c < 2^18 (cshift >= 34).
struct FastConst {
  uint64_t cmn;
  int tn;
};

QHTP_HD FastConst fast_const(uint64_t cm, int cshift) {
  if (cshift <= 96) return FastConst{cm, 96 - cshift};
  const int d = cshift - 96;
  if (d >= 64) return FastConst{0, 0};
  return FastConst{(cm + (1ull << (d - 1))) >> d, 0};
}

// Branch-free fast path.  Returns clip(round_half_up(T*c) + zp) and sets *near when the result may
// differ from round-half-even of the exact value: the 30 fraction bits below the binary point are
// within 2 units (2^-29) of a tie.  Error budget of V: truncation of the low product bits < 2^-30,
// cmn rounding <= 2^-34, c itself (a float64) <= 2^-33 for |V| < 2^19.  |T| >= 2^(63-tn) means
// |V| >= 2^19, which saturates.
QHTP_HD int32_t requant_fast96(int64_t T, uint64_t cmn, int tn, int32_t zp_out, int32_t qmax, bool* near,
                               int64_t* floor_v) {
  const bool neg = T < 0;
  const uint64_t a = neg ? static_cast<uint64_t>(-(T + 1)) + 1u : static_cast<uint64_t>(T);
  const bool big = (a >> (63 - tn)) != 0;
  const uint64_t ap = a << tn;  // < 2^63 unless big
#ifdef __CUDA_ARCH__
  const uint64_t hi = __umul64hi(ap, cmn);
#else
  const uint64_t hi = static_cast<uint64_t>((static_cast<unsigned __int128>(ap) * cmn) >> 64);
#endif
  // W = floor((P + 2^95) / 2^66): rounded magnitude above 30 fraction bits
  const uint64_t W = (hi + (1ull << 31)) >> 2;
  const uint32_t win = static_cast<uint32_t>(W) & 0x3FFFFFFFu;
  *near = !big && (((win + 2u) & 0x3FFFFFFFu) < 4u);
  const int64_t mag = static_cast<int64_t>(W >> 30);
  // floor of the signed value (meaningful when *near): |V| + 1/2 sits next to an integer boundary
  const int64_t fl_mag = win < (1u << 29) ? mag - 1 : mag;  // floor(|V|)
  *floor_v = (neg ? -fl_mag - 1 : fl_mag) + zp_out;
  int64_t r = (neg ? -mag : mag) + zp_out;
  if (big) r = neg ? 0 : qmax;
  r = r < 0 ? 0 : r;
  r = r > qmax ? qmax : r;
  return static_cast<int32_t>(r);
}

// Signed form of requant_fast96 (same constants, same error budget, same tie window).  With
// ap = T << tn and P = ap * cmn (signed 128-bit), V = P / 2^96 and
//     W = floor((floor(P / 2^64) + 2^31) / 4) = floor((V + 1/2) * 2^30)   (arithmetic shifts)
// carries round_half_up(V) in W >> 30 and the 30 fraction bits of V + 1/2 in its low bits for either
// sign, so no absolute value or re-negation is needed.  Returns clip(round_half_up(V) + zp) and sets
// *near as requant_fast96 does; *w_out receives W for requant_tie_w.
QHTP_HD int32_t requant_fast96s(int64_t T, uint64_t cmn, int tn, int32_t zp_out, int32_t qmax, bool* near,
                                int64_t* w_out) {
  const int64_t top = T >> (63 - tn);  // 0 or -1 unless |T| >= 2^(63-tn)
  const bool big = (top != 0) & (top != -1);
  const int64_t ap = static_cast<int64_t>(static_cast<uint64_t>(T) << tn);
#ifdef __CUDA_ARCH__
  const int64_t hi = __mul64hi(ap, static_cast<int64_t>(cmn));
#else
  const int64_t hi = static_cast<int64_t>((static_cast<__int128>(ap) * static_cast<__int128>(cmn)) >> 64);
#endif
  const int64_t W = (hi + (int64_t{1} << 31)) >> 2;
  const uint32_t win = static_cast<uint32_t>(W) & 0x3FFFFFFFu;
  *near = !big && (((win + 2u) & 0x3FFFFFFFu) < 4u);
  *w_out = W;
  int32_t r = static_cast<int32_t>(W >> 30) + zp_out;  // |V| < 2^20 unless big
  r = r < 0 ? 0 : r;
  r = r > qmax ? qmax : r;
  return big ? (T < 0 ? 0 : qmax) : r;
}

// Exact code for an element flagged by requant_fast96s, from its W: floor(z*) = floor(V) + zp with
// floor(V) = floor(V + 1/2) - [frac(V + 1/2) < 1/2].
QHTP_HD int32_t requant_tie_w(int64_t T, int64_t W, uint32_t mul, int e2, uint64_t mA, uint64_t mO, int eO,
                              int32_t zp_out, int32_t qmax) {
  const uint32_t win = static_cast<uint32_t>(W) & 0x3FFFFFFFu;
  const int64_t fl = (W >> 30) - (win < (1u << 29) ? 1 : 0) + zp_out;
  int64_t r = exact_round_near_tie(T, mul, mA, e2, mO, eO, zp_out, fl);
  r = r < 0 ? 0 : r;
  r = r > qmax ? qmax : r;
  return static_cast<int32_t>(r);
}

// Exact code for an element flagged by requant_fast96; floor_v = floor(z*) from the fast path.
QHTP_HD int32_t requant_tie(int64_t T, int64_t floor_v, uint32_t mul, int e2, uint64_t mA, uint64_t mO, int eO,
                            int32_t zp_out, int32_t qmax) {
  int64_t r = exact_round_near_tie(T, mul, mA, e2, mO, eO, zp_out, floor_v);
  r = r < 0 ? 0 : r;
  r = r > qmax ? qmax : r;
  return static_cast<int32_t>(r);
}

// Output code of one element.  cm/s: requant multiplier c = cm * 2^-s (1 <= s <= 127).
QHTP_HD int32_t requant_code(int64_t T, uint64_t cm, int s, uint32_t mul, int e2, uint64_t mA, uint64_t mO, int eO,
                             int32_t zp_out, int32_t qmax) {
  const bool neg = T < 0;
  const uint64_t a = neg ? static_cast<uint64_t>(-(T + 1)) + 1u : static_cast<uint64_t>(T);
  const U128 P = mul_64x64(a, cm);  // |T| * cm, exact
  const U128 ip = shr128(P, s);
  if (ip.hi != 0 || ip.lo > (1ull << 20)) return neg ? 0 : qmax;  // |z - zp| > 2^20: far outside the range
  const U128 f = low_bits(P, s);
  const U128 half = shl128(U128{1, 0}, s - 1);
  const int c = cmp128(f, half);
  const U128 d = c >= 0 ? sub128(f, half) : sub128(half, f);
  const int tol_bits = s - 30;  // tie window 2^-30, in units of 2^-s
  const bool near = tol_bits > 0 ? (bitlen128(d) <= tol_bits) : (d.hi == 0 && d.lo <= 1);
  int64_t r;
  if (near) {
    const int64_t r0 = (neg ? -static_cast<int64_t>(ip.lo) - 1 : static_cast<int64_t>(ip.lo)) + zp_out;
    r = exact_round_near_tie(T, mul, mA, e2, mO, eO, zp_out, r0);
  } else {
    const int64_t mag = static_cast<int64_t>(ip.lo) + (c > 0 ? 1 : 0);
    r = (neg ? -mag : mag) + zp_out;
  }
  if (r < 0) r = 0;
  if (r > qmax) r = qmax;
  return static_cast<int32_t>(r);
}

}  // namespace qhtp
