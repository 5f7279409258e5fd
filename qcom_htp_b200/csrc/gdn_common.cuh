// Pieces shared by the two GDN C=256 kernels (gdn256.cu: one CTA per SM with next-chunk prefetch,
// the bf16 -> f32 carrier; gdn256x2.cu: two CTAs per SM, the u16 code carrier): swizzled image
// addressing, operand and output tile writers, the code carriers, the 32x32 forward substitution,
// the MMA K-step and the upper-triangle stores.  See gdn256.cu for the algorithm.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"
#include "ptx.cuh"

namespace qhtp {
namespace gdn {

constexpr int kThreads = 256;
constexpr int kC = 256;
constexpr uint32_t KB = 1024;
constexpr uint32_t kTile = 4 * KB;  // one 32-row x 128-byte image or staging tile


// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled image.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * 128 + (((c ^ r) & 7) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

// 32 consecutive f32 values (TMEM columns) of row r -> bf16 chunks c0..c0+3 of an image.
__device__ __forceinline__ void put_row_bf16(uint8_t* img, int r, int c0, const uint32_t (&v)[32]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 w = make_uint4(pack_bf16(__uint_as_float(v[8 * c + 0]), __uint_as_float(v[8 * c + 1])),
                               pack_bf16(__uint_as_float(v[8 * c + 2]), __uint_as_float(v[8 * c + 3])),
                               pack_bf16(__uint_as_float(v[8 * c + 4]), __uint_as_float(v[8 * c + 5])),
                               pack_bf16(__uint_as_float(v[8 * c + 6]), __uint_as_float(v[8 * c + 7])));
    *reinterpret_cast<uint4*>(img + swz(r, c0 + c)) = w;
  }
}

struct OutCodes {   // u16 output carrier: code = clip(rint(t / sT) + zpT, 0, 65535)
  float inv_sT, zpT;
};

__device__ __forceinline__ uint32_t to_code(float t, const OutCodes& oc) {
  const float q = fminf(fmaxf(rintf(t * oc.inv_sT) + oc.zpT, 0.0f), 65535.0f);
  return static_cast<uint32_t>(q);
}

// 32 consecutive f32 values of row r -> a 32x32 staging tile of the output type, in the swizzle of
// the T tensor map: f32 rows of 128 bytes with the 128-byte swizzle, or u16 code rows of 64 bytes
// with the 64-byte swizzle (16-byte chunk c at ((c ^ (r >> 1)) & 3) * 16).
template <bool U16>
__device__ __forceinline__ void put_row_out(uint8_t* tile, int r, const uint32_t (&v)[32], const OutCodes& oc) {
  if constexpr (U16) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        w[i] = to_code(__uint_as_float(v[8 * c + 2 * i]), oc) | (to_code(__uint_as_float(v[8 * c + 2 * i + 1]), oc) << 16);
      *reinterpret_cast<uint4*>(tile + r * 64 + (((c ^ (r >> 1)) & 3) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(tile + swz(r, c)) = make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  }
}

// Input element pair -> f32: bf16 bits, or u16 codes (value = (code - zpA) * sA).
struct InCodes {
  float sA;
  int zpA;  // value = (code - zpA) * sA: exact integer difference, one rounding
};

template <bool U16>
__device__ __forceinline__ float in_lo(uint32_t w, const InCodes& ic) {
  if constexpr (U16) return static_cast<float>(static_cast<int>(w & 0xFFFFu) - ic.zpA) * ic.sA;
  return __uint_as_float(w << 16);
}
template <bool U16>
__device__ __forceinline__ float in_hi(uint32_t w, const InCodes& ic) {
  if constexpr (U16) return static_cast<float>(static_cast<int>(w >> 16) - ic.zpA) * ic.sA;
  return __uint_as_float(w & 0xFFFF0000u);
}

// u16 codes -> bf16 values in place, 16 bytes (8 elements) at a time.
__device__ __forceinline__ void codes_to_bf16(uint8_t* p, const InCodes& ic) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = pack_bf16(in_lo<true>(w[i], ic), in_hi<true>(w[i], ic));
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Level 0: forward substitution on one 32x32 diagonal block held in a swizzled bf16 tile (rows 0..31,
// columns chunk_off*8 .. chunk_off*8+31).  Lane j computes column j:
//     t[i] = delta(i, j) + sum_{k<i} A[i][k] * t[k]
// with four partial sums (k mod 4) to shorten the dependency chain.  Entries with k >= i are
// never read.  t[i] is exactly 0 for i < j and exactly 1 for i == j.
template <bool U16>
__device__ __forceinline__ void solve_diag32(const uint8_t* tile, int chunk_off, int lane, float (&t)[32],
                                             const InCodes& ic) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float s[4] = {(i == lane) ? 1.0f : 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (8 * c < i) {
        const uint4 raw = *reinterpret_cast<const uint4*>(tile + swz(i, c + chunk_off));
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int k = 8 * c + e;
          if (k < i) {
            const float a = (e & 1) ? in_hi<U16>(w[e >> 1], ic) : in_lo<U16>(w[e >> 1], ic);
            s[k & 3] = fmaf(a, t[k], s[k & 3]);
          }
        }
      }
    }
    t[i] = (s[0] + s[1]) + (s[2] + s[3]);
  }
}

// 16 K steps of one M=128 bf16 MMA group: A K-major at a_addr(s), B MN-major at b_addr(s).
__device__ __forceinline__ void mma_k16(uint32_t d, uint32_t a, uint32_t b, uint32_t lbo, uint32_t idesc,
                                        uint32_t acc) {
  mma_bf16(d, desc_kmajor_sw128(a), desc_mnmajor_sw128(b, lbo), idesc, acc);
}

// Upper-triangle zero box e (0..27) of a chunk, 32x32 elements: (column, row) of its top-left corner.
__device__ __forceinline__ void zero_box(int e, int& x, int& y) {
  if (e < 4) {  // level 1: rows 64q..64q+31, columns 64q+32..64q+63
    x = 64 * e + 32;
    y = 64 * e;
  } else if (e < 12) {  // level 2: rows 128h..128h+63, columns 128h+64..128h+127
    const int f = e - 4, h = f >> 2, a = (f >> 1) & 1, b = f & 1;
    x = 128 * h + 64 + 32 * b;
    y = 128 * h + 32 * a;
  } else {  // level 3: rows 0..127, columns 128..255
    const int f = e - 12;
    x = 128 + 32 * (f & 3);
    y = 32 * (f >> 2);
  }
}

// Part `part` (0..3) of a chunk's strict upper triangle outside the 32x32 diagonal blocks, written by
// one warp with coalesced 16-byte stores of the output zero (0.0f, or the zero-point code): rows
// 64q..64q+31 x columns 64q+32.. (q = 0..3), rows 128h..128h+63 x columns 128h+64.. (h = 0..1), rows
// 0..127 x columns 128..255.
template <bool U16>
__device__ __forceinline__ void store_zeros(void* T, int64_t y0, int part, int lane, uint32_t zword) {
  constexpr int es = U16 ? 2 : 4;
  const uint4 z = make_uint4(zword, zword, zword, zword);
  uint8_t* base = static_cast<uint8_t*>(T) + y0 * kC * es;
  const int t = part * 32 + lane;
#pragma unroll
  for (int reg = 0; reg < 7; ++reg) {
    const int row0 = reg < 4 ? 64 * reg : (reg < 6 ? 128 * (reg - 4) : 0);
    const int nrows = reg < 4 ? 32 : (reg < 6 ? 64 : 128);
    const int col0 = reg < 4 ? 64 * reg + 32 : (reg < 6 ? 128 * (reg - 4) + 64 : 128);
    const int cpr = (reg < 4 ? 32 : (reg < 6 ? 64 : 128)) * es / 16;  // 16-byte chunks per row
    for (int idx = t; idx < nrows * cpr; idx += 128) {
      const int r = idx / cpr, c = idx - r * cpr;
      *reinterpret_cast<uint4*>(base + (static_cast<int64_t>(row0 + r) * kC + col0) * es + c * 16) = z;
    }
  }
}

struct Gdn256Args {
  void* T;
  InCodes ic;
  OutCodes oc;
  int64_t n_chunks;
  int* err;
};


}  // namespace gdn
}  // namespace qhtp
