// GDN / KDA chunk triangular inverse on B200:  T = (I - A)^-1, A strictly lower triangular [C,C].
//
// Algorithm (recursive doubling on the block structure; reference algorithm family:
// example/gdn_native/solve_op/gdn_solve_ref.c:19-69 (BL=16 forward substitution + block merge),
// example/gdn_native/solve_br_op (BL=64 block-recursive), pure_hmx_solve/gdn_pure_solve.cpp:900-1030):
//   level 0  each 32x32 diagonal block is inverted by forward substitution in fp32 registers, one
//            warp per block, lane j owning column j  (T[i,:] = e_i + sum_{k<i} A[i,k] T[k,:]);
//   level 1  each 64x64 diagonal block: T10 = T11 * (A10 * T00) with 32x32 blocks, fp32 CUDA cores;
//   level 2  each 128x128 diagonal block: T10 = T11 * (A10 * T00) with 64x64 blocks, two bf16
//            tcgen05 MMAs (M=128 rows; rows 0..63 of each product are unused padding) with fp32
//            accumulators in TMEM;
//   level 3  the 256x256 chunk: T10 = T11 * (A10 * T00) with 128x128 blocks, two bf16 tcgen05 MMAs.
// With L = I - A the 2x2 block inverse is [[T00, 0], [T11 A10 T00, T11]] (A10 = -L10).
// One persistent CTA (256 threads) per SM walks the chunks; TMEM (512 columns) is allocated once.
// The strict upper triangle of every output chunk is written as zero; input entries on or above the
// diagonal are ignored.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"
#include "ptx.cuh"

namespace qhtp {

namespace {

constexpr int kThreads = 256;

struct GdnIO {
  const void* A;
  void* T;
  int64_t n_chunks;
  int zpA, zpT;
  float sA, inv_sT;
  int* err;
};

// 8 consecutive input elements of one row, as fp32.
template <bool U16>
__device__ __forceinline__ void load8(const GdnIO& io, size_t off, float (&v)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(io.A) + off);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = w[i] & 0xFFFFu, hi = w[i] >> 16;
    if constexpr (U16) {
      v[2 * i] = static_cast<float>(static_cast<int>(lo) - io.zpA) * io.sA;
      v[2 * i + 1] = static_cast<float>(static_cast<int>(hi) - io.zpA) * io.sA;
    } else {
      v[2 * i] = __uint_as_float(lo << 16);
      v[2 * i + 1] = __uint_as_float(hi << 16);
    }
  }
}

__device__ __forceinline__ uint32_t code_of(float t, float inv_sT, int zpT) {
  float q = rintf(t * inv_sT) + static_cast<float>(zpT);
  q = fminf(fmaxf(q, 0.0f), 65535.0f);
  return static_cast<uint32_t>(q);
}

// Store 4 consecutive output elements of one row.
template <bool U16>
__device__ __forceinline__ void store4(const GdnIO& io, size_t off, float a, float b, float c, float d) {
  if constexpr (U16) {
    const uint32_t x = code_of(a, io.inv_sT, io.zpT) | (code_of(b, io.inv_sT, io.zpT) << 16);
    const uint32_t y = code_of(c, io.inv_sT, io.zpT) | (code_of(d, io.inv_sT, io.zpT) << 16);
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(io.T) + off) = make_uint2(x, y);
  } else {
    *reinterpret_cast<float4*>(static_cast<float*>(io.T) + off) = make_float4(a, b, c, d);
  }
}

// Byte offset of bf16 element (r, c) in a K-major 128-byte-swizzled operand tile of `rows` rows;
// K is split into 64-element regions of rows*128 bytes each.
__device__ __forceinline__ uint32_t sw_off(int r, int c, int rows) {
  const int region = c >> 6, cc = c & 63;
  return static_cast<uint32_t>(region * rows * 128 + r * 128 + (((cc >> 3) ^ (r & 7)) << 4) + ((cc & 7) << 1));
}

__device__ __forceinline__ void st_bf16(uint8_t* tile, int r, int c, int rows, float v) {
  *reinterpret_cast<__nv_bfloat16*>(tile + sw_off(r, c, rows)) = __float2bfloat16_rn(v);
}

// 8 consecutive K elements (c % 8 == 0) as one 16-byte store.
__device__ __forceinline__ void st_bf16x8(uint8_t* tile, int r, int c, int rows, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  *reinterpret_cast<uint4*>(tile + sw_off(r, c, rows)) = make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[128 x N] (TMEM, fp32) = A_tile[128 x K] * B_tile[N x K]^T, both bf16 K-major SW128 in smem.
__device__ __forceinline__ void issue_mma_bf16(uint32_t d_tmem, uint32_t a_smem, uint32_t b_smem, int N, int K) {
  const uint32_t idesc = (N == 64) ? idesc_bf16(128, 64) : idesc_bf16(128, 128);
  for (int kk = 0; kk < K / 16; ++kk) {
    const int region = kk >> 2, within = kk & 3;
    const uint64_t da = desc_kmajor_sw128(a_smem + region * 128 * 128 + within * 32);
    const uint64_t db = desc_kmajor_sw128(b_smem + region * N * 128 + within * 32);
    mma_bf16(d_tmem, da, db, idesc, kk > 0 ? 1u : 0u);
  }
}

// smem plan (bytes), C = 256.  R0 = [0, 96K): T64f (4 x 64x64 fp32) | T10f (2 x 64x64 fp32);
// later SA3 (A[128:256, 0:128] bf16) | SB4.  R1 = [96K, 192K): stage-1 A64f (4 x 64x64 fp32) and
// X32 (4 x 32x32 fp32); stage-2 per-half operands; stage-3 SB3 | SA4.
template <int C>
struct GdnSmem {
  static constexpr int NB64 = C >= 64 ? C / 64 : 1;
  static constexpr int kT64 = 0;
  static constexpr int kT10 = NB64 * 64 * 64 * 4;
  static constexpr int kR1 = C == 256 ? 96 * 1024 : (C == 128 ? 48 * 1024 : 16 * 1024 + 0);
  static constexpr int kA64 = C == 32 ? 4096 : kR1;
  static constexpr int kX32 = kA64 + NB64 * 64 * 64 * 4;
  static constexpr int kStage2 = kR1;   // per half: SA 16K | SA2 16K | SB1 8K | SB2 8K
  static constexpr int kBytesRaw = C == 256 ? 192 * 1024 : (C == 128 ? 96 * 1024 : (C == 64 ? 48 * 1024 : 8192));
  static constexpr int kBar = kBytesRaw;
  static constexpr int kTotal = kBytesRaw + 64 + 1024;
};

template <int C, bool U16>
__global__ void __launch_bounds__(kThreads, 1) gdn_inverse_kernel(GdnIO io) {
  using SM = GdnSmem<C>;
  constexpr int NB64 = SM::NB64;
  constexpr int NB32 = C / 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* T64f = reinterpret_cast<float*>(smem + SM::kT64);   // [NB64][64][64] (C=32: [32][32])
  float* T10f = reinterpret_cast<float*>(smem + SM::kT10);   // [2][64][64]
  float* A64f = reinterpret_cast<float*>(smem + SM::kA64);   // [NB64][64][64]
  float* X32 = reinterpret_cast<float*>(smem + SM::kX32);    // [NB64][32][32]
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SM::kBar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr bool kTensor = C >= 128;
  if (kTensor) {
    if (tid == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
    }
    if (warp == 0) {
      tmem_alloc(tslot, 512);
      tmem_relinquish();
    }
    tc_fence_before();
  }
  __syncthreads();
  uint32_t tmem = 0;
  if (kTensor) {
    tc_fence_after();
    tmem = *tslot;
  }
  uint32_t mma_phase = 0;
  bool failed = false;
  constexpr int BW = C >= 64 ? 64 : 32;  // diagonal block width held in T64f / A64f

  for (int64_t ch = blockIdx.x; ch < io.n_chunks && !failed; ch += gridDim.x) {
    const size_t base = static_cast<size_t>(ch) * C * C;
    // ---------------------------------------------------------------- stage 1: diagonal blocks
    // A64f[q] = strictly-lower part of the q-th BWxBW diagonal block of A (fp32), T64f zeroed.
    for (int e = tid; e < NB64 * BW * BW / 8; e += kThreads) {
      const int q = e / (BW * BW / 8), rem = e % (BW * BW / 8);
      const int r = rem / (BW / 8), c0 = (rem % (BW / 8)) * 8;
      float v[8];
      load8<U16>(io, base + static_cast<size_t>(q * BW + r) * C + q * BW + c0, v);
      float* dst = A64f + (q * BW + r) * BW + c0;
      float* tz = T64f + (q * BW + r) * BW + c0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dst[i] = (c0 + i < r) ? v[i] : 0.0f;
        tz[i] = 0.0f;
      }
    }
    __syncthreads();
    // level 0: warp w inverts 32x32 diagonal block w by forward substitution
    if (warp < NB32) {
      const int q = warp / (BW / 32), o = (warp % (BW / 32)) * 32;
      const float* a = A64f + q * BW * BW;
      float t[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float s = (i == lane) ? 1.0f : 0.0f;
#pragma unroll
        for (int k = 0; k < i; ++k) s = fmaf(a[(o + i) * BW + o + k], t[k], s);
        t[i] = s;
      }
      float* tb = T64f + q * BW * BW;
#pragma unroll
      for (int i = 0; i < 32; ++i) tb[(o + i) * BW + o + lane] = t[i];
    }
    __syncthreads();
    if constexpr (C >= 64) {
      // level 1: within each 64-block q, X = A10 * T00, then T10 = T11 * X (32x32 blocks)
      constexpr int TPB = kThreads / NB64;
      const int q = tid / TPB, lt = tid % TPB;
      const float* a = A64f + q * 4096;
      float* tq = T64f + q * 4096;
      float* x = X32 + q * 1024;
      for (int e = lt; e < 1024; e += TPB) {
        const int r = e >> 5, c = e & 31;
        float s = 0.0f;
        for (int k = c; k < 32; ++k) s = fmaf(a[(32 + r) * 64 + k], tq[k * 64 + c], s);
        x[r * 32 + c] = s;
      }
      __syncthreads();
      for (int e = lt; e < 1024; e += TPB) {
        const int r = e >> 5, c = e & 31;
        float s = 0.0f;
        for (int k = 0; k <= r; ++k) s = fmaf(tq[(32 + r) * 64 + 32 + k], x[k * 32 + c], s);
        tq[(32 + r) * 64 + c] = s;
      }
      __syncthreads();
    }
    // write the diagonal BWxBW blocks (zeros above their diagonal included)
    for (int e = tid; e < NB64 * BW * BW / 4; e += kThreads) {
      const int q = e / (BW * BW / 4), rem = e % (BW * BW / 4);
      const int r = rem / (BW / 4), c0 = (rem % (BW / 4)) * 4;
      const float* s = T64f + (q * BW + r) * BW + c0;
      store4<U16>(io, base + static_cast<size_t>(q * BW + r) * C + q * BW + c0, s[0], s[1], s[2], s[3]);
    }
    // zero the strict upper triangle outside the diagonal blocks
    if constexpr (C >= 128) {
      for (int e = tid; e < C * C / 4; e += kThreads) {
        const int r = e / (C / 4), c0 = (e % (C / 4)) * 4;
        if (c0 / 64 > r / 64) store4<U16>(io, base + static_cast<size_t>(r) * C + c0, 0.f, 0.f, 0.f, 0.f);
      }
    }
    if constexpr (C >= 128) {
      // ---------------------------------------------------------------- stage 2: 64 -> 128
      constexpr int NH = C / 128;
      for (int h = 0; h < NH; ++h) {
        uint8_t* sa = smem + SM::kStage2 + h * 48 * 1024;  // rows 64..127 = A[128h+64+r][128h+c]
        uint8_t* sa2 = sa + 16 * 1024;                      // rows 64..127 = T64_{2h+1}
        uint8_t* sb1 = sa + 32 * 1024;                      // (n,k) = T64_{2h}[k][n]
        for (int e = tid; e < 64 * 8; e += kThreads) {
          const int r = e >> 3, c0 = (e & 7) * 8;
          float v[8];
          load8<U16>(io, base + static_cast<size_t>(128 * h + 64 + r) * C + 128 * h + c0, v);
          st_bf16x8(sa, 64 + r, c0, 128, v);
          const float* t1 = T64f + (2 * h + 1) * 4096 + r * 64 + c0;
          float w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = t1[i];
          st_bf16x8(sa2, 64 + r, c0, 128, w);
          // SB1 row n = r, K elements k = c0..c0+7 : T64_{2h}[k][n]
          const float* t0 = T64f + (2 * h) * 4096;
          float u[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) u[i] = t0[(c0 + i) * 64 + r];
          st_bf16x8(sb1, r, c0, 64, u);
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        for (int h = 0; h < NH; ++h) {
          const uint32_t sa = smem_u32(smem + SM::kStage2 + h * 48 * 1024);
          issue_mma_bf16(tmem + 128 * h, sa, sa + 32 * 1024, 64, 64);
        }
        mma_commit(bar);
      }
      failed = __syncthreads_or(mbar_wait(bar, mma_phase, io.err, kErrTimeoutOther) ? 0 : 1) != 0;
      mma_phase ^= 1;
      if (failed) break;
      tc_fence_after();
      // X_h = rows 64..127 of D1 -> SB2 (n,k) = X[k][n]; lanes 64..127 belong to warps 2,3,6,7
      {
        const int quad = warp & 3;
        if (quad >= 2) {
          const int k = (quad - 2) * 32 + lane;
          const int cb = (warp >= 4) ? 32 : 0;
          for (int h = 0; h < NH; ++h) {
            uint8_t* sb2 = smem + SM::kStage2 + h * 48 * 1024 + 40 * 1024;
            for (int c0 = cb; c0 < cb + 32; c0 += 16) {
              uint32_t rr[16];
              tmem_ld16(tmem + 128 * h + c0 + (static_cast<uint32_t>(quad * 32) << 16), rr);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j) st_bf16(sb2, c0 + j, k, 64, __uint_as_float(rr[j]));
            }
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        for (int h = 0; h < NH; ++h) {
          const uint32_t sa = smem_u32(smem + SM::kStage2 + h * 48 * 1024);
          issue_mma_bf16(tmem + 128 * h + 64, sa + 16 * 1024, sa + 40 * 1024, 64, 64);
        }
        mma_commit(bar);
      }
      failed = __syncthreads_or(mbar_wait(bar, mma_phase, io.err, kErrTimeoutOther) ? 0 : 1) != 0;
      mma_phase ^= 1;
      if (failed) break;
      tc_fence_after();
      // T10_h = rows 64..127 of D2 -> global and T10f
      {
        const int quad = warp & 3;
        if (quad >= 2) {
          const int r = (quad - 2) * 32 + lane;
          const int cb = (warp >= 4) ? 32 : 0;
          for (int h = 0; h < NH; ++h) {
            for (int c0 = cb; c0 < cb + 32; c0 += 16) {
              uint32_t rr[16];
              tmem_ld16(tmem + 128 * h + 64 + c0 + (static_cast<uint32_t>(quad * 32) << 16), rr);
              tmem_ld_wait();
              float* t10 = T10f + h * 4096 + r * 64 + c0;
#pragma unroll
              for (int j = 0; j < 16; ++j) t10[j] = __uint_as_float(rr[j]);
              const size_t off = base + static_cast<size_t>(128 * h + 64 + r) * C + 128 * h + c0;
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                store4<U16>(io, off + j, __uint_as_float(rr[j]), __uint_as_float(rr[j + 1]),
                            __uint_as_float(rr[j + 2]), __uint_as_float(rr[j + 3]));
            }
          }
        }
      }
      tc_fence_before();
      __syncthreads();
    }
    if constexpr (C == 256) {
      // ---------------------------------------------------------------- stage 3: 128 -> 256
      uint8_t* sb3 = smem + 96 * 1024;   // (n,k) = T128_0[k][n], 128 x 128
      uint8_t* sa4 = smem + 128 * 1024;  // T128_1 row-major, 128 x 128
      // T128_h = [[T64_{2h}, 0], [T10_h, T64_{2h+1}]]
      for (int e = tid; e < 128 * 16; e += kThreads) {
        const int r = e >> 4, c0 = (e & 15) * 8;
        float v[8], u[8];
        // sa4 row r, k = c0..c0+7 of T128_1
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = c0 + i;
          float val;
          if (r < 64) val = (c < 64) ? T64f[2 * 4096 + r * 64 + c] : 0.0f;
          else val = (c < 64) ? T10f[4096 + (r - 64) * 64 + c] : T64f[3 * 4096 + (r - 64) * 64 + c - 64];
          v[i] = val;
        }
        st_bf16x8(sa4, r, c0, 128, v);
        // sb3 row n = r, k = c0..c0+7: T128_0[k][n]
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k = c0 + i, n = r;
          float val;
          if (k < 64) val = (n < 64) ? T64f[k * 64 + n] : 0.0f;
          else val = (n < 64) ? T10f[(k - 64) * 64 + n] : T64f[4096 + (k - 64) * 64 + n - 64];
          u[i] = val;
        }
        st_bf16x8(sb3, r, c0, 128, u);
      }
      __syncthreads();  // R0 (T64f/T10f) is free from here on
      uint8_t* sa3 = smem;               // A[128+r][k], 128 x 128
      for (int e = tid; e < 128 * 16; e += kThreads) {
        const int r = e >> 4, c0 = (e & 15) * 8;
        float v[8];
        load8<U16>(io, base + static_cast<size_t>(128 + r) * C + c0, v);
        st_bf16x8(sa3, r, c0, 128, v);
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        issue_mma_bf16(tmem + 256, smem_u32(sa3), smem_u32(sb3), 128, 128);
        mma_commit(bar);
      }
      failed = __syncthreads_or(mbar_wait(bar, mma_phase, io.err, kErrTimeoutOther) ? 0 : 1) != 0;
      mma_phase ^= 1;
      if (failed) break;
      tc_fence_after();
      uint8_t* sb4 = smem + 32 * 1024;   // (n,k) = X[k][n]
      {
        const int quad = warp & 3;
        const int k = quad * 32 + lane;
        const int cb = (warp >= 4) ? 64 : 0;
        for (int c0 = cb; c0 < cb + 64; c0 += 16) {
          uint32_t rr[16];
          tmem_ld16(tmem + 256 + c0 + (static_cast<uint32_t>(quad * 32) << 16), rr);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) st_bf16(sb4, c0 + j, k, 128, __uint_as_float(rr[j]));
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        issue_mma_bf16(tmem + 384, smem_u32(sa4), smem_u32(sb4), 128, 128);
        mma_commit(bar);
      }
      failed = __syncthreads_or(mbar_wait(bar, mma_phase, io.err, kErrTimeoutOther) ? 0 : 1) != 0;
      mma_phase ^= 1;
      if (failed) break;
      tc_fence_after();
      {
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const int cb = (warp >= 4) ? 64 : 0;
        for (int c0 = cb; c0 < cb + 64; c0 += 16) {
          uint32_t rr[16];
          tmem_ld16(tmem + 384 + c0 + (static_cast<uint32_t>(quad * 32) << 16), rr);
          tmem_ld_wait();
          const size_t off = base + static_cast<size_t>(128 + r) * C + c0;
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            store4<U16>(io, off + j, __uint_as_float(rr[j]), __uint_as_float(rr[j + 1]), __uint_as_float(rr[j + 2]),
                        __uint_as_float(rr[j + 3]));
        }
      }
      tc_fence_before();
      __syncthreads();
    }
  }
  if (kTensor) {
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
      tc_fence_after();
      tmem_dealloc(tmem, 512);
    }
  }
}

template <int C, bool U16>
cudaError_t launch_c(const GdnIO& io, cudaStream_t stream) {
  using SM = GdnSmem<C>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e =
        cudaFuncSetAttribute(gdn_inverse_kernel<C, U16>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kTotal);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t grid = io.n_chunks < sms ? io.n_chunks : sms;
  gdn_inverse_kernel<C, U16><<<static_cast<unsigned>(grid), kThreads, SM::kTotal, stream>>>(io);
  return cudaGetLastError();
}

template <bool U16>
cudaError_t launch_any(const GdnIO& io, int C, cudaStream_t stream) {
  switch (C) {
    case 32: return launch_c<32, U16>(io, stream);
    case 64: return launch_c<64, U16>(io, stream);
    case 128: return launch_c<128, U16>(io, stream);
    case 256: return launch_c<256, U16>(io, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_gdn_bf16(const void* A, float* T, int64_t n_chunks, int C, cudaStream_t stream) {
  if (C == 256 && gdn256_supported(A, T, n_chunks)) return launch_gdn256_bf16(A, T, n_chunks, stream);
  GdnIO io{A, T, n_chunks, 0, 0, 1.0f, 1.0f, nullptr};
  return launch_any<false>(io, C, stream);
}

cudaError_t launch_gdn_u16(const uint16_t* A, int64_t n_chunks, int C, int zpA, float sA, int zpT, float sT,
                           uint16_t* T, cudaStream_t stream) {
  if (C == 256 && gdn256_supported(A, T, n_chunks)) return launch_gdn256_u16(A, n_chunks, zpA, sA, zpT, sT, T, stream);
  GdnIO io{A, T, n_chunks, zpA, zpT, sA, 1.0f / sT, nullptr};
  return launch_any<true>(io, C, stream);
}

}  // namespace qhtp
