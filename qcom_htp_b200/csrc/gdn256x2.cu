// GDN / KDA chunk inverse, C = 256, the u16 code carrier of GdnSolve / gdnbm_solve (value =
// (code - zp) * scale, example/gdn_native/solve_op/src/GdnSolveOp.cpp:195-281, gdnbm.idl:10-12): the
// same recursive-doubling algorithm and operand images as gdn256.cu, laid out for two CTAs per SM.
//
// The code conversions (codes -> fp32 in the substitutions, -> bf16 for the MMA inputs, fp32 -> codes
// for every output element) lengthen each chunk's chain of dependent steps; with two chunks in flight
// per SM one CTA's conversions, MMA round trips and TMEM drains overlap the other's.  That takes the
// shared memory down to 112 KB per CTA (no second buffer for the next chunk's tiles: they load during
// the level-3 products into the buffers the level-2 stores have released; A2 shares the 32 KB A3
// region and A3's second K-region loads over it after the level-2 first product) and 128 registers.
// The upper triangle is written as zero-point codes with coalesced stores while the last product runs.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "gdn_common.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace qhtp {

namespace {

using namespace gdn;

// Shared memory map (bytes from the 1024-aligned base), sized for two CTAs per SM: each SM keeps two
// chunks in flight, so one CTA's MMA round trips, TMEM drains and loads overlap the other's work.
constexpr uint32_t kAU = 0;          // AU[q] (q=0..3, 4K each): A[64q + r][64q + c], r < 32
constexpr uint32_t kAL = 16 * KB;    // AL[q]: A[64q + 32 + r][64q + c]; rows of the four q stack to M=128
constexpr uint32_t kA3 = 32 * KB;    // A3 K-region g (16K each): A[128 + r][64g + c], r < 128; region 1
constexpr uint32_t kA2 = 48 * KB;    //   first holds A2[h] (8K each): A[128h + 64 + r][128h + c], r < 64
constexpr uint32_t kRS0 = 64 * KB;   // 64x64 row images of the level-1 results T_q (8K each) and of the
constexpr uint32_t kRS1 = 72 * KB;   // level-2 off-diagonal blocks, ordered so that [RS1; RS3],
constexpr uint32_t kRS3 = 80 * KB;   // [RS2; L2R1] and [0; RS3] are M=128 operands
constexpr uint32_t kRS2 = 88 * KB;
constexpr uint32_t kL2R1 = 96 * KB;
constexpr uint32_t kL2R0 = 104 * KB;
constexpr uint32_t kBar = 112 * KB;
constexpr uint32_t kNeed = kBar + 64;     // bytes used above the 1024-aligned base
constexpr uint32_t kSmemBytes = 115712;   // (228 KB per SM - 2 x 1 KB reserved) / 2 CTAs
static_assert(kNeed + 896 <= kSmemBytes, "aligning a 128-byte-aligned base must fit");

__device__ __forceinline__ uint32_t rs_off(int q) {
  return q == 0 ? kRS0 : (q == 1 ? kRS1 : (q == 2 ? kRS2 : kRS3));
}

template <bool U16>
__global__ void __launch_bounds__(kThreads, 2)
    gdn256_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmT,
                  const Gdn256Args args) {
  extern __shared__ uint8_t smem_raw[];
  const uintptr_t raw = reinterpret_cast<uintptr_t>(smem_raw);
  uint8_t* sm = reinterpret_cast<uint8_t*>((raw + 1023) & ~uintptr_t(1023));
  if (reinterpret_cast<uintptr_t>(sm) + kNeed > raw + kSmemBytes) {  // base alignment below 128 bytes
    if (threadIdx.x == 0) record_error(args.err, kErrTimeoutOther);
    return;
  }
  const uint32_t sb = smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kBar);
  uint64_t* ld_bar = bars;       // AU + AL (the diagonal tiles)
  uint64_t* a23_bar = bars + 1;  // A3 K-region 0 + A2
  uint64_t* a3_bar = bars + 2;   // A3 K-region 1 (loaded over A2 once the level-2 first product is done)
  uint64_t* mma_bar = bars + 3;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, half = warp >> 2;  // TMEM lane quadrant, column half
  int* err = args.err;
  void* T = args.T;
  const InCodes ic = args.ic;
  const OutCodes oc = args.oc;
  const int64_t n_chunks = args.n_chunks;
  const uint32_t zword = U16 ? to_code(0.0f, oc) * 0x10001u : 0u;

  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmT);
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  // Loads (thread 0).  pend*: issued and not yet observed complete (an early exit waits for them
  // before shared memory goes away); every barrier completes once per chunk, parity it & 1.
  bool pend_d = false, pend_23 = false, pend_3 = false;
  uint32_t par_d = 0, par_23 = 0, par_3 = 0;
  const uint32_t id64 = idesc_bf16(128, 64, 1), id128 = idesc_bf16(128, 128, 1);
  uint32_t mma_par = 0;
  bool ok = true;

  // diagonal tiles of chunk `c` into AU / AL (thread 0); parity `p` of their ld_bar phase
  auto issue_diag = [&](int64_t c, uint32_t p) {
    const int yc = static_cast<int>(c * kC);
    mbar_arrive_expect_tx(ld_bar, 32 * KB);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      tma_load_2d(sm + kAU + q * kTile, &tmA, ld_bar, 64 * q, yc + 64 * q);
      tma_load_2d(sm + kAL + q * kTile, &tmA, ld_bar, 64 * q, yc + 64 * q + 32);
    }
    pend_d = true;
    par_d = p;
  };
  if (tid == 0 && static_cast<int64_t>(blockIdx.x) < n_chunks) issue_diag(blockIdx.x, 0u);

  int it = 0;
  for (int64_t ch = blockIdx.x; ch < n_chunks; ch += gridDim.x, ++it) {
    const uint32_t par = static_cast<uint32_t>(it) & 1u;
    const int y0 = static_cast<int>(ch * kC);

    // ---- S0: the previous chunk's staged stores have read their tiles; every generic access to
    // the buffers refilled below is ordered before the refill.
    if (lane == 0) bulk_wait_read_all();
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      mbar_arrive_expect_tx(a23_bar, 32 * KB);
#pragma unroll
      for (int j = 0; j < 4; ++j) tma_load_2d(sm + kA3 + j * kTile, &tmA, a23_bar, 0, y0 + 128 + 32 * j);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < 2; ++j)
          tma_load_2d(sm + kA2 + h * 8 * KB + j * kTile, &tmA, a23_bar, 128 * h, y0 + 128 * h + 64 + 32 * j);
      pend_23 = true;
      par_23 = par;
    }

    // ---- S1: level 0, warp w inverts diagonal block w (rows/columns 32w..32w+31)
    ok = mbar_wait(ld_bar, par, err, kErrTimeoutFull);
    if (ok) {
      const int q = warp >> 1, odd = warp & 1;
      const uint8_t* src = sm + (odd ? kAL : kAU) + q * kTile;
      float t[32];
      solve_diag32<U16>(src, odd * 4, lane, t, ic);
      __syncwarp();  // all lanes are done reading `src` before odd blocks overwrite it below
      // result rows (coalesced: lane j writes column 32w + j of row 32w + i)
      const int64_t o0 = static_cast<int64_t>(y0 + 32 * warp) * kC + 32 * warp + lane;
      if constexpr (U16) {
        uint16_t* out = static_cast<uint16_t*>(T) + o0;
#pragma unroll
        for (int i = 0; i < 32; ++i) out[static_cast<int64_t>(i) * kC] = static_cast<uint16_t>(to_code(t[i], oc));
      } else {
        float* out = static_cast<float*>(T) + o0;
#pragma unroll
        for (int i = 0; i < 32; ++i) out[static_cast<int64_t>(i) * kC] = t[i];
      }
      // bf16 row image of the 64x64 block T_q: this block at rows/columns 32*odd..
      uint8_t* rs = sm + rs_off(q);
      const int cc = 32 * odd + lane;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int r = 32 * odd + i;
        *reinterpret_cast<__nv_bfloat16*>(rs + swz(r, cc >> 3) + (cc & 7) * 2) = __float2bfloat16_rn(t[i]);
      }
      if (odd) {
        // T_{2q+1} rows also go to columns 32..63 of AL[q], making AL the stacked A operand
        // [T_1; T_3; T_5; T_7] of the level-1 second product (columns 0..31 still hold A10).
        uint8_t* al = sm + kAL + q * kTile;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          *reinterpret_cast<__nv_bfloat16*>(al + swz(i, cc >> 3) + (cc & 7) * 2) = __float2bfloat16_rn(t[i]);
      } else {
        // the zero upper-right 32x32 of T_q (rows 0..31, columns 32..63)
#pragma unroll
        for (int m = 0; m < 4; ++m)
          *reinterpret_cast<uint4*>(rs + swz(8 * m + (lane >> 2), 4 + (lane & 3))) = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (U16) {
          // A10_q (columns 0..31 of AL[q]) feeds the level-1 MMA: codes -> bf16 in place
          uint8_t* al = sm + kAL + q * kTile;
#pragma unroll
          for (int m = 0; m < 4; ++m) codes_to_bf16(al + swz(8 * m + (lane >> 2), lane & 3), ic);
        }
      }
    }
    if (tid == 0 && ok) pend_d = false;
    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(ok ? 0 : 1)) break;

    // ---- S2: level 1, X_q = A10_q * T_{2q}   (A: AL rows, K 0..31; B: RS_q rows 0..31, MN-major)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int s = 0; s < 2; ++s)
          mma_k16(tmem + 64 * q, sb + kAL + 32 * s, sb + rs_off(q) + 2048 * s, 8 * KB, id64, s);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_par, err, kErrTimeoutAccum);
    mma_par ^= 1u;
    tc_fence_after();
    // ---- S3: X_q (TMEM lanes 32q.., columns 64q..64q+31) -> XB1[q] image in AU[q] (rows k = 0..31)
    if (ok && warp < 4) {
      uint32_t v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + 64 * warp, v);
      tmem_ld_wait();
      put_row_bf16(sm + kAU + warp * kTile, lane, 0, v);
    } else if constexpr (U16) {
      // warps 4..7 are free here: A3 K-region 0 and A2, u16 codes -> bf16 in place, once landed
      if (ok) ok = mbar_wait(a23_bar, par, err, kErrTimeoutFull);
      if (ok)
        for (int e = tid - 128; e < static_cast<int>(32 * KB / 16); e += 128) codes_to_bf16(sm + kA3 + 16 * e, ic);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(ok ? 0 : 1)) break;

    // ---- S4: level 1, T10_q = T_{2q+1} * X_q   (A: AL rows, K 32..63; B: XB1[q], MN-major)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int s = 0; s < 2; ++s)
          mma_k16(tmem + 64 * q, sb + kAL + 64 + 32 * s, sb + kAU + q * kTile + 2048 * s, 8 * KB, id64, s);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_par, err, kErrTimeoutAccum);
    mma_par ^= 1u;
    tc_fence_after();
    // ---- S5: T10_q -> rows 32..63, columns 0..31 of RS_q, and out (rows 64q+32.., columns 64q..);
    // warps 4..7 store the chunk's upper-triangle zeros.
    if (ok && warp < 4) {
      uint32_t v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + 64 * warp, v);
      tmem_ld_wait();
      put_row_bf16(sm + rs_off(warp), 32 + lane, 0, v);
      uint8_t* st = sm + kAU + warp * kTile;  // XB1[q] is dead: the second product has completed
      put_row_out<U16>(st, lane, v, oc);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&tmT, st, 64 * warp, y0 + 64 * warp + 32);
        bulk_commit();
      }
    }
    if (ok) ok = mbar_wait(a23_bar, par, err, kErrTimeoutFull);
    if (tid == 0 && ok) pend_23 = false;
    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(ok ? 0 : 1)) break;

    // ---- S6: level 2, X2_h = A10_h * T_{2h}   (A: A2, rows [h0; h1]; B: RS_{2h}, MN-major); then
    // A3 K-region 1 loads over A2
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int s = 0; s < 4; ++s) mma_k16(tmem + 64 * h, sb + kA2 + 32 * s, sb + rs_off(2 * h) + 2048 * s, 8 * KB, id64, s);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_par, err, kErrTimeoutAccum);
    mma_par ^= 1u;
    tc_fence_after();
    if (tid == 0 && ok) {
      mbar_arrive_expect_tx(a3_bar, 16 * KB);
#pragma unroll
      for (int j = 0; j < 4; ++j) tma_load_2d(sm + kA2 + j * kTile, &tmA, a3_bar, 64, y0 + 128 + 32 * j);
      pend_3 = true;
      par_3 = par;
    }
    // ---- S7: X2_h (TMEM lanes 64h.., columns 64h..) -> XB2[h] image in AL (64 rows each)
    const int h2 = qd >> 1, r2 = 32 * (qd & 1) + lane;
    if (ok) {
      uint32_t v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * qd) << 16) + 64 * h2 + 32 * half, v);
      tmem_ld_wait();
      put_row_bf16(sm + kAL + h2 * 8 * KB, r2, 4 * half, v);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(ok ? 0 : 1)) break;

    // ---- S8: level 2, T10_h = T_{2h+1} * X2_h   (A: [RS1; RS3]; B: XB2[h], MN-major)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int s = 0; s < 4; ++s)
          mma_k16(tmem + 64 * h, sb + kRS1 + 32 * s, sb + kAL + h * 8 * KB + 2048 * s, 8 * KB, id64, s);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_par, err, kErrTimeoutAccum);
    mma_par ^= 1u;
    tc_fence_after();
    // ---- S9: T10_h -> L2R_h image and out (rows 128h+64.., columns 128h..), staged in AU (warps
    // 0..3, after their S5 tiles were read) or AL (warps 4..7: XB2 is dead); A3 K-region 1 landed
    if (ok) {
      uint32_t v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * qd) << 16) + 64 * h2 + 32 * half, v);
      tmem_ld_wait();
      put_row_bf16(sm + (h2 ? kL2R1 : kL2R0), r2, 4 * half, v);
      uint8_t* st = warp < 4 ? sm + kAU + warp * kTile : sm + kAL + (warp - 4) * kTile;
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
      put_row_out<U16>(st, lane, v, oc);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&tmT, st, 128 * h2 + 32 * half, y0 + 128 * h2 + 64 + 32 * (qd & 1));
        bulk_commit();
      }
    }
    if (ok) ok = mbar_wait(a3_bar, par, err, kErrTimeoutFull);
    if (tid == 0 && ok) pend_3 = false;
    if constexpr (U16) {
      if (ok)
        for (int e = tid; e < static_cast<int>(16 * KB / 16); e += kThreads) codes_to_bf16(sm + kA2 + 16 * e, ic);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(ok ? 0 : 1)) break;

    // ---- S10: level 3, X3 = A3 * T_lo, T_lo = [[T_0, 0], [T10_0, T_1]]
    //   columns 0..63:   K rows 0..63 from RS0, 64..127 from L2R0;   columns 64..127: K rows 64..127 from RS1
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_k16(tmem, sb + kA3 + (s >> 2) * 16 * KB + (s & 3) * 32,
                sb + (s < 4 ? kRS0 + 2048 * s : kL2R0 + 2048 * (s - 4)), 8 * KB, id64, s);
#pragma unroll
      for (int s = 4; s < 8; ++s)
        mma_k16(tmem + 64, sb + kA3 + 16 * KB + (s & 3) * 32, sb + kRS1 + 2048 * (s - 4), 8 * KB, id64, s - 4);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_par, err, kErrTimeoutAccum);
    mma_par ^= 1u;
    tc_fence_after();
    // ---- S11: X3 -> XB3 image over A3 (two 64-column groups of 128 rows); RS1 -> zeros.  After the
    // issuing lanes' wait here, every staging tile written in S5 and S9 has been read.
    if (ok) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(32 * qd) << 16) + 64 * half + 32 * j, v);
        tmem_ld_wait();
        put_row_bf16(sm + kA3 + half * 16 * KB, 32 * qd + lane, 4 * j, v);
      }
      reinterpret_cast<uint4*>(sm + kRS1)[2 * tid] = make_uint4(0u, 0u, 0u, 0u);
      reinterpret_cast<uint4*>(sm + kRS1)[2 * tid + 1] = make_uint4(0u, 0u, 0u, 0u);
    }
    if (lane == 0) bulk_wait_read_all();
    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(ok ? 0 : 1)) break;

    // ---- S12: level 3, T[128:256, 0:128] = T_hi * X3, T_hi = [[T_2, 0], [T10_1, T_3]]
    //   A K-region 0: [RS2; L2R1], K-region 1: [0; RS3];  B: XB3, MN-major, N = 128 (groups 16K apart)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_k16(tmem, sb + (s < 4 ? kRS2 : kRS1) + (s & 3) * 32, sb + kA3 + 2048 * s, 16 * KB, id128, s);
      mma_commit(mma_bar);
      // AU / AL are free (their S9 staging tiles were read): the next chunk's diagonal tiles load now
      const int64_t nx = ch + gridDim.x;
      if (nx < n_chunks) issue_diag(nx, par ^ 1u);
    }
    // while the product runs, warps 4..7 store the chunk's strict upper triangle: f32 zeros straight
    // from RS1 (all zero since S11, 4 KB per 32x32 box), u16 zero-point codes with coalesced stores
    if (warp >= 4) {
      if constexpr (U16) {
        store_zeros<U16>(T, y0, warp - 4, lane, zword);
      } else if (lane == 0) {
        for (int e = warp - 4; e < 28; e += 4) {
          int x, y;
          zero_box(e, x, y);
          tma_store_2d(&tmT, sm + kRS1, x, y0 + y);
        }
        bulk_commit();
      }
    }
    ok = mbar_wait(mma_bar, mma_par, err, kErrTimeoutAccum);
    mma_par ^= 1u;
    tc_fence_after();
    // ---- S13: out (rows 128 + 32qd.., columns 64*half + 32j..), staged over A3 (XB3 is dead) and
    // the level-1/2 images (RS0..RS2, dead once the last product has completed); AU / AL already
    // hold the next chunk's diagonal tiles
    if (ok) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(32 * qd) << 16) + 64 * half + 32 * j, v);
        tmem_ld_wait();
        // j = 1 slots: RS0, L2R1 / L2R0, RS3, RS2 (dead after S12), never RS1 -- the zero-box stores
        // of S12 may still be reading it
        constexpr uint32_t kSlot1[8] = {kRS0, kRS0 + kTile, kL2R1, kL2R1 + kTile, kRS3, kRS3 + kTile, kRS2,
                                        kRS2 + kTile};
        uint8_t* st = j == 0 ? sm + kA3 + warp * kTile : sm + kSlot1[warp];
        put_row_out<U16>(st, lane, v, oc);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tma_store_2d(&tmT, st, 64 * half + 32 * j, y0 + 128 + 32 * qd);
      }
      if (lane == 0) bulk_commit();
    }
    tc_fence_before();
    if (__syncthreads_or(ok ? 0 : 1)) break;
  }

  // Drain: stores complete, outstanding loads land (bounded), TMEM released.
  if (lane == 0) bulk_wait_all();
  if (tid == 0) {
    if (pend_d) mbar_wait(ld_bar, par_d, err, kErrTimeoutOther);
    if (pend_23) mbar_wait(a23_bar, par_23, err, kErrTimeoutOther);
    if (pend_3) mbar_wait(a3_bar, par_3, err, kErrTimeoutOther);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

__device__ int g_gdn256x2_err;

}  // namespace

namespace {

template <bool U16>
cudaError_t launch_gdn256(const void* A, void* T, int64_t n_chunks, InCodes ic, OutCodes oc, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  static int attr_set[64] = {0};
  static int sms[64] = {0};
  static int* err_ptr[64] = {nullptr};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      e = cudaFuncSetAttribute(gdn256_kernel<U16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess) return e;
      e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return e;
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_gdn256x2_err);
      if (e != cudaSuccess) return e;
      err_ptr[dev] = static_cast<int*>(p);
      attr_set[dev] = 1;
    }
  }
  CUtensorMap ta, tt;
  const uint64_t rows = static_cast<uint64_t>(n_chunks) * kC;
  const CUtensorMapDataType at = U16 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (!make_tmap_2d(&ta, at, A, kC, rows, kC * 2, 64, 32)) return cudaErrorInvalidValue;
  const bool okT = U16 ? make_tmap_2d(&tt, CU_TENSOR_MAP_DATA_TYPE_UINT16, T, kC, rows, kC * 2, 32, 32,
                                      CU_TENSOR_MAP_SWIZZLE_64B)
                       : make_tmap_2d(&tt, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, T, kC, rows, kC * 4, 32, 32);
  if (!okT) return cudaErrorInvalidValue;
  const int64_t grid = n_chunks < 2 * sms[dev] ? n_chunks : 2 * sms[dev];  // two CTAs per SM
  Gdn256Args args{T, ic, oc, n_chunks, err_ptr[dev]};
  gdn256_kernel<U16><<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(ta, tt, args);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gdn256_u16(const uint16_t* A, int64_t n_chunks, int zpA, float sA, int zpT, float sT, uint16_t* T,
                              cudaStream_t stream) {
  return launch_gdn256<true>(A, T, n_chunks, InCodes{sA, zpA}, OutCodes{1.0f / sT, static_cast<float>(zpT)}, stream);
}

}  // namespace qhtp
