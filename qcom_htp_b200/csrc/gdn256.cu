// GDN / KDA chunk triangular inverse for C = 256 on B200:  T = (I - A)^-1 per chunk, A strictly
// lower triangular, bf16 in / f32 out (the u16 code carrier runs the same algorithm in gdn256x2.cu).
//
// Same algorithm family as the reference's block solvers (example/gdn_native/solve_op/
// gdn_solve_ref.c:19-69 forward substitution + block merge; solve_br_op block recursion): the
// chunk is inverted by recursive doubling on its block structure.  With L = I - A and
// T_b = inverse of the b x b diagonal block,
//     [[T00, 0], [T10, T11]],   T10 = T11 * (A10 * T00)                        (A10 = -L10)
//   level 0   the eight 32x32 diagonal blocks, forward substitution in fp32 on CUDA cores
//             (one warp per block, lane j owns column j);
//   level 1   32 -> 64,  four block pairs;     level 2   64 -> 128, two pairs;
//   level 3   128 -> 256, one pair;
// every level is two bf16 tcgen05 MMAs (X = A10 * T00, then T10 = T11 * X) with fp32 accumulators
// in TMEM.  Independent block pairs of one level share one M = 128 instruction: their A10 (or T11)
// rows are stacked along M and each pair's B operand goes to its own TMEM column range, so only the
// diagonal sub-blocks of each product are kept.
//
// Every matrix that feeds an MMA lives in shared memory in one form only: a row-major bf16 image
// with the 128-byte swizzle (row r at r*128 bytes, 16-byte chunk c at ((c ^ r) & 7)*16).  The same
// bytes are a K-major A operand (rows = M, K contiguous) and an MN-major B operand (rows = K, 64
// N-contiguous elements per row), which is exactly what T10 = T11 * (A10 * T00) needs: A10 and T11
// as A, T00 and X as B.  TMEM rows come back one per thread, so each product is written to its
// next image as whole swizzled rows.
//
// One persistent CTA (8 warps) per SM walks the chunks.  TMA loads bring the A tiles in (the next
// chunk's diagonal tiles are prefetched into a second buffer while the current chunk runs); the
// f32 output leaves through TMA stores of swizzled 32x32 staging tiles, and the strict upper
// triangle is stored from a zero tile.  Input entries on or above the diagonal are never read.
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

// Shared memory map (bytes from the 1024-aligned base).
constexpr uint32_t kAULBytes = 32 * KB;  // one diagonal-tile buffer: AU (16K) | AL (16K); two of them
constexpr uint32_t kAU = 0;              //   AU[q] (q=0..3, 4K each): A[64q + r][64q + c], r < 32
constexpr uint32_t kAL = 16 * KB;        //   AL[q]: A[64q + 32 + r][64q + c]; rows of the four q stack to M=128
constexpr uint32_t kA2 = 64 * KB;        // A2[h] (8K each): A[128h + 64 + r][128h + c], r < 64
constexpr uint32_t kA3 = 80 * KB;        // A3 K-region g (16K each): A[128 + r][64g + c], r < 128
constexpr uint32_t kRS0 = 112 * KB;      // 64x64 row images of the level-1 results T_q (8K each) ...
constexpr uint32_t kL2R0 = 120 * KB;     // ... and of the level-2 off-diagonal blocks, ordered so that
constexpr uint32_t kRS2 = 128 * KB;      //     [RS1; RS3], [RS2; L2R1] and [0; RS3] are M=128 operands
constexpr uint32_t kL2R1 = 136 * KB;
constexpr uint32_t kRS1 = 144 * KB;
constexpr uint32_t kRS3 = 152 * KB;
constexpr uint32_t kZero = 160 * KB;     // 32x32 zero tile of the output type (upper-triangle stores)
constexpr uint32_t kBar = 164 * KB;
constexpr uint32_t kSmemBytes = kBar + 64 + 1024;  // barriers + alignment slack

__device__ __forceinline__ uint32_t rs_off(int q) {
  return q == 0 ? kRS0 : (q == 1 ? kRS1 : (q == 2 ? kRS2 : kRS3));
}

template <bool U16>
__global__ void __launch_bounds__(kThreads, 1)
    gdn256_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmT,
                  const Gdn256Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(sm);
  uint64_t* ld_bar = reinterpret_cast<uint64_t*>(sm + kBar);  // [2] diagonal-tile buffers
  uint64_t* ld23_bar = ld_bar + 2;                           // A2 + A3
  uint64_t* mma_bar = ld_bar + 3;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(ld_bar + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, half = warp >> 2;  // TMEM lane quadrant, column half
  int* err = args.err;
  void* T = args.T;
  const InCodes ic = args.ic;
  const OutCodes oc = args.oc;
  const int64_t n_chunks = args.n_chunks;

  if (tid == 0) {
    mbar_init(&ld_bar[0], 1);
    mbar_init(&ld_bar[1], 1);
    mbar_init(ld23_bar, 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmT);
  }
  for (int e = tid; e < static_cast<int>(kTile / 16); e += kThreads)
    if constexpr (U16) {
      const uint32_t z = to_code(0.0f, oc) * 0x10001u;
      reinterpret_cast<uint4*>(sm + kZero)[e] = make_uint4(z, z, z, z);
    } else {
      reinterpret_cast<uint4*>(sm + kZero)[e] = make_uint4(0u, 0u, 0u, 0u);
    }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  // Load issue (thread 0 only).  pend*: loads issued and not yet observed complete, with the parity
  // of the phase they complete, so an early exit can wait for them before shared memory goes away.
  bool pend[2] = {false, false}, pend23 = false;
  uint32_t pend_par[2] = {0u, 0u}, pend23_par = 0u;
  auto issue_diag = [&](int buf, int64_t ch, uint32_t parity) {
    uint64_t* bar = &ld_bar[buf];
    mbar_arrive_expect_tx(bar, kAULBytes);
    const int y0 = static_cast<int>(ch * kC);
    uint8_t* base = sm + buf * kAULBytes;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      tma_load_2d(base + kAU + q * kTile, &tmA, bar, 64 * q, y0 + 64 * q);
      tma_load_2d(base + kAL + q * kTile, &tmA, bar, 64 * q, y0 + 64 * q + 32);
    }
    pend[buf] = true;
    pend_par[buf] = parity;
  };
  auto issue_a23 = [&](int64_t ch, uint32_t parity) {
    mbar_arrive_expect_tx(ld23_bar, 48 * KB);
    const int y0 = static_cast<int>(ch * kC);
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int j = 0; j < 2; ++j) tma_load_2d(sm + kA2 + h * 8 * KB + j * kTile, &tmA, ld23_bar, 128 * h, y0 + 128 * h + 64 + 32 * j);
#pragma unroll
    for (int g = 0; g < 2; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j) tma_load_2d(sm + kA3 + g * 16 * KB + j * kTile, &tmA, ld23_bar, 64 * g, y0 + 128 + 32 * j);
    pend23 = true;
    pend23_par = parity;
  };

  const uint32_t id64 = idesc_bf16(128, 64, 1), id128 = idesc_bf16(128, 128, 1);
  uint32_t mma_par = 0;
  bool failed = false;
  if (tid == 0 && static_cast<int64_t>(blockIdx.x) < n_chunks) issue_diag(0, blockIdx.x, 0u);

  int it = 0;
  for (int64_t ch = blockIdx.x; ch < n_chunks; ch += gridDim.x, ++it) {
    const int buf = it & 1;
    uint8_t* aul = sm + buf * kAULBytes;
    const uint32_t aul_s = sb + buf * kAULBytes;
    const int y0 = static_cast<int>(ch * kC);

    // ---- S0: the previous chunk's staging tiles have been read by their stores; every generic access
    // to the buffers refilled below is ordered before the refill.
    if (lane == 0) bulk_wait_read_all();
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      issue_a23(ch, it & 1);
      const int64_t nx = ch + gridDim.x;
      if (nx < n_chunks) issue_diag(buf ^ 1, nx, ((it + 1) >> 1) & 1);
    }

    // ---- S1: level 0, warp w inverts diagonal block w (rows/columns 32w..32w+31)
    bool ok = mbar_wait(&ld_bar[buf], (it >> 1) & 1, err, kErrTimeoutFull);
    if (ok) {
      const int q = warp >> 1, odd = warp & 1;
      const uint8_t* src = aul + (odd ? kAL : kAU) + q * kTile;
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
        uint8_t* al = aul + kAL + q * kTile;
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
          uint8_t* al = aul + kAL + q * kTile;
#pragma unroll
          for (int m = 0; m < 4; ++m) codes_to_bf16(al + swz(8 * m + (lane >> 2), lane & 3), ic);
        }
      }
    }
    if (tid == 0 && ok) pend[buf] = false;
    fence_proxy_async_smem();
    tc_fence_before();
    failed = __syncthreads_or(ok ? 0 : 1) != 0;
    if (failed) break;

    // ---- S2: level 1, X_q = A10_q * T_{2q}   (A: AL rows, K 0..31; B: RS_q rows 0..31, MN-major)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int s = 0; s < 2; ++s)
          mma_k16(tmem + 64 * q, aul_s + kAL + 32 * s, sb + rs_off(q) + 2048 * s, 8 * KB, id64, s);
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
      put_row_bf16(aul + kAU + warp * kTile, lane, 0, v);
    } else if constexpr (U16) {
      // warps 4..7 are free here: the level-2 and level-3 A operands (A2 16 KB, A3 32 KB), u16 codes
      // -> bf16 in place, once their loads have landed
      if (ok) ok = mbar_wait(ld23_bar, it & 1, err, kErrTimeoutFull);
      if (ok)
        for (int e = tid - 128; e < static_cast<int>(48 * KB / 16); e += 128) codes_to_bf16(sm + kA2 + 16 * e, ic);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    failed = __syncthreads_or(ok ? 0 : 1) != 0;
    if (failed) break;

    // ---- S4: level 1, T10_q = T_{2q+1} * X_q   (A: AL rows, K 32..63; B: XB1[q], MN-major)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int s = 0; s < 2; ++s)
          mma_k16(tmem + 64 * q, aul_s + kAL + 64 + 32 * s, aul_s + kAU + q * kTile + 2048 * s, 8 * KB, id64, s);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_par, err, kErrTimeoutAccum);
    mma_par ^= 1u;
    tc_fence_after();
    // ---- S5: T10_q -> rows 32..63, columns 0..31 of RS_q, and f32 out (rows 64q+32.., columns 64q..);
    // warps 4..7 store the chunk's upper-triangle zero boxes.
    if (ok && warp < 4) {
      uint32_t v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + 64 * warp, v);
      tmem_ld_wait();
      put_row_bf16(sm + rs_off(warp), 32 + lane, 0, v);
      uint8_t* st = aul + kAU + warp * kTile;  // XB1[q] is dead: the second product has completed
      put_row_out<U16>(st, lane, v, oc);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&tmT, st, 64 * warp, y0 + 64 * warp + 32);
        bulk_commit();
      }
    } else if (ok && lane == 0) {
      for (int e = warp - 4; e < 28; e += 4) {
        int x, y;
        zero_box(e, x, y);
        tma_store_2d(&tmT, sm + kZero, x, y0 + y);
      }
      bulk_commit();
    }
    if (ok) ok = mbar_wait(ld23_bar, it & 1, err, kErrTimeoutFull);
    if (tid == 0 && ok) pend23 = false;

    fence_proxy_async_smem();
    tc_fence_before();
    failed = __syncthreads_or(ok ? 0 : 1) != 0;
    if (failed) break;

    // ---- S6: level 2, X2_h = A10_h * T_{2h}   (A: A2, rows [h0; h1]; B: RS_{2h}, MN-major)
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
    // ---- S7: X2_h (TMEM lanes 64h.., columns 64h..) -> XB2[h] image in AL (64 rows each)
    const int h2 = qd >> 1, r2 = 32 * (qd & 1) + lane;
    if (ok) {
      uint32_t v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * qd) << 16) + 64 * h2 + 32 * half, v);
      tmem_ld_wait();
      put_row_bf16(aul + kAL + h2 * 8 * KB, r2, 4 * half, v);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    failed = __syncthreads_or(ok ? 0 : 1) != 0;
    if (failed) break;

    // ---- S8: level 2, T10_h = T_{2h+1} * X2_h   (A: [RS1; RS3]; B: XB2[h], MN-major)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int s = 0; s < 4; ++s)
          mma_k16(tmem + 64 * h, sb + kRS1 + 32 * s, aul_s + kAL + h * 8 * KB + 2048 * s, 8 * KB, id64, s);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_par, err, kErrTimeoutAccum);
    mma_par ^= 1u;
    tc_fence_after();
    // ---- S9: T10_h -> L2R_h image and f32 out (rows 128h+64.., columns 128h..)
    if (ok) {
      uint32_t v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * qd) << 16) + 64 * h2 + 32 * half, v);
      tmem_ld_wait();
      put_row_bf16(sm + (h2 ? kL2R1 : kL2R0), r2, 4 * half, v);
      uint8_t* st = warp < 4 ? aul + kAU + warp * kTile : sm + kA2 + (warp - 4) * kTile;
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
    fence_proxy_async_smem();
    tc_fence_before();
    failed = __syncthreads_or(ok ? 0 : 1) != 0;
    if (failed) break;

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
    // ---- S11: X3 -> XB3 image in A3 (two 64-column groups of 128 rows); RS1 -> zeros
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
    fence_proxy_async_smem();
    tc_fence_before();
    failed = __syncthreads_or(ok ? 0 : 1) != 0;
    if (failed) break;

    // ---- S12: level 3, T[128:256, 0:128] = T_hi * X3, T_hi = [[T_2, 0], [T10_1, T_3]]
    //   A K-region 0: [RS2; L2R1], K-region 1: [0; RS3];  B: XB3, MN-major, N = 128 (groups 16K apart)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_k16(tmem, sb + (s < 4 ? kRS2 : kRS1) + (s & 3) * 32, sb + kA3 + 2048 * s, 16 * KB, id128, s);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_par, err, kErrTimeoutAccum);
    mma_par ^= 1u;
    tc_fence_after();
    // ---- S13: f32 out (rows 128 + 32qd.., columns 64*half + 32j..)
    if (ok) {
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(32 * qd) << 16) + 64 * half + 32 * j, v);
        tmem_ld_wait();
        uint8_t* st = j == 0 ? (warp < 4 ? aul + kAU + warp * kTile : sm + kA2 + (warp - 4) * kTile)
                             : (warp < 4 ? aul + kAL + warp * kTile : sm + kRS0 + (warp - 4) * kTile);
        put_row_out<U16>(st, lane, v, oc);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tma_store_2d(&tmT, st, 64 * half + 32 * j, y0 + 128 + 32 * qd);
      }
      if (lane == 0) bulk_commit();
    }
    failed = !ok;
    if (__syncthreads_or(failed ? 1 : 0)) {
      failed = true;
      break;
    }
  }

  // Drain: stores complete, outstanding loads land (bounded), TMEM released.
  if (lane == 0) bulk_wait_all();
  if (tid == 0) {
    for (int b = 0; b < 2; ++b)
      if (pend[b]) mbar_wait(&ld_bar[b], pend_par[b], err, kErrTimeoutOther);
    if (pend23) mbar_wait(ld23_bar, pend23_par, err, kErrTimeoutOther);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

__device__ int g_gdn256_err;

}  // namespace

bool gdn256_supported(const void* A, const void* T, int64_t n_chunks) {
  // TMA: 16-byte aligned bases; row coordinates (chunk * 256 + 255) must fit in int32.
  return (reinterpret_cast<uintptr_t>(A) & 15u) == 0 && (reinterpret_cast<uintptr_t>(T) & 15u) == 0 &&
         n_chunks > 0 && n_chunks <= (int64_t{1} << 23) - 1;
}

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
      e = cudaGetSymbolAddress(&p, g_gdn256_err);
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
  const int64_t grid = n_chunks < sms[dev] ? n_chunks : sms[dev];
  Gdn256Args args{T, ic, oc, n_chunks, err_ptr[dev]};
  gdn256_kernel<U16><<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(ta, tt, args);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gdn256_bf16(const void* A, float* T, int64_t n_chunks, cudaStream_t stream) {
  return launch_gdn256<false>(A, T, n_chunks, InCodes{1.0f, 0}, OutCodes{1.0f, 0.0f}, stream);
}


}  // namespace qhtp
