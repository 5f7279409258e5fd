// Fused GDN chunk A-construction + triangular inverse for C = 256, Dk = 128 on B200: from the raw
// gated-delta-rule inputs of a chunk -- keys k (bf16 [C, Dk]), beta and per-token log gates (f32 [C])
// -- to T = (I - A)^-1 (f32 [C, C]) in one pass, A never leaving the SM.
//
// A is built as the reference's chunk kernel builds it (Stage A of gdn_chunk,
// scripts/gdn_ref_kernel.py:66-82): k L2-normalised, g = cumsum of the log gates over the chunk,
//     A[i][j] = -beta_i * (k_i . k_j) / (|k_i| |k_j|) * exp(g_i - g_j)     for i > j, else 0.
// The Gram matrix k k^T of the raw keys comes from two bf16 tcgen05 MMAs with both operands the
// same K-major swizzled image of k (rows 0..127 x columns 0..127, and rows 128..255 x all 256
// columns -- the strictly-lower blocks the inverse needs); the epilogue scales each entry by the
// row and column inverse norms, beta_i and the decay, rounds to bf16 and writes the swizzled A
// images the inverse reads (the A tiles gdn256.cu loads from HBM).  The inverse itself is
// gdn256.cu's recursive doubling, unchanged (see there).
//
// HBM per chunk: k 64 KB + beta, g 2 KB in, T 256 KB out, against 80 KB of A tiles read by the
// inverse alone -- and the 128 KB A write + read of a separate construction kernel are gone.  k is
// needed only by the Gram MMAs, so one k buffer suffices: the next chunk's k loads as soon as they
// complete.
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
constexpr uint32_t kK = 0;               // k: two K-major swizzled images (Dk 0..63, 64..127), 256 rows, 32K each
constexpr uint32_t kRN = 64 * KB;        // 1 / |k_i| (f32 [256])
constexpr uint32_t kGC = 65 * KB;        // g_i * log2(e), g = cumsum of the log gates (f32 [256])
constexpr uint32_t kBE = 66 * KB;        // beta_i (f32 [256]), copied out of the load area
constexpr uint32_t kBGL = 67 * KB;       // load area: beta (1K) | log gates (1K) of the chunk
constexpr uint32_t kAUL = 70 * KB;       // diagonal-tile images: AU (16K) | AL (16K)
constexpr uint32_t kAU = 0;              //   AU[q] (q=0..3, 4K each): A[64q + r][64q + c], r < 32
constexpr uint32_t kAL = 16 * KB;        //   AL[q]: A[64q + 32 + r][64q + c]; rows of the four q stack to M=128
constexpr uint32_t kA2 = 102 * KB;       // A2[h] (8K each): A[128h + 64 + r][128h + c], r < 64
constexpr uint32_t kA3 = 118 * KB;       // A3 K-region g (16K each): A[128 + r][64g + c], r < 128
constexpr uint32_t kRS0 = 150 * KB;      // 64x64 row images of the level-1 results T_q (8K each) ...
constexpr uint32_t kL2R0 = 158 * KB;     // ... and of the level-2 off-diagonal blocks, ordered so that
constexpr uint32_t kRS2 = 166 * KB;      //     [RS1; RS3], [RS2; L2R1] and [0; RS3] are M=128 operands
constexpr uint32_t kL2R1 = 174 * KB;
constexpr uint32_t kRS1 = 182 * KB;
constexpr uint32_t kRS3 = 190 * KB;
constexpr uint32_t kZero = 198 * KB;     // 32x32 zero tile (upper-triangle stores)
constexpr uint32_t kBar = 202 * KB;
constexpr uint32_t kSmemBytes = kBar + 64 + 1024;  // barriers + alignment slack
constexpr uint32_t kKBytes = 64 * KB + 2 * KB;     // one chunk's k, beta, log gates

__device__ __forceinline__ uint32_t rs_off(int q) {
  return q == 0 ? kRS0 : (q == 1 ? kRS1 : (q == 2 ? kRS2 : kRS3));
}

struct GdnKbgArgs {
  float* T;
  const float* beta;   // [n_chunks, 256]
  const float* g;      // [n_chunks, 256] per-token log gates
  int64_t n_chunks;
  int* err;
};

// 2^x by the SFU's base-2 exponential, results below the normal range flushed to zero.
__device__ __forceinline__ float exp2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One 32-column group of the Gram matrix row i (TMEM) -> A[i][j0..j0+31] as bf16 into row r,
// columns c0..c0+31 of a swizzled image:  A = -beta_i / |k_i| * (k_i . k_j) / |k_j| * exp(g_i - g_j)
// below the diagonal, 0 on and above it; the decay is 2^(g2_i - g2_j) with g2 = g * log2(e), one SFU
// instruction per entry.  All lanes read the same column constants (broadcast).
template <bool DIAG>
__device__ __forceinline__ void build_a32(uint32_t taddr, int i, int j0, uint8_t* img, int r, int c0, float bi_rn,
                                          float gi, const float* rn, const float* gc) {
  uint32_t v[32];
  tmem_ld32(taddr, v);
  // the group's column constants: j0 is a multiple of 32, so 16-byte broadcast loads
  const float4* rn4 = reinterpret_cast<const float4*>(rn + j0);
  const float4* gc4 = reinterpret_cast<const float4*>(gc + j0);
  tmem_ld_wait();
#pragma unroll
  for (int e4 = 0; e4 < 8; ++e4) {
    const float4 rj = rn4[e4], gj = gc4[e4];
    const float rr[4] = {rj.x, rj.y, rj.z, rj.w}, gg[4] = {gj.x, gj.y, gj.z, gj.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = 4 * e4 + u;
      float a = -(bi_rn * rr[u]) * __uint_as_float(v[e]) * exp2_ftz(gi - gg[u]);
      if constexpr (DIAG) a = i > j0 + e ? a : 0.0f;  // the diagonal block: strictly lower part only
      v[e] = __float_as_uint(a);
    }
  }
  put_row_bf16(img, r, c0 >> 3, v);
}

// The k images hold the key rows in 32-row blocks ordered 0, 1, 2, 3, 7, 6, 5, 4: the Gram rows of
// TMEM lane quadrant q are then key blocks q (top half) and 7 - q (bottom half), whose
// below-diagonal work (q + 1 and 8 - q blocks of 32 columns) adds up to 9 blocks in every quadrant.
__host__ __device__ __forceinline__ int kb_of_image(int p) { return p < 4 ? p : 11 - p; }

// Where A's 32 x 32 block (key row block rb, key column block cb <= rb) goes: the image the inverse
// reads it from, the image row of its first row, and the image column of its first column.
//   rb, cb in the same 64-block q:   AU[q] (rb even) / AL[q] (rb odd), columns 32 * (cb - 2q)
//   rb, cb in the same 128-block h:  A2[h], rows 32 * (rb - 4h - 2), columns 32 * (cb - 4h)
//   otherwise (rb >= 4, cb <= 3):    A3 K-region cb / 2, rows 32 * (rb - 4), columns 32 * (cb % 2)
__device__ __forceinline__ uint32_t a_block_image(int rb, int cb, int& r0, int& c0) {
  if ((rb >> 1) == (cb >> 1)) {
    const int q = rb >> 1;
    r0 = 0;
    c0 = 32 * (cb - 2 * q);
    return kAUL + ((rb & 1) ? kAL : kAU) + q * kTile;
  }
  if ((rb >> 2) == (cb >> 2)) {
    const int h = rb >> 2;
    r0 = 32 * (rb - 4 * h - 2);
    c0 = 32 * (cb - 4 * h);
    return kA2 + h * 8 * KB;
  }
  r0 = 32 * (rb - 4);
  c0 = 32 * (cb & 1);
  return kA3 + (cb >> 1) * 16 * KB;
}

__global__ void __launch_bounds__(kThreads, 1)
    gdn256f_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmT,
                   const GdnKbgArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(sm);
  uint64_t* k_bar = reinterpret_cast<uint64_t*>(sm + kBar);  // k, beta, log gates of a chunk landed
  uint64_t* mma_bar = k_bar + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(k_bar + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, half = warp >> 2;  // TMEM lane quadrant, column half
  int* err = args.err;
  float* T = args.T;
  const OutCodes oc{1.0f, 0.0f};
  const int64_t n_chunks = args.n_chunks;
  uint8_t* aul = sm + kAUL;
  const uint32_t aul_s = sb + kAUL;
  float* rn = reinterpret_cast<float*>(sm + kRN);
  float* gc = reinterpret_cast<float*>(sm + kGC);
  float* be = reinterpret_cast<float*>(sm + kBE);

  if (tid == 0) {
    mbar_init(k_bar, 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmT);
  }
  for (int e = tid; e < static_cast<int>(kTile / 16); e += kThreads)
    reinterpret_cast<uint4*>(sm + kZero)[e] = make_uint4(0u, 0u, 0u, 0u);
  if (warp == 0) {
    tmem_alloc(tslot, 512);  // Gram matrix: columns 0..127 (rows 0..127) and 128..383 (rows 128..255)
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  // Load issue (thread 0 only).  pend: a load issued and not yet observed complete (with the parity of
  // the phase it completes), so an early exit can wait for it before shared memory goes away.
  bool pend = false;
  uint32_t pend_par = 0u;
  auto issue_kbg = [&](int64_t ch, uint32_t parity) {
    mbar_arrive_expect_tx(k_bar, kKBytes);
    const int y0 = static_cast<int>(ch * kC);
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int p = 0; p < 8; ++p)  // image block p holds key rows 32 * kb_of_image(p) ..
        tma_load_2d(sm + kK + h * 32 * KB + p * kTile, &tmK, k_bar, 64 * h, y0 + 32 * kb_of_image(p));
    bulk_load(sm + kBGL, args.beta + ch * kC, kC * 4, k_bar);
    bulk_load(sm + kBGL + KB, args.g + ch * kC, kC * 4, k_bar);
    pend = true;
    pend_par = parity;
  };

  const uint32_t id64 = idesc_bf16(128, 64, 1), id128 = idesc_bf16(128, 128, 1);
  const uint32_t idG1 = idesc_bf16(128, 128, 0), idG2 = idesc_bf16(128, 256, 0);  // Gram: K-major B
  uint32_t mma_par = 0;
  bool failed = false;
  if (tid == 0 && static_cast<int64_t>(blockIdx.x) < n_chunks) issue_kbg(blockIdx.x, 0u);

  int it = 0;
  for (int64_t ch = blockIdx.x; ch < n_chunks; ch += gridDim.x, ++it) {
    const int y0 = static_cast<int>(ch * kC);

    // ---- S0: the previous chunk's staging tiles have been read by their stores; every generic access
    // to the images rewritten below is ordered after that.
    if (lane == 0) bulk_wait_read_all();
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- B0: this chunk's k, beta and log gates have landed.  Warp 1 lane 0 issues the Gram MMAs
    // (both operands the K-major images of k); meanwhile every thread forms 1/|k| of its image row,
    // copies beta_i out of the load area, and warp 2 forms g = cumsum of the log gates (the MMAs are
    // issued from warp 1, so no warp carries more than one of these jobs besides its norms).
    bool ok = mbar_wait(k_bar, it & 1, err, kErrTimeoutFull);
    if (ok) {
      if (tid == 0) pend = false;
      if (tid == 32) {
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t dTop = desc_kmajor_sw128(sb + kK + h * 32 * KB) + 2 * kk;           // rows 0..127
            const uint64_t dBot = desc_kmajor_sw128(sb + kK + h * 32 * KB + 128 * 128) + 2 * kk;  // rows 128..255
            const uint32_t acc = (h | kk) ? 1u : 0u;
            mma_bf16(tmem, dTop, dTop, idG1, acc);         // rows 0..127 x columns 0..127
            mma_bf16(tmem + 128, dBot, dTop, idG2, acc);   // rows 128..255 x columns 0..255
          }
        mma_commit(mma_bar);
      }
      float ss = 0.0f;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 w = *reinterpret_cast<const uint4*>(sm + kK + h * 32 * KB + swz(tid, c));
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = __uint_as_float(ws[e] << 16), hi = __uint_as_float(ws[e] & 0xFFFF0000u);
            ss = fmaf(lo, lo, ss);
            ss = fmaf(hi, hi, ss);
          }
        }
      // the reference's l2norm: x / sqrt(sum x^2 + 1e-6); image row tid holds key row
      // 32 * kb_of_image(tid / 32) + tid % 32
      rn[32 * kb_of_image(tid >> 5) + (tid & 31)] = rsqrtf(ss + 1e-6f);
      be[tid] = reinterpret_cast<const float*>(sm + kBGL)[tid];
      if (warp == 2) {
        const float* gl = reinterpret_cast<const float*>(sm + kBGL + KB);
        float x[8], run = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          run += gl[8 * lane + e];
          x[e] = run;
        }
        float pre = run;  // inclusive scan of the lanes' totals
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float y = __shfl_up_sync(0xFFFFFFFFu, pre, off);
          if (lane >= off) pre += y;
        }
        constexpr float kLog2e = 1.4426950408889634f;
#pragma unroll
        for (int e = 0; e < 8; ++e) gc[8 * lane + e] = (pre - run + x[e]) * kLog2e;
      }
    }
    failed = __syncthreads_or(ok ? 0 : 1) != 0;  // also publishes rn, be, gc
    if (failed) break;
    ok = mbar_wait(mma_bar, mma_par, err, kErrTimeoutAccum);
    mma_par ^= 1u;
    tc_fence_after();
    // k is dead (its MMAs completed; every norm was read before the barrier): the next chunk loads now
    if (tid == 0 && ok) {
      const int64_t nx = ch + gridDim.x;
      if (nx < n_chunks) issue_kbg(nx, (it + 1) & 1);
    }

    // ---- B1: Gram rows -> the A images (AU / AL: the diagonal 64x64 blocks, A2: the level-2 blocks,
    // A3: rows 128..255 x columns 0..127).  Warp (qd, half) owns Gram rows 32qd + lane of each half.
    if (ok) {
      // Quadrant qd's 9 blocks of 32 Gram columns, alternately to its two warps: key row block qd
      // (TMEM columns = key columns 32 cb, cb = 0..qd), then key row block 7 - qd (TMEM column 128 +
      // image column of key block cb, cb = 0..7-qd).  Blocks wholly above the diagonal never occur.
      const uint32_t tl = tmem + (static_cast<uint32_t>(32 * qd) << 16);
#pragma unroll 1
      for (int idx = half; idx < 9; idx += 2) {
        const bool top = idx <= qd;
        const int rb = top ? qd : 7 - qd;
        const int cb = top ? idx : idx - qd - 1;
        const int icol = 32 * (cb < 4 ? cb : 11 - cb);  // image column of key block cb
        const int i = 32 * rb + lane;
        int r0, c0;
        const uint32_t img = a_block_image(rb, cb, r0, c0);
        const uint32_t ta = tl + (top ? 0u : 128u) + static_cast<uint32_t>(icol);
        if (cb == rb)  // warp-uniform
          build_a32<true>(ta, i, 32 * cb, sm + img, r0 + lane, c0, be[i] * rn[i], gc[i], rn, gc);
        else
          build_a32<false>(ta, i, 32 * cb, sm + img, r0 + lane, c0, be[i] * rn[i], gc[i], rn, gc);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    failed = __syncthreads_or(ok ? 0 : 1) != 0;
    if (failed) break;
    tc_fence_after();

    // ---- S1: level 0, warp w inverts diagonal block w (rows/columns 32w..32w+31)
    {
      const int q = warp >> 1, odd = warp & 1;
      const uint8_t* src = aul + (odd ? kAL : kAU) + q * kTile;
      float t[32];
      solve_diag32<false>(src, odd * 4, lane, t, InCodes{1.0f, 0});
      __syncwarp();  // all lanes are done reading `src` before odd blocks overwrite it below
      // result rows (coalesced: lane j writes column 32w + j of row 32w + i)
      const int64_t o0 = static_cast<int64_t>(y0 + 32 * warp) * kC + 32 * warp + lane;
      float* out = T + o0;
#pragma unroll
      for (int i = 0; i < 32; ++i) out[static_cast<int64_t>(i) * kC] = t[i];
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
      }
    }
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
      put_row_out<false>(st, lane, v, oc);
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
      put_row_out<false>(st, lane, v, oc);
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
        put_row_out<false>(st, lane, v, oc);
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

  // Drain: stores complete, an outstanding load lands (bounded), TMEM released.
  if (lane == 0) bulk_wait_all();
  if (tid == 0 && pend) mbar_wait(k_bar, pend_par, err, kErrTimeoutOther);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

__device__ int g_gdn256f_err;

}  // namespace

bool gdn256f_supported(const void* k, const float* beta, const float* g, const float* T, int64_t n_chunks) {
  // TMA / bulk copies: 16-byte aligned bases; row coordinates (chunk * 256 + 255) fit in int32.
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return al16(k) && al16(beta) && al16(g) && al16(T) && n_chunks > 0 && n_chunks <= (int64_t{1} << 23) - 1;
}

cudaError_t launch_gdn256_fused(const void* k, const float* beta, const float* g, float* T, int64_t n_chunks,
                                cudaStream_t stream) {
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
      e = cudaFuncSetAttribute(gdn256f_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess) return e;
      e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return e;
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_gdn256f_err);
      if (e != cudaSuccess) return e;
      err_ptr[dev] = static_cast<int*>(p);
      attr_set[dev] = 1;
    }
  }
  CUtensorMap tk, tt;
  const uint64_t rows = static_cast<uint64_t>(n_chunks) * kC;
  // k [n_chunks * 256, 128] bf16: boxes of 64 Dk columns (128 bytes, the swizzle span) x 32 rows
  if (!make_tmap_2d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, k, 128, rows, 128 * 2, 64, 32)) return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tt, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, T, kC, rows, kC * 4, 32, 32)) return cudaErrorInvalidValue;
  const int64_t grid = n_chunks < sms[dev] ? n_chunks : sms[dev];
  GdnKbgArgs args{T, beta, g, n_chunks, err_ptr[dev]};
  gdn256f_kernel<<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(tk, tt, args);
  return cudaGetLastError();
}

}  // namespace qhtp
