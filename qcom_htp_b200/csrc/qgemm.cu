// Quantized MatMul family on B200: persistent tcgen05 kind::i8 GEMM with TMEM accumulators,
// TMA-staged 128-byte-swizzled shared-memory tiles, and a fused exact requant epilogue.
//
// Mapping of the reference arithmetic (scripts/generate_qnn_matmul_python_cases.py:426-481) onto
// integer tensor-core products:
//   * u8 activations feed the MMA as-is (unsigned A operand); the activation zero-point is folded
//     into the per-channel effective bias (bias_q - zp * sum_k w, gen_quant_chain.py:879).
//   * u16 activations are split into two u8 byte planes (hi, lo); each plane is its own MMA into
//     its own s32 TMEM accumulator, recombined exactly in int64 (256*hi + lo) in the epilogue.
//   * float32 weight dequant (w_deq = f32(q*s)) is reproduced exactly: s = m_s*2^e_s, and
//     f32(q*s) = (q*m_s + e')*2^e_s with the integer residual e' in [-64,64].  The prepared weight
//     tile is [q rows | e' rows]: one N=256 MMA yields both sum(x*q) and sum(x*e').
//   * int16 weights (W16A16) are two byte planes, hi (s8) and lo (u8) (verify_w16a16_two_w8a16.py:21-48),
//     giving three accumulators (hi*hi, hi*lo+lo*hi, lo*lo) combined with x65536 / x256 / x1.
//
// Persistent CTAs (one per SM) walk 128x128 output tiles.  Roles (384 threads, 3 warpgroups):
//   warp 0      TMA producer (one lane): activation plane(s) + weight planes per 128-byte K step
//   warp 1      TMEM allocator + MMA issuer (one lane)
//   warps 2,3   idle (they complete warpgroup 0, which gives its registers to the epilogue)
//   warps 4..11 epilogue: each thread owns one output row and 64 channels; it drains the TMEM
//               accumulators into int64 registers, releases TMEM (the next tile's MMAs start),
//               then requantizes from registers with integer fixed-point math and stores.
// Register split: launched at 168 registers/thread (384 x 168 = 64512); warpgroup 0 drops to 40
// (setmaxnreg.dec) and the two epilogue warpgroups rise to 232 (setmaxnreg.inc):
// 128*40 + 256*232 = 64512, the launch total.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"
#include "requant.cuh"

namespace qhtp {

// ------------------------------------------------------------------------------------------------
// Tensor maps (driver entry point fetched once through the runtime; no -lcuda needed)
// ------------------------------------------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t rows,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  PFN_encodeTiled enc = get_encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                     uint32_t box_inner, uint32_t box_rows) {
  return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, inner, rows, row_stride_bytes, box_inner, box_rows);
}

// The prepared weight planes as [n_tiles * kblocks * b_rows, 128] bytes: each (tile, K block) is one
// contiguous, already swizzled operand image, copied verbatim (no TMA swizzle) into a stage.
bool make_tmap_planes(CUtensorMap* map, const QhtpMatmulPlan* plan) {
  const uint64_t rows = static_cast<uint64_t>(plan->n_tiles) * (plan->k_pad / kTileK) * b_rows_for_mode(plan->mode);
  return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, plan->prepared, kTileK, rows, kTileK, kTileK,
                      b_rows_for_mode(plan->mode), CU_TENSOR_MAP_SWIZZLE_NONE);
}

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// ------------------------------------------------------------------------------------------------
// GEMM kernel
// ------------------------------------------------------------------------------------------------
struct GemmParams {
  int M, N, m_tiles, n_tiles, kblocks, a_plane_rows, K;
  const uint8_t* a_lo;      // the activation's lo byte plane [M][K] (u16 activations)
  const int8_t* wplanes;    // the prepared weight images (the e' rows are read by the exact fix-up)
  const ChannelRecord* rec;
  void* out;
  int zp_out, qmax;
  uint64_t act_mant, out_mant;
  int act_exp2, out_exp2;
  int* err;
};

#ifndef QHTP_LO_DOT_BATCH
#define QHTP_LO_DOT_BATCH 8  // chunks per lane in flight in the exact lo x e' fix-up
#endif

constexpr int kEpiWarps = 8;
constexpr int kEpiWarp0 = 4;  // first epilogue warp (warpgroups 1 and 2)
constexpr int kGemmThreads = 32 * (kEpiWarp0 + kEpiWarps);
constexpr int kRegsLaunch = 168, kRegsCtrl = 40, kRegsEpi = 232;
static_assert(kGemmThreads * kRegsLaunch == 128 * kRegsCtrl + 32 * kEpiWarps * kRegsEpi, "register split");

// 16-byte global -> shared copy that bypasses the registers (completed by cp_async_wait).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// TMEM is released in two halves (activation-hi accumulators, then lo) when the activation has two
// byte planes and the planes' MMAs are separate instructions.
template <int PA, int MODE>
constexpr bool kSplitRelease = PA == 2 && MODE != kModeW16;

template <int PA, int MODE>
struct GemmCfg {
  static constexpr int kBRows = MODE == kModeExact ? 128 : 256;
  static constexpr int kStageA = kTileM * kTileK;  // 16 KB per activation plane
  static constexpr int kStageB = kBRows * kTileK;  // weight planes
  static constexpr int kStage = PA * kStageA + kStageB;
  static constexpr int kStagesRaw = (200 * 1024) / kStage;
  static constexpr int kStages = kStagesRaw > 6 ? 6 : kStagesRaw;
  static constexpr int kRecBytes = kTileN * 32;  // a tile's channel records, staged for the epilogue
  static constexpr int kSmem = kStages * kStage + 2 * kRecBytes + 1024 + 256;  // two record buffers
};

// Named barrier 1 over the epilogue warps, and the same barrier ANDing a predicate (every thread
// leaves with the same answer, so a bounded wait that gave up anywhere stops all of them together).
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory"); }
__device__ __forceinline__ bool epi_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.cta.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(32 * kEpiWarps)
      : "memory");
  return r != 0;
}

// sum_k x_lo[mm, k] * e'[nn, k] over the real K, by the whole warp (lane l takes the 16-byte chunks
// l, l + 32, ...: u8 activation bytes times s8 residuals, 4 per dp4a), returned to every lane.  A
// lane's chunks are loaded kLoDotBatch at a time, all in flight together: the fix-up sits in the
// epilogue, and in a launch of one or two tiles per CTA its latency is the kernel's.
constexpr int kLoDotBatch = QHTP_LO_DOT_BATCH;
__device__ __forceinline__ void lo_dot16(int32_t& acc, const uint4& xv, const uint4& ev) {
  asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(xv.x), "r"(ev.x));
  asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(xv.y), "r"(ev.y));
  asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(xv.z), "r"(ev.z));
  asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(xv.w), "r"(ev.w));
}
__device__ __forceinline__ int32_t lo_residual_dot(const GemmParams& p, int mm, int nn, int lane) {
  constexpr int B = kLoDotBatch;
  const uint8_t* xr = p.a_lo + static_cast<size_t>(mm) * p.K;
  const int nt = nn / kTileN, rr = nn % kTileN;
  const int8_t* wr = p.wplanes + (static_cast<size_t>(nt) * p.kblocks * 256 + 128 + rr) * kTileK;
  auto e_at = [&](int ch) {
    return *reinterpret_cast<const uint4*>(wr + static_cast<size_t>(ch >> 3) * 256 * kTileK +
                                           ((((ch & 7) ^ rr) & 7) << 4));
  };
  const int nch = p.K / 16;
  int32_t acc = 0;
  int ch = lane;
  for (; ch + 32 * (B - 1) < nch; ch += 32 * B) {
    uint4 xv[B], ev[B];
#pragma unroll
    for (int u = 0; u < B; ++u) {
      xv[u] = *reinterpret_cast<const uint4*>(xr + (ch + 32 * u) * 16);
      ev[u] = e_at(ch + 32 * u);
    }
#pragma unroll
    for (int u = 0; u < B; ++u) lo_dot16(acc, xv[u], ev[u]);
  }
  for (; ch < nch; ch += 32) lo_dot16(acc, *reinterpret_cast<const uint4*>(xr + ch * 16), e_at(ch));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return acc;
}

// LO3 (u16 activation, f32 dequant, plan flag kPlanLoResidualByBound): the lo-plane MMA multiplies
// the q rows only (N = 128); the lo x e' part of T, at most ChannelRecord::lo_win output units of
// 2^-30, is added exactly (lo_residual_dot) only where the fast path's value lies within that
// window of a rounding boundary.
template <int PA, int MODE, bool LO3 = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
  static_assert(!LO3 || (PA == 2 && MODE == kModeF32), "LO3 is the u16-activation f32-dequant variant");
  using Cfg = GemmCfg<PA, MODE>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t kTmemCols = 512;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  ChannelRecord* rec_s = reinterpret_cast<ChannelRecord*>(smem + S * Cfg::kStage);  // [2][128]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStage + 2 * Cfg::kRecBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 1;      // [2]: TMEM half A / half B handed back by the epilogue
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(&tempty[0], kEpiWarps);
    mbar_init(&tempty[1], kEpiWarps);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp < kEpiWarp0) {
  // warpgroup 0: give registers to the epilogue warpgroups (setmaxnreg must dominate the code it governs)
  regs_dec<kRegsCtrl>();
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      uint32_t it = 0;
      bool ok = true;
      // First tile: the weight planes of the first stages load before the activation is awaited,
      // overlapping the activation producer (the u16 plane split, launched just before with
      // programmatic dependent launch); a no-op wait otherwise.
      const int D = p.kblocks < S ? p.kblocks : S;
      if (static_cast<int>(blockIdx.x) < total_tiles) {
        const int m0 = (blockIdx.x % p.m_tiles) * kTileM;
        const int nt = blockIdx.x / p.m_tiles;
        for (int d = 0; d < D; ++d) {
          mbar_arrive_expect_tx(&full[d], Cfg::kStage);
          tma_load_2d(stages + d * Cfg::kStage + PA * Cfg::kStageA, &tmB, &full[d], 0, (nt * p.kblocks + d) * Cfg::kBRows);
        }
        griddep_wait();
        for (int d = 0; d < D; ++d) {
#pragma unroll
          for (int pl = 0; pl < PA; ++pl)
            tma_load_2d(stages + d * Cfg::kStage + pl * Cfg::kStageA, &tmA, &full[d], d * kTileK,
                        pl * p.a_plane_rows + m0);
        }
        it = static_cast<uint32_t>(D);
      }
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % p.m_tiles) * kTileM;
        const int nt = tile / p.m_tiles;
        for (int kb = (tile == static_cast<int>(blockIdx.x) ? D : 0); kb < p.kblocks; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::kStage);
          uint8_t* st = stages + s * Cfg::kStage;
#pragma unroll
          for (int pl = 0; pl < PA; ++pl)
            tma_load_2d(st + pl * Cfg::kStageA, &tmA, &full[s], kb * kTileK, pl * p.a_plane_rows + m0);
          tma_load_2d(st + PA * Cfg::kStageA, &tmB, &full[s], 0, (nt * p.kblocks + kb) * Cfg::kBRows);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, tc = 0;
      bool ok = true;
      // One K block's MMAs on stage s: the activation-hi plane (TMEM half A) and/or the lo plane
      // (half B; A16 only).
      auto issue_kb = [&](uint32_t st_addr, int kb, bool do_hi, bool do_lo) {
        const uint64_t dA0 = desc_kmajor_sw128(st_addr);
        const uint64_t dA1 = desc_kmajor_sw128(st_addr + (PA > 1 ? Cfg::kStageA : 0));
        const uint64_t dB = desc_kmajor_sw128(st_addr + PA * Cfg::kStageA);
#pragma unroll
        for (int kk = 0; kk < kTileK / 32; ++kk) {
          const uint32_t acc = (kb | kk) ? 1u : 0u;
          const uint64_t ko = static_cast<uint64_t>(kk * 2);  // 32 bytes, in 16-byte units
          if constexpr (MODE == kModeW16) {
            constexpr uint32_t idS = idesc_i8(128, 128, 0, 1);  // u8 act x s8 hi-byte weight
            constexpr uint32_t idU = idesc_i8(128, 128, 0, 0);  // u8 act x u8 lo-byte weight
            const uint64_t dBhi = dB + ko;
            const uint64_t dBlo = dB + ko + (128 * kTileK >> 4);
            mma_i8(tmem + 0, dA0 + ko, dBhi, idS, acc);
            mma_i8(tmem + 128, dA0 + ko, dBlo, idU, acc);
            mma_i8(tmem + 128, dA1 + ko, dBhi, idS, 1u);
            mma_i8(tmem + 256, dA1 + ko, dBlo, idU, acc);
          } else {
            constexpr int N = Cfg::kBRows;  // 256 = [q | e'] (f32 mode), 128 = q (exact mode)
            constexpr uint32_t id = idesc_i8(128, N, 0, 1);
            constexpr uint32_t id_lo = idesc_i8(128, LO3 ? 128 : N, 0, 1);  // LO3: lo plane x q rows only
            if (do_hi) mma_i8(tmem + 0, dA0 + ko, dB + ko, id, acc);
            if constexpr (PA == 2) {
              if (do_lo) mma_i8(tmem + N, dA1 + ko, dB + ko, id_lo, acc);
            }
          }
        }
      };
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x, ++tc) {
        if (!mbar_wait(&tempty[0], (tc & 1) ^ 1, p.err, kErrTimeoutOther)) break;
        tc_fence_after();
        int kb = 0;
        if constexpr (kSplitRelease<PA, MODE>) {
          // Half A is free: run the hi-plane MMAs of every stage already loaded while the epilogue
          // still drains half B, then the lo-plane MMAs of those stages.
          const int D = p.kblocks < S ? p.kblocks : S;
          for (int d = 0; d < D; ++d) {
            const int s = (it + d) % S;
            if (!mbar_wait(&full[s], ((it + d) / S) & 1, p.err, kErrTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_kb(smem_u32(stages + s * Cfg::kStage), d, true, false);
          }
          if (!ok) break;
          if (!mbar_wait(&tempty[1], (tc & 1) ^ 1, p.err, kErrTimeoutOther)) break;
          tc_fence_after();
          for (int d = 0; d < D; ++d) {
            const int s = (it + d) % S;
            issue_kb(smem_u32(stages + s * Cfg::kStage), d, false, true);
            mma_commit(&empty[s]);  // stage free once these MMAs have read it
          }
          kb = D;
          it += D;
        } else {
          if (!mbar_wait(&tempty[1], (tc & 1) ^ 1, p.err, kErrTimeoutOther)) break;
          tc_fence_after();
        }
        for (; kb < p.kblocks; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&full[s], ph, p.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_kb(smem_u32(stages + s * Cfg::kStage), kb, true, true);
          mma_commit(&empty[s]);  // stage free once these MMAs have read it
        }
        if (ok) mma_commit(tfull);  // accumulators of this tile complete
      }
    }
  }  // warps 2, 3: idle
  } else {
    regs_inc<kRegsEpi>();
    // ------------------------------------------------------------------ epilogue (warps 4..11)
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may access
    const int half = (warp - kEpiWarp0) >> 2;  // which 64 of the 128 channels
    const int row = quad * 32 + lane;
    const bool u16 = p.qmax > 255;
    // A tile's 128 channel records (4 KB) are copied into shared memory (cp.async, 16 bytes per
    // thread) one tile ahead, into the other of two buffers: the drain and the requant read their
    // constants there, and the copy's latency hides behind the previous tile's requant.
    const int et = static_cast<int>(threadIdx.x) - 32 * kEpiWarp0;  // 0..255, 16 bytes each
    auto stage_records = [&](int t, uint32_t buf) {
      if (t < total_tiles)
        cp_async16(smem_u32(rec_s + buf * kTileN) + 16 * et,
                   reinterpret_cast<const uint4*>(p.rec + (t / p.m_tiles) * kTileN) + et);
      cp_async_commit();  // an empty group past the last tile keeps the group count per tile
    };
    stage_records(blockIdx.x, 0);
    uint32_t tc = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++tc) {
      const int m = (tile % p.m_tiles) * kTileM + row;
      const int n0 = (tile / p.m_tiles) * kTileN + half * 64;
      epi_bar();  // every epilogue warp is done with the previous tile's records (the other buffer)
      stage_records(tile + gridDim.x, (tc + 1) & 1);
      cp_async_wait<1>();  // this tile's records (all but the newest group) have landed
      if (!epi_bar_and(mbar_wait(tfull, tc & 1, p.err, kErrTimeoutAccum))) break;  // also publishes them
      const ChannelRecord* rec = rec_s + (tc & 1) * kTileN + half * 64;
      tc_fence_after();
      const uint32_t tl = tmem + (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
      // ---- drain: TMEM -> int64 accumulators in registers (64 channels of this thread's row).  The
      // effective bias joins T in the requant phase (its record load is already there).
      int64_t T[64];
      if constexpr (kSplitRelease<PA, MODE>) {
        // half A (activation-hi accumulators) in one TMEM wait, handed back at once; then half B,
        // combined in place into T while the MMA warp already runs the next tile's hi-plane MMAs
        constexpr int N = Cfg::kBRows;
        uint32_t sq0[32], sq1[32], se0[32], se1[32];
        tmem_ld32(tl + 0, sq0);
        tmem_ld32(tl + 32, sq1);
        if constexpr (MODE == kModeF32) {
          tmem_ld32(tl + 128, se0);
          tmem_ld32(tl + 160, se1);
        }
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[0]);
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) {
          int32_t mqv[16];
          if constexpr (MODE == kModeF32) {
#pragma unroll
            for (int j = 0; j < 16; ++j) mqv[j] = rec[c0 + j].m_q;
          }
          uint32_t lq[16], le[16];
          tmem_ld16(tl + N + c0, lq);                                    // sum x_lo * q
          if constexpr (MODE == kModeF32 && !LO3) tmem_ld16(tl + N + 128 + c0, le);  // sum x_lo * e'
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t hq = c0 < 32 ? sq0[c0 + j] : sq1[c0 - 32 + j];
            const int64_t pq = static_cast<int64_t>(static_cast<int32_t>(hq)) * 256 + static_cast<int32_t>(lq[j]);
            if constexpr (MODE == kModeF32) {
              const uint32_t he = c0 < 32 ? se0[c0 + j] : se1[c0 - 32 + j];
              const int64_t pe = static_cast<int64_t>(static_cast<int32_t>(he)) * 256 +
                                 (LO3 ? 0 : static_cast<int32_t>(le[j]));
              T[c0 + j] = static_cast<int64_t>(mqv[j]) * pq + pe;
            } else {
              T[c0 + j] = pq;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[1]);
      } else {
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 8) {
          uint32_t s0[8], s1[8], s2[8];
          if constexpr (MODE == kModeF32) {
            tmem_ld8(tl + c0, s0);             // sum x * q
            tmem_ld8(tl + 128 + c0, s1);       // sum x * e'
          } else if constexpr (MODE == kModeExact) {
            tmem_ld8(tl + c0, s0);
          } else {
            tmem_ld8(tl + c0, s0);             // hi x hi
            tmem_ld8(tl + 128 + c0, s1);       // hi x lo + lo x hi
            tmem_ld8(tl + 256 + c0, s2);       // lo x lo
          }
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if constexpr (MODE == kModeF32) {
              const int64_t mq = rec[c0 + j].m_q;
              T[c0 + j] = mq * static_cast<int32_t>(s0[j]) + static_cast<int32_t>(s1[j]);
            } else if constexpr (MODE == kModeExact) {
              T[c0 + j] = static_cast<int32_t>(s0[j]);
            } else {
              T[c0 + j] = static_cast<int64_t>(static_cast<int32_t>(s0[j])) * 65536 +
                          static_cast<int64_t>(static_cast<int32_t>(s1[j])) * 256 + static_cast<int32_t>(s2[j]);
            }
          }
        }
        // accumulators are in registers: hand TMEM back to the MMA warp
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&tempty[0]);
          mbar_arrive(&tempty[1]);
        }
      }
      // ---- requant + store, 16 channels per iteration; the register array rotates by 16 so the
      // loop body is emitted once (small instruction footprint).  The whole warp runs every
      // iteration (rows past M compute and store nothing) so that the LO3 fix-up can be cooperative.
      const bool row_ok = m < p.M;
#pragma unroll 1
      for (int c0 = 0; c0 < 64; c0 += 16) {
        const int n = n0 + c0;
        if (n < p.N) {  // channels past N (tile padding) have no record; uniform across the warp
          uint32_t code[16];
          uint32_t near_mask = 0;
          int64_t fl[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint4 rb = *reinterpret_cast<const uint4*>(rec + c0 + j);       // beff | cmn
            const int tn = rec[c0 + j].tn;
            const uint64_t cmn = (static_cast<uint64_t>(rb.w) << 32) | rb.z;
            T[j] += static_cast<int64_t>((static_cast<uint64_t>(rb.y) << 32) | rb.x);  // + effective bias
            bool nr;
            code[j] = static_cast<uint32_t>(requant_fast96s(T[j], cmn, tn, p.zp_out, p.qmax, &nr, &fl[j]));
            if constexpr (LO3) {
              // the missing lo x e' term moves the value by at most lo_win units of 2^-30: flag the
              // elements whose fraction lies within lo_win + 2 units of a rounding boundary
              const uint32_t w = static_cast<uint32_t>(rec[c0 + j].lo_win) + 2u;
              const uint32_t win = static_cast<uint32_t>(fl[j]) & 0x3FFFFFFFu;
              const int64_t top = T[j] >> (63 - tn);
              const bool big = (top != 0) & (top != -1);
              nr = !big && (((win + w) & 0x3FFFFFFFu) < 2u * w);
            }
            near_mask |= nr ? (1u << j) : 0u;
          }
          if (!row_ok) near_mask = 0;
          if constexpr (LO3) {
            // exact lo x e' sums of the flagged elements, one element at a time by the whole warp,
            // added into T (which is then complete for those elements)
            uint32_t pending = near_mask;
            while (true) {
              const uint32_t lanes = __ballot_sync(0xffffffffu, pending != 0);
              if (lanes == 0) break;
              const int src = __ffs(lanes) - 1;
              const int jj = __shfl_sync(0xffffffffu, __ffs(pending) - 1, src);
              const int mm = __shfl_sync(0xffffffffu, m, src);
              const int32_t dot = lo_residual_dot(p, mm, n + jj, lane);
              if (lane == src) {
                pending &= ~(1u << jj);
#pragma unroll
                for (int j = 0; j < 16; ++j) T[j] += j == jj ? dot : 0;
              }
            }
            if (near_mask != 0) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                if (near_mask & (1u << j)) {
                  const uint64_t cmn = rec[c0 + j].cmn;
                  const int tn = rec[c0 + j].tn;
                  bool nr;  // T is complete: the exact decision of the full-MMA kernel
                  code[j] = static_cast<uint32_t>(requant_fast96s(T[j], cmn, tn, p.zp_out, p.qmax, &nr, &fl[j]));
                  if (nr) {
                    const uint32_t wb = rec[c0 + j].wbits;
                    const int es = static_cast<int>((wb >> 23) & 0xFFu) - 150;
                    code[j] = static_cast<uint32_t>(requant_tie_w(T[j], fl[j], 1u, es + p.act_exp2, p.act_mant,
                                                                p.out_mant, p.out_exp2, p.zp_out, p.qmax));
                  }
                }
              }
            }
          } else if (near_mask != 0) {  // rare: within 2^-29 of a tie -> exact decision
            for (int j = 0; j < 16; ++j) {
              if (near_mask & (1u << j)) {
                const uint32_t wb = rec[c0 + j].wbits;
                const uint32_t ms = (wb & 0x7FFFFFu) | 0x800000u;
                const int es = static_cast<int>((wb >> 23) & 0xFFu) - 150;
                const uint32_t mul = MODE == kModeF32 ? 1u : ms;
                code[j] = static_cast<uint32_t>(requant_tie_w(T[j], fl[j], mul, es + p.act_exp2, p.act_mant,
                                                            p.out_mant, p.out_exp2, p.zp_out, p.qmax));
              }
            }
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (row_ok && n + 8 * h < p.N) {
              const uint32_t* cd = code + 8 * h;
              if (u16) {
                uint4 v;
                v.x = cd[0] | (cd[1] << 16);
                v.y = cd[2] | (cd[3] << 16);
                v.z = cd[4] | (cd[5] << 16);
                v.w = cd[6] | (cd[7] << 16);
                // streaming (evict-first) store: the output does not displace the operand tiles in L2
                __stcs(reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + static_cast<size_t>(m) * p.N +
                                                n + 8 * h), v);
              } else {
                uint2 v;
                v.x = cd[0] | (cd[1] << 8) | (cd[2] << 16) | (cd[3] << 24);
                v.y = cd[4] | (cd[5] << 8) | (cd[6] << 16) | (cd[7] << 24);
                __stcs(reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(p.out) + static_cast<size_t>(m) * p.N +
                                                n + 8 * h), v);
              }
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 48; ++j) T[j] = T[j + 16];
      }
    }
    cp_async_wait<0>();  // no record copy is still in flight when the CTA's shared memory goes away
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// u16 activation [M,K] -> byte planes hi [M,K] and lo [M,K] (u8), the A operands of the A16 GEMM.
__global__ void split_u16_planes(const uint16_t* __restrict__ act, uint8_t* __restrict__ hi,
                                 uint8_t* __restrict__ lo, size_t n8) {
  griddep_launch_dependents();  // the GEMM may start its prologue and weight loads now
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint4 v = reinterpret_cast<const uint4*>(act)[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      h0 |= ((w[j] >> 8) & 0xFFu) << (16 * j);
      h0 |= ((w[j] >> 24) & 0xFFu) << (16 * j + 8);
      l0 |= (w[j] & 0xFFu) << (16 * j);
      l0 |= ((w[j] >> 16) & 0xFFu) << (16 * j + 8);
      h1 |= ((w[j + 2] >> 8) & 0xFFu) << (16 * j);
      h1 |= ((w[j + 2] >> 24) & 0xFFu) << (16 * j + 8);
      l1 |= (w[j + 2] & 0xFFu) << (16 * j);
      l1 |= ((w[j + 2] >> 16) & 0xFFu) << (16 * j + 8);
    }
    reinterpret_cast<uint2*>(hi)[i] = make_uint2(h0, h1);
    reinterpret_cast<uint2*>(lo)[i] = make_uint2(l0, l1);
  }
}

template <int PA, int MODE, bool LO3 = false>
static cudaError_t launch_variant(const GemmLaunch& g, const CUtensorMap& ta, const CUtensorMap& tb,
                                  const GemmParams& prm) {
  using Cfg = GemmCfg<PA, MODE>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(qgemm_kernel<PA, MODE, LO3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmem);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const int total = prm.m_tiles * prm.n_tiles;
  int slots = sm_count();
  if (g.max_ctas != 0 && static_cast<int>(g.max_ctas) < slots) slots = static_cast<int>(g.max_ctas);
  const int grid = total < slots ? total : slots;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = g.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = PA == 2 ? 1 : 0;  // only behind this library's own plane split
  return cudaLaunchKernelEx(&cfg, qgemm_kernel<PA, MODE, LO3>, ta, tb, prm);
}

cudaError_t launch_split_u16(const uint16_t* act, uint8_t* planes, size_t total, cudaStream_t stream) {
  const size_t n8 = total / 8;
  int blocks = static_cast<int>((n8 + 255) / 256);
  if (blocks > sm_count() * 16) blocks = sm_count() * 16;
  if (blocks < 1) blocks = 1;
  split_u16_planes<<<blocks, 256, 0, stream>>>(act, planes, planes + total, n8);
  return cudaGetLastError();
}

// The lo-plane residual bound on a row-tiled launch of `tiles` tiles: where it is valid and either
// forced by the caller, or worth it (few expected fix-ups) on a launch of at least
// kLoResidualMinWaves waves -- with fewer, the last tile's fix-ups are not hidden behind a next
// tile's MMAs (measured: M = 128, N = 14336 in one wave 48.2 us with it, 42.0 us without).
static bool lo_residual_launch(const QhtpMatmulPlan* pl, int tiles, uint32_t max_ctas) {
  if (!(pl->flags & kPlanLoResidualByBound)) return false;
  if (pl->flags & kPlanForceLoResidual) return true;
  int slots = sm_count();
  if (max_ctas != 0 && static_cast<int>(max_ctas) < slots) slots = static_cast<int>(max_ctas);
  return (pl->flags & kPlanLoResidualPays) && tiles >= kLoResidualMinWaves * slots;
}

cudaError_t launch_gemm(const GemmLaunch& g) {
  const QhtpMatmulPlan* pl = g.plan;
  const uint32_t K = pl->k;
  CUtensorMap ta, tb;
  const uint8_t* a_base;
  uint64_t a_rows;
  if (g.dec4 != nullptr && dec4_supported(pl, g.m)) return launch_dec4(g);  // int4 codes, M <= 16
  if (pl->a_planes == 2) {
    const size_t total = static_cast<size_t>(g.m) * K;
    cudaError_t e = launch_split_u16(static_cast<const uint16_t*>(g.act), g.planes, total, g.stream);
    if (e != cudaSuccess) return e;
    a_base = g.planes;
    a_rows = 2ull * g.m;
  } else {
    a_base = static_cast<const uint8_t*>(g.act);
    a_rows = g.m;
  }
  if (pl->mode == kModeGroup) return launch_gemm_group(g, a_base, a_rows, sm_count());
  if (decode_supported(pl, g.m)) return launch_decode(g, a_base);
  if (!make_tmap_2d_u8(&ta, a_base, K, a_rows, K, kTileK, kTileM)) return cudaErrorInvalidValue;
  const uint32_t brows = b_rows_for_mode(pl->mode);
  const uint8_t* planes = static_cast<const uint8_t*>(pl->prepared);
  if (!make_tmap_planes(&tb, pl)) return cudaErrorInvalidValue;
  GemmParams prm;
  prm.M = static_cast<int>(g.m);
  prm.N = static_cast<int>(pl->n);
  prm.m_tiles = static_cast<int>((g.m + kTileM - 1) / kTileM);
  prm.n_tiles = static_cast<int>(pl->n_tiles);
  prm.kblocks = static_cast<int>(pl->k_pad / kTileK);
  prm.a_plane_rows = static_cast<int>(g.m);
  prm.K = static_cast<int>(K);
  prm.a_lo = pl->a_planes == 2 ? a_base + static_cast<size_t>(g.m) * K : nullptr;
  prm.wplanes = reinterpret_cast<const int8_t*>(planes);
  prm.rec = reinterpret_cast<const ChannelRecord*>(planes + pl->plane_bytes);
  prm.out = g.out;
  prm.zp_out = pl->out_zp;
  prm.qmax = pl->out_qmax;
  prm.act_mant = pl->act_mant;
  prm.out_mant = pl->out_mant;
  prm.act_exp2 = pl->act_exp2;
  prm.out_exp2 = pl->out_exp2;
  prm.err = g.err;
  switch (pl->mode * 2 + (pl->a_planes - 1)) {
    case kModeF32 * 2 + 0: return launch_variant<1, kModeF32>(g, ta, tb, prm);
    case kModeF32 * 2 + 1:
      if (lo_residual_launch(pl, prm.m_tiles * prm.n_tiles, g.max_ctas))
        return launch_variant<2, kModeF32, true>(g, ta, tb, prm);
      return launch_variant<2, kModeF32>(g, ta, tb, prm);
    case kModeExact * 2 + 0: return launch_variant<1, kModeExact>(g, ta, tb, prm);
    case kModeExact * 2 + 1: return launch_variant<2, kModeExact>(g, ta, tb, prm);
    case kModeW16 * 2 + 1: return launch_variant<2, kModeW16>(g, ta, tb, prm);
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------------------------------------
// Prepare: weight byte planes + per-channel records
// ------------------------------------------------------------------------------------------------
struct PrepParams {
  uint32_t family, schema, mode, K, N, k_pad, b_rows, lpbq_block;
  const void* weight;
  const uint8_t* lpbq;
  int8_t* planes;
  long long* sums;  // [Npad][kSumsPerChannel]
};

__device__ __forceinline__ int load_weight(const PrepParams& p, uint32_t n, uint32_t k) {
  if (p.family == QHTP_FAMILY_U8I8 || p.family == QHTP_FAMILY_W8A16) {
    return static_cast<const int8_t*>(p.weight)[static_cast<size_t>(n) * p.K + k];
  }
  if (p.family == QHTP_FAMILY_W16A16) {
    return static_cast<const int16_t*>(p.weight)[static_cast<size_t>(n) * p.K + k];
  }
  const uint8_t b = static_cast<const uint8_t*>(p.weight)[static_cast<size_t>(k >> 1) * p.N + n];
  int q = (k & 1) ? (b >> 4) : (b & 0xF);
  q = q >= 8 ? q - 16 : q;  // two's-complement nibble
  if (p.schema == QHTP_SCHEMA_LPBQ) {
    const int f = p.lpbq[static_cast<size_t>(n) * (p.K / p.lpbq_block) + k / p.lpbq_block];
    q *= f;
    q = q < -128 ? -128 : (q > 127 ? 127 : q);  // HmxW4LpbqExpandToI8Op.cpp:42-47
  }
  return q;
}

// One thread per (channel, 16-wide K chunk).
__global__ void prepare_planes_kernel(PrepParams p, const float* __restrict__ scale) {
  const uint32_t chunks = p.K / 16;
  const size_t total = static_cast<size_t>(p.N) * chunks;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint32_t n = static_cast<uint32_t>(idx / chunks);
    const uint32_t k0 = static_cast<uint32_t>(idx % chunks) * 16;
    // blocked, pre-swizzled layout: (tile, K block) -> b_rows x 128-byte operand image, row r's
    // 16-byte chunk c at r*128 + ((c ^ r) & 7)*16
    const uint32_t tile = n / kTileN, rr = n % kTileN, kb = k0 / kTileK, c = (k0 % kTileK) / 16;
    const size_t blk = (static_cast<size_t>(tile) * (p.k_pad / kTileK) + kb) * p.b_rows * kTileK;
    int8_t* r0 = p.planes + blk + rr * kTileK + (((c ^ rr) & 7u) << 4);
    int8_t* r1 = r0 + 128 * kTileK;  // second plane (f32 / W16 modes): rows 128..255 of the image
    long long sq = 0, se = 0, sa = 0;
    if (p.mode == kModeF32) {
      const uint32_t bits = __float_as_uint(scale[n]);
      const int32_t ms = static_cast<int32_t>((bits & 0x7FFFFFu) | 0x800000u);
#pragma unroll 4
      for (int j = 0; j < 16; ++j) {
        const int q = load_weight(p, n, k0 + j);
        const int32_t prod = q * ms;                                    // |prod| < 2^31
        const int32_t rnd = __float2int_rz(__int2float_rn(prod));     // round to 24 significant bits
        const int e = rnd - prod;                                       // |e| <= 64
        r0[j] = static_cast<int8_t>(q);
        r1[j] = static_cast<int8_t>(e);
        sq += q;
        se += e;
        sa += e < 0 ? -e : e;
      }
    } else if (p.mode == kModeExact) {
#pragma unroll 4
      for (int j = 0; j < 16; ++j) {
        const int q = load_weight(p, n, k0 + j);
        r0[j] = static_cast<int8_t>(q);
        sq += q;
      }
    } else {
#pragma unroll 4
      for (int j = 0; j < 16; ++j) {
        const int q = load_weight(p, n, k0 + j);
        r0[j] = static_cast<int8_t>(q >> 8);                           // arithmetic high byte, s8
        r1[j] = static_cast<int8_t>(static_cast<uint8_t>(q & 0xFF));   // low byte, u8 carrier
        sq += q;
      }
    }
    long long* sn = p.sums + kSumsPerChannel * n;
    atomicAdd(reinterpret_cast<unsigned long long*>(sn), static_cast<unsigned long long>(sq));
    atomicAdd(reinterpret_cast<unsigned long long*>(sn + 1), static_cast<unsigned long long>(se));
    if (sa != 0) atomicAdd(reinterpret_cast<unsigned long long*>(sn + 2), static_cast<unsigned long long>(sa));
  }
}

__global__ void prepare_records_kernel(uint32_t mode, uint32_t N, const float* __restrict__ scale,
                                       const int32_t* __restrict__ bias, const long long* __restrict__ sums,
                                       double act_scale, double out_scale, int32_t act_zp, int32_t act_exp2,
                                       uint32_t a_planes, ChannelRecord* __restrict__ rec, int* bad_scale) {
  const uint32_t n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const float s = scale[n];
  const uint32_t bits = __float_as_uint(s);
  const uint32_t ex = (bits >> 23) & 0xFFu;
  ChannelRecord r;
  r.lo_win = 0;
  r.wbits = bits;
  if ((bits >> 31) != 0 || ex == 0 || ex == 0xFF) {  // negative, zero/subnormal, inf/nan
    atomicCAS(bad_scale, 0, 1);
    r.beff = 0;
    r.cmn = 0;
    r.m_q = 0;
    r.tn = 0;
    rec[n] = r;
    return;
  }
  const int64_t ms = static_cast<int64_t>((bits & 0x7FFFFFu) | 0x800000u);
  const int es = static_cast<int>(ex) - 150;
  const int64_t sq = sums[kSumsPerChannel * n], se = sums[kSumsPerChannel * n + 1];
  const int64_t sa = sums[kSumsPerChannel * n + 2];
  const int64_t b = bias[n];
  double c;
  if (mode == kModeF32) {
    r.beff = ms * (b - static_cast<int64_t>(act_zp) * sq) - static_cast<int64_t>(act_zp) * se;
    c = ldexp(act_scale, es) / out_scale;
    r.m_q = static_cast<int32_t>(ms);
    if (a_planes == 2) {
      // |sum_k x_lo[k] e'[k]| <= 255 * sum_k |e'[k]|, in units of 2^-30 of the output scale; the
      // products are exact or rounded once each (no contraction: no additions)
      const double x = __dmul_rn(__dmul_rn(static_cast<double>(255 * sa), c), 1073741824.0);
      r.lo_win = x >= 1073741824.0 ? (1 << 30) : static_cast<int32_t>(ceil(x)) + 1;
      atomicMax(bad_scale + 1, r.lo_win);
      atomicAdd(reinterpret_cast<unsigned long long*>(bad_scale + 4), static_cast<unsigned long long>(r.lo_win));
    }
  } else {
    r.beff = b - static_cast<int64_t>(act_zp) * sq;
    c = __dmul_rn(act_scale, static_cast<double>(s)) / out_scale;
    r.m_q = 1;
  }
  // c = cm * 2^-cshift with cm the 53-bit integer mantissa (c is a normal double)
  const uint64_t cb = static_cast<uint64_t>(__double_as_longlong(c));
  const int cex = static_cast<int>((cb >> 52) & 0x7FF);
  const int cshift = 1075 - cex;
  if (cex == 0 || cex == 0x7FF || cshift < 34) {
    atomicCAS(bad_scale, 0, 2);  // requant multiplier outside the supported range (c >= 2^18)
  }
  const FastConst fc = fast_const((cb & ((1ull << 52) - 1)) | (1ull << 52), cshift);
  r.cmn = fc.cmn;
  r.tn = fc.tn;
  (void)act_exp2;
  rec[n] = r;
}

cudaError_t launch_prepare(const QhtpMatmulPlan* plan, const QhtpMatmulWeights* w, void* prepared, int* bad_scale,
                           cudaStream_t stream) {
  if (plan->mode == kModeGroup) return launch_prepare_group(plan, w, prepared, bad_scale, stream, sm_count());
  uint8_t* base = static_cast<uint8_t*>(prepared);
  long long* sums = reinterpret_cast<long long*>(base + plan->plane_bytes + plan->record_bytes);
  cudaError_t e = cudaMemsetAsync(base, 0, plan->prepared_bytes, stream);
  if (e != cudaSuccess) return e;
  PrepParams p;
  p.family = plan->family;
  p.schema = plan->schema;
  p.mode = plan->mode;
  p.K = plan->k;
  p.N = plan->n;
  p.k_pad = plan->k_pad;
  p.b_rows = b_rows_for_mode(plan->mode);
  p.lpbq_block = plan->lpbq_block;
  p.weight = w->weight;
  p.lpbq = w->lpbq_block_scale;
  p.planes = reinterpret_cast<int8_t*>(base);
  p.sums = sums;
  const size_t total = static_cast<size_t>(plan->n) * (plan->k / 16);
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > sm_count() * 32) blocks = sm_count() * 32;
  prepare_planes_kernel<<<blocks, 256, 0, stream>>>(p, w->weight_scale);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  ChannelRecord* rec = reinterpret_cast<ChannelRecord*>(base + plan->plane_bytes);
  prepare_records_kernel<<<static_cast<unsigned>((plan->n + 127) / 128), 128, 0, stream>>>(
      plan->mode, plan->n, w->weight_scale, w->bias_q, sums, plan->act_scale, plan->out_scale, plan->act_zp,
      plan->act_exp2, plan->a_planes, rec, bad_scale);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------
// Failure-path check: one CTA whose warps wait on an mbarrier that no thread ever arrives on, with
// the kernels' own bounded wait.  Every wait runs out after `limit` cycles, records
// kErrTimeoutOther in the error word (first writer wins) and the kernel returns; the caller reads
// the word with qhtp_matmul_check.  Nothing faults, traps or hangs.
// ------------------------------------------------------------------------------------------------
__global__ void wait_timeout_kernel(int* err, long long limit, int* gave_up) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none comes
    fence_barrier_init();
  }
  __syncthreads();
  const bool ok = mbar_wait_limit(&bar, 0, err, kErrTimeoutOther, limit);
  if (!ok && (threadIdx.x & 31) == 0) atomicAdd(gave_up, 1);  // one count per warp that gave up
}

cudaError_t launch_wait_timeout(int* err, long long limit, int* gave_up, cudaStream_t stream) {
  wait_timeout_kernel<<<1, 128, 0, stream>>>(err, limit, gave_up);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------
// Stand-alone LPBQ expand (HmxW4LpbqExpandToI8 semantics), row-major [N,K] int8 output.
// ------------------------------------------------------------------------------------------------
__global__ void lpbq_expand_kernel(const uint8_t* __restrict__ w4, const uint8_t* __restrict__ bs, uint32_t K,
                                   uint32_t N, uint32_t block, int8_t* __restrict__ out) {
  const size_t total = static_cast<size_t>(N) * K;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint32_t n = static_cast<uint32_t>(i / K), k = static_cast<uint32_t>(i % K);
    const uint8_t b = w4[static_cast<size_t>(k >> 1) * N + n];
    int q = (k & 1) ? (b >> 4) : (b & 0xF);
    q = q >= 8 ? q - 16 : q;
    q *= bs[static_cast<size_t>(n) * (K / block) + k / block];
    out[i] = static_cast<int8_t>(q < -128 ? -128 : (q > 127 ? 127 : q));
  }
}

cudaError_t launch_lpbq_expand(const uint8_t* w4, const uint8_t* bs, uint32_t k, uint32_t n, uint32_t block,
                               int8_t* out, cudaStream_t stream) {
  const size_t total = static_cast<size_t>(n) * k;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > sm_count() * 32) blocks = sm_count() * 32;
  lpbq_expand_kernel<<<blocks, 256, 0, stream>>>(w4, bs, k, n, block, out);
  return cudaGetLastError();
}

}  // namespace qhtp
