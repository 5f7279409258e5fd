// Per-group W4 schema on B200: int4 weights with one float32 scale per 64 weights along K
// (scripts/generate_qnn_matmul_python_cases.py:392-423, families w4a8_per_group / w4a16_per_group)
// and a float32 bias (:460-470).  The reference output is, in float64,
//
//     y   = ((x_q - zp_A) * s_A) @ w_deq.T + bias          w_deq = float32(q * s[n, g])
//     out = clip(rint(y / s_O + zp_O), 0, qmax)
//
// Every group scale is s[n,g] = m*2^e (m a 24-bit integer), and float32(q*s) = (q*m + e')*2^e with
// the integer residual e' (|e'| <= 8 for int4 codes).  So one group's contribution to a row is
//
//     Z[g] * 2^e[n,g],   Z[g] = m[n,g]*sum_g(x*q) + sum_g(x*e') - zp*(m[n,g]*sum_g q + sum_g e')
//
// with Z an exact integer (|Z| < 2^50, exact in float64).  The kernel forms the two integer sums of
// a group on the tensor cores (kind::i8), drains them from TMEM after every group and accumulates
// acc += Z*2^e in float64, groups in K order.  The multiply by 2^e is exact, so this is the float64
// sum of the exact group contributions; then y = s_A*acc + bias and the output rounding follow the
// reference formula operation by operation (IEEE double, no contraction).  The oracle restates the
// same sequence (oracle.mm_oracle.per_group_output), and that sequence reproduces the reference's
// output_ref_q on its per-group golden cases.
//
// Channel-major tiles (swap-AB): the weight images are the M = 128 operand (TMEM lane = output
// channel) and 64 activation rows the N operand, so each epilogue thread owns one channel and reads
// its group constants (m, 2^e, zero-point term) once per group instead of once per element.  Per
// group and activation byte plane two MMAs (q rows, e' rows) of M=128, N=64 fill 2 x 64 TMEM columns;
// a 128-byte K block is one pipeline stage and two groups; groups rotate through 512 / (PA*128) TMEM
// buffers (2 for u16 activations, 4 for u8) so the MMAs of later groups overlap the drain of one.
// Roles (640 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer, warps 2-3 idle,
// warps 4..19 the drain/accumulate epilogue (thread = one channel, 16 of the 64 rows; four warps per
// TMEM lane quadrant, four per scheduler, which hides the TMEM-load and float64 latencies).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"
#include "ptx.cuh"

namespace qhtp {

namespace {

constexpr int kGroupK = 64;  // weights per scale group (along K)
constexpr int kGRows = 64;   // activation rows per tile (the MMA N)
// 1.5*2^52: the double whose bit pattern plus an integer Z (|Z| < 2^51) is the double 1.5*2^52 + Z
constexpr double kMagic = 6755399441055744.0;
constexpr int64_t kMagicBits = 0x4338000000000000ll;
constexpr int kGWRows = 2 * kGroupTileN;        // weight image rows per tile: [q 128 | e' 128]
constexpr int kGRecStage = 2 * kGroupRecBytes;  // the two groups of one 128-byte K block
constexpr int kEpiW = 16, kEpiW0 = 4;  // 16 drain warps: four per scheduler hide the TMEM-load latency
constexpr int kThreads = 32 * (kEpiW0 + kEpiW);
static_assert(kTileK == 2 * kGroupK, "a K block holds two groups");
static_assert(kGroupTileN == 128, "one TMEM lane per channel");

template <int PA>
struct GCfg {
  static constexpr int kStageW = kGWRows * kTileK;       // 32 KB: [q | e'] rows of 128 channels
  static constexpr int kStageX = kGRows * kTileK;        // 8 KB per activation plane
  static constexpr int kStage = kStageW + PA * kStageX;  // 48 KB (A16) / 40 KB (A8)
  static constexpr int kStages = 4;
  static constexpr int kSmem = kStages * (kStage + kGRecStage) + 1024 + 256;
};
static_assert(GCfg<2>::kSmem <= 227 * 1024 && GCfg<1>::kSmem <= 227 * 1024, "shared memory");

struct GroupParams {
  int M, N, m_tiles, n_tiles, kblocks, a_plane_rows;
  const uint8_t* grec;  // [n_tiles][kblocks][2 groups][K i64 x128 | 2^e f64 x128 | m i32 x128]
  const double* bias;   // [n_tiles * 128] float64 of the float32 bias
  void* out;
  double act_scale, out_scale;
  int zp_out, qmax;
  int* err;
};

template <int PA>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_group_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                       const GroupParams p) {
  using Cfg = GCfg<PA>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kBufCols = PA * 128;  // one group: per activation plane [q 64 rows | e' 64 rows]
  constexpr uint32_t NB = kTmemCols / kBufCols;  // group buffers in TMEM: 2 (A16), 4 (A8)

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* recs = smem + S * Cfg::kStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(recs + S * kGRecStage);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;    // [NB]: group buffer holds accumulators
  uint64_t* tempty = tfull + NB;  // [NB]: group buffer drained
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + NB);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + kEpiW);  // the MMAs have read the operands, every epilogue warp the constants
    }
    for (uint32_t b = 0; b < NB; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiW);
    }
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

  if (warp < kEpiW0) {
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      tma_prefetch_desc(&tmX);
      tma_prefetch_desc(&tmW);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % p.m_tiles) * kGRows;
        const int nt = tile / p.m_tiles;
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, p.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::kStage + kGRecStage);
          uint8_t* st = stages + s * Cfg::kStage;
          const size_t blk = static_cast<size_t>(nt) * p.kblocks + kb;
          tma_load_2d(st, &tmW, &full[s], 0, static_cast<int>(blk * kGWRows));
#pragma unroll
          for (int pl = 0; pl < PA; ++pl)
            tma_load_2d(st + Cfg::kStageW + pl * Cfg::kStageX, &tmX, &full[s], kb * kTileK, pl * p.a_plane_rows + m0);
          bulk_load(recs + s * kGRecStage, p.grec + blk * kGRecStage, kGRecStage, &full[s]);
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      constexpr uint32_t id = idesc_i8(128, kGRows, 1, 0);  // s8 weight rows x u8 activation rows
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1, p.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(stages + s * Cfg::kStage);
          const uint64_t dQ = desc_kmajor_sw128(st);                         // q rows of 128 channels
          const uint64_t dE = desc_kmajor_sw128(st + kGroupTileN * kTileK);  // e' rows
          const uint64_t dX0 = desc_kmajor_sw128(st + Cfg::kStageW);
          const uint64_t dX1 = desc_kmajor_sw128(st + Cfg::kStageW + (PA > 1 ? Cfg::kStageX : 0));
#pragma unroll
          for (int b = 0; b < 2; ++b) {  // group 2*kb + b -> TMEM buffer b
            const uint32_t gi = 2 * it + b, bf = gi % NB;  // group counter -> TMEM buffer
            if (!mbar_wait(&tempty[bf], ((gi / NB) & 1) ^ 1, p.err, kErrTimeoutOther)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem + bf * kBufCols;
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const uint64_t ko = static_cast<uint64_t>((2 * b + kk) * 2);  // 32 bytes, in 16-byte units
              const uint32_t accum = static_cast<uint32_t>(kk);
              mma_i8(d + 0, dQ + ko, dX0 + ko, id, accum);   // sum x(_hi) * q
              mma_i8(d + 64, dE + ko, dX0 + ko, id, accum);  // sum x(_hi) * e'
              if constexpr (PA == 2) {
                mma_i8(d + 128, dQ + ko, dX1 + ko, id, accum);  // sum x_lo * q
                mma_i8(d + 192, dE + ko, dX1 + ko, id, accum);  // sum x_lo * e'
              }
            }
            mma_commit(&tfull[bf]);
          }
          if (!ok) break;
          mma_commit(&empty[s]);  // operands read
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ drain + float64 accumulate
    const int quad = warp & 3;                 // TMEM lane quadrant: channels 32*quad .. +32
    const int rquart = (warp - kEpiW0) >> 2;   // rows 16*rquart .. +16 of the tile
    const int ch = quad * 32 + lane;           // this thread's channel within the tile
    const uint32_t tl = tmem + (static_cast<uint32_t>(quad * 32) << 16) + rquart * 16;
    const bool u16 = p.qmax > 255;
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      const int r0 = (tile % p.m_tiles) * kGRows + rquart * 16;
      const int n = (tile / p.m_tiles) * kGroupTileN + ch;
      double acc[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) acc[r] = 0.0;
      for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
        const int s = it % S;
        // Acquire the bulk copy of the stage's group constants on its own barrier.  The phase is
        // already complete (the MMAs of this stage waited on it) and cannot advance before this
        // warp arrives on empty[], so this returns at once.
        if (!mbar_wait(&full[s], (it / S) & 1, p.err, kErrTimeoutFull)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const uint8_t* rg = recs + s * kGRecStage + b * kGroupRecBytes;
          const int64_t kz = reinterpret_cast<const int64_t*>(rg)[ch];  // bits(1.5*2^52) - zero-point term
          const double sc = reinterpret_cast<const double*>(rg + 8 * kGroupTileN)[ch];   // 2^e
          const int32_t mg = reinterpret_cast<const int32_t*>(rg + 16 * kGroupTileN)[ch];  // m
          const uint32_t gi = 2 * it + b, bf = gi % NB;  // group counter -> TMEM buffer
          if (!mbar_wait(&tfull[bf], (gi / NB) & 1, p.err, kErrTimeoutAccum)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t tb = tl + bf * kBufCols;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t qh[8], eh[8], ql[8], el[8];
            tmem_ld8(tb + h * 8, qh);       // sum x(_hi) * q, rows 8h..
            tmem_ld8(tb + 64 + h * 8, eh);  // sum x(_hi) * e'
            if constexpr (PA == 2) {
              tmem_ld8(tb + 128 + h * 8, ql);  // sum x_lo * q
              tmem_ld8(tb + 192 + h * 8, el);  // sum x_lo * e'
            }
            tmem_ld_wait();
            if (h == 1) {  // buffer b fully in registers: the next group's MMAs may overwrite it
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&tempty[bf]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              int32_t pq, pe;
              if constexpr (PA == 2) {
                pq = static_cast<int32_t>(qh[j]) * 256 + static_cast<int32_t>(ql[j]);  // |.| < 2^26
                pe = static_cast<int32_t>(eh[j]) * 256 + static_cast<int32_t>(el[j]);
              } else {
                pq = static_cast<int32_t>(qh[j]);
                pe = static_cast<int32_t>(eh[j]);
              }
              // bits of the double 1.5*2^52 + Z; exact for |Z| < 2^51, and |Z| < 2^50 here
              const int64_t t = static_cast<int64_t>(mg) * pq + (kz + pe);
              const double z = __dsub_rn(__longlong_as_double(t), kMagic);  // Z, exact
              acc[h * 8 + j] = __fma_rn(z, sc, acc[h * 8 + j]);            // Z*2^e exact: one rounding
            }
          }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage's group constants
      }
      if (!ok) break;
      if (n < p.N) {
        const double bias = __ldg(p.bias + n);
#pragma unroll
        for (int r = 0; r < 16; ++r) {  // fully unrolled: acc[] stays in registers
          if (r0 + r < p.M) {
            const double y = __dadd_rn(__dmul_rn(p.act_scale, acc[r]), bias);
            double z = rint(__dadd_rn(__ddiv_rn(y, p.out_scale), static_cast<double>(p.zp_out)));
            z = fmin(fmax(z, 0.0), static_cast<double>(p.qmax));
            const size_t o = static_cast<size_t>(r0 + r) * p.N + n;  // a warp: 32 consecutive channels
            if (u16)
              reinterpret_cast<uint16_t*>(p.out)[o] = static_cast<uint16_t>(z);
            else
              reinterpret_cast<uint8_t*>(p.out)[o] = static_cast<uint8_t>(z);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int PA>
cudaError_t launch_group_variant(cudaStream_t stream, const CUtensorMap& tx, const CUtensorMap& tw,
                                 const GroupParams& prm, int sms) {
  using Cfg = GCfg<PA>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(qgemm_group_kernel<PA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmem);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const int total = prm.m_tiles * prm.n_tiles;
  const int grid = total < sms ? total : sms;
  qgemm_group_kernel<PA><<<grid, kThreads, Cfg::kSmem, stream>>>(tx, tw, prm);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------
// Prepare: one thread per (channel, group).  Writes the group's 64 q and 64 e' bytes into the
// pre-swizzled operand image of its (tile, K block) and the group's constants into its block.
// ------------------------------------------------------------------------------------------------
__global__ void prepare_group_kernel(const uint8_t* __restrict__ w4, const float* __restrict__ scale,
                                     const float* __restrict__ bias, uint32_t K, uint32_t N, uint32_t kblocks,
                                     int32_t act_zp, int8_t* __restrict__ planes, uint8_t* __restrict__ grec,
                                     double* __restrict__ bias_d, int* bad_scale) {
  const uint32_t G = K / kGroupK;
  const size_t total = static_cast<size_t>(N) * G;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint32_t n = static_cast<uint32_t>(idx / G), g = static_cast<uint32_t>(idx % G);
    const uint32_t bits = __float_as_uint(scale[idx]);  // scale [N, G] row-major: idx == n*G + g
    const uint32_t ex = (bits >> 23) & 0xFFu;
    const uint32_t tile = n / kGroupTileN, rr = n % kGroupTileN, kb = g / 2, half = g % 2;
    const size_t blk = static_cast<size_t>(tile) * kblocks + kb;
    uint8_t* rg = grec + blk * kGRecStage + half * kGroupRecBytes;
    if (g == 0) bias_d[n] = static_cast<double>(bias[n]);
    if ((bits >> 31) != 0 || ex == 0 || ex == 0xFF) {  // negative, zero/subnormal, inf/nan
      atomicCAS(bad_scale, 0, 1);
      continue;
    }
    const int32_t ms = static_cast<int32_t>((bits & 0x7FFFFFu) | 0x800000u);
    const int es = static_cast<int>(ex) - 150;  // scale = ms * 2^es
    int8_t* img = planes + blk * (kGWRows * kTileK);
    long long sq = 0, se = 0;
#pragma unroll 1
    for (uint32_t c4 = 0; c4 < 4; ++c4) {
      const uint32_t k0 = g * kGroupK + c4 * 16;
      const uint32_t c = half * 4 + c4;  // 16-byte chunk of the 128-byte K row
      int8_t* rq = img + rr * kTileK + (((c ^ rr) & 7u) << 4);
      int8_t* re = img + (kGroupTileN + rr) * kTileK + (((c ^ rr) & 7u) << 4);  // row 128+rr: same swizzle phase
#pragma unroll 4
      for (int j = 0; j < 16; ++j) {
        const uint32_t k = k0 + j;
        const uint8_t byte = w4[static_cast<size_t>(k >> 1) * N + n];  // K-pair carrier [K/2, N]
        int q = (k & 1) ? (byte >> 4) : (byte & 0xF);
        q = q >= 8 ? q - 16 : q;
        const int32_t prod = q * ms;                                 // |prod| < 2^28
        const int32_t rnd = __float2int_rz(__int2float_rn(prod));  // float32(q * scale), in units of 2^es
        const int e = rnd - prod;                                    // |e| <= 8
        rq[j] = static_cast<int8_t>(q);
        re[j] = static_cast<int8_t>(e);
        sq += q;
        se += e;
      }
    }
    reinterpret_cast<int64_t*>(rg)[rr] =
        kMagicBits - static_cast<int64_t>(act_zp) * (static_cast<int64_t>(ms) * sq + se);
    reinterpret_cast<double*>(rg + 8 * kGroupTileN)[rr] = ldexp(1.0, es);
    reinterpret_cast<int32_t*>(rg + 16 * kGroupTileN)[rr] = ms;
  }
}

}  // namespace

cudaError_t launch_prepare_group(const QhtpMatmulPlan* plan, const QhtpMatmulWeights* w, void* prepared,
                                 int* bad_scale, cudaStream_t stream, int sms) {
  uint8_t* base = static_cast<uint8_t*>(prepared);
  cudaError_t e = cudaMemsetAsync(base, 0, plan->prepared_bytes, stream);
  if (e != cudaSuccess) return e;
  const uint32_t kblocks = plan->k_pad / kTileK;
  uint8_t* grec = base + plan->plane_bytes;
  double* bias_d = reinterpret_cast<double*>(grec + group_rec_bytes(plan));
  const size_t total = static_cast<size_t>(plan->n) * (plan->k / kGroupK);
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > sms * 32) blocks = sms * 32;
  prepare_group_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(w->weight), w->weight_scale,
                                                   w->bias_float, plan->k, plan->n, kblocks, plan->act_zp,
                                                   reinterpret_cast<int8_t*>(base), grec, bias_d, bad_scale);
  return cudaGetLastError();
}

cudaError_t launch_gemm_group(const GemmLaunch& g, const uint8_t* a_base, uint64_t a_rows, int sms) {
  const QhtpMatmulPlan* pl = g.plan;
  CUtensorMap tx, tw;
  if (!make_tmap_2d_u8(&tx, a_base, pl->k, a_rows, pl->k, kTileK, kGRows)) return cudaErrorInvalidValue;
  const uint32_t kblocks = pl->k_pad / kTileK;
  const uint64_t wrows = static_cast<uint64_t>(pl->n_tiles) * kblocks * kGWRows;
  if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, pl->prepared, kTileK, wrows, kTileK, kTileK, kGWRows,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  const uint8_t* base = static_cast<const uint8_t*>(pl->prepared);
  GroupParams prm;
  prm.M = static_cast<int>(g.m);
  prm.N = static_cast<int>(pl->n);
  prm.m_tiles = static_cast<int>((g.m + kGRows - 1) / kGRows);
  prm.n_tiles = static_cast<int>(pl->n_tiles);
  prm.kblocks = static_cast<int>(kblocks);
  prm.a_plane_rows = static_cast<int>(g.m);
  prm.grec = base + pl->plane_bytes;
  prm.bias = reinterpret_cast<const double*>(base + pl->plane_bytes + group_rec_bytes(pl));
  prm.out = g.out;
  prm.act_scale = pl->act_scale;
  prm.out_scale = pl->out_scale;
  prm.zp_out = pl->out_zp;
  prm.qmax = pl->out_qmax;
  prm.err = g.err;
  return pl->a_planes == 2 ? launch_group_variant<2>(g.stream, tx, tw, prm, sms)
                           : launch_group_variant<1>(g.stream, tx, tw, prm, sms);
}

}  // namespace qhtp
