// Decode-shaped quantized GEMM (few activation rows, M <= 128) on B200.
//
// Same operation and exactness model as qgemm.cu (HmxU16I4ToU16MatMul and the rest of the QNN
// MatMul family, requant as generate_qnn_matmul_python_cases.py:426-525), with the roles of the
// operands swapped for small M:
//   D[ch, tok] = sum_k W[ch, k] * X[tok, k]
// The 128 output channels of a weight tile are the MMA's M = 128 (one TMEM lane per channel) and
// the M activation rows are its N (16, 32, 64 or 128 columns), so for small M the tensor work per
// weight byte is N/128 of the row-tiled kernel's and the kernel is bound by streaming the prepared
// weight planes.
// The prepared planes are used as they are: for each 128-channel tile, rows [q | e'] (f32 weight
// dequant), [q] (exact dequant) or [hi | lo] (int16 weights), K contiguous, which is the K-major
// A operand; the activation (u8, or the hi/lo byte planes of u16) is the K-major B operand.
//
// Weight tiles alone (N/128 of them) cannot fill 148 SMs for N = 4096, so K is split over the CTAs
// of a thread-block cluster.  Each CTA accumulates its K range in TMEM and parks its int32 partial
// accumulators in its own shared memory; then each CTA sums one slice of the activation rows over
// the whole cluster through distributed shared memory and requantizes that slice.  The int32 plane sums are exact for the
// supported K (<= 32768), so the split changes no output bit.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocation + MMA issue, warps 2..5
// epilogue (TMEM lane quadrants 2, 3, 0, 1).  Every mbarrier wait is bounded.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"
#include "requant.cuh"

namespace qhtp {

namespace {

constexpr int kDecThreads = 192;
constexpr int kDecEpiWarp0 = 2;

struct DecodeParams {
  int M, N, kblocks, splits;
  const ChannelRecord* rec;
  void* out;
  int zp_out, qmax;
  uint64_t act_mant, out_mant;
  int act_exp2, out_exp2;
  int* err;
};

// Accumulators per mode and activation-plane count (TMEM column groups of MP columns each).
template <int MODE, int PA>
struct DecAcc {
  static constexpr int kWPlanes = MODE == kModeExact ? 1 : 2;  // weight planes per tile
  static constexpr int kAcc = MODE == kModeW16 ? 3 : kWPlanes * PA;
};

template <int MODE, int PA, int MP>
struct DecCfg {
  static constexpr int kAcc = DecAcc<MODE, PA>::kAcc;
  static constexpr int kWRows = 128 * DecAcc<MODE, PA>::kWPlanes;
  static constexpr int kStageW = kWRows * kTileK;    // weight planes of one 128-deep K block
  static constexpr int kStageX = MP * kTileK;        // one activation plane
  static constexpr int kStage = kStageW + PA * kStageX;
  static constexpr int kStages = (192 * 1024) / kStage > 8 ? 8 : (192 * 1024) / kStage;
  static constexpr int kRound = MP < 64 ? MP : 64;           // activation rows reduced per round
  static constexpr int kRedBytes = kAcc * kRound * 128 * 4;  // int32 partials of one round
  static constexpr int kPipeBytes = kStages * kStage;
  static constexpr int kSmem = (kPipeBytes > kRedBytes ? kPipeBytes : kRedBytes) + 1024 + 256;
  static constexpr uint32_t kTmemCols =
      kAcc * MP <= 32 ? 32 : (kAcc * MP <= 64 ? 64 : (kAcc * MP <= 128 ? 128 : (kAcc * MP <= 256 ? 256 : 512)));
  static_assert(kAcc * MP <= 512, "accumulators exceed TMEM");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
// Plain (non-volatile) load from distributed shared memory: ordering against the partial-sum stores
// comes from the cluster barrier, so independent loads may be scheduled together.
__device__ __forceinline__ int4 ld_cluster_v4(uint32_t addr) {
  int4 v;
  asm("ld.shared::cluster.v4.s32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// Requant constants of one output channel (its prepared record).
struct ChanConst {
  int64_t beff, mq;
  uint64_t cmn;
  int tn, es;
  uint32_t mul;
};

template <int MODE>
__device__ __forceinline__ ChanConst load_chan(const ChannelRecord* rc) {
  ChanConst c;
  c.beff = rc->beff;
  c.cmn = rc->cmn;
  c.tn = rc->tn;
  c.mq = rc->m_q;
  const uint32_t wb = rc->wbits;
  c.es = static_cast<int>((wb >> 23) & 0xFFu) - 150;
  c.mul = MODE == kModeF32 ? 1u : ((wb & 0x7FFFFFu) | 0x800000u);
  return c;
}

// One output code from the int32 plane accumulators of one (row, channel): the accumulator T of
// the exactness model (same combination as the row-tiled kernel), then the exact requant.
template <int MODE, int PA, int NA>
__device__ __forceinline__ uint32_t requant_one(const int32_t (&a)[NA], const ChanConst& c, const DecodeParams& p) {
  int64_t T;
  if constexpr (MODE == kModeF32) {
    int64_t pq = a[0], pe = a[1];
    if constexpr (PA == 2) {
      pq = pq * 256 + a[2];
      pe = pe * 256 + a[3];
    }
    T = c.mq * pq + pe + c.beff;
  } else if constexpr (MODE == kModeExact) {
    int64_t pq = a[0];
    if constexpr (PA == 2) pq = pq * 256 + a[1];
    T = pq + c.beff;
  } else {
    T = static_cast<int64_t>(a[0]) * 65536 + static_cast<int64_t>(a[1]) * 256 + a[2] + c.beff;
  }
  bool near = false;
  int64_t fl = 0;
  int32_t code = requant_fast96s(T, c.cmn, c.tn, p.zp_out, p.qmax, &near, &fl);
  if (near) code = requant_tie_w(T, fl, c.mul, c.es + p.act_exp2, p.act_mant, p.out_mant, p.out_exp2, p.zp_out, p.qmax);
  return static_cast<uint32_t>(code);
}

template <int MODE, int PA, int MP>
__global__ void __launch_bounds__(kDecThreads, 1)
    qdecode_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                   const DecodeParams p) {
  using Cfg = DecCfg<MODE, PA, MP>;
  constexpr int S = Cfg::kStages;
  constexpr int NA = Cfg::kAcc;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int red_region = Cfg::kPipeBytes > Cfg::kRedBytes ? Cfg::kPipeBytes : Cfg::kRedBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + red_region);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tfull + 1);
  int32_t* red = reinterpret_cast<int32_t*>(smem);  // [acc][tok][ch] partials (after the K loop)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int splits = p.splits;
  const uint32_t crank = splits > 1 ? cluster_rank() : 0u;
  const int tile = blockIdx.x / splits;
  const int kb0 = static_cast<int>((static_cast<int64_t>(p.kblocks) * crank) / splits);
  const int kb1 = static_cast<int>((static_cast<int64_t>(p.kblocks) * (crank + 1)) / splits);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  bool ok = true;
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmX);
      tma_prefetch_desc(&tmW);
      // The weight planes of the first stages load before the activation is awaited (the u16 plane
      // split runs just before, launched with programmatic dependent launch; a no-op wait otherwise).
      const int D = (kb1 - kb0) < S ? (kb1 - kb0) : S;
      for (int d = 0; d < D; ++d) {
        mbar_arrive_expect_tx(&full[d], Cfg::kStage);
        tma_load_2d(smem + d * Cfg::kStage, &tmW, &full[d], 0, (tile * p.kblocks + kb0 + d) * Cfg::kWRows);
      }
      griddep_wait();
      for (int d = 0; d < D; ++d) {
#pragma unroll
        for (int pl = 0; pl < PA; ++pl)
          tma_load_2d(smem + d * Cfg::kStage + Cfg::kStageW + pl * Cfg::kStageX, &tmX, &full[d], (kb0 + d) * kTileK,
                      pl * p.M);
      }
      int i = D;
      for (int kb = kb0 + D; kb < kb1; ++kb, ++i) {
        const int s = i % S;
        if (!mbar_wait(&empty[s], ((i / S) & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&full[s], Cfg::kStage);
        uint8_t* st = smem + s * Cfg::kStage;
        tma_load_2d(st, &tmW, &full[s], 0, (tile * p.kblocks + kb) * Cfg::kWRows);
#pragma unroll
        for (int pl = 0; pl < PA; ++pl)
          tma_load_2d(st + Cfg::kStageW + pl * Cfg::kStageX, &tmX, &full[s], kb * kTileK, pl * p.M);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int i = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++i) {
        const int s = i % S;
        if (!mbar_wait(&full[s], (i / S) & 1, p.err, kErrTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * Cfg::kStage);
        const uint64_t dW0 = desc_kmajor_sw128(st);
        const uint64_t dW1 = desc_kmajor_sw128(st + 128 * kTileK);
        const uint64_t dX0 = desc_kmajor_sw128(st + Cfg::kStageW);
        const uint64_t dX1 = desc_kmajor_sw128(st + Cfg::kStageW + (PA > 1 ? Cfg::kStageX : 0));
#pragma unroll
        for (int kk = 0; kk < kTileK / 32; ++kk) {
          const uint32_t acc = (i | kk) ? 1u : 0u;
          const uint64_t ko = static_cast<uint64_t>(kk * 2);  // 32 bytes, in 16-byte units
          if constexpr (MODE == kModeW16) {
            constexpr uint32_t idS = idesc_i8(128, MP, 1, 0);  // s8 hi-byte weight x u8 act
            constexpr uint32_t idU = idesc_i8(128, MP, 0, 0);  // u8 lo-byte weight x u8 act
            mma_i8(tmem + 0 * MP, dW0 + ko, dX0 + ko, idS, acc);   // hi x hi
            mma_i8(tmem + 1 * MP, dW0 + ko, dX1 + ko, idS, acc);   // hi x lo
            mma_i8(tmem + 1 * MP, dW1 + ko, dX0 + ko, idU, 1u);    // + lo x hi
            mma_i8(tmem + 2 * MP, dW1 + ko, dX1 + ko, idU, acc);   // lo x lo
          } else {
            constexpr uint32_t id = idesc_i8(128, MP, 1, 0);       // s8 weight x u8 act
            mma_i8(tmem + 0 * MP, dW0 + ko, dX0 + ko, id, acc);                     // q x x(_hi)
            if constexpr (MODE == kModeF32) mma_i8(tmem + 1 * MP, dW1 + ko, dX0 + ko, id, acc);  // e' x x(_hi)
            if constexpr (PA == 2) {
              constexpr int lo = MODE == kModeF32 ? 2 : 1;
              mma_i8(tmem + lo * MP, dW0 + ko, dX1 + ko, id, acc);                  // q x x_lo
              if constexpr (MODE == kModeF32) mma_i8(tmem + 3 * MP, dW1 + ko, dX1 + ko, id, acc);
            }
          }
        }
        mma_commit(&empty[s]);
      }
      if (ok) mma_commit(tfull);
    }
  }

  // All MMAs of this CTA complete (or it gave up) before the pipeline buffers turn into the
  // partial-sum area.
  const bool is_epi = warp >= kDecEpiWarp0;
  const int quad = warp & 3;
  const int ch_local = quad * 32 + lane;                       // TMEM lane = channel in the tile
  const uint32_t tl = tmem + (static_cast<uint32_t>(quad * 32) << 16);
  // The channel constants load while the MMAs run (the epilogue warps are idle until then): channel
  // ch_local without a K split, channels c4..c4+3 (the reduce step's layout) with one.
  const int c4 = 4 * lane;
  ChanConst cc, cc4[4];
  bool cok[4];
  if (splits == 1) {
    const int n = tile * 128 + ch_local;
    cc = load_chan<MODE>(p.rec + (is_epi && n < p.N ? n : 0));
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = tile * 128 + c4 + i;
      cok[i] = is_epi && n < p.N;
      cc4[i] = load_chan<MODE>(p.rec + (cok[i] ? n : 0));
    }
  }
  if (is_epi) {
    ok = mbar_wait(tfull, 0, p.err, kErrTimeoutAccum);
    tc_fence_after();
  }
  __syncthreads();

  const bool u16 = p.qmax > 255;

  if (splits == 1) {
    // ---------------------------------------------------------------- whole K here: TMEM -> requant
    // (one channel per epilogue thread, all activation rows)
    const int n = tile * 128 + ch_local;
    if (is_epi && n < p.N) {
#pragma unroll 1
      for (int t0 = 0; t0 < MP && t0 < p.M; t0 += 16) {
        uint32_t v[NA][16];
#pragma unroll
        for (int g = 0; g < NA; ++g) tmem_ld16(tl + g * MP + t0, v[g]);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (t0 + j >= p.M) break;
          int32_t a[NA];
#pragma unroll
          for (int g = 0; g < NA; ++g) a[g] = ok ? static_cast<int32_t>(v[g][j]) : 0;
          const uint32_t code = requant_one<MODE, PA, NA>(a, cc, p);
          if (u16)
            reinterpret_cast<uint16_t*>(p.out)[static_cast<size_t>(t0 + j) * p.N + n] = static_cast<uint16_t>(code);
          else
            reinterpret_cast<uint8_t*>(p.out)[static_cast<size_t>(t0 + j) * p.N + n] = static_cast<uint8_t>(code);
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- K split over the cluster:
    // in rounds of kRound activation rows, every CTA parks its int32 partials [acc][row][ch] in its
    // own shared memory; then CTA r sums rows [r*kRound/S, (r+1)*kRound/S) of the round over all
    // CTAs through distributed shared memory and requantizes them.  In that step each epilogue warp
    // takes whole rows and each lane four adjacent channels (16-byte loads, every peer's loads of
    // a row issued before they are summed).
    constexpr int RT = Cfg::kRound;
    const int ew = warp - kDecEpiWarp0;           // 0..3 for the epilogue warps
    const uint32_t red_s = smem_u32(red);
    uint32_t peer[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) peer[r] = map_to_rank(red_s, static_cast<uint32_t>(r < splits ? r : 0));
#pragma unroll 1
    for (int rb = 0; rb < MP; rb += RT) {
      if (rb > 0) cluster_sync();  // the previous round's partials have been read everywhere
      if (is_epi) {
#pragma unroll 1
        for (int g = 0; g < NA; ++g) {
#pragma unroll 1
          for (int c0 = 0; c0 < RT; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(tl + g * MP + rb + c0, v);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) red[(g * RT + c0 + j) * 128 + ch_local] = ok ? static_cast<int32_t>(v[j]) : 0;
          }
        }
      }
      cluster_sync();  // every CTA's partials of this round are visible cluster-wide
      if (is_epi && tile * 128 + c4 < p.N) {
        const int per = RT / splits;
        const int tb = rb + static_cast<int>(crank) * per;
#pragma unroll 1
        for (int ti = ew; ti < per && tb + ti < p.M; ti += 4) {
          const int tok = tb + ti;
          const uint32_t off = static_cast<uint32_t>(((tok - rb) * 128 + c4) * 4);
          int4 v[8][NA];
#pragma unroll
          for (int r = 0; r < 8; ++r)
            if (r < splits) {
#pragma unroll
              for (int g = 0; g < NA; ++g) v[r][g] = ld_cluster_v4(peer[r] + off + static_cast<uint32_t>(g * RT * 128 * 4));
            }
          int32_t a[4][NA];
#pragma unroll
          for (int g = 0; g < NA; ++g) {
            a[0][g] = a[1][g] = a[2][g] = a[3][g] = 0;
#pragma unroll
            for (int r = 0; r < 8; ++r)
              if (r < splits) {
                a[0][g] += v[r][g].x;
                a[1][g] += v[r][g].y;
                a[2][g] += v[r][g].z;
                a[3][g] += v[r][g].w;
              }
          }
          uint32_t code[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) code[i] = requant_one<MODE, PA, NA>(a[i], cc4[i], p);
          const size_t o = static_cast<size_t>(tok) * p.N + tile * 128 + c4;
          if (cok[3]) {  // all four channels exist (N is a multiple of 32)
            if (u16)
              *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p.out) + o) =
                  make_uint2(code[0] | (code[1] << 16), code[2] | (code[3] << 16));
            else
              *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(p.out) + o) =
                  code[0] | (code[1] << 8) | (code[2] << 16) | (code[3] << 24);
          }
        }
      }
    }
    cluster_sync();  // no CTA leaves while others may still read its partials
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

int sm_count_dec() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// K splits: enough CTAs to cover the SMs, each keeping at least 4 K blocks, at most 8 (portable
// cluster size), and only where the partial-sum area fits in shared memory.
int choose_splits(int n_tiles, int kblocks) {
  const int sms = sm_count_dec();
  int s = 1;
  while (s < 8 && n_tiles * (s * 2) <= sms + sms / 4 && kblocks / (s * 2) >= 4) s *= 2;
  return s;
}

template <int MODE, int PA, int MP>
cudaError_t launch_dec(const CUtensorMap& tx, const CUtensorMap& tw, DecodeParams prm, int n_tiles,
                       cudaStream_t stream) {
  using Cfg = DecCfg<MODE, PA, MP>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(qdecode_kernel<MODE, PA, MP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg::kSmem);
  });
  if (attr_err != cudaSuccess) return attr_err;
  prm.splits = choose_splits(n_tiles, prm.kblocks);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n_tiles * prm.splits), 1, 1);
  cfg.blockDim = dim3(kDecThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(prm.splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = PA == 2 ? 2 : 1;  // dependent launch only behind this library's own plane split
  return cudaLaunchKernelEx(&cfg, qdecode_kernel<MODE, PA, MP>, tx, tw, prm);
}

template <int MODE, int PA>
cudaError_t launch_dec_mp(int mp, const CUtensorMap& tx, const CUtensorMap& tw, const DecodeParams& prm,
                          int n_tiles, cudaStream_t stream) {
  switch (mp) {
    case 16: return launch_dec<MODE, PA, 16>(tx, tw, prm, n_tiles, stream);
    case 32: return launch_dec<MODE, PA, 32>(tx, tw, prm, n_tiles, stream);
    case 64: return launch_dec<MODE, PA, 64>(tx, tw, prm, n_tiles, stream);
    case 128: return launch_dec<MODE, PA, 128>(tx, tw, prm, n_tiles, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool decode_supported(const QhtpMatmulPlan* plan, uint32_t m) {
  if (m == 0 || m > kDecodeMaxM) return false;
  // Above 64 rows with channel tiles enough to occupy the SMs without a K split, the row-tiled
  // kernel is faster (W4A16 LPBQ K=4096, M=128: N=14336 42.0 us vs 46.4 us; N=4096, 32 tiles, the
  // split decode kernel 30.9 us vs 37.9 us)
  if (m > 64 && 2 * static_cast<int>(plan->n_tiles) > sm_count_dec()) return false;
  if (plan->mode == kModeW16 && plan->a_planes != 2) return false;
  return true;
}

cudaError_t launch_decode(const GemmLaunch& g, const uint8_t* a_base) {
  const QhtpMatmulPlan* pl = g.plan;
  const int mp = g.m <= 16 ? 16 : (g.m <= 32 ? 32 : (g.m <= 64 ? 64 : 128));
  CUtensorMap tx, tw;
  const uint64_t x_rows = static_cast<uint64_t>(g.m) * pl->a_planes;
  if (!make_tmap_2d_u8(&tx, a_base, pl->k, x_rows, pl->k, kTileK, static_cast<uint32_t>(mp)))
    return cudaErrorInvalidValue;
  const uint8_t* planes = static_cast<const uint8_t*>(pl->prepared);
  if (!make_tmap_planes(&tw, pl)) return cudaErrorInvalidValue;
  DecodeParams prm;
  prm.M = static_cast<int>(g.m);
  prm.N = static_cast<int>(pl->n);
  prm.kblocks = static_cast<int>(pl->k_pad / kTileK);
  prm.splits = 1;
  prm.rec = reinterpret_cast<const ChannelRecord*>(planes + pl->plane_bytes);
  prm.out = g.out;
  prm.zp_out = pl->out_zp;
  prm.qmax = pl->out_qmax;
  prm.act_mant = pl->act_mant;
  prm.out_mant = pl->out_mant;
  prm.act_exp2 = pl->act_exp2;
  prm.out_exp2 = pl->out_exp2;
  prm.err = g.err;
  const int n_tiles = static_cast<int>(pl->n_tiles);
  switch (pl->mode * 2 + (pl->a_planes - 1)) {
    case kModeF32 * 2 + 0: return launch_dec_mp<kModeF32, 1>(mp, tx, tw, prm, n_tiles, g.stream);
    case kModeF32 * 2 + 1: return launch_dec_mp<kModeF32, 2>(mp, tx, tw, prm, n_tiles, g.stream);
    case kModeExact * 2 + 0: return launch_dec_mp<kModeExact, 1>(mp, tx, tw, prm, n_tiles, g.stream);
    case kModeExact * 2 + 1: return launch_dec_mp<kModeExact, 2>(mp, tx, tw, prm, n_tiles, g.stream);
    case kModeW16 * 2 + 1: return launch_dec_mp<kModeW16, 2>(mp, tx, tw, prm, n_tiles, g.stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qhtp
