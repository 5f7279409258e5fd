// CHAIN=N quantized MatMul (the reference's chain graphs, gen_quant_chain.py:1346-1362 and :1542-1545:
// the same op applied `chain` times, each output code tensor feeding the next op as its activation),
// fused into one kernel: the requantized output of a step is written straight into shared memory as
// the next step's activation operand, so the intermediate results never reach HBM.
//
// Shape: K == N <= 256 (the reference's chain gates run at 256^3), any M.  Output rows are
// independent across the chain, so every 128-row block is its own thread-block cluster of
// ceil(N / 64) CTAs, CTA r owning output channels [64 r, 64 r + 64):
//   * the CTA's rows of the weight image (its 64 channels' q and e' rows -- or hi and lo bytes -- for
//     all of K) and its channel records stay resident in shared memory;
//   * each step: one thread issues the tcgen05 kind::i8 MMAs over K (N = 128: [q | e'] of the 64
//     channels), all 8 warps drain TMEM, requantize with the exact epilogue of qgemm_kernel (32
//     channels per thread), and write the codes as bytes [64 r, 64 r + 64) of every row of the next
//     step's activation image (u16: split into the hi and lo byte planes), into this CTA's shared
//     memory and through distributed shared memory into every other CTA's of the cluster; a cluster
//     barrier publishes them;
//   * the last step stores the codes to global memory.
// The requant work of a step, which bounds the kernel, is spread over N / 64 SMs per row block.
// Activation images are double-buffered: step s reads buffer s & 1 and writes buffer (s + 1) & 1.  A
// CTA writes a peer's buffer only after the cluster barrier that ends the previous step, which the
// peer reaches after its MMAs of that step completed, so no MMA still reads a buffer being written.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"
#include "ptx.cuh"
#include "requant.cuh"

namespace qhtp {
namespace {

constexpr int kChainThreads = 256;  // 8 warps: warp w drains TMEM lane quadrant w % 4, channels 32*(w/4)..
constexpr int kChainCh = 64;        // output channels per CTA
constexpr int kChainMaxCtas = 4;    // K == N <= 256
constexpr int kActBlock = kTileM * kTileK;  // 16 KB: one 128-row x 128-byte K block of one byte plane

struct ChainParams {
  int M, N, kblocks, a_plane_rows, chain;
  const ChannelRecord* rec;
  void* out;
  int zp_out, qmax;
  uint64_t act_mant, out_mant;
  int act_exp2, out_exp2;
  int* err;
};

template <int PA, int MODE>
struct ChainCfg {
  static constexpr int kImgRows = MODE == kModeExact ? 128 : 256;  // rows of a tile's weight image
  static constexpr int kBRows = MODE == kModeExact ? 64 : 128;     // this CTA's rows of it
  static constexpr int kWBlock = kBRows * kTileK;                  // one K block of them
  static constexpr int kActBuf(int kb) { return PA * kb * kActBlock; }
};

// Dynamic shared memory: weights + two activation images + records + barriers; at least 120 KB so
// that one CTA occupies an SM (its TMEM allocation is then never contended by a second CTA of this
// kernel).
template <int PA, int MODE>
constexpr int chain_smem_bytes(int kb) {
  const int b = kb * ChainCfg<PA, MODE>::kWBlock + 2 * ChainCfg<PA, MODE>::kActBuf(kb) + kChainCh * 32 + 64 + 1024;
  return b < 120 * 1024 ? 120 * 1024 : b;
}

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// 16 byte codes (one per channel) packed little-endian into a 16-byte vector
__device__ __forceinline__ uint4 pack16(const uint32_t (&b)[16]) {
  uint4 v;
  v.x = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
  v.y = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
  v.z = b[8] | (b[9] << 8) | (b[10] << 16) | (b[11] << 24);
  v.w = b[12] | (b[13] << 8) | (b[14] << 16) | (b[15] << 24);
  return v;
}

template <int PA, int MODE>
__global__ void __launch_bounds__(kChainThreads, 1)
    qchain_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const ChainParams p) {
  using Cfg = ChainCfg<PA, MODE>;
  const int KB = p.kblocks;                       // 128-byte K blocks (1 or 2)
  const int NC = static_cast<int>(gridDim.x) / ((p.M + kTileM - 1) / kTileM);  // CTAs per cluster
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wimg = smem;                                     // [KB][kBRows][128]
  uint8_t* act = wimg + KB * Cfg::kWBlock;                  // [2][PA][KB][128][128]
  ChannelRecord* rec_s = reinterpret_cast<ChannelRecord*>(act + 2 * Cfg::kActBuf(KB));
  uint64_t* load_bar = reinterpret_cast<uint64_t*>(rec_s + kChainCh);
  uint64_t* mma_bar = load_bar + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mma_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();        // this CTA's 64-channel slice
  const int rb = blockIdx.x / NC;                 // 128-row block
  const int quad = warp & 3, half = warp >> 2;
  const int row = quad * 32 + lane;               // TMEM lane = output row in the block
  const int m = rb * kTileM + row;
  const int tile = static_cast<int>(rank) >> 1, hsel = static_cast<int>(rank) & 1;  // image tile, its half

  if (threadIdx.x == 0) {
    mbar_init(load_bar, 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  // this slice's 64 channel records (2 KB) into shared memory
  for (int i = threadIdx.x; i < kChainCh * 2; i += kChainThreads)
    reinterpret_cast<uint4*>(rec_s)[i] = __ldg(reinterpret_cast<const uint4*>(p.rec + rank * kChainCh) + i);
  tc_fence_before();
  cluster_sync_all();  // barriers initialised, TMEM allocated, every CTA of the cluster running
  tc_fence_after();
  const uint32_t tmem = *tslot;

  bool ok = true;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    mbar_arrive_expect_tx(load_bar, KB * Cfg::kWBlock + PA * KB * kActBlock);
    for (int kb = 0; kb < KB; ++kb) {
      const int img = (tile * KB + kb) * Cfg::kImgRows + 64 * hsel;  // first row of this slice's q rows
      tma_load_2d(wimg + kb * Cfg::kWBlock, &tmB, load_bar, 0, img);
      if constexpr (Cfg::kBRows == 128)  // the e' (or lo-byte) rows of the same channels
        tma_load_2d(wimg + kb * Cfg::kWBlock + 64 * kTileK, &tmB, load_bar, 0, img + 128);
      for (int pl = 0; pl < PA; ++pl)
        tma_load_2d(act + (pl * KB + kb) * kActBlock, &tmA, load_bar, kb * kTileK, pl * p.a_plane_rows + rb * kTileM);
    }
    ok = mbar_wait(load_bar, 0, p.err, kErrTimeoutFull);
  }

  const bool u16 = p.qmax > 255;
  const uint32_t tl = tmem + (static_cast<uint32_t>(quad * 32) << 16);
  // the byte column of this slice's channels in the next activation's rows
  const int kb_out = static_cast<int>(rank) >> 1, col_out = 64 * (static_cast<int>(rank) & 1);
  for (int step = 0; step < p.chain; ++step) {
    const int bin = step & 1;
    // ---------------------------------------------------------------- MMAs of this step (one thread)
    if (threadIdx.x == 0) {
      tc_fence_after();
      if (ok) {
        const uint32_t abase = smem_u32(act + bin * Cfg::kActBuf(KB));
        for (int kb = 0; kb < KB; ++kb) {
          const uint64_t dA0 = desc_kmajor_sw128(abase + kb * kActBlock);
          const uint64_t dA1 = desc_kmajor_sw128(abase + ((PA - 1) * KB + kb) * kActBlock);
          const uint64_t dB = desc_kmajor_sw128(smem_u32(wimg + kb * Cfg::kWBlock));
#pragma unroll
          for (int kk = 0; kk < kTileK / 32; ++kk) {
            const uint32_t acc = (kb | kk) ? 1u : 0u;
            const uint64_t ko = static_cast<uint64_t>(kk * 2);
            if constexpr (MODE == kModeW16) {
              constexpr uint32_t idS = idesc_i8(128, 64, 0, 1);
              constexpr uint32_t idU = idesc_i8(128, 64, 0, 0);
              const uint64_t dBhi = dB + ko, dBlo = dB + ko + (64 * kTileK >> 4);
              mma_i8(tmem + 0, dA0 + ko, dBhi, idS, acc);
              mma_i8(tmem + 64, dA0 + ko, dBlo, idU, acc);
              mma_i8(tmem + 64, dA1 + ko, dBhi, idS, 1u);
              mma_i8(tmem + 128, dA1 + ko, dBlo, idU, acc);
            } else {
              constexpr int N = Cfg::kBRows;  // 128 = [q | e'] of 64 channels (f32 mode), 64 = q (exact mode)
              constexpr uint32_t id = idesc_i8(128, N, 0, 1);
              mma_i8(tmem + 0, dA0 + ko, dB + ko, id, acc);
              if constexpr (PA == 2) mma_i8(tmem + N, dA1 + ko, dB + ko, id, acc);
            }
          }
        }
      }
      mma_commit(mma_bar);
    }
    // ---------------------------------------------------------------- epilogue (all 8 warps)
    mbar_wait(mma_bar, step & 1, p.err, kErrTimeoutAccum);
    tc_fence_after();
    const bool last = step == p.chain - 1;
    const uint32_t obase = smem_u32(act + (bin ^ 1) * Cfg::kActBuf(KB));
#pragma unroll 1
    for (int g = 0; g < 2; ++g) {
      const int c0 = half * 32 + g * 16;  // first of this group's 16 channels within the slice
      int64_t T[16];
      {
        uint32_t a0[16], a1[16], a2[16], a3[16];
        tmem_ld16(tl + c0, a0);
        if constexpr (MODE == kModeF32) {
          tmem_ld16(tl + c0 + 64, a1);
          if constexpr (PA == 2) {
            tmem_ld16(tl + c0 + 128, a2);
            tmem_ld16(tl + c0 + 192, a3);
          }
        } else if constexpr (MODE == kModeW16) {
          tmem_ld16(tl + c0 + 64, a1);
          tmem_ld16(tl + c0 + 128, a2);
        } else if constexpr (PA == 2) {
          tmem_ld16(tl + c0 + 64, a1);
        }
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int64_t s0 = static_cast<int32_t>(a0[j]);
          if constexpr (MODE == kModeF32) {
            const int64_t mq = rec_s[c0 + j].m_q;
            if constexpr (PA == 2) {
              T[j] = mq * (s0 * 256 + static_cast<int32_t>(a2[j])) +
                     (static_cast<int64_t>(static_cast<int32_t>(a1[j])) * 256 + static_cast<int32_t>(a3[j]));
            } else {
              T[j] = mq * s0 + static_cast<int32_t>(a1[j]);
            }
          } else if constexpr (MODE == kModeW16) {
            T[j] = s0 * 65536 + static_cast<int64_t>(static_cast<int32_t>(a1[j])) * 256 + static_cast<int32_t>(a2[j]);
          } else if constexpr (PA == 2) {
            T[j] = s0 * 256 + static_cast<int32_t>(a1[j]);
          } else {
            T[j] = s0;
          }
        }
      }
      uint32_t code[16];
      const int n_first = static_cast<int>(rank) * kChainCh + c0;
      const bool real = n_first < p.N;  // 16-channel groups lie wholly inside or past N (N % 32 == 0)
      if (real) {
        uint32_t near_mask = 0;
        int64_t wv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const ChannelRecord& r = rec_s[c0 + j];
          T[j] += r.beff;
          bool nr;
          code[j] = static_cast<uint32_t>(requant_fast96s(T[j], r.cmn, r.tn, p.zp_out, p.qmax, &nr, &wv[j]));
          near_mask |= nr ? (1u << j) : 0u;
        }
        if (near_mask != 0) {
          for (int j = 0; j < 16; ++j) {
            if (near_mask & (1u << j)) {
              const uint32_t wb = rec_s[c0 + j].wbits;
              const uint32_t ms = (wb & 0x7FFFFFu) | 0x800000u;
              const int es = static_cast<int>((wb >> 23) & 0xFFu) - 150;
              const uint32_t mul = MODE == kModeF32 ? 1u : ms;
              code[j] = static_cast<uint32_t>(requant_tie_w(T[j], wv[j], mul, es + p.act_exp2, p.act_mant, p.out_mant,
                                                          p.out_exp2, p.zp_out, p.qmax));
            }
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) code[j] = 0;
      }
      if (!last) {
        // next activation: K block kb_out, bytes col_out + c0 .. +15 of row `row` (one swizzled
        // 16-byte chunk), here and in every other CTA of the cluster
        const int chunk = (col_out + c0) >> 4;
        const uint32_t off = static_cast<uint32_t>(kb_out * kActBlock + row * kTileK + (((chunk ^ row) & 7) << 4));
        uint32_t hb[16], lb[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          hb[j] = u16 ? (code[j] >> 8) : code[j];
          lb[j] = code[j] & 0xFFu;
        }
        const uint4 vh = pack16(hb);
        const uint32_t a_hi = obase + off;
        st_shared_v4(a_hi, vh);
        for (int r = 0; r < NC; ++r)
          if (r != static_cast<int>(rank)) st_cluster_v4(mapa_shared(a_hi, static_cast<uint32_t>(r)), vh);
        if constexpr (PA == 2) {
          const uint4 vl = pack16(lb);
          const uint32_t a_lo = obase + KB * kActBlock + off;
          st_shared_v4(a_lo, vl);
          for (int r = 0; r < NC; ++r)
            if (r != static_cast<int>(rank)) st_cluster_v4(mapa_shared(a_lo, static_cast<uint32_t>(r)), vl);
        }
      } else if (real && m < p.M) {
        const size_t o = static_cast<size_t>(m) * p.N + n_first;
        if (u16) {
          uint4 v0, v1;
          v0.x = code[0] | (code[1] << 16);
          v0.y = code[2] | (code[3] << 16);
          v0.z = code[4] | (code[5] << 16);
          v0.w = code[6] | (code[7] << 16);
          v1.x = code[8] | (code[9] << 16);
          v1.y = code[10] | (code[11] << 16);
          v1.z = code[12] | (code[13] << 16);
          v1.w = code[14] | (code[15] << 16);
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + o);
          dst[0] = v0;
          dst[1] = v1;
        } else {
          uint32_t b[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) b[j] = code[j];
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.out) + o) = pack16(b);
        }
      }
    }
    // every TMEM read of this step is done and the next activation is in place (every CTA): the
    // generic-proxy shared-memory writes are made visible to the tensor core's async proxy
    tc_fence_before();
    asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
    cluster_sync_all();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

template <int PA, int MODE>
cudaError_t launch_chain_variant(const CUtensorMap& ta, const CUtensorMap& tb, const ChainParams& prm, int m_blocks,
                                 int ctas, cudaStream_t stream) {
  const int smem = chain_smem_bytes<PA, MODE>(prm.kblocks);
  cudaError_t e = cudaFuncSetAttribute(qchain_kernel<PA, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(m_blocks * ctas), 1, 1);
  cfg.blockDim = dim3(kChainThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(ctas);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qchain_kernel<PA, MODE>, ta, tb, prm);
}

}  // namespace

bool chain_fusable(const QhtpMatmulPlan* pl) {
  return pl->mode != kModeGroup && pl->k == pl->n && pl->n <= kChainMaxCtas * kChainCh && pl->act_bits == pl->out_bits &&
         pl->k_pad / kTileK == pl->n_tiles;
}

cudaError_t launch_chain(const GemmLaunch& g, uint32_t chain) {
  const QhtpMatmulPlan* pl = g.plan;
  const uint32_t K = pl->k;
  const uint8_t* a_base;
  uint64_t a_rows;
  if (pl->a_planes == 2) {
    cudaError_t e = launch_split_u16(static_cast<const uint16_t*>(g.act), g.planes, static_cast<size_t>(g.m) * K,
                                     g.stream);
    if (e != cudaSuccess) return e;
    a_base = g.planes;
    a_rows = 2ull * g.m;
  } else {
    a_base = static_cast<const uint8_t*>(g.act);
    a_rows = g.m;
  }
  CUtensorMap ta, tb;
  if (!make_tmap_2d_u8(&ta, a_base, K, a_rows, K, kTileK, kTileM)) return cudaErrorInvalidValue;
  // the weight images as 64-row boxes: one CTA's q (or hi-byte) rows, then its e' (or lo-byte) rows
  const uint64_t img_rows = static_cast<uint64_t>(pl->n_tiles) * (pl->k_pad / kTileK) * b_rows_for_mode(pl->mode);
  if (!make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, pl->prepared, kTileK, img_rows, kTileK, kTileK, 64,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  ChainParams prm;
  prm.M = static_cast<int>(g.m);
  prm.N = static_cast<int>(pl->n);
  prm.kblocks = static_cast<int>(pl->n_tiles);
  prm.a_plane_rows = static_cast<int>(g.m);
  prm.chain = static_cast<int>(chain);
  prm.rec = reinterpret_cast<const ChannelRecord*>(static_cast<const uint8_t*>(pl->prepared) + pl->plane_bytes);
  prm.out = g.out;
  prm.zp_out = pl->out_zp;
  prm.qmax = pl->out_qmax;
  prm.act_mant = pl->act_mant;
  prm.out_mant = pl->out_mant;
  prm.act_exp2 = pl->act_exp2;
  prm.out_exp2 = pl->out_exp2;
  prm.err = g.err;
  const int m_blocks = static_cast<int>((g.m + kTileM - 1) / kTileM);
  const int ctas = static_cast<int>((pl->n + kChainCh - 1) / kChainCh);
  switch (pl->mode * 2 + (pl->a_planes - 1)) {
    case kModeF32 * 2 + 0: return launch_chain_variant<1, kModeF32>(ta, tb, prm, m_blocks, ctas, g.stream);
    case kModeF32 * 2 + 1: return launch_chain_variant<2, kModeF32>(ta, tb, prm, m_blocks, ctas, g.stream);
    case kModeExact * 2 + 0: return launch_chain_variant<1, kModeExact>(ta, tb, prm, m_blocks, ctas, g.stream);
    case kModeExact * 2 + 1: return launch_chain_variant<2, kModeExact>(ta, tb, prm, m_blocks, ctas, g.stream);
    case kModeW16 * 2 + 1: return launch_chain_variant<2, kModeW16>(ta, tb, prm, m_blocks, ctas, g.stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qhtp
