// CHAIN=N quantized MatMul (the reference's chain graphs, gen_quant_chain.py:1346-1362 and :1542-1545:
// the same op applied `chain` times, each output code tensor feeding the next op as its activation),
// fused into one kernel: the requantized output of a step is written straight into shared memory as
// the next step's activation operand, so the intermediate results never reach HBM.
//
// Shape: K == N <= 256 (one or two 128-channel tiles; the reference's chain gates run at 256^3),
// any M.  Output rows are independent across the chain, so every 128-row block is its own
// thread-block cluster of n_tiles CTAs, CTA t owning output channels [128 t, 128 t + 128):
//   * the CTA's weight planes (all of K) and channel records stay resident in shared memory;
//   * each step: one thread issues the tcgen05 kind::i8 MMAs over K (accumulators in TMEM, the
//     same operand images and TMEM layout as qgemm_kernel), all 8 warps drain TMEM, requantize with
//     the exact epilogue of qgemm_kernel, and write the codes as the K block t of the next step's
//     activation image (u16: split into the hi and lo byte planes), into this CTA's shared memory and
//     through distributed shared memory into the peer CTA's; a cluster barrier publishes them;
//   * the last step stores the codes to global memory.
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

constexpr int kChainThreads = 256;  // 8 warps: warp w drains TMEM lane quadrant w % 4, channels 64*(w/4)..
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
  static constexpr int kBRows = MODE == kModeExact ? 128 : 256;
  static constexpr int kWBlock = kBRows * kTileK;  // one K block of the weight image
  static constexpr int kActBuf(int kb) { return PA * kb * kActBlock; }
};

// bytes of dynamic shared memory: weights + two activation images + records + barriers; at least
// 120 KB so that one CTA occupies an SM (the TMEM allocation of 512 columns is then never contended
// by a second CTA of this kernel)
template <int PA, int MODE>
constexpr int chain_smem_bytes(int kb) {
  const int b = kb * ChainCfg<PA, MODE>::kWBlock + 2 * ChainCfg<PA, MODE>::kActBuf(kb) + kTileN * 32 + 64 + 1024;
  return b < 120 * 1024 ? 120 * 1024 : b;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_peer(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
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
  const int KB = p.kblocks;  // == number of channel tiles == cluster size
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wimg = smem;                                     // [KB][kBRows][128]
  uint8_t* act = wimg + KB * Cfg::kWBlock;                  // [2][PA][KB][128][128]
  ChannelRecord* rec_s = reinterpret_cast<ChannelRecord*>(act + 2 * Cfg::kActBuf(KB));
  uint64_t* load_bar = reinterpret_cast<uint64_t*>(rec_s + kTileN);
  uint64_t* mma_bar = load_bar + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mma_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ct = cluster_rank();                       // this CTA's channel tile
  const int rb = blockIdx.x / KB;                           // 128-row block
  const int quad = warp & 3, half = warp >> 2;
  const int row = quad * 32 + lane;                         // TMEM lane = output row in the block
  const int m = rb * kTileM + row;

  if (threadIdx.x == 0) {
    mbar_init(load_bar, 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  // this tile's channel records (4 KB) into shared memory
  for (int i = threadIdx.x; i < kTileN * 2; i += kChainThreads)
    reinterpret_cast<uint4*>(rec_s)[i] = __ldg(reinterpret_cast<const uint4*>(p.rec + ct * kTileN) + i);
  tc_fence_before();
  cluster_sync();  // barriers initialised, TMEM allocated, every CTA of the cluster running
  tc_fence_after();
  const uint32_t tmem = *tslot;

  bool ok = true;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    mbar_arrive_expect_tx(load_bar, KB * Cfg::kWBlock + PA * KB * kActBlock);
    for (int kb = 0; kb < KB; ++kb) {
      tma_load_2d(wimg + kb * Cfg::kWBlock, &tmB, load_bar, 0, (ct * KB + kb) * Cfg::kBRows);
      for (int pl = 0; pl < PA; ++pl)
        tma_load_2d(act + (pl * KB + kb) * kActBlock, &tmA, load_bar, kb * kTileK, pl * p.a_plane_rows + rb * kTileM);
    }
    ok = mbar_wait(load_bar, 0, p.err, kErrTimeoutFull);
  }

  const bool u16 = p.qmax > 255;
  const uint32_t tl = tmem + (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
  const uint32_t peer = ct ^ 1u;
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
              constexpr uint32_t idS = idesc_i8(128, 128, 0, 1);
              constexpr uint32_t idU = idesc_i8(128, 128, 0, 0);
              const uint64_t dBhi = dB + ko, dBlo = dB + ko + (128 * kTileK >> 4);
              mma_i8(tmem + 0, dA0 + ko, dBhi, idS, acc);
              mma_i8(tmem + 128, dA0 + ko, dBlo, idU, acc);
              mma_i8(tmem + 128, dA1 + ko, dBhi, idS, 1u);
              mma_i8(tmem + 256, dA1 + ko, dBlo, idU, acc);
            } else {
              constexpr int N = Cfg::kBRows;
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
    const bool got = mbar_wait(mma_bar, step & 1, p.err, kErrTimeoutAccum);
    tc_fence_after();
    const bool last = step == p.chain - 1;
    const uint32_t obase = smem_u32(act + (bin ^ 1) * Cfg::kActBuf(KB));
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      const int c0 = half * 64 + g * 16;  // first of this group's 16 channels within the tile
      int64_t T[16];
      {
        uint32_t a0[16], a1[16], a2[16], a3[16];
        tmem_ld16(tl + g * 16, a0);
        if constexpr (MODE == kModeF32) {
          tmem_ld16(tl + g * 16 + 128, a1);
          if constexpr (PA == 2) {
            tmem_ld16(tl + g * 16 + 256, a2);
            tmem_ld16(tl + g * 16 + 384, a3);
          }
        } else if constexpr (MODE == kModeW16) {
          tmem_ld16(tl + g * 16 + 128, a1);
          tmem_ld16(tl + g * 16 + 256, a2);
        } else if constexpr (PA == 2) {
          tmem_ld16(tl + g * 16 + 128, a1);
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
      const bool real = ct * kTileN + c0 < p.N;  // 16-channel groups lie wholly inside or past N
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
        // next activation: K block ct, bytes c0..c0+15 of row `row` (one swizzled 16-byte chunk)
        const uint32_t chunk = static_cast<uint32_t>(row * kTileK + ((((c0 >> 4) ^ row) & 7) << 4));
        uint32_t hb[16], lb[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          hb[j] = u16 ? (code[j] >> 8) : code[j];
          lb[j] = code[j] & 0xFFu;
        }
        const uint4 vh = pack16(hb);
        const uint32_t a_hi = obase + ct * kActBlock + chunk;
        st_shared_v4(a_hi, vh);
        if (KB == 2) st_cluster_v4(map_peer(a_hi, peer), vh);
        if constexpr (PA == 2) {
          const uint4 vl = pack16(lb);
          const uint32_t a_lo = obase + (KB + ct) * kActBlock + chunk;
          st_shared_v4(a_lo, vl);
          if (KB == 2) st_cluster_v4(map_peer(a_lo, peer), vl);
        }
      } else if (real && m < p.M) {
        const size_t o = static_cast<size_t>(m) * p.N + ct * kTileN + c0;
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
    (void)got;
    // every TMEM read of this step is done and the next activation is in place (both CTAs): the
    // generic-proxy shared-memory writes are made visible to the tensor core's async proxy
    tc_fence_before();
    asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
    cluster_sync();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <int PA, int MODE>
cudaError_t launch_chain_variant(const CUtensorMap& ta, const CUtensorMap& tb, const ChainParams& prm, int m_blocks,
                                 cudaStream_t stream) {
  const int smem = chain_smem_bytes<PA, MODE>(prm.kblocks);
  cudaError_t e = cudaFuncSetAttribute(qchain_kernel<PA, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(m_blocks * prm.kblocks), 1, 1);
  cfg.blockDim = dim3(kChainThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(prm.kblocks);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qchain_kernel<PA, MODE>, ta, tb, prm);
}

}  // namespace

bool chain_fusable(const QhtpMatmulPlan* pl) {
  return pl->mode != kModeGroup && pl->k == pl->n && pl->n <= 2 * kTileN && pl->act_bits == pl->out_bits &&
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
  if (!make_tmap_planes(&tb, pl)) return cudaErrorInvalidValue;
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
  switch (pl->mode * 2 + (pl->a_planes - 1)) {
    case kModeF32 * 2 + 0: return launch_chain_variant<1, kModeF32>(ta, tb, prm, m_blocks, g.stream);
    case kModeF32 * 2 + 1: return launch_chain_variant<2, kModeF32>(ta, tb, prm, m_blocks, g.stream);
    case kModeExact * 2 + 0: return launch_chain_variant<1, kModeExact>(ta, tb, prm, m_blocks, g.stream);
    case kModeExact * 2 + 1: return launch_chain_variant<2, kModeExact>(ta, tb, prm, m_blocks, g.stream);
    case kModeW16 * 2 + 1: return launch_chain_variant<2, kModeW16>(ta, tb, prm, m_blocks, g.stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qhtp
