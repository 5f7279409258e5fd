// Tensor-pipe rate probe: the dense tcgen05.mma rate of this GPU, kind::i8 (the quantized GEMMs'
// instruction) or kind::f16 with bf16 operands, with no memory traffic in the timed loop.
//
// One CTA per SM (the dynamic shared memory keeps a second CTA off the SM).  The CTA fills a
// 128-row A tile and a 256-row B tile (128 bytes of K each, 128-byte swizzle) with pseudo-random
// bytes, allocates 512 TMEM columns, and one thread issues `iters` rounds of four M=128, N=256,
// K=32-byte MMAs -- the shape and K step of qgemm_kernel's mainloop -- alternating between two
// 256-column accumulators.  A commit on an mbarrier (bounded wait, as in the GEMMs) ends the CTA.
// The host times the launch with CUDA events: executed ops = ctas * iters * 4 * 2*128*256*K_inst,
// K_inst = 32 (i8) or 16 (bf16).  The operand values do not change the instruction count; they are
// non-zero so the datapath toggles as it does on real data.
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"
#include "ptx.cuh"

namespace qhtp {
namespace {

constexpr int kProbeThreads = 128;
constexpr int kProbeSmem = 160 * 1024;  // forces one CTA per SM; the operands use 48 KB of it

__global__ void __launch_bounds__(kProbeThreads, 1) mma_rate_kernel(uint32_t kind, uint32_t iters, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tslot;
  uint8_t* a = smem;               // 128 x 128 B
  uint8_t* b = smem + 128 * 128;   // 256 x 128 B
  // operand bytes: a hash of the index; for bf16 each 16-bit word keeps its sign and 7 mantissa bits
  // and gets the exponent of 2^-7 (magnitudes in [2^-7, 2^-6): finite, no overflow in f32)
  for (int i = threadIdx.x; i < (384 * 128) / 4; i += blockDim.x) {
    uint32_t h = static_cast<uint32_t>(i) * 2654435761u + blockIdx.x * 40503u;
    h ^= h >> 15;
    if (kind == 1) h = (h & 0x807F807Fu) | 0x3C003C00u;
    reinterpret_cast<uint32_t*>(a)[i] = h;
  }
  fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core (async proxy)
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(&tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  if (threadIdx.x == 0) {
    const uint64_t dA = desc_kmajor_sw128(smem_u32(a));
    const uint64_t dB = desc_kmajor_sw128(smem_u32(b));
    constexpr uint32_t id_i8 = idesc_i8(128, 256, 0, 1);
    constexpr uint32_t id_bf = idesc_bf16(128, 256);
    for (uint32_t it = 0; it < iters; ++it) {
      const uint32_t d = tmem + (it & 1u) * 256u;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t acc = (it < 2 && kk == 0) ? 0u : 1u;
        const uint64_t ko = static_cast<uint64_t>(kk * 2);  // 32 bytes of K, in 16-byte units
        if (kind == 0)
          mma_i8(d, dA + ko, dB + ko, id_i8, acc);
        else
          mma_bf16(d, dA + ko, dB + ko, id_bf, acc);
      }
    }
    mma_commit(&done);
  }
  mbar_wait(&done, 0, err, kErrTimeoutAccum);
  tc_fence_after();
  __syncthreads();
  if (threadIdx.x < 32) tmem_dealloc(tmem, 512);
}

}  // namespace
}  // namespace qhtp

extern "C" QhtpStatus qhtp_selftest_mma_rate(uint32_t kind, uint32_t iters, uint32_t ctas, int* err_word,
                                             void* stream) {
  if (kind > 1 || iters == 0 || iters > (1u << 24) || ctas == 0 || ctas > 4096 || err_word == nullptr)
    return QHTP_STATUS_INVALID_ARGUMENT;
  static bool attr_done = false;
  if (!attr_done) {
    const cudaError_t e = cudaFuncSetAttribute(qhtp::mma_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               qhtp::kProbeSmem);
    if (e != cudaSuccess) return qhtp::status_from_cuda(e);
    attr_done = true;
  }
  qhtp::mma_rate_kernel<<<ctas, qhtp::kProbeThreads, qhtp::kProbeSmem, static_cast<cudaStream_t>(stream)>>>(
      kind, iters, err_word);
  return qhtp::status_from_cuda(cudaGetLastError());
}
