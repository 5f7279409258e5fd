// Reference weight wire formats -> the library's plain weight carriers (qhtp_weights_from_wire).
//
// The reference packs MatMul weights into several layouts for its QNN ops (the packers of
// example/qnn_hmx_matmul_common/gen_quant_chain.py:285-742: HMX K-major tiles, K-pair and
// channel-pair nibble orders, XOR-0x80 int8 carriers, "hilo" and "biased" nibble variants).  Each
// layout is an address map: logical weight (k, n) lives at one byte (and, for int4, one nibble) of
// the carrier.  One gather kernel evaluates that map for every byte of the plain output -- int8
// [N, K], or int4 K-pairs [K/2, N] (two logical elements per output byte) -- so the writes are
// coalesced and each output byte is written once.  A one-time prepare step, HBM-bound.
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"

namespace qhtp {

namespace {

__device__ __forceinline__ uint64_t kmajor32(uint64_t k, uint64_t n, uint64_t N) {
  const uint64_t kt = k / 32, r = k % 32, nt = n / 32, c = n % 32;
  return (kt * (N / 32) + nt) * 1024 + (r / 4) * 128 + c * 4 + r % 4;
}

// Byte address of logical element (k, n) and its nibble (0 low, 1 high) before the HILO flag.
__device__ __forceinline__ uint64_t wire_addr(uint32_t fmt, uint64_t k, uint64_t n, uint64_t K, uint64_t N,
                                              uint32_t* nib) {
  *nib = 0;
  switch (fmt) {
    case QHTP_WIRE_W8_RAW_KN: return k * N + n;
    case QHTP_WIRE_W8_KMAJOR_TILE32: return kmajor32(k, n, N);
    case QHTP_WIRE_W8_KMAJOR_SPLIT128: return (n / 128) * (K * 128) + kmajor32(k, n % 128, 128);
    case QHTP_WIRE_W4_TILE32X64_NPAIR32: {
      const uint64_t nb = n / 64, nc = n % 64;
      *nib = nc >= 32;
      return ((k / 32) * (N / 64) + nb) * 1024 + ((k % 32) / 4) * 128 + (nc % 32) * 4 + k % 4;
    }
    case QHTP_WIRE_W4_KPAIR: *nib = k & 1; return (k / 2) * N + n;
    case QHTP_WIRE_W4_NMAJOR_KPAIR: *nib = k & 1; return n * (K / 2) + k / 2;
    case QHTP_WIRE_W4_NMAJOR_K4:
      *nib = (k % 8) >= 4;
      return (((n / 32) * (K / 8) + k / 8) * 32 + n % 32) * 4 + k % 4;
    case QHTP_WIRE_W4_KBLOCK32_NMAJOR_K4:
      *nib = (k % 8) >= 4;
      return ((((k / 32) * (N / 32) + n / 32) * 4 + (k % 32) / 8) * 32 + n % 32) * 4 + k % 4;
    case QHTP_WIRE_W4_NPAIR_ADJACENT: *nib = n & 1; return (n / 2) * K + k;
    case QHTP_WIRE_W4_NPAIR_TILE32: *nib = (n % 64) >= 32; return ((n / 64) * 32 + n % 32) * K + k;
    default: return k * N + n;  // QHTP_WIRE_W4_FULL_CODES
  }
}

// int4 code of logical element (k, n), two's complement in the low nibble.
__device__ __forceinline__ uint32_t w4_code(const uint8_t* wire, uint32_t fmt, uint32_t flags, uint64_t k, uint64_t n,
                                            uint64_t K, uint64_t N) {
  uint32_t nib;
  uint32_t b = wire[wire_addr(fmt, k, n, K, N, &nib)];
  if (flags & QHTP_WIRE_XOR80) b ^= 0x80u;
  if (fmt != QHTP_WIRE_W4_FULL_CODES && (flags & QHTP_WIRE_HILO)) nib ^= 1u;
  uint32_t c = (b >> (4 * nib)) & 15u;
  if (flags & QHTP_WIRE_BIASED) c ^= 8u;  // v + 8 -> v (mod 16)
  return c;
}

__global__ void wire_w8_kernel(const uint8_t* __restrict__ wire, uint32_t fmt, uint32_t flags, uint64_t K, uint64_t N,
                               uint8_t* __restrict__ plain) {
  const uint8_t x = (flags & QHTP_WIRE_XOR80) ? 0x80u : 0u;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < K * N;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t n = i / K, k = i % K;  // plain int8 [N, K]
    uint32_t nib;
    plain[i] = wire[wire_addr(fmt, k, n, K, N, &nib)] ^ x;
  }
}

__global__ void wire_w4_kernel(const uint8_t* __restrict__ wire, uint32_t fmt, uint32_t flags, uint64_t K, uint64_t N,
                               uint8_t* __restrict__ plain) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < (K / 2) * N;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t k2 = i / N, n = i % N;  // plain K-pair [K/2, N]
    const uint32_t lo = w4_code(wire, fmt, flags, 2 * k2, n, K, N);
    const uint32_t hi = w4_code(wire, fmt, flags, 2 * k2 + 1, n, K, N);
    plain[i] = static_cast<uint8_t>(lo | (hi << 4));
  }
}

bool is_w8(uint32_t fmt) { return fmt >= QHTP_WIRE_W8_RAW_KN && fmt <= QHTP_WIRE_W8_KMAJOR_SPLIT128; }
bool known(uint32_t fmt) { return fmt >= QHTP_WIRE_W8_RAW_KN && fmt <= QHTP_WIRE_W4_FULL_CODES; }

// Whether a [K, N] weight fits the layout's tiles (the reference packers' own shape checks).
bool shape_ok(uint32_t fmt, uint32_t k, uint32_t n) {
  if (!is_w8(fmt) && k % 2) return false;  // the plain int4 carrier pairs K
  switch (fmt) {
    case QHTP_WIRE_W8_KMAJOR_TILE32: return k % 32 == 0 && n % 32 == 0;
    case QHTP_WIRE_W8_KMAJOR_SPLIT128: return k % 32 == 0 && n % 128 == 0;
    case QHTP_WIRE_W4_TILE32X64_NPAIR32: return k % 32 == 0 && n % 64 == 0;
    case QHTP_WIRE_W4_NMAJOR_K4: return k % 8 == 0 && n % 32 == 0;
    case QHTP_WIRE_W4_KBLOCK32_NMAJOR_K4: return k % 32 == 0 && n % 32 == 0;
    case QHTP_WIRE_W4_NPAIR_ADJACENT: return n % 2 == 0;
    case QHTP_WIRE_W4_NPAIR_TILE32: return n % 64 == 0;
    default: return true;
  }
}

}  // namespace

}  // namespace qhtp

using namespace qhtp;

extern "C" {

size_t qhtp_wire_bytes(uint32_t format, uint32_t k, uint32_t n) {
  if (!known(format)) return 0;
  const size_t kn = static_cast<size_t>(k) * n;
  return (is_w8(format) || format == QHTP_WIRE_W4_FULL_CODES) ? kn : kn / 2;
}

QhtpStatus qhtp_weights_from_wire(uint32_t format, uint32_t flags, const void* wire, size_t wire_bytes, uint32_t k,
                                  uint32_t n, void* plain, size_t plain_bytes, void* stream) {
  if (wire == nullptr || plain == nullptr || k == 0 || n == 0 || !known(format) ||
      (flags & ~(QHTP_WIRE_XOR80 | QHTP_WIRE_HILO | QHTP_WIRE_BIASED)) != 0)
    return QHTP_STATUS_INVALID_ARGUMENT;
  if (!shape_ok(format, k, n)) return QHTP_STATUS_UNSUPPORTED;
  const size_t kn = static_cast<size_t>(k) * n;
  const size_t out_bytes = is_w8(format) ? kn : kn / 2;
  if (wire_bytes < qhtp_wire_bytes(format, k, n) || plain_bytes < out_bytes) return QHTP_STATUS_INVALID_ARGUMENT;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  size_t blocks = (out_bytes + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (is_w8(format))
    wire_w8_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(static_cast<const uint8_t*>(wire), format, flags, k,
                                                                n, static_cast<uint8_t*>(plain));
  else
    wire_w4_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(static_cast<const uint8_t*>(wire), format, flags, k,
                                                                n, static_cast<uint8_t*>(plain));
  return status_from_cuda(cudaGetLastError());
}

}  // extern "C"
