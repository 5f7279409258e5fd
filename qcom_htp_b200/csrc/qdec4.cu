// Decode rows (M <= 2) of the int4-weight MatMul families, streaming the 4-bit weight codes.
//
// Same operation and exactness model as qdecode.cu (HmxU16I4ToU16MatMul / HmxU8I4ToU8MatMul and
// the LPBQ variants; requant as generate_qnn_matmul_python_cases.py:426-525).  For the int4
// families the weight of output channel n at depth k is q8 = v * f (v the signed 4-bit code, f the
// LPBQ block factor, 1 per channel otherwise; HmxW4LpbqExpandToI8Op.cpp:26-47), and in the
// float32-dequant mode the accumulator is
//   T = m_s * sum_k x_k q8_k + sum_k x_k e'(q8_k) + beff,   e'(q8) = round24(q8 m_s) - q8 m_s,
// e' the float32 rounding residual of the dequantized weight (|e'| <= 64).  qdecode.cu streams
// q8 and e' as prepared byte planes (2 bytes per weight) into tensor-core tiles.  For one or two
// activation rows this kernel streams the 4-bit code image instead (0.5 byte per weight, plus one
// factor byte per 32 weights for LPBQ) and does the arithmetic on the CUDA cores:
//   * q part: with u = v + 8 the offset-binary code, sum_k x_k q8_k = f * (sum_k x_k u_k - 8 sum_k x_k)
//     per 32-deep K step (one factor per step).  The codes are unpacked to bytes with two masks and
//     multiplied with the activation by dp2a (u16 activation pairs) or dp4a (u8 activations); the
//     bytes come out in K order 0,2,4,6 | 1,3,5,7 of each group of eight, so a copy of the activation
//     is kept in that order, together with the sum of every 32 consecutive values.
//   * e' part: 16-entry table lookups with byte permutes.  Per (channel, f) a prepared 16-byte table
//     holds e'((u - 8) f) for u = 0..15; prmt selects bytes with the code word as selector, the
//     entries u < 8 from the table's first half and u >= 8 (code XOR 8) from its second, and a
//     third prmt in sign-replicate mode turns bit 3 of each code into the byte mask that picks
//     between them.  The bytes (K order 0..3 | 4..7) go through dp2a / dp4a with the activation.
// A thread owns one channel and accumulates int32 sums per K step (exact: |sum| < 2^31) into int64.
// (A tensor-core version that formed the q8 and e' images in TMEM and ran kind::i8 MMAs with A from
// TMEM was built and is bit-exact, but each MMA (M = 128, N <= 64, K = 32) costs 46-60 cycles in
// isolation and ~120 inside the pipeline, 16 per 256-deep stage, and it was no faster than the
// byte-plane kernel.)
//
// Work split: the K range of every 128-channel tile is cut into stages of 256; the stages of all
// tiles, tile-major, are divided evenly over one persistent CTA per SM (contiguous ranges).  A
// tile a CTA covers alone is requantized there; for a tile shared by several CTAs each writes its
// int64 partial T to the workspace and moves on, and a small combine kernel, launched right behind
// with programmatic dependent launch, sums the partials and requantizes once the stream has
// finished (one thread per output, no loads queued behind the weight stream).  No CTA waits for
// another.
//
// Warp roles: 0 TMA producer (code and factor tiles, per-tile e' tables), 1..16 compute (channel
// group (w - 1) & 3 of 32 channels, K steps (w - 1) >> 2 and that + 4 of every stage, interleaved as
// two independent instruction streams; the four K-step groups of a channel meet in shared memory at
// the end of a tile).  Every mbarrier wait is
// bounded, and a compute warp whose wait gave up still takes every named barrier.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"
#include "requant.cuh"

namespace qhtp {

namespace {

constexpr int kD4StageK = 256;                  // K per stage: 128 code bytes per channel
constexpr int kD4Steps = kD4StageK / 32;        // 32-deep K steps per stage (one factor each)
constexpr int kD4MaxCtas = 160;                 // partial slots are sized for this many CTAs
constexpr int kD4Codes = 128 * 128;             // code bytes of one stage (128 channels x 128 B)
constexpr size_t kD4SmemMax = 227 * 1024;       // dynamic shared memory of one CTA

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

bool lpbq_plan(const QhtpMatmulPlan* p) { return p->schema == QHTP_SCHEMA_LPBQ; }
int n_tables(const QhtpMatmulPlan* p) { return p->mode != kModeF32 ? 0 : (lpbq_plan(p) ? 16 : 1); }

size_t codes_bytes(const QhtpMatmulPlan* p) { return align256(static_cast<size_t>(p->n_tiles) * 128 * (p->k / 2)); }
size_t factor_bytes(const QhtpMatmulPlan* p) {
  return lpbq_plan(p) ? align256(static_cast<size_t>(p->n_tiles) * (p->k / 32) * 128) : 0;
}
size_t table_tile_bytes(const QhtpMatmulPlan* p) { return static_cast<size_t>(n_tables(p)) * 128 * 16; }

}  // namespace

bool int4_stream_layout(const QhtpMatmulPlan* p) {
  if (p->weight_bits != 4) return false;
  if (p->schema != QHTP_SCHEMA_PER_CHANNEL && p->schema != QHTP_SCHEMA_LPBQ) return false;
  if (p->mode != kModeF32 && p->mode != kModeExact) return false;
  if (p->k % kD4StageK) return false;
  if (lpbq_plan(p) && p->lpbq_block % 32) return false;
  return true;
}

size_t int4_image_bytes(const QhtpMatmulPlan* p) {
  if (!int4_stream_layout(p)) return 0;
  return codes_bytes(p) + factor_bytes(p) + align256(p->n_tiles * table_tile_bytes(p));
}

size_t int4_image_offset(const QhtpMatmulPlan* p) {
  const size_t npad = static_cast<size_t>(p->n_tiles) * p->ch_per_tile;
  return p->plane_bytes + p->record_bytes + align256(npad * 8 * kSumsPerChannel);
}

size_t dec4_workspace_bytes(const QhtpMatmulPlan* p, uint32_t m) {
  if (!int4_stream_layout(p) || m == 0 || m > kDec4MaxM) return 0;
  return align256(static_cast<size_t>(kD4MaxCtas) * 2 * m * 128 * 8);  // partial T, 2 slots per CTA
}

namespace {
size_t gemv_smem(const QhtpMatmulPlan* p, uint32_t m);
}

int sm_count_d4();

// Dispatch: the code stream pays where every CTA streams several stages (measured, W4A16 LPBQ
// K = 4096, M = 1: N = 14336 (12 stages per SM) 27.4 us vs 31.8 us for the byte-plane kernel;
// N = 4096 (3.5 stages per SM) 18.3 us vs 17.5 us; M = 4 loses at both widths).
bool dec4_supported(const QhtpMatmulPlan* p, uint32_t m) {
  const uint64_t units = static_cast<uint64_t>(p->n_tiles) * (p->k / kD4StageK);
  return (p->flags & kPlanInt4Stream) != 0 && dec4_workspace_bytes(p, m) != 0 &&
         units * kD4MaxCtas < (1ull << 31) && gemv_smem(p, m) <= kD4SmemMax &&
         (units >= 6ull * sm_count_d4() || (p->flags & kPlanForceInt4Stream) != 0);
}

// ------------------------------------------------------------------------------------------------
// Prepare: code image, block factors per K step, e' tables
// ------------------------------------------------------------------------------------------------
namespace {

struct Int4Prep {
  uint32_t N, K, npad, n_tiles, lpbq_block, n_tab;
  bool lpbq;
  const uint8_t* w4;    // reference layout: byte (k/2, n) holds k (low nibble) and k+1, two's complement
  const uint8_t* fac;   // LPBQ factors [N][K / block]
  uint8_t* codes;       // [n_tiles][K/256][128][128]: one contiguous 16 KB image per (tile, stage); byte
                        // (row, k/2 mod 128) = (u_k | u_{k+1} << 4), u = v + 8
  uint8_t* factors;     // [n_tiles][K/32][128]
  uint8_t* tables;      // [n_tiles][n_tab][128][16]: byte u = e'(clip((u - 8) f) * m_s)
  int* status;
};

// One thread per (channel, 16 code bytes): 32 weights, read down the reference layout's columns.
__global__ void int4_codes_kernel(Int4Prep p) {
  const uint32_t chunks = p.K / 32;
  const size_t total = static_cast<size_t>(chunks) * p.npad;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint32_t n = static_cast<uint32_t>(i % p.npad), j = static_cast<uint32_t>(i / p.npad);
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t v = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t kp = 16 * j + 4 * q + b;  // k-pair index
        const uint32_t byte = n < p.N ? p.w4[static_cast<size_t>(kp) * p.N + n] : 0u;
        v |= (byte ^ 0x88u) << (8 * b);  // two's-complement nibble -> offset binary (v = 0 in padding)
      }
      w[q] = v;
    }
    const uint32_t kb = 16 * j;  // byte offset along K / 2
    const size_t tile_stage = static_cast<size_t>(n / 128) * (p.K / kD4StageK) + kb / 128;
    *reinterpret_cast<uint4*>(p.codes + (tile_stage * 128 + n % 128) * 128 + kb % 128) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__global__ void int4_factors_kernel(Int4Prep p) {
  const uint32_t steps = p.K / 32;
  const size_t total = static_cast<size_t>(p.n_tiles) * steps * 128;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint32_t c = static_cast<uint32_t>(i % 128), ks = static_cast<uint32_t>((i / 128) % steps),
                   t = static_cast<uint32_t>(i / (128ull * steps));
    const uint32_t n = t * 128 + c;
    uint32_t f = 1;
    if (n < p.N) {
      f = p.fac[static_cast<size_t>(n) * (p.K / p.lpbq_block) + ks * 32 / p.lpbq_block];
      if (f < 1 || f > 16) atomicOr(p.status + 2, 1);  // u * f must fit a byte, table index f - 1
    }
    p.factors[i] = static_cast<uint8_t>(f);
  }
}

__global__ void int4_tables_kernel(Int4Prep p, const float* __restrict__ scale) {
  const size_t total = static_cast<size_t>(p.n_tiles) * p.n_tab * 128;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint32_t c = static_cast<uint32_t>(i % 128), fi = static_cast<uint32_t>((i / 128) % p.n_tab),
                   t = static_cast<uint32_t>(i / (128ull * p.n_tab));
    const uint32_t n = t * 128 + c;
    uint32_t w[4] = {0, 0, 0, 0};
    if (n < p.N) {
      const uint32_t bits = __float_as_uint(scale[n]);
      const int32_t ms = static_cast<int32_t>((bits & 0x7FFFFFu) | 0x800000u);
      const int f = p.lpbq ? static_cast<int>(fi) + 1 : 1;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        int q = (u - 8) * f;
        q = q < -128 ? -128 : (q > 127 ? 127 : q);
        const int32_t prod = q * ms;                                 // |prod| < 2^31
        const int32_t e = __float2int_rz(__int2float_rn(prod)) - prod;  // round to 24 bits; |e| <= 64
        w[u >> 2] |= (static_cast<uint32_t>(e) & 0xFFu) << (8 * (u & 3));
      }
    }
    *reinterpret_cast<uint4*>(p.tables + 16 * i) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace

int sm_count_d4() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

namespace {

int grid_for(size_t total) {
  size_t b = (total + 255) / 256;
  const size_t cap = static_cast<size_t>(sm_count_d4()) * 32;
  if (b > cap) b = cap;
  return b < 1 ? 1 : static_cast<int>(b);
}

}  // namespace

cudaError_t launch_prepare_int4(const QhtpMatmulPlan* plan, const QhtpMatmulWeights* w, void* prepared, int* status,
                                cudaStream_t stream) {
  if (!int4_stream_layout(plan)) return cudaSuccess;
  uint8_t* base = static_cast<uint8_t*>(prepared) + int4_image_offset(plan);
  Int4Prep p;
  p.N = plan->n;
  p.K = plan->k;
  p.n_tiles = plan->n_tiles;
  p.npad = plan->n_tiles * 128;
  p.lpbq = lpbq_plan(plan);
  p.lpbq_block = plan->lpbq_block;
  p.n_tab = static_cast<uint32_t>(n_tables(plan));
  p.w4 = static_cast<const uint8_t*>(w->weight);
  p.fac = w->lpbq_block_scale;
  p.codes = base;
  p.factors = base + codes_bytes(plan);
  p.tables = p.factors + factor_bytes(plan);
  p.status = status;
  int4_codes_kernel<<<grid_for(static_cast<size_t>(p.K / 32) * p.npad), 256, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && p.lpbq) {
    int4_factors_kernel<<<grid_for(static_cast<size_t>(p.n_tiles) * (p.K / 32) * 128), 256, 0, stream>>>(p);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && p.n_tab > 0) {
    int4_tables_kernel<<<grid_for(static_cast<size_t>(p.n_tiles) * p.n_tab * 128), 256, 0, stream>>>(p, w->weight_scale);
    e = cudaGetLastError();
  }
  return e;
}

// ------------------------------------------------------------------------------------------------
// The decode kernel
// ------------------------------------------------------------------------------------------------
namespace {

struct D4Params {
  int M, N, K, cps;       // cps: stages per tile (K / 256)
  int units, grid;        // stages of all tiles; CTAs
  int fac_rows;           // K / 32: factor rows per tile
  const void* act;        // [M][K], u16 or u8
  const ChannelRecord* rec;
  const uint8_t* tables;  // [n_tiles][n_tab][128][16]
  void* out;
  long long* partial;     // [grid][2][M][128]: the first and the last segment of each CTA
  int zp_out, qmax;
  uint64_t act_mant, out_mant;
  int act_exp2, out_exp2;
  int* err;
};

constexpr int kD4KGroups = 4;                      // K-step groups: compute warps per channel group
constexpr int kD4Warps = 4 * kD4KGroups;           // compute warps: 4 channel groups x the K-step groups
constexpr int kD4Threads = (1 + kD4Warps) * 32;    // + the TMA producer warp

// Shared memory: the activation (natural and q order) and its per-32-K sums, the stage ring (codes
// and, for LPBQ, factors), two e' table buffers, the cross-warp reduction area, mbarriers.
template <int PA, int MODE, bool LPBQ, int MR>
struct D4Cfg {
  static constexpr bool kF32 = MODE == kModeF32;
  static constexpr int kFac = LPBQ ? kD4Steps * 128 : 0;
  static constexpr int kStage = kD4Codes + kFac;
  static constexpr int kTab = kF32 ? (LPBQ ? 16 : 1) * 128 * 16 : 0;
  static constexpr int kStages = MR >= 4 ? 3 : (MR == 2 ? 5 : 6);
  static constexpr int kRed = kD4KGroups * 128 * MR * 16;  // [K-step group][channel][row] x (q, e' part)
  static constexpr int kFixed = kStages * kStage + 2 * kTab + kRed + 1024 + 256;
  static size_t smem(int K) { return kFixed + static_cast<size_t>(MR) * K * PA * 2 + static_cast<size_t>(MR) * (K / 32) * 4; }
};

struct D4Chan {
  int64_t beff, mq;
  uint64_t cmn;
  int tn, es;
  uint32_t mul;
};

template <int MODE>
__device__ __forceinline__ D4Chan d4_chan(const ChannelRecord* rc) {
  D4Chan c;
  c.beff = rc->beff;
  c.cmn = rc->cmn;
  c.tn = rc->tn;
  c.mq = rc->m_q;
  const uint32_t wb = rc->wbits;
  c.es = static_cast<int>((wb >> 23) & 0xFFu) - 150;
  c.mul = MODE == kModeF32 ? 1u : ((wb & 0x7FFFFFu) | 0x800000u);
  return c;
}

__device__ __forceinline__ uint32_t d4_requant(int64_t T, const D4Chan& c, const D4Params& p) {
  bool near = false;
  int64_t fl = 0;
  int32_t code = requant_fast96s(T, c.cmn, c.tn, p.zp_out, p.qmax, &near, &fl);
  if (near) code = requant_tie_w(T, fl, c.mul, c.es + p.act_exp2, p.act_mant, p.out_mant, p.out_exp2, p.zp_out, p.qmax);
  return static_cast<uint32_t>(code);
}

__device__ __forceinline__ void d4_store(const D4Params& p, int row, int n, uint32_t code) {
  if (p.qmax > 255)
    reinterpret_cast<uint16_t*>(p.out)[static_cast<size_t>(row) * p.N + n] = static_cast<uint16_t>(code);
  else
    reinterpret_cast<uint8_t*>(p.out)[static_cast<size_t>(row) * p.N + n] = static_cast<uint8_t>(code);
}

// Contiguous stage ranges: CTA g owns units [start(g), start(g+1)).  units * grid < 2^31
// (dec4_supported), so 32-bit products are exact.
__device__ __forceinline__ int d4_start(int g, const D4Params& p) { return (p.units * g) / p.grid; }
__device__ __forceinline__ int d4_owner(int u, const D4Params& p) { return ((u + 1) * p.grid - 1) / p.units; }

__device__ __forceinline__ uint32_t pick(uint32_t n, uint32_t p, uint32_t m) { return (n & ~m) | (p & m); }

// e' bytes of one code word (8 weights, nibble i = K position i, offset binary u) by 16-entry table
// lookup: byte u of the table is e' for code u.  With the code's bit 3 cleared (u & 7, every
// selector nibble in plain byte-select mode), one prmt reads the table's first half (entries 0..7)
// and one its second half (8..15); the bit-3 mask (prmt in sign-replicate mode over the code shifted
// into each byte's sign bit) picks between them.  K positions 0..3 | 4..7.  The shifts run on the
// multiply pipe (w * 16 and the high word of w7 * 2^16), the permutes and selects on the integer pipe.
__device__ __forceinline__ void d4_lookup(uint32_t w, const uint4& et, uint32_t& e0, uint32_t& e1) {
  const uint32_t w7 = w & 0x77777777u;
  const uint32_t w4 = w * 16u;
  const uint32_t m0 = prmt(w4, w, 0xD9C8u);  // 0xFF where the code of K position i (0..3) is >= 8
  const uint32_t m1 = prmt(w4, w, 0xFBEAu);  // the same for K positions 4..7
  const uint32_t w7h = __umulhi(w7, 0x10000u);
  e0 = pick(prmt(et.x, et.y, w7), prmt(et.z, et.w, w7), m0);
  e1 = pick(prmt(et.x, et.y, w7h), prmt(et.z, et.w, w7h), m1);
}

// dot products of 16-bit activation pairs with byte lanes (dp2a) and of 8-bit activation quads
// with byte lanes (dp4a); u = unsigned weight bytes, s = signed weight bytes
__device__ __forceinline__ uint32_t dp2lo_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d; asm("dp2a.lo.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ uint32_t dp2hi_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d; asm("dp2a.hi.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int32_t dp2lo_s(uint32_t a, uint32_t b, int32_t c) {
  int32_t d; asm("dp2a.lo.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int32_t dp2hi_s(uint32_t a, uint32_t b, int32_t c) {
  int32_t d; asm("dp2a.hi.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ uint32_t dp4_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d; asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int32_t dp4_s(uint32_t a, uint32_t b, int32_t c) {
  int32_t d; asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}

// AND of a predicate over the 16 compute warps (named barrier 1): a warp whose bounded wait gave up
// still takes every barrier, so the others never wait for it.
__device__ __forceinline__ bool compute_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(kD4Warps * 32)
      : "memory");
  return r != 0;
}

template <int PA, int MODE, bool LPBQ, int MR>
__global__ void __launch_bounds__(kD4Threads, 1)
    qgemv4_kernel(const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmF,
                  const D4Params p) {
  using Cfg = D4Cfg<PA, MODE, LPBQ, MR>;
  constexpr int S = Cfg::kStages;
  constexpr bool F32 = Cfg::kF32;

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base by pointer arithmetic on the shared array, so that the compiler keeps
  // every derived access in the shared window (32-bit shared loads, not generic ones)
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* tbl = smem + S * Cfg::kStage;                                        // [2][n_tab][128][16]
  long long* red = reinterpret_cast<long long*>(tbl + 2 * Cfg::kTab);           // [KGroups][128][MR][2]
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + Cfg::kRed);
  uint64_t* empty = full + S;
  uint64_t* tblfull = empty + S;
  uint64_t* tblfree = tblfull + 2;
  uint64_t* actfull = tblfree + 2;
  uint8_t* act_nat = smem + Cfg::kFixed - 1024;                                  // [MR][K], act width
  uint8_t* act_q = act_nat + MR * p.K * PA;                                     // q order
  int32_t* asum = reinterpret_cast<int32_t*>(act_q + MR * p.K * PA);            // [MR][K/32]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x;
  const int u0 = d4_start(g, p), u1 = d4_start(g + 1, p);
  const int nst = u1 - u0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kD4Warps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tblfull[b], 1);
      mbar_init(&tblfree[b], kD4Warps);
    }
    mbar_init(actfull, 1);
    fence_barrier_init();
    griddep_launch_dependents();  // the combine kernel may be scheduled now
  }
  __syncthreads();

  // The producer's loads of one stage (and, at a tile's first stage, its e' tables); stages are issued
  // in order, so the tile t_p and chunk c_p of stage i_p advance by counting (no division per stage).
  int seg_p = -1, i_p = 0, t_p = u0 / p.cps, c_p = u0 % p.cps;
  bool ok_p = true;
  auto issue = [&](int i, bool may_wait) -> bool {
    const int t = t_p, c = c_p;
    if (i == 0 || c == 0) {
      if constexpr (F32) {
        const int tb = (seg_p + 1) & 1;
        if (!may_wait && seg_p + 1 >= 2) return false;  // would wait for the compute warps
        if (!mbar_wait_suspend(&tblfree[tb], (((seg_p + 1) >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty)) {
          ok_p = false;
          return false;
        }
        mbar_arrive_expect_tx(&tblfull[tb], Cfg::kTab);
        bulk_load(tbl + tb * Cfg::kTab, p.tables + static_cast<size_t>(t) * Cfg::kTab, Cfg::kTab, &tblfull[tb]);
      }
      ++seg_p;
    }
    const int s = i % S;
    if (!mbar_wait_suspend(&empty[s], ((i / S) & 1) ^ 1, p.err, kErrTimeoutEmpty)) {
      ok_p = false;
      return false;
    }
    uint8_t* st = smem + s * Cfg::kStage;
    mbar_arrive_expect_tx(&full[s], Cfg::kStage);
    tma_load_2d(st, &tmC, &full[s], 0, (t * p.cps + c) * 128);
    if constexpr (LPBQ) tma_load_2d(st + kD4Codes, &tmF, &full[s], 0, t * p.fac_rows + c * kD4Steps);
    if (++c_p == p.cps) {
      c_p = 0;
      ++t_p;
    }
    return true;
  };
  if (warp == 0 && lane == 0) {  // the activation and the first stages start streaming together
    const uint32_t act_bytes = static_cast<uint32_t>(p.M) * p.K * PA;
    mbar_arrive_expect_tx(actfull, act_bytes);
    bulk_load(act_nat, p.act, act_bytes, actfull);
    tma_prefetch_desc(&tmC);
    if (LPBQ) tma_prefetch_desc(&tmF);
    for (; i_p < nst && i_p < S; ++i_p)
      if (!issue(i_p, false)) break;
  }

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && ok_p)
      for (; i_p < nst; ++i_p)
        if (!issue(i_p, true)) break;
  } else {
    // ---------------------------------------------------------------- compute warps
    // activation rows (rows >= M are zero; rows < M arrive by bulk copy in the natural copy): the
    // q-order copy (K positions 0,2,4,6,1,3,5,7 of each group of eight) and the sum of every 32
    // consecutive values, one K step per thread and iteration
    const int ksteps = p.K / 32;
    bool ok = mbar_wait(actfull, 0, p.err, kErrTimeoutFull);
    for (int it = threadIdx.x - 32; it < MR * ksteps; it += kD4Warps * 32) {
      const int r = it / ksteps, kk = it % ksteps;
      uint4* dn = reinterpret_cast<uint4*>(act_nat + (r * p.K + kk * 32) * PA);
      uint4* dq = reinterpret_cast<uint4*>(act_q + (r * p.K + kk * 32) * PA);
      int32_t sum = 0;
#pragma unroll
      for (int q = 0; q < PA * 2; ++q) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < p.M) v = dn[q];
        else dn[q] = v;
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        if constexpr (PA == 2) {  // eight u16 values per uint4
          dq[q] = make_uint4(prmt(w[0], w[1], 0x5410), prmt(w[2], w[3], 0x5410), prmt(w[0], w[1], 0x7632),
                             prmt(w[2], w[3], 0x7632));
#pragma unroll
          for (int e = 0; e < 4; ++e) sum += static_cast<int32_t>((w[e] & 0xFFFFu) + (w[e] >> 16));
        } else {  // sixteen u8 values per uint4: two groups of eight
          dq[q] = make_uint4(prmt(w[0], w[1], 0x6420), prmt(w[0], w[1], 0x7531), prmt(w[2], w[3], 0x6420),
                             prmt(w[2], w[3], 0x7531));
#pragma unroll
          for (int e = 0; e < 4; ++e)
            sum += static_cast<int32_t>((w[e] & 0xFFu) + ((w[e] >> 8) & 0xFFu) + ((w[e] >> 16) & 0xFFu) + (w[e] >> 24));
        }
      }
      asum[r * ksteps + kk] = sum;
    }
    ok = compute_bar_and(ok);  // the activation copies are complete
    const int wi = warp - 1, grp = wi & 3, kj = wi >> 2;  // channel group, K-step group
    const int ch = grp * 32 + lane;
    int64_t tq[MR], te[MR];
    int seg = -1;
    const int t0 = u0 / p.cps, c0 = u0 % p.cps;  // tile and chunk of this CTA's first stage
    int t = t0, c = c0;                           // of stage i, advanced by counting
    for (int i = 0; i < nst; ++i) {
      const bool first = i == 0 || c == 0, last = i == nst - 1 || c == p.cps - 1;
      if (first) {
        ++seg;
#pragma unroll
        for (int r = 0; r < MR; ++r) tq[r] = te[r] = 0;
        if constexpr (F32)
          if (ok) ok = mbar_wait(&tblfull[seg & 1], (seg >> 1) & 1, p.err, kErrTimeoutFull);
      }
      const int s = i % S;
      if (ok) ok = mbar_wait(&full[s], (i / S) & 1, p.err, kErrTimeoutFull);
      if (ok) {
        const uint8_t* st = smem + s * Cfg::kStage;
        const uint4* tab = reinterpret_cast<const uint4*>(tbl + (seg & 1) * Cfg::kTab) + ch;
        constexpr int RK = kD4Steps / kD4KGroups;  // K steps per warp and stage
        uint32_t f[RK];
        uint4 et[RK], cw[RK];
#pragma unroll
        for (int rk = 0; rk < RK; ++rk) {  // every shared-memory load of the stage first
          const int ks = kj + kD4KGroups * rk;
          f[rk] = LPBQ ? static_cast<uint32_t>(st[kD4Codes + ks * 128 + ch]) : 1u;
          cw[rk] = *reinterpret_cast<const uint4*>(st + ch * 128 + ((ks ^ (ch & 7)) << 4));
        }
#pragma unroll
        for (int rk = 0; rk < RK; ++rk) {
          et[rk] = make_uint4(0, 0, 0, 0);
          if constexpr (F32) et[rk] = tab[(LPBQ ? f[rk] - 1 : 0) * 128];
        }
        uint32_t su[RK][MR];
        int32_t se[RK][MR];
#pragma unroll
        for (int rk = 0; rk < RK; ++rk)
#pragma unroll
          for (int r = 0; r < MR; ++r) su[rk][r] = 0, se[rk][r] = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
#pragma unroll
          for (int rk = 0; rk < RK; ++rk) {  // independent streams, interleaved
            const int kg = c * kD4Steps + kj + kD4KGroups * rk;  // K step within K
            const uint32_t w = q == 0 ? cw[rk].x : (q == 1 ? cw[rk].y : (q == 2 ? cw[rk].z : cw[rk].w));
            const uint32_t x0 = w & 0x0F0F0F0Fu, x1 = __umulhi(w, 1u << 28) & 0x0F0F0F0Fu;
            uint32_t e0 = 0, e1 = 0;
            if constexpr (F32) d4_lookup(w, et[rk], e0, e1);
#pragma unroll
            for (int r = 0; r < MR; ++r) {
              const int off = (r * p.K + kg * 32 + q * 8) * PA;
              if constexpr (PA == 2) {
                const uint4 aq = *reinterpret_cast<const uint4*>(act_q + off);
                su[rk][r] = dp2lo_u(aq.x, x0, su[rk][r]);
                su[rk][r] = dp2hi_u(aq.y, x0, su[rk][r]);
                su[rk][r] = dp2lo_u(aq.z, x1, su[rk][r]);
                su[rk][r] = dp2hi_u(aq.w, x1, su[rk][r]);
                if constexpr (F32) {
                  const uint4 an = *reinterpret_cast<const uint4*>(act_nat + off);
                  se[rk][r] = dp2lo_s(an.x, e0, se[rk][r]);
                  se[rk][r] = dp2hi_s(an.y, e0, se[rk][r]);
                  se[rk][r] = dp2lo_s(an.z, e1, se[rk][r]);
                  se[rk][r] = dp2hi_s(an.w, e1, se[rk][r]);
                }
              } else {
                const uint2 aq = *reinterpret_cast<const uint2*>(act_q + off);
                su[rk][r] = dp4_u(aq.x, x0, su[rk][r]);
                su[rk][r] = dp4_u(aq.y, x1, su[rk][r]);
                if constexpr (F32) {
                  const uint2 an = *reinterpret_cast<const uint2*>(act_nat + off);
                  se[rk][r] = dp4_s(an.x, e0, se[rk][r]);
                  se[rk][r] = dp4_s(an.y, e1, se[rk][r]);
                }
              }
            }
          }
        }
        // sum_k x_k q8_k = f * sum_k x_k (u_k - 8), per K step
#pragma unroll
        for (int rk = 0; rk < RK; ++rk) {
          const int kg = c * kD4Steps + kj + kD4KGroups * rk;
#pragma unroll
          for (int r = 0; r < MR; ++r) {
            tq[r] += static_cast<int64_t>(static_cast<int32_t>(f[rk]) *
                                          (static_cast<int32_t>(su[rk][r]) - 8 * asum[r * ksteps + kg]));
            te[r] += se[rk][r];
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[s]);
        if (F32 && last) mbar_arrive(&tblfree[seg & 1]);
      }
      if (last) {
        // the K-step groups of each channel meet in shared memory; warp kj finishes rows kj, kj+8..
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          red[((kj * 128 + ch) * MR + r) * 2] = tq[r];
          red[((kj * 128 + ch) * MR + r) * 2 + 1] = te[r];
        }
        ok = compute_bar_and(ok);
        const int ca = seg == 0 ? c0 : 0;  // first chunk of this segment
        const bool whole = ca == 0 && c == p.cps - 1;
        const int n = t * 128 + ch;
        if (ok && n < p.N) {
          const D4Chan cc = d4_chan<MODE>(p.rec + n);
          const int slot = t0 == t ? 0 : 1;
          for (int r = kj; r < MR && r < p.M; r += kD4KGroups) {
            int64_t Tq = 0, Te = 0;
#pragma unroll
            for (int k = 0; k < kD4KGroups; ++k) {
              Tq += red[((k * 128 + ch) * MR + r) * 2];
              Te += red[((k * 128 + ch) * MR + r) * 2 + 1];
            }
            const int64_t T = cc.mq * Tq + Te;
            if (whole)
              d4_store(p, r, n, d4_requant(T + cc.beff, cc, p));
            else
              p.partial[((static_cast<size_t>(g) * 2 + slot) * p.M + r) * 128 + ch] = T;
          }
        }
        ok = compute_bar_and(ok);  // the reduction area is free again
      }
      if (++c == p.cps) {
        c = 0;
        ++t;
      }
    }
  }
  __syncthreads();
}

// Tiles shared by several CTAs: sum the partial T of every contributor (block x = tile, block y =
// a group of four activation rows, thread = channel), add the effective bias and requantize.
template <int MODE>
__global__ void __launch_bounds__(128) dec4_combine_kernel(const D4Params p) {
  const int t = blockIdx.x;
  const int gf = d4_owner(t * p.cps, p), gl = d4_owner(t * p.cps + p.cps - 1, p);
  const int n = t * 128 + static_cast<int>(threadIdx.x);
  if (gf == gl || n >= p.N) return;  // a tile covered by one CTA was requantized there
  const D4Chan cc = d4_chan<MODE>(p.rec + n);
  // the contributors' slots: the tile is the first segment of every contributor but the first
  int off[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int gc = gf + q;
    off[q] = ((gc * 2 + (q == 0 && d4_start(gf, p) / p.cps != t ? 1 : 0)) * p.M) * 128 + static_cast<int>(threadIdx.x);
  }
  const int nc = gl - gf + 1;
  griddep_wait();  // every partial of the decode kernel is written and visible
  const int r0 = blockIdx.y * 4;
  int64_t T[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) T[r] = cc.beff;
#pragma unroll
  for (int q = 0; q < 8; ++q)
#pragma unroll
    for (int r = 0; r < 4; ++r)
      if (q < nc && r0 + r < p.M) T[r] += p.partial[off[q] + (r0 + r) * 128];
  for (int gc = gf + 8; gc <= gl; ++gc)  // more than 8 contributors (few tiles over a long K)
#pragma unroll
    for (int r = 0; r < 4; ++r)
      if (r0 + r < p.M) T[r] += p.partial[(gc * 2 * p.M + r0 + r) * 128 + threadIdx.x];
#pragma unroll
  for (int r = 0; r < 4; ++r)
    if (r0 + r < p.M) d4_store(p, r0 + r, n, d4_requant(T[r], cc, p));
}

template <int PA, int MODE, bool LPBQ, int MR>
cudaError_t launch_d4(const CUtensorMap& tc, const CUtensorMap& tf, const D4Params& prm, cudaStream_t stream) {
  using Cfg = D4Cfg<PA, MODE, LPBQ, MR>;
  const size_t smem = Cfg::smem(prm.K);
  static int attr_set = 0;  // largest dynamic shared memory size set so far
  if (static_cast<int>(smem) > attr_set) {
    cudaError_t e = cudaFuncSetAttribute(qgemv4_kernel<PA, MODE, LPBQ, MR>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    attr_set = static_cast<int>(smem);
  }
  qgemv4_kernel<PA, MODE, LPBQ, MR><<<prm.grid, kD4Threads, smem, stream>>>(tc, tf, prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cc = {};
  cc.gridDim = dim3(static_cast<unsigned>(prm.units / prm.cps), static_cast<unsigned>((prm.M + 3) / 4), 1);
  cc.blockDim = dim3(128, 1, 1);
  cc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cc.attrs = attr;
  cc.numAttrs = 1;
  return cudaLaunchKernelEx(&cc, dec4_combine_kernel<MODE>, prm);
}

template <int PA, int MODE, bool LPBQ>
cudaError_t launch_d4_rows(int mr, const CUtensorMap& tc, const CUtensorMap& tf, const D4Params& prm,
                           cudaStream_t stream) {
  switch (mr) {
    case 1: return launch_d4<PA, MODE, LPBQ, 1>(tc, tf, prm, stream);
    case 2: return launch_d4<PA, MODE, LPBQ, 2>(tc, tf, prm, stream);
    default: return cudaErrorInvalidValue;
  }
}

int rows_bucket(uint32_t m) { return m <= 1 ? 1 : 2; }

size_t gemv_smem(const QhtpMatmulPlan* p, uint32_t m) {
  const int mr = rows_bucket(m);
  const bool lp = lpbq_plan(p), f32 = p->mode == kModeF32;
  const int pa = static_cast<int>(p->a_planes);
  const int fac = lp ? kD4Steps * 128 : 0;
  const int stages = mr >= 4 ? 3 : (mr == 2 ? 5 : 6);
  const int tab = f32 ? (lp ? 16 : 1) * 128 * 16 : 0;
  return static_cast<size_t>(stages) * (kD4Codes + fac) + 2 * tab + kD4KGroups * 128 * mr * 16 + 1024 + 256 +
         static_cast<size_t>(mr) * p->k * pa * 2 + static_cast<size_t>(mr) * (p->k / 32) * 4;
}

}  // namespace

cudaError_t launch_dec4(const GemmLaunch& g) {
  const QhtpMatmulPlan* pl = g.plan;
  if (!dec4_supported(pl, g.m) || g.dec4 == nullptr) return cudaErrorInvalidValue;
  const int M = static_cast<int>(g.m), K = static_cast<int>(pl->k);
  const int n_tiles = static_cast<int>(pl->n_tiles);
  const bool f32 = pl->mode == kModeF32, lpbq = lpbq_plan(pl);
  const uint8_t* img = static_cast<const uint8_t*>(pl->prepared) + int4_image_offset(pl);
  const uint8_t* codes = img;
  const uint8_t* factors = img + codes_bytes(pl);
  const uint8_t* tables = factors + factor_bytes(pl);
  CUtensorMap tc, tf;
  if (!make_tmap_2d_u8(&tc, codes, 128, static_cast<uint64_t>(n_tiles) * (K / kD4StageK) * 128, 128, 128, 128))
    return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tf, CU_TENSOR_MAP_DATA_TYPE_UINT8, lpbq ? factors : codes, 128,
                    lpbq ? static_cast<uint64_t>(n_tiles) * (K / 32) : 8, 128, 128, kD4Steps, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  D4Params prm;
  prm.M = M;
  prm.N = static_cast<int>(pl->n);
  prm.K = K;
  prm.cps = K / kD4StageK;
  prm.units = n_tiles * prm.cps;
  int grid = sm_count_d4();
  if (grid > kD4MaxCtas) grid = kD4MaxCtas;
  if (grid > prm.units) grid = prm.units;
  prm.grid = grid;
  prm.fac_rows = K / 32;
  prm.act = g.act;
  prm.rec = reinterpret_cast<const ChannelRecord*>(static_cast<const uint8_t*>(pl->prepared) + pl->plane_bytes);
  prm.tables = tables;
  prm.out = g.out;
  prm.partial = reinterpret_cast<long long*>(g.dec4);
  prm.zp_out = pl->out_zp;
  prm.qmax = pl->out_qmax;
  prm.act_mant = pl->act_mant;
  prm.out_mant = pl->out_mant;
  prm.act_exp2 = pl->act_exp2;
  prm.out_exp2 = pl->out_exp2;
  prm.err = g.err;
  const int mr = rows_bucket(g.m);
  const int key = (pl->a_planes == 2 ? 4 : 0) + (f32 ? 2 : 0) + (lpbq ? 1 : 0);
  switch (key) {
    case 0: return launch_d4_rows<1, kModeExact, false>(mr, tc, tf, prm, g.stream);
    case 1: return launch_d4_rows<1, kModeExact, true>(mr, tc, tf, prm, g.stream);
    case 2: return launch_d4_rows<1, kModeF32, false>(mr, tc, tf, prm, g.stream);
    case 3: return launch_d4_rows<1, kModeF32, true>(mr, tc, tf, prm, g.stream);
    case 4: return launch_d4_rows<2, kModeExact, false>(mr, tc, tf, prm, g.stream);
    case 5: return launch_d4_rows<2, kModeExact, true>(mr, tc, tf, prm, g.stream);
    case 6: return launch_d4_rows<2, kModeF32, false>(mr, tc, tf, prm, g.stream);
    case 7: return launch_d4_rows<2, kModeF32, true>(mr, tc, tf, prm, g.stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qhtp
