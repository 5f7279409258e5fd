// Declarations shared between the .cu translation units of libqhtp (not part of the public ABI).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/qhtp.h"

namespace qhtp {

constexpr uint32_t kPlanMagic = 0x51485450u;  // "QHTP"

// Kernel variants of the quantized GEMM.  Every tile covers 128 output rows x 128 output channels.
enum GemmMode : uint32_t {
  kModeF32 = 0,    // f32 weight dequant: B tile = [q (128 ch) | e' (128 ch)], s8
  kModeExact = 1,  // exact dequant, 8-bit weights: B tile = q (128 ch), s8
  kModeW16 = 2,    // exact dequant, int16 weights: B tile = [hi s8 (128 ch) | lo u8 (128 ch)]
  kModeGroup = 3,  // per-group W4 (float32 scale per 64 weights of K): channel-major tiles,
                   // weight image = [q (128 ch) | e' (128 ch)], s8; qgroup.cu
};

// QhtpMatmulPlan.flags (set by qhtp_matmul_prepare)
constexpr uint32_t kPlanLoResidualByBound = 1u;  // the lo-plane x e' product is bounded per channel
                                                 // (ChannelRecord::lo_win), so the GEMM may leave it out of
                                                 // the MMAs; elements within that bound of a rounding
                                                 // boundary then get it exactly
constexpr int32_t kLoWinMax = 1 << 20;           // widest per-channel window that enables it (~1e-3 units)
constexpr uint32_t kPlanLoResidualPays = 8u;     // mean window <= kLoWinMeanMax: the bound is worth using
constexpr uint32_t kPlanForceLoResidual = 16u;   // set by the caller: use the bound on every launch
// A value is sent to the exact fix-up with probability ~2 (lo_win + 2) / 2^30, so a 128 x 128 tile
// expects 2^15 (mean lo_win + 2) / 2^30 fix-ups; 3 * 2^16 is ~6 per tile.  Measured on B200 at
// K = 4096: ~3 per tile (W4A16) gains 8 %, ~8.5 (W8A16) loses 5 %.
constexpr uint64_t kLoWinMeanMax = 3u << 16;
constexpr int kLoResidualMinWaves = 3;           // row-tiled launches of fewer waves keep the full product
constexpr uint32_t kPlanInt4Stream = 2u;         // the int4 code image was built (qdec4.cu): decode rows
                                                 // stream 4-bit codes instead of the byte planes
constexpr uint32_t kPlanForceInt4Stream = 4u;    // set by the caller: M <= 2 takes the code stream at any shape
constexpr int kSumsPerChannel = 4;               // prepare scratch: sum q, sum e', sum |e'|, unused

constexpr int kTileM = 128;      // rows per CTA tile (TMEM lanes)
constexpr int kTileN = 128;      // output channels per tile
constexpr int kTileK = 128;      // bytes of K per pipeline stage (one 128-byte swizzle row)

// weight-plane rows per tile in the prepared layout
inline constexpr uint32_t b_rows_for_mode(uint32_t mode) { return mode == kModeExact ? 128u : 256u; }

// Per-group schema: channels per tile, and the constants of one (tile, group) in the prepared
// buffer: K int64[128] = bits(1.5*2^52) - zp*(m*sum q + sum e') | 2^e float64[128] | m int32[128]
constexpr int kGroupTileN = 128;
constexpr int kGroupRecBytes = kGroupTileN * (8 + 8 + 4);
inline size_t group_rec_bytes(const QhtpMatmulPlan* p) {
  const size_t b = static_cast<size_t>(p->n_tiles) * (p->k_pad / kTileK) * 2 * kGroupRecBytes;
  return (b + 255) / 256 * 256;
}

struct ChannelRecord {  // 32 bytes, one per output channel (padded to the tile)
  int64_t beff;         // effective bias, in accumulator units
  uint64_t cmn;         // requant multiplier, applied as (|T| << tn) * cmn * 2^-96 (see fast_const)
  int32_t m_q;          // multiplier of the q-plane accumulator inside T
  uint32_t wbits;       // float32 weight-scale bits: mantissa/exponent for the exact tie check
  int32_t tn;           // left shift of |T| in the fast path
  int32_t lo_win;       // f32 mode, u16 activation: bound on |sum_k x_lo * e'| * c in 2^-30 output
                        // units, ceil(255 * sum_k |e'| * c * 2^30) + 1 (capped at 2^30); else 0
};
static_assert(sizeof(ChannelRecord) == 32, "record layout");

struct GemmLaunch {
  const QhtpMatmulPlan* plan;
  const void* act;        // user activation [M,K]
  uint32_t m;
  void* out;
  uint8_t* planes;        // workspace: u16 act byte planes [2][M][K] (A16 only)
  int* err;               // workspace: device error word
  cudaStream_t stream;
  uint32_t max_ctas = 0;  // row-tiled GEMM: at most this many persistent CTAs (0: one per SM)
  uint8_t* dec4 = nullptr;  // workspace area of the int4-stream decode kernel (dec4_workspace_bytes)
};

// qhtp_abi.cu: status of a CUDA result (records the error for qhtp_last_error_string), and a
// validation message for qhtp_last_error_string (static storage only)
QhtpStatus status_from_cuda(cudaError_t e);
void set_last_message(const char* msg);

// qgemm.cu
cudaError_t launch_gemm(const GemmLaunch& g);
// u16 activation [total elements] -> byte planes hi [total] | lo [total] at `planes`
cudaError_t launch_split_u16(const uint16_t* act, uint8_t* planes, size_t total, cudaStream_t stream);
// qchain.cu: CHAIN=N in one kernel (K == N <= 256, act width == out width, not per-group)
bool chain_fusable(const QhtpMatmulPlan* plan);
cudaError_t launch_chain(const GemmLaunch& g, uint32_t chain);
// qdecode.cu: channel-major (swap-AB) kernel for M <= kDecodeMaxM activation rows; a_base is the
// u8 activation or the [hi; lo] byte planes of a u16 activation
constexpr uint32_t kDecodeMaxM = 128;
bool decode_supported(const QhtpMatmulPlan* plan, uint32_t m);
cudaError_t launch_decode(const GemmLaunch& g, const uint8_t* a_base);
cudaError_t launch_prepare(const QhtpMatmulPlan* plan, const QhtpMatmulWeights* w, void* prepared,
                           int* bad_scale, cudaStream_t stream);
// qdec4.cu: decode rows (M <= kDec4MaxM) of int4-weight plans (per-channel or LPBQ, K % 256 == 0),
// streaming the 4-bit codes; the prepared buffer holds its code image after the per-channel sums
constexpr uint32_t kDec4MaxM = 2;
bool int4_stream_layout(const QhtpMatmulPlan* plan);                 // the plan has the code image
size_t int4_image_bytes(const QhtpMatmulPlan* plan);                 // 0 when it has none
size_t int4_image_offset(const QhtpMatmulPlan* plan);                // in the prepared buffer
size_t dec4_workspace_bytes(const QhtpMatmulPlan* plan, uint32_t m);  // 0 when the kernel cannot run
bool dec4_supported(const QhtpMatmulPlan* plan, uint32_t m);         // prepared, flag set, m in range
// status[2] != 0 after the stream completes: a block factor outside [1, 16] (the codes stay unused)
cudaError_t launch_prepare_int4(const QhtpMatmulPlan* plan, const QhtpMatmulWeights* w, void* prepared,
                                int* status, cudaStream_t stream);
cudaError_t launch_dec4(const GemmLaunch& g);
// qhtp_abi.cu: the int4-stream decode area inside a run's workspace (nullptr when it has none)
uint8_t* dec4_area(const QhtpMatmulPlan* plan, uint32_t m, uint8_t* workspace);
// qgroup.cu: the per-group W4 schema (prepare, and the GEMM on the u8 activation or byte planes)
cudaError_t launch_prepare_group(const QhtpMatmulPlan* plan, const QhtpMatmulWeights* w, void* prepared,
                                 int* bad_scale, cudaStream_t stream, int sms);
cudaError_t launch_gemm_group(const GemmLaunch& g, const uint8_t* a_base, uint64_t a_rows, int sms);
cudaError_t launch_wait_timeout(int* err, long long limit, int* gave_up, cudaStream_t stream);
cudaError_t launch_lpbq_expand(const uint8_t* w4, const uint8_t* bs, uint32_t k, uint32_t n, uint32_t block,
                               int8_t* out, cudaStream_t stream);

// gdn.cu
cudaError_t launch_gdn_bf16(const void* A, float* T, int64_t n_chunks, int C, cudaStream_t stream);
cudaError_t launch_gdn_u16(const uint16_t* A, int64_t n_chunks, int C, int zpA, float sA, int zpT, float sT,
                           uint16_t* T, cudaStream_t stream);
// gdn256.cu: C = 256, tensor-core doubling kernel (bf16 in / f32 out, or u16 codes in / out)
bool gdn256_supported(const void* A, const void* T, int64_t n_chunks);
cudaError_t launch_gdn256_bf16(const void* A, float* T, int64_t n_chunks, cudaStream_t stream);
// gdn256f.cu: fused A construction (k, beta, log gates) + inverse, C = 256, Dk = 128
bool gdn256f_supported(const void* k, const float* beta, const float* g, const float* T, int64_t n_chunks);
cudaError_t launch_gdn256_fused(const void* k, const float* beta, const float* g, float* T, int64_t n_chunks,
                                cudaStream_t stream);
cudaError_t launch_gdn256_u16(const uint16_t* A, int64_t n_chunks, int zpA, float sA, int zpT, float sT, uint16_t* T,
                              cudaStream_t stream);

// tensor maps (qgemm.cu)
bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t rows,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);
// prepared weight planes: box (tile, K block) at row (tile * kblocks + kb) * b_rows, copied verbatim
bool make_tmap_planes(CUtensorMap* map, const QhtpMatmulPlan* plan);
bool make_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                     uint32_t box_inner, uint32_t box_rows);

}  // namespace qhtp
