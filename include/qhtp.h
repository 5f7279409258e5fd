/* qhtp.h -- C ABI of the B200 (sm_100a) quantized MatMul family and GDN chunk inverse.
 *
 * Plain pointers and sizes only.  Every buffer is caller-owned device memory unless stated
 * otherwise; nothing here allocates device memory.  Work is enqueued on the caller's CUDA
 * stream (`stream` is a cudaStream_t passed as void*; NULL = legacy default stream) and is
 * asynchronous unless a function says it synchronizes.
 *
 * Reference interfaces replaced (paths inside the zzh-www/qcom_htp tree):
 *   - handwritten C ABI   example/handwritten_hmx_matmul/include/handwritten_hmx_matmul.h:11-52
 *       HmStatus, HmPreparedRun, hm_<family>_run_prepared, hm_status_string
 *   - QNN custom ops       HmxU8I8ToU8MatMul  (example/qnn_hmx_matmul_u8i8/src/HmxU8I8ToU8MatMulOp.cpp:481-792)
 *                          HmxU8I4ToU8MatMul  (example/qnn_hmx_matmul_w4a8/src/HmxU8I4ToU8MatMulOp.cpp:1113-1122)
 *                          HmxU16I8ToU16MatMul (example/qnn_hmx_matmul_w8a16/src/HmxU16I8ToU16MatMulOp.cpp)
 *                          HmxU16I4ToU16MatMul (example/qnn_hmx_matmul_w4a16/src/HmxU16I4ToU16MatMulOp.cpp)
 *                          HmxU16I16ToU16MatMul (example/qnn_hmx_matmul_w16a16/src/HmxU16I16ToU16MatMulOp.cpp:912,1214)
 *                          HmxW4LpbqExpandToI8 (example/qnn_hmx_matmul_common/HmxW4LpbqExpandToI8Op.cpp:49-157)
 *   - GDN solve            gdnbm_solve (example/gdn_native/baremetal/inc/gdnbm.idl:10-12),
 *                          GdnSolve op (example/gdn_native/solve_op/src/GdnSolveOp.cpp:195-281)
 */
#ifndef QHTP_H_
#define QHTP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: same values and meaning as HmStatus (handwritten_hmx_matmul.h:11-16). */
typedef enum QhtpStatus {
  QHTP_STATUS_OK = 0,
  QHTP_STATUS_INVALID_ARGUMENT = 1,
  QHTP_STATUS_UNSUPPORTED = 2,
  QHTP_STATUS_RUNTIME_ERROR = 3
} QhtpStatus;

/* Replaces hm_status_string (handwritten_hmx_matmul.h:52). */
const char *qhtp_status_string(QhtpStatus status);

/* ------------------------------------------------------------------------------------------
 * Quantized MatMul:  out[M,N] = requant( act[M,K] (x) weight[N,K] + bias )
 *
 * Semantics (QNN affine, offset = -zero_point):  x = (x_q + act_offset) * act_scale,
 * w = deq(w_q), b = bias_q * act_scale * weight_scale[n],
 * out_q = clip(round_half_even(y / out_scale - out_offset), 0, 2^out_bits - 1).
 * Dequant modes:
 *   QHTP_DEQUANT_F32_WEIGHT  deq(w_q) = float32(w_q * weight_scale[n]) -- the reference oracle's
 *                            rule (scripts/generate_qnn_matmul_python_cases.py:307,361); outputs
 *                            are bit-exact to it.
 *   QHTP_DEQUANT_EXACT       deq(w_q) = w_q * weight_scale[n] exactly (W16A16 semantics,
 *                            docs/w16a16_is_two_w8a16.md:14-36).
 * ------------------------------------------------------------------------------------------ */
typedef enum QhtpFamily {
  QHTP_FAMILY_U8I8 = 0,   /* u8 act  x int8 weight  -> u8   */
  QHTP_FAMILY_W4A8 = 1,   /* u8 act  x int4 weight  -> u8   */
  QHTP_FAMILY_W8A16 = 2,  /* u16 act x int8 weight  -> u16  */
  QHTP_FAMILY_W4A16 = 3,  /* u16 act x int4 weight  -> u16  */
  QHTP_FAMILY_W16A16 = 4  /* u16 act x int16 weight -> u16 (two byte-weight passes) */
} QhtpFamily;

typedef enum QhtpWeightSchema {
  QHTP_SCHEMA_PER_CHANNEL = 0, /* symmetric per-output-channel scale                         */
  QHTP_SCHEMA_LPBQ = 1,        /* int4 x per-block uint8 factor (1..16) x per-channel scale;  */
                               /* expanded exactly like HmxW4LpbqExpandToI8Op.cpp:94-97        */
  QHTP_SCHEMA_PER_GROUP = 2    /* W4 families only: float32 scale per (channel, 64 weights of  */
                               /* K), float32 bias; scripts/generate_qnn_matmul_python_cases.py */
                               /* :392-423 (weights) and :460-470 (bias kept float)             */
} QhtpWeightSchema;

typedef enum QhtpDequant {
  QHTP_DEQUANT_F32_WEIGHT = 0,
  QHTP_DEQUANT_EXACT = 1
} QhtpDequant;

/* Weight-side inputs (all device pointers).
 * weight layout by family:
 *   U8I8, W8A16 : int8  [N, K] row-major (the reference's weight_q_nk)
 *   W4A8, W4A16 : int4 K-pair bytes [K/2, N]: byte (k>>1)*N + n, even k in the low nibble,
 *                 two's-complement nibbles (HmxW4LpbqExpandToI8Op.cpp:5,32-40)
 *   W16A16      : int16 [N, K] row-major
 * lpbq_block_scale: uint8 [N, K/lpbq_block] (n*(K/lpbq_block) + kb), LPBQ only, else NULL.
 * QHTP_SCHEMA_PER_GROUP: weight_scale is float32 [N, K/64] (n*(K/64) + g), K a multiple of 64 and
 * above 64, dequant QHTP_DEQUANT_F32_WEIGHT; bias_q is unused and bias_float (float32 [N]) is the
 * bias, added in float64 like the reference (y = x_deq @ w_deq.T + bias). */
typedef struct QhtpMatmulWeights {
  uint32_t family;      /* QhtpFamily       */
  uint32_t schema;      /* QhtpWeightSchema */
  uint32_t dequant;     /* QhtpDequant      */
  uint32_t k;
  uint32_t n;
  uint32_t lpbq_block;  /* 32 or 64 (multiple of 32, divides K); 0 when not LPBQ */
  const void *weight;
  const float *weight_scale;         /* [N] float32, finite, > 0, normal */
  const int32_t *bias_q;             /* [N] int32                        */
  const uint8_t *lpbq_block_scale;
  double act_scale;
  int32_t act_offset;                /* QNN offset = -zero_point (-128 for u8, -32768 for u16) */
  double out_scale;
  int32_t out_offset;                /* 0 for u8 outputs, -32768 for u16 outputs */
  const float *bias_float;           /* [N] float32, QHTP_SCHEMA_PER_GROUP only, else NULL */
} QhtpMatmulWeights;

/* Host-side plan: filled by qhtp_matmul_plan (host only) and bound to a prepared device buffer by
 * qhtp_matmul_prepare.  Treat as opaque; it is plain data and may be copied. */
typedef struct QhtpMatmulPlan {
  uint32_t magic;
  uint32_t family, schema, dequant, k, n, lpbq_block;
  uint32_t act_bits, weight_bits, out_bits;
  uint32_t mode;          /* kernel variant */
  uint32_t a_planes;      /* 1 (u8 act) or 2 (u16 act as hi/lo byte planes) */
  uint32_t ch_per_tile;   /* output channels per 128-row tile */
  uint32_t n_tiles;
  uint32_t k_pad;         /* K rounded up to 128 */
  int32_t act_zp, out_zp, out_qmax;
  double act_scale, out_scale;
  uint64_t act_mant;      /* act_scale = act_mant * 2^act_exp2, 53-bit mantissa */
  int32_t act_exp2;
  uint32_t flags;         /* kernel options (QHTP_PLAN_FLAG_*), set by qhtp_matmul_prepare but the FORCE_* ones */
  uint64_t out_mant;
  int32_t out_exp2;
  uint64_t plane_bytes;   /* prepared weight planes */
  uint64_t record_bytes;  /* per-channel records (32 bytes each) */
  uint64_t prepared_bytes;
  void *prepared;         /* device buffer bound by qhtp_matmul_prepare */
} QhtpMatmulPlan;

/* QhtpMatmulPlan.flags.  LO_RESIDUAL_BY_BOUND: the lo-plane x e' product of the u16 row-tiled GEMM
 * is bounded per channel, so the GEMM may leave it out of its MMAs (exact fix-up of the elements near
 * a rounding boundary).  LO_RESIDUAL_PAYS: the expected fix-ups are few enough (at most ~6 per
 * 128 x 128 tile on average over the channels) that leaving it out is faster; the GEMM then does so
 * for launches of at least three waves of tiles (with fewer, the last tile's fix-ups are not hidden
 * behind a next tile).  INT4_STREAM: the prepared buffer holds the 4-bit code image (int4 families,
 * per-channel or LPBQ with factors in [1, 16], K % 256 == 0) and runs of M <= 2 rows over a long
 * enough weight stream (at least six 256-deep stages per SM) read it instead of the byte planes.
 * FORCE_INT4_STREAM / FORCE_LO_RESIDUAL: set by the caller before or after prepare; M <= 2 then takes
 * the code stream at any shape, and every row-tiled launch with a valid bound leaves the lo-plane x
 * e' product out (tests, benchmarks).  Every variant gives the same output bytes. */
#define QHTP_PLAN_FLAG_LO_RESIDUAL_BY_BOUND 1u
#define QHTP_PLAN_FLAG_INT4_STREAM 2u
#define QHTP_PLAN_FLAG_FORCE_INT4_STREAM 4u
#define QHTP_PLAN_FLAG_LO_RESIDUAL_PAYS 8u
#define QHTP_PLAN_FLAG_FORCE_LO_RESIDUAL 16u

/* Validate shapes / family / schema and fill *plan (host only, no device access).
 * Requirements: K % 32 == 0, 32 <= K <= 32768, N % 32 == 0, N >= 32; LPBQ only for int4 families. */
QhtpStatus qhtp_matmul_plan(const QhtpMatmulWeights *w, QhtpMatmulPlan *plan);

/* Device bytes qhtp_matmul_prepare needs (== plan->prepared_bytes). */
size_t qhtp_matmul_prepared_bytes(const QhtpMatmulPlan *plan);

/* Build the prepared record in `prepared` (device, >= prepared_bytes, 256-byte aligned):
 * byte-plane weights in the tiled layout the kernel streams, one 32-byte record per output
 * channel (effective bias, requant multiplier, exact-path exponents) and, for the int4 families,
 * the 4-bit code image with its per-(channel, factor) e' tables.  This is the B200 analogue
 * of the reference's prepare-time const-fold (HmxW4LpbqExpandToI8Op.cpp:107-157,
 * gen_quant_chain.py:879).  Synchronizes `stream` to validate the scales. */
QhtpStatus qhtp_matmul_prepare(QhtpMatmulPlan *plan, const QhtpMatmulWeights *w, void *prepared,
                               size_t prepared_bytes, void *stream);

/* Device workspace qhtp_matmul_run needs for M rows (u16 byte planes + error word). */
size_t qhtp_matmul_workspace_bytes(const QhtpMatmulPlan *plan, uint32_t m);

/* out[M,N] (u8 or u16, row-major) from act[M,K] (u8 or u16, row-major).  act and out must be
 * 16-byte aligned.  Asynchronous.  Device-side failures (a timed-out pipeline wait) are reported
 * by qhtp_matmul_check. */
QhtpStatus qhtp_matmul_run(const QhtpMatmulPlan *plan, const void *act, uint32_t m, void *out,
                           void *workspace, size_t workspace_bytes, void *stream);

/* qhtp_matmul_run with the row-tiled GEMM's persistent grid limited to max_ctas CTAs, one per SM
 * (0: every SM), so that the other SMs stay free for work running at the same time on other streams --
 * e.g. the NCCL all-gather of the previous row chunk's output in a sharded multi-GPU GEMM, which cannot
 * start while the GEMM holds every SM.  The output is the same bytes as qhtp_matmul_run's.  No
 * counterpart in the reference (its HTP ops run alone on the device). */
QhtpStatus qhtp_matmul_run_ctas(const QhtpMatmulPlan *plan, const void *act, uint32_t m, void *out,
                                void *workspace, size_t workspace_bytes, uint32_t max_ctas, void *stream);

/* qhtp_matmul_run without a caller workspace.  No counterpart in the reference.
 * For callers that may not allocate device memory when they run the op -- e.g. an inference-runtime
 * plugin called from the runtime's execute step, where the runtime owns and pre-plans every device
 * buffer, or a latency-critical thread that cannot afford an allocation's implicit synchronization.
 * The u16 activation planes and the error word live in a fixed area inside the library
 * (QHTP_NOALLOC_SCRATCH_BYTES of device memory, held by every GPU that loads the library until the
 * process exits), so M*K is limited: the call needs qhtp_matmul_workspace_bytes(plan, m) <=
 * QHTP_NOALLOC_SCRATCH_BYTES (u16 byte planes, int4 decode partials for M <= 2, the error word)
 * and returns QHTP_STATUS_INVALID_ARGUMENT with a qhtp_last_error_string message otherwise.  The
 * first call on each device looks up the area's device address: make it before any stream capture.
 * All calls share the area: calls whose work overlaps on the GPU race, so serialize them.  Calls no
 * cudaMalloc / cudaFree.  M above 2^24 is QHTP_STATUS_UNSUPPORTED, as for qhtp_matmul_run.
 * Device-side pipeline timeouts are recorded in the area's error word; qhtp_matmul_noalloc_check
 * reads it. */
#define QHTP_NOALLOC_SCRATCH_BYTES (8u << 20)
QhtpStatus qhtp_matmul_run_noalloc(const QhtpMatmulPlan *plan, const void *act, uint32_t m, void *out,
                                   void *stream);

/* qhtp_matmul_check for qhtp_matmul_run_noalloc: synchronize `stream` and read (and clear) the error
 * word an M-row qhtp_matmul_run_noalloc call on the current device wrote.  No counterpart in the
 * reference.  Allocates nothing. */
QhtpStatus qhtp_matmul_noalloc_check(const QhtpMatmulPlan *plan, uint32_t m, int *device_code, void *stream);

/* qhtp_matmul_run from and to HOST memory: out_host[M,N] from act_host[M,K].  No counterpart in
 * the reference (its op runs on buffers the QNN runtime has placed); for serving from host memory.
 * The rows are processed in chunks of chunk_rows (0: the library picks ~8 chunks of a multiple of
 * 128 rows): chunk i's host->device copy runs on a library stream, its GEMM on `stream`, its
 * device->host copy on a second library stream, so copies in both directions overlap the GEMMs of
 * the other chunks.  act_dev [M,K] and out_dev [M,N] are device staging buffers (16-byte aligned);
 * workspace >= qhtp_matmul_workspace_bytes(plan, chunk_rows) (the error word for qhtp_matmul_check
 * is the one of an M = chunk_rows call; *chunk_rows_used reports the chunk size if non-NULL).  The
 * host buffers must be pinned (page-locked) for the copies to be asynchronous.  The whole
 * operation is ordered after prior work on `stream`, and later work on `stream` after it: the
 * host output is complete once `stream` is.  Calls no cudaMalloc / cudaFree (the library's two
 * copy streams and its events are created once per device). */
QhtpStatus qhtp_matmul_run_host(const QhtpMatmulPlan *plan, const void *act_host, uint32_t m, void *out_host,
                                void *act_dev, void *out_dev, void *workspace, size_t workspace_bytes,
                                uint32_t chunk_rows, uint32_t *chunk_rows_used, void *stream);

/* Synchronize `stream` and read the device error word of `workspace`; clears it.  Returns
 * QHTP_STATUS_RUNTIME_ERROR if a kernel recorded an error (code in *device_code if non-NULL). */
QhtpStatus qhtp_matmul_check(const QhtpMatmulPlan *plan, void *workspace, uint32_t m, int *device_code,
                             void *stream);

/* Failure-path self-test (no counterpart in the reference, whose kernels report nothing).  Launches
 * one 4-warp CTA that waits, with the library's bounded pipeline wait, on an mbarrier that no thread
 * arrives on.  Each wait gives up after limit_cycles (1 .. 2^32) cycles of the SM clock, records
 * code 4 (the code of a timed-out pipeline wait) in the device word *err_word unless it is already
 * non-zero, adds 1 per warp to the device counter *warps_gave_up, and the kernel returns.  Point
 * err_word at a workspace's error word and qhtp_matmul_check reports QHTP_STATUS_RUNTIME_ERROR with
 * that code, exactly as it would for a GEMM whose pipeline stalled.  Asynchronous. */
QhtpStatus qhtp_selftest_wait_timeout(int *err_word, int *warps_gave_up, uint64_t limit_cycles, void *stream);

/* Tensor-pipe rate probe (no counterpart in the reference): `ctas` CTAs (one per SM) each issue
 * `iters` rounds of four tcgen05.mma of M = 128, N = 256 -- kind 0: kind::i8 (u8 x s8, s32
 * accumulate, 32 bytes of K per instruction), kind 1: kind::f16 with bf16 operands (f32 accumulate,
 * 16 elements of K) -- on shared-memory operands, with no memory traffic.  Time the launch on
 * `stream` with CUDA events: executed ops = ctas * iters * 4 * 2 * 128 * 256 * (32 | 16).  A timed-out
 * completion wait records code 3 in the device word *err_word.  Asynchronous. */
QhtpStatus qhtp_selftest_mma_rate(uint32_t kind, uint32_t iters, uint32_t ctas, int *err_word, void *stream);

/* Read back the prepared per-channel records (the B200 "sidecar", 32 bytes per channel, padded to
 * the tile) into host memory: sizes in bytes.  Synchronizes `stream`. */
QhtpStatus qhtp_matmul_read_records(const QhtpMatmulPlan *plan, void *host_dst, size_t bytes, void *stream);

/* LPBQ expand (HmxW4LpbqExpandToI8 semantics, HmxW4LpbqExpandToI8Op.cpp:26-47,94-97):
 * int4 K-pair [K/2, N] x uint8 factor [N, K/block] -> int8 [N, K] row-major, saturated. */
QhtpStatus qhtp_lpbq_expand_i8(const uint8_t *w4_kpair, const uint8_t *block_scale, uint32_t k, uint32_t n,
                               uint32_t block, int8_t *out_nk, void *stream);

/* ---- Reference weight wire formats -> this library's plain weight carriers.
 * The layouts the reference's QNN MatMul ops read from their ONNX initializers
 * (example/qnn_hmx_matmul_common/gen_quant_chain.py:285-742), so existing weight files load
 * unchanged: decode once on the device, then pass the plain carrier to qhtp_matmul_plan/prepare.
 * Output: int8 [N, K] row-major for the W8 formats; int4 K-pair bytes [K/2, N] (byte (k/2)*N + n,
 * low nibble = even k, two's complement) for the W4 formats. ---- */
typedef enum QhtpWireFormat {
  QHTP_WIRE_W8_RAW_KN = 1,            /* int8 [K, N] (w8a16 "raw"; u8i8 with QHTP_WIRE_XOR80), :728-741 */
  QHTP_WIRE_W8_KMAJOR_TILE32 = 2,     /* 32x32 K-major HMX tiles, dst = (r/4)*128 + c*4 + r%4, :285-303 */
  QHTP_WIRE_W8_KMAJOR_SPLIT128 = 3,   /* K-major tiles per 128-channel stream, :306-314 */
  QHTP_WIRE_W4_TILE32X64_NPAIR32 = 4, /* W4A8 HMX: 32x64 K-major tiles, byte = channels n | n+32, :686-712 */
  QHTP_WIRE_W4_KPAIR = 5,             /* [K/2, N] K-pairs (also the LPBQ pre-chain weight), :369-382 */
  QHTP_WIRE_W4_NMAJOR_KPAIR = 6,      /* [N, K/2] K-pairs, :385-398 */
  QHTP_WIRE_W4_NMAJOR_K4 = 7,         /* N32 tiles, K8 groups, k / k+4 pairs, :401-422 */
  QHTP_WIRE_W4_KBLOCK32_NMAJOR_K4 = 8,/* K32 blocks, then N32 tiles, k / k+4 pairs, :425-452 */
  QHTP_WIRE_W4_NPAIR_ADJACENT = 9,    /* [N/2, K], byte = channels 2j | 2j+1, :455-468 */
  QHTP_WIRE_W4_NPAIR_TILE32 = 10,     /* [N/2, K], byte = channels n | n+32 per 64-channel tile, :471-489 */
  QHTP_WIRE_W4_FULL_CODES = 11        /* [K, N], one code per byte, :619-627 */
} QhtpWireFormat;
#define QHTP_WIRE_XOR80 1u  /* every carrier byte XOR 0x80 (the int8 carriers of the QNN sidecar) */
#define QHTP_WIRE_HILO 2u   /* "hilo" orders: the first element of a byte pair in the high nibble */
#define QHTP_WIRE_BIASED 4u /* "biased" nibble encoding: code = v + 8 */

/* Bytes of a wire-format weight [K, N] (0 for an unknown format). */
size_t qhtp_wire_bytes(uint32_t format, uint32_t k, uint32_t n);

/* Decode `wire` (device, qhtp_wire_bytes) into `plain` (device, K*N bytes for W8 formats, K*N/2
 * for W4).  QHTP_STATUS_UNSUPPORTED for shapes the layout cannot hold (tile multiples of K / N).
 * Asynchronous on `stream`. */
QhtpStatus qhtp_weights_from_wire(uint32_t format, uint32_t flags, const void *wire, size_t wire_bytes, uint32_t k,
                                  uint32_t n, void *plain, size_t plain_bytes, void *stream);

/* ---- prepared-run entry points, one per family (hm_<family>_run_prepared,
 *      handwritten_hmx_matmul.h:28-50).  chain > 1 re-applies the same op chain times, each
 *      output feeding the next activation (requires K == N and equal act/out widths); the
 *      intermediate results live in `scratch` after the workspace. ---- */
typedef struct QhtpBuffer {
  void *data;
  size_t bytes;
} QhtpBuffer;

typedef struct QhtpConstBuffer {
  const void *data;
  size_t bytes;
} QhtpConstBuffer;

typedef struct QhtpPreparedRun {
  uint32_t m, k, n, chain;
  QhtpConstBuffer activation;   /* device [M,K] */
  const QhtpMatmulPlan *plan;   /* prepared by qhtp_matmul_prepare */
  QhtpBuffer scratch;           /* device, >= qhtp_prepared_run_scratch_bytes */
  QhtpBuffer output;            /* device [M,N] */
  void *stream;
} QhtpPreparedRun;

size_t qhtp_prepared_run_scratch_bytes(const QhtpMatmulPlan *plan, uint32_t m, uint32_t chain);
QhtpStatus qhtp_u8i8_run_prepared(const QhtpPreparedRun *run);
QhtpStatus qhtp_w4a8_run_prepared(const QhtpPreparedRun *run);
QhtpStatus qhtp_w8a16_run_prepared(const QhtpPreparedRun *run);
QhtpStatus qhtp_w4a16_run_prepared(const QhtpPreparedRun *run);
QhtpStatus qhtp_w16a16_run_prepared(const QhtpPreparedRun *run);

/* ------------------------------------------------------------------------------------------
 * GDN / KDA chunk triangular inverse  T = (I - A)^-1,  A strictly lower triangular [C, C].
 * n_chunks independent (batch, head, chunk) matrices, row-major, contiguous.
 * C in {32, 64, 128, 256}.  Inputs above the diagonal are ignored (treated as zero); the output
 * upper triangle is written as zero.
 * ------------------------------------------------------------------------------------------ */

/* A bf16 [n_chunks, C, C] -> T float32 [n_chunks, C, C]. */
QhtpStatus qhtp_gdn_inverse_bf16(const void *A, float *T, int64_t n_chunks, int32_t C, void *stream);

/* The chunk's A built on the GPU from the gated-delta-rule inputs and inverted in the same kernel, as
 * the reference's chunk kernel does (Stage A of gdn_chunk, scripts/gdn_ref_kernel.py:66-82):
 * k L2-normalised (eps 1e-6), g = cumsum of the per-token log gates over the chunk,
 * A[i][j] = -beta_i (k_i . k_j) exp(g_i - g_j) for i > j, T = (I - A)^-1.  A never reaches memory.
 * k bf16 [n_chunks, C, Dk] (raw keys), beta and g float32 [n_chunks, C] -> T float32 [n_chunks, C, C].
 * C = 256 and Dk = 128 (QHTP_STATUS_UNSUPPORTED otherwise); 16-byte aligned buffers. */
QhtpStatus qhtp_gdn_chunk_inverse(const void *k, const float *beta, const float *g, float *T, int64_t n_chunks,
                                  int32_t C, int32_t dk, void *stream);

/* u16-code carrier (gdnbm.idl:10-12, gdn_solve_oc_check.py:28-29): value = (code - zp) * scale.
 * A codes [n_chunks, C, C] -> T codes, T_code = clip(rint(T / sT) + zpT, 0, 65535). */
QhtpStatus qhtp_gdn_solve_u16(const uint16_t *A, int64_t n_chunks, int32_t C, int32_t zpA, float sA,
                              int32_t zpT, float sT, uint16_t *T, void *stream);

/* ------------------------------------------------------------------------------------------
 * Host-only helpers (no GPU needed).
 * ------------------------------------------------------------------------------------------ */

/* Library version string. */
const char *qhtp_version(void);

/* Text of the last CUDA error behind a QHTP_STATUS_RUNTIME_ERROR on the calling thread. */
const char *qhtp_last_error_string(void);

/* The exact requant decision the kernels use, on the host (for tests):
 * clip(round_half_even(T*mul*act_mant*2^e2 / (out_mant*2^out_exp2) + zp_out), 0, qmax), with the
 * same fixed-point fast path (multiplier c = cm * 2^-cshift, cshift >= 34, i.e. c < 2^18) and 128-bit exact
 * tie check as the device epilogue.  Returns -1 for a cshift outside [34, 1074]. */
int32_t qhtp_requant_code_host(int64_t T, uint64_t cm, int32_t cshift, uint32_t mul, int32_t e2,
                               uint64_t act_mant, uint64_t out_mant, int32_t out_exp2, int32_t zp_out,
                               int32_t qmax);

#ifdef __cplusplus
}
#endif

#endif /* QHTP_H_ */
