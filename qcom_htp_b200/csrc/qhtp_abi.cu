// C ABI of libqhtp: argument validation, planning, and dispatch to the kernels.
//
// Error behaviour follows the reference's handwritten ABI (HmStatus, handwritten_hmx_matmul.cpp:8-46):
// any null pointer, zero size or undersized buffer is QHTP_STATUS_INVALID_ARGUMENT; a shape the
// kernels do not cover is QHTP_STATUS_UNSUPPORTED; a CUDA failure is QHTP_STATUS_RUNTIME_ERROR.
// Unlike the QHPI kernels (which return QHPI_Success on bad inputs, HmxU8I8ToU8MatMulOp.cpp:500),
// nothing here fails silently.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "requant.cuh"

using namespace qhtp;

namespace {

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool family_bits(uint32_t family, uint32_t* act, uint32_t* wt, uint32_t* out) {
  switch (family) {
    case QHTP_FAMILY_U8I8: *act = 8; *wt = 8; *out = 8; return true;
    case QHTP_FAMILY_W4A8: *act = 8; *wt = 4; *out = 8; return true;
    case QHTP_FAMILY_W8A16: *act = 16; *wt = 8; *out = 16; return true;
    case QHTP_FAMILY_W4A16: *act = 16; *wt = 4; *out = 16; return true;
    case QHTP_FAMILY_W16A16: *act = 16; *wt = 16; *out = 16; return true;
    default: return false;
  }
}

// x = mant * 2^exp2 with a 53-bit integer mantissa (x finite, > 0).
void split_f64(double x, uint64_t* mant, int32_t* exp2) {
  int e = 0;
  const double fr = std::frexp(x, &e);          // x = fr * 2^e, fr in [0.5, 1)
  *mant = static_cast<uint64_t>(std::ldexp(fr, 53));
  *exp2 = e - 53;
}

size_t a16_plane_bytes(const QhtpMatmulPlan* p, uint32_t m) {
  return p->a_planes == 2 ? align_up(2ull * m * p->k, 256) : 0;
}

bool plan_ok(const QhtpMatmulPlan* p) { return p != nullptr && p->magic == kPlanMagic; }

// Workspace of a run over m rows: u16 byte planes | int4-stream decode area | 256-byte error area.
size_t err_offset(const QhtpMatmulPlan* p, uint32_t m) { return a16_plane_bytes(p, m) + dec4_workspace_bytes(p, m); }

}  // namespace

namespace qhtp {

uint8_t* dec4_area(const QhtpMatmulPlan* plan, uint32_t m, uint8_t* workspace) {
  return dec4_workspace_bytes(plan, m) != 0 ? workspace + a16_plane_bytes(plan, m) : nullptr;
}

}  // namespace qhtp

namespace qhtp {

// Last failure on the calling thread: a CUDA error, or a message from host-side validation.
thread_local cudaError_t g_last_cuda_error = cudaSuccess;
thread_local const char* g_last_message = nullptr;

QhtpStatus status_from_cuda(cudaError_t e) {
  if (e == cudaSuccess) return QHTP_STATUS_OK;
  g_last_cuda_error = e;
  g_last_message = nullptr;
  return QHTP_STATUS_RUNTIME_ERROR;
}

void set_last_message(const char* msg) { g_last_message = msg; }

}  // namespace qhtp

namespace {
QhtpStatus from_cuda(cudaError_t e) { return qhtp::status_from_cuda(e); }

// qhtp_matmul_run_host: per device, two copy streams (host->device, device->host) and the events
// that chain each row chunk's copy in, GEMM and copy out.  Created on first use, kept until the
// process exits; one call at a time uses them (the events are re-recorded by every call).
constexpr uint32_t kHostMaxChunks = 64;
constexpr int kHostMaxDevices = 64;
struct HostPipe {
  std::mutex mu;
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t start = nullptr, done = nullptr;
  cudaEvent_t copied[kHostMaxChunks] = {}, computed[kHostMaxChunks] = {};
};

HostPipe* host_pipe() {
  static std::mutex init_mu;
  static HostPipe* pipes[kHostMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kHostMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(init_mu);
  if (pipes[dev] == nullptr) {
    HostPipe* hp = new HostPipe();
    bool ok = cudaStreamCreateWithFlags(&hp->in, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&hp->out, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&hp->start, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&hp->done, cudaEventDisableTiming) == cudaSuccess;
    for (uint32_t i = 0; ok && i < kHostMaxChunks; ++i)
      ok = cudaEventCreateWithFlags(&hp->copied[i], cudaEventDisableTiming) == cudaSuccess &&
           cudaEventCreateWithFlags(&hp->computed[i], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) return nullptr;  // what was created stays with the process
    pipes[dev] = hp;
  }
  return pipes[dev];
}

// Rows per chunk: the caller's choice, or ~8 chunks of a multiple of 128 rows (the GEMM's row
// tile); never more than kHostMaxChunks chunks, never more than M rows.
uint32_t host_chunk_rows(uint32_t m, uint32_t req) {
  uint32_t r = req;
  if (r == 0) r = ((m + 7) / 8 + 127) / 128 * 128;
  const uint32_t min_r = (m + kHostMaxChunks - 1) / kHostMaxChunks;
  if (r < min_r) r = min_r;
  if (r > m) r = m;
  return r;
}
}  // namespace

extern "C" {

const char* qhtp_status_string(QhtpStatus status) {
  switch (status) {
    case QHTP_STATUS_OK: return "ok";
    case QHTP_STATUS_INVALID_ARGUMENT: return "invalid_argument";
    case QHTP_STATUS_UNSUPPORTED: return "unsupported";
    case QHTP_STATUS_RUNTIME_ERROR: return "runtime_error";
  }
  return "unknown";
}

const char* qhtp_version(void) { return "qhtp-b200 0.1 (sm_100a)"; }

const char* qhtp_last_error_string(void) {
  if (qhtp::g_last_message != nullptr) return qhtp::g_last_message;
  return qhtp::g_last_cuda_error == cudaSuccess ? "no error" : cudaGetErrorString(qhtp::g_last_cuda_error);
}

int32_t qhtp_requant_code_host(int64_t T, uint64_t cm, int32_t cshift, uint32_t mul, int32_t e2, uint64_t act_mant,
                               uint64_t out_mant,
                               int32_t out_exp2, int32_t zp_out, int32_t qmax) {
  if (cshift < 34 || cshift > 1074) return -1;
  // same sequence as the GEMM epilogue: per-channel fast constants, branch-free fast path, exact
  // decision near a tie
  const FastConst fc = fast_const(cm, cshift);
  bool near = false;
  int64_t w = 0;
  const int32_t code = requant_fast96s(T, fc.cmn, fc.tn, zp_out, qmax, &near, &w);
  if (!near) return code;
  return requant_tie_w(T, w, mul, e2, act_mant, out_mant, out_exp2, zp_out, qmax);
}

QhtpStatus qhtp_matmul_plan(const QhtpMatmulWeights* w, QhtpMatmulPlan* plan) {
  if (w == nullptr || plan == nullptr) return QHTP_STATUS_INVALID_ARGUMENT;
  QhtpMatmulPlan p;
  std::memset(&p, 0, sizeof(p));
  if (!family_bits(w->family, &p.act_bits, &p.weight_bits, &p.out_bits)) return QHTP_STATUS_INVALID_ARGUMENT;
  if (w->schema != QHTP_SCHEMA_PER_CHANNEL && w->schema != QHTP_SCHEMA_LPBQ && w->schema != QHTP_SCHEMA_PER_GROUP)
    return QHTP_STATUS_INVALID_ARGUMENT;
  if (w->dequant != QHTP_DEQUANT_F32_WEIGHT && w->dequant != QHTP_DEQUANT_EXACT) return QHTP_STATUS_INVALID_ARGUMENT;
  if (w->k == 0 || w->n == 0) return QHTP_STATUS_INVALID_ARGUMENT;
  if (w->k % 32 || w->n % 32) return QHTP_STATUS_UNSUPPORTED;     // reference: M/K/N multiples of 32
  if (w->k > 32768) return QHTP_STATUS_UNSUPPORTED;               // int32 plane accumulators / int64 T
  if (w->schema == QHTP_SCHEMA_LPBQ) {
    if (p.weight_bits != 4) return QHTP_STATUS_UNSUPPORTED;
    if (w->lpbq_block == 0 || w->lpbq_block % 32 || w->k % w->lpbq_block || w->k <= w->lpbq_block)
      return QHTP_STATUS_UNSUPPORTED;
  }
  if (w->schema == QHTP_SCHEMA_PER_GROUP) {  // generate_qnn_matmul_python_cases.py:392-396
    if (p.weight_bits != 4 || w->dequant != QHTP_DEQUANT_F32_WEIGHT) return QHTP_STATUS_UNSUPPORTED;
    if (w->k % 64 || w->k <= 64) return QHTP_STATUS_UNSUPPORTED;
  }
  if (p.weight_bits == 16 && w->dequant != QHTP_DEQUANT_EXACT) return QHTP_STATUS_UNSUPPORTED;
  if (!(w->act_scale > 0.0) || !std::isfinite(w->act_scale) || !(w->out_scale > 0.0) ||
      !std::isfinite(w->out_scale))
    return QHTP_STATUS_INVALID_ARGUMENT;
  p.act_zp = -w->act_offset;
  p.out_zp = -w->out_offset;
  p.out_qmax = (1 << p.out_bits) - 1;
  if (p.act_zp < 0 || p.act_zp > (1 << p.act_bits) - 1) return QHTP_STATUS_INVALID_ARGUMENT;
  if (p.out_zp < 0 || p.out_zp > p.out_qmax) return QHTP_STATUS_INVALID_ARGUMENT;
  p.magic = kPlanMagic;
  p.family = w->family;
  p.schema = w->schema;
  p.dequant = w->dequant;
  p.k = w->k;
  p.n = w->n;
  p.lpbq_block = w->schema == QHTP_SCHEMA_LPBQ ? w->lpbq_block : 0;
  p.a_planes = p.act_bits == 16 ? 2 : 1;
  if (w->schema == QHTP_SCHEMA_PER_GROUP) {
    p.mode = kModeGroup;
    p.ch_per_tile = kGroupTileN;
  } else if (p.weight_bits == 16) {
    p.mode = kModeW16;
    p.ch_per_tile = 128;
  } else if (w->dequant == QHTP_DEQUANT_F32_WEIGHT) {
    p.mode = kModeF32;
    p.ch_per_tile = 128;
  } else {
    p.mode = kModeExact;
    p.ch_per_tile = 128;
  }
  p.n_tiles = (p.n + p.ch_per_tile - 1) / p.ch_per_tile;
  p.k_pad = static_cast<uint32_t>(align_up(p.k, kTileK));
  p.act_scale = w->act_scale;
  p.out_scale = w->out_scale;
  split_f64(w->act_scale, &p.act_mant, &p.act_exp2);
  split_f64(w->out_scale, &p.out_mant, &p.out_exp2);
  p.plane_bytes = align_up(static_cast<size_t>(p.n_tiles) * b_rows_for_mode(p.mode) * p.k_pad, 256);
  const size_t npad = static_cast<size_t>(p.n_tiles) * p.ch_per_tile;
  // per-group: the (tile, group) constant blocks, then the float64 bias per channel
  p.record_bytes = p.mode == kModeGroup ? group_rec_bytes(&p) + align_up(npad * sizeof(double), 256)
                                        : align_up(npad * sizeof(ChannelRecord), 256);
  // planes | records | per-channel sums (prepare scratch) | int4 code image (int4 families) |
  // 256-byte status word area
  p.prepared_bytes =
      p.plane_bytes + p.record_bytes + align_up(npad * 8 * kSumsPerChannel, 256) + int4_image_bytes(&p) + 256;
  p.prepared = nullptr;
  *plan = p;
  return QHTP_STATUS_OK;
}

size_t qhtp_matmul_prepared_bytes(const QhtpMatmulPlan* plan) { return plan_ok(plan) ? plan->prepared_bytes : 0; }

QhtpStatus qhtp_matmul_prepare(QhtpMatmulPlan* plan, const QhtpMatmulWeights* w, void* prepared, size_t bytes,
                               void* stream) {
  if (!plan_ok(plan) || w == nullptr || prepared == nullptr) return QHTP_STATUS_INVALID_ARGUMENT;
  if (bytes < plan->prepared_bytes || !aligned(prepared, 256)) return QHTP_STATUS_INVALID_ARGUMENT;
  if (w->family != plan->family || w->k != plan->k || w->n != plan->n || w->schema != plan->schema)
    return QHTP_STATUS_INVALID_ARGUMENT;
  if (w->weight == nullptr || w->weight_scale == nullptr) return QHTP_STATUS_INVALID_ARGUMENT;
  if (plan->schema == QHTP_SCHEMA_PER_GROUP ? w->bias_float == nullptr : w->bias_q == nullptr)
    return QHTP_STATUS_INVALID_ARGUMENT;
  if (plan->schema == QHTP_SCHEMA_LPBQ && w->lpbq_block_scale == nullptr) return QHTP_STATUS_INVALID_ARGUMENT;
  cudaStream_t s = as_stream(stream);
  // status word: last 256-byte area of the prepared buffer (zeroed by the prepare memset)
  int* dflag = reinterpret_cast<int*>(static_cast<uint8_t*>(prepared) + plan->prepared_bytes - 256);
  cudaError_t e = launch_prepare(plan, w, prepared, dflag, s);
  if (e == cudaSuccess) e = launch_prepare_int4(plan, w, prepared, dflag, s);
  if (e != cudaSuccess) return QHTP_STATUS_RUNTIME_ERROR;
  // [0] bad-scale flag, [1] widest per-channel lo-plane residual window, [2] LPBQ factor outside [1, 16],
  // [4..5] sum of the channels' windows (uint64)
  int h[6] = {0, 0, 0, 0, 0, 0};
  e = cudaMemcpyAsync(h, dflag, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return QHTP_STATUS_RUNTIME_ERROR;
  if (h[0] != 0) return QHTP_STATUS_INVALID_ARGUMENT;  // a scale was zero, negative, subnormal or not finite
  plan->flags &= kPlanForceInt4Stream | kPlanForceLoResidual;  // the caller's overrides survive a re-prepare
  if (plan->mode == kModeF32 && plan->a_planes == 2 && h[1] > 0 && h[1] <= kLoWinMax) {
    plan->flags |= kPlanLoResidualByBound;
    const uint64_t win_sum = static_cast<uint64_t>(static_cast<uint32_t>(h[4])) |
                             (static_cast<uint64_t>(static_cast<uint32_t>(h[5])) << 32);
    if (win_sum <= kLoWinMeanMax * plan->n) plan->flags |= kPlanLoResidualPays;
  }
  if (int4_stream_layout(plan) && h[2] == 0) plan->flags |= kPlanInt4Stream;
  plan->prepared = prepared;
  return QHTP_STATUS_OK;
}

size_t qhtp_matmul_workspace_bytes(const QhtpMatmulPlan* plan, uint32_t m) {
  if (!plan_ok(plan)) return 0;
  return err_offset(plan, m) + 256;
}

QhtpStatus qhtp_matmul_run(const QhtpMatmulPlan* plan, const void* act, uint32_t m, void* out, void* workspace,
                           size_t workspace_bytes, void* stream) {
  return qhtp_matmul_run_ctas(plan, act, m, out, workspace, workspace_bytes, 0, stream);
}

QhtpStatus qhtp_matmul_run_ctas(const QhtpMatmulPlan* plan, const void* act, uint32_t m, void* out, void* workspace,
                                size_t workspace_bytes, uint32_t max_ctas, void* stream) {
  if (!plan_ok(plan) || plan->prepared == nullptr) return QHTP_STATUS_INVALID_ARGUMENT;
  if (act == nullptr || out == nullptr || workspace == nullptr || m == 0) return QHTP_STATUS_INVALID_ARGUMENT;
  if (!aligned(act, 16) || !aligned(out, 16) || !aligned(workspace, 256)) return QHTP_STATUS_INVALID_ARGUMENT;
  if (workspace_bytes < qhtp_matmul_workspace_bytes(plan, m)) return QHTP_STATUS_INVALID_ARGUMENT;
  if (m > (1u << 24)) return QHTP_STATUS_UNSUPPORTED;
  GemmLaunch g;
  g.plan = plan;
  g.act = act;
  g.m = m;
  g.out = out;
  g.planes = static_cast<uint8_t*>(workspace);
  g.err = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + err_offset(plan, m));
  g.dec4 = dec4_area(plan, m, static_cast<uint8_t*>(workspace));
  g.stream = as_stream(stream);
  g.max_ctas = max_ctas;
  return from_cuda(launch_gemm(g));
}

QhtpStatus qhtp_matmul_run_host(const QhtpMatmulPlan* plan, const void* act_host, uint32_t m, void* out_host,
                                void* act_dev, void* out_dev, void* workspace, size_t workspace_bytes,
                                uint32_t chunk_rows, uint32_t* chunk_rows_used, void* stream) {
  if (!plan_ok(plan) || plan->prepared == nullptr) return QHTP_STATUS_INVALID_ARGUMENT;
  if (act_host == nullptr || out_host == nullptr || act_dev == nullptr || out_dev == nullptr || workspace == nullptr ||
      m == 0)
    return QHTP_STATUS_INVALID_ARGUMENT;
  if (!aligned(act_dev, 16) || !aligned(out_dev, 16) || !aligned(workspace, 256)) return QHTP_STATUS_INVALID_ARGUMENT;
  if (m > (1u << 24)) return QHTP_STATUS_UNSUPPORTED;
  const uint32_t rows = host_chunk_rows(m, chunk_rows);
  if (workspace_bytes < qhtp_matmul_workspace_bytes(plan, rows)) {
    set_last_message("qhtp_matmul_run_host: workspace smaller than qhtp_matmul_workspace_bytes(plan, chunk rows)");
    return QHTP_STATUS_INVALID_ARGUMENT;
  }
  if (chunk_rows_used) *chunk_rows_used = rows;
  HostPipe* hp = host_pipe();
  if (hp == nullptr) return QHTP_STATUS_RUNTIME_ERROR;
  std::lock_guard<std::mutex> lock(hp->mu);  // the pipe's streams and events serve one call at a time
  const size_t act_row = static_cast<size_t>(plan->k) * (plan->act_bits / 8);
  const size_t out_row = static_cast<size_t>(plan->n) * (plan->out_bits / 8);
  cudaStream_t s = as_stream(stream);
  // the copies start after prior work on `stream` (which may still use the staging buffers)
  cudaError_t e = cudaEventRecord(hp->start, s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(hp->in, hp->start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(hp->out, hp->start, 0);
  GemmLaunch g;
  g.plan = plan;
  g.planes = static_cast<uint8_t*>(workspace);
  g.err = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + err_offset(plan, rows));
  g.stream = s;
  const uint32_t chunks = (m + rows - 1) / rows;
  for (uint32_t c = 0; c < chunks && e == cudaSuccess; ++c) {
    const uint32_t r0 = c * rows, rc = m - r0 < rows ? m - r0 : rows;
    uint8_t* a_d = static_cast<uint8_t*>(act_dev) + r0 * act_row;
    uint8_t* o_d = static_cast<uint8_t*>(out_dev) + r0 * out_row;
    // chunk c: host -> device (copy stream 1), GEMM (the caller's stream), device -> host (stream 2)
    e = cudaMemcpyAsync(a_d, static_cast<const uint8_t*>(act_host) + r0 * act_row, rc * act_row,
                        cudaMemcpyHostToDevice, hp->in);
    if (e == cudaSuccess) e = cudaEventRecord(hp->copied[c], hp->in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, hp->copied[c], 0);
    if (e == cudaSuccess) {
      g.act = a_d;
      g.m = rc;
      g.out = o_d;
      g.dec4 = dec4_area(plan, rc, static_cast<uint8_t*>(workspace));
      e = launch_gemm(g);
    }
    if (e == cudaSuccess) e = cudaEventRecord(hp->computed[c], s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(hp->out, hp->computed[c], 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(static_cast<uint8_t*>(out_host) + r0 * out_row, o_d, rc * out_row, cudaMemcpyDeviceToHost,
                          hp->out);
  }
  // later work on `stream` follows the last copy back
  if (e == cudaSuccess) e = cudaEventRecord(hp->done, hp->out);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, hp->done, 0);
  return from_cuda(e);
}

QhtpStatus qhtp_matmul_check(const QhtpMatmulPlan* plan, void* workspace, uint32_t m, int* device_code,
                             void* stream) {
  if (!plan_ok(plan) || workspace == nullptr) return QHTP_STATUS_INVALID_ARGUMENT;
  cudaStream_t s = as_stream(stream);
  int* err = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + err_offset(plan, m));
  int h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(err, 0, sizeof(int), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return QHTP_STATUS_RUNTIME_ERROR;
  if (device_code) *device_code = h;
  return h == 0 ? QHTP_STATUS_OK : QHTP_STATUS_RUNTIME_ERROR;
}

QhtpStatus qhtp_selftest_wait_timeout(int* err_word, int* warps_gave_up, uint64_t limit_cycles, void* stream) {
  if (err_word == nullptr || warps_gave_up == nullptr || limit_cycles == 0 || limit_cycles > (1ull << 32))
    return QHTP_STATUS_INVALID_ARGUMENT;
  if (!aligned(err_word, 4) || !aligned(warps_gave_up, 4)) return QHTP_STATUS_INVALID_ARGUMENT;
  return from_cuda(launch_wait_timeout(err_word, static_cast<long long>(limit_cycles), warps_gave_up,
                                       as_stream(stream)));
}

QhtpStatus qhtp_matmul_read_records(const QhtpMatmulPlan* plan, void* host_dst, size_t bytes, void* stream) {
  if (!plan_ok(plan) || plan->prepared == nullptr || host_dst == nullptr) return QHTP_STATUS_INVALID_ARGUMENT;
  if (plan->mode == kModeGroup) return QHTP_STATUS_UNSUPPORTED;  // per-(channel, group) constants, no record
  const size_t need = static_cast<size_t>(plan->n_tiles) * plan->ch_per_tile * sizeof(ChannelRecord);
  if (bytes < need) return QHTP_STATUS_INVALID_ARGUMENT;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemcpyAsync(host_dst, static_cast<const uint8_t*>(plan->prepared) + plan->plane_bytes, need,
                                  cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return from_cuda(e);
}

QhtpStatus qhtp_lpbq_expand_i8(const uint8_t* w4_kpair, const uint8_t* block_scale, uint32_t k, uint32_t n,
                               uint32_t block, int8_t* out_nk, void* stream) {
  if (w4_kpair == nullptr || block_scale == nullptr || out_nk == nullptr || k == 0 || n == 0 || block == 0)
    return QHTP_STATUS_INVALID_ARGUMENT;
  if (k % 2 || k % block) return QHTP_STATUS_UNSUPPORTED;
  return from_cuda(launch_lpbq_expand(w4_kpair, block_scale, k, n, block, out_nk, as_stream(stream)));
}

size_t qhtp_prepared_run_scratch_bytes(const QhtpMatmulPlan* plan, uint32_t m, uint32_t chain) {
  if (!plan_ok(plan)) return 0;
  const size_t ws = qhtp_matmul_workspace_bytes(plan, m);
  if (chain <= 1) return ws;
  const size_t inter = align_up(static_cast<size_t>(m) * plan->n * (plan->out_bits / 8), 256);
  return ws + inter;
}

}  // extern "C"

namespace {

QhtpStatus run_prepared(const QhtpPreparedRun* run, uint32_t family) {
  if (run == nullptr || !plan_ok(run->plan)) return QHTP_STATUS_INVALID_ARGUMENT;
  const QhtpMatmulPlan* pl = run->plan;
  if (pl->family != family) return QHTP_STATUS_INVALID_ARGUMENT;
  if (run->m == 0 || run->k == 0 || run->n == 0 || run->chain == 0) return QHTP_STATUS_INVALID_ARGUMENT;
  if (run->k != pl->k || run->n != pl->n) return QHTP_STATUS_INVALID_ARGUMENT;
  if (run->activation.data == nullptr || run->output.data == nullptr || run->scratch.data == nullptr)
    return QHTP_STATUS_INVALID_ARGUMENT;
  const size_t act_bytes = static_cast<size_t>(run->m) * run->k * (pl->act_bits / 8);
  const size_t out_bytes = static_cast<size_t>(run->m) * run->n * (pl->out_bits / 8);
  if (run->activation.bytes < act_bytes || run->output.bytes < out_bytes) return QHTP_STATUS_INVALID_ARGUMENT;
  if (run->scratch.bytes < qhtp_prepared_run_scratch_bytes(pl, run->m, run->chain)) return QHTP_STATUS_INVALID_ARGUMENT;
  if (run->chain > 1 && (pl->k != pl->n || pl->act_bits != pl->out_bits)) return QHTP_STATUS_UNSUPPORTED;
  const size_t ws = qhtp_matmul_workspace_bytes(pl, run->m);
  if (run->chain > 1 && run->m <= (1u << 24) && chain_fusable(pl)) {
    // K == N <= 256: one kernel for the whole chain, intermediates kept in shared memory
    if (!aligned(run->activation.data, 16) || !aligned(run->output.data, 16) || !aligned(run->scratch.data, 256))
      return QHTP_STATUS_INVALID_ARGUMENT;
    GemmLaunch g;
    g.plan = pl;
    g.act = run->activation.data;
    g.m = run->m;
    g.out = run->output.data;
    g.planes = static_cast<uint8_t*>(run->scratch.data);
    g.err = reinterpret_cast<int*>(static_cast<uint8_t*>(run->scratch.data) + err_offset(pl, run->m));
    g.stream = as_stream(run->stream);
    return from_cuda(launch_chain(g, run->chain));
  }
  uint8_t* inter = static_cast<uint8_t*>(run->scratch.data) + ws;
  // ping-pong so that the last pass writes `output`
  const void* src = run->activation.data;
  for (uint32_t i = 0; i < run->chain; ++i) {
    const uint32_t left = run->chain - 1 - i;  // passes after this one
    void* dst = (left % 2 == 0) ? run->output.data : static_cast<void*>(inter);
    QhtpStatus st = qhtp_matmul_run(pl, src, run->m, dst, run->scratch.data, ws, run->stream);
    if (st != QHTP_STATUS_OK) return st;
    src = dst;
  }
  return QHTP_STATUS_OK;
}

}  // namespace

extern "C" {

QhtpStatus qhtp_u8i8_run_prepared(const QhtpPreparedRun* run) { return run_prepared(run, QHTP_FAMILY_U8I8); }
QhtpStatus qhtp_w4a8_run_prepared(const QhtpPreparedRun* run) { return run_prepared(run, QHTP_FAMILY_W4A8); }
QhtpStatus qhtp_w8a16_run_prepared(const QhtpPreparedRun* run) { return run_prepared(run, QHTP_FAMILY_W8A16); }
QhtpStatus qhtp_w4a16_run_prepared(const QhtpPreparedRun* run) { return run_prepared(run, QHTP_FAMILY_W4A16); }
QhtpStatus qhtp_w16a16_run_prepared(const QhtpPreparedRun* run) { return run_prepared(run, QHTP_FAMILY_W16A16); }

QhtpStatus qhtp_gdn_inverse_bf16(const void* A, float* T, int64_t n_chunks, int32_t C, void* stream) {
  if (A == nullptr || T == nullptr || n_chunks <= 0) return QHTP_STATUS_INVALID_ARGUMENT;
  if (C != 32 && C != 64 && C != 128 && C != 256) return QHTP_STATUS_UNSUPPORTED;
  if (!aligned(A, 16) || !aligned(T, 16)) return QHTP_STATUS_INVALID_ARGUMENT;
  return from_cuda(launch_gdn_bf16(A, T, n_chunks, C, as_stream(stream)));
}

QhtpStatus qhtp_gdn_chunk_inverse(const void* k, const float* beta, const float* g, float* T, int64_t n_chunks,
                                  int32_t C, int32_t dk, void* stream) {
  if (k == nullptr || beta == nullptr || g == nullptr || T == nullptr || n_chunks <= 0)
    return QHTP_STATUS_INVALID_ARGUMENT;
  if (C != 256 || dk != 128) return QHTP_STATUS_UNSUPPORTED;
  if (!gdn256f_supported(k, beta, g, T, n_chunks)) return QHTP_STATUS_INVALID_ARGUMENT;
  return from_cuda(launch_gdn256_fused(k, beta, g, T, n_chunks, as_stream(stream)));
}

QhtpStatus qhtp_gdn_solve_u16(const uint16_t* A, int64_t n_chunks, int32_t C, int32_t zpA, float sA, int32_t zpT,
                              float sT, uint16_t* T, void* stream) {
  if (A == nullptr || T == nullptr || n_chunks <= 0) return QHTP_STATUS_INVALID_ARGUMENT;
  if (C != 32 && C != 64 && C != 128 && C != 256) return QHTP_STATUS_UNSUPPORTED;
  if (!(sA > 0.0f) || !(sT > 0.0f) || !std::isfinite(sA) || !std::isfinite(sT)) return QHTP_STATUS_INVALID_ARGUMENT;
  if (zpA < 0 || zpA > 65535 || zpT < 0 || zpT > 65535) return QHTP_STATUS_INVALID_ARGUMENT;
  if (!aligned(A, 16) || !aligned(T, 16)) return QHTP_STATUS_INVALID_ARGUMENT;
  return from_cuda(launch_gdn_u16(A, n_chunks, C, zpA, sA, zpT, sT, T, as_stream(stream)));
}

}  // extern "C"
