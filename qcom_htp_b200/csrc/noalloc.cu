// qhtp_matmul_run_noalloc: the quantized MatMul for callers that cannot allocate device memory.
//
// Some callers are not allowed to call cudaMalloc when they run the op: an inference-runtime
// plugin invoked from the runtime's execute callback (the runtime owns and pre-plans every device
// buffer -- the position the QNN/QHPI custom ops hold in the reference, where the op never
// allocates), or code on a latency-critical thread where an allocation's implicit synchronization
// and unpredictable latency are not acceptable.  qhtp_matmul_run needs a caller-provided workspace
// (the u16 activation byte planes and a device error word); this entry point uses a fixed scratch
// area that lives in the library instead:
//
//   * g_noalloc_scratch is a file-scope device array of QHTP_NOALLOC_SCRATCH_BYTES (8 MiB).  Every
//     GPU that loads libqhtp holds it until the process exits.
//   * Host code cannot pass g_noalloc_scratch to a kernel (in host code the name is a host-side
//     stand-in, not a device address).  The first call on each device looks up the device address
//     with cudaGetSymbolAddress while that device is current and caches it; make that first call
//     before any stream capture begins.
//   * Every call shares the one area and it keeps the previous call's contents: the error word is
//     cleared at the start of each call.  Calls whose kernels overlap on the GPU (different streams,
//     or several host threads) race on the area; serialize them.
//   * Sizes whose workspace exceeds the area are rejected with QHTP_STATUS_INVALID_ARGUMENT and a
//     message from qhtp_last_error_string.  Nothing here calls cudaMalloc, cudaFree or any
//     allocating library routine.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "internal.h"

namespace {

constexpr size_t kScratchBytes = QHTP_NOALLOC_SCRATCH_BYTES;
static_assert(kScratchBytes % 256 == 0, "scratch size");

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint8_t* g_dev_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
cudaError_t scratch_on_current_device(uint8_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_dev_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_dev_ptr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_dev_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" QhtpStatus qhtp_matmul_run_noalloc(const QhtpMatmulPlan* plan, const void* act, uint32_t m, void* out,
                                              void* stream) {
  if (plan == nullptr || plan->magic != qhtp::kPlanMagic || plan->prepared == nullptr)
    return QHTP_STATUS_INVALID_ARGUMENT;
  if (act == nullptr || out == nullptr || m == 0) return QHTP_STATUS_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(act) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return QHTP_STATUS_INVALID_ARGUMENT;
  if (m > (1u << 24)) return QHTP_STATUS_UNSUPPORTED;  // the row limit of qhtp_matmul_run
  const size_t need = qhtp_matmul_workspace_bytes(plan, m);  // run workspace, error word last
  if (need == 0 || need > kScratchBytes) {
    qhtp::set_last_message(
        "qhtp_matmul_run_noalloc: qhtp_matmul_workspace_bytes(plan, M) exceeds the library's fixed 8 MiB "
        "scratch; use qhtp_matmul_run with a "
        "caller workspace");
    return QHTP_STATUS_INVALID_ARGUMENT;
  }
  uint8_t* scratch = nullptr;
  cudaError_t e = scratch_on_current_device(&scratch);
  if (e != cudaSuccess) return qhtp::status_from_cuda(e);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* err = reinterpret_cast<int*>(scratch + need - 256);
  e = cudaMemsetAsync(err, 0, sizeof(int), s);  // the area keeps the last call's contents
  if (e != cudaSuccess) return qhtp::status_from_cuda(e);
  qhtp::GemmLaunch g;
  g.plan = plan;
  g.act = act;
  g.m = m;
  g.out = out;
  g.planes = scratch;
  g.err = err;
  g.dec4 = qhtp::dec4_area(plan, m, scratch);
  g.stream = s;
  return qhtp::status_from_cuda(qhtp::launch_gemm(g));
}

extern "C" QhtpStatus qhtp_matmul_noalloc_check(const QhtpMatmulPlan* plan, uint32_t m, int* device_code,
                                               void* stream) {
  if (plan == nullptr || plan->magic != qhtp::kPlanMagic || m == 0 || m > (1u << 24))
    return QHTP_STATUS_INVALID_ARGUMENT;
  const size_t need = qhtp_matmul_workspace_bytes(plan, m);
  if (need == 0 || need > kScratchBytes) return QHTP_STATUS_INVALID_ARGUMENT;
  uint8_t* scratch = nullptr;
  cudaError_t e = scratch_on_current_device(&scratch);
  if (e != cudaSuccess) return qhtp::status_from_cuda(e);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* err = reinterpret_cast<int*>(scratch + need - 256);  // where an M-row call keeps its error word
  int h = 0;
  e = cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(err, 0, sizeof(int), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return qhtp::status_from_cuda(e);
  if (device_code) *device_code = h;
  return h == 0 ? QHTP_STATUS_OK : QHTP_STATUS_RUNTIME_ERROR;
}
