// rldx_gemm_static_ws: the K-split grouped GEMM of rldx_gemm_ws, with its workspace in a
// file-scope device array of this library instead of memory the caller allocates.
//
// Who needs it: callers that cannot call cudaMalloc when they run a GEMM.  Typical cases are a
// serving loop whose request path must not touch the CUDA allocator (cudaMalloc / cudaFree
// synchronise the device and stall every stream), and foreign hosts that bind the C ABI
// without owning any CUDA allocator to hand out a workspace.  This entry point makes no
// cudaMalloc, cudaFree or other allocating call; the caller still passes inputs and outputs.
//
// Limits and contract:
//   * The scratch holds kStaticScratchBytes (8 MiB) and every GPU that loads the library keeps
//     it until the process exits.  A launch whose K-split plan needs more workspace (see
//     rldx_gemm_workspace_size) is rejected with RLDX_ERR_UNSUPPORTED and nothing is launched
//     (rldx_gemm_ws, given too small a workspace, runs such a launch unsplit instead).
//   * Host code cannot use the array's name as a device address.  The first call on each
//     device, with that device current, looks the address up with cudaGetSymbolAddress and
//     keeps it for the process (a failed look-up is not kept: the next call tries again); make
//     that first call before any stream capture.  The address does not survive a
//     cudaDeviceReset of that device.
//   * Every call first clears the per-tile arrival counters at the head of the scratch (one
//     cudaMemsetAsync of a few KB on `stream`), so a call never depends on how an earlier one
//     ended; the fp32 partial tiles after them keep the last call's contents and need no
//     clearing.
//   * One scratch per device for the whole process: calls that overlap on the GPU (different
//     streams, or unordered host threads) race on it.  Keep them ordered on one stream.
#include <mutex>

#include "host_util.h"

namespace rldx {

constexpr size_t kStaticScratchBytes = size_t{8} << 20;
static __device__ __align__(256) unsigned char g_gemm_scratch[kStaticScratchBytes];

namespace {
constexpr int kScratchDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kScratchDevices];

// Device address of the scratch on device `dev` (current), looked up once per device.
cudaError_t scratch_address(int dev, void** out) {
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gemm_scratch);
    if (e != cudaSuccess) return e;  // not cached: the next call looks again
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}
}  // namespace

}  // namespace rldx

using namespace rldx;

extern "C" int rldx_gemm_static_ws(const rldx_gemm_desc* problems, int nproblems, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!problems) return set_error(RLDX_ERR_ARG, "gemm_static_ws: null problems");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kScratchDevices) return set_error(RLDX_ERR_UNSUPPORTED, "device index");
  void* scratch = nullptr;
  e = scratch_address(dev, &scratch);
  if (e != cudaSuccess) return cuda_fail(e, "static scratch address");

  static thread_local GemmParams params;
  std::string err;
  size_t need = 0;
  if (!build_gemm_params(problems, nproblems, nullptr, 0, &params, &need, &err))
    return set_error(RLDX_ERR_ARG, err);
  if (need > kStaticScratchBytes)
    return set_error(RLDX_ERR_UNSUPPORTED,
                     "gemm_static_ws: the K-split plan needs " + std::to_string(need) +
                         " bytes of workspace, the static scratch holds " +
                         std::to_string(kStaticScratchBytes) + " (use rldx_gemm_ws)");
  if (!build_gemm_params(problems, nproblems, scratch, kStaticScratchBytes, &params, nullptr, &err))
    return set_error(RLDX_ERR_ARG, err);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bool split = false;
  for (int i = 0; i < params.nprob; ++i) split = split || params.p[i].nsplit > 1;
  if (split) {
    e = cudaMemsetAsync(params.counters, 0, kCounterBytes, st);
    if (e != cudaSuccess) return cuda_fail(e, "static scratch counters");
  }
  e = launch_gemm(params, st, false);
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  return RLDX_OK;
}
