// Per-step device status of the runtimes (MSAT control step, decoder-stack prefill), the
// run-time wait bound and a self-test of the bounded wait.
//
// Every bounded wait of the library records its error code in the device word g_rldx_err.  A
// runtime brackets its launch list with two one-thread kernels: the first moves a code left by
// earlier work into the handle's status slot 0 and clears the word, so the step starts from a
// clean word (a set word makes every wait of the step give up at its first slow poll); the
// last moves a code raised during the step into slot 1.  The slots are mapped pinned host
// memory: after the step's completion event the host reads them with no copy.  This replaces
// the reference's fall-back-on-failure of its compiled dispatcher
// (rldx/inference/serve_optimization.py:432-516) with an error the caller sees on the step
// that failed.
#include "host_util.h"

namespace rldx {

__global__ void status_take_kernel(unsigned int* slot) {
  *reinterpret_cast<volatile unsigned int*>(slot) = atomicExch(&g_rldx_err, 0u);
}

cudaError_t launch_status_take(unsigned int* slot_dev, cudaStream_t stream) {
  status_take_kernel<<<1, 1, 0, stream>>>(slot_dev);
  return cudaGetLastError();
}

// One warp waits on a shared-memory barrier that nothing ever arrives on: the wait runs out
// after `limit_cycles`, records kErrSelftestTimeout and the kernel returns.
__global__ void wait_selftest_kernel(long long limit_cycles) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) mbar_wait(&bar, 0u, kErrSelftestTimeout, limit_cycles);
  __syncwarp();
}

bool StepStatus::init() {
  void* p = nullptr;
  if (cudaHostAlloc(&p, 2 * sizeof(unsigned int), cudaHostAllocMapped) != cudaSuccess) return false;
  host = static_cast<unsigned int*>(p);
  host[0] = host[1] = 0u;
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, p, 0) != cudaSuccess) return false;
  dev = static_cast<unsigned int*>(d);
  return cudaEventCreateWithFlags(&done, cudaEventDisableTiming) == cudaSuccess;
}

void StepStatus::release() {
  if (done) cudaEventDestroy(done);
  if (host) cudaFreeHost(host);
  done = nullptr;
  host = dev = nullptr;
}

// 0: no error; else the first code (slot 0: left by earlier work, slot 1: raised in the step).
// wait = 0 only looks when the last step has completed; both slots are cleared once read.
int StepStatus::read(bool wait, unsigned int* code, unsigned int* which) {
  *code = 0u;
  if (which) *which = 0u;
  if (!host || !done) return RLDX_OK;
  cudaError_t e = wait ? cudaEventSynchronize(done) : cudaEventQuery(done);
  if (e == cudaErrorNotReady) return RLDX_OK;
  if (e != cudaSuccess) return cuda_fail(e, "step status event");
  volatile unsigned int* h = host;
  const unsigned int before = h[0], during = h[1];
  h[0] = h[1] = 0u;
  if (during) {
    *code = during;
    if (which) *which = 1u;
  } else if (before) {
    *code = before;
  }
  return RLDX_OK;
}

}  // namespace rldx

using namespace rldx;

extern "C" {

int rldx_set_wait_limit(int64_t cycles) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (cycles < 1000 || cycles > 100000000000ll)
    return set_error(RLDX_ERR_ARG, "wait limit must be in [1e3, 1e11] SM cycles");
  const long long v = cycles;
  cudaError_t e = cudaMemcpyToSymbol(g_rldx_wait_limit, &v, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "set wait limit");
  return RLDX_OK;
}

int rldx_get_wait_limit(int64_t* cycles) {
  if (!cycles) return set_error(RLDX_ERR_ARG, "null cycles");
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  long long v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_rldx_wait_limit, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "get wait limit");
  *cycles = v;
  return RLDX_OK;
}

int rldx_wait_selftest(int64_t limit_cycles, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (limit_cycles < 1000 || limit_cycles > 4000000000ll)
    return set_error(RLDX_ERR_ARG, "self-test limit must be in [1e3, 4e9] SM cycles");
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_cycles);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "wait self-test launch");
  return RLDX_OK;
}

}  // extern "C"
