// Host-side helpers shared by the C-ABI entry points and the MSAT runtime.
#pragma once
#include <string>

#include "../../include/rldx_b200.h"
#include "kernels.cuh"

namespace rldx {

// Records the message returned by rldx_last_error() and returns `code`.
int set_error(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

// Makes sure the current device is sm_100 and kernel attributes are set (once per device).
int ensure_device();

// 2D / 3D bf16 tensor maps with 128-byte swizzle; box inner extent is 64 elements (128 bytes).
bool make_tmap_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                  std::string* err);
bool make_tmap_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                  uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                  uint32_t b2, std::string* err);

// Validates one GEMM description and fills the shape-only fields of the device problem.
bool validate_gemm_problem(const rldx_gemm_desc& d, GemmProblem* p, std::string* err);
// Plans up to kMaxProblems problems as one persistent launch: tile widths and K splits from a
// cost model, ring sizing, tensor maps and the longest-first unit schedule.  K splits need a
// workspace (`ws`, `ws_bytes`: tile counters that start at zero, then fp32 partial tiles);
// with ws == nullptr no problem is split.  *ws_needed (optional) receives the workspace bytes
// the plan would use if a workspace were given.
bool build_gemm_params(const rldx_gemm_desc* d, int n, void* ws, size_t ws_bytes,
                       GemmParams* params, size_t* ws_needed, std::string* err);

int sm_count();

// Device status of one runtime handle (status.cu): two mapped pinned host words written by
// the one-thread kernels that open and close its launch list (slot 0: an error code left by
// earlier work, slot 1: a code raised during the step) and the completion event of its last
// step.
struct StepStatus {
  unsigned int* host = nullptr;
  unsigned int* dev = nullptr;
  cudaEvent_t done = nullptr;
  bool init();
  void release();
  // *code = the recorded code (0: none; nothing is known yet when !wait and the last step is
  // still running), *which = 1 when it was raised during the step.  Clears both slots.
  int read(bool wait, unsigned int* code, unsigned int* which);
};
// *slot = g_rldx_err, g_rldx_err = 0 (one thread)
cudaError_t launch_status_take(unsigned int* slot_dev, cudaStream_t stream);

}  // namespace rldx
