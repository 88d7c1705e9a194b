// Single translation unit of librldx_b200.so: every kernel and the C ABI.
#include "gemm.cu"
#include "attention.cu"
#include "rownorm.cu"
#include "relayout.cu"
#include "capi.cu"
#include "static_ws.cu"
#include "msat.cu"
#include "llm.cu"
