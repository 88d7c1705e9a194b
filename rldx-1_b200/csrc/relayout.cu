// Bind-time weight re-layout kernels (run once per handle, never on the control-step path).
#include "kernels.cuh"

namespace rldx {

__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ src, long long ld_src,
                                   __nv_bfloat16* __restrict__ dst, long long ld_dst,
                                   const int* __restrict__ idx, int rows, int cols) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const __nv_bfloat16* s = src + static_cast<long long>(idx[r]) * ld_src;
  __nv_bfloat16* d = dst + static_cast<long long>(r) * ld_dst;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) d[c] = s[c];
}

cudaError_t launch_gather_rows(const __nv_bfloat16* src, long long ld_src, __nv_bfloat16* dst,
                               long long ld_dst, const int* idx, int rows, int cols,
                               cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  gather_rows_kernel<<<rows, 256, 0, stream>>>(src, ld_src, dst, ld_dst, idx, rows, cols);
  return cudaGetLastError();
}

// dst[c][n][k] = src[c][k][n] for k < K, 0 for K <= k < Kp; 32x32 tiles through shared memory.
__global__ void transpose_cat_kernel(const __nv_bfloat16* __restrict__ src,
                                     __nv_bfloat16* __restrict__ dst, int K, int N, int Kp) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int c = blockIdx.z;
  const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  const __nv_bfloat16* s = src + static_cast<long long>(c) * K * N;
  __nv_bfloat16* d = dst + static_cast<long long>(c) * N * Kp;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int k = k0 + i, n = n0 + threadIdx.x;
    tile[i][threadIdx.x] = (k < K && n < N) ? s[static_cast<long long>(k) * N + n]
                                            : __float2bfloat16_rn(0.0f);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int n = n0 + i, k = k0 + threadIdx.x;
    if (n < N && k < Kp) d[static_cast<long long>(n) * Kp + k] = tile[threadIdx.x][i];
  }
}

cudaError_t launch_transpose_cat(const __nv_bfloat16* src, __nv_bfloat16* dst, int cats, int K,
                                 int N, int Kp, cudaStream_t stream) {
  dim3 grid((N + 31) / 32, (Kp + 31) / 32, cats);
  dim3 block(32, 8, 1);
  transpose_cat_kernel<<<grid, block, 0, stream>>>(src, dst, K, N, Kp);
  return cudaGetLastError();
}

__global__ void elementwise_kernel(const __nv_bfloat16* __restrict__ x,
                                   __nv_bfloat16* __restrict__ y, long long n, int mode) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float v = __bfloat162float(x[i]);
    const float r = (mode == 0) ? v / (1.0f + expf(-v)) : 1.0f + v;
    y[i] = __float2bfloat16_rn(r);
  }
}

cudaError_t launch_elementwise(const __nv_bfloat16* x, __nv_bfloat16* y, long long n, int mode,
                               cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  long long grid = (n + 255) / 256;
  if (grid > 4096) grid = 4096;
  elementwise_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(x, y, n, mode);
  return cudaGetLastError();
}

}  // namespace rldx
