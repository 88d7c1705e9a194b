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

// Deepstack injection (modeling_qwen3_vl.py:1102-1113: hidden[mask] = hidden[mask] + embeds):
// one thread per 8 columns of a listed row; bf16 + bf16 rounds once (packed, exactly rounded).
__global__ void rows_add_kernel(__nv_bfloat16* __restrict__ x, const int* __restrict__ rows, int nrows,
                                const __nv_bfloat16* __restrict__ f, int B, int T, int D) {
  const int nv = D / 8;
  const long long total = static_cast<long long>(B) * nrows * nv;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int v = static_cast<int>(i % nv);
    const long long bj = i / nv;  // b * nrows + j
    const int j = static_cast<int>(bj % nrows);
    const int b = static_cast<int>(bj / nrows);
    uint4* xp = reinterpret_cast<uint4*>(x + (static_cast<long long>(b) * T + rows[j]) * D) + v;
    const uint4 fv = reinterpret_cast<const uint4*>(f + bj * D)[v];
    uint4 xv = *xp;
    __nv_bfloat162* xh = reinterpret_cast<__nv_bfloat162*>(&xv);
    const __nv_bfloat162* fh = reinterpret_cast<const __nv_bfloat162*>(&fv);
#pragma unroll
    for (int k = 0; k < 4; ++k) xh[k] = __hadd2_rn(xh[k], fh[k]);
    *xp = xv;
  }
}

cudaError_t launch_rows_add(__nv_bfloat16* x, const int* rows, int nrows, const __nv_bfloat16* f, int B, int T,
                            int D, cudaStream_t stream) {
  if (nrows <= 0 || B <= 0) return cudaSuccess;
  if (D % 8) return cudaErrorInvalidValue;
  const long long total = static_cast<long long>(B) * nrows * (D / 8);
  long long grid = (total + 255) / 256;
  if (grid > 4096) grid = 4096;
  rows_add_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(x, rows, nrows, f, B, T, D);
  return cudaGetLastError();
}

// Key mask of the joint sequence [VL | SA | P] of every observation: VL keys from the backbone
// mask, action / state / time keys visible, physics keys from the observation's physics mask.
__global__ void key_mask_kernel(uint8_t* __restrict__ kmask, const uint8_t* __restrict__ vl,
                                const uint8_t* __restrict__ p, int B, int L, int nvl, int nsa) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < B * L; i += gridDim.x * blockDim.x) {
    const int b = i / L, t = i - b * L;
    const uint8_t m = t < nvl ? vl[b * nvl + t] : (t < nvl + nsa ? 1 : p[b]);
    kmask[i] = m != 0 ? 1 : 0;
  }
}

cudaError_t launch_key_mask(uint8_t* kmask, const uint8_t* vl, const uint8_t* p, int B, int L, int nvl,
                            int nsa, cudaStream_t stream) {
  const int n = B * L;
  key_mask_kernel<<<(n + 255) / 256 < 148 ? (n + 255) / 256 : 148, 256, 0, stream>>>(kmask, vl, p, B, L, nvl, nsa);
  return cudaGetLastError();
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
