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

// Video-token compression of B sequences [B, T, D] -> [B, T2, D], T2 = T - (end - begin) + 1:
// the rows [begin, end) become one row, their mean, at `begin`; the rows before and after are
// copied in order.  Blocks [0, mean_blocks) each own 64 columns of one sequence's mean row:
// 8 column groups x 32 row lanes sum the dropped rows in fp32 (lane l takes rows begin + l,
// begin + l + 32, ...), the lane partials are added in lane order through shared memory (a fixed
// order, so the result does not depend on scheduling), the sum is rounded to bf16, divided by the
// row count and rounded again (the module's bf16 sum followed by a bf16 true division).  The
// other blocks copy the kept rows, 16 bytes per thread.
__global__ void __launch_bounds__(256) compress_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                            __nv_bfloat16* __restrict__ y, int B, int T, int D,
                                                            int begin, int end, int mean_blocks) {
  const int T2 = T - (end - begin) + 1;
  if (static_cast<int>(blockIdx.x) < mean_blocks) {
    __shared__ float part[32][65];
    const int per_seq = D / 64;
    const int b = blockIdx.x / per_seq, c0 = (blockIdx.x % per_seq) * 64;
    const int grp = threadIdx.x & 7, lane = threadIdx.x >> 3;
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    const __nv_bfloat16* base = x + static_cast<long long>(b) * T * D + c0 + grp * 8;
#pragma unroll 4
    for (int r = begin + lane; r < end; r += 32) {
      const uint4 v = *reinterpret_cast<const uint4*>(base + static_cast<long long>(r) * D);
      const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(hv[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) part[lane][grp * 8 + k] = acc[k];
    __syncthreads();
    if (threadIdx.x < 64) {
      float sum = 0.f;
      for (int l = 0; l < 32; ++l) sum += part[l][threadIdx.x];
      const float rounded = __bfloat162float(__float2bfloat16_rn(sum));
      const float mean = __fdiv_rn(rounded, static_cast<float>(end - begin));
      y[(static_cast<long long>(b) * T2 + begin) * D + c0 + threadIdx.x] = __float2bfloat16_rn(mean);
    }
    return;
  }
  const int kept = T2 - 1;
  if (kept <= 0) return;
  const int nv = D / 8;
  const long long total = static_cast<long long>(B) * kept * nv;
  const long long stride = static_cast<long long>(gridDim.x - mean_blocks) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x - mean_blocks) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int v = static_cast<int>(i % nv);
    const long long br = i / nv;
    const int j = static_cast<int>(br % kept);
    const int b = static_cast<int>(br / kept);
    const int r2 = j < begin ? j : j + 1;                  // output row (the mean row is skipped)
    const int r = r2 < begin ? r2 : r2 - begin - 1 + end;  // source row
    reinterpret_cast<uint4*>(y + (static_cast<long long>(b) * T2 + r2) * D)[v] =
        reinterpret_cast<const uint4*>(x + (static_cast<long long>(b) * T + r) * D)[v];
  }
}

cudaError_t launch_compress_rows(const __nv_bfloat16* x, __nv_bfloat16* y, int B, int T, int D, int begin, int end,
                                 cudaStream_t stream) {
  if (B <= 0 || D % 64 || begin < 0 || end <= begin || end > T) return cudaErrorInvalidValue;
  const long long mean_blocks = static_cast<long long>(B) * (D / 64);
  const long long kept = static_cast<long long>(B) * (T - (end - begin)) * (D / 8);
  long long copy_blocks = (kept + 255) / 256;
  if (copy_blocks > 4 * 148) copy_blocks = 4 * 148;
  if (mean_blocks + copy_blocks > (1LL << 31) - 1) return cudaErrorInvalidValue;
  compress_rows_kernel<<<static_cast<unsigned>(mean_blocks + copy_blocks), 256, 0, stream>>>(
      x, y, B, T, D, begin, end, static_cast<int>(mean_blocks));
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
