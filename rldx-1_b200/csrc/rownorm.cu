// Memory-bound row kernels: 128-bit coalesced loads/stores, one warp (or half-warp) per row,
// warp-shuffle reductions, fp32 math, bf16 rounding at the same points as the reference.
//
//   ln_rows_kernel        LayerNorm without affine (eps 1e-6), optionally followed by the
//                         AdaLN modulation y*(1+scale)+shift of the MSAT output projection.
//                         nn.LayerNorm(elementwise_affine=False): rldx/model/modules/norms.py:35-36;
//                         output projection: rldx/model/modules/action_model/msat.py:771-781.
//   copy_rows_kernel      row copies between buffers (stream initialisation inside the graph).
//   qk_rmsnorm_rope_kernel  Qwen3-style per-head RMSNorm (cast, then weight) + rotate-half RoPE,
//                         modeling_qwen3_vl.py:118-122, 357-371, 377-401 (backbone path).
//   swiglu_kernel         silu(gate) * up, rldx/model/modules/action_model/ops.py:157-161.
#include "kernels.cuh"

namespace rldx {

// One warp per row; D <= 32 * 8 * kVec.  Instantiated for rows up to 1536 (6 vectors per
// lane, few registers, so the CTAs fit next to a running GEMM and start the moment it
// completes) and up to 4096.
template <int kVec>
__global__ void __launch_bounds__(128) ln_rows_kernel(const __grid_constant__ LnParams P) {
  constexpr int kLnMaxVec = kVec;
  griddep_wait();
  griddep_launch();
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_global >= P.total_rows) return;
  int si = 0;
#pragma unroll
  for (int i = 1; i < kMaxLnSegments; ++i)
    if (i < P.nseg && warp_global >= P.seg[i].row_begin) si = i;
  const LnSegment& sg = P.seg[si];
  const int row = warp_global - sg.row_begin;
  const int D = sg.D > 0 ? sg.D : P.D;
  const int nvec = D / 8;
  const uint4* src = reinterpret_cast<const uint4*>(sg.in + static_cast<size_t>(row) * sg.ld_in);
  float x[kLnMaxVec][8];
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      const uint4 u = src[v];
      unpack_bf16x2(u.x, x[i][0], x[i][1]);
      unpack_bf16x2(u.y, x[i][2], x[i][3]);
      unpack_bf16x2(u.z, x[i][4], x[i][5]);
      unpack_bf16x2(u.w, x[i][6], x[i][7]);
#pragma unroll
      for (int e = 0; e < 8; ++e) sum += x[i][e];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / static_cast<float>(D);
  float var = 0.0f;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = x[i][e] - mean;
        var += d * d;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
  const float rstd = rsqrtf(var / static_cast<float>(D) + P.eps);
  uint4* dst = reinterpret_cast<uint4*>(sg.out + static_cast<size_t>(row) * sg.ld_out);
  const uint4* sc = reinterpret_cast<const uint4*>(sg.scale1p);
  const uint4* sh = reinterpret_cast<const uint4*>(sg.shift);
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = bf16r((x[i][e] - mean) * rstd);
      if (sc != nullptr) {
        float a[8], c[8];
        const uint4 ua = sc[v], uc = sh[v];
        unpack_bf16x2(ua.x, a[0], a[1]);
        unpack_bf16x2(ua.y, a[2], a[3]);
        unpack_bf16x2(ua.z, a[4], a[5]);
        unpack_bf16x2(ua.w, a[6], a[7]);
        unpack_bf16x2(uc.x, c[0], c[1]);
        unpack_bf16x2(uc.y, c[2], c[3]);
        unpack_bf16x2(uc.z, c[4], c[5]);
        unpack_bf16x2(uc.w, c[6], c[7]);
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = bf16r(bf16r(y[e] * a[e]) + c[e]);
      }
      uint4 u;
      u.x = pack_bf16x2(y[0], y[1]);
      u.y = pack_bf16x2(y[2], y[3]);
      u.z = pack_bf16x2(y[4], y[5]);
      u.w = pack_bf16x2(y[6], y[7]);
      dst[v] = u;
    }
  }
}

cudaError_t launch_ln(const LnParams& p, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  // 4 warps (rows) per CTA: small enough in registers to sit next to a 608-thread GEMM CTA and
  // start the moment it completes
  const int warps_per_block = 4;
  cfg.gridDim = dim3((p.total_rows + warps_per_block - 1) / warps_per_block, 1, 1);
  cfg.blockDim = dim3(32 * warps_per_block, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (p.D <= 32 * 8 * 6) return cudaLaunchKernelEx(&cfg, ln_rows_kernel<6>, p);
  return cudaLaunchKernelEx(&cfg, ln_rows_kernel<16>, p);
}

// ---------------------------------------------------------------------------------------------
// Row copies: dst[r] = src[r] for `rows` rows of `bytes` bytes (multiples of 16); a src pitch
// of 0 broadcasts one source row.  Used for stream initialisation inside the captured graph.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) copy_rows_kernel(const __grid_constant__ CopyParams P) {
  griddep_wait();
  griddep_launch();
  for (int ri = 0; ri < P.n; ++ri) {
    const CopyRegion& rg = P.r[ri];
    const int vec_per_row = rg.bytes / 16;
    const long long total = static_cast<long long>(vec_per_row) * rg.rows;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
      const long long row = i / vec_per_row;
      const long long c = i - row * vec_per_row;
      long long g = 0, rr = row;
      if (rg.group_rows > 0) {
        g = row / rg.group_rows;
        rr = row - g * rg.group_rows;
      }
      const uint4 v = reinterpret_cast<const uint4*>(rg.src + g * rg.src_group_pitch +
                                                     rr * rg.src_pitch)[c];
      reinterpret_cast<uint4*>(rg.dst + g * rg.dst_group_pitch + rr * rg.dst_pitch)[c] = v;
    }
  }
}

cudaError_t launch_copy(const CopyParams& p, int blocks, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, copy_rows_kernel, p);
}

// ---------------------------------------------------------------------------------------------
// Qwen3-style QK RMSNorm + rotate-half RoPE on [T, H, 128] (in place allowed).
//   n   = bf16(x * rsqrt(mean(x^2) + eps))          (cast to the input dtype first)
//   y   = bf16(w * n)                                (then the bf16 weight)
//   out = bf16( bf16(y * cos) + bf16(rotate_half(y) * sin) ),  cos/sin bf16 [P, 128]
// A half-warp owns one (token, head) row: lane l of the half holds elements 8l..8l+7, the
// rotate-half partner sits 8 lanes away.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) qk_rmsnorm_rope_kernel(
    const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
    const __nv_bfloat16* __restrict__ w, const int* __restrict__ pos,
    const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t,
    long long nrows, int heads, float eps) {
  const long long half_global = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 4;
  const int hl = threadIdx.x & 15;
  const bool active = half_global < nrows;
  const long long row = active ? half_global : 0;
  const uint4 u = reinterpret_cast<const uint4*>(x + row * 128)[hl];
  float v[8];
  unpack_bf16x2(u.x, v[0], v[1]);
  unpack_bf16x2(u.y, v[2], v[3]);
  unpack_bf16x2(u.z, v[4], v[5]);
  unpack_bf16x2(u.w, v[6], v[7]);
  float ss = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss * (1.0f / 128.0f) + eps);
  const uint4 uw = reinterpret_cast<const uint4*>(w)[hl];
  float wv[8];
  unpack_bf16x2(uw.x, wv[0], wv[1]);
  unpack_bf16x2(uw.y, wv[2], wv[3]);
  unpack_bf16x2(uw.z, wv[4], wv[5]);
  unpack_bf16x2(uw.w, wv[6], wv[7]);
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = bf16r(wv[e] * bf16r(v[e] * rstd));
  float pv[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) pv[e] = __shfl_xor_sync(0xffffffffu, v[e], 8);
  const long long tok = row / heads;
  const int p = pos[tok];
  const uint4 uc = reinterpret_cast<const uint4*>(cos_t + static_cast<size_t>(p) * 128)[hl];
  const uint4 us = reinterpret_cast<const uint4*>(sin_t + static_cast<size_t>(p) * 128)[hl];
  float c[8], s[8];
  unpack_bf16x2(uc.x, c[0], c[1]);
  unpack_bf16x2(uc.y, c[2], c[3]);
  unpack_bf16x2(uc.z, c[4], c[5]);
  unpack_bf16x2(uc.w, c[6], c[7]);
  unpack_bf16x2(us.x, s[0], s[1]);
  unpack_bf16x2(us.y, s[2], s[3]);
  unpack_bf16x2(us.z, s[4], s[5]);
  unpack_bf16x2(us.w, s[6], s[7]);
  const float sign = (hl < 8) ? -1.0f : 1.0f;  // rotate_half = cat(-x2, x1)
  float o[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = bf16r(bf16r(v[e] * c[e]) + bf16r(sign * pv[e] * s[e]));
  if (active) {
    uint4 r;
    r.x = pack_bf16x2(o[0], o[1]);
    r.y = pack_bf16x2(o[2], o[3]);
    r.z = pack_bf16x2(o[4], o[5]);
    r.w = pack_bf16x2(o[6], o[7]);
    reinterpret_cast<uint4*>(y + row * 128)[hl] = r;
  }
}

cudaError_t launch_qk_rmsnorm_rope(const __nv_bfloat16* x, __nv_bfloat16* y, const __nv_bfloat16* w,
                                   const int* pos, const __nv_bfloat16* cos_t,
                                   const __nv_bfloat16* sin_t, long long nrows, int heads,
                                   float eps, cudaStream_t stream) {
  const long long threads = nrows * 16;
  const int block = 256;
  const long long grid = (threads + block - 1) / block;
  qk_rmsnorm_rope_kernel<<<static_cast<unsigned>(grid), block, 0, stream>>>(x, y, w, pos, cos_t,
                                                                           sin_t, nrows, heads, eps);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// SwiGLU activation: out[t, i] = bf16( bf16(silu(gate[t, i])) * up[t, i] ).
// gate/up rows are `ld_in` elements apart (the fused [T, 2H] w12 output has gate at column 0
// and up at column H); 8 elements per thread, grid-stride.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) swiglu_kernel(const __nv_bfloat16* __restrict__ gate,
                                                     const __nv_bfloat16* __restrict__ up,
                                                     __nv_bfloat16* __restrict__ out,
                                                     long long rows, int H, long long ld_in,
                                                     long long ld_out) {
  const int vpr = H / 8;
  const long long total = rows * vpr;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / vpr;
    const int c = static_cast<int>(i - r * vpr);
    const uint4 ug = reinterpret_cast<const uint4*>(gate + r * ld_in)[c];
    const uint4 uu = reinterpret_cast<const uint4*>(up + r * ld_in)[c];
    float g[8], u[8], o[8];
    unpack_bf16x2(ug.x, g[0], g[1]);
    unpack_bf16x2(ug.y, g[2], g[3]);
    unpack_bf16x2(ug.z, g[4], g[5]);
    unpack_bf16x2(ug.w, g[6], g[7]);
    unpack_bf16x2(uu.x, u[0], u[1]);
    unpack_bf16x2(uu.y, u[2], u[3]);
    unpack_bf16x2(uu.z, u[4], u[5]);
    unpack_bf16x2(uu.w, u[6], u[7]);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = bf16r(bf16r(g[e] / (1.0f + expf(-g[e]))) * u[e]);
    uint4 res;
    res.x = pack_bf16x2(o[0], o[1]);
    res.y = pack_bf16x2(o[2], o[3]);
    res.z = pack_bf16x2(o[4], o[5]);
    res.w = pack_bf16x2(o[6], o[7]);
    reinterpret_cast<uint4*>(out + r * ld_out)[c] = res;
  }
}

cudaError_t launch_swiglu(const __nv_bfloat16* gate, const __nv_bfloat16* up, __nv_bfloat16* out,
                          long long rows, int H, long long ld_in, long long ld_out, int sms,
                          cudaStream_t stream) {
  const long long total = rows * (H / 8);
  long long grid = (total + 255) / 256;
  const long long cap = static_cast<long long>(sms) * 8;
  if (grid > cap) grid = cap;
  swiglu_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(gate, up, out, rows, H, ld_in,
                                                                  ld_out);
  return cudaGetLastError();
}

}  // namespace rldx
