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
//   res_ln_kernel, swiglu_bias_kernel, qkv_prep_kernel  the op-level epilogue / preparation
//                         steps of the reference's ds:: and ss:: custom ops (see each kernel).
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
// A half-warp owns kQkRows consecutive (token, head) rows: lane l of the half holds elements
// 8l..8l+7 of each, the rotate-half partner sits 8 lanes away.  All x loads of a thread are
// issued before any arithmetic.  Products and sums of two bf16 values are exact in fp32, so the
// packed bf16x2 multiply / add (one rounding of the exact result) give the same bits as the
// fp32-compute-then-round of the reference's bf16 tensor ops, at a quarter of the instructions;
// the _rn forms keep the compiler from contracting a multiply and an add into one fma.
// ---------------------------------------------------------------------------------------------
constexpr int kQkRows = 4;

__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 h) { return *reinterpret_cast<uint32_t*>(&h); }

__global__ void __launch_bounds__(256) qk_rmsnorm_rope_kernel(const __grid_constant__ QkNormRopeParams P) {
  const unsigned half_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const int hl = threadIdx.x & 15;
  const int hd = P.hd, nl = hd / 8, hh = nl / 2;  // lanes of a row, lanes of half a row
  const bool act = hl < nl;                      // lanes past the head's dims idle (96-dim heads)
  const int hle = act ? hl : 0;
  const unsigned row0 = half_global * kQkRows;
  uint4 u[kQkRows], uc[kQkRows], us[kQkRows], uw[kQkRows];
#pragma unroll
  for (int k = 0; k < kQkRows; ++k) {
    const unsigned row = min(row0 + k, P.nrows - 1);  // clamped: the tail rows are not stored
    const unsigned tok = row / P.heads, head = row - tok * P.heads;
    u[k] = __ldcs(reinterpret_cast<const uint4*>(P.x + tok * P.x_tok_stride + head * hd) + hle);
  }
#pragma unroll
  for (int k = 0; k < kQkRows; ++k) {
    const unsigned row = min(row0 + k, P.nrows - 1);
    const unsigned tok = row / P.heads, head = row - tok * P.heads;
    const int p = P.pos ? __ldg(P.pos + tok) : static_cast<int>(tok % P.T);
    uc[k] = __ldg(reinterpret_cast<const uint4*>(P.cos + static_cast<size_t>(p) * hd) + hle);
    us[k] = __ldg(reinterpret_cast<const uint4*>(P.sin + static_cast<size_t>(p) * hd) + hle);
    uw[k] = P.norm ? __ldg(reinterpret_cast<const uint4*>(head < P.Hq ? P.wq : P.wk) + hle) : make_uint4(0, 0, 0, 0);
  }
  const uint32_t sign = (hl < hh) ? 0x80008000u : 0u;  // rotate_half = cat(-x2, x1)
  // rotate_half partner: the lane half a row away (within this half-warp)
  const int src_lane = (threadIdx.x & 16) + (hl < hh ? hl + hh : (act ? hl - hh : hl));
#pragma unroll
  for (int k = 0; k < kQkRows; ++k) {
    const uint32_t xv[4] = {u[k].x, u[k].y, u[k].z, u[k].w};
    const uint32_t wv[4] = {uw[k].x, uw[k].y, uw[k].z, uw[k].w};
    uint32_t yv[4], pv[4];
    if (P.norm) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) unpack_bf16x2(xv[i], v[2 * i], v[2 * i + 1]);
      float ss = 0.0f;
      if (act)
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rstd = rsqrtf(ss / static_cast<float>(hd) + P.eps);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        yv[i] = as_u32(__hmul2_rn(as_bf2(wv[i]), __floats2bfloat162_rn(v[2 * i] * rstd, v[2 * i + 1] * rstd)));
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) yv[i] = xv[i];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) pv[i] = __shfl_sync(0xffffffffu, yv[i], src_lane) ^ sign;
    const uint32_t cv[4] = {uc[k].x, uc[k].y, uc[k].z, uc[k].w};
    const uint32_t sv[4] = {us[k].x, us[k].y, us[k].z, us[k].w};
    uint32_t ov[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      ov[i] = as_u32(__hadd2_rn(__hmul2_rn(as_bf2(yv[i]), as_bf2(cv[i])), __hmul2_rn(as_bf2(pv[i]), as_bf2(sv[i]))));
    const unsigned row = row0 + k;
    if (row < P.nrows && act) {
      __nv_bfloat16* dst;
      if (P.layout == 0) {
        dst = P.y + static_cast<size_t>(row) * hd;
      } else {  // attention layout: q [B, Hq, T, out_hd] or k [B, H - Hq, T, out_hd]
        const unsigned tok = row / P.heads, head = row - tok * P.heads;
        const unsigned b = tok / P.T, t = tok - b * P.T;
        dst = head < P.Hq ? P.q + ((static_cast<size_t>(b) * P.Hq + head) * P.T + t) * P.out_hd
                          : P.k + ((static_cast<size_t>(b) * (P.heads - P.Hq) + head - P.Hq) * P.T + t) * P.out_hd;
      }
      __stcs(reinterpret_cast<uint4*>(dst) + hl, make_uint4(ov[0], ov[1], ov[2], ov[3]));
    }
  }
}

cudaError_t launch_qk_rmsnorm_rope(const QkNormRopeParams& p, cudaStream_t stream) {
  if (p.nrows == 0 || p.nrows >= (1u << 31) || p.heads == 0 || p.Hq == 0 || p.Hq > p.heads || p.T == 0 ||
      (p.hd != 96 && p.hd != 128) || (p.layout == 1 && p.out_hd < p.hd))
    return cudaErrorInvalidValue;
  const long long halves = (static_cast<long long>(p.nrows) + kQkRows - 1) / kQkRows;
  const int block = 256;
  const long long grid = (halves * 16 + block - 1) / block;
  qk_rmsnorm_rope_kernel<<<static_cast<unsigned>(grid), block, 0, stream>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// V^T for the attention kernel from projected rows: v [B*T tokens, row stride ld] with kv head
// h at columns h*128..h*128+127  ->  vt [B, Hkv, 128, Tp].  One CTA = 32 tokens x one kv head
// of one batch element, through shared memory so both sides move 16-byte vectors.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) v_transpose_kernel(const __nv_bfloat16* __restrict__ v, long long ld,
                                                          __nv_bfloat16* __restrict__ vt, int T, int Tp, int Hkv,
                                                          int hd, int out_hd) {
  __shared__ __align__(16) __nv_bfloat16 tile[128][40];  // [dim][token]
  const int t0 = blockIdx.x * 32, hv = blockIdx.y, b = blockIdx.z;
#pragma unroll
  for (int i = 0; i < 2; ++i) {  // 32 tokens x 16 chunks of 8 dims
    const int idx = threadIdx.x + 256 * i;
    const int tl = idx >> 4, ch = idx & 15;
    const int t = t0 + tl;
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (t < T && ch * 8 < hd)
      u = *reinterpret_cast<const uint4*>(v + (static_cast<size_t>(b) * T + t) * ld + hv * hd + ch * 8);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) tile[ch * 8 + j][tl] = e[j];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 2; ++i) {  // 128 dims x 4 groups of 8 tokens
    const int idx = threadIdx.x + 256 * i;
    const int d = idx >> 2, grp = idx & 3;
    const int t = t0 + grp * 8;
    if (t < Tp && d < hd)
      *reinterpret_cast<uint4*>(vt + ((static_cast<size_t>(b) * Hkv + hv) * out_hd + d) * Tp + t) =
          *reinterpret_cast<const uint4*>(&tile[d][grp * 8]);
  }
}

cudaError_t launch_v_transpose(const __nv_bfloat16* v, long long ld, __nv_bfloat16* vt, int B, int T, int Tp,
                               int Hkv, int hd, int out_hd, cudaStream_t stream) {
  if (B <= 0 || T <= 0 || Tp < T || Tp % 8 || Hkv <= 0 || hd % 8 || hd > 128 || out_hd < hd) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>((T + 31) / 32), static_cast<unsigned>(Hkv), static_cast<unsigned>(B));
  v_transpose_kernel<<<grid, 256, 0, stream>>>(v, ld, vt, T, Tp, Hkv, hd, out_hd);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// SwiGLU activation: out[t, i] = bf16( bf16(silu(gate[t, i])) * up[t, i] ).
// gate/up rows are `ld_in` elements apart (the fused [T, 2H] w12 output has gate at column 0
// and up at column H).  One CTA row-slice: blockIdx.x is the row, blockIdx.y a slice of
// 256 * kV 16-byte vectors; every load of a thread is issued before the arithmetic.  silu in
// fp32 with the fast exponential and division intrinsics; the product of two bf16 values is
// exact, so the packed bf16x2 multiply rounds it exactly like the reference's bf16 tensor op.
// ---------------------------------------------------------------------------------------------
template <int kV>
__global__ void __launch_bounds__(256) swiglu_kernel(const __nv_bfloat16* __restrict__ gate,
                                                     const __nv_bfloat16* __restrict__ up,
                                                     __nv_bfloat16* __restrict__ out, int H,
                                                     long long ld_in, long long ld_out) {
  const int vpr = H / 8;
  const size_t r = blockIdx.x;
  const int c0 = blockIdx.y * (256 * kV) + threadIdx.x;
  const uint4* g4 = reinterpret_cast<const uint4*>(gate + r * ld_in);
  const uint4* u4 = reinterpret_cast<const uint4*>(up + r * ld_in);
  uint4* o4 = reinterpret_cast<uint4*>(out + r * ld_out);
  uint4 ug[kV], uu[kV];
#pragma unroll
  for (int j = 0; j < kV; ++j) {
    const int c = c0 + 256 * j;
    if (c < vpr) {
      ug[j] = __ldcs(g4 + c);
      uu[j] = __ldcs(u4 + c);
    }
  }
#pragma unroll
  for (int j = 0; j < kV; ++j) {
    const int c = c0 + 256 * j;
    if (c < vpr) {
      const uint32_t gv[4] = {ug[j].x, ug[j].y, ug[j].z, ug[j].w};
      const uint32_t uv[4] = {uu[j].x, uu[j].y, uu[j].z, uu[j].w};
      uint32_t ov[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float a, b;
        unpack_bf16x2(gv[i], a, b);
        const __nv_bfloat162 s =
            __floats2bfloat162_rn(__fdividef(a, 1.0f + __expf(-a)), __fdividef(b, 1.0f + __expf(-b)));
        ov[i] = as_u32(__hmul2_rn(s, as_bf2(uv[i])));
      }
      __stcs(o4 + c, make_uint4(ov[0], ov[1], ov[2], ov[3]));
    }
  }
}

cudaError_t launch_swiglu(const __nv_bfloat16* gate, const __nv_bfloat16* up, __nv_bfloat16* out,
                          long long rows, int H, long long ld_in, long long ld_out, int sms,
                          cudaStream_t stream) {
  (void)sms;
  if (rows <= 0 || rows >= (1ll << 31) || H <= 0) return cudaErrorInvalidValue;
  const int vpr = H / 8;
  int v = 1;
  while (v < 8 && 256 * v < vpr) v *= 2;
  const int slices = (vpr + 256 * v - 1) / (256 * v);
  if (slices > 65535) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(rows), static_cast<unsigned>(slices));
  switch (v) {
    case 1: swiglu_kernel<1><<<grid, 256, 0, stream>>>(gate, up, out, H, ld_in, ld_out); break;
    case 2: swiglu_kernel<2><<<grid, 256, 0, stream>>>(gate, up, out, H, ld_in, ld_out); break;
    case 4: swiglu_kernel<4><<<grid, 256, 0, stream>>>(gate, up, out, H, ld_in, ld_out); break;
    default: swiglu_kernel<8><<<grid, 256, 0, stream>>>(gate, up, out, H, ld_in, ld_out); break;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// QKV preparation for the joint attention, from projected [q | k | v] rows (the input of the
// reference's ds::/ss::fused_attention_{2,3}way ops): per-head RMSNorm of q and k (fp32 rstd,
// weight then cast, norms.py:18-22), rotation of interleaved pairs with fp32 cos / sin and one
// rounding (ops.py:48-67), scatter to q, k [B, H, L, 64] and V^T [B, H, 64, Lp].
// One CTA = 32 consecutive tokens of the joint sequence x one head of one batch element; a warp
// takes 4 tokens, a lane 2 of the 64 dims.  V goes through shared memory so that V^T is
// written as 64-byte rows.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) qkv_prep_kernel(const __grid_constant__ QkvPrepParams P) {
  __shared__ __align__(16) __nv_bfloat16 sv[64][40];  // [dim][token], rows 80 bytes apart
  const int t0 = blockIdx.x * 32;
  const int head = blockIdx.y;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int inner = P.H * 64;
  const size_t bh = static_cast<size_t>(b) * P.H + head;
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    const int tl = warp * 4 + i;
    const int t = t0 + tl;
    float vx = 0.0f, vy = 0.0f;
    if (t < P.L) {  // uniform over the warp
      int s = 0, off = 0;
      while (s + 1 < P.nseg && t >= off + P.seg[s].rows) {
        off += P.seg[s].rows;
        ++s;
      }
      const QkvPrepSeg& sg = P.seg[s];
      const int r = t - off;
      const __nv_bfloat16* row = sg.qkv + b * sg.batch_stride + static_cast<long long>(r) * sg.ld + head * 64;
      const bool rot = sg.cos != nullptr && r >= sg.rope_from;
      float c = 1.0f, sn = 0.0f;
      if (rot) {
        c = sg.cos[static_cast<size_t>(r - sg.rope_from) * 32 + lane];
        sn = sg.sin[static_cast<size_t>(r - sg.rope_from) * 32 + lane];
      }
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        float x0, x1;
        unpack_bf16x2(*reinterpret_cast<const uint32_t*>(row + part * inner + 2 * lane), x0, x1);
        float ss = x0 * x0 + x1 * x1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rstd = rsqrtf(ss * (1.0f / 64.0f) + P.eps);
        const __nv_bfloat16* w = part == 0 ? sg.qn : sg.kn;
        float w0, w1;
        unpack_bf16x2(*reinterpret_cast<const uint32_t*>(w + 2 * lane), w0, w1);
        const float a = bf16r(w0 * (x0 * rstd));
        const float bb = bf16r(w1 * (x1 * rstd));
        const uint32_t out = pack_bf16x2(a * c - bb * sn, a * sn + bb * c);
        __nv_bfloat16* dst = (part == 0 ? P.q : P.k) + (bh * P.L + t) * 64 + 2 * lane;
        *reinterpret_cast<uint32_t*>(dst) = out;
      }
      unpack_bf16x2(*reinterpret_cast<const uint32_t*>(row + 2 * inner + 2 * lane), vx, vy);
    }
    sv[2 * lane][tl] = __float2bfloat16_rn(vx);
    sv[2 * lane + 1][tl] = __float2bfloat16_rn(vy);
  }
  __syncthreads();
  // V^T rows: thread -> (dim d, 8-token group); tokens past L write zeros inside Lp only
  const int d = threadIdx.x >> 2, grp = threadIdx.x & 3;
  const int tok = t0 + grp * 8;
  if (tok < P.Lp) {
    const uint4 u = *reinterpret_cast<const uint4*>(&sv[d][grp * 8]);
    *reinterpret_cast<uint4*>(P.vt + (bh * 64 + d) * P.Lp + tok) = u;
  }
}

cudaError_t launch_qkv_prep(const QkvPrepParams& p, cudaStream_t stream) {
  if (p.nseg < 1 || p.nseg > 3 || p.B <= 0 || p.H <= 0 || p.L <= 0 || p.Lp < p.L || p.Lp % 8)
    return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>((p.L + 31) / 32), static_cast<unsigned>(p.H), static_cast<unsigned>(p.B));
  qkv_prep_kernel<<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// Residual sums + LayerNorm of the reference's epilogue ops (one warp per row):
//   ds::vl_epilogue_ln  new = bf16 sequence x + v1 + v2 + y, ln = LN(new)
//     (rldx/inference/action_model/double_stream/engine/kernels/vl_epilogue_ln.py:53-75)
//   ss::fused_epilogue_ln  new = bf16(x + y), ln = LN(new)
//     (rldx/inference/action_model/single_stream/engine/kernels/ss_epilogue_ln.py:57-84)
//   ds::grouped_res_ln  ln = LN(x + y + v1) summed in fp32
//     (rldx/inference/action_model/double_stream/engine/kernels/grouped_res_ln.py:70-147)
// ---------------------------------------------------------------------------------------------
template <int kVec>
__global__ void __launch_bounds__(128) res_ln_kernel(const __grid_constant__ ResLnParams P) {
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_global >= P.total_rows) return;
  const ResLnSeg& sg = (P.nseg > 1 && warp_global >= P.seg[1].row_begin) ? P.seg[1] : P.seg[0];
  const int row = warp_global - sg.row_begin;
  const int nvec = sg.D / 8;
  const size_t off = static_cast<size_t>(row) * sg.ld;
  float x[kVec][8];
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      float a[8], t[8];
      const uint4 ua = reinterpret_cast<const uint4*>(sg.x + off)[v];
      unpack_bf16x2(ua.x, a[0], a[1]);
      unpack_bf16x2(ua.y, a[2], a[3]);
      unpack_bf16x2(ua.z, a[4], a[5]);
      unpack_bf16x2(ua.w, a[6], a[7]);
      auto add = [&](const __nv_bfloat16* p, bool round) {
        const uint4 u = reinterpret_cast<const uint4*>(p)[v];
        unpack_bf16x2(u.x, t[0], t[1]);
        unpack_bf16x2(u.y, t[2], t[3]);
        unpack_bf16x2(u.z, t[4], t[5]);
        unpack_bf16x2(u.w, t[6], t[7]);
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = round ? bf16r(a[e] + t[e]) : a[e] + t[e];
      };
      if (P.fp32_sum) {
        if (sg.y) add(sg.y + off, false);
        if (sg.v1) add(sg.v1, false);
        if (sg.v2) add(sg.v2, false);
      } else {
        if (sg.v1) add(sg.v1, true);
        if (sg.v2) add(sg.v2, true);
        if (sg.y) add(sg.y + off, true);
      }
      if (sg.sum_out) {
        uint4 r;
        r.x = pack_bf16x2(a[0], a[1]);
        r.y = pack_bf16x2(a[2], a[3]);
        r.z = pack_bf16x2(a[4], a[5]);
        r.w = pack_bf16x2(a[6], a[7]);
        reinterpret_cast<uint4*>(sg.sum_out + off)[v] = r;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        x[i][e] = a[e];
        sum += a[e];
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = P.rms ? 0.0f : sum / static_cast<float>(sg.D);  // RMSNorm: no centring
  float var = 0.0f;
#pragma unroll
  for (int i = 0; i < kVec; ++i)
    if (lane + 32 * i < nvec)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = x[i][e] - mean;
        var += d * d;
      }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
  const float rstd = rsqrtf(var / static_cast<float>(sg.D) + P.eps);
  if (P.rms && P.rms_weight_first) {  // weight times the fp32 normalised value, one rounding
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      const int v = lane + 32 * i;
      if (v < nvec) {
        const uint4 uw = reinterpret_cast<const uint4*>(sg.w)[v];
        float wv[8];
        unpack_bf16x2(uw.x, wv[0], wv[1]);
        unpack_bf16x2(uw.y, wv[2], wv[3]);
        unpack_bf16x2(uw.z, wv[4], wv[5]);
        unpack_bf16x2(uw.w, wv[6], wv[7]);
        uint4 r;
        r.x = pack_bf16x2(wv[0] * (x[i][0] * rstd), wv[1] * (x[i][1] * rstd));
        r.y = pack_bf16x2(wv[2] * (x[i][2] * rstd), wv[3] * (x[i][3] * rstd));
        r.z = pack_bf16x2(wv[4] * (x[i][4] * rstd), wv[5] * (x[i][5] * rstd));
        r.w = pack_bf16x2(wv[6] * (x[i][6] * rstd), wv[7] * (x[i][7] * rstd));
        reinterpret_cast<uint4*>(sg.ln_out + off)[v] = r;
      }
    }
    return;
  }
  if (P.rms) {  // cast, then the bf16 weight (packed multiply: exact product, one rounding)
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      const int v = lane + 32 * i;
      if (v < nvec) {
        const uint4 uw = reinterpret_cast<const uint4*>(sg.w)[v];
        const uint32_t wv[4] = {uw.x, uw.y, uw.z, uw.w};
        uint32_t ov[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ov[k] = as_u32(__hmul2_rn(as_bf2(wv[k]), __floats2bfloat162_rn(x[i][2 * k] * rstd, x[i][2 * k + 1] * rstd)));
        reinterpret_cast<uint4*>(sg.ln_out + off)[v] = make_uint4(ov[0], ov[1], ov[2], ov[3]);
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      uint4 r;
      r.x = pack_bf16x2((x[i][0] - mean) * rstd, (x[i][1] - mean) * rstd);
      r.y = pack_bf16x2((x[i][2] - mean) * rstd, (x[i][3] - mean) * rstd);
      r.z = pack_bf16x2((x[i][4] - mean) * rstd, (x[i][5] - mean) * rstd);
      r.w = pack_bf16x2((x[i][6] - mean) * rstd, (x[i][7] - mean) * rstd);
      reinterpret_cast<uint4*>(sg.ln_out + off)[v] = r;
    }
  }
}

cudaError_t launch_res_ln(const ResLnParams& p, cudaStream_t stream) {
  if (p.total_rows <= 0 || p.dmax <= 0 || p.dmax > 4096) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>((p.total_rows + 3) / 4);
  if (p.dmax <= 32 * 8 * 6) res_ln_kernel<6><<<grid, 128, 0, stream>>>(p);
  else res_ln_kernel<16><<<grid, 128, 0, stream>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// ds::grouped_swiglu: out = bf16( silu(gate + bg) * (up + bu) ), every step in fp32
// (rldx/inference/action_model/double_stream/engine/kernels/grouped_swiglu.py:150-170).
// blockIdx.x is the row of the concatenated segments, blockIdx.y a slice of 256 x 8 columns.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) swiglu_bias_kernel(const __grid_constant__ SwigluBiasParams P) {
  const int grow = blockIdx.x;
  const SwigluBiasSeg& sg = (P.nseg > 1 && grow >= P.seg[1].row_begin) ? P.seg[1] : P.seg[0];
  const size_t r = grow - sg.row_begin;
  const int c = blockIdx.y * 256 + threadIdx.x;
  if (c >= sg.H / 8) return;
  const uint4 ug = reinterpret_cast<const uint4*>(sg.gate + r * sg.ld_in)[c];
  const uint4 uu = reinterpret_cast<const uint4*>(sg.up + r * sg.ld_in)[c];
  const uint4 bg = reinterpret_cast<const uint4*>(sg.bg)[c];
  const uint4 bu = reinterpret_cast<const uint4*>(sg.bu)[c];
  const uint32_t gv[4] = {ug.x, ug.y, ug.z, ug.w}, uv[4] = {uu.x, uu.y, uu.z, uu.w};
  const uint32_t bgv[4] = {bg.x, bg.y, bg.z, bg.w}, buv[4] = {bu.x, bu.y, bu.z, bu.w};
  uint32_t ov[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float g0, g1, u0, u1, a0, a1, b0, b1;
    unpack_bf16x2(gv[i], g0, g1);
    unpack_bf16x2(uv[i], u0, u1);
    unpack_bf16x2(bgv[i], a0, a1);
    unpack_bf16x2(buv[i], b0, b1);
    g0 += a0;
    g1 += a1;
    u0 += b0;
    u1 += b1;
    ov[i] = pack_bf16x2(g0 * __fdividef(1.0f, 1.0f + __expf(-g0)) * u0, g1 * __fdividef(1.0f, 1.0f + __expf(-g1)) * u1);
  }
  reinterpret_cast<uint4*>(sg.out + r * sg.ld_out)[c] = make_uint4(ov[0], ov[1], ov[2], ov[3]);
}

cudaError_t launch_swiglu_bias(const SwigluBiasParams& p, cudaStream_t stream) {
  if (p.total_rows <= 0 || p.hmax <= 0) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(p.total_rows), static_cast<unsigned>((p.hmax / 8 + 255) / 256));
  swiglu_bias_kernel<<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace rldx
