// Grouped tcgen05 GEMM with fused row epilogues (see gemm.cuh for the CTA layout).
//
// Rounding follows the reference bf16 eager path step by step: nn.Linear rounds once after
// the fused bias (cuBLASLt bias epilogue), CategorySpecificLinear (bmm + b) rounds the matmul
// and then the bias add, every elementwise op (SiLU, swish, products, residual adds, the
// Euler update) rounds its bf16 result.  References:
//   nn.Linear / SwiGLUFFN            rldx/model/modules/action_model/ops.py:137-161
//   CategorySpecificLinear            rldx/model/modules/embodiment_conditioned_mlp.py:72-82
//   swish (x * sigmoid(x))            rldx/model/modules/embodiment_conditioned_mlp.py:24-26
//   QK RMSNorm (weight then cast)     rldx/model/modules/norms.py:18-22
//   RoPE on interleaved pairs         rldx/model/modules/action_model/ops.py:48-67
//   Euler update                      rldx/model/core/rldx.py:716-723
#include "gemm.cuh"

namespace rldx {

__device__ __forceinline__ float apply_act(float y, int act) {
  if (act == kActRelu) return fmaxf(y, 0.0f);
  if (act == kActSilu) return bf16r(y / (1.0f + expf(-y)));
  if (act == kActSwish) {  // sigmoid rounded to bf16, then the product rounded
    const float sg = bf16r(1.0f / (1.0f + expf(-y)));
    return bf16r(y * sg);
  }
  return y;
}

__device__ __forceinline__ float finish_acc(float acc, float b, int bias_mode) {
  if (bias_mode == kBiasFused) return bf16r(acc + b);
  if (bias_mode == kBiasPostRound) return bf16r(bf16r(acc) + b);
  return bf16r(acc);
}

__device__ __forceinline__ void load_bf16x64(const __nv_bfloat16* src, bool vec_ok, int nvalid,
                                             float (&dst)[64]) {
  if (vec_ok && nvalid >= 64) {
    const uint4* p = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint4 u = p[i];
      unpack_bf16x2(u.x, dst[8 * i + 0], dst[8 * i + 1]);
      unpack_bf16x2(u.y, dst[8 * i + 2], dst[8 * i + 3]);
      unpack_bf16x2(u.z, dst[8 * i + 4], dst[8 * i + 5]);
      unpack_bf16x2(u.w, dst[8 * i + 6], dst[8 * i + 7]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) dst[i] = (i < nvalid) ? __bfloat162float(src[i]) : 0.0f;
  }
}

__device__ __forceinline__ void store_bf16x64(__nv_bfloat16* dst, bool vec_ok, int nvalid,
                                              const float (&v)[64]) {
  if (vec_ok && nvalid >= 64) {
    uint4* p = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint4 u;
      u.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
      u.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
      u.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
      u.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
      p[i] = u;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i)
      if (i < nvalid) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

// Epilogue of one 128 x BN tile; thread = accumulator row (TMEM lane).
__device__ __forceinline__ void gemm_epilogue(const GemmProblem& pr, uint32_t tmem_acc, int tm,
                                              int tn, int lane_grp, int lane) {
  const GemmEpilogue& ep = pr.ep;
  const int r_local = lane_grp * 32 + lane;
  const int row = tm * pr.m_step + r_local;
  const bool valid = (r_local < pr.m_step) && (row < pr.M);
  int bidx = 0, t = row;
  if (ep.rows_in > 0) {
    bidx = row / ep.rows_in;
    t = row - bidx * ep.rows_in;
  }
  const bool dropped = (ep.rows_in > 0) && (t < ep.row_skip);
  const int out_row = (ep.rows_in > 0) ? bidx * ep.rows_out + t - ep.row_skip : row;
  int cat = 0;
  if (pr.cat_ids != nullptr) cat = static_cast<int>(pr.cat_ids[tm]);
  const __nv_bfloat16* bias =
      ep.bias ? ep.bias + static_cast<size_t>(cat) * ep.bias_cat_stride : nullptr;
  const uint32_t tbase = tmem_acc + (static_cast<uint32_t>(lane_grp * 32) << 16);

  for (int c = 0; c < pr.bn / 64; ++c) {
    float lo[32], hi[32];
    tmem_ld32(tbase + c * 64, lo);
    tmem_ld32(tbase + c * 64 + 32, hi);
    tmem_wait_ld();
    const int n0 = tn * pr.bn + c * 64;
    if (!valid || dropped || n0 >= pr.N) continue;
    const int nvalid = min(64, pr.N - n0);
    float v[64];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      v[i] = lo[i];
      v[32 + i] = hi[i];
    }
    float bv[64];
    if (bias) {
      load_bf16x64(bias + n0, (n0 % 8) == 0, nvalid, bv);
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) bv[i] = 0.0f;
    }

    if (ep.mode == kEpiStore || ep.mode == kEpiEuler) {
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = apply_act(finish_acc(v[i], bv[i], ep.bias_mode), ep.act);
      if (ep.add) {
        const int arow = ep.add_row_mod > 0 ? (t % ep.add_row_mod) : row;
        float av[64];
        const __nv_bfloat16* ap = ep.add + static_cast<size_t>(arow) * ep.ld_add + n0;
        load_bf16x64(ap, (ep.ld_add % 8 == 0) && (n0 % 8 == 0), nvalid, av);
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = bf16r(v[i] + av[i]);
      }
      __nv_bfloat16* op = ep.out + static_cast<size_t>(out_row) * ep.ldo + ep.col_off + n0;
      const bool vec_ok = (ep.ldo % 8 == 0) && ((ep.col_off + n0) % 8 == 0);
      if (ep.mode == kEpiEuler) {
        float xv[64];
        load_bf16x64(op, vec_ok, nvalid, xv);
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = bf16r(xv[i] + bf16r(ep.dt * v[i]));
      }
      store_bf16x64(op, vec_ok, nvalid, v);
    } else if (ep.mode == kEpiSwiGLU) {
      // columns [0,32) gate, [32,64) up of hidden units n0/2 .. n0/2+31
      float h[64];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float g = finish_acc(v[i], bv[i], ep.bias_mode);
        const float u = finish_acc(v[32 + i], bv[32 + i], ep.bias_mode);
        const float sg = bf16r(g / (1.0f + expf(-g)));
        h[i] = bf16r(sg * u);
        h[32 + i] = 0.0f;
      }
      const int hcol = n0 / 2;
      __nv_bfloat16* op = ep.out + static_cast<size_t>(out_row) * ep.ldo + ep.col_off + hcol;
      const bool vec_ok = (ep.ldo % 8 == 0) && ((ep.col_off + hcol) % 8 == 0);
      if (vec_ok) {
        uint4* p = reinterpret_cast<uint4*>(op);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 u;
          u.x = pack_bf16x2(h[8 * i + 0], h[8 * i + 1]);
          u.y = pack_bf16x2(h[8 * i + 2], h[8 * i + 3]);
          u.z = pack_bf16x2(h[8 * i + 4], h[8 * i + 5]);
          u.w = pack_bf16x2(h[8 * i + 6], h[8 * i + 7]);
          p[i] = u;
        }
      } else {
        for (int i = 0; i < 32; ++i) op[i] = __float2bfloat16_rn(h[i]);
      }
    } else {  // kEpiQKV: chunk = one head of q, k or v
      const int inner = ep.H * 64;
      const int part = n0 / inner;
      const int head = (n0 - part * inner) / 64;
      const int tok = ep.tok_off + t;
      const size_t bh = static_cast<size_t>(bidx) * ep.H + head;
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = finish_acc(v[i], bv[i], kBiasFused);
      if (part < 2) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 64; ++i) ss += v[i] * v[i];
        const float rstd = rsqrtf(ss * (1.0f / 64.0f) + ep.eps);
        const __nv_bfloat16* w = (part == 0) ? ep.qn_w : ep.kn_w;
        float wv[64];
        load_bf16x64(w, true, 64, wv);
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = bf16r(wv[i] * (v[i] * rstd));
        const float* cs = ep.rope_cos + static_cast<size_t>(tok) * 32;
        const float* sn = ep.rope_sin + static_cast<size_t>(tok) * 32;
#pragma unroll
        for (int p = 0; p < 32; ++p) {
          const float c0 = cs[p], s0 = sn[p];
          const float a = v[2 * p], b = v[2 * p + 1];
          v[2 * p] = bf16r(a * c0 - b * s0);
          v[2 * p + 1] = bf16r(a * s0 + b * c0);
        }
        __nv_bfloat16* dst = ((part == 0) ? ep.q : ep.k) + (bh * ep.L + tok) * 64;
        store_bf16x64(dst, true, 64, v);
      } else {
        __nv_bfloat16* dst = ep.vt + bh * 64 * ep.Lp + tok;
#pragma unroll
        for (int d = 0; d < 64; ++d) dst[static_cast<size_t>(d) * ep.Lp] = __float2bfloat16_rn(v[d]);
      }
    }
  }
}

__global__ void __launch_bounds__(kGemmThreads, 1) gemm_bf16_kernel(const __grid_constant__ GemmParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int S = P.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * P.stage_bytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* accum = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int bid = blockIdx.x;
  int pi = 0;
#pragma unroll
  for (int i = 1; i < kMaxProblems; ++i)
    if (i < P.nprob && bid >= P.p[i].tile_begin) pi = i;
  const GemmProblem& pr = P.p[pi];
  const int local = bid - pr.tile_begin;
  const int tm = local % pr.tiles_m;
  const int tn = local / pr.tiles_m;
  const int nk = (pr.K + 63) / 64;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&pr.ta);
    tma_prefetch_desc(&pr.tb);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_acc = *tmem_slot;
  if (threadIdx.x == 0) griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t a_bytes = static_cast<uint32_t>(pr.a_rows) * 128u;
      const uint32_t b_bytes = static_cast<uint32_t>(pr.bn) * 128u;
      const uint64_t pol_a = l2_policy_evict_last();
      const uint64_t pol_b = (pr.tiles_m == 1) ? l2_policy_evict_first() : l2_policy_evict_last();
      const int a_row0 = tm * pr.m_step;
      const int n0 = tn * pr.bn;
      const int cat = pr.cat_ids ? static_cast<int>(pr.cat_ids[tm]) : 0;
      const int npre = min(S, nk);
      // Weight tiles do not depend on the previous kernel: issue them first.
      for (int kb = 0; kb < npre; ++kb) {
        uint8_t* st = smem + kb * P.stage_bytes;
        mbar_arrive_expect_tx(&full[kb], a_bytes + b_bytes);
        if (pr.cat_ids)
          tma_load_3d(st + kATileBytes, &pr.tb, &full[kb], kb * 64, n0, cat, pol_b);
        else
          tma_load_2d(st + kATileBytes, &pr.tb, &full[kb], kb * 64, n0, pol_b);
      }
      griddep_wait();
      for (int kb = 0; kb < npre; ++kb)
        tma_load_2d(smem + kb * P.stage_bytes, &pr.ta, &full[kb], kb * 64, a_row0, pol_a);
      for (int kb = npre; kb < nk; ++kb) {
        const int s = kb % S;
        const uint32_t ph = static_cast<uint32_t>(kb / S) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, kErrGemmTimeout + 1)) break;
        uint8_t* st = smem + s * P.stage_bytes;
        mbar_arrive_expect_tx(&full[s], a_bytes + b_bytes);
        if (pr.cat_ids)
          tma_load_3d(st + kATileBytes, &pr.tb, &full[s], kb * 64, n0, cat, pol_b);
        else
          tma_load_2d(st + kATileBytes, &pr.tb, &full[s], kb * 64, n0, pol_b);
        tma_load_2d(st, &pr.ta, &full[s], kb * 64, a_row0, pol_a);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(128, pr.bn);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S;
        const uint32_t ph = static_cast<uint32_t>(kb / S) & 1u;
        if (!mbar_wait(&full[s], ph, kErrGemmTimeout + 2)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * P.stage_bytes);
        const uint32_t b_addr = a_addr + kATileBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          umma_f16(tmem_acc, umma_desc_sw128(a_addr + 32 * k), umma_desc_sw128(b_addr + 32 * k),
                   idesc, (kb | k) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else {
    griddep_wait();
    if (mbar_wait(accum, 0, kErrGemmTimeout + 3)) {
      tc_fence_after();
      gemm_epilogue(pr, tmem_acc, tm, tn, warp & 3, lane);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_acc, 256);
  }
}

size_t gemm_smem_bytes(int stages, int stage_bytes) {
  return 1024 + static_cast<size_t>(stages) * stage_bytes + (2 * kMaxStages + 2) * 8;
}

cudaError_t gemm_prepare_device() {
  return cudaFuncSetAttribute(gemm_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              227 * 1024);
}

cudaError_t launch_gemm(const GemmParams& params, int total_tiles, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(total_tiles, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = gemm_smem_bytes(params.stages, params.stage_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemm_bf16_kernel, params);
}

}  // namespace rldx
