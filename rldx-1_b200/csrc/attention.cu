// Joint-stream attention for sm_100a: non-causal softmax(Q K^T / sqrt(64)) V over the
// concatenated [cognition | action | physics] token sequence of one batch element and head.
//
// Reference: F.scaled_dot_product_attention over torch.cat([vl, sa, p]) in
// rldx/model/modules/action_model/blocks.py:826-870 (ExpandedDoubleStreamBlock) and
// blocks.py:559-581 (DoubleStreamBlock); the output split back into streams follows
// blocks.py:867-869.  The optional key mask reproduces the -inf masking of masked VL tokens /
// masked physics samples (blocks.py:843-864).
//
// One CTA = one (128-query tile, head, batch element).  Q, K come as [B*H, L, 64] and V as
// V^T [B*H, 64, Lp] (written by the QKV GEMM epilogue), so every tcgen05 operand is K-major:
//   S_j  = Q K_j^T          (M=128, N=64 keys, K=64 dims)   -> TMEM, double buffered
//   O_j  = P_j V_j          (M=128, N=64 dims, K=64 keys)   -> TMEM, double buffered
// The four softmax warps own one query row per thread: row max / sum need no shuffles, P_j is
// written to shared memory in the 128-byte-swizzled K-major layout the next MMA reads, and the
// per-tile O_j is folded into a register accumulator with the online-softmax rescale.
#include "kernels.cuh"

namespace rldx {

constexpr int kAttnThreads = 192;
constexpr int kKvStages = 3;
constexpr int kQBytes = 128 * 128;
constexpr int kKvTileBytes = 64 * 128;
constexpr int kPBytes = 128 * 128;

__global__ void __launch_bounds__(kAttnThreads, 1) joint_attention_kernel(const __grid_constant__ AttnParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kQBytes;                       // kKvStages x 8 KB
  uint8_t* sV = sK + kKvStages * kKvTileBytes;      // kKvStages x 8 KB
  uint8_t* sP = sV + kKvStages * kKvTileBytes;      // 2 x 16 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kPBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kKvStages;
  uint64_t* s_full = kv_empty + kKvStages;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* p_empty = p_full + 2;
  uint64_t* o_full = p_empty + 2;
  uint64_t* o_empty = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 2);

  const int q0 = blockIdx.x * 128;
  const int head = blockIdx.y;
  const int b = blockIdx.z;
  const int bh = b * P.H + head;
  const int L = P.L;
  const int nkv = (L + 63) / 64;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&P.tq);
    tma_prefetch_desc(&P.tk);
    tma_prefetch_desc(&P.tv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) griddep_launch();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      griddep_wait();
      mbar_arrive_expect_tx(q_full, kQBytes);
      tma_load_3d(sQ, &P.tq, q_full, 0, q0, bh, pol);
      for (int j = 0; j < nkv; ++j) {
        const int s = j % kKvStages;
        const uint32_t ph = static_cast<uint32_t>(j / kKvStages) & 1u;
        if (!mbar_wait(&kv_empty[s], ph ^ 1u, kErrAttnTimeout + 1)) break;
        mbar_arrive_expect_tx(&kv_full[s], 2 * kKvTileBytes);
        tma_load_3d(sK + s * kKvTileBytes, &P.tk, &kv_full[s], 0, j * 64, bh, pol);
        tma_load_3d(sV + s * kKvTileBytes, &P.tv, &kv_full[s], j * 64, 0, bh, pol);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(128, 64);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, kErrAttnTimeout + 2);
      auto issue_s = [&](int j) -> bool {
        const int s = j % kKvStages;
        const int sb = j & 1;
        if (!mbar_wait(&kv_full[s], static_cast<uint32_t>(j / kKvStages) & 1u, kErrAttnTimeout + 2))
          return false;
        if (!mbar_wait(&s_empty[sb], (static_cast<uint32_t>(j >> 1) & 1u) ^ 1u, kErrAttnTimeout + 2))
          return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + s * kKvTileBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(tmem + sb * 64, umma_desc_sw128(q_addr + 32 * k),
                   umma_desc_sw128(k_addr + 32 * k), idesc, k != 0 ? 1u : 0u);
        umma_commit(&s_full[sb]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nkv; ++j) {
        if (j + 1 < nkv) {
          ok = issue_s(j + 1);
          if (!ok) break;
        }
        const int pb = j & 1;
        const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
        if (!mbar_wait(&p_full[pb], ph, kErrAttnTimeout + 2)) break;
        if (!mbar_wait(&o_empty[pb], ph ^ 1u, kErrAttnTimeout + 2)) break;
        tc_fence_after();
        const int s = j % kKvStages;
        const uint32_t p_addr = smem_u32(sP + pb * kPBytes);
        const uint32_t v_addr = smem_u32(sV + s * kKvTileBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(tmem + 128 + pb * 64, umma_desc_sw128(p_addr + 32 * k),
                   umma_desc_sw128(v_addr + 32 * k), idesc, k != 0 ? 1u : 0u);
        umma_commit(&o_full[pb]);
        umma_commit(&kv_empty[s]);
        umma_commit(&p_empty[pb]);
      }
    }
  } else {
    // ---------------- softmax / output warps ----------------
    griddep_wait();
    const int lane_grp = warp & 3;
    const int r = lane_grp * 32 + lane;
    const int qrow = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(lane_grp * 32) << 16;
    const unsigned char* kmask = P.key_mask ? P.key_mask + static_cast<size_t>(b) * L : nullptr;
    float m_run = -INFINITY, l_run = 0.0f, alpha_pend = 0.0f;
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.0f;
    bool ok = true;

    auto consume_o = [&](int i, float alpha) -> bool {
      const int ob = i & 1;
      if (!mbar_wait(&o_full[ob], static_cast<uint32_t>(i >> 1) & 1u, kErrAttnTimeout + 3))
        return false;
      tc_fence_after();
      float lo[32], hi[32];
      tmem_ld32(tmem + lane_off + 128 + ob * 64, lo);
      tmem_ld32(tmem + lane_off + 128 + ob * 64 + 32, hi);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[ob]);
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        acc[c] = acc[c] * alpha + lo[c];
        acc[32 + c] = acc[32 + c] * alpha + hi[c];
      }
      return true;
    };

    for (int j = 0; j < nkv; ++j) {
      const int sb = j & 1;
      const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
      if (!mbar_wait(&s_full[sb], ph, kErrAttnTimeout + 3)) { ok = false; break; }
      tc_fence_after();
      float s[64];
      {
        float lo[32], hi[32];
        tmem_ld32(tmem + lane_off + sb * 64, lo);
        tmem_ld32(tmem + lane_off + sb * 64 + 32, hi);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          s[c] = lo[c];
          s[32 + c] = hi[c];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);

      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const int key = j * 64 + c;
        bool vis = key < L;
        if (vis && kmask) vis = kmask[key] != 0;
        s[c] = vis ? s[c] * P.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[c]);
      }
      const float m_new = fmaxf(m_run, mx);
      const float m_use = (m_new == -INFINITY) ? 0.0f : m_new;
      const float alpha = exp2f(m_run - m_use);
      float psum = 0.0f;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        s[c] = exp2f(s[c] - m_use);
        psum += s[c];
      }
      l_run = l_run * alpha + psum;
      m_run = m_new;

      // P_j -> shared memory (K-major, 128-byte swizzle: chunk c of row r at (c ^ (r & 7)) * 16)
      if (!mbar_wait(&p_empty[sb], ph ^ 1u, kErrAttnTimeout + 3)) { ok = false; break; }
      uint8_t* prow = sP + sb * kPBytes + r * 128;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint4 u;
        u.x = pack_bf16x2(s[8 * cc + 0], s[8 * cc + 1]);
        u.y = pack_bf16x2(s[8 * cc + 2], s[8 * cc + 3]);
        u.z = pack_bf16x2(s[8 * cc + 4], s[8 * cc + 5]);
        u.w = pack_bf16x2(s[8 * cc + 6], s[8 * cc + 7]);
        *reinterpret_cast<uint4*>(prow + ((cc ^ (r & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);

      if (j >= 1) {
        if (!consume_o(j - 1, alpha_pend)) { ok = false; break; }
      }
      alpha_pend = alpha;
    }
    if (ok && nkv > 0) ok = consume_o(nkv - 1, alpha_pend);

    if (ok && qrow < L) {
      int seg = 0, off = 0;
      while (seg + 1 < P.nseg && qrow >= off + P.seg_len[seg]) {
        off += P.seg_len[seg];
        ++seg;
      }
      const float inv_l = 1.0f / l_run;
      __nv_bfloat16* dst = P.seg_out[seg] +
                           (static_cast<size_t>(b) * P.seg_len[seg] + (qrow - off)) * (P.H * 64) +
                           head * 64;
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint4 u;
        u.x = pack_bf16x2(acc[8 * cc + 0] * inv_l, acc[8 * cc + 1] * inv_l);
        u.y = pack_bf16x2(acc[8 * cc + 2] * inv_l, acc[8 * cc + 3] * inv_l);
        u.z = pack_bf16x2(acc[8 * cc + 4] * inv_l, acc[8 * cc + 5] * inv_l);
        u.w = pack_bf16x2(acc[8 * cc + 6] * inv_l, acc[8 * cc + 7] * inv_l);
        d4[cc] = u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

size_t attention_smem_bytes() {
  return 1024 + kQBytes + 2 * kKvStages * kKvTileBytes + 2 * kPBytes + 32 * 8;
}

cudaError_t attention_prepare_device() {
  return cudaFuncSetAttribute(joint_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(attention_smem_bytes()));
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.L + 127) / 128, p.H, p.B);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = attention_smem_bytes();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, joint_attention_kernel, p);
}

}  // namespace rldx
