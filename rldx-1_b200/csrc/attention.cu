// Joint-stream attention for sm_100a: non-causal softmax(Q K^T / sqrt(d)) V over the
// concatenated [cognition | action | physics] token sequence of one batch element and head,
// head_dim d = 64 (MSAT) or 128 (the joint-attention sweep shapes).  The same kernel serves the
// decoder prefill of the VLM backbone: causal masking (key j visible to query i iff j <= i; a
// CTA stops at the key tile of its last query row) and grouped-query heads (query head h reads
// K / V head h / (H / kv_heads)), as Qwen3's sdpa / eager attention with repeat_kv
// (rldx/model/modules/backbone/modeling_qwen3_vl.py:139-175, 404-490).
//
// Reference: F.scaled_dot_product_attention over torch.cat([vl, sa, p]) in
// rldx/model/modules/action_model/blocks.py:826-870 (ExpandedDoubleStreamBlock) and
// blocks.py:559-581 (DoubleStreamBlock); the output split back into streams follows
// blocks.py:867-869.  The optional key mask reproduces the -inf masking of masked VL tokens /
// masked physics samples (blocks.py:843-864).
//
// One CTA = one or two 128-query tiles of one (head, batch element).  Q, K come as [B*H, L, d] and V as
// V^T [B*H, d, Lp] (written by the QKV GEMM epilogue), so every tcgen05 operand is K-major:
//   S_j  = Q K_j^T          (M=128, N=64 keys, K=d dims)    -> TMEM, double buffered
//   O   += P_j V_j          (M=128, N=d dims, K=64 keys)    -> one TMEM accumulator
// Q and K tiles are held as d/64 chunks of 64 dims (one 128-byte swizzle atom per row each).
// Each softmax warpgroup (four warps) owns one query tile, one row per thread, so row max / sum
// need no shuffles.
// P_j goes to shared memory in the 128-byte-swizzled K-major layout the PV MMA reads.  The
// running max is rescaled lazily: exponentials use a reference max that only moves when a
// row's max grows by more than 2^8 (P then stays <= 256, exact in the final O / l); only then
// is that row of O read from TMEM, scaled and written back, after the previous PV MMA landed.
#include "host_util.h"
#include "kernels.cuh"

namespace rldx {

constexpr int kPBytes = 128 * 128;
constexpr float kRescaleLog2 = 8.0f;  // lazy-rescale threshold (log2 units)

// kG query tiles of 128 rows per CTA share every K / V tile: kG = 1 for latency (more CTAs),
// kG = 2 for throughput (two softmax warpgroups keep the special-function and ALU pipes busy
// while the tensor core works on the other tile, and K / V are read once per 256 queries).
// TMEM columns: S of group g, buffer b at (2g + b) * 64; O of group g at kG * 128 + g * d.
template <int kHD, int kG>
struct AttnShape {
  static constexpr int kChunks = kHD / 64;           // 64-dim chunks of a Q / K row
  static constexpr int kQBytes = 128 * kHD * 2;      // 128 queries
  static constexpr int kQChunk = 128 * 128;          // one 64-dim chunk of a Q tile
  static constexpr int kKTileBytes = 64 * kHD * 2;   // 64 keys
  static constexpr int kKChunk = 64 * 128;           // one 64-dim chunk of a K tile
  static constexpr int kVTileBytes = kHD * 64 * 2;   // V^T: d rows x 64 keys
  // separate K and V rings: K(j) is free once the S MMAs of tile j are done, V(j) once its PV
  // MMAs are, so the K loads run ahead of the PV work
  static constexpr int kKStages = 3;
  static constexpr int kVStages = (kHD == 128 && kG == 2) ? 2 : 3;
  static constexpr int kThreads = 64 + 128 * kG;
  static constexpr uint32_t kOCol = 128 * kG;
  static constexpr uint32_t kTmemCols = (kG == 1) ? 256 : 512;
  static constexpr int kBars = 1 + 2 * kKStages + 2 * kVStages + 10 * kG;
  static constexpr size_t kSmem = 1024 + static_cast<size_t>(kG) * kQBytes +
                                  static_cast<size_t>(kKStages) * kKTileBytes +
                                  static_cast<size_t>(kVStages) * kVTileBytes +
                                  static_cast<size_t>(kG) * 2 * kPBytes + 8 * kBars + 16;
};

template <int kHD, int kG>
__global__ void __launch_bounds__(AttnShape<kHD, kG>::kThreads, 1)
    joint_attention_kernel(const __grid_constant__ AttnParams P) {
  using Sh = AttnShape<kHD, kG>;
  constexpr int kQBytes = Sh::kQBytes;
  constexpr int kKTileBytes = Sh::kKTileBytes;
  constexpr int kVTileBytes = Sh::kVTileBytes;
  constexpr int kKS = Sh::kKStages;
  constexpr int kVS = Sh::kVStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                               // kG Q tiles
  uint8_t* sK = sQ + kG * kQBytes;                  // kKS K tiles
  uint8_t* sV = sK + kKS * kKTileBytes;             // kVS V^T tiles
  uint8_t* sP = sV + kVS * kVTileBytes;             // kG x 2 x 16 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kG * 2 * kPBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + kKS;
  uint64_t* v_full = k_empty + kKS;
  uint64_t* v_empty = v_full + kVS;
  // per group: s_full[2], s_empty[2], p_full[2], p_empty[2], o_done (one phase per PV MMA),
  // o_final (one phase: the group's last PV MMA landed)
  uint64_t* gbar = v_empty + kVS;
  auto s_full = [&](int g) { return gbar + 10 * g; };
  auto s_empty = [&](int g) { return gbar + 10 * g + 2; };
  auto p_full = [&](int g) { return gbar + 10 * g + 4; };
  auto p_empty = [&](int g) { return gbar + 10 * g + 6; };
  auto o_done = [&](int g) { return gbar + 10 * g + 8; };
  auto o_final = [&](int g) { return gbar + 10 * g + 9; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbar + 10 * kG);

  const int q0 = blockIdx.x * (128 * kG);
  const int head = blockIdx.y;
  const int b = blockIdx.z;
  const int bh = b * P.H + head;
  const int kvh = P.kv_heads > 0 ? P.kv_heads : P.H;
  const int bh_kv = b * kvh + head / (P.H / kvh);  // GQA: K / V row of this query head
  const int L = P.L;
  // key tiles this CTA needs: all of them, or (causal) those a query row of the CTA can see:
  // keys j < (i / cb + 1) * cb for row i (cb = 1: j <= i)
  const int cb = P.causal_block > 1 ? P.causal_block : 1;
  const int last_row = min(L, q0 + 128 * kG) - 1;
  const int nkv = P.causal ? min((L + 63) / 64, (min(L, (last_row / cb + 1) * cb) - 1) / 64 + 1) : (L + 63) / 64;
  const int ng = (kG == 2 && q0 + 128 < L) ? 2 : 1;  // query tiles with rows inside L
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int g = 0; g < kG; ++g) {
      for (int i = 0; i < 2; ++i) {
        mbar_init(&s_full(g)[i], 1);
        mbar_init(&s_empty(g)[i], 4);
        mbar_init(&p_full(g)[i], 4);
        mbar_init(&p_empty(g)[i], 1);
      }
      mbar_init(o_done(g), 1);
      mbar_init(o_final(g), 1);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&P.tq);
    tma_prefetch_desc(&P.tk);
    tma_prefetch_desc(&P.tv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Sh::kTmemCols);
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
      mbar_arrive_expect_tx(q_full, ng * kQBytes);
      for (int g = 0; g < ng; ++g)
#pragma unroll
        for (int c = 0; c < Sh::kChunks; ++c)
          tma_load_3d(sQ + g * kQBytes + c * Sh::kQChunk, &P.tq, q_full, c * 64, q0 + 128 * g, bh, pol);
      // K(i) and V(i - 1) per step: K leads by one tile (S_{j+1} is issued before PV_j)
      for (int i = 0; i <= nkv; ++i) {
        if (i < nkv) {
          const int s = i % kKS;
          if (!mbar_wait(&k_empty[s], (static_cast<uint32_t>(i / kKS) & 1u) ^ 1u, kErrAttnTimeout + 1)) break;
          mbar_arrive_expect_tx(&k_full[s], kKTileBytes);
#pragma unroll
          for (int c = 0; c < Sh::kChunks; ++c)
            tma_load_3d(sK + s * kKTileBytes + c * Sh::kKChunk, &P.tk, &k_full[s], c * 64, i * 64, bh_kv, pol);
        }
        if (i >= 1) {
          const int j = i - 1;
          const int s = j % kVS;
          if (!mbar_wait(&v_empty[s], (static_cast<uint32_t>(j / kVS) & 1u) ^ 1u, kErrAttnTimeout + 1)) break;
          mbar_arrive_expect_tx(&v_full[s], kVTileBytes);
          tma_load_3d(sV + s * kVTileBytes, &P.tv, &v_full[s], j * 64, 0, bh_kv, pol);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(128, 64);
      const uint32_t idesc_pv = umma_idesc_bf16(128, kHD);
      bool ok = mbar_wait(q_full, 0, kErrAttnTimeout + 2);
      auto issue_s = [&](int j) -> bool {
        const int s = j % kKS;
        const int sb = j & 1;
        if (!mbar_wait(&k_full[s], static_cast<uint32_t>(j / kKS) & 1u, kErrAttnTimeout + 2))
          return false;
        const uint32_t k_addr = smem_u32(sK + s * kKTileBytes);
        for (int g = 0; g < ng; ++g) {
          if (!mbar_wait(&s_empty(g)[sb], (static_cast<uint32_t>(j >> 1) & 1u) ^ 1u, kErrAttnTimeout + 2))
            return false;
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sQ + g * kQBytes);
#pragma unroll
          for (int k = 0; k < 4 * Sh::kChunks; ++k)
            umma_f16(tmem + (2 * g + sb) * 64, umma_desc_sw128(q_addr + (k >> 2) * Sh::kQChunk + 32 * (k & 3)),
                     umma_desc_sw128(k_addr + (k >> 2) * Sh::kKChunk + 32 * (k & 3)), idesc, k != 0 ? 1u : 0u);
          umma_commit(&s_full(g)[sb]);
        }
        umma_commit(&k_empty[s]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nkv; ++j) {
        if (j + 1 < nkv) {
          ok = issue_s(j + 1);
          if (!ok) break;
        }
        const int pb = j & 1;
        const int s = j % kVS;
        if (!mbar_wait(&v_full[s], static_cast<uint32_t>(j / kVS) & 1u, kErrAttnTimeout + 2)) break;
        const uint32_t v_addr = smem_u32(sV + s * kVTileBytes);
        for (int g = 0; ok && g < ng; ++g) {
          if (!mbar_wait(&p_full(g)[pb], static_cast<uint32_t>(j >> 1) & 1u, kErrAttnTimeout + 2)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t p_addr = smem_u32(sP + (2 * g + pb) * kPBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + Sh::kOCol + g * kHD, umma_desc_sw128(p_addr + 32 * k),
                     umma_desc_sw128(v_addr + 32 * k), idesc_pv, (j | k) != 0 ? 1u : 0u);
          umma_commit(o_done(g));
          umma_commit(&p_empty(g)[pb]);
          if (j == nkv - 1) umma_commit(o_final(g));
        }
        if (ok) umma_commit(&v_empty[s]);
      }
    }
  } else {
    // ---------------- softmax warpgroups ----------------
    griddep_wait();
    const int g = (warp - 2) >> 2;
    const int quad = warp & 3;  // TMEM lane quadrant of this warp
    const int r = quad * 32 + lane;
    const int qrow = q0 + 128 * g + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t o_col = Sh::kOCol + g * kHD;
    const unsigned char* kmask = P.key_mask ? P.key_mask + static_cast<size_t>(b) * L : nullptr;
    const float scale = P.scale_log2;
    float m_ref = -INFINITY;  // reference max of the exponentials (log2 units)
    float l_run = 0.0f;
    bool ok = g < ng;

    for (int j = 0; ok && j < nkv; ++j) {
      const int sb = j & 1;
      const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
      // every exit is warp-uniform: the warp-collective TMEM loads / stores and the vote below
      // need all 32 lanes
      ok = mbar_wait(&s_full(g)[sb], ph, kErrAttnTimeout + 3);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      float sv[64];
      tmem_ld32(tmem + lane_off + (2 * g + sb) * 64, *reinterpret_cast<float(*)[32]>(&sv[0]));
      tmem_ld32(tmem + lane_off + (2 * g + sb) * 64 + 32, *reinterpret_cast<float(*)[32]>(&sv[32]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty(g)[sb]);

      // mask, row max of the raw scores (four independent chains; the scale is positive, so it
      // is applied to the max and folded into the exponent's fma).  Tiles wholly inside the
      // sequence without a key mask skip the masking; the key mask, when there is one, is read
      // as 64 bytes once per tile, so the per-element work stays branch-free.
      const int kbase = j * 64;
      // keys of this tile visible to this row: inside the sequence and, when causal, <= the row
      const int nvis = P.causal ? min(L, (qrow / cb + 1) * cb) - kbase : L - kbase;
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      // a tile below the diagonal for every row of the group needs no mask (warp-uniform test)
      const bool full_tile = L - kbase >= 64 && (!P.causal || kbase + 63 < ((q0 + 128 * g) / cb + 1) * cb);
      if (kmask == nullptr && full_tile) {
#pragma unroll
        for (int c = 0; c < 64; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], sv[c]);
      } else if (kmask == nullptr) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          sv[c] = (c < nvis) ? sv[c] : -INFINITY;
          mx4[c & 3] = fmaxf(mx4[c & 3], sv[c]);
        }
      } else {
        uint32_t mbits[2] = {0u, 0u};  // bit c: key kbase + c visible
#pragma unroll 1
        for (int c = 0; c < 64; ++c)
          if (c < nvis && kmask[kbase + c] != 0) mbits[c >> 5] |= 1u << (c & 31);
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          sv[c] = ((mbits[c >> 5] >> (c & 31)) & 1u) ? sv[c] : -INFINITY;
          mx4[c & 3] = fmaxf(mx4[c & 3], sv[c]);
        }
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * scale;

      // lazy rescale of O and l when this row's max outgrows the reference by 2^8
      const bool grow = mx > m_ref + kRescaleLog2;
      float alpha = 1.0f;
      if (grow) {
        alpha = (m_ref == -INFINITY) ? 0.0f : ex2_approx(m_ref - mx);
        m_ref = mx;
        l_run *= alpha;
      }
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // O holds PV_0..PV_{j-1}: wait for the last one, scale the rows that moved (S_j was
        // issued after PV_{j-2}, so o_done is at most one phase behind here)
        ok = mbar_wait(o_done(g), static_cast<uint32_t>(j - 1) & 1u, kErrAttnTimeout + 3);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < kHD / 32; ++h) {
          float o[32];
          tmem_ld32(tmem + lane_off + o_col + 32 * h, o);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] *= alpha;
          tmem_st32(tmem + lane_off + o_col + 32 * h, o);
        }
        tmem_wait_st();
      }
      const float m_use = (m_ref == -INFINITY) ? 0.0f : m_ref;
      float ps4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        sv[c] = ex2_approx(fmaf(sv[c], scale, -m_use));
        ps4[c & 3] += sv[c];
      }
      l_run += (ps4[0] + ps4[1]) + (ps4[2] + ps4[3]);

      // P_j -> shared memory (K-major, 128-byte swizzle: chunk c of row r at (c ^ (r & 7)) * 16)
      ok = mbar_wait(&p_empty(g)[sb], ph ^ 1u, kErrAttnTimeout + 3);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      uint8_t* prow = sP + (2 * g + sb) * kPBytes + r * 128;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint4 u;
        u.x = pack_bf16x2(sv[8 * cc + 0], sv[8 * cc + 1]);
        u.y = pack_bf16x2(sv[8 * cc + 2], sv[8 * cc + 3]);
        u.z = pack_bf16x2(sv[8 * cc + 4], sv[8 * cc + 5]);
        u.w = pack_bf16x2(sv[8 * cc + 6], sv[8 * cc + 7]);
        *reinterpret_cast<uint4*>(prow + ((cc ^ (r & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full(g)[sb]);
    }

    // O = (sum of PV) / l after the last PV MMA.  Its own one-phase barrier: at this point
    // o_done may be anywhere from two phases behind to complete, which a parity wait on it
    // cannot tell apart.
    if (ok && nkv > 0) ok = mbar_wait(o_final(g), 0u, kErrAttnTimeout + 3);
    if (__all_sync(0xffffffffu, ok) && nkv > 0) {
      tc_fence_after();
      int seg = 0, off = 0;
      while (seg + 1 < P.nseg && qrow >= off + P.seg_len[seg]) {
        off += P.seg_len[seg];
        ++seg;
      }
      const float inv_l = 1.0f / l_run;
      const int od = P.out_dim > 0 ? P.out_dim : kHD;  // dims of a head written out
      const int ld = P.seg_ld[seg] > 0 ? P.seg_ld[seg] : P.H * od;
      uint4* d4 = reinterpret_cast<uint4*>(
          P.seg_out[seg] + (static_cast<size_t>(b) * P.seg_len[seg] + (qrow - off)) * ld + head * od);
#pragma unroll
      for (int half = 0; half < kHD / 64; ++half) {  // 64 output dims at a time
        float o[64];
        tmem_ld32(tmem + lane_off + o_col + 64 * half, *reinterpret_cast<float(*)[32]>(&o[0]));
        tmem_ld32(tmem + lane_off + o_col + 64 * half + 32, *reinterpret_cast<float(*)[32]>(&o[32]));
        tmem_wait_ld();
        if (qrow < L) {
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            if (64 * half + 8 * cc >= od) break;
            uint4 u;
            u.x = pack_bf16x2(o[8 * cc + 0] * inv_l, o[8 * cc + 1] * inv_l);
            u.y = pack_bf16x2(o[8 * cc + 2] * inv_l, o[8 * cc + 3] * inv_l);
            u.z = pack_bf16x2(o[8 * cc + 4] * inv_l, o[8 * cc + 5] * inv_l);
            u.w = pack_bf16x2(o[8 * cc + 6] * inv_l, o[8 * cc + 7] * inv_l);
            d4[8 * half + cc] = u;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Sh::kTmemCols);
  }
}

namespace {
template <int kHD, int kG>
cudaError_t set_smem() {
  return cudaFuncSetAttribute(joint_attention_kernel<kHD, kG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(AttnShape<kHD, kG>::kSmem));
}

template <int kHD, int kG>
cudaError_t launch_variant(const AttnParams& p, cudaStream_t stream, bool pdl) {
  using Sh = AttnShape<kHD, kG>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.L + 128 * kG - 1) / (128 * kG), p.H, p.B);
  cfg.blockDim = dim3(Sh::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Sh::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, joint_attention_kernel<kHD, kG>, p);
}
}  // namespace

size_t attention_smem_bytes(int head_dim) {
  return head_dim == 128 ? AttnShape<128, 2>::kSmem : AttnShape<64, 2>::kSmem;
}

cudaError_t attention_prepare_device() {
  cudaError_t e = set_smem<64, 1>();
  if (e == cudaSuccess) e = set_smem<64, 2>();
  if (e == cudaSuccess) e = set_smem<128, 1>();
  if (e == cudaSuccess) e = set_smem<128, 2>();
  return e;
}

// One query tile per CTA unless two are asked for: measured on the head_dim-128 sweep
// (L 544-4128, batch 1-16) the two-warpgroup form is no faster yet (within 3%), and one tile
// per CTA gives the batch-1 MSAT step twice the CTAs.
int attention_tiles_per_cta(const AttnParams& p, int sms) {
  (void)sms;
  return p.tiles_per_cta == 2 ? 2 : 1;
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl) {
  const int hd = p.head_dim > 0 ? p.head_dim : 64;
  if (hd != 64 && hd != 128) return cudaErrorInvalidValue;
  const int g = attention_tiles_per_cta(p, sm_count());
  if (hd == 128) return g == 2 ? launch_variant<128, 2>(p, stream, pdl) : launch_variant<128, 1>(p, stream, pdl);
  return g == 2 ? launch_variant<64, 2>(p, stream, pdl) : launch_variant<64, 1>(p, stream, pdl);
}

}  // namespace rldx
