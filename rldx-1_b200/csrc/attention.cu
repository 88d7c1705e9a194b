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
//   S_j  = Q K_j^T          (M=128, N=kBN keys, K=d dims)   -> TMEM
//   O   += P_j V_j          (M=128, N=d dims, K=kBN keys)   -> one TMEM accumulator
// Q and K tiles are held as d/64 chunks of 64 dims (one 128-byte swizzle atom per row each).
// Each softmax warpgroup (four warps) owns one query tile, one row per thread, so row max / sum
// need no shuffles.
// P_j goes to TMEM as bf16 pairs (the PV MMA takes its A operand from tensor memory), or, for
// head_dim 128 with two query tiles, to shared memory in the 128-byte-swizzled K-major layout.  The
// running max is rescaled lazily: exponentials use a reference max that only moves when a
// row's max grows by more than 2^8 (P then stays <= 256, exact in the final O / l); only then
// is that row of O read from TMEM, scaled and written back, after the previous PV MMA landed.
#include "host_util.h"
#include "kernels.cuh"

namespace rldx {

constexpr float kRescaleLog2 = 8.0f;  // lazy-rescale threshold (log2 units)

// Of every four exponent pairs of a tile, this many are computed on the FMA pipe
// (exp2_fma_x2) and the rest by the special-function unit (16 results per cycle per SM: 1024
// cycles for a 128 x 128 tile).  Measured on the config-4 sweep: one in four +1.5-2.4 %, two
// in four no gain, three in four slower (the polynomial's instructions then cost more issue
// slots than the special-function unit saves).
#ifndef RLDX_ATTN_EXP_FMA
#define RLDX_ATTN_EXP_FMA 1
#endif
constexpr int kExpFmaPairs = RLDX_ATTN_EXP_FMA;

// 2^x for two values on the FMA pipe: n = round(x) through the 1.5 * 2^23 shift (exact for
// |x| < 2^22), 2^(x - n) by a degree-4 polynomial fitted to 2^f on [-1/2, 1/2] (weighted least
// squares on Chebyshev nodes, relative error below 3e-6 in fp32 evaluation), then n added to
// the exponent field; arguments below -126 (and -inf) give 0.
__device__ __forceinline__ float2 exp2_fma_x2(float2 x) {
  const float2 t = add_f32x2(x, make_float2(12582912.0f, 12582912.0f));
  const float2 n = add_f32x2(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = fma_f32x2(n, make_float2(-1.0f, -1.0f), x);
  float2 p = make_float2(0.009570094756782055f, 0.009570094756782055f);
  p = fma_f32x2(p, f, make_float2(0.05591786280274391f, 0.05591786280274391f));
  p = fma_f32x2(p, f, make_float2(0.240247443318367f, 0.240247443318367f));
  p = fma_f32x2(p, f, make_float2(0.6931217908859253f, 0.6931217908859253f));
  p = fma_f32x2(p, f, make_float2(0.9999992847442627f, 0.9999992847442627f));
  // the low bits of t hold n; shifted by 23 they add n to the exponent field of p
  const float ex = __int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23));
  const float ey = __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23));
  return make_float2(x.x >= -126.0f ? ex : 0.0f, x.y >= -126.0f ? ey : 0.0f);
}

// kG query tiles of 128 rows per CTA share every K / V tile: kG = 1 for latency (more CTAs),
// kG = 2 for throughput (two softmax warpgroups keep the special-function and ALU pipes busy
// while the tensor core works on the other tile, and K / V are read once per 256 queries).
// kW softmax warpgroups per query tile split each key tile's columns (kW = 2: half the keys per
// thread), so the exponentials of one tile take half as long (the short-sequence, batch-1 case
// is bound by that chain).  Each keeps its own reference max, row sum and O accumulator over
// its keys; the row maxima and sums meet through shared memory once, after the last tile.
// Key tile width kBN: the variants that run one CTA per SM (head_dim 128 with one query tile,
// head_dim 64 with the column split) take 128 keys per tile, so the S MMAs have N = 128 (an
// M = 128 MMA takes as long at N = 64 as at N = 128) and the softmax chain's fixed costs per tile
// (waits, TMEM load latency, barrier round trips) cover twice the keys.  Their softmax reads S
// into registers at the start of a tile, so one S buffer suffices (S_{j+1} is issued once
// softmax j has read S_j).  The other variants keep 64-key tiles and two S buffers.  K and V^T
// tiles of 128 keys arrive as two 64-key boxes each (the tensor maps' boxes stay 64 rows / keys).
// TMEM columns: S of group g, buffer b at (kNS g + b) kBN; O of group g at kG kNS kBN + g d.
template <int kHD, int kG, int kW = 1>
struct AttnShape {
  static constexpr int kBN = (kG == 1 && (kW == 2 || kHD == 128)) ? 128 : 64;  // keys per tile
  static constexpr int kNS = (kBN == 128) ? 1 : 2;   // S buffers per query tile
  static constexpr int kChunks = kHD / 64;           // 64-dim chunks of a Q / K row
  static constexpr int kQBytes = 128 * kHD * 2;      // 128 queries
  static constexpr int kQChunk = 128 * 128;          // one 64-dim chunk of a Q tile
  static constexpr int kKTileBytes = kBN * kHD * 2;  // kBN keys
  static constexpr int kKChunk = kBN * 128;          // one 64-dim chunk of a K tile
  static constexpr int kVTileBytes = kHD * kBN * 2;  // V^T: d rows x kBN keys
  static constexpr int kVChunk = kHD * 128;          // one 64-key chunk of a V^T tile
  // P lives in TMEM (the PV MMA reads its A operand from there: no shared-memory round trip, no
  // proxy fence) wherever two P buffers fit beside S and O: every variant but head_dim 128 with
  // two query tiles, which keeps P in shared memory
  static constexpr bool kPT = !(kHD == 128 && kG == 2);
  static constexpr int kPBytes = kPT ? 0 : 128 * kBN * 2;  // smem P: 128 rows x kBN keys, 64-key chunks
  static constexpr int kPChunk = 128 * 128;
  static constexpr int kPCols = kPT ? kBN / 2 : 0;         // TMEM columns of one P buffer (bf16 pairs)
  // separate K and V rings: K(j) is free once the S MMAs of tile j are done, V(j) once its PV
  // MMAs are, so the K loads run ahead of the PV work
  static constexpr int kKStages = 3;
  static constexpr int kVStages = (kHD == 128 && kG == 2) ? 2 : 3;
  static constexpr int kThreads = 64 + 128 * kG * kW;
  static constexpr int kCols = kBN / kW;  // keys of a tile per softmax thread
  static constexpr uint32_t kOCol = kG * kNS * kBN;
  // one O accumulator per column warpgroup: each keeps its own reference max, row sum and O over
  // its share of the keys, merged once at the end (no exchange of row maxima per tile)
  static constexpr uint32_t kPCol = kOCol + kG * kW * kHD;  // P buffers (2 per group) when kPT
  static constexpr uint32_t kTmemCols = (kPCol + 2 * kG * kPCols <= 256) ? 256 : 512;
  static constexpr int kBars = 1 + 2 * kKStages + 2 * kVStages + 14 * kG + 1;  // + drain
  static constexpr int kXchFloats = kG * (2 + 1) * kW * 128;  // per-tile maxima (2 buffers), sums
  static constexpr size_t kSmem = 1024 + static_cast<size_t>(kG) * kQBytes +
                                  static_cast<size_t>(kKStages) * kKTileBytes +
                                  static_cast<size_t>(kVStages) * kVTileBytes +
                                  static_cast<size_t>(kG) * 2 * kPBytes + 8 * kBars + 16 +
                                  4 * static_cast<size_t>(kXchFloats);
  static_assert(kSmem <= 232448, "shared memory of one CTA");
  static_assert(kPCol + 2 * kG * kPCols <= 512, "TMEM columns");
  static_assert(kW == 1 || kPT, "column split: P in TMEM");
};

template <int kHD, int kG, int kW>
__global__ void __launch_bounds__(AttnShape<kHD, kG, kW>::kThreads, 1)
    joint_attention_kernel(const __grid_constant__ AttnParams P) {
  using Sh = AttnShape<kHD, kG, kW>;
  static_assert(kW == 1 || (kW == 2 && kHD == 64 && kG == 1), "column split: head_dim 64, one tile");
  constexpr int kQBytes = Sh::kQBytes;
  constexpr int kKTileBytes = Sh::kKTileBytes;
  constexpr int kVTileBytes = Sh::kVTileBytes;
  constexpr int kPBytes = Sh::kPBytes;
  constexpr int kBN = Sh::kBN;
  constexpr int kNS = Sh::kNS;
  constexpr int kKS = Sh::kKStages;
  constexpr int kVS = Sh::kVStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                               // kG Q tiles
  uint8_t* sK = sQ + kG * kQBytes;                  // kKS K tiles
  uint8_t* sV = sK + kKS * kKTileBytes;             // kVS V^T tiles
  uint8_t* sP = sV + kVS * kVTileBytes;             // kG x 2 P tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kG * 2 * kPBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + kKS;
  uint64_t* v_full = k_empty + kKS;
  uint64_t* v_empty = v_full + kVS;
  // per group: s_full[2], s_empty[2], p_full[2], p_empty[2], o_done[2] (PV_j commits to
  // o_done[j & 1]), o_final (one phase: the group's last PV MMA landed), xch[2] (initialised
  // but no longer waited on: the column warpgroups keep their own row maxima), l_xch (their
  // reference maxima and row sums are in shared memory, once, after the last tile)
  uint64_t* gbar = v_empty + kVS;
  auto s_full = [&](int g) { return gbar + 14 * g; };
  auto s_empty = [&](int g) { return gbar + 14 * g + 2; };
  auto p_full = [&](int g) { return gbar + 14 * g + 4; };
  auto p_empty = [&](int g) { return gbar + 14 * g + 6; };
  auto o_done = [&](int g) { return gbar + 14 * g + 8; };
  auto o_final = [&](int g) { return gbar + 14 * g + 10; };
  auto xch = [&](int g) { return gbar + 14 * g + 11; };
  auto l_xch = [&](int g) { return gbar + 14 * g + 13; };
  uint64_t* drain = gbar + 14 * kG;  // failure path: the issued MMAs have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  // exchange floats: group g, buffer sb, warpgroup w, row r at xf[((g * 3 + sb) * kW + w) * 128 + r]
  // (sb = 2: the final row sums)
  float* xf = reinterpret_cast<float*>(tmem_slot + 4);

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
  const int nkv = P.causal ? min((L + kBN - 1) / kBN, (min(L, (last_row / cb + 1) * cb) - 1) / kBN + 1)
                           : (L + kBN - 1) / kBN;
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
        mbar_init(&s_empty(g)[i], 4 * kW);
        mbar_init(&p_full(g)[i], 4 * kW);
        mbar_init(&p_empty(g)[i], 1);
        mbar_init(&xch(g)[i], 4 * kW);
        mbar_init(&o_done(g)[i], 1);
      }
      mbar_init(o_final(g), 1);
      mbar_init(l_xch(g), 4 * kW);
    }
    mbar_init(drain, 1);
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
      // K(i) and V(i - kNS) per step: K leads by kNS tiles (S_{j+kNS} is issued before PV_j)
      bool ok = true;
      for (int i = 0; ok && i < nkv + kNS; ++i) {
        if (i < nkv) {
          const int s = i % kKS;
          if (!mbar_wait(&k_empty[s], (static_cast<uint32_t>(i / kKS) & 1u) ^ 1u, kErrAttnTimeout + 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[s], kKTileBytes);  // keys past L arrive zero-filled
#pragma unroll
          for (int hb = 0; hb < kBN / 64; ++hb)
#pragma unroll
            for (int c = 0; c < Sh::kChunks; ++c)
              tma_load_3d(sK + s * kKTileBytes + c * Sh::kKChunk + hb * 64 * 128, &P.tk, &k_full[s], c * 64,
                          i * kBN + hb * 64, bh_kv, pol);
        }
        if (i >= kNS && i - kNS < nkv) {
          const int j = i - kNS;
          const int s = j % kVS;
          if (!mbar_wait(&v_empty[s], (static_cast<uint32_t>(j / kVS) & 1u) ^ 1u, kErrAttnTimeout + 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[s], kVTileBytes);
#pragma unroll
          for (int hb = 0; hb < kBN / 64; ++hb)
            tma_load_3d(sV + s * kVTileBytes + hb * Sh::kVChunk, &P.tv, &v_full[s], j * kBN + hb * 64, 0, bh_kv, pol);
        }
      }
      if (!ok) settle_issued_copies();  // loads already issued land before the CTA exits
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(128, kBN);
      const uint32_t idesc_pv = umma_idesc_bf16(128, kHD);
      bool ok = mbar_wait(q_full, 0, kErrAttnTimeout + 2);
      auto issue_s = [&](int j) -> bool {
        const int s = j % kKS;
        const int sb = j % kNS;
        if (!mbar_wait(&k_full[s], static_cast<uint32_t>(j / kKS) & 1u, kErrAttnTimeout + 2))
          return false;
        const uint32_t k_addr = smem_u32(sK + s * kKTileBytes);
        for (int g = 0; g < ng; ++g) {
          if (!mbar_wait(&s_empty(g)[sb], (static_cast<uint32_t>(j / kNS) & 1u) ^ 1u, kErrAttnTimeout + 2))
            return false;
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sQ + g * kQBytes);
#pragma unroll
          for (int k = 0; k < 4 * Sh::kChunks; ++k)
            umma_f16(tmem + (kNS * g + sb) * kBN, umma_desc_sw128(q_addr + (k >> 2) * Sh::kQChunk + 32 * (k & 3)),
                     umma_desc_sw128(k_addr + (k >> 2) * Sh::kKChunk + 32 * (k & 3)), idesc, k != 0 ? 1u : 0u);
          umma_commit(&s_full(g)[sb]);
        }
        umma_commit(&k_empty[s]);
        return true;
      };
      // S runs kNS key tiles ahead of PV: S_{j+kNS} goes to the S buffer that softmax j has just
      // read into registers, before PV_j (which waits for P_j), so the scores of the next tile
      // are ready when its softmax turn comes
      for (int t = 0; ok && t < kNS && t < nkv; ++t) ok = issue_s(t);
      for (int j = 0; ok && j < nkv; ++j) {
        if (j + kNS < nkv) {
          ok = issue_s(j + kNS);
          if (!ok) break;
        }
        const int pb = j & 1;
        const int s = j % kVS;
        if (!mbar_wait(&v_full[s], static_cast<uint32_t>(j / kVS) & 1u, kErrAttnTimeout + 2)) {
          ok = false;
          break;
        }
        const uint32_t v_addr = smem_u32(sV + s * kVTileBytes);
        for (int g = 0; ok && g < ng; ++g) {
          if (!mbar_wait(&p_full(g)[pb], static_cast<uint32_t>(j >> 1) & 1u, kErrAttnTimeout + 2)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if constexpr (Sh::kPT) {  // P from TMEM: 16 keys = 8 columns per MMA
            const uint32_t p_tmem = tmem + Sh::kPCol + static_cast<uint32_t>((2 * g + pb) * Sh::kPCols);
#pragma unroll
            for (int k = 0; k < kBN / 16; ++k) {
              constexpr int kPerW = kBN / 16 / kW;  // MMAs over one column warpgroup's keys
              const int w = k / kPerW;
              umma_f16_ts(tmem + Sh::kOCol + (g * kW + w) * kHD, p_tmem + 8 * k,
                          umma_desc_sw128(v_addr + (k >> 2) * Sh::kVChunk + 32 * (k & 3)), idesc_pv,
                          (j > 0 || k % kPerW != 0) ? 1u : 0u);
            }
          } else {
            const uint32_t p_addr = smem_u32(sP + (2 * g + pb) * kPBytes);
#pragma unroll
            for (int k = 0; k < kBN / 16; ++k)  // 16 keys per MMA; 64-key chunks of P and V^T
              umma_f16(tmem + Sh::kOCol + g * kHD, umma_desc_sw128(p_addr + (k >> 2) * Sh::kPChunk + 32 * (k & 3)),
                       umma_desc_sw128(v_addr + (k >> 2) * Sh::kVChunk + 32 * (k & 3)), idesc_pv,
                       (j | k) != 0 ? 1u : 0u);
          }
          umma_commit(&o_done(g)[pb]);
          umma_commit(&p_empty(g)[pb]);
          if (j == nkv - 1) umma_commit(o_final(g));
        }
        if (ok) umma_commit(&v_empty[s]);
      }
      if (!ok) {  // the MMAs already issued finish before TMEM is released
        umma_commit(drain);
        mbar_wait_teardown(drain, 0u);
      }
    }
  } else {
    // ---------------- softmax warpgroups ----------------
    griddep_wait();
    const int g = (warp - 2) / (4 * kW);
    const int wsub = ((warp - 2) >> 2) % kW;  // column share: keys [c0, c0 + kCols) of each tile
    constexpr int kCols = Sh::kCols;
    const int c0 = wsub * kCols;
    const int quad = warp & 3;  // TMEM lane quadrant of this warp
    const int r = quad * 32 + lane;
    const int qrow = q0 + 128 * g + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t o_col = Sh::kOCol + (g * kW + wsub) * kHD;  // this warpgroup's O
    const unsigned char* kmask = P.key_mask ? P.key_mask + static_cast<size_t>(b) * L : nullptr;
    const float scale = P.scale_log2;
    float m_ref = -INFINITY;  // reference max of the exponentials (log2 units)
    float l_run = 0.0f;
    bool ok = g < ng;

    for (int j = 0; ok && j < nkv; ++j) {
      const int sb = j & 1;  // P buffer and exchange buffer of this tile
      const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
      const int ssb = j % kNS;  // S buffer
      // every exit is warp-uniform: the warp-collective TMEM loads / stores and the vote below
      // need all 32 lanes
      ok = mbar_wait(&s_full(g)[ssb], static_cast<uint32_t>(j / kNS) & 1u, kErrAttnTimeout + 3);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      float sv[kCols];
#pragma unroll
      for (int h = 0; h < kCols / 32; ++h)
        tmem_ld32(tmem + lane_off + (kNS * g + ssb) * kBN + c0 + 32 * h,
                  *reinterpret_cast<float(*)[32]>(&sv[32 * h]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty(g)[ssb]);

      // mask, row max of the raw scores (four independent chains; the scale is positive, so it
      // is applied to the max and folded into the exponent's fma).  Tiles wholly inside the
      // sequence without a key mask skip the masking; the key mask, when there is one, is read
      // as kBN bytes once per tile, so the per-element work stays branch-free.
      const int kbase = j * kBN;
      // keys of this thread's columns visible to this row: inside the sequence and, when causal,
      // <= the row
      const int nvis = (P.causal ? min(L, (qrow / cb + 1) * cb) - kbase : L - kbase) - c0;
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      // a tile below the diagonal for every row of the group needs no mask (warp-uniform test)
      const bool full_tile = L - kbase >= kBN && (!P.causal || kbase + kBN - 1 < ((q0 + 128 * g) / cb + 1) * cb);
      if (kmask == nullptr && full_tile) {
#pragma unroll
        for (int c = 0; c < kCols; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], sv[c]);
      } else if (kmask == nullptr) {
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
          sv[c] = (c < nvis) ? sv[c] : -INFINITY;
          mx4[c & 3] = fmaxf(mx4[c & 3], sv[c]);
        }
      } else {
        uint32_t mbits[kCols / 32] = {};  // bit c: key kbase + c0 + c visible
#pragma unroll 1
        for (int c = 0; c < kCols; ++c)
          if (c < nvis && kmask[kbase + c0 + c] != 0) mbits[c >> 5] |= 1u << (c & 31);
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
          sv[c] = ((mbits[c >> 5] >> (c & 31)) & 1u) ? sv[c] : -INFINITY;
          mx4[c & 3] = fmaxf(mx4[c & 3], sv[c]);
        }
      }
      // the maximum over this warpgroup's keys only: each column warpgroup keeps its own
      // reference max, row sum and O accumulator, merged after the last tile
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      mx *= scale;

      // lazy rescale of O and l when this row's max outgrows the reference by 2^8
      const bool grow = mx > m_ref + kRescaleLog2;
      float alpha = 1.0f;
      if (grow) {
        alpha = (m_ref == -INFINITY) ? 0.0f : ex2_approx(m_ref - mx);
        m_ref = mx;
        l_run *= alpha;
      }
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // O holds PV_0..PV_{j-1}: wait for the last one, scale the rows that moved.  S_j was
        // issued after PV_{j-kNS-1} (so after PV_{j-3}), whose commit went to the same barrier as
        // PV_{j-1}'s when kNS = 2; S_j has landed, so PV_{j-3} has too and the parity wait for
        // PV_{j-1} is unambiguous
        ok = mbar_wait(&o_done(g)[(j - 1) & 1], static_cast<uint32_t>((j - 1) >> 1) & 1u, kErrAttnTimeout + 3);
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
      // exponent arguments two at a time (packed fma), the row sum in four chains (column c adds
      // to chain c & 3, in column order) two chains per packed add
      const float2 sc2 = make_float2(scale, scale), nm2 = make_float2(-m_use, -m_use);
#pragma unroll
      for (int c = 0; c < kCols; c += 2) {
        const float2 t = fma_f32x2(make_float2(sv[c], sv[c + 1]), sc2, nm2);
        if (((c >> 1) & 3) < kExpFmaPairs) {
          const float2 e = exp2_fma_x2(t);
          sv[c] = e.x;
          sv[c + 1] = e.y;
        } else {
          sv[c] = ex2_approx(t.x);
          sv[c + 1] = ex2_approx(t.y);
        }
      }
      float2 ps01 = make_float2(0.0f, 0.0f), ps23 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int c = 0; c < kCols; c += 4) {
        ps01 = add_f32x2(ps01, make_float2(sv[c], sv[c + 1]));
        ps23 = add_f32x2(ps23, make_float2(sv[c + 2], sv[c + 3]));
      }
      l_run += (ps01.x + ps01.y) + (ps23.x + ps23.y);

      // P_j -> shared memory: 64-key chunks of [128 rows x 128 bytes], K-major, 128-byte swizzle
      // (16-byte group c of row r at (c ^ (r & 7)) * 16)
      ok = mbar_wait(&p_empty(g)[sb], ph ^ 1u, kErrAttnTimeout + 3);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      if constexpr (Sh::kPT) {  // P -> TMEM: column c of this row's share holds keys 2c, 2c + 1
        const uint32_t pcol = tmem + lane_off + Sh::kPCol + static_cast<uint32_t>((2 * g + sb) * Sh::kPCols + c0 / 2);
#pragma unroll
        for (int h = 0; h < kCols / 64; ++h) {
          float pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = __uint_as_float(pack_bf16x2(sv[64 * h + 2 * i], sv[64 * h + 2 * i + 1]));
          tmem_st32(pcol + 32 * h, pk);
        }
        tmem_wait_st();
      } else {
        uint8_t* prow = sP + (2 * g + sb) * kPBytes + r * 128;
#pragma unroll
        for (int cc = 0; cc < kCols / 8; ++cc) {
          uint4 u;
          u.x = pack_bf16x2(sv[8 * cc + 0], sv[8 * cc + 1]);
          u.y = pack_bf16x2(sv[8 * cc + 2], sv[8 * cc + 3]);
          u.z = pack_bf16x2(sv[8 * cc + 4], sv[8 * cc + 5]);
          u.w = pack_bf16x2(sv[8 * cc + 6], sv[8 * cc + 7]);
          const int grp = c0 / 8 + cc;  // 8-key group within the tile
          *reinterpret_cast<uint4*>(prow + (grp >> 3) * Sh::kPChunk + (((grp & 7) ^ (r & 7)) << 4)) = u;
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full(g)[sb]);
    }

    // O = (sum of PV) / l after the last PV MMA.  Its own one-phase barrier: at this point
    // o_done may be anywhere from two phases behind to complete, which a parity wait on it
    // cannot tell apart.
    if (ok && nkv > 0) ok = mbar_wait(o_final(g), 0u, kErrAttnTimeout + 3);
    // merge of the column warpgroups: O = sum_w O_w 2^(m_w - m) / sum_w l_w 2^(m_w - m) with m
    // the largest reference max (a warpgroup that saw no visible key contributes nothing)
    float wscale[kW];
    wscale[0] = 1.0f;
    if constexpr (kW > 1) {
      if (__all_sync(0xffffffffu, ok) && nkv > 0) {
        xf[((g * 3 + 0) * kW + wsub) * 128 + r] = m_ref;
        xf[((g * 3 + 2) * kW + wsub) * 128 + r] = l_run;
        __syncwarp();
        if (lane == 0) mbar_arrive(l_xch(g));
        ok = mbar_wait(l_xch(g), 0u, kErrAttnTimeout + 3);
        if (__all_sync(0xffffffffu, ok)) {
          float m = -INFINITY;
#pragma unroll
          for (int w = 0; w < kW; ++w) m = fmaxf(m, xf[((g * 3 + 0) * kW + w) * 128 + r]);
          l_run = 0.0f;
#pragma unroll
          for (int w = 0; w < kW; ++w) {
            const float mw = xf[((g * 3 + 0) * kW + w) * 128 + r];
            wscale[w] = (mw == -INFINITY) ? 0.0f : ex2_approx(mw - m);
            l_run += xf[((g * 3 + 2) * kW + w) * 128 + r] * wscale[w];
          }
        }
      }
    }
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
      // the column warpgroups split the output dims too: warpgroup w writes dims [w * 64 / kW, ...)
      constexpr int kODims = 64 / kW;
#pragma unroll
      for (int half = 0; half < kHD / 64; ++half) {  // 64 output dims at a time
        float o[kODims];
        const uint32_t ocol = Sh::kOCol + g * kW * kHD + 64 * half + wsub * kODims;
#pragma unroll
        for (int h = 0; h < kODims / 32; ++h)
          tmem_ld32(tmem + lane_off + ocol + 32 * h, *reinterpret_cast<float(*)[32]>(&o[32 * h]));
        tmem_wait_ld();
        if constexpr (kW > 1) {
#pragma unroll
          for (int c = 0; c < kODims; ++c) o[c] *= wscale[0];
#pragma unroll
          for (int w = 1; w < kW; ++w) {
            float o2[kODims];
#pragma unroll
            for (int h = 0; h < kODims / 32; ++h)
              tmem_ld32(tmem + lane_off + ocol + w * kHD + 32 * h, *reinterpret_cast<float(*)[32]>(&o2[32 * h]));
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < kODims; ++c) o[c] = fmaf(o2[c], wscale[w], o[c]);
          }
        }
        if (qrow < L) {
#pragma unroll
          for (int cc0 = 0; cc0 < kODims / 8; ++cc0) {
            const int cc = wsub * (kODims / 8) + cc0;  // 8-dim chunk of the 64 of this half
            if (64 * half + 8 * cc >= od) break;
            uint4 u;
            u.x = pack_bf16x2(o[8 * cc0 + 0] * inv_l, o[8 * cc0 + 1] * inv_l);
            u.y = pack_bf16x2(o[8 * cc0 + 2] * inv_l, o[8 * cc0 + 3] * inv_l);
            u.z = pack_bf16x2(o[8 * cc0 + 4] * inv_l, o[8 * cc0 + 5] * inv_l);
            u.w = pack_bf16x2(o[8 * cc0 + 6] * inv_l, o[8 * cc0 + 7] * inv_l);
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
template <int kHD, int kG, int kW = 1>
cudaError_t set_smem() {
  return cudaFuncSetAttribute(joint_attention_kernel<kHD, kG, kW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(AttnShape<kHD, kG, kW>::kSmem));
}

template <int kHD, int kG, int kW = 1>
cudaError_t launch_variant(const AttnParams& p, cudaStream_t stream, bool pdl) {
  using Sh = AttnShape<kHD, kG, kW>;
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
  return cudaLaunchKernelEx(&cfg, joint_attention_kernel<kHD, kG, kW>, p);
}
}  // namespace

size_t attention_smem_bytes(int head_dim) {
  return head_dim == 128 ? std::max(AttnShape<128, 1>::kSmem, AttnShape<128, 2>::kSmem)
                         : std::max(AttnShape<64, 1>::kSmem, std::max(AttnShape<64, 2>::kSmem, AttnShape<64, 1, 2>::kSmem));
}

cudaError_t attention_prepare_device() {
  cudaError_t e = set_smem<64, 1>();
  if (e == cudaSuccess) e = set_smem<64, 1, 2>();
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

// Two column warpgroups per query tile (head_dim 64) when the launch has no more query tiles
// than SMs: then every CTA sits alone on its SM and the softmax chain of its tiles is the
// critical path (the batch-1 control step: 5 tiles x 24 heads).  Larger launches keep one
// warpgroup per tile, which lets two CTAs share an SM.  RLDX_ATTN_COLS=1 turns the split off.
bool attention_column_split(const AttnParams& p, int sms) {
  static int off = [] {
    const char* e = std::getenv("RLDX_ATTN_COLS");
    return (e && e[0] == '1') ? 1 : 0;
  }();
  const long long tiles = static_cast<long long>((p.L + 127) / 128) * p.H * p.B;
  return off == 0 && tiles <= sms;
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl) {
  const int hd = p.head_dim > 0 ? p.head_dim : 64;
  if (hd != 64 && hd != 128) return cudaErrorInvalidValue;
  const int g = attention_tiles_per_cta(p, sm_count());
  if (hd == 128) return g == 2 ? launch_variant<128, 2>(p, stream, pdl) : launch_variant<128, 1>(p, stream, pdl);
  if (g == 2) return launch_variant<64, 2>(p, stream, pdl);
  return attention_column_split(p, sm_count()) ? launch_variant<64, 1, 2>(p, stream, pdl)
                                                : launch_variant<64, 1>(p, stream, pdl);
}

}  // namespace rldx
