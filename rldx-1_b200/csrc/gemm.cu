// Grouped persistent tcgen05 GEMM with fused row epilogues (see gemm.cuh for the CTA layout).
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
#include <type_traits>

#include "gemm.cuh"

namespace rldx {

namespace {

// Activation of one bias-finished bf16 value.  The exponential and the reciprocal use the fast
// hardware paths (a couple of fp32 ulps); the result is rounded to bf16 like the reference.
template <int kAct>
__device__ __forceinline__ float act_fn(float y) {
  if constexpr (kAct == kActRelu) {
    return fmaxf(y, 0.0f);
  } else if constexpr (kAct == kActSilu) {  // F.silu: one rounding
    return bf16r(__fdividef(y, 1.0f + __expf(-y)));
  } else if constexpr (kAct == kActSwish) {  // x * torch.sigmoid(x): sigmoid rounded, then product
    return bf16r(y * bf16r(__fdividef(1.0f, 1.0f + __expf(-y))));
  } else {
    return y;
  }
}

// Bias epilogue without branches: an absent bias reads as zeros (bf16(acc + 0) = bf16(acc)),
// the post-rounded form (torch.bmm then + b) rounds the product first.
__device__ __forceinline__ float finish_acc(float acc, float b, int bias_mode) {
  const float a = (bias_mode == kBiasPostRound) ? bf16r(acc) : acc;
  return bf16r(a + b);
}

__device__ __forceinline__ bool al16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float bf_at(const uint4& q, int i) {
  const uint32_t w = (i < 2) ? q.x : (i < 4) ? q.y : (i < 6) ? q.z : q.w;
  return (i & 1) ? bf_hi(w) : bf_lo(w);
}

// Output-row bookkeeping of one accumulator row (thread) of one M tile.
struct RowCtx {
  int row, r_local, bidx, t, out_row, cat;
  bool live;  // row exists and is not dropped
};

__device__ __forceinline__ RowCtx row_ctx(const GemmProblem& pr, int tm, int r_local) {
  const GemmEpilogue& ep = pr.ep;
  RowCtx c;
  c.r_local = r_local;
  c.row = tm * pr.m_step + r_local;
  c.bidx = 0;
  c.t = c.row;
  if (ep.rows_in > 0) {
    c.bidx = c.row / ep.rows_in;
    c.t = c.row - c.bidx * ep.rows_in;
  }
  const bool dropped = (ep.rows_in > 0) && (c.t < ep.row_skip);
  c.out_row = (ep.rows_in > 0) ? c.bidx * ep.rows_out + c.t - ep.row_skip : c.row;
  c.live = (r_local < pr.m_step) && (c.row < pr.M) && !dropped;
  c.cat = pr.cat_ids ? static_cast<int>(pr.cat_ids[tm]) : 0;
  return c;
}

// Accumulator sources of the epilogue: 8 fp32 columns of this thread's row.
//   TmemSrc  the unit's own TMEM accumulator (tcgen05.ld: every lane of the warp calls it).
//   PartSrc  the sum, in split order, of a K-split tile's fp32 partials in the workspace.
struct TmemSrc {
  uint32_t taddr;
  __device__ __forceinline__ void get8(int col, bool /*live*/, float (&v)[8]) const {
    __syncwarp();
    tmem_ld8(taddr + static_cast<uint32_t>(col), v);
    tmem_wait_ld();
  }
  // two 8-column groups under one wait
  __device__ __forceinline__ void get8x2(int c0, int c1, bool /*live*/, float (&v0)[8], float (&v1)[8]) const {
    __syncwarp();
    tmem_ld8(taddr + static_cast<uint32_t>(c0), v0);
    tmem_ld8(taddr + static_cast<uint32_t>(c1), v1);
    tmem_wait_ld();
  }
  __device__ __forceinline__ void get16(int col, bool /*live*/, float (&v)[16]) const {
    __syncwarp();
    tmem_ld16(taddr + static_cast<uint32_t>(col), v);
    tmem_wait_ld();
  }
};

// Partial tiles are stored column-major, [split][column][128 rows] per tile, so that the 32
// rows of a warp read and write 128 contiguous bytes per column.
struct PartSrc {
  const float* col0;  // split 0, column 0, this thread's row
  size_t split_stride;  // floats between splits (= 128 * BN)
  int nsplit;
  static constexpr int kSplitsInFlight = 4;  // splits whose loads are issued before adding
  // two groups: the loads of both (two splits at a time) are issued before their sums are formed,
  // so one L2 round trip serves 16 columns
  __device__ __forceinline__ void get8x2(int c0, int c1, bool live, float (&v0)[8], float (&v1)[8]) const {
#pragma unroll
    for (int i = 0; i < 8; ++i) v0[i] = v1[i] = 0.0f;
    if (!live) return;
    const float* b0 = col0 + static_cast<size_t>(c0) * 128;
    const float* b1 = col0 + static_cast<size_t>(c1) * 128;
#pragma unroll 1
    for (int s0 = 0; s0 < nsplit; s0 += 2) {
      float a0[2][8], a1[2][8];
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const bool on = s0 + t < nsplit;
          a0[t][i] = on ? __ldcg(b0 + (s0 + t) * split_stride + i * 128) : 0.0f;
          a1[t][i] = on ? __ldcg(b1 + (s0 + t) * split_stride + i * 128) : 0.0f;
        }
#pragma unroll
      for (int t = 0; t < 2; ++t)  // added in split order
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (s0 + t < nsplit) {
            v0[i] += a0[t][i];
            v1[i] += a1[t][i];
          }
    }
  }
  __device__ __forceinline__ void get16(int col, bool live, float (&v)[16]) const {
    float a[8], b[8];
    get8(col, live, a);
    get8(col + 8, live, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[i] = a[i];
      v[8 + i] = b[i];
    }
  }
  __device__ __forceinline__ void get8(int col, bool live, float (&v)[8]) const {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    if (!live) return;
    const float* base = col0 + static_cast<size_t>(col) * 128;
#pragma unroll 1
    for (int s0 = 0; s0 < nsplit; s0 += kSplitsInFlight) {
      float a[kSplitsInFlight][8];
#pragma unroll
      for (int t = 0; t < kSplitsInFlight; ++t)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          a[t][i] = (s0 + t < nsplit) ? __ldcg(base + (s0 + t) * split_stride + i * 128) : 0.0f;
#pragma unroll
      for (int t = 0; t < kSplitsInFlight; ++t)  // added in split order
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (s0 + t < nsplit) v[i] += a[t][i];
    }
  }
};

// 8 bf16 at p (n of them valid; one 16-byte load when full and aligned), or zeros when !on.
__device__ __forceinline__ uint4 load8q(const __nv_bfloat16* p, bool on, int n) {
  if (!on) return make_uint4(0, 0, 0, 0);
  if (n >= 8 && al16(p)) return *reinterpret_cast<const uint4*>(p);
  uint16_t h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = (i < n) ? __bfloat16_as_ushort(p[i]) : 0;
  return make_uint4(h[0] | (static_cast<uint32_t>(h[1]) << 16), h[2] | (static_cast<uint32_t>(h[3]) << 16),
                    h[4] | (static_cast<uint32_t>(h[5]) << 16), h[6] | (static_cast<uint32_t>(h[7]) << 16));
}

// 8 bf16-exact values to p (n of them valid).
__device__ __forceinline__ void store8q(__nv_bfloat16* p, int n, const float (&y)[8]) {
  if (n >= 8 && al16(p)) {
    uint4 u;
    u.x = pack_exact_bf16x2(y[0], y[1]);
    u.y = pack_exact_bf16x2(y[2], y[3]);
    u.z = pack_exact_bf16x2(y[4], y[5]);
    u.w = pack_exact_bf16x2(y[6], y[7]);
    *reinterpret_cast<uint4*>(p) = u;
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < n) p[i] = __ushort_as_bfloat16(static_cast<unsigned short>(__float_as_uint(y[i]) >> 16));
}

// Epilogue of one unit by one of the kEpiSets epilogue warp sets (every set holds the same 32
// rows of a TMEM lane quadrant; the sets split the columns).  The loop bodies are small
// (8 columns per iteration) so the code stays resident in the instruction caches.
template <int kMode, int kAct, class Src>
__device__ __forceinline__ void unit_epilogue(const GemmProblem& pr, const RowCtx& rc, int n_base,
                                              int set, const Src& src) {
  const GemmEpilogue& ep = pr.ep;
  const int bn = pr.bn;
  const __nv_bfloat16* bias_row =
      ep.bias ? ep.bias + static_cast<size_t>(rc.cat) * ep.bias_cat_stride : nullptr;
  const int bias_mode = ep.bias_mode;

  if constexpr (kMode == kEpiStore || kMode == kEpiEuler) {
    __nv_bfloat16* orow = ep.out + static_cast<size_t>(rc.out_row) * ep.ldo + ep.col_off;
    const __nv_bfloat16* arow = nullptr;
    if (ep.add) {
      const int r = ep.add_row_mod > 0 ? (rc.t % ep.add_row_mod) : rc.row;
      arow = ep.add + static_cast<size_t>(r) * ep.ld_add;
    }
    const float dt = ep.dt;
    // set s takes the 8-column groups s, s + kEpiSets, ...; the operand loads of the next group
    // are issued before the current group is computed (one group of software pipelining)
    auto next_col = [](int col) { return col + 8 * kEpiSets; };
    auto fetch = [&](int col, uint4& bq, uint4& aq, uint4& xq) {
      const int n0 = n_base + col;
      const int n = pr.N - n0;
      const bool on = rc.live && n > 0 && col < bn;
      bq = load8q(bias_row + n0, on && bias_row, n);
      aq = load8q(arow + n0, on && arow, n);
      xq = load8q(orow + n0, on && kMode == kEpiEuler, n);
    };
    uint4 nb, na, nx;
    fetch(set * 8, nb, na, nx);
    // Plain store (no activation, bias added before the one rounding): two fp32 adds, one paired
    // round-to-bf16 and, with a residual, one exactly rounded bf16x2 add per two columns -- the
    // same roundings as the general path below, in a third of the instructions.
    const bool packed = (kMode == kEpiStore) && (kAct == kActNone) && bias_mode != kBiasPostRound &&
                        ((ep.ldo | ep.col_off | ep.ld_add) & 7) == 0 && al16(ep.out) &&
                        (!ep.add || al16(ep.add)) && (!bias_row || al16(bias_row));
    if constexpr (std::is_same<Src, PartSrc>::value) {
      // the last unit of a K-split tile: two column groups per L2 round trip for the partials,
      // their bias / residual loads issued in the same round
#pragma unroll 1
      for (int col = set * 8; col < bn; col += 16 * kEpiSets) {
        const int colb = min(col + 8 * kEpiSets, bn - 8);
        const bool second = col + 8 * kEpiSets < bn;
        uint4 b0, a0, x0, b1, a1, x1;
        fetch(col, b0, a0, x0);
        fetch(second ? col + 8 * kEpiSets : bn, b1, a1, x1);
        float v[2][8];
        src.get8x2(col, colb, rc.live, v[0], v[1]);
        if (!rc.live) continue;
        const uint4 bb[2] = {b0, b1}, aa[2] = {a0, a1}, xx[2] = {x0, x1};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c = col + h * 8 * kEpiSets;
          const int n0 = n_base + c;
          const int n = pr.N - n0;
          if ((h == 1 && !second) || n <= 0) continue;
          float y[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float t = act_fn<kAct>(finish_acc(v[h][i], bf_at(bb[h], i), bias_mode));
            t = bf16r(t + bf_at(aa[h], i));
            if constexpr (kMode == kEpiEuler) t = bf16r(bf_at(xx[h], i) + bf16r(dt * t));
            y[i] = t;
          }
          store8q(orow + n0, n, y);
        }
      }
      return;
    }
    if (packed) {
#pragma unroll 1
      for (int col = set * 8; col < bn; col = next_col(col)) {
        const int n0 = n_base + col;
        const int n = pr.N - n0;
        const uint4 bq = nb, aq = na;
        fetch(next_col(col), nb, na, nx);
        float v[8];
        src.get8(col, rc.live, v);
        if (!rc.live || n <= 0) continue;
        if (n < 8) {
          float y[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = bf16r(bf16r(v[i] + bf_at(bq, i)) + bf_at(aq, i));
          store8q(orow + n0, n, y);
          continue;
        }
        const uint32_t bw[4] = {bq.x, bq.y, bq.z, bq.w};
        const uint32_t aw[4] = {aq.x, aq.y, aq.z, aq.w};
        uint32_t h[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          __nv_bfloat162 t = __floats2bfloat162_rn(v[2 * p] + bf_lo(bw[p]), v[2 * p + 1] + bf_hi(bw[p]));
          if (arow) t = __hadd2_rn(t, *reinterpret_cast<const __nv_bfloat162*>(&aw[p]));
          h[p] = *reinterpret_cast<const uint32_t*>(&t);
        }
        *reinterpret_cast<uint4*>(orow + n0) = make_uint4(h[0], h[1], h[2], h[3]);
      }
      return;
    }
#pragma unroll 1
    for (int col = set * 8; col < bn; col = next_col(col)) {
      const int n0 = n_base + col;
      const int n = pr.N - n0;  // valid columns from n0 (uniform over the warp)
      const bool on = rc.live && n > 0;
      const uint4 bq = nb, aq = na, xq = nx;
      fetch(next_col(col), nb, na, nx);
      float v[8];
      src.get8(col, rc.live, v);
      if (!on) continue;
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float t = act_fn<kAct>(finish_acc(v[i], bf_at(bq, i), bias_mode));
        t = bf16r(t + bf_at(aq, i));  // an absent add reads as zeros: exact no-op
        if constexpr (kMode == kEpiEuler) t = bf16r(bf_at(xq, i) + bf16r(dt * t));
        y[i] = t;
      }
      store8q(orow + n0, n, y);
    }
  } else if constexpr (kMode == kEpiSwiGLU) {
    // every 64 columns: [0,32) gate, [32,64) up of hidden units n0/2 .. n0/2+31 (N % 64 == 0);
    // set s takes the 8-unit groups j = s, s + kEpiSets, ... (j < 4) of each chunk
    // The bias words of the next group are loaded while the current one is computed; the gate
    // and up columns come from TMEM under one wait; silu(g) and u are bf16-exact, so their
    // product rounds once in packed bf16x2 arithmetic exactly as bf16(float(s) * float(u)).
    __nv_bfloat16* orow = ep.out + static_cast<size_t>(rc.out_row) * ep.ldo + ep.col_off;
    auto bias_of = [&](int c, int j, uint4& bg, uint4& bu) {
      const int n0 = n_base + c;
      const bool on = rc.live && c < bn && n0 < pr.N && bias_row;
      bg = load8q(bias_row + n0 + 8 * j, on, 8);
      bu = load8q(bias_row + n0 + 32 + 8 * j, on, 8);
    };
    int c = 0, j = set;
    uint4 nbg, nbu;
    bias_of(c, j, nbg, nbu);
#pragma unroll 1
    while (c < bn) {
      const uint4 bg = nbg, bu = nbu;
      int c2 = c, j2 = j + kEpiSets;
      if (j2 >= 4) {
        j2 = set;
        c2 = c + 64;
      }
      bias_of(c2, j2, nbg, nbu);
      const int n0 = n_base + c;
      float g[8], u[8];
      src.get8x2(c + 8 * j, c + 32 + 8 * j, rc.live, g, u);
      if (rc.live && n0 < pr.N) {
        const uint32_t gw[4] = {bg.x, bg.y, bg.z, bg.w};
        const uint32_t uw[4] = {bu.x, bu.y, bu.z, bu.w};
        uint32_t hw[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float a0 = finish_acc(g[2 * p], bf_lo(gw[p]), bias_mode);
          const float a1 = finish_acc(g[2 * p + 1], bf_hi(gw[p]), bias_mode);
          const float b0 = finish_acc(u[2 * p], bf_lo(uw[p]), bias_mode);
          const float b1 = finish_acc(u[2 * p + 1], bf_hi(uw[p]), bias_mode);
          const uint32_t sw = pack_exact_bf16x2(act_fn<kActSilu>(a0), act_fn<kActSilu>(a1));
          const uint32_t bw = pack_exact_bf16x2(b0, b1);
          const __nv_bfloat162 h = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162*>(&sw),
                                              *reinterpret_cast<const __nv_bfloat162*>(&bw));
          hw[p] = *reinterpret_cast<const uint32_t*>(&h);
        }
        __nv_bfloat16* dst = orow + n0 / 2 + 8 * j;
        if (al16(dst)) {
          *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        } else {
          float h[8];
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            h[2 * p] = bf_lo(hw[p]);
            h[2 * p + 1] = bf_hi(hw[p]);
          }
          store8q(dst, 8, h);
        }
      }
      c = c2;
      j = j2;
    }
  } else {  // kEpiQKV: every 64 columns = one head of q, k or v; set s takes heads s, s+kEpiSets, ...
    const int inner = ep.H * 64;
    const int tok = ep.tok_off + rc.t;
    // rows whose RoPE is the identity (cos 1, sin 0) read no tables: their per-row table loads
    // are the epilogue's L1 misses (bias and norm weights are shared by every row)
    const bool rope = !ep.rope_identity;
#pragma unroll 1
    for (int c = 64 * set; c < bn; c += 64 * kEpiSets) {
      const int n0 = n_base + c;
      if (n0 >= pr.N) break;  // uniform over the warp
      const int part = n0 / inner;
      const int head = (n0 - part * inner) / 64;
      const size_t bh = static_cast<size_t>(rc.bidx) * ep.H + head;
      const __nv_bfloat16* hb = bias_row ? bias_row + n0 : nullptr;
      if (part < 2) {
        const __nv_bfloat16* w = (part == 0) ? ep.qn_w : ep.kn_w;
        const float4* cp = reinterpret_cast<const float4*>(ep.rope_cos + static_cast<size_t>(tok) * 32);
        const float4* sp = reinterpret_cast<const float4*>(ep.rope_sin + static_cast<size_t>(tok) * 32);
        const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
        // operands of pass 2's first group: in flight during pass 1
        uint4 nw = load8q(w, rc.live, 8);
        const float4 one4 = make_float4(1.f, 1.f, 1.f, 1.f);
        float4 nc = (rc.live && rope) ? cp[0] : one4, ns = (rc.live && rope) ? sp[0] : z4;
        float ss = 0.0f;
        uint4 nb = load8q(hb, rc.live && hb, 8);
        uint4 nb2 = load8q(hb + 8, rc.live && hb, 8);
#pragma unroll 1
        for (int g = 0; g < 64; g += 16) {  // pass 1: sum of squares of the finished head
          const uint4 bq = nb, bq2 = nb2;
          nb = load8q(hb + ((g + 16) & 63), rc.live && hb, 8);  // wraps to pass 2's first group
          nb2 = load8q(hb + ((g + 24) & 63), rc.live && hb && g + 16 < 64, 8);
          float v[16];
          src.get16(c + g, rc.live, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) {  // columns in order: the same fp32 sum as one at a time
            const float y = finish_acc(v[i], bf_at(i < 8 ? bq : bq2, i & 7), kBiasFused);
            ss += y * y;
          }
        }
        const float rstd = rsqrtf(ss * (1.0f / 64.0f) + ep.eps);
        __nv_bfloat16* dst = ((part == 0) ? ep.q : ep.k) + (bh * ep.L + tok) * 64;
#pragma unroll 1
        for (int g = 0; g < 64; g += 8) {  // pass 2: RMSNorm (weight then cast) + pair RoPE
          const uint4 bq = nb, wq = nw;
          const float4 c4 = nc, s4 = ns;
          const bool more = rc.live && g + 8 < 64;
          nb = load8q(hb + g + 8, more && hb, 8);
          nw = load8q(w + g + 8, more, 8);
          nc = (more && rope) ? cp[g / 8 + 1] : one4;
          ns = (more && rope) ? sp[g / 8 + 1] : z4;
          float v[8];
          src.get8(c + g, rc.live, v);
          if (!rc.live) continue;
          const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
          const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
          float y[8];
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const float x0 = finish_acc(v[2 * p], bf_at(bq, 2 * p), kBiasFused);
            const float x1 = finish_acc(v[2 * p + 1], bf_at(bq, 2 * p + 1), kBiasFused);
            const float a = bf16r(bf_at(wq, 2 * p) * (x0 * rstd));
            const float b = bf16r(bf_at(wq, 2 * p + 1) * (x1 * rstd));
            if (rope) {
              y[2 * p] = bf16r(a * cc[p] - b * sv[p]);
              y[2 * p + 1] = bf16r(a * sv[p] + b * cc[p]);
            } else {  // cos 1, sin 0: the rotation returns a and b (bf16 already)
              y[2 * p] = a;
              y[2 * p + 1] = b;
            }
          }
          store8q(dst + g, 8, y);
        }
      } else {
        __nv_bfloat16* dst = ep.vt + bh * 64 * ep.Lp + tok;
#pragma unroll 1
        for (int g = 0; g < 64; g += 8) {
          const uint4 bq = load8q(hb + g, rc.live && hb, 8);
          float v[8];
          src.get8(c + g, rc.live, v);
          if (!rc.live) continue;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float y = finish_acc(v[i], bf_at(bq, i), kBiasFused);
            dst[static_cast<size_t>(g + i) * ep.Lp] =
                __ushort_as_bfloat16(static_cast<unsigned short>(__float_as_uint(y) >> 16));
          }
        }
      }
    }
  }
}

// Dispatch of the activation (uniform per problem) outside the per-element loops.
template <int kMode, class Src>
__device__ __forceinline__ void unit_epilogue_act(const GemmProblem& pr, const RowCtx& rc,
                                                  int n_base, int set, const Src& src) {
  if constexpr (kMode == kEpiStore || kMode == kEpiEuler) {
    switch (pr.ep.act) {
      case kActRelu:
        unit_epilogue<kMode, kActRelu>(pr, rc, n_base, set, src);
        return;
      case kActSilu:
        unit_epilogue<kMode, kActSilu>(pr, rc, n_base, set, src);
        return;
      case kActSwish:
        unit_epilogue<kMode, kActSwish>(pr, rc, n_base, set, src);
        return;
      default:
        unit_epilogue<kMode, kActNone>(pr, rc, n_base, set, src);
        return;
    }
  } else {
    unit_epilogue<kMode, kActNone>(pr, rc, n_base, set, src);
  }
}

// Unit `i` of this CTA's list (host LPT schedule or plain striding).
__device__ __forceinline__ int cta_units(const GemmParams& P, int& first) {
  const int cta = blockIdx.x;
  if (P.explicit_sched) {
    first = P.cta_begin[cta];
    return P.cta_begin[cta + 1] - first;
  }
  first = 0;
  return (P.nunits - cta + P.ncta - 1) / P.ncta;
}

__device__ __forceinline__ int unit_id(const GemmParams& P, int first, int i) {
  return P.explicit_sched ? static_cast<int>(P.sched[first + i]) : blockIdx.x + i * P.ncta;
}

struct UnitInfo {
  int pi, tile, tm, tn, ks, c_begin, c_end, nslots;
};

__device__ __forceinline__ UnitInfo decode_unit(const GemmParams& P, int u) {
  UnitInfo d;
  d.pi = 0;
#pragma unroll
  for (int i = 1; i < kMaxProblems; ++i)
    if (i < P.nprob && u >= P.p[i].unit_begin) d.pi = i;
  const GemmProblem& pr = P.p[d.pi];
  const int local = u - pr.unit_begin;
  d.ks = local % pr.nsplit;
  d.tile = local / pr.nsplit;
  d.tm = d.tile % pr.tiles_m;
  d.tn = d.tile / pr.tiles_m;
  d.c_begin = d.ks * pr.split_chunks;
  d.c_end = min(pr.nchunks, d.c_begin + pr.split_chunks);
  d.nslots = (d.c_end - d.c_begin + pr.ksub - 1) / pr.ksub;
  return d;
}

}  // namespace

// kSplit: whether any problem of the launch is split along K.  Launches without splits use the
// instantiation without the reduction code, which keeps the hot loops compact.
template <int kMode, bool kSplit>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_bf16_kernel(const __grid_constant__ GemmParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int S = P.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * P.slot_bytes + kRingSlack);
  uint64_t* empty = full + kMaxStages;
  uint64_t* acc_full = empty + kMaxStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;  // failure path: the issued MMAs have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  uint32_t* bcast = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int first = 0;
  const int nunits = cta_units(P, first);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 2);  // A producer + B producer
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < P.nprob; ++i) tma_prefetch_desc(&P.p[i].ta);
  }
  if (warp == 2 && lane == 0) {
    for (int i = 0; i < P.nprob; ++i) tma_prefetch_desc(&P.p[i].tb);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * kAccCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // TMEM is held from here on: only now may dependent grids be scheduled next to this CTA.
  if (threadIdx.x == 0) griddep_launch();

  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers: warp 0 = A (activations), warp 2 = B (weights) ----------
    if (lane == 0) {
      const bool is_a = (warp == 0);
      if (is_a) griddep_wait();  // activations come from the previous kernel; weights do not
      const uint64_t pol_keep = l2_policy_evict_last();
      const uint64_t pol_once = l2_policy_evict_first();
      int it = 0;
      bool ok = true;
      for (int i = 0; ok && i < nunits; ++i) {
        const UnitInfo u = decode_unit(P, unit_id(P, first, i));
        const GemmProblem& pr = P.p[u.pi];
        const uint32_t a_sub = static_cast<uint32_t>(pr.a_rows) * 128u;
        const uint32_t b_sub = static_cast<uint32_t>(pr.bn) * 128u;
        const uint32_t bytes = (is_a ? a_sub : b_sub) * static_cast<uint32_t>(pr.ksub);
        const int a_row0 = u.tm * pr.m_step;
        const int n0 = u.tn * pr.bn;
        const int cat = pr.cat_ids ? static_cast<int>(pr.cat_ids[u.tm]) : 0;
        const uint64_t pol = is_a ? pol_keep : ((pr.tiles_m == 1 && !pr.cat_ids) ? pol_once : pol_keep);
        for (int sl = 0; sl < u.nslots; ++sl, ++it) {
          const int s = it % S;
          const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, kErrGemmTimeout + 1)) {
            ok = false;
            break;
          }
          uint8_t* slot = smem + s * P.slot_bytes;
          const int chunk = u.c_begin + sl * pr.ksub;
          mbar_arrive_expect_tx(&full[s], bytes);
          if (is_a) {
            if (pr.kdim3)
              tma_load_3d(slot, &pr.ta, &full[s], 0, a_row0, chunk, pol);
            else
              tma_load_2d(slot, &pr.ta, &full[s], chunk * 64, a_row0, pol);
          } else {
            uint8_t* dst = slot + a_sub * pr.ksub;
            if (pr.kdim3) {
              if (pr.cat_ids)
                tma_load_4d(dst, &pr.tb, &full[s], 0, n0, chunk, cat, pol);
              else
                tma_load_3d(dst, &pr.tb, &full[s], 0, n0, chunk, pol);
            } else {
              if (pr.cat_ids)
                tma_load_3d(dst, &pr.tb, &full[s], chunk * 64, n0, cat, pol);
              else
                tma_load_2d(dst, &pr.tb, &full[s], chunk * 64, n0, pol);
            }
          }
        }
      }
      if (!ok) settle_issued_copies();  // loads already issued land before the CTA exits
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int j = 0; ok && j < nunits; ++j) {
        const UnitInfo u = decode_unit(P, unit_id(P, first, j));
        const GemmProblem& pr = P.p[u.pi];
        const int ab = j & 1;
        if (!mbar_wait(&acc_empty[ab], (static_cast<uint32_t>(j >> 1) & 1u) ^ 1u, kErrGemmTimeout + 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * kAccCols);
        const uint32_t idesc = umma_idesc_bf16(128, pr.bn);
        const uint32_t a_sub = static_cast<uint32_t>(pr.a_rows) * 128u;
        const uint32_t b_sub = static_cast<uint32_t>(pr.bn) * 128u;
        for (int sl = 0; sl < u.nslots; ++sl, ++it) {
          const int s = it % S;
          const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
          if (!mbar_wait(&full[s], ph, kErrGemmTimeout + 2)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * P.slot_bytes);
          const uint32_t b_addr = a_addr + a_sub * static_cast<uint32_t>(pr.ksub);
          const int nsub = min(pr.ksub, u.c_end - (u.c_begin + sl * pr.ksub));
          for (int sub = 0; sub < nsub; ++sub) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              umma_f16(d_tmem, umma_desc_sw128(a_addr + sub * a_sub + 32 * k),
                       umma_desc_sw128(b_addr + sub * b_sub + 32 * k), idesc,
                       (sl | sub | k) != 0 ? 1u : 0u);
            }
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[ab]);
      }
      if (!ok) {  // the MMAs already issued finish before TMEM is released
        umma_commit(drain);
        mbar_wait_teardown(drain, 0u);
      }
    }
  } else {
    // ---------------- epilogue warps ----------------
    griddep_wait();
    const int quad = warp & 3;           // TMEM lane quadrant this warp may read
    const int set = (warp - kEpiWarp0) >> 2;  // column share of the unit (0 .. kEpiSets-1)
    const int r_local = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    // After a failed wait the warps keep walking the unit list (every wait then returns at
    // once) so that all of them still meet at the named barriers of the K-split units.
    bool ok = true;
    for (int j = 0; j < nunits; ++j) {
      const UnitInfo u = decode_unit(P, unit_id(P, first, j));
      const GemmProblem& pr = P.p[u.pi];
      const int ab = j & 1;
      if (ok && !mbar_wait(&acc_full[ab], static_cast<uint32_t>(j >> 1) & 1u, kErrGemmTimeout + 3))
        ok = false;
      tc_fence_after();
      const uint32_t tacc = tmem_base + lane_off + static_cast<uint32_t>(ab * kAccCols);
      const RowCtx rc = row_ctx(pr, u.tm, r_local);
      const int n_base = u.tn * pr.bn;
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[ab]);
      };

      if (!kSplit || pr.nsplit == 1) {
        if (!ok) continue;
        unit_epilogue_act<kMode>(pr, rc, n_base, set, TmemSrc{tacc});
        release();
        continue;
      }
      if constexpr (kSplit) {

      // K split: write this unit's fp32 partial tile, count arrivals, the last one reduces.
      const size_t split_stride = static_cast<size_t>(128) * pr.bn;
      float* col0 = P.ws + pr.ws_off + static_cast<size_t>(u.tile) * pr.nsplit * split_stride +
                    static_cast<size_t>(r_local);
      if (ok) {
        const TmemSrc src{tacc};
#pragma unroll 1
        for (int col = set * 8; col < pr.bn; col += 8 * kEpiSets) {
          float v[8];
          src.get8(col, rc.live, v);
          if (rc.live && n_base + col < pr.N) {
            float* dst = col0 + u.ks * split_stride + static_cast<size_t>(col) * 128;
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i * 128] = v[i];
          }
        }
        release();
      }
      __threadfence();
      named_bar_sync(1, kEpiWarps * 32);
      if (threadIdx.x == kEpiWarp0 * 32) {
        unsigned int* cnt = P.counters + pr.cnt_off + u.tile;
        const unsigned int prev = atomicAdd(cnt, 1u);
        const bool last = (prev == static_cast<unsigned int>(pr.nsplit - 1));
        if (last) *cnt = 0u;  // every split of this tile has arrived: ready for the next launch
        *bcast = last ? 1u : 0u;
      }
      named_bar_sync(1, kEpiWarps * 32);
      const bool last = (*reinterpret_cast<volatile uint32_t*>(bcast) != 0u);
      named_bar_sync(1, kEpiWarps * 32);  // bcast is rewritten by the next split unit
      if (!last || !ok) continue;
      __threadfence();
      unit_epilogue_act<kMode>(pr, rc, n_base, set, PartSrc{col0, split_stride, pr.nsplit});
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kAccCols);
  }
}

// ---------------------------------------------------------------------------------------------
// CTA-pair kernel: clusters of 2 CTAs, cta_group::2 MMAs over 256-row M tiles.
//
// Barriers live in both CTAs at the same offsets; which ones are used:
//   full[s]       rank 0 only: its two producers arrive with the bytes of BOTH CTAs' loads
//                 (expect_tx of 2x their own), and the TMA loads of both CTAs complete on it;
//   empty[s]      each CTA's own: the MMA thread commits to both CTAs' barriers after stage s;
//   acc_full[ab]  each CTA's own: committed to both after the unit's last MMA;
//   acc_empty[ab] rank 0 only: every epilogue warp of both CTAs arrives (2 x kEpiWarps).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ int pair_units(const GemmParams& P, int pair, int& first) {
  const int npairs = P.ncta >> 1;
  if (P.explicit_sched) {
    first = P.cta_begin[pair];
    return P.cta_begin[pair + 1] - first;
  }
  first = 0;
  return (P.nunits - pair + npairs - 1) / npairs;
}

__device__ __forceinline__ int pair_unit_id(const GemmParams& P, int pair, int first, int i) {
  return P.explicit_sched ? static_cast<int>(P.sched[first + i]) : pair + i * (P.ncta >> 1);
}

template <int kMode>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_pair_kernel(const __grid_constant__ GemmParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int S = P.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * P.slot_bytes + kRingSlack);
  uint64_t* empty = full + kMaxStages;
  uint64_t* acc_full = empty + kMaxStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;  // failure path (rank 0): the issued pair MMAs have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  int first = 0;
  const int nunits = pair_units(P, pair, first);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 2);  // rank 0's A producer + B producer
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 2 * kEpiWarps);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < P.nprob; ++i) tma_prefetch_desc(&P.p[i].ta);
  }
  if (warp == 2 && lane == 0) {
    for (int i = 0; i < P.nprob; ++i) tma_prefetch_desc(&P.p[i].tb);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, 2 * kAccCols);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any pair traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) griddep_launch();

  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers: warp 0 = A (this CTA's 128 rows), warp 2 = B (half) -----
    if (lane == 0) {
      const bool is_a = (warp == 0);
      if (is_a) griddep_wait();
      const uint64_t pol = l2_policy_evict_last();
      int it = 0;
      bool ok = true;
      for (int i = 0; ok && i < nunits; ++i) {
        const UnitInfo u = decode_unit(P, pair_unit_id(P, pair, first, i));
        const GemmProblem& pr = P.p[u.pi];
        const uint32_t a_sub = 128u * 128u;
        const uint32_t b_sub = static_cast<uint32_t>(pr.bn >> 1) * 128u;
        const uint32_t bytes = (is_a ? a_sub : b_sub) * static_cast<uint32_t>(pr.ksub);
        const int a_row0 = u.tm * 256 + static_cast<int>(rank) * 128;
        const int n0 = u.tn * pr.bn + static_cast<int>(rank) * (pr.bn >> 1);
        for (int sl = 0; sl < u.nslots; ++sl, ++it) {
          const int s = it % S;
          const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, kErrGemmTimeout + 1)) {
            ok = false;
            break;
          }
          uint8_t* slot = smem + s * P.slot_bytes;
          const int chunk = u.c_begin + sl * pr.ksub;
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2u * bytes);
          const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0u);
          if (is_a) {
            if (pr.kdim3)
              tma_load_3d_pair(slot, &pr.ta, bar, 0, a_row0, chunk, pol);
            else
              tma_load_2d_pair(slot, &pr.ta, bar, chunk * 64, a_row0, pol);
          } else {
            uint8_t* dst = slot + a_sub * pr.ksub;
            if (pr.kdim3)
              tma_load_3d_pair(dst, &pr.tb, bar, 0, n0, chunk, pol);
            else
              tma_load_2d_pair(dst, &pr.tb, bar, chunk * 64, n0, pol);
          }
        }
      }
      // The MMA thread's commits arrive on this CTA's empty barriers asynchronously: wait for the
      // release of every slot still in flight so that none lands after the CTA has exited.
      for (int t = (it > S ? it - S : 0); ok && t < it; ++t)
        ok = mbar_wait(&empty[t % S], static_cast<uint32_t>(t / S) & 1u, kErrGemmTimeout + 1);
      if (!ok) settle_issued_copies();  // loads already issued land before the CTA exits
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: one thread of rank 0 drives both CTAs' tensor cores ----------
    if (lane == 0 && rank == 0) {
      int it = 0;
      bool ok = true;
      for (int j = 0; ok && j < nunits; ++j) {
        const UnitInfo u = decode_unit(P, pair_unit_id(P, pair, first, j));
        const GemmProblem& pr = P.p[u.pi];
        const int ab = j & 1;
        if (!mbar_wait(&acc_empty[ab], (static_cast<uint32_t>(j >> 1) & 1u) ^ 1u, kErrGemmTimeout + 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * kAccCols);
        const uint32_t idesc = umma_idesc_bf16(256, pr.bn);
        const uint32_t a_sub = 128u * 128u;
        const uint32_t b_sub = static_cast<uint32_t>(pr.bn >> 1) * 128u;
        for (int sl = 0; sl < u.nslots; ++sl, ++it) {
          const int s = it % S;
          const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
          if (!mbar_wait(&full[s], ph, kErrGemmTimeout + 2)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * P.slot_bytes);
          const uint32_t b_addr = a_addr + a_sub * static_cast<uint32_t>(pr.ksub);
          const int nsub = min(pr.ksub, u.c_end - (u.c_begin + sl * pr.ksub));
          for (int sub = 0; sub < nsub; ++sub) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              umma_f16_pair(d_tmem, umma_desc_sw128(a_addr + sub * a_sub + 32 * k),
                            umma_desc_sw128(b_addr + sub * b_sub + 32 * k), idesc,
                            (sl | sub | k) != 0 ? 1u : 0u);
            }
          }
          const uint32_t e = smem_u32(&empty[s]);
          umma_commit_pair(mapa_shared(e, 0u));
          umma_commit_pair(mapa_shared(e, 1u));
        }
        if (!ok) break;
        const uint32_t f = smem_u32(&acc_full[ab]);
        umma_commit_pair(mapa_shared(f, 0u));
        umma_commit_pair(mapa_shared(f, 1u));
      }
      if (!ok) {  // the pair MMAs already issued finish before either CTA releases TMEM
        umma_commit_pair(mapa_shared(smem_u32(drain), 0u));
        mbar_wait_teardown(drain, 0u);
      }
    }
  } else {
    // ---------------- epilogue warps (both CTAs, each over its own 128 rows) ----------------
    griddep_wait();
    const int quad = warp & 3;
    const int set = (warp - kEpiWarp0) >> 2;
    const int r_local = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t rel0 = mapa_shared(smem_u32(&acc_empty[0]), 0u);
    const uint32_t rel1 = mapa_shared(smem_u32(&acc_empty[1]), 0u);
    bool ok = true;
    for (int j = 0; ok && j < nunits; ++j) {
      const UnitInfo u = decode_unit(P, pair_unit_id(P, pair, first, j));
      const GemmProblem& pr = P.p[u.pi];
      const int ab = j & 1;
      if (!mbar_wait(&acc_full[ab], static_cast<uint32_t>(j >> 1) & 1u, kErrGemmTimeout + 3)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tacc = tmem_base + lane_off + static_cast<uint32_t>(ab * kAccCols);
      const RowCtx rc = row_ctx(pr, 2 * u.tm + static_cast<int>(rank), r_local);
      unit_epilogue_act<kMode>(pr, rc, u.tn * pr.bn, set, TmemSrc{tacc});
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(ab ? rel1 : rel0);
    }
  }
  tc_fence_before();
  cluster_sync();  // no pair traffic (MMA reads, commits, remote arrivals) outlives either CTA
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * kAccCols);
  }
}

// At least 116 KB so that two CTAs never share an SM: a second CTA would only wait in
// tcgen05.alloc for the first one's 512 TMEM columns.
size_t gemm_smem_bytes(int stages, int slot_bytes) {
  const size_t need = 1024 + static_cast<size_t>(stages) * slot_bytes + kRingSlack + 256;
  return need < 116 * 1024 ? 116 * 1024 : need;
}

cudaError_t gemm_prepare_device() {
  cudaError_t e = cudaSuccess;
  auto set = [&](const void* fn) {
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  };
  set(reinterpret_cast<const void*>(gemm_bf16_kernel<kEpiStore, false>));
  set(reinterpret_cast<const void*>(gemm_bf16_kernel<kEpiSwiGLU, false>));
  set(reinterpret_cast<const void*>(gemm_bf16_kernel<kEpiQKV, false>));
  set(reinterpret_cast<const void*>(gemm_bf16_kernel<kEpiEuler, false>));
  set(reinterpret_cast<const void*>(gemm_bf16_kernel<kEpiStore, true>));
  set(reinterpret_cast<const void*>(gemm_bf16_kernel<kEpiSwiGLU, true>));
  set(reinterpret_cast<const void*>(gemm_bf16_kernel<kEpiQKV, true>));
  set(reinterpret_cast<const void*>(gemm_bf16_kernel<kEpiEuler, true>));
  set(reinterpret_cast<const void*>(gemm_pair_kernel<kEpiStore>));
  set(reinterpret_cast<const void*>(gemm_pair_kernel<kEpiSwiGLU>));
  set(reinterpret_cast<const void*>(gemm_pair_kernel<kEpiQKV>));
  set(reinterpret_cast<const void*>(gemm_pair_kernel<kEpiEuler>));
  return e;
}

cudaError_t launch_gemm(const GemmParams& params, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(params.ncta, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = gemm_smem_bytes(params.stages, params.slot_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (params.pair) {
    if (params.ncta % 2 != 0) return cudaErrorInvalidValue;
    attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[cfg.numAttrs].val.clusterDim.x = 2;
    attr[cfg.numAttrs].val.clusterDim.y = 1;
    attr[cfg.numAttrs].val.clusterDim.z = 1;
    cfg.numAttrs += 1;
    switch (params.p[0].ep.mode) {
      case kEpiSwiGLU:
        return cudaLaunchKernelEx(&cfg, gemm_pair_kernel<kEpiSwiGLU>, params);
      case kEpiQKV:
        return cudaLaunchKernelEx(&cfg, gemm_pair_kernel<kEpiQKV>, params);
      case kEpiEuler:
        return cudaLaunchKernelEx(&cfg, gemm_pair_kernel<kEpiEuler>, params);
      default:
        return cudaLaunchKernelEx(&cfg, gemm_pair_kernel<kEpiStore>, params);
    }
  }
  bool split = false;
  for (int i = 0; i < params.nprob; ++i) split = split || params.p[i].nsplit > 1;
  switch (params.p[0].ep.mode) {  // every problem of a launch shares the epilogue mode
    case kEpiSwiGLU:
      return split ? cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<kEpiSwiGLU, true>, params)
                   : cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<kEpiSwiGLU, false>, params);
    case kEpiQKV:
      return split ? cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<kEpiQKV, true>, params)
                   : cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<kEpiQKV, false>, params);
    case kEpiEuler:
      return split ? cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<kEpiEuler, true>, params)
                   : cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<kEpiEuler, false>, params);
    default:
      return split ? cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<kEpiStore, true>, params)
                   : cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<kEpiStore, false>, params);
  }
}

}  // namespace rldx
