// Launch parameters and host launchers of every kernel in the library.
#pragma once
#include "gemm.cuh"

namespace rldx {

// ---- joint attention (attention.cu) ----
struct AttnParams {
  CUtensorMap tq;  // [B*H, L, 64], box (64, 128, 1)
  CUtensorMap tk;  // [B*H, L, 64], box (64, 64, 1)
  CUtensorMap tv;  // [B*H, 64, Lp] (V transposed), box (64 keys, 64 dims, 1)
  int L, H, B;
  const unsigned char* key_mask;  // [B, L] (1 = visible) or null
  __nv_bfloat16* seg_out[3];      // per-stream outputs [B * seg_len, H*64]
  int seg_len[3];
  int seg_ld[3];                  // row stride of seg_out[s] in elements (0: H*64)
  int nseg;
  float scale_log2;  // log2(e) / sqrt(head_dim)
  int head_dim;      // 64 or 128 (0: 64)
  int tiles_per_cta; // 128-query tiles per CTA: 1, 2, or 0 = chosen from the grid size
  int kv_heads;      // K / V heads (GQA: query head h reads kv head h / (H / kv_heads)); 0: H
  int causal;        // 1: key j visible to query i only for j < (i / causal_block + 1) * causal_block
  int causal_block;  // 1 (or 0): token-causal; n: block-causal over blocks of n tokens
  int out_dim;       // dims per head written to seg_out (<= head_dim, multiple of 8; 0: head_dim);
                     // a 96-dim head runs zero-padded to 128 and writes its first 96 dims
};
int attention_tiles_per_cta(const AttnParams& p, int sms);
size_t attention_smem_bytes(int head_dim);
cudaError_t attention_prepare_device();
cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl);

// ---- row kernels (rownorm.cu) ----
struct LnSegment {
  const __nv_bfloat16* in;
  __nv_bfloat16* out;
  const __nv_bfloat16* scale1p;  // optional [D]: (1 + scale), bf16
  const __nv_bfloat16* shift;    // optional [D]
  int rows, ld_in, ld_out, row_begin;
  int D;  // row width of this segment (0: LnParams::D)
};
constexpr int kMaxLnSegments = 4;
struct LnParams {
  LnSegment seg[kMaxLnSegments];
  int nseg;
  int D;  // widest segment (selects the kernel variant)
  int total_rows;
  float eps;
};
cudaError_t launch_ln(const LnParams& p, cudaStream_t stream, bool pdl);

// x[(b * T + rows[j]) * D + c] = bf16(x + f[(b * nrows + j) * D + c]) for b < B, j < nrows
// (deepstack feature injection; D % 8 == 0, 16-byte aligned rows)
cudaError_t launch_rows_add(__nv_bfloat16* x, const int* rows, int nrows, const __nv_bfloat16* f, int B, int T,
                            int D, cudaStream_t stream);

// Row copy: row i -> group g = i / group_rows, r = i % group_rows (group_rows 0: g = 0, r = i);
// src + g*src_group_pitch + r*src_pitch -> dst + g*dst_group_pitch + r*dst_pitch.
struct CopyRegion {
  const uint8_t* src;
  uint8_t* dst;
  long long src_pitch, dst_pitch;
  long long src_group_pitch, dst_group_pitch;
  int group_rows;
  int rows, bytes;  // bytes % 16 == 0
};
constexpr int kMaxCopyRegions = 8;
struct CopyParams {
  CopyRegion r[kMaxCopyRegions];
  int n;
};
cudaError_t launch_copy(const CopyParams& p, int blocks, cudaStream_t stream, bool pdl);

// Qwen3 per-head RMSNorm (cast, then weight) + rotate-half RoPE over rows (token, head) of
// 128 dims.  Token tok's head h is at x + tok * x_tok_stride + h * 128; heads < Hq use wq, the
// others wk; the RoPE row of a token is pos[tok] (or tok % T without pos).  layout 0 writes
// y[row * 128]; layout 1 writes the attention layout q [B, Hq, T, 128] / k [B, heads - Hq, T, 128].
// hd: head dims (96 or 128; a row's lanes past hd / 8 idle); out_hd: the head stride of the
// attention layout (128: 96-dim heads are written into zero-padded 128-dim rows); norm = 0 skips
// the RMSNorm (RoPE only, the memory module's attention, rldx/model/modules/memory.py:95-112).
struct QkNormRopeParams {
  const __nv_bfloat16* x;
  long long x_tok_stride;
  int hd, out_hd, norm;
  __nv_bfloat16* y;
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  const __nv_bfloat16* wq;
  const __nv_bfloat16* wk;
  const int* pos;
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  unsigned nrows, heads, Hq, T;
  int layout;
  float eps;
};
cudaError_t launch_qk_rmsnorm_rope(const QkNormRopeParams& p, cudaStream_t stream);
cudaError_t launch_v_transpose(const __nv_bfloat16* v, long long ld, __nv_bfloat16* vt, int B, int T, int Tp,
                               int Hkv, int hd, int out_hd, cudaStream_t stream);
cudaError_t launch_swiglu(const __nv_bfloat16* gate, const __nv_bfloat16* up, __nv_bfloat16* out,
                          long long rows, int H, long long ld_in, long long ld_out, int sms,
                          cudaStream_t stream);

// ---- residual sums + LayerNorm, bias + SwiGLU (rownorm.cu): the reference's epilogue ops ----
// sum = x (+ y) (+ v1) (+ v2): rows x, y [rows, D] (row stride ld), vectors v1, v2 [D];
// fp32_sum = 0: bf16 rounding after each add in the order x, v1, v2, y (eager order of
// ds::vl_epilogue_ln / ss::fused_epilogue_ln); 1: one fp32 sum in the order x, y, v1, v2 with no
// rounding (ds::grouped_res_ln).  sum_out (optional) gets bf16(sum); ln_out = LN(sum).
// rms = 1: Qwen3 RMSNorm instead of LayerNorm: ln_out = bf16(w * bf16(sum * rsqrt(mean(sum^2) + eps)))
// (rldx/model/modules/backbone/modeling_qwen3_vl.py:357-374), w [D] per segment.
struct ResLnSeg {
  const __nv_bfloat16* x;
  const __nv_bfloat16* y;
  const __nv_bfloat16* v1;
  const __nv_bfloat16* v2;
  const __nv_bfloat16* w;
  __nv_bfloat16* sum_out;
  __nv_bfloat16* ln_out;
  int rows, D, ld, row_begin;
};
struct ResLnParams {
  ResLnSeg seg[2];
  int nseg, total_rows, dmax, fp32_sum, rms;
  int rms_weight_first;  // 1: bf16(w * (sum * rstd)) in fp32 (rldx/model/modules/norms.py:18-22)
  float eps;
};
cudaError_t launch_res_ln(const ResLnParams& p, cudaStream_t stream);

// out = bf16( silu(gate + bg) * (up + bu) ) in fp32 (ds::grouped_swiglu), up to 2 segments.
struct SwigluBiasSeg {
  const __nv_bfloat16* gate;
  const __nv_bfloat16* up;
  const __nv_bfloat16* bg;
  const __nv_bfloat16* bu;
  __nv_bfloat16* out;
  long long ld_in, ld_out;
  int rows, H, row_begin;
};
struct SwigluBiasParams {
  SwigluBiasSeg seg[2];
  int nseg, total_rows, hmax;
};
cudaError_t launch_swiglu_bias(const SwigluBiasParams& p, cudaStream_t stream);

// ---- QKV preparation of the joint attention (rownorm.cu) ----
// Segments of the joint sequence, in order: rows of [q | k | v] (3*H*64 wide, row stride ld),
// per-segment QK RMSNorm weights and RoPE tables ([rows - rope_from, 32] fp32 cos / sin for the
// segment's rows from rope_from on; null cos: no rotation).
struct QkvPrepSeg {
  const __nv_bfloat16* qkv;
  long long ld, batch_stride;  // elements
  int rows, rope_from;
  const __nv_bfloat16* qn;
  const __nv_bfloat16* kn;
  const float* cos;
  const float* sin;
};
struct QkvPrepParams {
  QkvPrepSeg seg[3];
  int nseg, B, H, L, Lp;
  float eps;
  __nv_bfloat16* q;   // [B, H, L, 64]
  __nv_bfloat16* k;   // [B, H, L, 64]
  __nv_bfloat16* vt;  // [B, H, 64, Lp]
};
cudaError_t launch_qkv_prep(const QkvPrepParams& p, cudaStream_t stream);

// ---- bind-time helpers (relayout.cu) ----
// dst[i, :] = src[idx[i], :] for rows of `cols` bf16 (row gather).
cudaError_t launch_gather_rows(const __nv_bfloat16* src, long long ld_src, __nv_bfloat16* dst,
                               long long ld_dst, const int* idx, int rows, int cols,
                               cudaStream_t stream);
// dst[c, n, k] = src[c, k, n] (per-category transpose), zero-padding k in [K, Kp).
cudaError_t launch_transpose_cat(const __nv_bfloat16* src, __nv_bfloat16* dst, int cats, int K,
                                 int N, int Kp, cudaStream_t stream);
// y = silu(x) (mode 0) or y = 1 + x (mode 1), bf16 rounding once.
cudaError_t launch_elementwise(const __nv_bfloat16* x, __nv_bfloat16* y, long long n, int mode,
                               cudaStream_t stream);

// kmask [B, L]: VL keys (t < nvl) from vl [B, nvl], then nsa visible keys, then the physics
// keys from p [B] (nonzero = visible)
// Video-token compression: [B, T, D] -> [B, T - (end - begin) + 1, D], rows [begin, end) of
// every sequence replaced by their mean (bf16 sum, then bf16 division by the row count).
cudaError_t launch_compress_rows(const __nv_bfloat16* x, __nv_bfloat16* y, int B, int T, int D, int begin, int end,
                                 cudaStream_t stream);

cudaError_t launch_key_mask(uint8_t* kmask, const uint8_t* vl, const uint8_t* p, int B, int L, int nvl,
                            int nsa, cudaStream_t stream);

cudaError_t gemm_prepare_device();

}  // namespace rldx
