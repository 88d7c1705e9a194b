// Grouped bf16 GEMM for sm_100a: up to kMaxProblems independent problems (the cognition /
// action / physics streams of one MSAT projection) share one launch.  Each CTA owns one
// 128 x BN output tile of one problem and runs the full K loop:
//
//   warp 0      TMA producer: B (weight) tiles are issued before griddepcontrol.wait, so a
//               programmatic-dependent launch streams weights while the previous kernel drains;
//               A (activation) tiles after it.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16 steps).
//   warps 2..5  epilogue: tcgen05.ld of the fp32 accumulator (thread = output row) and the
//               fused row epilogue (bias / activation / residual / SwiGLU / QK-RMSNorm+RoPE /
//               Euler update), written straight to global memory.
//
// Operands are K-major in 128-byte-swizzled shared-memory tiles (64 bf16 of K per row).
// C = A[M,K] * B[N,K]^T, the nn.Linear convention, so weights are used in place.
#pragma once
#include "common.cuh"

namespace rldx {

constexpr int kMaxProblems = 4;
constexpr int kMaxStages = 8;
constexpr int kGemmThreads = 192;
constexpr int kATileBytes = 128 * 128;  // 128 rows x 128 bytes

enum EpiMode : int {
  kEpiStore = 0,   // y = act(bias(acc)) (+ add) -> out
  kEpiSwiGLU = 1,  // 64-col chunk = 32 gate + 32 up columns -> 32 outputs silu(g)*u
  kEpiQKV = 2,     // 64-col chunk = one head of q/k/v: RMSNorm + RoPE for q/k, transpose v
  kEpiEuler = 3,   // out = out + dt * act(bias(acc))   (flow-matching Euler step)
};
enum BiasMode : int { kBiasNone = 0, kBiasFused = 1, kBiasPostRound = 2 };
enum ActMode : int { kActNone = 0, kActRelu = 1, kActSilu = 2, kActSwish = 3 };

struct GemmEpilogue {
  int mode, bias_mode, act;
  const __nv_bfloat16* bias;  // [N] or [categories, N] (category bias stride = bias_cat_stride)
  int bias_cat_stride;
  const __nv_bfloat16* add;   // optional tensor added after the activation (residual / pos-emb)
  int ld_add, add_row_mod;    // add row = add_row_mod ? (t % add_row_mod) : r, t = row in batch
  __nv_bfloat16* out;
  int ldo, col_off;
  int rows_in, rows_out, row_skip;  // t = row % rows_in, b = row / rows_in; out row =
                                    // b*rows_out + t - row_skip; rows t < row_skip dropped
  float dt;
  // kEpiQKV
  const __nv_bfloat16* qn_w;
  const __nv_bfloat16* kn_w;
  const float* rope_cos;  // [L, 32]
  const float* rope_sin;  // [L, 32]
  __nv_bfloat16* q;       // [B, H, L, 64]
  __nv_bfloat16* k;       // [B, H, L, 64]
  __nv_bfloat16* vt;      // [B, H, 64, Lp]
  int L, Lp, H, tok_off;
  float eps;
};

struct __align__(64) GemmProblem {
  CUtensorMap ta;  // A [M, K] (2D), box (64, a_rows)
  CUtensorMap tb;  // B [N, K] (2D) or [categories, N, K] (3D), box (64, bn[, 1])
  int M, N, K;
  int bn;          // tile N (64..256, multiple of 64)
  int a_rows;      // A box rows (8..128)
  int m_step;      // output rows owned by one M tile (<= 128)
  int tiles_m, tiles_n, tile_begin;
  const long long* cat_ids;  // non-null: M tile index = batch element, B slab = cat_ids[tile]
  GemmEpilogue ep;
};

struct GemmParams {
  GemmProblem p[kMaxProblems];
  int nprob;
  int stages;
  int stage_bytes;  // kATileBytes + bn_max * 128
};

size_t gemm_smem_bytes(int stages, int stage_bytes);
cudaError_t launch_gemm(const GemmParams& params, int total_tiles, cudaStream_t stream, bool pdl);

}  // namespace rldx
