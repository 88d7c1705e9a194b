// Grouped bf16 GEMM for sm_100a: up to kMaxProblems independent problems (the cognition /
// action / physics streams of one MSAT projection) share one persistent launch.
//
// Work unit = (problem, 128-row M tile, BN-column N tile, K split).  The host orders the units
// longest-first and deals them to at most one CTA per SM (LPT schedule, kept in the launch
// parameters), so the weight-streaming work of all streams is spread evenly over the SMs.
// Large launches run on CTA pairs instead: the two CTAs of a cluster each load 128 rows of A and
// half of the B tile, one thread of rank 0 issues cta_group::2 MMAs (M = 256) that read both
// CTAs' tiles, and each CTA's epilogue finishes its own 128 rows from its own TMEM.  Per SM this
// halves the B traffic of a 256-wide tile (32 KB instead of 48 KB per 64-deep K chunk).
// Roles inside a CTA (3 + kEpiWarps warps):
//
//   warp 0      TMA producer of A (activations), after griddepcontrol.wait.
//   warp 2      TMA producer of B (weights).  Weights never depend on the previous kernel, so
//               this warp starts streaming them as soon as the CTA is resident, overlapping the
//               tail of the previous kernel under programmatic dependent launch.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16 steps)
//               into one of two TMEM accumulators (2 x 256 columns), so the epilogue of one
//               unit overlaps the main loop of the next.
//   warps 3..    epilogue: kEpiSets warps per TMEM lane quadrant (thread = output row) split
//               the unit's columns.  A unit's operands (bias, residual, norm weights, RoPE
//               rows) are fetched before its accumulator is ready, then tcgen05.ld brings up to
//               32 fp32 columns per wait into the fused row epilogue (bias / activation /
//               residual / SwiGLU / QK-RMSNorm+RoPE / Euler update), written straight to
//               global memory.  K-split units write fp32
//               partial tiles to a workspace; the last of a tile's units to finish (arrival
//               counter) adds the partials in split order and runs the epilogue, so results do
//               not depend on which CTA finishes last.
//
// Operands are K-major in 128-byte-swizzled shared-memory tiles (64 bf16 of K per row).  When
// K is a multiple of 64 the tensor maps view each operand as [K/64][rows][64], so one TMA box
// brings `ksub` consecutive 64-wide K chunks (one instruction per operand per ring slot).
// C = A[M,K] * B[N,K]^T, the nn.Linear convention, so weights are used in place.
#pragma once
#include "common.cuh"

namespace rldx {

constexpr int kMaxProblems = 4;
constexpr int kMaxStages = 8;
constexpr int kEpiWarp0 = 3;         // first epilogue warp
#ifndef RLDX_GEMM_EPI_WARPS
#define RLDX_GEMM_EPI_WARPS 16
#endif
constexpr int kEpiWarps = RLDX_GEMM_EPI_WARPS;  // kEpiSets warps per TMEM lane quadrant
constexpr int kEpiSets = kEpiWarps / 4;         // ... splitting the columns of a unit
constexpr int kGemmThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr int kMaxUnits = 1536;     // explicit schedule capacity; larger launches stride units
constexpr int kMaxCtas = 160;       // >= SM count of the part
constexpr int kRingSlack = 16384;   // the MMA reads 128 A rows from every A sub-tile
constexpr int kAccCols = 256;       // TMEM columns per accumulator (two accumulators)

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
  int rope_identity;  // every row's RoPE is the identity (cos 1, sin 0): the tables are not read
};

struct __align__(64) GemmProblem {
  CUtensorMap ta;  // A: [K/64][M][64] (kdim3) or [M][K] (2D)
  CUtensorMap tb;  // B: [K/64][N][64] / [cats][K/64][N][64] (kdim3) or [N][K] / [cats][N][K]
  int M, N, K;
  int bn;          // tile N (64..256, multiple of 64)
  int a_rows;      // A box rows (8..128, multiple of 8)
  int m_step;      // output rows owned by one M tile (<= 128)
  int tiles_m, tiles_n;
  int nchunks;     // ceil(K / 64)
  int ksub;        // 64-wide K chunks per TMA box (1 unless kdim3)
  int kdim3;       // 1: chunked tensor maps (K % 64 == 0)
  int nsplit;      // K splits per output tile
  int split_chunks;  // chunks per split (the last split may hold fewer)
  int unit_begin;  // first unit id of this problem
  long long ws_off;  // float offset of this problem's partial tiles in the workspace
  int cnt_off;     // offset of this problem's tile counters
  const long long* cat_ids;  // non-null: M tile index = batch element, B slab = cat_ids[tile]
  GemmEpilogue ep;
};

struct GemmParams {
  GemmProblem p[kMaxProblems];
  int nprob;
  int stages;
  int slot_bytes;
  int nunits;
  int ncta;
  int explicit_sched;       // 1: sched/cta_begin hold the unit list; 0: unit = cta + i * ncta
  int pair;                 // 1: CTA pairs (clusters of 2) run cta_group::2 MMAs on 256-row M
                            //    tiles: tiles_m counts 256-row tiles, bn is the pair's N (each
                            //    CTA loads bn/2 rows of B), a unit's list index is the pair's
                            //    (cta_begin / striding over ncta / 2 pairs); no K splits
  float* ws;                // K-split partial tiles (fp32)
  unsigned int* counters;   // one arrival counter per split tile; zero between launches
  unsigned short cta_begin[kMaxCtas + 1];
  unsigned short sched[kMaxUnits];
};

size_t gemm_smem_bytes(int stages, int slot_bytes);
cudaError_t launch_gemm(const GemmParams& params, cudaStream_t stream, bool pdl);

}  // namespace rldx
