/*
 * rldx_b200.h — C ABI of the B200 (sm_100a) MSAT inference library (librldx_b200.so).
 *
 * Plain pointers and sizes only.  All tensors are device pointers unless a function says
 * otherwise; bf16 tensors are row-major with the leading dimension given in elements.
 * `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * Every function returns RLDX_OK (0) or a negative RLDX_ERR_* code; rldx_last_error() gives
 * the message of the last failure on the calling thread.  Kernels never spin forever: a wait
 * that runs out records a device error code that rldx_get_device_error() reports.
 *
 * The library has no CPU fallback: without an sm_100 device every compute call fails.
 */
#ifndef RLDX_B200_H_
#define RLDX_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RLDX_OK 0
#define RLDX_ERR_ARG (-1)         /* bad shape, pointer, alignment or enum value        */
#define RLDX_ERR_CUDA (-2)        /* a CUDA runtime / driver call failed                 */
#define RLDX_ERR_DEVICE (-3)      /* a kernel recorded a device-side error (timeout)     */
#define RLDX_ERR_UNSUPPORTED (-4) /* configuration outside what the kernels implement    */
#define RLDX_ERR_STATE (-5)       /* call not valid in the object's current state        */

/* ABI version of this header (major * 100 + minor). */
int rldx_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* rldx_last_error(void);

/* Reads and clears the device-side error word (0 = none).  Synchronizes the device. */
int rldx_get_device_error(unsigned int* code);

/* Bound of every wait inside the kernels, in SM clock cycles (default 4e9, about 2 s at full
 * clock), for the current device; [1e3, 1e11].  A wait that runs out records a device error
 * and its kernel returns.  Set it between steps, not while kernels of the library run.
 * No counterpart in the reference (its Triton kernels have no waits). */
int rldx_set_wait_limit(int64_t cycles);
int rldx_get_wait_limit(int64_t* cycles);

/* Self-test of the bounded wait: one warp waits on a barrier that nothing arrives on, gives up
 * after limit_cycles ([1e3, 4e9]) and records device error 0x400; the kernel then returns.
 * Asynchronous on `stream`.  No counterpart in the reference. */
int rldx_wait_selftest(int64_t limit_cycles, void* stream);

/* 1 if the current device is an sm_100 part the kernels were built for, else 0. */
int rldx_device_supported(void);

/* ------------------------------------------------------------------------------------------
 * Grouped GEMM with fused epilogue:  out = epilogue(A[M,K] * B[N,K]^T).
 * Replaces the cuBLAS nn.Linear / torch.bmm calls of every MSAT block and encoder
 * (rldx/model/modules/action_model/blocks.py:314-351, 684-689;
 *  rldx/model/modules/embodiment_conditioned_mlp.py:72-82) and the Triton SwiGLU epilogue
 * ds::grouped_swiglu (rldx/inference/action_model/double_stream/engine/ops/op_grouped_swiglu.py:12-39).
 * ------------------------------------------------------------------------------------------ */
#define RLDX_EPI_STORE 0  /* out = act(bias(acc)) [+ add]                                       */
#define RLDX_EPI_SWIGLU 1 /* B rows interleaved [32 gate | 32 up] per 64: out = silu(g) * u     */
#define RLDX_EPI_QKV 2    /* per-head RMSNorm + RoPE of q/k into [B,H,L,64], v into [B,H,64,Lp] */
#define RLDX_EPI_EULER 3  /* out = out + dt * act(bias(acc))                                     */

#define RLDX_BIAS_NONE 0
#define RLDX_BIAS_FUSED 1      /* bf16(acc + b)          (nn.Linear)                         */
#define RLDX_BIAS_POST_ROUND 2 /* bf16(bf16(acc) + b)    (torch.bmm(x, W) + b)               */

#define RLDX_ACT_NONE 0
#define RLDX_ACT_RELU 1
#define RLDX_ACT_SILU 2  /* bf16(x * sigmoid(x)) in one rounding (F.silu)                    */
#define RLDX_ACT_SWISH 3 /* bf16(x * bf16(sigmoid(x)))             (x * torch.sigmoid(x))    */

typedef struct {
  const void* a; /* [M, K] bf16, row stride lda elements (lda*2 % 16 == 0, 16-byte aligned) */
  int64_t lda;
  const void* b; /* [N, K] bf16 (row stride ldb), or [cats, N, K] with cat_ids              */
  int64_t ldb;
  int64_t b_cat_stride;   /* elements between category slabs                              */
  const int64_t* cat_ids; /* device [M / rows_per_cat] category ids, or NULL               */
  int rows_per_cat;       /* rows sharing one category (<= 128)                            */
  int num_cats;           /* number of category slabs in b                                 */
  int M, N, K;
  const void* bias; /* [N] bf16 or [cats, N] with cat_ids (stride bias_cat_stride)         */
  int bias_mode;
  int64_t bias_cat_stride;
  int act;
  const void* add; /* optional bf16 added after the activation (residual / positions)      */
  int64_t ld_add;
  int add_row_mod; /* add row = (row % rows_in) % add_row_mod when > 0, else the row itself  */
  void* out;
  int64_t ldo;
  int col_off;
  int epilogue;
  int rows_in, rows_out, row_skip; /* batched row remap (0 = identity), see RLDX_EPI_*       */
  float dt;                        /* RLDX_EPI_EULER step                                    */
  /* RLDX_EPI_QKV */
  const void* q_norm_w; /* [64] bf16 */
  const void* k_norm_w; /* [64] bf16 */
  const float* rope_cos; /* [L, 32] fp32 */
  const float* rope_sin; /* [L, 32] fp32 */
  void* q;               /* [B, H, L, 64] bf16 */
  void* k;               /* [B, H, L, 64] bf16 */
  void* vt;              /* [B, H, 64, Lp] bf16 */
  int L, Lp, H, tok_off;
  float eps;
  int tile_n; /* 0 = choose automatically, else 64/128/192/256 */
  /* RLDX_EPI_QKV: 1 promises that the RoPE of every row of this problem is the identity (cos 1,
   * sin 0 in its table rows, e.g. position 0 on every axis): the epilogue then skips the tables.
   * 0 (the safe default) reads them. */
  int rope_identity;
} rldx_gemm_desc;

/* Runs up to 4 independent problems in one persistent launch (no K split). */
int rldx_gemm(const rldx_gemm_desc* problems, int nproblems, void* stream);

/* Bytes of workspace with which rldx_gemm_ws may split long K loops of these problems across
 * SMs (0 = the plan would not split).  Same validation as rldx_gemm; launches nothing. */
int rldx_gemm_workspace_size(const rldx_gemm_desc* problems, int nproblems, uint64_t* bytes);

/* The launch plan that rldx_gemm_ws (given a large enough workspace) uses for these problems;
 * launches nothing.  plan[0] = 1 when CTA pairs (clusters of two) run cta_group::2 MMAs on
 * 256-row tiles, plan[1] = CTAs launched, plan[2] = ring stages, plan[3] = tile width (N) of the
 * first problem (the pair's width in pair mode), plan[4] = its K splits. */
int rldx_gemm_plan(const rldx_gemm_desc* problems, int nproblems, int* plan);

/* rldx_gemm with a device workspace: problems whose K loop would leave SMs idle are split,
 * each split writes an fp32 partial tile, and the last split of a tile to finish adds the
 * partials in split order (the result does not depend on which finishes last) and runs the
 * epilogue.  The workspace must be 16-byte aligned and ZERO-FILLED before its first use; its
 * first bytes hold per-tile arrival counters that every call leaves at zero again.  Calls that
 * share one workspace must be ordered on one stream.  A workspace smaller than
 * rldx_gemm_workspace_size() (or NULL) runs the problems unsplit. */
int rldx_gemm_ws(const rldx_gemm_desc* problems, int nproblems, void* workspace,
                 uint64_t workspace_bytes, void* stream);

/* rldx_gemm_ws without a caller workspace: the K-split partials and arrival counters live in
 * an 8 MiB static device array of the library.  For callers that cannot allocate device
 * memory when they run a GEMM (allocator-free serving paths, C-ABI hosts without a CUDA
 * allocator).  No counterpart in the reference.  Allocates nothing.  The first call on a
 * device looks the scratch's device address up (cudaGetSymbolAddress, kept for the process;
 * not valid across a cudaDeviceReset): make it before any stream capture.  Every call clears
 * the arrival counters first (a cudaMemsetAsync of a few KB on `stream`).  Plans needing more
 * than 8 MiB of workspace fail with RLDX_ERR_UNSUPPORTED (rldx_gemm_ws with too small a
 * workspace runs them unsplit instead).  One scratch per device: calls that overlap on the
 * GPU race, so order them on one stream. */
int rldx_gemm_static_ws(const rldx_gemm_desc* problems, int nproblems, void* stream);

/* ------------------------------------------------------------------------------------------
 * Joint-stream attention (non-causal, scale 1/sqrt(head_dim)) over [seg0 | seg1 | seg2].
 * Replaces the F.scaled_dot_product_attention of ds::fused_attention_3way
 * (rldx/inference/action_model/double_stream/engine/ops/op_fused_attention_3way.py:13-116) and
 * rldx/model/modules/action_model/blocks.py:866-869 (split of the output back into streams).
 *   head_dim 64 (MSAT) or 128
 *   q, k  [B, H, L, head_dim] bf16;  vt [B, H, head_dim, Lp] bf16 (Lp >= L, Lp % 8 == 0)
 *   key_mask [B, L] uint8 (1 = attend) or NULL
 *   out[s] [B * seg_len[s], H*head_dim] bf16, nseg in 1..3, sum(seg_len) == L
 *   tiles_per_cta: 128-query tiles per CTA, 1 or 2 (two softmax warpgroups sharing each K / V
 *   tile), 0 = chosen from the grid size
 * ------------------------------------------------------------------------------------------ */
int rldx_joint_attention(const void* q, const void* k, const void* vt, int B, int H, int L, int Lp,
                         int head_dim, const uint8_t* key_mask, void* const* out, const int* seg_len,
                         int nseg, int tiles_per_cta, void* stream);

/* ------------------------------------------------------------------------------------------
 * Attention with every option of the kernel, described by a struct:
 *   q [B, H, L, head_dim]; k [B, kv_heads, L, head_dim]; vt [B, kv_heads, head_dim, Lp];
 *   kv_heads divides H (grouped-query attention: query head h reads kv head h / (H / kv_heads),
 *   repeat_kv of rldx/model/modules/backbone/modeling_qwen3_vl.py:139-151), 0 = H;
 *   causal 1: key j is visible to query i only for j <= i (the decoder prefill's causal mask);
 *   out[s] with row stride out_ld[s] elements (0: H*head_dim), nseg 1..3, sum(seg_len) == L;
 *   causal_block n > 1 makes the mask block-causal (key j visible to query i iff
 *   j < (i / n + 1) * n); out_dim < head_dim writes only the first out_dim dims of each head
 *   (a 96-dim head stored zero-padded to 128).
 * rldx_joint_attention is this with kv_heads = H, causal = 0 and dense outputs.
 * ------------------------------------------------------------------------------------------ */
typedef struct {
  const void* q;
  const void* k;
  const void* vt;
  int B, H, kv_heads, L, Lp, head_dim;
  int causal;
  int tiles_per_cta;
  const uint8_t* key_mask;
  void* out[3];
  int seg_len[3];
  int out_ld[3];
  int nseg;
  int causal_block;
  int out_dim;
} rldx_attention_desc;

int rldx_attention(const rldx_attention_desc* desc, void* stream);

/* ------------------------------------------------------------------------------------------
 * QKV preparation of the joint attention from projected [q | k | v] rows: per-head QK RMSNorm
 * (norms.py:18-22) and interleaved-pair RoPE (ops.py:48-67) into q, k [B, H, L, 64] and
 * V^T [B, H, 64, Lp].  The RMSNorm + RoPE half of ds::fused_attention_2way / _3way
 * (rldx/inference/action_model/double_stream/engine/ops/op_fused_attention.py:12-92,
 * op_fused_attention_3way.py:13-116) and ss::fused_attention_2way / _3way
 * (single_stream/engine/ops/op_fused_attention.py:12-80, op_fused_attention_3way.py:13-110);
 * rldx_joint_attention does the SDPA half.
 *   segments in joint-sequence order (1..3), rows summing to L; qkv rows 3*H*64 wide,
 *   ld % 8 == 0, 16-byte aligned; rope tables [rows - rope_from, 32] fp32 for the segment's
 *   rows from rope_from on (rope_cos NULL: no rotation), as the reference ops' per-stream
 *   tables; batch b of a segment starts batch_stride elements after batch b-1.
 * ------------------------------------------------------------------------------------------ */
typedef struct {
  const void* qkv;
  int64_t ld;
  int64_t batch_stride;
  int rows;
  int rope_from;
  const void* q_norm; /* [64] bf16 */
  const void* k_norm; /* [64] bf16 */
  const float* rope_cos;
  const float* rope_sin;
} rldx_qkv_segment;

int rldx_qkv_prep(const rldx_qkv_segment* segs, int nseg, int B, int H, int L, int Lp, float eps,
                  void* q, void* k, void* vt, void* stream);

/* ------------------------------------------------------------------------------------------
 * Residual sums + LayerNorm (no affine) over up to 2 row groups in one launch:
 *   sum = x (+ y) (+ v1) (+ v2), rows x, y [rows, D] with row stride ld, vectors v1, v2 [D];
 *   fp32_sum 0: bf16 rounding after each add in the order x, v1, v2, y -- ds::vl_epilogue_ln
 *     (rldx/inference/action_model/double_stream/engine/ops/op_vl_epilogue_ln.py:13-38,
 *     new = res + proj_bias + w3_bias + w3_out) and ss::fused_epilogue_ln
 *     (single_stream/engine/ops/op_fused_epilogue_ln.py:11-30, new = hidden + residual);
 *   fp32_sum 1: one fp32 sum x + y + v1 + v2 -- ds::grouped_res_ln
 *     (double_stream/engine/ops/op_grouped_res_ln.py:12-45, LN(res + proj + bias)).
 *   sum_out (optional) = bf16(sum); ln_out = LN(sum) in fp32, rounded once.  D % 8 == 0,
 *   D <= 4096, every pointer 16-byte aligned, ld % 8 == 0.
 * ------------------------------------------------------------------------------------------ */
typedef struct {
  const void* x;
  const void* y;  /* optional */
  const void* v1; /* optional [D] */
  const void* v2; /* optional [D] */
  void* sum_out;  /* optional */
  void* ln_out;
  int rows;
  int D;
  int64_t ld;
  const void* w;  /* [D] RMSNorm weight (rldx_res_rmsnorm only) */
} rldx_res_ln_segment;

int rldx_res_layernorm(const rldx_res_ln_segment* segs, int nseg, int fp32_sum, float eps, void* stream);

/* Same sums (bf16 after each add), then Qwen3 RMSNorm with weight instead of LayerNorm:
 * ln_out = bf16(w * bf16(sum * rsqrt(mean(sum^2) + eps)))  (Qwen3VLTextRMSNorm,
 * rldx/model/modules/backbone/modeling_qwen3_vl.py:357-374; with y = the residual it is the
 * reference's fused_epilogue_add2_rmsnorm, rldx/inference/backbone/llm/engine/ops/). */
int rldx_res_rmsnorm(const rldx_res_ln_segment* segs, int nseg, float eps, void* stream);

/* ------------------------------------------------------------------------------------------
 * Bias + SwiGLU over up to 2 row groups, all in fp32 with one rounding:
 * out = bf16( silu(gate + bias_gate) * (up + bias_up) ) -- ds::grouped_swiglu
 * (rldx/inference/action_model/double_stream/engine/ops/op_grouped_swiglu.py:12-41 on the
 * [gate | up] halves of an un-biased w12 output).  H % 8 == 0, 16-byte aligned rows.
 * ------------------------------------------------------------------------------------------ */
typedef struct {
  const void* gate;
  const void* up;
  const void* bias_gate; /* [H] */
  const void* bias_up;   /* [H] */
  void* out;
  int64_t ld_in;
  int64_t ld_out;
  int rows;
  int H;
} rldx_swiglu_bias_segment;

int rldx_swiglu_bias(const rldx_swiglu_bias_segment* segs, int nseg, void* stream);

/* ------------------------------------------------------------------------------------------
 * LayerNorm without affine (eps) over rows of width D (D % 8 == 0, D <= 4096), optionally
 * followed by y * scale1p + shift (AdaLN-zero output projection, both bf16 [D]).
 * Replaces nn.LayerNorm(elementwise_affine=False) (rldx/model/modules/norms.py:35-36), the LN of
 * ds::vl_epilogue_ln (rldx/inference/action_model/double_stream/engine/ops/op_vl_epilogue_ln.py:13-38)
 * and MSAT._output_projection (rldx/model/modules/action_model/msat.py:771-781).
 * ------------------------------------------------------------------------------------------ */
int rldx_layernorm(const void* in, int64_t ld_in, void* out, int64_t ld_out, int rows, int D,
                   float eps, const void* scale1p, const void* shift, void* stream);

/* ------------------------------------------------------------------------------------------
 * Qwen3-style per-head RMSNorm + rotate-half RoPE on x [T, H, 128] -> y (may alias x).
 *   pos [T] int32 rows of cos/sin [P, 128] bf16 tables; w [128] bf16.
 * Replaces the QK-norm + RoPE stage of fused_llm_attention
 * (rldx/inference/backbone/llm/engine/kernels/fused_llm_attention.py:100) and
 * modeling_qwen3_vl.py:357-401 (rldx/model/modules/backbone).
 * ------------------------------------------------------------------------------------------ */
int rldx_qk_rmsnorm_rope(const void* x, void* y, const void* w, const int32_t* pos,
                         const void* cos_table, const void* sin_table, int64_t tokens, int heads,
                         int head_dim, float eps, void* stream);

/* ------------------------------------------------------------------------------------------
 * SwiGLU activation out[t,i] = silu(gate[t,i]) * up[t,i]  (H % 8 == 0).
 * Replaces ds::grouped_swiglu's activation
 * (rldx/inference/action_model/double_stream/engine/kernels/grouped_swiglu.py:108) and
 * SwiGLUFFN.forward (rldx/model/modules/action_model/ops.py:157-161).
 * ------------------------------------------------------------------------------------------ */
int rldx_swiglu(const void* gate, const void* up, int64_t ld_in, void* out, int64_t ld_out,
                int64_t rows, int H, void* stream);

/* ------------------------------------------------------------------------------------------
 * MSAT control step (all-modality action head): state encoder, physics history encoder, then
 * num_steps flow-matching Euler steps of [action encoder + physics future encoder + depth
 * ExpandedDoubleStreamBlocks over [VL | SA | P] + output projections + action / physics
 * decoders + Euler updates], captured once as a single CUDA graph.
 * Replaces CustomExpandedActionHeadChain.__init__/forward
 * (rldx/inference/action_model/engine/custom_expanded_action_model_chain.py:19-213) and
 * GraphSafeActionModel.forward (rldx/inference/action_model/model/graph_safe_action_model.py:170-312);
 * semantics of RLDXActionModel.get_action_with_features (rldx/model/core/rldx.py:490-735)
 * without RTC.
 * ------------------------------------------------------------------------------------------ */
typedef struct rldx_msat rldx_msat;

#define RLDX_ROPE_SA_ONLY 0
#define RLDX_ROPE_VL_SA 1

typedef struct {
  int batch;           /* observations per call                                          */
  int n_vl;            /* cognition (VL) tokens per observation                          */
  int n_state;         /* state tokens (1)                                               */
  int horizon;         /* action tokens                                                  */
  int physics_hist;    /* physics history tokens (ignored on the standard path)          */
  int physics_fut;     /* physics future tokens (== horizon; ignored on the standard path) */
  int dim;             /* sa_dim == p_dim == heads * head_dim (single-block width)       */
  int heads;
  int head_dim;        /* 64                                                             */
  int depth;           /* double-stream blocks (Expanded... with physics)                */
  int mlp_hidden;      /* SwiGLU hidden of the SA and P streams                          */
  int vl_mlp_hidden;   /* SwiGLU hidden of the VL stream                                 */
  int out_dim;         /* MSAT output_dim (= action decoder input)                       */
  int action_dim;
  int state_dim;
  int dec_hidden;      /* action / state encoder hidden size                             */
  int physics_dim;
  int num_embodiments;
  int num_steps;       /* Euler steps (t = i / num_steps, dt = 1 / num_steps)            */
  int rope_mode;       /* RLDX_ROPE_*                                                    */
  int rope_cos_only;   /* 1: RoPE buffers were cast to a real dtype (bf16 module) -> cos  */
  float rope_theta;
  int rope_max_seq;    /* RoPE table length (action_model_max_seq_len)                   */
  int temb_channels;   /* Timesteps(num_channels) (256)                                  */
  int use_graph;       /* 1: capture the whole control step as one CUDA graph            */
  /* Topology (a zero-filled tail gives the all-modality form above: physics, double blocks) */
  int standard_path;   /* 1: no physics stream: DoubleStreamBlocks [VL | SA], then
                          SingleStreamBlocks [VL_proj | time | SA] (msat.py:363-556)       */
  int vl_dim;          /* VL stream width in the double blocks (0: dim)                  */
  int depth_single;    /* single-stream blocks after the double ones (Expanded... with P) */
  int single_expanded; /* SingleStreamBlock SwiGLU width: int(dim * mlp_ratio)            */
  int single_mlp_hidden; /* SingleStreamBlock mlp_proj output: int(2/3 * single_expanded) */
  int prefix_len;      /* RTC trained mode: first prefix_len actions locked to
                          io.prefix_actions, encoded at t = 1 (graph_safe_action_model.py:196-300;
                          custom_action_model_chain.py:86-165); 0 = off                       */
  int key_mask;        /* 1: steps may pass key masks (io.vl_mask / io.physics_mask): a second
                          graph whose attention masks those keys is captured beside the
                          unmasked one (rldx/model/modules/action_model/blocks.py:557-576,
                          843-864; msat.py:517-531, 716-745)                                  */
} rldx_msat_config;

typedef struct {
  const void* w; /* nn.Linear weight [out, in] bf16 */
  const void* b; /* [out] bf16 */
} rldx_linear;

typedef struct {
  const void* W; /* CategorySpecificLinear.W [cats, in, out] bf16 */
  const void* b; /* [cats, out] bf16 */
} rldx_cat_linear;

typedef struct {
  rldx_linear qkv, proj, w12, w3; /* {sa,vl,p}_qkv / _proj / _mlp.w12 / _mlp.w3        */
  const void* q_norm;             /* q_norm_{sa,vl,p}.weight [head_dim] bf16            */
  const void* k_norm;
} rldx_stream_weights;

typedef struct {
  rldx_stream_weights vl, sa, p;
} rldx_block_weights;

/* SingleStreamBlock (blocks.py:42-254) / ExpandedSingleStreamBlock (blocks.py:894-1089):
 * linear1 [3*inner + 2*expanded, dim] = [q | k | v | SwiGLU gate | SwiGLU up],
 * mlp_proj [mlp_hidden, expanded], linear2 [dim, inner + mlp_hidden]; p_* for the physics
 * stream of the expanded block (NULL on the standard path). */
typedef struct {
  rldx_linear linear1, linear2, mlp_proj;
  const void* q_norm; /* [head_dim] bf16 */
  const void* k_norm;
  rldx_linear p_linear1, p_linear2, p_mlp_proj;
  const void* p_q_norm;
  const void* p_k_norm;
} rldx_single_block_weights;

typedef struct {
  const rldx_block_weights* blocks; /* [depth] (host array of device pointers)       */
  rldx_linear temb_lin1, temb_lin2;  /* timestep_encoder.timestep_embedder.linear_1/2  */
  rldx_linear time_token_proj;       /* w == NULL: identity                            */
  rldx_linear proj_out_1, proj_out_2;
  rldx_linear proj_out_phys_1, proj_out_phys_2;
  rldx_cat_linear state_l1, state_l2;      /* state_encoder.layer1/2                    */
  rldx_cat_linear act_w1, act_w2, act_w3;  /* action_encoder.W1/W2/W3                   */
  rldx_cat_linear dec_l1, dec_l2;          /* action_decoder.layer1/2                   */
  const void* pos_emb;                     /* position_embedding.weight [max, dim]      */
  rldx_linear phc_w1, phc_w2, phc_w3;      /* physics.physics_cond_encoder.W1/W2/W3     */
  rldx_linear phf_w1, phf_w2, phf_w3;      /* physics.physics_fut_encoder.W1/W2/W3      */
  rldx_linear phd_l1, phd_l2;              /* physics.physics_decoder.net[0] / net[2]   */
  const rldx_single_block_weights* single_blocks; /* [depth_single] (host array)         */
  rldx_linear vl_proj_to_sa;               /* w == NULL: identity (vl_dim == dim)       */
  /* The module's own RoPE tables (RoPEEmbedder1D.freqs_cis_0 / _1, ops.py:11-25, 70-119):
   * cos and sin of axis i as [rope_max_seq, axes_i / 2] fp32 (host or device; sin ignored
   * with rope_cos_only, where cos is the real part the bf16 cast kept).  axes = [16, 48]
   * under rope_sa_only, [48, 16] under rope_vl_sa.  NULL: computed from rope_theta. */
  const float* rope_cos[2];
  const float* rope_sin[2];
} rldx_msat_weights;

typedef struct {
  const void* vl;            /* [B, n_vl, vl_dim] bf16                                  */
  const void* state;         /* [B, n_state, state_dim] bf16                            */
  const int64_t* emb_id;     /* [B] int64                                               */
  const void* init_noise;    /* [B, horizon, action_dim] bf16                           */
  const void* physics_hist;  /* [B, physics_hist, physics_dim] bf16 (NULL: standard)   */
  const void* physics_noise; /* [B, physics_fut, physics_dim] bf16 (NULL: standard)    */
  void* actions;             /* out: [B, horizon, action_dim] bf16                      */
  const void* prefix_actions; /* [B, prefix_len, action_dim] bf16 (NULL when prefix_len 0) */
  /* Key masks (handles created with key_mask = 1; NULL = every key visible): uint8, nonzero =
   * visible.  vl_mask [B, n_vl] masks backbone tokens as keys of every block (the reference's
   * backbone_attention_mask, rldx/model/core/rldx.py:619-621); physics_mask [B] masks all physics
   * tokens of an observation (PhysicsInferenceState.attn_mask, physics_head.py:232-244; the
   * all-modality path only).  Action / state / time keys are always visible.  An all-ones mask
   * gives the unmasked result. */
  const uint8_t* vl_mask;
  const uint8_t* physics_mask;
} rldx_msat_io;

/* Copies and re-lays out the weights into a device arena owned by the handle, precomputes the
 * step-constant tables (timestep embeddings, time tokens, AdaLN scale/shift, sinusoids, RoPE)
 * and plans every launch.  Must be called outside stream capture with the device current. */
int rldx_msat_create(const rldx_msat_config* cfg, const rldx_msat_weights* w, rldx_msat** out);
int rldx_msat_destroy(rldx_msat* h);

/* One control step on `stream`; io holds device pointers.  Asynchronous.  The first call
 * captures the graph (when cfg.use_graph), so it must not itself run under stream capture. */
int rldx_msat_step(rldx_msat* h, const rldx_msat_io* io, void* stream);

/* One control step with io in host memory (pinned for full speed): host->device copies, the
 * step, device->host copy of the actions, stream synchronize.  Returns RLDX_ERR_DEVICE when a
 * device error code was recorded: raised by a kernel of this step, or left by earlier work
 * (the step's first launch takes and clears such a code, so the step itself runs clean; the
 * message says which).  Replaces the reference's fall-back-on-failure
 * (rldx/inference/serve_optimization.py:432-516) with an error on the step that failed. */
int rldx_msat_step_host(rldx_msat* h, const rldx_msat_io* io, void* stream);

/* Device status of the handle's last step (rldx_msat_step is asynchronous): *code = 0 when no
 * device error was recorded, else the code (see rldx_msat_step_host).  wait = 1 waits for the
 * step to finish; wait = 0 reports 0 while it is still running.  Reading clears the status. */
int rldx_msat_status(rldx_msat* h, int wait, unsigned int* code);

/* Launches from the start of a control step up to and including the last one of block `block`
 * (double blocks first, then single blocks; -1: the launches before the first block, i.e. the
 * encoders) of Euler step `step`: with rldx_msat_run_partial
 * and rldx_msat_read_buffer this exposes the residual streams after every block (per-layer
 * parity against the reference's blocks).  No counterpart in the reference. */
int rldx_msat_block_end(const rldx_msat* h, int step, int block, int* n_ops);

/* Runs the first n_ops launches of a control step eagerly (no graph) on `stream` after the
 * input copies; io holds device pointers.  Asynchronous.  No counterpart in the reference. */
int rldx_msat_run_partial(rldx_msat* h, const rldx_msat_io* io, int n_ops, void* stream);

/* Number of kernel launches one control step performs (graph nodes when captured). */
int rldx_msat_launch_count(const rldx_msat* h);

typedef struct {
  int kind;     /* 0 GEMM, 1 joint attention, 2 layernorm, 3 row copy, 4 status word         */
  int grid;     /* CTAs launched                                                            */
  float ms;     /* device time between CUDA events recorded around the launch               */
  double bytes; /* algorithmic HBM bytes: every operand read once, every result written once */
  double flops; /* algorithmic FLOPs (2*M*N*K per GEMM problem, 4*L*L*64 per attention head) */
} rldx_op_profile;

/* Runs one control step eagerly (no graph, no programmatic overlap) with a CUDA event pair
 * around every launch; fills up to max_ops entries, sets *n_ops and synchronizes `stream`. */
int rldx_msat_profile(rldx_msat* h, const rldx_msat_io* io, rldx_op_profile* ops, int max_ops,
                      int* n_ops, void* stream);

/* Copies an intermediate buffer of the last control step into dst (device or host memory,
 * dst_bytes large enough) on `stream`: 0 X_vl ([B*n_vl, vl_dim]), 1 X_sa, 2 X_p (streams after
 * the last block of the last Euler step; with single blocks, X_sa / X_p after the last single
 * block and X_vl after the last double block unless vl_proj_to_sa is the identity), 3 the
 * action state; intermediates of the double blocks (as the last launch run left them):
 * 4-6 LayerNorm outputs (VL, SA, P), 7 q and 8 k ([B*H*L, 64], joint token order), 9 v^T
 * ([B*H*64, Lp]), 10-12 attention outputs ([B*n, H*64]), 13-15 SwiGLU hidden ([B*n, hidden
 * rounded up to 32]).  With dst == NULL only *rows / *cols are set. */
int rldx_msat_read_buffer(const rldx_msat* h, int which, void* dst, int64_t dst_bytes,
                          int64_t* rows, int64_t* cols, void* stream);

/* ------------------------------------------------------------------------------------------
 * VLM backbone prefill: a stack of Qwen3 decoder layers over B sequences of T tokens, captured
 * as one CUDA graph.  Replaces CustomLLMChain.forward
 * (rldx/inference/backbone/llm/engine/custom_llm_chain.py:63-170) and the eager
 * Qwen3VLTextDecoderLayer stack (rldx/model/modules/backbone/modeling_qwen3_vl.py:357-560):
 * per layer input RMSNorm -> fused q|k|v projection -> per-head q/k RMSNorm + rotate-half RoPE
 * -> causal grouped-query attention -> o_proj + residual -> post-attention RMSNorm -> SwiGLU MLP
 * (gate, up, down) + residual; optional final RMSNorm.  No projection has a bias (Qwen3).
 * RoPE tables are the caller's [T, head_dim] bf16 cos / sin (the rotary embedding's output,
 * mRoPE included; sin unsigned -- rotate_half supplies the sign).
 * ------------------------------------------------------------------------------------------ */
typedef struct rldx_llm rldx_llm;

typedef struct {
  int batch;      /* sequences per call */
  int tokens;     /* T, tokens per sequence */
  int hidden;     /* D */
  int q_heads;
  int kv_heads;   /* divides q_heads */
  int head_dim;   /* 128 */
  int ffn;        /* MLP intermediate size */
  int layers;
  float rms_eps;
  int final_norm; /* 1: apply the final RMSNorm (CustomLLMChain apply_final_norm) */
  int use_graph;  /* 1: capture the stack as one CUDA graph */
  /* Variants for the memory module's TransformerMemory (rldx/model/modules/memory.py:150-370),
   * a zero-filled tail gives the Qwen3 decoder: */
  int no_qk_norm;        /* 1: no per-head q / k RMSNorm (RoPE only) */
  int norm_weight_first; /* 1: RMSNorm = bf16(w * x * rsqrt(...)) in fp32 (norms.py:18-22);
                            0: Qwen3's cast, then weight */
  int causal_block;      /* 0 / 1: token-causal mask; n: block-causal over blocks of n tokens */
  /* Deepstack (Qwen3VLTextModel._deepstack_process, modeling_qwen3_vl.py:1086-1113;
   * CustomLLMChain.forward's deepstack_features, custom_llm_chain.py:137-161): after layer
   * i < deepstack_layers, hidden[b, row, :] += feature[i, b, j, :] (one bf16 rounding) for the
   * deepstack_rows token rows listed in rldx_llm_weights.deepstack_row_index.  0: none. */
  int deepstack_layers;
  int deepstack_rows;
  /* Video-token compression (LayerWrapper with internal_projection = compress_layer,
   * rldx/model/modules/backbone/layer_wrapper.py:73-113; the reference inference engine's static
   * form, graph_safe_qwen3vl_text_model.py:26-59 and 142-175): before layer compress_layer the
   * token rows [compress_begin, compress_end) of every sequence are replaced by one row, their
   * mean (bf16 sum over the rows, then bf16 division by their count), and the layers from there
   * on run on tokens - (compress_end - compress_begin) + 1 tokens with the RoPE rows
   * [0, compress_begin], [compress_end, tokens).  compress_end <= compress_begin: none (a
   * zero-filled tail).  deepstack_layers must not exceed compress_layer. */
  int compress_layer;
  int compress_begin;
  int compress_end;
} rldx_llm_config;

typedef struct {
  const void* input_norm; /* [D] */
  const void* q_proj;     /* [q_heads*head_dim, D] */
  const void* k_proj;     /* [kv_heads*head_dim, D] */
  const void* v_proj;     /* [kv_heads*head_dim, D] */
  const void* q_norm;     /* [head_dim] */
  const void* k_norm;     /* [head_dim] */
  const void* o_proj;     /* [D, q_heads*head_dim] */
  const void* post_norm;  /* [D] */
  const void* gate_proj;  /* [ffn, D] */
  const void* up_proj;    /* [ffn, D] */
  const void* down_proj;  /* [D, ffn] */
} rldx_llm_layer_weights;

typedef struct {
  const rldx_llm_layer_weights* layers; /* [layers] (host array of device or host pointers) */
  const void* final_norm;               /* [D] (final_norm = 1) */
  const void* rope_cos;                 /* [tokens, head_dim] bf16 */
  const void* rope_sin;                 /* [tokens, head_dim] bf16 */
  const int* deepstack_row_index;       /* [deepstack_rows] host array of token rows (< tokens) */
} rldx_llm_weights;

int rldx_llm_create(const rldx_llm_config* cfg, const rldx_llm_weights* w, rldx_llm** out);
int rldx_llm_destroy(rldx_llm* h);
/* hidden_in: [batch, tokens, hidden], hidden_out: [batch, rldx_llm_out_tokens(h), hidden] bf16
 * device (or pinned host) pointers; asynchronous on stream. */
int rldx_llm_prefill(rldx_llm* h, const void* hidden_in, void* hidden_out, void* stream);
/* tokens per sequence of the prefill's output: tokens, or the compressed count */
int rldx_llm_out_tokens(const rldx_llm* h);
/* kernel launches of one prefill (graph nodes when captured) */
int rldx_llm_launch_count(const rldx_llm* h);

/* Device status of the handle's last rldx_llm_prefill, as rldx_msat_status. */
int rldx_llm_status(rldx_llm* h, int wait, unsigned int* code);
/* Deepstack features of the next prefills: [deepstack_layers, batch, deepstack_rows, hidden]
 * bf16 (device or host pointer), copied into the handle's buffer asynchronously on stream
 * (the reference chain copies them into its _deepstack_add buffer per call,
 * custom_llm_chain.py:138-147).  Requires deepstack_layers > 0 at create. */
int rldx_llm_set_deepstack(rldx_llm* h, const void* features, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RLDX_B200_H_ */
