// MSAT control-step runtime: binds the action head's weights, precomputes every step-constant
// table, plans the whole control step as a list of kernel launches over static buffers and
// captures it as one CUDA graph.
//
// Two topologies (no RTC):
//   * all-modality (physics): ExpandedDoubleStreamBlocks over [VL | SA | P], then optional
//     ExpandedSingleStreamBlocks over [VL_proj + SA | P] (msat.py:558-781);
//   * standard (no add-ons): DoubleStreamBlocks over [VL | SA] with a VL stream of its own
//     width, then SingleStreamBlocks over [VL_proj | time | SA] (msat.py:363-556).
// Reference call sequence of the all-modality action head:
//   rldx/inference/action_model/model/graph_safe_action_model.py:170-312   (loop structure)
//   rldx/inference/action_model/engine/custom_expanded_action_model_chain.py:51-66 (baked temb,
//       time tokens and positional embeddings)
//   rldx/model/modules/action_model/msat.py:558-781  (_forward_physics, output projections)
//   rldx/model/modules/action_model/blocks.py:705-891 (ExpandedDoubleStreamBlock.forward)
//   rldx/model/modules/embodiment_conditioned_mlp.py:146-227 (category MLPs, action encoder)
//   rldx/model/modules/action_model/physics.py:9-70 (physics encoders / decoder)
//
// Buffer layout in HBM ("stream-major"): every stream keeps its own [B * tokens, dim] matrix
// (cognition X_vl, action X_sa = [time | state | actions], physics X_p = [hist | fut]); the QKV
// epilogue scatters into the joint attention layout Q, K [B, H, L, 64] and V^T [B, H, 64, Lp]
// with L = n_vl + n_sa + n_p, and attention writes its output back per stream.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <stdexcept>
#include <vector>

#include "host_util.h"

namespace rldx {
namespace {

using bf16 = __nv_bfloat16;

struct Op {
  enum Kind { kGemm, kAttn, kLn, kCopy, kStatus, kMask } kind;
  int grid;
  double bytes, flops;  // algorithmic traffic / work of the launch
  GemmParams g;
  AttnParams a;
  LnParams l;
  CopyParams c;
  unsigned int* slot;  // kStatus: device address of the status word this launch fills
};

uint16_t f2bf_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return static_cast<uint16_t>((u >> 16) | ((u & 0xffffu) ? 0x40u : 0u));
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return static_cast<uint16_t>(u >> 16);
}
float bf_round(float f) {
  uint32_t u = static_cast<uint32_t>(f2bf_bits(f)) << 16;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

// K-split GEMMs in the control step: on by default (the planner splits where its cost model
// says idle SMs outweigh the partial-tile traffic, chiefly the K = 4096 MLP down-projection);
// RLDX_MSAT_SPLIT_K=0 turns them off.
bool split_k_enabled() {
  const char* e = std::getenv("RLDX_MSAT_SPLIT_K");
  return !(e && e[0] == '0');
}

struct Fail : std::runtime_error {
  int code;
  Fail(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Fail(RLDX_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Sinusoid of SinusoidalPositionalEncoding (embodiment_conditioned_mlp.py:39-59): [sin | cos].
void sinusoid_sin_cos(float t, int dim, uint16_t* out) {
  const int half = dim / 2;
  const float scale = logf(10000.0f) / static_cast<float>(half);
  for (int i = 0; i < half; ++i) {
    const float e = -static_cast<float>(i) * scale;
    const float f = t * expf(e);
    out[i] = f2bf_bits(sinf(f));
    out[half + i] = f2bf_bits(cosf(f));
  }
}

// diffusers Timesteps(num_channels, flip_sin_to_cos=True, downscale_freq_shift=1): [cos | sin].
void timestep_proj(float t, int channels, uint16_t* out) {
  const int half = channels / 2;
  const float neg_log = static_cast<float>(-std::log(10000.0));
  for (int i = 0; i < half; ++i) {
    float e = neg_log * static_cast<float>(i);
    e = e / static_cast<float>(half - 1);
    const float f = t * expf(e);
    out[i] = f2bf_bits(cosf(f));
    out[half + i] = f2bf_bits(sinf(f));
  }
}

}  // namespace
}  // namespace rldx

using namespace rldx;

struct rldx_msat {
  rldx_msat_config c{};
  int device = 0;
  std::vector<void*> allocs;
  int B = 0, nvl = 0, nsa = 0, np = 0, L = 0, Lp = 0, D = 0, H = 0, hc = 0, S = 0;
  bool standard = false;  // no physics stream
  int Dv = 0;             // VL stream width in the double blocks
  int nx = 0;             // single-block x stream tokens per observation: [VL_proj | time | S/A]
  int E = 0, Mh = 0;      // single-block SwiGLU width and mlp_proj output width

  struct StreamW {
    bf16 *qkv_w, *qkv_b, *proj_w, *proj_b, *w12_w, *w12_b, *w3_w, *w3_b, *qn, *kn;
    int hidden;
  };
  std::vector<StreamW> wvl, wsa, wp;
  struct SingleW {
    bf16 *qkv_w, *qkv_b, *w12_w, *w12_b, *mp_w, *mp_b, *l2_w, *l2_b, *qn, *kn;
  };
  std::vector<SingleW> sgx, sgp;  // single blocks: x stream, physics stream (expanded form)
  bf16 *vlp_w = nullptr, *vlp_b = nullptr;  // vl_proj_to_sa (null: identity)
  float *rope_cos_s = nullptr, *rope_sin_s = nullptr;
  // Single-block row groups [VL_proj | time, S/A | P].  The x stream is the first two groups:
  // they share the x weights and run as two problems of one grouped GEMM, so the S/A rows stay
  // in xsa and VL_proj is xvl itself when vl_proj_to_sa is the identity.  The joint sequence
  // has the same length L as in the double blocks.
  bf16* sx[3] = {};    // group rows (residual stream)
  bf16* sln[3] = {};   // pre_norm output
  bf16* sh[3] = {};    // silu(x1) * x2
  bf16* scat[3] = {};  // [attention | mlp_proj] = linear2 input, row width inner + Mh
  bf16 *po2_w = nullptr, *po2_b = nullptr, *pp2_w = nullptr, *pp2_b = nullptr;
  bf16 *st1_W, *st1_b, *st2_W, *st2_b, *aw1_W, *aw1_b, *aw2_W, *aw2_b, *aw3_W, *aw3_b;
  bf16 *dl1_W, *dl1_b, *dl2_W, *dl2_b, *pos;
  bf16 *phc1_w, *phc1_b, *phc2_w, *phc2_b, *phc3_w, *phc3_b;
  bf16 *phf1_w, *phf1_b, *phf2_w, *phf2_b, *phf3_w, *phf3_b;
  bf16 *phd1_w, *phd1_b, *phd2_w, *phd2_b;
  int sdp = 0, adp = 0;  // padded state / action dims (multiples of 8)

  float *rope_cos = nullptr, *rope_sin = nullptr;
  // host copies of the two [L, 32] tables (double blocks, single blocks): which rows rotate
  std::vector<float> host_cos[2], host_sin[2];
  bf16 *time_tok = nullptr, *ada_sc1p = nullptr, *ada_shift = nullptr, *pada_sc1p = nullptr,
       *pada_shift = nullptr;

  bf16 *vl_in, *xvl, *xsa, *xp, *lnvl, *lnsa, *lnp, *q, *k, *vt, *ovl, *osa, *op, *hvl, *hsa, *hp;
  bf16 *state_in, *state_h, *state_feat, *x, *act_h, *phf_h, *phc_cat, *phc_h, *phist;
  bf16 *phys_hist_in, *phys_x, *oln_sa, *oln_p, *oproj_sa, *oproj_p, *dec_h, *pdec_h;
  int64_t* emb = nullptr;
  std::vector<bf16*> act_cat, phf_cat;

  std::vector<Op> ops;
  // Masked form of the step (cfg.key_mask): the same launches, the attention ones reading the key
  // mask kmask [B, L], built in the graph from the per-step inputs vlmask_in / pmask_in
  std::vector<Op> ops_m;
  uint8_t *kmask = nullptr, *vlmask_in = nullptr, *pmask_in = nullptr;
  cudaGraph_t graph_m = nullptr;
  cudaGraphExec_t exec_m = nullptr;
  // block_marks[step * nblocks + i]: launches from the start of the list up to and including
  // the last one of block i (double blocks, then single blocks) of Euler step `step`
  std::vector<int> block_marks;
  std::vector<int> step_marks;  // launches before the first block of each Euler step
  StepStatus status;
  // K-split workspace shared by every GEMM launch of the step (launches are stream-ordered):
  // tile arrival counters (zero between launches) followed by fp32 partial tiles.
  void* gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0, ws_need = 0;
  bool sizing = false;
  cudaStream_t stream = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  bool pdl = true;

  // Every bind-time copy, fill and re-layout kernel runs in order on the handle's own stream:
  // the legacy-stream forms (cudaMemcpy / cudaMemset) return before a device-to-device copy
  // has landed and are not ordered with a non-blocking stream, so a re-layout kernel on
  // `stream` could read a weight half copied.
  template <class T>
  T* alloc(size_t n) {
    void* p = nullptr;
    ck(cudaMalloc(&p, n * sizeof(T) + 256), "cudaMalloc");
    allocs.push_back(p);
    ck(cudaMemsetAsync(p, 0, n * sizeof(T) + 256, stream), "cudaMemset");
    return static_cast<T*>(p);
  }

  void copy(void* dst, const void* src, size_t bytes, const char* what) {
    ck(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream), what);
  }

  void release(void* p) {
    auto it = std::find(allocs.begin(), allocs.end(), p);
    if (it != allocs.end()) {
      ck(cudaStreamSynchronize(stream), "release sync");  // no queued work still reads it
      cudaFree(p);
      allocs.erase(it);
    }
  }

  bf16* copy_in(const void* src, size_t n, const char* what) {
    if (!src) throw Fail(RLDX_ERR_ARG, std::string("missing weight: ") + what);
    bf16* d = alloc<bf16>(n);
    copy(d, src, n * 2, what);
    return d;
  }

  // [rows, K] -> [rows, Kp] zero-padded
  bf16* copy_pad(const void* src, int rows, int K, int Kp, const char* what) {
    if (!src) throw Fail(RLDX_ERR_ARG, std::string("missing weight: ") + what);
    bf16* d = alloc<bf16>(static_cast<size_t>(rows) * Kp);
    ck(cudaMemcpy2DAsync(d, Kp * 2, src, K * 2, K * 2, rows, cudaMemcpyDefault, stream), what);
    return d;
  }

  // CategorySpecificLinear.W [cats, K, N] -> [cats, N, Kp]
  bf16* cat_weight(const void* W, int K, int N, int Kp, const char* what) {
    if (!W) throw Fail(RLDX_ERR_ARG, std::string("missing weight: ") + what);
    const int cats = c.num_embodiments;
    bf16* tmp = alloc<bf16>(static_cast<size_t>(cats) * K * N);
    copy(tmp, W, static_cast<size_t>(cats) * K * N * 2, what);
    bf16* d = alloc<bf16>(static_cast<size_t>(cats) * N * Kp);
    ck(launch_transpose_cat(tmp, d, cats, K, N, Kp, stream), "transpose");
    ck(cudaStreamSynchronize(stream), "transpose sync");
    release(tmp);
    return d;
  }

  // SwiGLUFFN.w12 [2h, dim] (gate rows then up rows) -> [32 gate | 32 up] row groups over hp =
  // h rounded up to 32; the padded gate / up rows are zero (silu(0) * 0 = 0, and w3's padded
  // columns are zero too), so a hidden size like int(2/3 * 16384) = 10922 runs exactly.
  void w12_interleave(const rldx_linear& l, int hidden, int hp, int dim, bf16** w, bf16** b) {
    if (!l.w || !l.b) throw Fail(RLDX_ERR_ARG, "missing w12");
    if (hp % 32 || hp < hidden) throw Fail(RLDX_ERR_UNSUPPORTED, "padded SwiGLU hidden must be a multiple of 32");
    const int zero_row = 2 * hidden;  // one zero row after the source rows
    std::vector<int> idx(2 * hp);
    for (int g = 0; g < hp / 32; ++g)
      for (int i = 0; i < 32; ++i) {
        const int r = g * 32 + i;
        idx[g * 64 + i] = r < hidden ? r : zero_row;
        idx[g * 64 + 32 + i] = r < hidden ? hidden + r : zero_row;
      }
    int* didx = alloc<int>(idx.size());
    copy(didx, idx.data(), idx.size() * 4, "idx");
    bf16* src = alloc<bf16>(static_cast<size_t>(2 * hidden + 1) * dim);  // zero-filled
    copy(src, l.w, static_cast<size_t>(2) * hidden * dim * 2, "w12");
    *w = alloc<bf16>(static_cast<size_t>(2) * hp * dim);
    ck(launch_gather_rows(src, dim, *w, dim, didx, 2 * hp, dim, stream), "gather");
    bf16* bsrc = alloc<bf16>(static_cast<size_t>(2 * hidden + 1));
    copy(bsrc, l.b, static_cast<size_t>(2) * hidden * 2, "w12 bias");
    *b = alloc<bf16>(static_cast<size_t>(2) * hp);
    ck(launch_gather_rows(bsrc, 1, *b, 1, didx, 2 * hp, 1, stream), "gather bias");
    ck(cudaStreamSynchronize(stream), "gather sync");
    release(src);
    release(bsrc);
    release(didx);
  }

  static int pad32(int v) { return (v + 31) / 32 * 32; }

  StreamW bind_stream(const rldx_stream_weights& s, int hidden, int width) {
    StreamW w{};
    const size_t inner = static_cast<size_t>(H) * 64;
    const int hp = pad32(hidden);
    w.hidden = hp;
    w.qkv_w = copy_in(s.qkv.w, 3 * inner * width, "qkv.w");
    w.qkv_b = copy_in(s.qkv.b, 3 * inner, "qkv.b");
    w.proj_w = copy_in(s.proj.w, static_cast<size_t>(width) * inner, "proj.w");
    w.proj_b = copy_in(s.proj.b, width, "proj.b");
    w12_interleave(s.w12, hidden, hp, width, &w.w12_w, &w.w12_b);
    w.w3_w = copy_pad(s.w3.w, width, hidden, hp, "w3.w");  // [width, hidden] -> [width, hp], zero columns
    w.w3_b = copy_in(s.w3.b, width, "w3.b");
    w.qn = copy_in(s.q_norm, 64, "q_norm");
    w.kn = copy_in(s.k_norm, 64, "k_norm");
    return w;
  }

  // SingleStreamBlock weights: linear1 = [q | k | v | gate | up] rows, split into the QKV part
  // and the SwiGLU part (re-laid as [32 gate | 32 up] row groups); mlp_proj; linear2.
  SingleW bind_single(const rldx_linear& l1, const rldx_linear& l2, const rldx_linear& mp,
                      const void* qn, const void* kn) {
    SingleW w{};
    const size_t inner3 = static_cast<size_t>(3) * H * 64;
    const size_t inner = static_cast<size_t>(H) * 64;
    if (!l1.w || !l1.b) throw Fail(RLDX_ERR_ARG, "missing single block linear1");
    w.qkv_w = copy_in(l1.w, inner3 * D, "linear1.w (qkv)");
    w.qkv_b = copy_in(l1.b, inner3, "linear1.b (qkv)");
    rldx_linear l12;
    l12.w = static_cast<const uint16_t*>(l1.w) + inner3 * D;
    l12.b = static_cast<const uint16_t*>(l1.b) + inner3;
    w12_interleave(l12, E, E, D, &w.w12_w, &w.w12_b);
    w.mp_w = copy_in(mp.w, static_cast<size_t>(Mh) * E, "mlp_proj.w");
    w.mp_b = copy_in(mp.b, Mh, "mlp_proj.b");
    w.l2_w = copy_in(l2.w, static_cast<size_t>(D) * (inner + Mh), "linear2.w");
    w.l2_b = copy_in(l2.b, D, "linear2.b");
    w.qn = copy_in(qn, 64, "q_norm");
    w.kn = copy_in(kn, 64, "k_norm");
    return w;
  }

  // ---- GEMM description helpers ----
  static rldx_gemm_desc lin(const bf16* a, int lda, const bf16* w, const bf16* b, int M, int N,
                            int K, bf16* out, int ldo) {
    rldx_gemm_desc d;
    std::memset(&d, 0, sizeof(d));
    d.a = a;
    d.lda = lda;
    d.b = w;
    d.ldb = K;
    d.M = M;
    d.N = N;
    d.K = K;
    d.bias = b;
    d.bias_mode = b ? RLDX_BIAS_FUSED : RLDX_BIAS_NONE;
    d.out = out;
    d.ldo = ldo;
    d.epilogue = RLDX_EPI_STORE;
    d.eps = 1e-6f;
    return d;
  }
  rldx_gemm_desc catlin(const bf16* a, int lda, const bf16* W, const bf16* b, int M, int N, int Kp,
                        int rows_per_cat, bf16* out, int ldo) const {
    rldx_gemm_desc d = lin(a, lda, W, b, M, N, Kp, out, ldo);
    d.cat_ids = emb;
    d.rows_per_cat = rows_per_cat;
    d.num_cats = c.num_embodiments;
    d.b_cat_stride = static_cast<int64_t>(N) * Kp;
    d.bias_cat_stride = N;
    d.bias_mode = RLDX_BIAS_POST_ROUND;
    return d;
  }

  void push_gemm(std::initializer_list<rldx_gemm_desc> ds) { push_gemm(std::vector<rldx_gemm_desc>(ds)); }
  void push_gemm(const std::vector<rldx_gemm_desc>& v) {
    Op o;
    std::memset(&o, 0, sizeof(o));
    o.kind = Op::kGemm;
    std::string err;
    size_t need = 0;
    if (!build_gemm_params(v.data(), static_cast<int>(v.size()), sizing ? nullptr : gemm_ws,
                           sizing ? 0 : gemm_ws_bytes, &o.g, sizing ? &need : nullptr, &err))
      throw Fail(RLDX_ERR_ARG, err);
    ws_need = std::max(ws_need, need);
    o.grid = o.g.ncta;
    for (const rldx_gemm_desc& d : v) {
      const double M = d.M, N = d.N, K = d.K;
      const double slabs = d.cat_ids ? static_cast<double>(d.M / d.rows_per_cat) : 1.0;
      const double nout = (d.epilogue == RLDX_EPI_SWIGLU) ? N / 2 : N;
      o.bytes += 2.0 * (slabs * N * K + M * K + M * nout);
      if (d.epilogue == RLDX_EPI_EULER) o.bytes += 2.0 * M * N;
      if (d.add) o.bytes += 2.0 * (d.add_row_mod > 0 ? d.add_row_mod : M) * N;
      o.flops += 2.0 * M * N * K;
    }
    ops.push_back(o);
  }

  void push_ln(const std::vector<LnSegment>& segs) {
    Op o;
    std::memset(&o, 0, sizeof(o));
    o.kind = Op::kLn;
    int row = 0, n = 0, dmax = 0;
    double elems = 0.0;
    for (const LnSegment& s : segs) {
      o.l.seg[n] = s;
      o.l.seg[n].row_begin = row;
      const int w = s.D > 0 ? s.D : D;
      o.l.seg[n].D = w;
      dmax = std::max(dmax, w);
      elems += static_cast<double>(s.rows) * w;
      row += s.rows;
      ++n;
    }
    o.l.nseg = n;
    o.l.D = dmax;
    o.l.total_rows = row;
    o.l.eps = 1e-6f;
    o.grid = (row + 7) / 8;
    o.bytes = 4.0 * elems;
    o.flops = 8.0 * elems;
    ops.push_back(o);
  }

  // QKV projection of one stream / row group with the fused RMS QK-norm + RoPE epilogue that
  // scatters q, k (and v transposed) into the joint sequence at token offset tok_off.
  rldx_gemm_desc qkv_desc(const bf16* a, int width, const bf16* w, const bf16* b, const bf16* qn,
                          const bf16* kn, int rows, int tok_off, const float* rc, const float* rs) const {
    const int inner = H * 64;
    rldx_gemm_desc d = lin(a, width, w, b, B * rows, 3 * inner, width, q, inner);
    d.epilogue = RLDX_EPI_QKV;
    d.q_norm_w = qn;
    d.k_norm_w = kn;
    d.rope_cos = rc;
    d.rope_sin = rs;
    d.q = q;
    d.k = k;
    d.vt = vt;
    d.L = L;
    d.Lp = Lp;
    d.H = H;
    d.tok_off = tok_off;
    d.rows_in = rows;
    d.rows_out = rows;
    // rows whose table entries are all cos 1 / sin 0 (position 0 on both axes: the VL tokens
    // under rope_sa_only) need no rotation: the epilogue then reads no tables
    const int which = (rc == rope_cos) ? 0 : 1;
    bool identity = !host_cos[which].empty();
    for (int t = tok_off; identity && t < tok_off + rows; ++t)
      for (int p = 0; p < 32 && identity; ++p)
        identity = host_cos[which][static_cast<size_t>(t) * 32 + p] == 1.0f &&
                   host_sin[which][static_cast<size_t>(t) * 32 + p] == 0.0f;
    d.rope_identity = identity ? 1 : 0;
    (void)rs;
    return d;
  }

  // Joint attention over the L tokens of each observation; query rows of segment i go to
  // outs[i] (row stride lds[i], or H*64 when lds is null).
  void push_attn(bf16* const* outs, const int* lens, const int* lds, int nseg) {
    Op o;
    std::memset(&o, 0, sizeof(o));
    o.kind = Op::kAttn;
    AttnParams& a = o.a;
    a.L = L;
    a.H = H;
    a.B = B;
    a.key_mask = nullptr;
    for (int i = 0; i < nseg; ++i) {
      a.seg_out[i] = outs[i];
      a.seg_len[i] = lens[i];
      a.seg_ld[i] = lds ? lds[i] : 0;
    }
    a.nseg = nseg;
    a.scale_log2 = 1.4426950408889634f / 8.0f;
    std::string err;
    const uint64_t bh = static_cast<uint64_t>(B) * H;
    o.grid = ((L + 127) / 128) * H * B;
    o.bytes = 2.0 * 4.0 * static_cast<double>(bh) * L * 64;
    o.flops = 4.0 * static_cast<double>(bh) * L * L * 64;
    if (!make_tmap_3d(&a.tq, q, 64, L, bh, 128, static_cast<uint64_t>(L) * 128, 64, 128, 1, &err) ||
        !make_tmap_3d(&a.tk, k, 64, L, bh, 128, static_cast<uint64_t>(L) * 128, 64, 64, 1, &err) ||
        !make_tmap_3d(&a.tv, vt, L, 64, bh, static_cast<uint64_t>(Lp) * 2, static_cast<uint64_t>(Lp) * 128, 64, 64, 1,
                      &err))
      throw Fail(RLDX_ERR_ARG, err);
    ops.push_back(o);
  }

  void push_copy(const std::vector<CopyRegion>& rs) {
    Op o;
    std::memset(&o, 0, sizeof(o));
    o.kind = Op::kCopy;
    for (size_t i = 0; i < rs.size(); ++i) o.c.r[i] = rs[i];
    o.c.n = static_cast<int>(rs.size());
    o.grid = 2 * sm_count();
    for (const CopyRegion& r : rs) o.bytes += 2.0 * r.rows * r.bytes;
    ops.push_back(o);
  }

  void push_status(int which) {
    Op o;
    std::memset(&o, 0, sizeof(o));
    o.kind = Op::kStatus;
    o.grid = 1;
    o.slot = status.dev + which;
    ops.push_back(o);
  }

  // Launches ops [0, n) of `list` (all of them when n < 0; `list` null: the unmasked step).
  void run_ops(cudaStream_t st, cudaEvent_t* ev = nullptr, int n = -1, const std::vector<Op>* list = nullptr) {
    const std::vector<Op>& L_ = list ? *list : ops;
    if (ev) ck(cudaEventRecord(ev[0], st), "event");
    const size_t end = n < 0 ? L_.size() : std::min(L_.size(), static_cast<size_t>(n));
    for (size_t i = 0; i < end; ++i) {
      const Op& o = L_[i];
      const bool p = pdl && i > 0 && !ev && L_[i - 1].kind != Op::kStatus && L_[i - 1].kind != Op::kMask;
      cudaError_t e = cudaSuccess;
      switch (o.kind) {
        case Op::kGemm:
          e = launch_gemm(o.g, st, p);
          break;
        case Op::kAttn:
          e = launch_attention(o.a, st, p);
          break;
        case Op::kLn:
          e = launch_ln(o.l, st, p);
          break;
        case Op::kCopy:
          e = launch_copy(o.c, o.grid, st, p);
          break;
        case Op::kStatus:
          e = launch_status_take(o.slot, st);
          break;
        case Op::kMask:
          e = launch_key_mask(kmask, vlmask_in, pmask_in, B, L, nvl, nsa, st);
          break;
      }
      ck(e, "launch");
      if (ev) ck(cudaEventRecord(ev[i + 1], st), "event");
    }
  }

  // Per-step key masks into the static mask inputs (an absent mask: every key visible).
  void copy_masks(const rldx_msat_io* io, cudaStream_t st) {
    if (io->vl_mask)
      ck(cudaMemcpyAsync(vlmask_in, io->vl_mask, static_cast<size_t>(B) * nvl, cudaMemcpyDefault, st), "vl_mask");
    else
      ck(cudaMemsetAsync(vlmask_in, 1, static_cast<size_t>(B) * nvl, st), "vl_mask");
    if (io->physics_mask)
      ck(cudaMemcpyAsync(pmask_in, io->physics_mask, static_cast<size_t>(B), cudaMemcpyDefault, st), "physics_mask");
    else
      ck(cudaMemsetAsync(pmask_in, 1, static_cast<size_t>(B), st), "physics_mask");
  }

  void copy_inputs(const rldx_msat_io* io, cudaStream_t st) {
    ck(cudaMemcpyAsync(vl_in, io->vl, static_cast<size_t>(B) * nvl * Dv * 2, cudaMemcpyDefault, st), "vl");
    ck(cudaMemcpy2DAsync(state_in, sdp * 2, io->state, c.state_dim * 2, c.state_dim * 2,
                         static_cast<size_t>(B) * c.n_state, cudaMemcpyDefault, st),
       "state");
    ck(cudaMemcpyAsync(emb, io->emb_id, static_cast<size_t>(B) * 8, cudaMemcpyDefault, st), "emb");
    ck(cudaMemcpyAsync(x, io->init_noise, static_cast<size_t>(B) * c.horizon * c.action_dim * 2,
                       cudaMemcpyDefault, st),
       "noise");
    if (c.prefix_len > 0) {  // RTC trained mode: the prefix rows of x hold the frozen actions
      const size_t row = static_cast<size_t>(c.action_dim) * 2;
      ck(cudaMemcpy2DAsync(x, c.horizon * row, io->prefix_actions, c.prefix_len * row, c.prefix_len * row, B,
                           cudaMemcpyDefault, st),
         "prefix_actions");
    }
    if (standard) return;
    ck(cudaMemcpy2DAsync(phys_hist_in, hc * 2, io->physics_hist, c.physics_dim * 2, c.physics_dim * 2,
                         static_cast<size_t>(B) * c.physics_hist, cudaMemcpyDefault, st),
       "physics_hist");
    ck(cudaMemcpy2DAsync(phys_x, hc * 2, io->physics_noise, c.physics_dim * 2, c.physics_dim * 2,
                         static_cast<size_t>(B) * c.physics_fut, cudaMemcpyDefault, st),
       "physics_noise");
  }

  void copy_outputs(const rldx_msat_io* io, cudaStream_t st) {
    ck(cudaMemcpyAsync(io->actions, x, static_cast<size_t>(B) * c.horizon * c.action_dim * 2,
                       cudaMemcpyDefault, st),
       "actions");
  }

  void create(const rldx_msat_config& cfg, const rldx_msat_weights& w);
  void precompute(const rldx_msat_weights& w);
  void plan();
};

void rldx_msat::create(const rldx_msat_config& cfg, const rldx_msat_weights& w) {
  c = cfg;
  if (c.head_dim != 64) throw Fail(RLDX_ERR_UNSUPPORTED, "head_dim must be 64");
  if (c.dim != c.heads * c.head_dim) throw Fail(RLDX_ERR_UNSUPPORTED, "dim must equal heads * head_dim");
  if (c.batch <= 0 || c.n_vl <= 0 || c.horizon <= 0 || c.depth <= 0 || c.num_steps <= 0)
    throw Fail(RLDX_ERR_ARG, "batch, n_vl, horizon, depth, num_steps must be positive");
  standard = c.standard_path != 0;
  Dv = c.vl_dim > 0 ? c.vl_dim : c.dim;
  if (!standard && c.physics_fut != c.horizon) throw Fail(RLDX_ERR_UNSUPPORTED, "physics_fut must equal horizon");
  if (c.n_state <= 0 || 1 + c.n_state + c.horizon > 128 || c.horizon > 128 ||
      (!standard && c.physics_hist + c.physics_fut > 128))
    throw Fail(RLDX_ERR_UNSUPPORTED, "per-observation action / physics streams must fit 128 rows");
  if (c.dim % 64 || Dv % 64 || c.mlp_hidden <= 0 || c.vl_mlp_hidden <= 0 || c.out_dim % 8 || c.dec_hidden % 8)
    throw Fail(RLDX_ERR_UNSUPPORTED, "dims must be multiples of 64 (dim, vl_dim) / 8 (out_dim, dec_hidden)");
  if (c.dim > 4096 || Dv > 4096) throw Fail(RLDX_ERR_UNSUPPORTED, "dim / vl_dim > 4096");
  if (!standard && (c.physics_dim <= 0 || c.physics_hist <= 0))
    throw Fail(RLDX_ERR_UNSUPPORTED, "the all-modality path needs the physics stream");
  if (c.depth_single < 0) throw Fail(RLDX_ERR_ARG, "depth_single must be >= 0");
  if (c.prefix_len < 0 || c.prefix_len >= c.horizon) throw Fail(RLDX_ERR_ARG, "prefix_len must be in [0, horizon)");
  if (c.depth_single > 0) {
    if (!w.single_blocks) throw Fail(RLDX_ERR_ARG, "missing single block weights");
    if (c.single_expanded <= 0 || c.single_expanded % 32 || c.single_mlp_hidden <= 0 ||
        c.single_mlp_hidden % 8)
      throw Fail(RLDX_ERR_UNSUPPORTED, "single-block widths must be multiples of 32 (SwiGLU) / 8");
    if (Dv != c.dim && !w.vl_proj_to_sa.w) throw Fail(RLDX_ERR_ARG, "missing vl_proj_to_sa");
  }
  if (!w.blocks) throw Fail(RLDX_ERR_ARG, "missing block weights");
  if (standard) c.physics_hist = c.physics_fut = c.physics_dim = 0;  // no physics buffers
  if (w.time_token_proj.w) throw Fail(RLDX_ERR_UNSUPPORTED, "time_token_proj must be identity (inner == sa_dim)");
  ck(cudaGetDevice(&device), "cudaGetDevice");
  ck(cudaDeviceSynchronize(), "weights ready");  // the caller's weights may come from any stream
  const char* env = getenv("RLDX_PDL");
  pdl = !(env && env[0] == '0');

  B = c.batch;
  D = c.dim;
  H = c.heads;
  nvl = c.n_vl;
  nsa = 1 + c.n_state + c.horizon;
  np = standard ? 0 : c.physics_hist + c.physics_fut;
  L = nvl + nsa + np;
  Lp = (L + 7) / 8 * 8;
  nx = nvl + nsa;
  E = c.single_expanded;
  Mh = c.single_mlp_hidden;
  S = c.num_steps;
  hc = (c.physics_dim + 7) / 8 * 8;
  sdp = (c.state_dim + 7) / 8 * 8;
  adp = (c.action_dim + 7) / 8 * 8;
  if (adp != c.action_dim) throw Fail(RLDX_ERR_UNSUPPORTED, "action_dim must be a multiple of 8");
  ck(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");

  // ---- weights ----
  for (int i = 0; i < c.depth; ++i) {
    const rldx_block_weights& bw = w.blocks[i];
    wvl.push_back(bind_stream(bw.vl, c.vl_mlp_hidden, Dv));
    wsa.push_back(bind_stream(bw.sa, c.mlp_hidden, D));
    if (!standard) wp.push_back(bind_stream(bw.p, c.mlp_hidden, D));
  }
  for (int i = 0; i < c.depth_single; ++i) {
    const rldx_single_block_weights& sw = w.single_blocks[i];
    sgx.push_back(bind_single(sw.linear1, sw.linear2, sw.mlp_proj, sw.q_norm, sw.k_norm));
    if (!standard) sgp.push_back(bind_single(sw.p_linear1, sw.p_linear2, sw.p_mlp_proj, sw.p_q_norm, sw.p_k_norm));
  }
  if (c.depth_single > 0 && Dv != D) {
    vlp_w = copy_in(w.vl_proj_to_sa.w, static_cast<size_t>(D) * Dv, "vl_proj_to_sa.w");
    vlp_b = copy_in(w.vl_proj_to_sa.b, D, "vl_proj_to_sa.b");
  }
  po2_w = copy_in(w.proj_out_2.w, static_cast<size_t>(c.out_dim) * D, "proj_out_2.w");
  po2_b = copy_in(w.proj_out_2.b, c.out_dim, "proj_out_2.b");
  if (!standard) {
    pp2_w = copy_in(w.proj_out_phys_2.w, static_cast<size_t>(c.out_dim) * D, "proj_out_physics_2.w");
    pp2_b = copy_in(w.proj_out_phys_2.b, c.out_dim, "proj_out_physics_2.b");
  }
  const int cats = c.num_embodiments;
  st1_W = cat_weight(w.state_l1.W, c.state_dim, c.dec_hidden, sdp, "state_encoder.layer1.W");
  st1_b = copy_in(w.state_l1.b, static_cast<size_t>(cats) * c.dec_hidden, "state_encoder.layer1.b");
  st2_W = cat_weight(w.state_l2.W, c.dec_hidden, D, c.dec_hidden, "state_encoder.layer2.W");
  st2_b = copy_in(w.state_l2.b, static_cast<size_t>(cats) * D, "state_encoder.layer2.b");
  aw1_W = cat_weight(w.act_w1.W, c.action_dim, D, adp, "action_encoder.W1.W");
  aw1_b = copy_in(w.act_w1.b, static_cast<size_t>(cats) * D, "action_encoder.W1.b");
  aw2_W = cat_weight(w.act_w2.W, 2 * D, D, 2 * D, "action_encoder.W2.W");
  aw2_b = copy_in(w.act_w2.b, static_cast<size_t>(cats) * D, "action_encoder.W2.b");
  aw3_W = cat_weight(w.act_w3.W, D, D, D, "action_encoder.W3.W");
  aw3_b = copy_in(w.act_w3.b, static_cast<size_t>(cats) * D, "action_encoder.W3.b");
  dl1_W = cat_weight(w.dec_l1.W, c.out_dim, c.dec_hidden, c.out_dim, "action_decoder.layer1.W");
  dl1_b = copy_in(w.dec_l1.b, static_cast<size_t>(cats) * c.dec_hidden, "action_decoder.layer1.b");
  dl2_W = cat_weight(w.dec_l2.W, c.dec_hidden, c.action_dim, c.dec_hidden, "action_decoder.layer2.W");
  dl2_b = copy_in(w.dec_l2.b, static_cast<size_t>(cats) * c.action_dim, "action_decoder.layer2.b");
  pos = copy_in(w.pos_emb, static_cast<size_t>(c.horizon) * D, "position_embedding");
  if (!standard) {
  phc1_w = copy_pad(w.phc_w1.w, D, c.physics_dim, hc, "physics_cond_encoder.W1");
  phc1_b = copy_in(w.phc_w1.b, D, "physics_cond_encoder.W1.b");
  phc2_w = copy_in(w.phc_w2.w, static_cast<size_t>(D) * 2 * D, "physics_cond_encoder.W2");
  phc2_b = copy_in(w.phc_w2.b, D, "physics_cond_encoder.W2.b");
  phc3_w = copy_in(w.phc_w3.w, static_cast<size_t>(D) * D, "physics_cond_encoder.W3");
  phc3_b = copy_in(w.phc_w3.b, D, "physics_cond_encoder.W3.b");
  phf1_w = copy_pad(w.phf_w1.w, D, c.physics_dim, hc, "physics_fut_encoder.W1");
  phf1_b = copy_in(w.phf_w1.b, D, "physics_fut_encoder.W1.b");
  phf2_w = copy_in(w.phf_w2.w, static_cast<size_t>(D) * 2 * D, "physics_fut_encoder.W2");
  phf2_b = copy_in(w.phf_w2.b, D, "physics_fut_encoder.W2.b");
  phf3_w = copy_in(w.phf_w3.w, static_cast<size_t>(D) * D, "physics_fut_encoder.W3");
  phf3_b = copy_in(w.phf_w3.b, D, "physics_fut_encoder.W3.b");
  phd1_w = copy_in(w.phd_l1.w, static_cast<size_t>(D) * c.out_dim, "physics_decoder.net.0");
  phd1_b = copy_in(w.phd_l1.b, D, "physics_decoder.net.0.b");
  phd2_w = copy_in(w.phd_l2.w, static_cast<size_t>(c.physics_dim) * D, "physics_decoder.net.2");
  phd2_b = copy_in(w.phd_l2.b, c.physics_dim, "physics_decoder.net.2.b");
  }

  // ---- activations ----
  const size_t inner = static_cast<size_t>(H) * 64;
  vl_in = alloc<bf16>(static_cast<size_t>(B) * nvl * Dv);
  xvl = alloc<bf16>(static_cast<size_t>(B) * nvl * Dv);
  xsa = alloc<bf16>(static_cast<size_t>(B) * nsa * D);
  xp = alloc<bf16>(static_cast<size_t>(B) * np * D);
  lnvl = alloc<bf16>(static_cast<size_t>(B) * nvl * Dv);
  lnsa = alloc<bf16>(static_cast<size_t>(B) * nsa * D);
  lnp = alloc<bf16>(static_cast<size_t>(B) * np * D);
  q = alloc<bf16>(static_cast<size_t>(B) * H * L * 64);
  k = alloc<bf16>(static_cast<size_t>(B) * H * L * 64);
  vt = alloc<bf16>(static_cast<size_t>(B) * H * 64 * Lp);
  if (c.depth_single > 0) {
    const int grows[3] = {nvl, nsa, np};
    sx[0] = (Dv != D) ? alloc<bf16>(static_cast<size_t>(B) * nvl * D) : xvl;
    sx[1] = xsa;
    sx[2] = xp;
    for (int g = 0; g < 3; ++g) {
      const size_t r = static_cast<size_t>(B) * grows[g];
      sln[g] = (g == 0) ? alloc<bf16>(r * D) : (g == 1 ? lnsa : lnp);
      sh[g] = alloc<bf16>(r * E);
      scat[g] = alloc<bf16>(r * (inner + Mh));
    }
  }
  ovl = alloc<bf16>(static_cast<size_t>(B) * nvl * inner);
  osa = alloc<bf16>(static_cast<size_t>(B) * nsa * inner);
  op = alloc<bf16>(static_cast<size_t>(B) * np * inner);
  hvl = alloc<bf16>(static_cast<size_t>(B) * nvl * pad32(c.vl_mlp_hidden));
  hsa = alloc<bf16>(static_cast<size_t>(B) * nsa * pad32(c.mlp_hidden));
  hp = alloc<bf16>(static_cast<size_t>(B) * np * pad32(c.mlp_hidden));
  state_in = alloc<bf16>(static_cast<size_t>(B) * c.n_state * sdp);
  state_h = alloc<bf16>(static_cast<size_t>(B) * c.n_state * c.dec_hidden);
  state_feat = alloc<bf16>(static_cast<size_t>(B) * c.n_state * D);
  emb = alloc<int64_t>(B);
  x = alloc<bf16>(static_cast<size_t>(B) * c.horizon * adp);
  for (int s = 0; s < S; ++s) {
    act_cat.push_back(alloc<bf16>(static_cast<size_t>(B) * c.horizon * 2 * D));
    phf_cat.push_back(alloc<bf16>(static_cast<size_t>(B) * c.physics_fut * 2 * D));
  }
  act_h = alloc<bf16>(static_cast<size_t>(B) * c.horizon * D);
  phf_h = alloc<bf16>(static_cast<size_t>(B) * c.physics_fut * D);
  phc_cat = alloc<bf16>(static_cast<size_t>(B) * c.physics_hist * 2 * D);
  phc_h = alloc<bf16>(static_cast<size_t>(B) * c.physics_hist * D);
  phist = alloc<bf16>(static_cast<size_t>(B) * c.physics_hist * D);
  phys_hist_in = alloc<bf16>(static_cast<size_t>(B) * c.physics_hist * hc);
  phys_x = alloc<bf16>(static_cast<size_t>(B) * c.physics_fut * hc);
  oln_sa = alloc<bf16>(static_cast<size_t>(B) * nsa * D);
  oln_p = alloc<bf16>(static_cast<size_t>(B) * np * D);
  oproj_sa = alloc<bf16>(static_cast<size_t>(B) * nsa * c.out_dim);
  oproj_p = alloc<bf16>(static_cast<size_t>(B) * np * c.out_dim);
  dec_h = alloc<bf16>(static_cast<size_t>(B) * nsa * c.dec_hidden);
  pdec_h = alloc<bf16>(static_cast<size_t>(B) * np * D);

  precompute(w);
  if (!status.init()) throw Fail(RLDX_ERR_CUDA, "step status: mapped host memory");
  if (split_k_enabled()) {
    sizing = true;  // first pass: workspace the K-split plans want
    plan();
    sizing = false;
    ops.clear();
    block_marks.clear();
    step_marks.clear();
    if (ws_need > 0) {
      gemm_ws = alloc<uint8_t>(ws_need);  // zero-filled: the tile counters start at zero
      gemm_ws_bytes = ws_need;
    }
  }
  plan();
  if (c.key_mask) {
    kmask = alloc<uint8_t>(static_cast<size_t>(B) * L);
    vlmask_in = alloc<uint8_t>(static_cast<size_t>(B) * nvl);
    pmask_in = alloc<uint8_t>(B);
    ck(cudaMemsetAsync(vlmask_in, 1, static_cast<size_t>(B) * nvl, stream), "mask fill");
    ck(cudaMemsetAsync(pmask_in, 1, B, stream), "mask fill");
    ops_m = ops;
    for (Op& o : ops_m)
      if (o.kind == Op::kAttn) o.a.key_mask = kmask;
    Op m;
    std::memset(&m, 0, sizeof(m));
    m.kind = Op::kMask;
    m.grid = 1;
    ops_m.insert(ops_m.begin() + 1, m);  // after the opening status launch
  }

  // Warm-up run (loads every kernel), then capture.
  run_ops(stream);
  if (c.key_mask) run_ops(stream, nullptr, -1, &ops_m);
  ck(cudaEventRecord(status.done, stream), "status event");
  ck(cudaStreamSynchronize(stream), "warm-up");
  unsigned int derr = 0, during = 0;
  if (status.read(true, &derr, &during) != RLDX_OK) throw Fail(RLDX_ERR_CUDA, "warm-up status");
  if (derr && during) throw Fail(RLDX_ERR_DEVICE, "device error during warm-up: " + std::to_string(derr));
  if (c.use_graph) {
    ck(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
      run_ops(stream);
    } catch (...) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    ck(cudaStreamEndCapture(stream, &graph), "end capture");
    ck(cudaGraphInstantiate(&exec, graph, 0), "instantiate");
    ck(cudaGraphUpload(exec, stream), "upload");
    if (c.key_mask) {
      ck(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "begin capture");
      try {
        run_ops(stream, nullptr, -1, &ops_m);
      } catch (...) {
        cudaGraph_t g = nullptr;
        cudaStreamEndCapture(stream, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      ck(cudaStreamEndCapture(stream, &graph_m), "end capture");
      ck(cudaGraphInstantiate(&exec_m, graph_m, 0), "instantiate");
      ck(cudaGraphUpload(exec_m, stream), "upload");
    }
    ck(cudaStreamSynchronize(stream), "upload sync");
  }
}

void rldx_msat::precompute(const rldx_msat_weights& w) {
  // ---- RoPE tables over the joint sequence [VL | time, S/A | P]: position ids of the double
  //      blocks (msat.py:583-631 with physics, msat.py:369-420 without) and of the single
  //      blocks (msat.py:460-505, 676-709), angles as ops.py:11-25 ----
  const int axes0 = (c.rope_mode == RLDX_ROPE_SA_ONLY) ? 16 : 48;
  const int axes1 = 64 - axes0;
  auto freq = [&](int dim, int i) {
    const float ex = static_cast<float>(2 * i) / static_cast<float>(dim);
    return 1.0f / powf(c.rope_theta, ex);
  };
  // S/A ids (after the time token at 0) start at 1 in the double blocks under rope_sa_only and
  // at 2 otherwise; the single blocks start them at 2 in both modes.
  // The module's per-axis tables when the binding passes them (exactly the reference's
  // values), else the same angles computed here.
  std::vector<float> mod_cos[2], mod_sin[2];
  const int axes[2] = {axes0, axes1};
  for (int a = 0; a < 2; ++a) {
    if (!w.rope_cos[a]) continue;
    const size_t n = static_cast<size_t>(c.rope_max_seq) * (axes[a] / 2);
    mod_cos[a].resize(n);
    mod_sin[a].assign(n, 0.0f);
    ck(cudaMemcpy(mod_cos[a].data(), w.rope_cos[a], n * 4, cudaMemcpyDefault), "rope table");
    if (!c.rope_cos_only) {
      if (!w.rope_sin[a]) throw Fail(RLDX_ERR_ARG, "rope_sin missing for a full-rotation table");
      ck(cudaMemcpy(mod_sin[a].data(), w.rope_sin[a], n * 4, cudaMemcpyDefault), "rope table");
    }
  }
  if (w.rope_cos[0] == nullptr || w.rope_cos[1] == nullptr) {
    mod_cos[0].clear();
    mod_cos[1].clear();
  }
  auto table = [&](int sa_start, float** dcos, float** dsin, int which) {
    std::vector<float> hc_cos(static_cast<size_t>(L) * 32), hc_sin(static_cast<size_t>(L) * 32);
    for (int t = 0; t < L; ++t) {
      int id0 = 0, id1 = 0;
      if (t < nvl) {
        if (c.rope_mode == RLDX_ROPE_VL_SA) id0 = t;
      } else if (t < nvl + nsa) {
        const int j = t - nvl;  // 0 = time token
        if (j > 0) id1 = sa_start + j - 1;
      } else {
        id0 = 1;
        id1 = t - nvl - nsa;
      }
      if (id0 >= c.rope_max_seq || id1 >= c.rope_max_seq)
        throw Fail(RLDX_ERR_ARG, "RoPE position beyond rope_max_seq");
      for (int p = 0; p < 32; ++p) {
        float cs, sn;
        if (!mod_cos[0].empty()) {
          const int a = p < axes0 / 2 ? 0 : 1;
          const size_t i = static_cast<size_t>(a == 0 ? id0 : id1) * (axes[a] / 2) + (a == 0 ? p : p - axes0 / 2);
          cs = mod_cos[a][i];
          sn = c.rope_cos_only ? 0.0f : mod_sin[a][i];
        } else {
          float ang;
          if (p < axes0 / 2)
            ang = static_cast<float>(id0) * freq(axes0, p);
          else
            ang = static_cast<float>(id1) * freq(axes1, p - axes0 / 2);
          cs = static_cast<float>(std::cos(static_cast<double>(ang)));
          sn = static_cast<float>(std::sin(static_cast<double>(ang)));
          if (c.rope_cos_only) {
            cs = bf_round(cs);
            sn = 0.0f;
          }
        }
        hc_cos[static_cast<size_t>(t) * 32 + p] = cs;
        hc_sin[static_cast<size_t>(t) * 32 + p] = sn;
      }
    }
    *dcos = alloc<float>(hc_cos.size());
    *dsin = alloc<float>(hc_sin.size());
    copy(*dcos, hc_cos.data(), hc_cos.size() * 4, "rope");
    copy(*dsin, hc_sin.data(), hc_sin.size() * 4, "rope");
    ck(cudaStreamSynchronize(stream), "rope sync");
    host_cos[which] = std::move(hc_cos);
    host_sin[which] = std::move(hc_sin);
  };
  table(c.rope_mode == RLDX_ROPE_SA_ONLY ? 1 : 2, &rope_cos, &rope_sin, 0);
  if (c.depth_single > 0) table(2, &rope_cos_s, &rope_sin_s, 1);

  // ---- timestep embedding per Euler step (ops.py:123-133), baked like
  //      custom_expanded_action_model_chain.py:57-66 ----
  std::vector<float> tvals(S);
  for (int s = 0; s < S; ++s) tvals[s] = bf_round(static_cast<float>(s) / static_cast<float>(S));
  const int tc = c.temb_channels;
  if (tc % 8 || tc <= 0) throw Fail(RLDX_ERR_UNSUPPORTED, "temb_channels must be a multiple of 8");
  std::vector<uint16_t> tproj(static_cast<size_t>(S) * tc);
  for (int s = 0; s < S; ++s) timestep_proj(tvals[s], tc, &tproj[static_cast<size_t>(s) * tc]);
  bf16* d_tproj = alloc<bf16>(tproj.size());
  copy(d_tproj, tproj.data(), tproj.size() * 2, "tproj");
  const size_t inner = static_cast<size_t>(H) * 64;
  bf16* t1 = alloc<bf16>(static_cast<size_t>(S) * inner);
  time_tok = alloc<bf16>(static_cast<size_t>(S) * inner);
  if (!w.temb_lin1.w || !w.temb_lin2.w) throw Fail(RLDX_ERR_ARG, "missing timestep embedder");
  std::string err;
  auto run = [&](std::initializer_list<rldx_gemm_desc> ds) {
    std::vector<rldx_gemm_desc> v(ds);
    static GemmParams gp;
    if (!build_gemm_params(v.data(), static_cast<int>(v.size()), nullptr, 0, &gp, nullptr, &err))
      throw Fail(RLDX_ERR_ARG, err);
    ck(launch_gemm(gp, stream, false), "bind gemm");
    ck(cudaStreamSynchronize(stream), "bind gemm sync");
  };
  {
    bf16* l1w = copy_in(w.temb_lin1.w, inner * tc, "temb linear_1");
    bf16* l1b = copy_in(w.temb_lin1.b, inner, "temb linear_1.b");
    bf16* l2w = copy_in(w.temb_lin2.w, inner * inner, "temb linear_2");
    bf16* l2b = copy_in(w.temb_lin2.b, inner, "temb linear_2.b");
    rldx_gemm_desc d1 = lin(d_tproj, tc, l1w, l1b, S, static_cast<int>(inner), tc, t1, static_cast<int>(inner));
    d1.act = RLDX_ACT_SILU;
    run({d1});
    run({lin(t1, static_cast<int>(inner), l2w, l2b, S, static_cast<int>(inner), static_cast<int>(inner), time_tok,
             static_cast<int>(inner))});
  }
  // time token = time_token_proj(temb) = identity here (inner == sa_dim); temb == time_tok.

  // ---- AdaLN scale / shift of the two output projections (msat.py:771-781) ----
  bf16* stemb = alloc<bf16>(static_cast<size_t>(S) * inner);
  ck(launch_elementwise(time_tok, stemb, static_cast<long long>(S) * inner, 0, stream), "silu");
  auto adaln = [&](const rldx_linear& l, bf16** sc1p, bf16** shift, const char* what) {
    bf16* lw = copy_in(l.w, static_cast<size_t>(2) * D * inner, what);
    bf16* lb = copy_in(l.b, static_cast<size_t>(2) * D, what);
    bf16* ss = alloc<bf16>(static_cast<size_t>(S) * 2 * D);
    run({lin(stemb, static_cast<int>(inner), lw, lb, S, 2 * D, static_cast<int>(inner), ss, 2 * D)});
    *shift = alloc<bf16>(static_cast<size_t>(S) * D);
    *sc1p = alloc<bf16>(static_cast<size_t>(S) * D);
    ck(cudaMemcpy2DAsync(*shift, D * 2, ss, 4 * D, D * 2, S, cudaMemcpyDeviceToDevice, stream), "shift");
    bf16* sc = alloc<bf16>(static_cast<size_t>(S) * D);
    ck(cudaMemcpy2DAsync(sc, D * 2, ss + D, 4 * D, D * 2, S, cudaMemcpyDeviceToDevice, stream), "scale");
    ck(launch_elementwise(sc, *sc1p, static_cast<long long>(S) * D, 1, stream), "1+scale");
  };
  adaln(w.proj_out_1, &ada_sc1p, &ada_shift, "proj_out_1");
  if (!standard) adaln(w.proj_out_phys_1, &pada_sc1p, &pada_shift, "proj_out_physics_1");

  // ---- sinusoids: action encoder / physics future encoder use t, the physics history
  //      encoder uses the token index (embodiment_conditioned_mlp.py:39-59, physics.py:19-25) ----
  // RTC trained mode: the prefix action tokens are encoded at t = 1 (clean), every step.
  std::vector<uint16_t> row(D), row_prefix(D);
  sinusoid_sin_cos(1.0f, D, row_prefix.data());
  for (int s = 0; s < S; ++s) {
    sinusoid_sin_cos(tvals[s], D, row.data());
    for (int r = 0; r < B * c.horizon; ++r)
      copy(act_cat[s] + static_cast<size_t>(r) * 2 * D + D,
           (r % c.horizon < c.prefix_len ? row_prefix : row).data(), D * 2, "tau");
    for (int r = 0; r < B * c.physics_fut; ++r)
      copy(phf_cat[s] + static_cast<size_t>(r) * 2 * D + D, row.data(), D * 2, "tau");
    ck(cudaStreamSynchronize(stream), "tau sync");  // `row` is rewritten for the next step
  }
  for (int t = 0; t < c.physics_hist; ++t) {
    sinusoid_sin_cos(static_cast<float>(t), D, row.data());
    for (int b = 0; b < B; ++b)
      copy(phc_cat + (static_cast<size_t>(b) * c.physics_hist + t) * 2 * D + D, row.data(), D * 2, "pos");
    ck(cudaStreamSynchronize(stream), "pos sync");  // `row` is rewritten for the next token
  }
  ck(cudaStreamSynchronize(stream), "precompute");
}

void rldx_msat::plan() {
  const int inner = H * 64;
  const int h = c.horizon;
  const int hist = c.physics_hist, fut = c.physics_fut;
  const float dt = 1.0f / static_cast<float>(S);
  const int ns = standard ? 2 : 3;  // streams / row groups: VL, SA (, P)
  push_status(0);  // a code left by earlier work -> slot 0; the step starts from a clean word

  // ---- once per control step: state encoder, physics history encoder ----
  {
    rldx_gemm_desc s1 = catlin(state_in, sdp, st1_W, st1_b, B * c.n_state, c.dec_hidden, sdp, c.n_state, state_h, c.dec_hidden);
    s1.act = RLDX_ACT_RELU;
    rldx_gemm_desc s2 = catlin(state_h, c.dec_hidden, st2_W, st2_b, B * c.n_state, D, c.dec_hidden, c.n_state, state_feat, D);
    if (standard) {
      push_gemm({s1});
      push_gemm({s2});
    } else {
      rldx_gemm_desc p1 = lin(phys_hist_in, hc, phc1_w, phc1_b, B * hist, D, hc, phc_cat, 2 * D);
      push_gemm({s1, p1});
      rldx_gemm_desc p2 = lin(phc_cat, 2 * D, phc2_w, phc2_b, B * hist, D, 2 * D, phc_h, D);
      p2.act = RLDX_ACT_SILU;
      push_gemm({s2, p2});
      push_gemm({lin(phc_h, D, phc3_w, phc3_b, B * hist, D, D, phist, D)});
    }
  }

  for (int s = 0; s < S; ++s) {
    // ---- stream initialisation: X_vl = vl, X_sa = [time token | state | .], X_p = [hist | .] ----
    {
      std::vector<CopyRegion> rs;
      CopyRegion r{};
      r.src = reinterpret_cast<const uint8_t*>(vl_in);
      r.dst = reinterpret_cast<uint8_t*>(xvl);
      r.src_pitch = r.dst_pitch = static_cast<long long>(Dv) * 2;
      r.rows = B * nvl;
      r.bytes = Dv * 2;
      rs.push_back(r);
      CopyRegion t{};
      t.src = reinterpret_cast<const uint8_t*>(time_tok + static_cast<size_t>(s) * inner);
      t.dst = reinterpret_cast<uint8_t*>(xsa);
      t.src_pitch = 0;
      t.dst_pitch = static_cast<long long>(nsa) * D * 2;
      t.rows = B;
      t.bytes = D * 2;
      rs.push_back(t);
      CopyRegion st{};
      st.src = reinterpret_cast<const uint8_t*>(state_feat);
      st.dst = reinterpret_cast<uint8_t*>(xsa + D);
      st.src_pitch = st.dst_pitch = static_cast<long long>(D) * 2;
      st.group_rows = c.n_state;
      st.src_group_pitch = static_cast<long long>(c.n_state) * D * 2;
      st.dst_group_pitch = static_cast<long long>(nsa) * D * 2;
      st.rows = B * c.n_state;
      st.bytes = D * 2;
      rs.push_back(st);
      if (!standard) {
        CopyRegion ph{};
        ph.src = reinterpret_cast<const uint8_t*>(phist);
        ph.dst = reinterpret_cast<uint8_t*>(xp);
        ph.src_pitch = ph.dst_pitch = static_cast<long long>(D) * 2;
        ph.group_rows = hist;
        ph.src_group_pitch = static_cast<long long>(hist) * D * 2;
        ph.dst_group_pitch = static_cast<long long>(np) * D * 2;
        ph.rows = B * hist;
        ph.bytes = D * 2;
        rs.push_back(ph);
      }
      push_copy(rs);
    }
    // ---- action encoder + physics future encoder ----
    {
      std::vector<rldx_gemm_desc> g1, g2, g3;
      g1.push_back(catlin(x, adp, aw1_W, aw1_b, B * h, D, adp, h, act_cat[s], 2 * D));
      rldx_gemm_desc a2 = catlin(act_cat[s], 2 * D, aw2_W, aw2_b, B * h, D, 2 * D, h, act_h, D);
      a2.act = RLDX_ACT_SWISH;
      g2.push_back(a2);
      rldx_gemm_desc a3 = catlin(act_h, D, aw3_W, aw3_b, B * h, D, D, h, xsa, D);
      a3.add = pos;
      a3.ld_add = D;
      a3.add_row_mod = h;
      a3.rows_in = h;
      a3.rows_out = nsa;
      a3.row_skip = -(1 + c.n_state);
      g3.push_back(a3);
      if (!standard) {
        g1.push_back(lin(phys_x, hc, phf1_w, phf1_b, B * fut, D, hc, phf_cat[s], 2 * D));
        rldx_gemm_desc f2 = lin(phf_cat[s], 2 * D, phf2_w, phf2_b, B * fut, D, 2 * D, phf_h, D);
        f2.act = RLDX_ACT_SILU;
        g2.push_back(f2);
        rldx_gemm_desc f3 = lin(phf_h, D, phf3_w, phf3_b, B * fut, D, D, xp, D);
        f3.rows_in = fut;
        f3.rows_out = np;
        f3.row_skip = -hist;
        g3.push_back(f3);
      }
      push_gemm(g1);
      push_gemm(g2);
      push_gemm(g3);
    }
    // ---- (Expanded)DoubleStreamBlocks over [VL | SA (| P)] ----
    bf16* xs[3] = {xvl, xsa, xp};
    bf16* lns[3] = {lnvl, lnsa, lnp};
    bf16* os[3] = {ovl, osa, op};
    bf16* hs[3] = {hvl, hsa, hp};
    const int rows[3] = {nvl, nsa, np};
    const int wd[3] = {Dv, D, D};
    const int toff[3] = {0, nvl, nvl + nsa};
    step_marks.push_back(static_cast<int>(ops.size()));
    for (int blk = 0; blk < c.depth; ++blk) {
      const StreamW* sw[3] = {&wvl[blk], &wsa[blk], standard ? nullptr : &wp[blk]};
      auto ln_all = [&]() {
        std::vector<LnSegment> v;
        for (int i = 0; i < ns; ++i)
          v.push_back(LnSegment{xs[i], lns[i], nullptr, nullptr, B * rows[i], wd[i], wd[i], 0, wd[i]});
        push_ln(v);
      };
      ln_all();
      {
        std::vector<rldx_gemm_desc> d(ns);
        for (int i = 0; i < ns; ++i)
          d[i] = qkv_desc(lns[i], wd[i], sw[i]->qkv_w, sw[i]->qkv_b, sw[i]->qn, sw[i]->kn, rows[i], toff[i],
                          rope_cos, rope_sin);
        push_gemm(d);
      }
      push_attn(os, rows, nullptr, ns);
      {
        std::vector<rldx_gemm_desc> d(ns);
        for (int i = 0; i < ns; ++i) {
          d[i] = lin(os[i], inner, sw[i]->proj_w, sw[i]->proj_b, B * rows[i], wd[i], inner, xs[i], wd[i]);
          d[i].add = xs[i];
          d[i].ld_add = wd[i];
        }
        push_gemm(d);
      }
      ln_all();
      {
        std::vector<rldx_gemm_desc> d(ns);
        for (int i = 0; i < ns; ++i) {
          const int hid = sw[i]->hidden;
          d[i] = lin(lns[i], wd[i], sw[i]->w12_w, sw[i]->w12_b, B * rows[i], 2 * hid, wd[i], hs[i], hid);
          d[i].epilogue = RLDX_EPI_SWIGLU;
        }
        push_gemm(d);
      }
      {
        std::vector<rldx_gemm_desc> d(ns);
        for (int i = 0; i < ns; ++i) {
          const int hid = sw[i]->hidden;
          d[i] = lin(hs[i], hid, sw[i]->w3_w, sw[i]->w3_b, B * rows[i], wd[i], hid, xs[i], wd[i]);
          d[i].add = xs[i];
          d[i].ld_add = wd[i];
        }
        push_gemm(d);
      }
      block_marks.push_back(static_cast<int>(ops.size()));
    }
    // ---- (Expanded)SingleStreamBlocks over [VL_proj | time, S/A (| P)] ----
    if (c.depth_single > 0) {
      if (Dv != D) push_gemm({lin(xvl, Dv, vlp_w, vlp_b, B * nvl, D, Dv, sx[0], D)});
      const int ld_cat = inner + Mh;
      for (int blk = 0; blk < c.depth_single; ++blk) {
        const SingleW* gw[3] = {&sgx[blk], &sgx[blk], standard ? nullptr : &sgp[blk]};
        {
          std::vector<LnSegment> v;
          for (int g = 0; g < ns; ++g)
            v.push_back(LnSegment{sx[g], sln[g], nullptr, nullptr, B * rows[g], D, D, 0, D});
          push_ln(v);
        }
        {
          std::vector<rldx_gemm_desc> d(ns);
          for (int g = 0; g < ns; ++g)
            d[g] = qkv_desc(sln[g], D, gw[g]->qkv_w, gw[g]->qkv_b, gw[g]->qn, gw[g]->kn, rows[g], toff[g],
                            rope_cos_s, rope_sin_s);
          push_gemm(d);
        }
        {
          std::vector<rldx_gemm_desc> d(ns);
          for (int g = 0; g < ns; ++g) {
            d[g] = lin(sln[g], D, gw[g]->w12_w, gw[g]->w12_b, B * rows[g], 2 * E, D, sh[g], E);
            d[g].epilogue = RLDX_EPI_SWIGLU;
          }
          push_gemm(d);
        }
        const int lds[3] = {ld_cat, ld_cat, ld_cat};
        push_attn(scat, rows, lds, ns);
        {
          std::vector<rldx_gemm_desc> d(ns);
          for (int g = 0; g < ns; ++g) {
            d[g] = lin(sh[g], E, gw[g]->mp_w, gw[g]->mp_b, B * rows[g], Mh, E, scat[g], ld_cat);
            d[g].col_off = inner;
          }
          push_gemm(d);
        }
        {
          std::vector<rldx_gemm_desc> d(ns);
          for (int g = 0; g < ns; ++g) {
            d[g] = lin(scat[g], ld_cat, gw[g]->l2_w, gw[g]->l2_b, B * rows[g], D, ld_cat, sx[g], D);
            d[g].add = sx[g];
            d[g].ld_add = D;
          }
          push_gemm(d);
        }
        block_marks.push_back(static_cast<int>(ops.size()));
      }
    }
    // ---- output projections, decoders, Euler updates ----
    {
      std::vector<LnSegment> v;
      v.push_back(LnSegment{xsa, oln_sa, ada_sc1p + static_cast<size_t>(s) * D, ada_shift + static_cast<size_t>(s) * D,
                            B * nsa, D, D, 0, D});
      if (!standard)
        v.push_back(LnSegment{xp, oln_p, pada_sc1p + static_cast<size_t>(s) * D,
                              pada_shift + static_cast<size_t>(s) * D, B * np, D, D, 0, D});
      push_ln(v);
    }
    {
      std::vector<rldx_gemm_desc> g1, g2, g3;
      g1.push_back(lin(oln_sa, D, po2_w, po2_b, B * nsa, c.out_dim, D, oproj_sa, c.out_dim));
      rldx_gemm_desc d1 = catlin(oproj_sa, c.out_dim, dl1_W, dl1_b, B * nsa, c.dec_hidden, c.out_dim, nsa, dec_h, c.dec_hidden);
      d1.act = RLDX_ACT_RELU;
      g2.push_back(d1);
      // Euler update of action tokens [prefix_len, h) of each observation: rows of the decoder
      // output before them (time, state, locked prefix) are dropped, so the prefix keeps the
      // frozen actions (the re-lock of graph_safe_action_model.py:296-300).
      const int pl = c.prefix_len;
      rldx_gemm_desc d2 = catlin(dec_h, c.dec_hidden, dl2_W, dl2_b, B * nsa, c.action_dim, c.dec_hidden, nsa,
                                 x + static_cast<size_t>(pl) * adp, adp);
      d2.epilogue = RLDX_EPI_EULER;
      d2.dt = dt;
      d2.rows_in = nsa;
      d2.rows_out = h;
      d2.row_skip = nsa - h + pl;
      g3.push_back(d2);
      if (!standard) {
        g1.push_back(lin(oln_p, D, pp2_w, pp2_b, B * np, c.out_dim, D, oproj_p, c.out_dim));
        rldx_gemm_desc p1 = lin(oproj_p, c.out_dim, phd1_w, phd1_b, B * np, D, c.out_dim, pdec_h, D);
        p1.act = RLDX_ACT_SILU;
        g2.push_back(p1);
        rldx_gemm_desc p2 = lin(pdec_h, D, phd2_w, phd2_b, B * np, c.physics_dim, D, phys_x, hc);
        p2.epilogue = RLDX_EPI_EULER;
        p2.dt = dt;
        p2.rows_in = np;
        p2.rows_out = fut;
        p2.row_skip = hist;
        g3.push_back(p2);
      }
      push_gemm(g1);
      push_gemm(g2);
      push_gemm(g3);
    }
  }
  push_status(1);  // a code raised during the step -> slot 1
}

namespace {
int guard(const std::function<void()>& f) {
  try {
    f();
    return RLDX_OK;
  } catch (const Fail& e) {
    return set_error(e.code, e.what());
  } catch (const std::exception& e) {
    return set_error(RLDX_ERR_CUDA, e.what());
  }
}

void free_all(rldx_msat* h) {
  if (h->exec) cudaGraphExecDestroy(h->exec);
  if (h->graph) cudaGraphDestroy(h->graph);
  if (h->exec_m) cudaGraphExecDestroy(h->exec_m);
  if (h->graph_m) cudaGraphDestroy(h->graph_m);
  for (void* p : h->allocs) cudaFree(p);
  if (h->stream) cudaStreamDestroy(h->stream);
  h->status.release();
  h->allocs.clear();
}

int device_status_error(unsigned int code, unsigned int during, const char* what) {
  return set_error(RLDX_ERR_DEVICE, std::string(what) + ": device error 0x" + [&] {
    char b[16];
    std::snprintf(b, sizeof(b), "%x", code);
    return std::string(b);
  }() + (during ? " raised during the step" : " left by earlier work (the step itself ran clean)"));
}
}  // namespace

extern "C" {

int rldx_msat_create(const rldx_msat_config* cfg, const rldx_msat_weights* w, rldx_msat** out) {
  if (!cfg || !w || !out) return set_error(RLDX_ERR_ARG, "msat_create: null argument");
  *out = nullptr;
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  rldx_msat* h = new rldx_msat();
  rc = guard([&] { h->create(*cfg, *w); });
  if (rc != RLDX_OK) {
    free_all(h);
    delete h;
    return rc;
  }
  *out = h;
  return RLDX_OK;
}

int rldx_msat_destroy(rldx_msat* h) {
  if (!h) return RLDX_OK;
  cudaStreamSynchronize(h->stream);
  free_all(h);
  delete h;
  return RLDX_OK;
}

static int msat_step_impl(rldx_msat* h, const rldx_msat_io* io, cudaStream_t st) {
  if (!h || !io) return set_error(RLDX_ERR_ARG, "msat_step: null argument");
  if (!io->vl || !io->state || !io->emb_id || !io->init_noise || !io->actions ||
      (!h->standard && (!io->physics_hist || !io->physics_noise)) || (h->c.prefix_len > 0 && !io->prefix_actions))
    return set_error(RLDX_ERR_ARG,
                     "msat_step: every io pointer is required (physics ones on the all-modality path, "
                     "prefix_actions with prefix_len > 0)");
  const bool masked = io->vl_mask != nullptr || io->physics_mask != nullptr;
  if (masked && !h->c.key_mask)
    return set_error(RLDX_ERR_STATE, "msat_step: key masks need a handle created with key_mask = 1");
  if (io->physics_mask && h->standard)
    return set_error(RLDX_ERR_ARG, "msat_step: physics_mask on a head without the physics stream");
  return guard([&] {
    h->copy_inputs(io, st);
    if (masked) {
      h->copy_masks(io, st);
      if (h->exec_m)
        ck(cudaGraphLaunch(h->exec_m, st), "graph launch");
      else
        h->run_ops(st, nullptr, -1, &h->ops_m);
    } else if (h->exec) {
      ck(cudaGraphLaunch(h->exec, st), "graph launch");
    } else {
      h->run_ops(st);
    }
    h->copy_outputs(io, st);
    ck(cudaEventRecord(h->status.done, st), "status event");
  });
}

int rldx_msat_step(rldx_msat* h, const rldx_msat_io* io, void* stream) {
  return msat_step_impl(h, io, static_cast<cudaStream_t>(stream));
}

int rldx_msat_step_host(rldx_msat* h, const rldx_msat_io* io, void* stream) {
  int rc = msat_step_impl(h, io, static_cast<cudaStream_t>(stream));
  if (rc != RLDX_OK) return rc;
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "msat_step_host sync");
  unsigned int code = 0, during = 0;
  rc = h->status.read(true, &code, &during);
  if (rc != RLDX_OK) return rc;
  if (code) return device_status_error(code, during, "msat_step_host");
  return RLDX_OK;
}

int rldx_msat_status(rldx_msat* h, int wait, unsigned int* code) {
  if (!h || !code) return set_error(RLDX_ERR_ARG, "msat_status: null argument");
  unsigned int during = 0;
  return h->status.read(wait != 0, code, &during);
}

int rldx_msat_block_end(const rldx_msat* h, int step, int block, int* n_ops) {
  if (!h || !n_ops) return set_error(RLDX_ERR_ARG, "msat_block_end: null argument");
  const int nblocks = h->c.depth + h->c.depth_single;
  if (step < 0 || step >= h->S || block < -1 || block >= nblocks)
    return set_error(RLDX_ERR_ARG, "msat_block_end: step / block out of range");
  *n_ops = block < 0 ? h->step_marks[step] : h->block_marks[static_cast<size_t>(step) * nblocks + block];
  return RLDX_OK;
}

int rldx_msat_run_partial(rldx_msat* h, const rldx_msat_io* io, int n_ops, void* stream) {
  if (!h || !io) return set_error(RLDX_ERR_ARG, "msat_run_partial: null argument");
  if (n_ops < 0 || n_ops > static_cast<int>(h->ops.size()))
    return set_error(RLDX_ERR_ARG, "msat_run_partial: n_ops outside [0, launch count]");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return guard([&] {
    h->copy_inputs(io, st);
    h->run_ops(st, nullptr, n_ops);
    ck(cudaEventRecord(h->status.done, st), "status event");
  });
}

int rldx_msat_profile(rldx_msat* h, const rldx_msat_io* io, rldx_op_profile* out, int max_ops,
                      int* n_ops, void* stream) {
  if (!h || !io || !n_ops || (max_ops > 0 && !out)) return set_error(RLDX_ERR_ARG, "profile: null argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<cudaEvent_t> ev(h->ops.size() + 1, nullptr);
  int rc = guard([&] {
    for (auto& e : ev) ck(cudaEventCreate(&e), "event create");
    h->copy_inputs(io, st);
    h->run_ops(st, ev.data());
    h->copy_outputs(io, st);
    ck(cudaStreamSynchronize(st), "profile sync");
    const int n = static_cast<int>(h->ops.size());
    *n_ops = n;
    for (int i = 0; i < n && i < max_ops; ++i) {
      float ms = 0.0f;
      ck(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]), "elapsed");
      const Op& o = h->ops[i];
      out[i].kind = static_cast<int>(o.kind);
      out[i].grid = o.grid;
      out[i].ms = ms;
      out[i].bytes = o.bytes;
      out[i].flops = o.flops;
    }
  });
  for (auto& e : ev)
    if (e) cudaEventDestroy(e);
  return rc;
}

int rldx_msat_launch_count(const rldx_msat* h) { return h ? static_cast<int>(h->ops.size()) : 0; }

int rldx_msat_read_buffer(const rldx_msat* h, int which, void* dst, int64_t dst_bytes,
                          int64_t* rows, int64_t* cols, void* stream) {
  if (!h || !rows || !cols) return set_error(RLDX_ERR_ARG, "read_buffer: null argument");
  const void* src = nullptr;
  switch (which) {
    case 0:
      src = h->xvl;
      *rows = static_cast<int64_t>(h->B) * h->nvl;
      *cols = h->Dv;
      break;
    case 1:
      src = h->xsa;
      *rows = static_cast<int64_t>(h->B) * h->nsa;
      *cols = h->D;
      break;
    case 2:
      src = h->xp;
      *rows = static_cast<int64_t>(h->B) * h->np;
      *cols = h->D;
      break;
    case 3:
      src = h->x;
      *rows = static_cast<int64_t>(h->B) * h->c.horizon;
      *cols = h->c.action_dim;
      break;
    case 4:  // LayerNorm outputs of the streams (the last LN of a double block)
    case 5:
    case 6: {
      const bf16* b[3] = {h->lnvl, h->lnsa, h->lnp};
      const int n[3] = {h->nvl, h->nsa, h->np};
      src = b[which - 4];
      *rows = static_cast<int64_t>(h->B) * n[which - 4];
      *cols = which == 4 ? h->Dv : h->D;
      break;
    }
    case 7:  // q, k [B*H*L, 64]
    case 8:
      src = which == 7 ? h->q : h->k;
      *rows = static_cast<int64_t>(h->B) * h->H * h->L;
      *cols = 64;
      break;
    case 9:  // v^T [B*H*64, Lp]
      src = h->vt;
      *rows = static_cast<int64_t>(h->B) * h->H * 64;
      *cols = h->Lp;
      break;
    case 10:  // attention outputs of the streams [B*n, H*64]
    case 11:
    case 12: {
      const bf16* b[3] = {h->ovl, h->osa, h->op};
      const int n[3] = {h->nvl, h->nsa, h->np};
      src = b[which - 10];
      *rows = static_cast<int64_t>(h->B) * n[which - 10];
      *cols = h->H * 64;
      break;
    }
    case 13:  // SwiGLU hidden of the streams [B*n, hidden padded to 32]
    case 14:
    case 15: {
      const bf16* b[3] = {h->hvl, h->hsa, h->hp};
      const int n[3] = {h->nvl, h->nsa, h->np};
      const int hid[3] = {rldx_msat::pad32(h->c.vl_mlp_hidden), rldx_msat::pad32(h->c.mlp_hidden),
                          rldx_msat::pad32(h->c.mlp_hidden)};
      src = b[which - 13];
      *rows = static_cast<int64_t>(h->B) * n[which - 13];
      *cols = hid[which - 13];
      break;
    }
    default:
      return set_error(RLDX_ERR_ARG, "read_buffer: unknown buffer");
  }
  if (!src || *rows == 0) return set_error(RLDX_ERR_ARG, "read_buffer: the handle has no such buffer");
  if (!dst) return RLDX_OK;
  const int64_t bytes = *rows * *cols * 2;
  if (dst_bytes < bytes) return set_error(RLDX_ERR_ARG, "read_buffer: destination too small");
  cudaError_t e = cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDefault,
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "read_buffer copy");
  return RLDX_OK;
}

}  // extern "C"
