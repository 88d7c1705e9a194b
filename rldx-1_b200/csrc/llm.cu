// VLM backbone prefill: a stack of Qwen3 decoder layers over B sequences of T tokens, planned
// once and replayed as one CUDA graph (the counterpart of CustomLLMChain,
// rldx/inference/backbone/llm/engine/custom_llm_chain.py:63-170).  The same runtime runs the
// memory module's TransformerMemory (rldx/model/modules/memory.py:150-370; CustomMemoryChain,
// rldx/inference/memory/engine/custom_memory_chain.py:43-174): no q / k norm, weight-then-cast
// RMSNorm, 96-dim heads (1536 / 16, run zero-padded to 128), block-wise positions.
//
// Per layer (Qwen3VLTextDecoderLayer, rldx/model/modules/backbone/modeling_qwen3_vl.py:509-560):
//   n   = RMSNorm_in(h)                               res_ln_kernel (rms)
//   qkv = n @ [Wq; Wk; Wv]^T                          gemm_bf16_kernel (store)
//   q, k = RoPE(RMSNorm_head(q | k)), V^T            qk_rmsnorm_rope_kernel (attention layout),
//                                                    v_transpose_kernel
//   a   = causal GQA attention                        joint_attention_kernel<128> (causal, kv heads)
//   h   = h + a @ Wo^T                                gemm_bf16_kernel (residual epilogue)
//   n   = RMSNorm_post(h)                             res_ln_kernel (rms)
//   g   = silu(n @ Wg^T) * (n @ Wu^T)                 gemm_bf16_kernel (SwiGLU epilogue on
//                                                    [32 gate | 32 up] interleaved rows)
//   h   = h + g @ Wd^T                                gemm_bf16_kernel (residual epilogue)
// and an optional final RMSNorm.  With video-token compression (the VTC backbone's LayerWrapper,
// rldx/model/modules/backbone/layer_wrapper.py:73-113, run with static rows as the reference
// inference engine does, graph_safe_qwen3vl_text_model.py:142-175) one compress_rows_kernel
// before layer compress_layer replaces the rows [begin, end) of every sequence with their mean,
// and the layers from there on run on the shorter sequence with the matching RoPE rows (front,
// row begin, back).  Every bf16 rounding follows the eager module: each linear
// rounds once, the residual adds round, RMSNorm casts before its weight, RoPE rounds each
// product and the sum, silu rounds before the product.
//
// Layout: token-major activations [B*T, width]; q [B, Hq, T, 128], k [B, Hkv, T, 128] and
// V^T [B, Hkv, 128, Tp] (Tp = T rounded up to 8) for the attention kernel.  A compressed stack
// has a second set of hidden / q / k / V^T buffers and RoPE tables for its T2 tokens; the
// token-major scratch (norm output, qkv, attention output, SwiGLU hidden) is shared.
#include "host_util.h"

using namespace rldx;

struct rldx_llm {
  rldx_llm_config c{};
  int B = 0, T = 0, Tp = 0, D = 0, Hq = 0, Hkv = 0, F = 0, Fp = 0, NQKV = 0, M = 0;
  int hd = 128, phd = 128;  // head dims, and the padded head dims of the attention layout
  std::vector<void*> allocs;
  struct LayerW {
    bf16 *in_norm, *qkv, *qn, *kn, *o, *post_norm, *w12, *down;
  };
  std::vector<LayerW> lw;
  bf16* final_norm = nullptr;
  // one sequence length of the stack: all layers, or the layers before / after compression
  struct Seq {
    int T = 0, Tp = 0, M = 0;
    bf16 *h = nullptr, *q = nullptr, *k = nullptr, *vt = nullptr, *cos = nullptr, *sin = nullptr;
  };
  Seq pre, post;  // post == pre without compression
  bool compress = false;
  bf16 *h = nullptr, *n = nullptr, *qkv = nullptr, *a = nullptr, *g = nullptr;
  bf16* out = nullptr;  // result of the last op (n after the final norm, else the last hidden)
  int out_rows = 0;     // B * tokens of the output
  int ds_layers = 0, ds_rows = 0;
  int* ds_index = nullptr;  // [ds_rows] token rows
  bf16* ds_feat = nullptr;  // [ds_layers][B][ds_rows][D]
  std::vector<std::function<cudaError_t(cudaStream_t, bool)>> ops;
  StepStatus status;  // device error codes of the last call (status.cu)
  void* ws = nullptr;
  size_t ws_bytes = 0, ws_need = 0;
  bool sizing = false;
  cudaStream_t stream = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  bool pdl = true;

  // Bind-time copies, fills and re-layout kernels all run in order on the handle's stream (a
  // legacy-stream cudaMemcpy between device buffers is asynchronous and unordered with it).
  template <class T_>
  T_* alloc(size_t count) {
    void* p = nullptr;
    ck(cudaMalloc(&p, count * sizeof(T_) + 256), "cudaMalloc");
    allocs.push_back(p);
    ck(cudaMemsetAsync(p, 0, count * sizeof(T_) + 256, stream), "cudaMemset");
    return static_cast<T_*>(p);
  }
  bf16* copy_rows(bf16* dst, const void* src, size_t count, const char* what) {
    if (!src) throw Fail(RLDX_ERR_ARG, std::string("missing weight: ") + what);
    ck(cudaMemcpyAsync(dst, src, count * 2, cudaMemcpyDefault, stream), what);
    return dst;
  }
  bf16* copy_in(const void* src, size_t count, const char* what) { return copy_rows(alloc<bf16>(count), src, count, what); }

  // gate [F, D] and up [F, D] -> [32 gate | 32 up] row groups over Fp = F rounded up to 32;
  // padded rows are zero (silu(0) * 0 = 0) and so are the matching columns of down_proj.
  bf16* interleave_w12(const void* gate, const void* up) {
    bf16* src = alloc<bf16>(static_cast<size_t>(2 * F + 1) * D);  // gate rows, up rows, one zero row
    copy_rows(src, gate, static_cast<size_t>(F) * D, "gate_proj");
    copy_rows(src + static_cast<size_t>(F) * D, up, static_cast<size_t>(F) * D, "up_proj");
    std::vector<int> idx(2 * Fp);
    for (int grp = 0; grp < Fp / 32; ++grp)
      for (int i = 0; i < 32; ++i) {
        const int r = grp * 32 + i;
        idx[grp * 64 + i] = r < F ? r : 2 * F;
        idx[grp * 64 + 32 + i] = r < F ? F + r : 2 * F;
      }
    int* didx = alloc<int>(idx.size());
    ck(cudaMemcpyAsync(didx, idx.data(), idx.size() * 4, cudaMemcpyHostToDevice, stream), "idx");
    bf16* dst = alloc<bf16>(static_cast<size_t>(2) * Fp * D);
    ck(launch_gather_rows(src, D, dst, D, didx, 2 * Fp, D, stream), "gather w12");
    ck(cudaStreamSynchronize(stream), "gather sync");
    return dst;
  }

  void push_gemm(const rldx_gemm_desc& d) {
    GemmParams gp;
    std::string err;
    size_t need = 0;
    if (!build_gemm_params(&d, 1, sizing ? nullptr : ws, sizing ? 0 : ws_bytes, &gp, sizing ? &need : nullptr, &err))
      throw Fail(RLDX_ERR_ARG, err);
    ws_need = std::max(ws_need, need);
    ops.push_back([gp](cudaStream_t st, bool p) { return launch_gemm(gp, st, p); });
  }
  void push_rmsnorm(const bf16* x, const bf16* w, bf16* outp, int M) {
    ResLnParams p;
    std::memset(&p, 0, sizeof(p));
    p.seg[0].x = x;
    p.seg[0].w = w;
    p.seg[0].ln_out = outp;
    p.seg[0].rows = M;
    p.seg[0].D = D;
    p.seg[0].ld = D;
    p.nseg = 1;
    p.total_rows = M;
    p.dmax = D;
    p.rms = 1;
    p.rms_weight_first = c.norm_weight_first ? 1 : 0;
    p.eps = c.rms_eps;
    ops.push_back([p](cudaStream_t st, bool) { return launch_res_ln(p, st); });
  }

  void create(const rldx_llm_config& cfg, const rldx_llm_weights& w) {
    c = cfg;
    B = c.batch;
    T = c.tokens;
    D = c.hidden;
    Hq = c.q_heads;
    Hkv = c.kv_heads;
    F = c.ffn;
    if (B <= 0 || T <= 0 || D <= 0 || Hq <= 0 || Hkv <= 0 || F <= 0 || c.layers <= 0)
      throw Fail(RLDX_ERR_ARG, "llm_create: batch, tokens, hidden, heads, ffn, layers must be positive");
    if (c.head_dim != 128 && c.head_dim != 96) throw Fail(RLDX_ERR_UNSUPPORTED, "llm_create: head_dim must be 96 or 128");
    hd = c.head_dim;  // 96-dim heads run zero-padded to 128 in q, k, V^T
    if (c.causal_block < 0) throw Fail(RLDX_ERR_ARG, "llm_create: causal_block must be >= 0");
    if (Hq % Hkv) throw Fail(RLDX_ERR_ARG, "llm_create: kv_heads must divide q_heads");
    if (D % 64 || D > 4096) throw Fail(RLDX_ERR_UNSUPPORTED, "llm_create: hidden must be a multiple of 64, <= 4096");
    if (static_cast<long long>(B) * T * (Hq + Hkv) >= (1LL << 31)) throw Fail(RLDX_ERR_UNSUPPORTED, "llm_create: too many rows");
    if (!w.layers || !w.rope_cos || !w.rope_sin) throw Fail(RLDX_ERR_ARG, "llm_create: missing layers or RoPE tables");
    if (c.final_norm && !w.final_norm) throw Fail(RLDX_ERR_ARG, "llm_create: missing final_norm");
    if (c.deepstack_layers < 0 || c.deepstack_layers > c.layers || c.deepstack_rows < 0 ||
        (c.deepstack_layers > 0) != (c.deepstack_rows > 0))
      throw Fail(RLDX_ERR_ARG, "llm_create: deepstack_layers in [0, layers] and deepstack_rows > 0 together");
    compress = c.compress_end > c.compress_begin;
    if (compress) {
      if (c.compress_begin < 0 || c.compress_end > c.tokens || c.compress_layer < 0 || c.compress_layer >= c.layers)
        throw Fail(RLDX_ERR_ARG, "llm_create: compression needs 0 <= compress_begin < compress_end <= tokens and "
                                 "0 <= compress_layer < layers");
      if (c.deepstack_layers > c.compress_layer)
        throw Fail(RLDX_ERR_UNSUPPORTED, "llm_create: deepstack layers must come before the compression layer");
    }
    if (c.deepstack_layers > 0) {
      if (!w.deepstack_row_index) throw Fail(RLDX_ERR_ARG, "llm_create: missing deepstack_row_index");
      for (int j = 0; j < c.deepstack_rows; ++j)
        if (w.deepstack_row_index[j] < 0 || w.deepstack_row_index[j] >= c.tokens)
          throw Fail(RLDX_ERR_ARG, "llm_create: deepstack row outside the sequence");
    }
    Tp = (T + 7) / 8 * 8;
    Fp = (F + 31) / 32 * 32;
    NQKV = (Hq + 2 * Hkv) * hd;
    M = B * T;
    const char* env = getenv("RLDX_PDL");
    pdl = !(env && env[0] == '0');
    ck(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
    ck(cudaDeviceSynchronize(), "weights ready");  // the caller's weights may come from any stream

    const size_t qd = static_cast<size_t>(Hq) * hd, kd = static_cast<size_t>(Hkv) * hd;
    for (int i = 0; i < c.layers; ++i) {
      const rldx_llm_layer_weights& s = w.layers[i];
      LayerW l{};
      l.in_norm = copy_in(s.input_norm, D, "input_layernorm");
      l.qkv = alloc<bf16>(static_cast<size_t>(NQKV) * D);
      copy_rows(l.qkv, s.q_proj, qd * D, "q_proj");
      copy_rows(l.qkv + qd * D, s.k_proj, kd * D, "k_proj");
      copy_rows(l.qkv + (qd + kd) * D, s.v_proj, kd * D, "v_proj");
      if (!c.no_qk_norm) {
        l.qn = copy_in(s.q_norm, hd, "q_norm");
        l.kn = copy_in(s.k_norm, hd, "k_norm");
      }
      l.o = copy_in(s.o_proj, static_cast<size_t>(D) * qd, "o_proj");
      l.post_norm = copy_in(s.post_norm, D, "post_attention_layernorm");
      l.w12 = interleave_w12(s.gate_proj, s.up_proj);
      if (!s.down_proj) throw Fail(RLDX_ERR_ARG, "missing weight: down_proj");
      l.down = alloc<bf16>(static_cast<size_t>(D) * Fp);  // [D, F] -> [D, Fp], zero columns
      ck(cudaMemcpy2DAsync(l.down, static_cast<size_t>(Fp) * 2, s.down_proj, static_cast<size_t>(F) * 2,
                           static_cast<size_t>(F) * 2, D, cudaMemcpyDefault, stream),
         "down_proj");
      lw.push_back(l);
    }
    if (c.final_norm) final_norm = copy_in(w.final_norm, D, "final norm");
    ds_layers = c.deepstack_layers;
    ds_rows = c.deepstack_rows;
    if (ds_layers > 0) {
      ds_index = alloc<int>(ds_rows);
      ck(cudaMemcpyAsync(ds_index, w.deepstack_row_index, static_cast<size_t>(ds_rows) * 4, cudaMemcpyHostToDevice,
                         stream),
         "deepstack rows");
      ds_feat = alloc<bf16>(static_cast<size_t>(ds_layers) * B * ds_rows * D);  // zero until set
    }
    pre = make_seq(T);
    pre.cos = copy_in(w.rope_cos, static_cast<size_t>(T) * hd, "rope cos");
    pre.sin = copy_in(w.rope_sin, static_cast<size_t>(T) * hd, "rope sin");
    post = pre;
    if (compress) {  // RoPE rows of the compressed sequence: [0, begin), begin, [end, T)
      const int b0 = c.compress_begin, e0 = c.compress_end;
      post = make_seq(T - (e0 - b0) + 1);
      post.cos = alloc<bf16>(static_cast<size_t>(post.T) * hd);
      post.sin = alloc<bf16>(static_cast<size_t>(post.T) * hd);
      const size_t row = static_cast<size_t>(hd) * 2;
      for (int t = 0; t < 2; ++t) {
        bf16* dst = t ? post.sin : post.cos;
        const bf16* src = t ? pre.sin : pre.cos;
        ck(cudaMemcpyAsync(dst, src, (b0 + 1) * row, cudaMemcpyDeviceToDevice, stream), "rope rows");
        if (e0 < T)
          ck(cudaMemcpyAsync(reinterpret_cast<char*>(dst) + (b0 + 1) * row, reinterpret_cast<const char*>(src) + e0 * row,
                             static_cast<size_t>(T - e0) * row, cudaMemcpyDeviceToDevice, stream),
             "rope rows");
      }
    }
    h = pre.h;
    n = alloc<bf16>(static_cast<size_t>(M) * D);
    qkv = alloc<bf16>(static_cast<size_t>(M) * NQKV);
    a = alloc<bf16>(static_cast<size_t>(M) * qd);
    g = alloc<bf16>(static_cast<size_t>(M) * Fp);

    if (!status.init()) throw Fail(RLDX_ERR_CUDA, "step status: mapped host memory");
    if (split_k_enabled()) {  // first pass: the workspace the K-split plans want
      sizing = true;
      plan();
      sizing = false;
      ops.clear();
      if (ws_need > 0) {
        ws = alloc<uint8_t>(ws_need);  // zero-filled: the tile counters start at zero
        ws_bytes = ws_need;
      }
    }
    plan();
    run_ops(stream);  // warm-up (loads every kernel)
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
        cudaGraph_t gr = nullptr;
        cudaStreamEndCapture(stream, &gr);
        if (gr) cudaGraphDestroy(gr);
        throw;
      }
      ck(cudaStreamEndCapture(stream, &graph), "end capture");
      ck(cudaGraphInstantiate(&exec, graph, 0), "instantiate");
      ck(cudaGraphUpload(exec, stream), "upload");
      ck(cudaStreamSynchronize(stream), "upload sync");
    }
  }

  // hidden / q / k / V^T buffers of a sequence of T_ tokens (zero-filled: padded head dims stay zero)
  Seq make_seq(int T_) {
    Seq s_;
    s_.T = T_;
    s_.Tp = (T_ + 7) / 8 * 8;
    s_.M = B * T_;
    s_.h = alloc<bf16>(static_cast<size_t>(s_.M) * D);
    s_.q = alloc<bf16>(static_cast<size_t>(B) * Hq * T_ * phd);
    s_.k = alloc<bf16>(static_cast<size_t>(B) * Hkv * T_ * phd);
    s_.vt = alloc<bf16>(static_cast<size_t>(B) * Hkv * phd * s_.Tp);
    return s_;
  }

  void push_status(int which) {
    unsigned int* slot = status.dev + which;
    ops.push_back([slot](cudaStream_t st, bool) { return launch_status_take(slot, st); });
  }

  void plan() {
    const int qd = Hq * hd;
    push_status(0);  // a code left by earlier work -> slot 0; the call starts from a clean word
    const Seq* last = &pre;
    for (int li = 0; li < c.layers; ++li) {
      const LayerW& l = lw[li];
      if (compress && li == c.compress_layer) {
        const bf16* x = pre.h;
        bf16* y = post.h;
        const int b_ = B, t_ = T, d_ = D, b0 = c.compress_begin, e0 = c.compress_end;
        ops.push_back([=](cudaStream_t st, bool) { return launch_compress_rows(x, y, b_, t_, d_, b0, e0, st); });
      }
      const Seq& sq = (compress && li >= c.compress_layer) ? post : pre;
      last = &sq;
      const int M = sq.M, T = sq.T, Tp = sq.Tp;
      bf16 *h = sq.h, *q = sq.q, *k = sq.k, *vt = sq.vt;
      push_rmsnorm(h, l.in_norm, n, M);
      push_gemm(rldx_msat::lin(n, D, l.qkv, nullptr, M, NQKV, D, qkv, NQKV));
      {
        QkNormRopeParams p;
        std::memset(&p, 0, sizeof(p));
        p.x = qkv;
        p.x_tok_stride = NQKV;
        p.q = q;
        p.k = k;
        p.wq = l.qn;
        p.wk = l.kn;
        p.cos = sq.cos;
        p.sin = sq.sin;
        p.nrows = static_cast<unsigned>(M * (Hq + Hkv));
        p.heads = static_cast<unsigned>(Hq + Hkv);
        p.Hq = static_cast<unsigned>(Hq);
        p.T = static_cast<unsigned>(T);
        p.layout = 1;
        p.hd = hd;
        p.out_hd = phd;
        p.norm = c.no_qk_norm ? 0 : 1;
        p.eps = c.rms_eps;
        ops.push_back([p](cudaStream_t st, bool) { return launch_qk_rmsnorm_rope(p, st); });
        const bf16* v = qkv + static_cast<size_t>(Hq + Hkv) * hd;
        bf16* vtp = vt;
        const int b_ = B, t_ = T, tp_ = Tp, hkv_ = Hkv, ld_ = NQKV, hd_ = hd, phd_ = phd;
        ops.push_back(
            [=](cudaStream_t st, bool) { return launch_v_transpose(v, ld_, vtp, b_, t_, tp_, hkv_, hd_, phd_, st); });
      }
      {
        AttnParams ap;
        std::memset(&ap, 0, sizeof(ap));
        ap.L = T;
        ap.H = Hq;
        ap.B = B;
        ap.kv_heads = Hkv;
        ap.causal = 1;
        ap.causal_block = c.causal_block > 1 ? c.causal_block : 1;
        ap.head_dim = phd;
        ap.out_dim = hd;
        ap.seg_out[0] = a;
        ap.seg_len[0] = T;
        ap.seg_ld[0] = qd;
        ap.nseg = 1;
        ap.scale_log2 = 1.4426950408889634f / std::sqrt(static_cast<float>(hd));
        std::string err;
        const uint64_t bq = static_cast<uint64_t>(B) * Hq, bkv = static_cast<uint64_t>(B) * Hkv;
        if (!make_tmap_3d(&ap.tq, q, 128, T, bq, 256, static_cast<uint64_t>(T) * 256, 64, 128, 1, &err) ||
            !make_tmap_3d(&ap.tk, k, 128, T, bkv, 256, static_cast<uint64_t>(T) * 256, 64, 64, 1, &err) ||
            !make_tmap_3d(&ap.tv, vt, T, 128, bkv, static_cast<uint64_t>(Tp) * 2, static_cast<uint64_t>(Tp) * 256, 64,
                          128, 1, &err))
          throw Fail(RLDX_ERR_ARG, err);
        ops.push_back([ap](cudaStream_t st, bool p) { return launch_attention(ap, st, p); });
      }
      {
        rldx_gemm_desc d = rldx_msat::lin(a, qd, l.o, nullptr, M, D, qd, h, D);
        d.add = h;
        d.ld_add = D;
        push_gemm(d);
      }
      push_rmsnorm(h, l.post_norm, n, M);
      {
        rldx_gemm_desc d = rldx_msat::lin(n, D, l.w12, nullptr, M, 2 * Fp, D, g, Fp);
        d.epilogue = RLDX_EPI_SWIGLU;
        push_gemm(d);
      }
      {
        rldx_gemm_desc d = rldx_msat::lin(g, Fp, l.down, nullptr, M, D, Fp, h, D);
        d.add = h;
        d.ld_add = D;
        push_gemm(d);
      }
      if (li < ds_layers) {  // deepstack: after the layer's output, before the next layer
        bf16* hp = h;
        const int* idx = ds_index;
        const bf16* f = ds_feat + static_cast<size_t>(li) * B * ds_rows * D;
        const int r_ = ds_rows, b_ = B, t_ = T, d_ = D;
        ops.push_back([=](cudaStream_t st, bool) { return launch_rows_add(hp, idx, r_, f, b_, t_, d_, st); });
      }
    }
    out = last->h;
    out_rows = last->M;
    if (c.final_norm) {
      push_rmsnorm(last->h, final_norm, n, last->M);
      out = n;
    }
    push_status(1);  // a code raised during the call -> slot 1
  }

  void run_ops(cudaStream_t st) {
    for (size_t i = 0; i < ops.size(); ++i) ck(ops[i](st, pdl && i > 0), "launch");
  }
};

namespace {
void free_llm(rldx_llm* h) {
  if (h->exec) cudaGraphExecDestroy(h->exec);
  if (h->graph) cudaGraphDestroy(h->graph);
  for (void* p : h->allocs) cudaFree(p);
  if (h->stream) cudaStreamDestroy(h->stream);
  h->status.release();
  h->allocs.clear();
}
}  // namespace

extern "C" {

int rldx_llm_create(const rldx_llm_config* cfg, const rldx_llm_weights* w, rldx_llm** out) {
  if (!cfg || !w || !out) return set_error(RLDX_ERR_ARG, "llm_create: null argument");
  *out = nullptr;
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  rldx_llm* h = new rldx_llm();
  rc = guard([&] { h->create(*cfg, *w); });
  if (rc != RLDX_OK) {
    free_llm(h);
    delete h;
    return rc;
  }
  *out = h;
  return RLDX_OK;
}

int rldx_llm_destroy(rldx_llm* h) {
  if (!h) return RLDX_OK;
  cudaStreamSynchronize(h->stream);
  free_llm(h);
  delete h;
  return RLDX_OK;
}

int rldx_llm_prefill(rldx_llm* h, const void* hidden_in, void* hidden_out, void* stream) {
  if (!h || !hidden_in || !hidden_out) return set_error(RLDX_ERR_ARG, "llm_prefill: null argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return guard([&] {
    const size_t bytes = static_cast<size_t>(h->M) * h->D * 2;
    ck(cudaMemcpyAsync(h->h, hidden_in, bytes, cudaMemcpyDefault, st), "hidden in");
    if (h->exec)
      ck(cudaGraphLaunch(h->exec, st), "graph launch");
    else
      h->run_ops(st);
    ck(cudaMemcpyAsync(hidden_out, h->out, static_cast<size_t>(h->out_rows) * h->D * 2, cudaMemcpyDefault, st),
       "hidden out");
    ck(cudaEventRecord(h->status.done, st), "status event");
  });
}

int rldx_llm_status(rldx_llm* h, int wait, unsigned int* code) {
  if (!h || !code) return set_error(RLDX_ERR_ARG, "llm_status: null argument");
  unsigned int during = 0;
  return h->status.read(wait != 0, code, &during);
}

int rldx_llm_launch_count(const rldx_llm* h) { return h ? static_cast<int>(h->ops.size()) : 0; }

int rldx_llm_out_tokens(const rldx_llm* h) { return h ? h->post.T : 0; }

int rldx_llm_set_deepstack(rldx_llm* h, const void* features, void* stream) {
  if (!h || !features) return set_error(RLDX_ERR_ARG, "llm_set_deepstack: null argument");
  if (h->ds_layers == 0) return set_error(RLDX_ERR_ARG, "llm_set_deepstack: the handle was created without deepstack");
  return guard([&] {
    const size_t bytes = static_cast<size_t>(h->ds_layers) * h->B * h->ds_rows * h->D * 2;
    ck(cudaMemcpyAsync(h->ds_feat, features, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)),
       "deepstack features");
  });
}

}  // extern "C"
