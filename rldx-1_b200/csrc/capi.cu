// C-ABI entry points of the per-op kernels, error reporting and the host helpers that turn
// plain pointers and sizes into TMA descriptors and launch parameters.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "host_util.h"

namespace rldx {

namespace {
thread_local std::string t_last_error;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

constexpr int kMaxDevices = 64;
std::once_flag g_dev_once[kMaxDevices];
int g_dev_status[kMaxDevices];
int g_dev_sms[kMaxDevices];

int round_up(int x, int m) { return (x + m - 1) / m * m; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

int set_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return set_error(RLDX_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int ensure_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return set_error(RLDX_ERR_UNSUPPORTED, "device index");
  std::call_once(g_dev_once[dev], [dev] {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
      g_dev_status[dev] = -1;
      return;
    }
    if (prop.major != 10 || prop.minor != 0) {
      g_dev_status[dev] = -2;
      return;
    }
    g_dev_sms[dev] = prop.multiProcessorCount;
    if (gemm_prepare_device() != cudaSuccess || attention_prepare_device() != cudaSuccess) {
      g_dev_status[dev] = -3;
      return;
    }
    g_dev_status[dev] = 1;
  });
  switch (g_dev_status[dev]) {
    case 1:
      return RLDX_OK;
    case -2:
      return set_error(RLDX_ERR_UNSUPPORTED, "device is not sm_100 (B200/GB200)");
    case -3:
      return set_error(RLDX_ERR_CUDA, "setting kernel attributes failed");
    default:
      return set_error(RLDX_ERR_CUDA, "cudaGetDeviceProperties failed");
  }
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  return (dev >= 0 && dev < kMaxDevices && g_dev_sms[dev] > 0) ? g_dev_sms[dev] : 148;
}

bool make_tmap_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                  std::string* err) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled(2d) failed with code " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

bool make_tmap_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                  uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                  uint32_t b2, std::string* err) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled(3d) failed with code " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

bool build_gemm_problem(const rldx_gemm_desc& d, GemmProblem* p, std::string* err) {
  std::memset(p, 0, sizeof(*p));
  if (!d.a || !d.b || !d.out) return (*err = "gemm: null a/b/out"), false;
  if (d.M <= 0 || d.N <= 0 || d.K <= 0) return (*err = "gemm: M, N, K must be positive"), false;
  if (d.K % 8 != 0) return (*err = "gemm: K must be a multiple of 8"), false;
  if (d.lda < d.K || d.ldb < d.K || (d.lda % 8) || (d.ldb % 8))
    return (*err = "gemm: lda/ldb must be >= K and multiples of 8"), false;
  if (!aligned16(d.a) || !aligned16(d.b)) return (*err = "gemm: a/b must be 16-byte aligned"), false;
  if (d.epilogue < RLDX_EPI_STORE || d.epilogue > RLDX_EPI_EULER)
    return (*err = "gemm: bad epilogue"), false;
  if (d.bias_mode < 0 || d.bias_mode > 2 || d.act < 0 || d.act > 3)
    return (*err = "gemm: bad bias_mode / act"), false;
  if (d.bias_mode != RLDX_BIAS_NONE && !d.bias) return (*err = "gemm: bias_mode needs bias"), false;
  if (d.ldo <= 0) return (*err = "gemm: ldo must be positive"), false;

  int m_step, tiles_m;
  if (d.cat_ids) {
    if (d.rows_per_cat <= 0 || d.rows_per_cat > 128 || d.M % d.rows_per_cat != 0)
      return (*err = "gemm: rows_per_cat must divide M and be <= 128"), false;
    if (d.num_cats <= 0 || d.b_cat_stride < static_cast<int64_t>(d.N) * d.ldb ||
        d.b_cat_stride % 8 != 0)
      return (*err = "gemm: bad num_cats / b_cat_stride"), false;
    m_step = d.rows_per_cat;
    tiles_m = d.M / d.rows_per_cat;
  } else {
    m_step = 128;
    tiles_m = (d.M + 127) / 128;
  }
  const int a_rows = std::min(128, round_up(std::min(m_step, d.M), 8));

  int bn = d.tile_n;
  if (bn == 0) {
    const int t256 = tiles_m * ((d.N + 255) / 256);
    const int t128 = tiles_m * ((d.N + 127) / 128);
    if (d.N >= 256 && t256 >= 96)
      bn = 256;
    else if (d.N >= 128 && t128 >= 96)
      bn = 128;
    else
      bn = 64;
  }
  if (bn < 64 || bn > 256 || bn % 64 != 0) return (*err = "gemm: tile_n must be 64..256, x64"), false;

  if (d.epilogue == RLDX_EPI_SWIGLU && d.N % 64 != 0)
    return (*err = "gemm: SwiGLU needs N % 64 == 0 (interleaved 32 gate + 32 up)"), false;
  if (d.epilogue == RLDX_EPI_QKV) {
    if (!d.q || !d.k || !d.vt || !d.q_norm_w || !d.k_norm_w || !d.rope_cos || !d.rope_sin)
      return (*err = "gemm: QKV epilogue needs q, k, vt, norms and rope tables"), false;
    if (d.H <= 0 || d.N != 3 * 64 * d.H) return (*err = "gemm: QKV needs N == 3 * H * 64"), false;
    if (d.L <= 0 || d.Lp < d.L || d.Lp % 8 != 0) return (*err = "gemm: QKV needs Lp >= L, Lp % 8 == 0"), false;
    if (d.rows_in <= 0 || d.tok_off < 0 || d.tok_off + d.rows_in > d.L)
      return (*err = "gemm: QKV rows_in/tok_off outside L"), false;
  }
  if (d.rows_in < 0 || (d.rows_in > 0 && d.rows_out <= 0))
    return (*err = "gemm: bad rows_in / rows_out"), false;

  p->M = d.M;
  p->N = d.N;
  p->K = d.K;
  p->bn = bn;
  p->a_rows = a_rows;
  p->m_step = m_step;
  p->tiles_m = tiles_m;
  p->tiles_n = (d.N + bn - 1) / bn;
  p->cat_ids = reinterpret_cast<const long long*>(d.cat_ids);

  if (!make_tmap_2d(&p->ta, d.a, d.K, d.M, static_cast<uint64_t>(d.lda) * 2, 64, a_rows, err))
    return false;
  if (d.cat_ids) {
    if (!make_tmap_3d(&p->tb, d.b, d.K, d.N, d.num_cats, static_cast<uint64_t>(d.ldb) * 2,
                      static_cast<uint64_t>(d.b_cat_stride) * 2, 64, bn, 1, err))
      return false;
  } else {
    if (!make_tmap_2d(&p->tb, d.b, d.K, d.N, static_cast<uint64_t>(d.ldb) * 2, 64, bn, err))
      return false;
  }

  GemmEpilogue& e = p->ep;
  e.mode = d.epilogue;
  e.bias_mode = d.bias_mode;
  e.act = d.act;
  e.bias = static_cast<const __nv_bfloat16*>(d.bias);
  e.bias_cat_stride = static_cast<int>(d.bias_cat_stride);
  e.add = static_cast<const __nv_bfloat16*>(d.add);
  e.ld_add = static_cast<int>(d.ld_add);
  e.add_row_mod = d.add_row_mod;
  e.out = static_cast<__nv_bfloat16*>(d.out);
  e.ldo = static_cast<int>(d.ldo);
  e.col_off = d.col_off;
  e.rows_in = d.rows_in;
  e.rows_out = d.rows_out;
  e.row_skip = d.row_skip;
  e.dt = d.dt;
  e.qn_w = static_cast<const __nv_bfloat16*>(d.q_norm_w);
  e.kn_w = static_cast<const __nv_bfloat16*>(d.k_norm_w);
  e.rope_cos = d.rope_cos;
  e.rope_sin = d.rope_sin;
  e.q = static_cast<__nv_bfloat16*>(d.q);
  e.k = static_cast<__nv_bfloat16*>(d.k);
  e.vt = static_cast<__nv_bfloat16*>(d.vt);
  e.L = d.L;
  e.Lp = d.Lp;
  e.H = d.H;
  e.tok_off = d.tok_off;
  e.eps = d.eps > 0.0f ? d.eps : 1e-6f;
  return true;
}

bool build_gemm_params(const rldx_gemm_desc* d, int n, GemmParams* params, int* tiles,
                       std::string* err) {
  if (n <= 0 || n > kMaxProblems) return (*err = "gemm: 1..4 problems per launch"), false;
  std::memset(params, 0, sizeof(*params));
  int total = 0, bn_max = 64;
  for (int i = 0; i < n; ++i) {
    if (!build_gemm_problem(d[i], &params->p[i], err)) return false;
    params->p[i].tile_begin = total;
    total += params->p[i].tiles_m * params->p[i].tiles_n;
    bn_max = std::max(bn_max, params->p[i].bn);
  }
  params->nprob = n;
  params->stage_bytes = kATileBytes + bn_max * 128;
  const int budget = 227 * 1024 - 1024 - 512;
  params->stages = std::min(kMaxStages, budget / params->stage_bytes);
  *tiles = total;
  return true;
}

}  // namespace rldx

using namespace rldx;

extern "C" {

int rldx_version(void) { return 100; }

const char* rldx_last_error(void) { return t_last_error.c_str(); }

int rldx_device_supported(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return 0;
  return ensure_device() == RLDX_OK ? 1 : 0;
}

int rldx_get_device_error(unsigned int* code) {
  if (!code) return set_error(RLDX_ERR_ARG, "null code");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  unsigned int v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, g_rldx_err, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "read device error");
  e = cudaMemcpyToSymbol(g_rldx_err, &zero, sizeof(zero));
  if (e != cudaSuccess) return cuda_fail(e, "clear device error");
  *code = v;
  return RLDX_OK;
}

int rldx_gemm(const rldx_gemm_desc* problems, int nproblems, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!problems) return set_error(RLDX_ERR_ARG, "gemm: null problems");
  GemmParams params;
  int tiles = 0;
  std::string err;
  if (!build_gemm_params(problems, nproblems, &params, &tiles, &err))
    return set_error(RLDX_ERR_ARG, err);
  cudaError_t e = launch_gemm(params, tiles, static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  return RLDX_OK;
}

int rldx_joint_attention(const void* q, const void* k, const void* vt, int B, int H, int L, int Lp,
                         const uint8_t* key_mask, void* const* out, const int* seg_len, int nseg,
                         void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!q || !k || !vt || !out || !seg_len) return set_error(RLDX_ERR_ARG, "attention: null pointer");
  if (B <= 0 || H <= 0 || L <= 0 || Lp < L || Lp % 8 != 0)
    return set_error(RLDX_ERR_ARG, "attention: need B, H, L > 0, Lp >= L, Lp % 8 == 0");
  if (nseg < 1 || nseg > 3) return set_error(RLDX_ERR_ARG, "attention: nseg must be 1..3");
  if (!aligned16(q) || !aligned16(k) || !aligned16(vt))
    return set_error(RLDX_ERR_ARG, "attention: q/k/vt must be 16-byte aligned");
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  int sum = 0;
  for (int s = 0; s < nseg; ++s) {
    if (seg_len[s] <= 0 || !out[s] || !aligned16(out[s]))
      return set_error(RLDX_ERR_ARG, "attention: bad segment");
    p.seg_out[s] = static_cast<__nv_bfloat16*>(out[s]);
    p.seg_len[s] = seg_len[s];
    sum += seg_len[s];
  }
  if (sum != L) return set_error(RLDX_ERR_ARG, "attention: segment lengths must sum to L");
  p.nseg = nseg;
  p.L = L;
  p.H = H;
  p.B = B;
  p.key_mask = key_mask;
  p.scale_log2 = 1.4426950408889634f / 8.0f;
  std::string err;
  const uint64_t bh = static_cast<uint64_t>(B) * H;
  if (!make_tmap_3d(&p.tq, q, 64, L, bh, 128, static_cast<uint64_t>(L) * 128, 64, 128, 1, &err) ||
      !make_tmap_3d(&p.tk, k, 64, L, bh, 128, static_cast<uint64_t>(L) * 128, 64, 64, 1, &err) ||
      !make_tmap_3d(&p.tv, vt, L, 64, bh, static_cast<uint64_t>(Lp) * 2,
                    static_cast<uint64_t>(Lp) * 128, 64, 64, 1, &err))
    return set_error(RLDX_ERR_ARG, err);
  cudaError_t e = launch_attention(p, static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return RLDX_OK;
}

int rldx_layernorm(const void* in, int64_t ld_in, void* out, int64_t ld_out, int rows, int D,
                   float eps, const void* scale1p, const void* shift, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!in || !out || rows <= 0 || D <= 0 || D % 8 != 0 || D > 4096)
    return set_error(RLDX_ERR_ARG, "layernorm: need rows > 0, D % 8 == 0, D <= 4096");
  if (ld_in % 8 || ld_out % 8 || !aligned16(in) || !aligned16(out))
    return set_error(RLDX_ERR_ARG, "layernorm: rows must be 16-byte aligned");
  if ((scale1p == nullptr) != (shift == nullptr))
    return set_error(RLDX_ERR_ARG, "layernorm: scale1p and shift go together");
  LnParams p;
  std::memset(&p, 0, sizeof(p));
  p.seg[0].in = static_cast<const __nv_bfloat16*>(in);
  p.seg[0].out = static_cast<__nv_bfloat16*>(out);
  p.seg[0].scale1p = static_cast<const __nv_bfloat16*>(scale1p);
  p.seg[0].shift = static_cast<const __nv_bfloat16*>(shift);
  p.seg[0].rows = rows;
  p.seg[0].ld_in = static_cast<int>(ld_in);
  p.seg[0].ld_out = static_cast<int>(ld_out);
  p.seg[0].row_begin = 0;
  p.nseg = 1;
  p.D = D;
  p.total_rows = rows;
  p.eps = eps;
  cudaError_t e = launch_ln(p, static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "layernorm launch");
  return RLDX_OK;
}

int rldx_qk_rmsnorm_rope(const void* x, void* y, const void* w, const int32_t* pos,
                         const void* cos_table, const void* sin_table, int64_t tokens, int heads,
                         int head_dim, float eps, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!x || !y || !w || !pos || !cos_table || !sin_table || tokens <= 0 || heads <= 0)
    return set_error(RLDX_ERR_ARG, "qk_rmsnorm_rope: null pointer or empty shape");
  if (head_dim != 128) return set_error(RLDX_ERR_UNSUPPORTED, "qk_rmsnorm_rope: head_dim must be 128");
  if (!aligned16(x) || !aligned16(y) || !aligned16(w) || !aligned16(cos_table) || !aligned16(sin_table))
    return set_error(RLDX_ERR_ARG, "qk_rmsnorm_rope: pointers must be 16-byte aligned");
  cudaError_t e = launch_qk_rmsnorm_rope(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y),
      static_cast<const __nv_bfloat16*>(w), pos, static_cast<const __nv_bfloat16*>(cos_table),
      static_cast<const __nv_bfloat16*>(sin_table), tokens * heads, heads, eps,
      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "qk_rmsnorm_rope launch");
  return RLDX_OK;
}

int rldx_swiglu(const void* gate, const void* up, int64_t ld_in, void* out, int64_t ld_out,
                int64_t rows, int H, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!gate || !up || !out || rows <= 0 || H <= 0 || H % 8 != 0)
    return set_error(RLDX_ERR_ARG, "swiglu: need rows > 0, H % 8 == 0");
  if (ld_in % 8 || ld_out % 8 || !aligned16(gate) || !aligned16(up) || !aligned16(out))
    return set_error(RLDX_ERR_ARG, "swiglu: rows must be 16-byte aligned");
  cudaError_t e = launch_swiglu(static_cast<const __nv_bfloat16*>(gate),
                                static_cast<const __nv_bfloat16*>(up),
                                static_cast<__nv_bfloat16*>(out), rows, H, ld_in, ld_out,
                                sm_count(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "swiglu launch");
  return RLDX_OK;
}

}  // extern "C"
