// C-ABI entry points of the per-op kernels, error reporting and the host helpers that turn
// plain pointers and sizes into TMA descriptors and launch parameters.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <functional>
#include <map>
#include <queue>
#include <vector>
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

namespace {

bool make_tmap_4d(CUtensorMap* m, const void* base, const cuuint64_t (&dims)[4],
                  const cuuint64_t (&strides)[3], const cuuint32_t (&box)[4], std::string* err) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled(4d) failed with code " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

// ---- GEMM planning ----------------------------------------------------------------------------
// Cost model of one work unit on one SM, in nanoseconds, from measurements on B200: the SM's
// copy engine takes one TMA box at a time, at least ~400 cycles per box (up to ~32 KB) and
// ~92 bytes per cycle beyond, so a ring slot costs the sum of its A and B boxes; the tensor
// core does ~15 TFLOP/s per SM (dense bf16 near 1.9 GHz, M = 128 whatever the live rows) on the slots
// already landed; a unit pays a fixed pipeline fill, an epilogue proportional to its columns,
// and a K-split unit also writes its fp32 partial tile and (for the last one) reads all
// partials of the tile back from L2 (~114 bytes per ns).
constexpr double kFillBytesPerNs = 114.0;
constexpr double kMmaFlopsPerNs = 15000.0;
constexpr double kChunkNs = 20.0;
constexpr double kUnitNs = 1500.0;
constexpr double kTmaOpNs = 210.0;        // one TMA box occupies the SM's copy engine >= ~400 cycles
constexpr double kTmaBytesPerNs = 175.0;  // ... and streams ~92 bytes per cycle beyond ~36 KB
// A K-split unit also pays for its tile's arrival count and the epilogue warps' barrier rounds,
// and the last one waits for the partials of its tile before its epilogue can start: ~1 us
// beyond the partials' traffic (B200: the config-2 output projection runs 15.6 us on 64-column
// tiles without splits, 18.2 us on 128-column tiles split in two, which the model without this
// term ranked the other way round).
constexpr double kSplitNs = 1000.0;
constexpr int kMinSplitChunks = 4;
constexpr int kMaxSplit = 8;
constexpr size_t kCounterBytes = ((kMaxUnits * 4 + 255) / 256) * 256;

struct ProbShape {
  int M, N, K, m_step, tiles_m, a_rows, live_rows, nchunks, kdim3, cat, epi;
};

// Epilogue time per output column of a unit (ns), by epilogue mode, measured on B200 for the
// 16-warp epilogue: per-head RMSNorm + RoPE and SwiGLU cost about twice the plain store.
double epi_ns_per_col(int epi) {
  return (epi == RLDX_EPI_QKV || epi == RLDX_EPI_SWIGLU) ? 26.0 : 15.0;
}

// Ring slots of up to 64 KB: three stages fit beside the barriers, and boxes of 16-64 KB keep
// the copy engine's per-box cost below the tensor core's time for the slot.
constexpr int kSlotTargetBytes = 64 * 1024;

// 64-deep K chunks per ring slot (= per TMA box) for a tile of `bn` columns.
int ksub_for(const ProbShape& s, int bn) {
  const int per_chunk = (s.a_rows + bn) * 128;
  return s.kdim3 ? std::max(1, std::min(kSlotTargetBytes / per_chunk, 8)) : 1;
}

// One ring slot: the A and B boxes go through the SM's copy engine one after the other, the
// tensor core works on the previous slots meanwhile.
double slot_ns(const ProbShape& s, int bn, int ksub) {
  auto op = [](double bytes) { return std::max(kTmaOpNs, bytes / kTmaBytesPerNs); };
  const double tma = op(s.a_rows * 128.0 * ksub) + op(bn * 128.0 * ksub);
  const double mma = ksub * 128.0 * bn * 64.0 * 2.0 / kMmaFlopsPerNs;
  return std::max(tma, mma) + kChunkNs;
}

double unit_ns(const ProbShape& s, int bn, int chunks, int nsplit) {
  const int ksub = std::max(1, std::min(ksub_for(s, bn), chunks));
  double t = ((chunks + ksub - 1) / ksub) * slot_ns(s, bn, ksub);
  t += kUnitNs + bn * epi_ns_per_col(s.epi);
  if (nsplit > 1) t += s.live_rows * bn * 4.0 * 2.0 / kFillBytesPerNs + kSplitNs;
  return t;
}

// Units of one problem for a (bn, nsplit) choice, appended as costs.
void unit_costs(const ProbShape& s, int bn, int nsplit, std::vector<double>* out) {
  const int tiles = s.tiles_m * ((s.N + bn - 1) / bn);
  const int per = (s.nchunks + nsplit - 1) / nsplit;
  for (int t = 0; t < tiles; ++t)
    for (int k = 0; k < nsplit; ++k) {
      const int c = std::min(per, s.nchunks - k * per);
      out->push_back(unit_ns(s, bn, c, nsplit));
    }
}

// Makespan of the longest-processing-time-first assignment of `costs` to `ncta` CTAs.
double lpt_makespan(std::vector<double> costs, int nsm) {
  if (costs.empty()) return 0.0;
  std::sort(costs.begin(), costs.end(), std::greater<double>());
  const int ncta = std::min<int>(nsm, static_cast<int>(costs.size()));
  std::priority_queue<double, std::vector<double>, std::greater<double>> loads;
  for (int i = 0; i < ncta; ++i) loads.push(0.0);
  double mk = 0.0;
  for (double c : costs) {
    double l = loads.top() + c;
    loads.pop();
    loads.push(l);
    mk = std::max(mk, l);
  }
  return mk;
}

int normalize_split(int nchunks, int nsplit) {
  const int per = (nchunks + nsplit - 1) / nsplit;
  return (nchunks + per - 1) / per;  // no empty trailing split
}

// Tile width (from 64/128/256) and K-split count of every problem of one launch: for each
// tile-width combination, splits are added greedily while they shorten the modelled makespan;
// the best combination wins.  Results are cached per shape set (an MSAT control step repeats
// a handful of shape sets hundreds of times).
void choose_tiles_uncached(const ProbShape* sh, const int* fixed_bn, int n, int nsm,
                           bool can_split, int* best_bn, int* best_split) {
  double best_mk = 1e300;
  int cand[kMaxProblems][3], ncand[kMaxProblems];
  // 64-column tiles for multi-tile problems only when 128-column tiles leave SMs idle: there
  // they fill the SMs without K splits; elsewhere they only multiply the A re-reads
  long long tiles128 = 0;
  for (int i = 0; i < n; ++i) tiles128 += static_cast<long long>(sh[i].tiles_m) * ((sh[i].N + 127) / 128);
  const bool narrow = tiles128 < nsm;
  for (int i = 0; i < n; ++i) {
    if (fixed_bn[i]) {
      cand[i][0] = fixed_bn[i];
      ncand[i] = 1;
      continue;
    }
    const int nmax = std::max(64, round_up(sh[i].N, 64));
    int k = 0;
    for (int bn : {64, 128, 256}) {
      if (bn > nmax) continue;
      if (sh[i].tiles_m >= 2 && bn == 64 && nmax > 64 && !narrow) continue;  // A re-reads: keep tiles wide
      cand[i][k++] = bn;
    }
    ncand[i] = k;
  }
  int idx[kMaxProblems] = {0, 0, 0, 0};
  std::vector<double> c;
  while (true) {
    int bn[kMaxProblems], sp[kMaxProblems];
    for (int i = 0; i < n; ++i) {
      bn[i] = cand[i][idx[i]];
      sp[i] = 1;
    }
    auto eval = [&]() {
      c.clear();
      int units = 0;
      for (int i = 0; i < n; ++i) {
        unit_costs(sh[i], bn[i], sp[i], &c);
        units += sh[i].tiles_m * ((sh[i].N + bn[i] - 1) / bn[i]) * sp[i];
      }
      if (units > kMaxUnits) {
        // Beyond the explicit schedule's capacity the kernel deals units round-robin; bound
        // its makespan by the mean load plus the longest unit.
        double sum = 0.0, mx = 0.0;
        for (double x : c) {
          sum += x;
          mx = std::max(mx, x);
        }
        return sum / nsm + mx;
      }
      return lpt_makespan(c, nsm);
    };
    double mk = eval();
    if (can_split) {
      for (int iter = 0; iter < 16; ++iter) {
        int bi = -1, bs = 0;
        double bm = mk;
        for (int i = 0; i < n; ++i) {
          const int maxs = std::min(kMaxSplit, std::max(1, sh[i].nchunks / kMinSplitChunks));
          int ns = sp[i];
          do {
            ns = normalize_split(sh[i].nchunks, ns + 1);
          } while (ns == sp[i] && ns < maxs);
          if (ns <= sp[i] || ns > maxs) continue;
          const int old = sp[i];
          sp[i] = ns;
          const double m = eval();
          sp[i] = old;
          if (m < bm * 0.99) {
            bm = m;
            bi = i;
            bs = ns;
          }
        }
        // group move: every problem one split further at once (identical problems only gain
        // together, since the longest unit of any one of them bounds the makespan)
        int gsp[kMaxProblems];
        bool gmove = false;
        for (int i = 0; i < n; ++i) {
          const int maxs = std::min(kMaxSplit, std::max(1, sh[i].nchunks / kMinSplitChunks));
          int ns = sp[i];
          do {
            ns = normalize_split(sh[i].nchunks, ns + 1);
          } while (ns == sp[i] && ns < maxs);
          gsp[i] = (ns > sp[i] && ns <= maxs) ? ns : sp[i];
          gmove = gmove || gsp[i] != sp[i];
        }
        if (gmove) {
          int old[kMaxProblems];
          for (int i = 0; i < n; ++i) {
            old[i] = sp[i];
            sp[i] = gsp[i];
          }
          const double m = eval();
          for (int i = 0; i < n; ++i) sp[i] = old[i];
          if (m < bm * 0.99) {
            bm = m;
            bi = n;  // marks the group move
          }
        }
        if (bi < 0) break;
        if (bi == n) {
          for (int i = 0; i < n; ++i) sp[i] = gsp[i];
        } else {
          sp[bi] = bs;
        }
        mk = bm;
      }
    }
    if (mk < best_mk) {
      best_mk = mk;
      for (int i = 0; i < n; ++i) {
        best_bn[i] = bn[i];
        best_split[i] = sp[i];
      }
    }
    int i = 0;
    for (; i < n; ++i) {
      if (++idx[i] < ncand[i]) break;
      idx[i] = 0;
    }
    if (i == n) break;
  }
}

void choose_tiles(const ProbShape* sh, const int* fixed_bn, int n, int nsm, bool can_split,
                  int* best_bn, int* best_split) {
  std::vector<int> key = {n, nsm, can_split ? 1 : 0};
  for (int i = 0; i < n; ++i) {
    const ProbShape& s = sh[i];
    key.insert(key.end(), {s.M, s.N, s.K, s.m_step, s.a_rows, s.cat, s.epi, fixed_bn[i]});
  }
  static std::mutex mu;
  static std::map<std::vector<int>, std::vector<int>> cache;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      for (int i = 0; i < n; ++i) {
        best_bn[i] = it->second[2 * i];
        best_split[i] = it->second[2 * i + 1];
      }
      return;
    }
  }
  choose_tiles_uncached(sh, fixed_bn, n, nsm, can_split, best_bn, best_split);
  std::vector<int> v;
  for (int i = 0; i < n; ++i) v.insert(v.end(), {best_bn[i], best_split[i]});
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = v;
}

// Modelled makespan of a single-CTA plan (tile widths and splits given).
double single_makespan(const ProbShape* sh, int n, int nsm, const int* bn, const int* split) {
  std::vector<double> c;
  int units = 0;
  for (int i = 0; i < n; ++i) {
    unit_costs(sh[i], bn[i], split[i], &c);
    units += sh[i].tiles_m * ((sh[i].N + bn[i] - 1) / bn[i]) * split[i];
  }
  if (units > kMaxUnits) {
    double sum = 0.0, mx = 0.0;
    for (double x : c) {
      sum += x;
      mx = std::max(mx, x);
    }
    return sum / nsm + mx;
  }
  return lpt_makespan(c, nsm);
}

// One unit of a CTA pair: 256 rows x bn columns, each CTA loading 128 rows of A and bn/2 rows of
// B per slot and computing 128 x bn on its own tensor core.
double pair_unit_ns(const ProbShape& s, int bn) {
  const int bh = bn / 2;
  const int ksub = s.kdim3 ? std::max(1, std::min(kSlotTargetBytes / ((128 + bh) * 128), 8)) : 1;
  auto op = [](double bytes) { return std::max(kTmaOpNs, bytes / kTmaBytesPerNs); };
  const double tma = op(128.0 * 128.0 * ksub) + op(bh * 128.0 * ksub);
  const double mma = ksub * 128.0 * bn * 64.0 * 2.0 / kMmaFlopsPerNs;
  const int slots = (s.nchunks + ksub - 1) / ksub;
  return slots * (std::max(tma, mma) + kChunkNs) + kUnitNs + bn * epi_ns_per_col(s.epi);
}

double pair_makespan(const ProbShape* sh, int n, int nsm) {
  std::vector<double> c;
  for (int i = 0; i < n; ++i) {
    const int bn = sh[i].N > 128 ? 256 : 128;
    const int units = ((sh[i].M + 255) / 256) * ((sh[i].N + bn - 1) / bn);
    const double u = pair_unit_ns(sh[i], bn);
    for (int k = 0; k < units; ++k) c.push_back(u);
  }
  const int npairs = nsm / 2;
  if (static_cast<int>(c.size()) > kMaxUnits) {
    double sum = 0.0;
    for (double x : c) sum += x;
    return sum / npairs + c[0];
  }
  return lpt_makespan(c, npairs);
}

// RLDX_GEMM_PAIR=0 keeps every launch on single-CTA tiles; =2 runs every launch that can on
// CTA pairs (A/B measurement).
int pair_mode() {
  static int v = [] {
    const char* e = std::getenv("RLDX_GEMM_PAIR");
    return (e && e[0] == '0') ? 0 : (e && e[0] == '2') ? 2 : 1;
  }();
  return v;
}

bool split_disabled() {
  static int v = [] {
    const char* e = std::getenv("RLDX_GEMM_SPLIT");
    return (e && e[0] == '0') ? 1 : 0;
  }();
  return v != 0;
}

}  // namespace

// Validates one GEMM description and fills the shape-only fields of the device problem.
bool validate_gemm_problem(const rldx_gemm_desc& d, GemmProblem* p, std::string* err) {
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
  if (d.tile_n != 0 && (d.tile_n < 64 || d.tile_n > 256 || d.tile_n % 64 != 0))
    return (*err = "gemm: tile_n must be 64..256, x64"), false;

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
  if (d.epilogue == RLDX_EPI_SWIGLU && d.N % 64 != 0)
    return (*err = "gemm: SwiGLU needs N % 64 == 0 (interleaved 32 gate + 32 up)"), false;
  if (d.epilogue == RLDX_EPI_QKV) {
    if (!d.q || !d.k || !d.vt || !d.q_norm_w || !d.k_norm_w || !d.rope_cos || !d.rope_sin)
      return (*err = "gemm: QKV epilogue needs q, k, vt, norms and rope tables"), false;
    if (d.H <= 0 || d.N != 3 * 64 * d.H) return (*err = "gemm: QKV needs N == 3 * H * 64"), false;
    if (d.L <= 0 || d.Lp < d.L || d.Lp % 8 != 0) return (*err = "gemm: QKV needs Lp >= L, Lp % 8 == 0"), false;
    if (d.rows_in <= 0 || d.tok_off < 0 || d.tok_off + d.rows_in > d.L)
      return (*err = "gemm: QKV rows_in/tok_off outside L"), false;
    if (!aligned16(d.q) || !aligned16(d.k) || !aligned16(d.q_norm_w) || !aligned16(d.k_norm_w) ||
        !aligned16(d.rope_cos) || !aligned16(d.rope_sin))
      return (*err = "gemm: QKV buffers must be 16-byte aligned"), false;
  }
  if (d.rows_in < 0 || (d.rows_in > 0 && d.rows_out <= 0))
    return (*err = "gemm: bad rows_in / rows_out"), false;

  p->M = d.M;
  p->N = d.N;
  p->K = d.K;
  p->m_step = m_step;
  p->tiles_m = tiles_m;
  p->a_rows = std::min(128, round_up(std::min(m_step, d.M), 8));
  p->nchunks = (d.K + 63) / 64;
  p->kdim3 = (d.K % 64 == 0) ? 1 : 0;
  p->cat_ids = reinterpret_cast<const long long*>(d.cat_ids);

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
  e.rope_identity = d.rope_identity ? 1 : 0;
  return true;
}

bool build_gemm_params(const rldx_gemm_desc* d, int n, void* ws, size_t ws_bytes,
                       GemmParams* params, size_t* ws_needed, std::string* err) {
  if (n <= 0 || n > kMaxProblems) return (*err = "gemm: 1..4 problems per launch"), false;
  std::memset(params, 0, sizeof(*params));
  const int nsm = std::min(sm_count(), kMaxCtas);
  for (int i = 1; i < n; ++i)
    if (d[i].epilogue != d[0].epilogue)
      return (*err = "gemm: every problem of one launch must use the same epilogue"), false;
  ProbShape sh[kMaxProblems];
  for (int i = 0; i < n; ++i) {
    GemmProblem& p = params->p[i];
    if (!validate_gemm_problem(d[i], &p, err)) return false;
    ProbShape& s = sh[i];
    s.M = p.M;
    s.N = p.N;
    s.K = p.K;
    s.m_step = p.m_step;
    s.tiles_m = p.tiles_m;
    s.a_rows = p.a_rows;
    s.live_rows = std::min(p.m_step, p.M);
    s.nchunks = p.nchunks;
    s.kdim3 = p.kdim3;
    s.cat = d[i].cat_ids ? 1 : 0;
    s.epi = d[i].epilogue;
  }

  // ---- tile width and K splits: minimise the modelled LPT makespan ----
  const bool can_split = (ws != nullptr || ws_needed != nullptr) && !split_disabled();
  int fixed_bn[kMaxProblems], best_bn[kMaxProblems], best_split[kMaxProblems];
  for (int i = 0; i < n; ++i) fixed_bn[i] = d[i].tile_n;
  choose_tiles(sh, fixed_bn, n, nsm, can_split, best_bn, best_split);

  // ---- CTA pairs (cta_group::2, 256-row M tiles): launches with plenty of large tiles, and
  // smaller ones whose modelled makespan on pairs beats the single-CTA plan (a pair halves each
  // SM's copy-engine boxes per tile: the small-batch projections whose rows fit a few tiles) ----
  bool pair = pair_mode() != 0 && nsm >= 2;
  bool large = true;
  long long tiles128 = 0;
  for (int i = 0; i < n && pair; ++i) {
    pair = !d[i].cat_ids && d[i].tile_n == 0;
    large = large && d[i].M >= 512;
    tiles128 += static_cast<long long>((d[i].M + 127) / 128) * ((d[i].N + 127) / 128);
  }
  if (pair && pair_mode() != 2 && !(large && tiles128 >= 4LL * nsm)) {
    const double single_mk = single_makespan(sh, n, nsm, best_bn, best_split);
    pair = pair_makespan(sh, n, nsm) < 0.9 * single_mk;
  }
  if (pair) {
    for (int i = 0; i < n; ++i) {
      best_bn[i] = d[i].N > 128 ? 256 : 128;
      best_split[i] = 1;
    }
  }

  // ---- workspace layout: [tile counters][fp32 partial tiles] ----
  size_t need = 0;
  for (int pass = 0; pass < 2; ++pass) {
    size_t off_f = 0;
    int cnt = 0;
    bool any = false;
    for (int i = 0; i < n; ++i) {
      GemmProblem& p = params->p[i];
      p.bn = best_bn[i];
      p.tiles_n = (p.N + p.bn - 1) / p.bn;
      p.nsplit = best_split[i];
      p.split_chunks = (p.nchunks + p.nsplit - 1) / p.nsplit;
      p.ws_off = 0;
      p.cnt_off = 0;
      if (p.nsplit > 1) {
        any = true;
        p.ws_off = static_cast<long long>(off_f);
        p.cnt_off = cnt;
        off_f += static_cast<size_t>(p.tiles_m) * p.tiles_n * p.nsplit * 128 * p.bn;
        cnt += p.tiles_m * p.tiles_n;
      }
    }
    // the arrival counters of every split tile must fit the counter block ahead of the partials
    const bool counters_fit = static_cast<size_t>(cnt) * sizeof(unsigned int) <= kCounterBytes;
    need = (any && counters_fit) ? kCounterBytes + off_f * 4 : 0;
    if (ws_needed) *ws_needed = std::max(*ws_needed, need);
    if (!any || (counters_fit && ws != nullptr && need <= ws_bytes)) break;
    for (int i = 0; i < n; ++i) best_split[i] = 1;  // no (or too small a) workspace
  }
  params->pair = pair ? 1 : 0;
  if (pair) {
    for (int i = 0; i < n; ++i) {
      GemmProblem& p = params->p[i];
      p.tiles_m = (p.M + 255) / 256;  // pair tiles; each CTA owns 128 rows (m_step)
      p.m_step = 128;
      p.a_rows = 128;
    }
  }
  params->ws = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kCounterBytes);
  params->counters = static_cast<unsigned int*>(ws);
  if (!ws) {
    params->ws = nullptr;
    params->counters = nullptr;
  }

  // ---- ring slot: ksub chunks of every problem must fit one slot ----
  int slot = 0;
  for (int i = 0; i < n; ++i) {
    GemmProblem& p = params->p[i];
    const int per_chunk = (p.a_rows + (pair ? p.bn / 2 : p.bn)) * 128;
    p.ksub = p.kdim3 ? std::max(1, std::min({kSlotTargetBytes / per_chunk, 8, p.split_chunks})) : 1;
    slot = std::max(slot, p.ksub * per_chunk);
  }
  params->slot_bytes = slot;
  const int budget = 227 * 1024 - 1024 - kRingSlack - 256;
  params->stages = std::min(kMaxStages, budget / slot);
  if (params->stages < 2) return (*err = "gemm: ring does not fit shared memory"), false;

  // ---- tensor maps ----
  for (int i = 0; i < n; ++i) {
    GemmProblem& p = params->p[i];
    const rldx_gemm_desc& q = d[i];
    if (p.kdim3) {
      if (!make_tmap_3d(&p.ta, q.a, 64, p.M, p.nchunks, static_cast<uint64_t>(q.lda) * 2, 128, 64,
                        p.a_rows, p.ksub, err))
        return false;
      if (q.cat_ids) {
        const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(p.N), static_cast<cuuint64_t>(p.nchunks),
                                    static_cast<cuuint64_t>(q.num_cats)};
        const cuuint64_t strides[3] = {static_cast<cuuint64_t>(q.ldb) * 2, 128,
                                       static_cast<cuuint64_t>(q.b_cat_stride) * 2};
        const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(p.bn), static_cast<cuuint32_t>(p.ksub), 1};
        if (!make_tmap_4d(&p.tb, q.b, dims, strides, box, err)) return false;
      } else if (!make_tmap_3d(&p.tb, q.b, 64, p.N, p.nchunks, static_cast<uint64_t>(q.ldb) * 2, 128,
                               64, pair ? p.bn / 2 : p.bn, p.ksub, err)) {
        return false;
      }
    } else {
      if (!make_tmap_2d(&p.ta, q.a, q.K, p.M, static_cast<uint64_t>(q.lda) * 2, 64, p.a_rows, err))
        return false;
      if (q.cat_ids) {
        if (!make_tmap_3d(&p.tb, q.b, q.K, p.N, q.num_cats, static_cast<uint64_t>(q.ldb) * 2,
                          static_cast<uint64_t>(q.b_cat_stride) * 2, 64, p.bn, 1, err))
          return false;
      } else if (!make_tmap_2d(&p.tb, q.b, q.K, p.N, static_cast<uint64_t>(q.ldb) * 2, 64,
                               pair ? p.bn / 2 : p.bn, err)) {
        return false;
      }
    }
  }

  // ---- units and the LPT schedule ----
  int total = 0;
  for (int i = 0; i < n; ++i) {
    GemmProblem& p = params->p[i];
    p.unit_begin = total;
    total += p.tiles_m * p.tiles_n * p.nsplit;
  }
  params->nprob = n;
  params->nunits = total;
  params->ncta = pair ? 2 * std::min(nsm / 2, total) : std::min(nsm, total);
  const int nlists = pair ? params->ncta / 2 : params->ncta;  // unit lists: one per CTA or pair
  if (total > kMaxUnits) {
    params->explicit_sched = 0;
    return true;
  }
  params->explicit_sched = 1;
  struct U {
    double cost;
    int id;
  };
  std::vector<U> us;
  us.reserve(total);
  for (int i = 0; i < n; ++i) {
    const GemmProblem& p = params->p[i];
    for (int local = 0; local < p.tiles_m * p.tiles_n * p.nsplit; ++local) {
      const int ks = local % p.nsplit;
      const int c = std::min(p.split_chunks, p.nchunks - ks * p.split_chunks);
      us.push_back({unit_ns(sh[i], p.bn, c, p.nsplit), p.unit_begin + local});
    }
  }
  std::stable_sort(us.begin(), us.end(), [](const U& a, const U& b) { return a.cost > b.cost; });
  using Load = std::pair<double, int>;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> loads;
  for (int c = 0; c < nlists; ++c) loads.push({0.0, c});
  std::vector<std::vector<int>> lists(nlists);
  for (const U& u : us) {
    Load l = loads.top();
    loads.pop();
    lists[l.second].push_back(u.id);
    l.first += u.cost;
    loads.push(l);
  }
  int off = 0;
  for (int c = 0; c < nlists; ++c) {
    params->cta_begin[c] = static_cast<unsigned short>(off);
    for (int id : lists[c]) params->sched[off++] = static_cast<unsigned short>(id);
  }
  params->cta_begin[nlists] = static_cast<unsigned short>(off);
  return true;
}

}  // namespace rldx

using namespace rldx;

extern "C" {

int rldx_version(void) { return 111; }

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
  static thread_local GemmParams params;
  std::string err;
  if (!build_gemm_params(problems, nproblems, nullptr, 0, &params, nullptr, &err))
    return set_error(RLDX_ERR_ARG, err);
  cudaError_t e = launch_gemm(params, static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  return RLDX_OK;
}

int rldx_gemm_workspace_size(const rldx_gemm_desc* problems, int nproblems, uint64_t* bytes) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!problems || !bytes) return set_error(RLDX_ERR_ARG, "gemm_workspace_size: null argument");
  static thread_local GemmParams params;
  std::string err;
  size_t need = 0;
  if (!build_gemm_params(problems, nproblems, nullptr, 0, &params, &need, &err))
    return set_error(RLDX_ERR_ARG, err);
  *bytes = need;
  return RLDX_OK;
}

int rldx_gemm_plan(const rldx_gemm_desc* problems, int nproblems, int* plan) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!problems || !plan) return set_error(RLDX_ERR_ARG, "gemm_plan: null argument");
  static thread_local GemmParams params;
  std::string err;
  // planned as if an unbounded workspace were given (the pointer is only recorded, never read)
  void* any_ws = reinterpret_cast<void*>(static_cast<uintptr_t>(256));
  if (!build_gemm_params(problems, nproblems, any_ws, SIZE_MAX, &params, nullptr, &err))
    return set_error(RLDX_ERR_ARG, err);
  plan[0] = params.pair;
  plan[1] = params.ncta;
  plan[2] = params.stages;
  plan[3] = params.p[0].bn;
  plan[4] = params.p[0].nsplit;
  return RLDX_OK;
}

int rldx_gemm_ws(const rldx_gemm_desc* problems, int nproblems, void* workspace,
                 uint64_t workspace_bytes, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!problems) return set_error(RLDX_ERR_ARG, "gemm: null problems");
  if (workspace && !aligned16(workspace)) return set_error(RLDX_ERR_ARG, "gemm: workspace must be 16-byte aligned");
  static thread_local GemmParams params;
  std::string err;
  if (!build_gemm_params(problems, nproblems, workspace, workspace ? workspace_bytes : 0, &params,
                         nullptr, &err))
    return set_error(RLDX_ERR_ARG, err);
  cudaError_t e = launch_gemm(params, static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  return RLDX_OK;
}

int rldx_attention(const rldx_attention_desc* d, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!d || !d->q || !d->k || !d->vt) return set_error(RLDX_ERR_ARG, "attention: null pointer");
  const int B = d->B, H = d->H, L = d->L, Lp = d->Lp, hd = d->head_dim;
  const int kvh = d->kv_heads > 0 ? d->kv_heads : H;
  if (B <= 0 || H <= 0 || L <= 0 || Lp < L || Lp % 8 != 0 || H % kvh != 0)
    return set_error(RLDX_ERR_ARG, "attention: need B, H, L > 0, Lp >= L, Lp % 8 == 0, kv_heads | H");
  if (hd != 64 && hd != 128) return set_error(RLDX_ERR_UNSUPPORTED, "attention: head_dim must be 64 or 128");
  if (d->tiles_per_cta < 0 || d->tiles_per_cta > 2) return set_error(RLDX_ERR_ARG, "attention: tiles_per_cta must be 0, 1 or 2");
  if (d->nseg < 1 || d->nseg > 3) return set_error(RLDX_ERR_ARG, "attention: nseg must be 1..3");
  if (!aligned16(d->q) || !aligned16(d->k) || !aligned16(d->vt))
    return set_error(RLDX_ERR_ARG, "attention: q/k/vt must be 16-byte aligned");
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  int sum = 0;
  for (int s = 0; s < d->nseg; ++s) {
    const int ld = d->out_ld[s] > 0 ? d->out_ld[s] : H * hd;
    if (d->seg_len[s] <= 0 || !d->out[s] || !aligned16(d->out[s]) || ld % 8 != 0 || ld < H * hd)
      return set_error(RLDX_ERR_ARG, "attention: bad segment");
    p.seg_out[s] = static_cast<__nv_bfloat16*>(d->out[s]);
    p.seg_len[s] = d->seg_len[s];
    p.seg_ld[s] = ld;
    sum += d->seg_len[s];
  }
  if (sum != L) return set_error(RLDX_ERR_ARG, "attention: segment lengths must sum to L");
  p.nseg = d->nseg;
  p.L = L;
  p.H = H;
  p.B = B;
  p.kv_heads = kvh;
  p.causal = d->causal ? 1 : 0;
  p.causal_block = d->causal_block > 1 ? d->causal_block : 1;
  if (d->out_dim < 0 || d->out_dim > hd || d->out_dim % 8 != 0) return set_error(RLDX_ERR_ARG, "attention: bad out_dim");
  p.out_dim = d->out_dim;
  p.key_mask = d->key_mask;
  p.head_dim = hd;
  p.tiles_per_cta = d->tiles_per_cta;
  p.scale_log2 = 1.4426950408889634f / std::sqrt(static_cast<float>(hd));
  std::string err;
  const uint64_t bq = static_cast<uint64_t>(B) * H, bkv = static_cast<uint64_t>(B) * kvh;
  const uint64_t h64 = static_cast<uint64_t>(hd);
  if (!make_tmap_3d(&p.tq, d->q, h64, L, bq, h64 * 2, static_cast<uint64_t>(L) * h64 * 2, 64, 128, 1, &err) ||
      !make_tmap_3d(&p.tk, d->k, h64, L, bkv, h64 * 2, static_cast<uint64_t>(L) * h64 * 2, 64, 64, 1, &err) ||
      !make_tmap_3d(&p.tv, d->vt, L, h64, bkv, static_cast<uint64_t>(Lp) * 2, static_cast<uint64_t>(Lp) * h64 * 2, 64,
                    static_cast<uint32_t>(h64), 1, &err))
    return set_error(RLDX_ERR_ARG, err);
  cudaError_t e = launch_attention(p, static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return RLDX_OK;
}

int rldx_joint_attention(const void* q, const void* k, const void* vt, int B, int H, int L, int Lp,
                         int head_dim, const uint8_t* key_mask, void* const* out, const int* seg_len,
                         int nseg, int tiles_per_cta, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!q || !k || !vt || !out || !seg_len) return set_error(RLDX_ERR_ARG, "attention: null pointer");
  if (B <= 0 || H <= 0 || L <= 0 || Lp < L || Lp % 8 != 0)
    return set_error(RLDX_ERR_ARG, "attention: need B, H, L > 0, Lp >= L, Lp % 8 == 0");
  if (head_dim != 64 && head_dim != 128) return set_error(RLDX_ERR_UNSUPPORTED, "attention: head_dim must be 64 or 128");
  if (tiles_per_cta < 0 || tiles_per_cta > 2) return set_error(RLDX_ERR_ARG, "attention: tiles_per_cta must be 0, 1 or 2");
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
  p.head_dim = head_dim;
  p.tiles_per_cta = tiles_per_cta;
  p.scale_log2 = 1.4426950408889634f / std::sqrt(static_cast<float>(head_dim));
  std::string err;
  const uint64_t bh = static_cast<uint64_t>(B) * H;
  const uint64_t hd = static_cast<uint64_t>(head_dim);
  // Q, K: [bh, L, hd] loaded as 64-dim chunks (128-byte rows); V^T: [bh, hd, Lp], 64-key boxes
  if (!make_tmap_3d(&p.tq, q, hd, L, bh, hd * 2, static_cast<uint64_t>(L) * hd * 2, 64, 128, 1, &err) ||
      !make_tmap_3d(&p.tk, k, hd, L, bh, hd * 2, static_cast<uint64_t>(L) * hd * 2, 64, 64, 1, &err) ||
      !make_tmap_3d(&p.tv, vt, L, hd, bh, static_cast<uint64_t>(Lp) * 2, static_cast<uint64_t>(Lp) * hd * 2, 64,
                    static_cast<uint32_t>(hd), 1, &err))
    return set_error(RLDX_ERR_ARG, err);
  cudaError_t e = launch_attention(p, static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return RLDX_OK;
}

int rldx_qkv_prep(const rldx_qkv_segment* segs, int nseg, int B, int H, int L, int Lp, float eps,
                  void* q, void* k, void* vt, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!segs || !q || !k || !vt) return set_error(RLDX_ERR_ARG, "qkv_prep: null pointer");
  if (nseg < 1 || nseg > 3 || B <= 0 || H <= 0 || L <= 0 || Lp < L || Lp % 8 != 0)
    return set_error(RLDX_ERR_ARG, "qkv_prep: need 1..3 segments, B, H, L > 0, Lp >= L, Lp % 8 == 0");
  if (!aligned16(q) || !aligned16(k) || !aligned16(vt)) return set_error(RLDX_ERR_ARG, "qkv_prep: q/k/vt must be 16-byte aligned");
  QkvPrepParams p;
  std::memset(&p, 0, sizeof(p));
  int sum = 0;
  for (int i = 0; i < nseg; ++i) {
    const rldx_qkv_segment& s = segs[i];
    if (!s.qkv || !s.q_norm || !s.k_norm || s.rows <= 0 || s.ld < 3LL * H * 64 || s.ld % 8 != 0 ||
        !aligned16(s.qkv) || s.rope_from < 0 || (s.rope_cos != nullptr) != (s.rope_sin != nullptr) ||
        (B > 1 && s.batch_stride < static_cast<int64_t>(s.rows) * s.ld))
      return set_error(RLDX_ERR_ARG, "qkv_prep: bad segment");
    p.seg[i].qkv = static_cast<const __nv_bfloat16*>(s.qkv);
    p.seg[i].ld = s.ld;
    p.seg[i].batch_stride = s.batch_stride;
    p.seg[i].rows = s.rows;
    p.seg[i].rope_from = s.rope_from;
    p.seg[i].qn = static_cast<const __nv_bfloat16*>(s.q_norm);
    p.seg[i].kn = static_cast<const __nv_bfloat16*>(s.k_norm);
    p.seg[i].cos = s.rope_cos;
    p.seg[i].sin = s.rope_sin;
    sum += s.rows;
  }
  if (sum != L) return set_error(RLDX_ERR_ARG, "qkv_prep: segment rows must sum to L");
  p.nseg = nseg;
  p.B = B;
  p.H = H;
  p.L = L;
  p.Lp = Lp;
  p.eps = eps;
  p.q = static_cast<__nv_bfloat16*>(q);
  p.k = static_cast<__nv_bfloat16*>(k);
  p.vt = static_cast<__nv_bfloat16*>(vt);
  cudaError_t e = launch_qkv_prep(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "qkv_prep launch");
  return RLDX_OK;
}

static int res_norm_impl(const rldx_res_ln_segment* segs, int nseg, int fp32_sum, int rms, float eps, void* stream);

int rldx_res_layernorm(const rldx_res_ln_segment* segs, int nseg, int fp32_sum, float eps, void* stream) {
  return res_norm_impl(segs, nseg, fp32_sum, 0, eps, stream);
}

int rldx_res_rmsnorm(const rldx_res_ln_segment* segs, int nseg, float eps, void* stream) {
  return res_norm_impl(segs, nseg, 0, 1, eps, stream);
}

static int res_norm_impl(const rldx_res_ln_segment* segs, int nseg, int fp32_sum, int rms, float eps, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!segs || nseg < 1 || nseg > 2) return set_error(RLDX_ERR_ARG, "res_layernorm: need 1 or 2 segments");
  ResLnParams p;
  std::memset(&p, 0, sizeof(p));
  int row = 0;
  for (int i = 0; i < nseg; ++i) {
    const rldx_res_ln_segment& s = segs[i];
    if (!s.x || !s.ln_out || s.rows <= 0 || s.D <= 0 || s.D % 8 || s.D > 4096 || s.ld < s.D || s.ld % 8 ||
        !aligned16(s.x) || !aligned16(s.ln_out) || (s.y && !aligned16(s.y)) || (s.v1 && !aligned16(s.v1)) ||
        (s.v2 && !aligned16(s.v2)) || (s.sum_out && !aligned16(s.sum_out)))
      return set_error(RLDX_ERR_ARG, "res_layernorm: bad segment (D % 8, D <= 4096, 16-byte aligned rows)");
    ResLnSeg& d = p.seg[i];
    d.x = static_cast<const __nv_bfloat16*>(s.x);
    d.y = static_cast<const __nv_bfloat16*>(s.y);
    d.v1 = static_cast<const __nv_bfloat16*>(s.v1);
    d.v2 = static_cast<const __nv_bfloat16*>(s.v2);
    if (rms && (!s.w || !aligned16(s.w))) return set_error(RLDX_ERR_ARG, "res_rmsnorm: need a 16-byte aligned weight");
    d.w = static_cast<const __nv_bfloat16*>(s.w);
    d.sum_out = static_cast<__nv_bfloat16*>(s.sum_out);
    d.ln_out = static_cast<__nv_bfloat16*>(s.ln_out);
    d.rows = s.rows;
    d.D = s.D;
    d.ld = static_cast<int>(s.ld);
    d.row_begin = row;
    row += s.rows;
    p.dmax = std::max(p.dmax, s.D);
  }
  p.nseg = nseg;
  p.total_rows = row;
  p.fp32_sum = fp32_sum ? 1 : 0;
  p.rms = rms ? 1 : 0;
  p.eps = eps;
  cudaError_t e = launch_res_ln(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "res_layernorm launch");
  return RLDX_OK;
}

int rldx_swiglu_bias(const rldx_swiglu_bias_segment* segs, int nseg, void* stream) {
  int rc = ensure_device();
  if (rc != RLDX_OK) return rc;
  if (!segs || nseg < 1 || nseg > 2) return set_error(RLDX_ERR_ARG, "swiglu_bias: need 1 or 2 segments");
  SwigluBiasParams p;
  std::memset(&p, 0, sizeof(p));
  int row = 0;
  for (int i = 0; i < nseg; ++i) {
    const rldx_swiglu_bias_segment& s = segs[i];
    if (!s.gate || !s.up || !s.bias_gate || !s.bias_up || !s.out || s.rows <= 0 || s.H <= 0 || s.H % 8 ||
        s.ld_in % 8 || s.ld_out % 8 || !aligned16(s.gate) || !aligned16(s.up) || !aligned16(s.bias_gate) ||
        !aligned16(s.bias_up) || !aligned16(s.out))
      return set_error(RLDX_ERR_ARG, "swiglu_bias: bad segment (H % 8, 16-byte aligned rows)");
    SwigluBiasSeg& d = p.seg[i];
    d.gate = static_cast<const __nv_bfloat16*>(s.gate);
    d.up = static_cast<const __nv_bfloat16*>(s.up);
    d.bg = static_cast<const __nv_bfloat16*>(s.bias_gate);
    d.bu = static_cast<const __nv_bfloat16*>(s.bias_up);
    d.out = static_cast<__nv_bfloat16*>(s.out);
    d.ld_in = s.ld_in;
    d.ld_out = s.ld_out;
    d.rows = s.rows;
    d.H = s.H;
    d.row_begin = row;
    row += s.rows;
    p.hmax = std::max(p.hmax, s.H);
  }
  p.nseg = nseg;
  p.total_rows = row;
  cudaError_t e = launch_swiglu_bias(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "swiglu_bias launch");
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
  if (tokens * heads >= (1LL << 31)) return set_error(RLDX_ERR_UNSUPPORTED, "qk_rmsnorm_rope: too many rows");
  QkNormRopeParams p;
  std::memset(&p, 0, sizeof(p));
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.x_tok_stride = static_cast<long long>(heads) * 128;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.wq = p.wk = static_cast<const __nv_bfloat16*>(w);
  p.pos = pos;
  p.cos = static_cast<const __nv_bfloat16*>(cos_table);
  p.sin = static_cast<const __nv_bfloat16*>(sin_table);
  p.nrows = static_cast<unsigned>(tokens * heads);
  p.heads = p.Hq = static_cast<unsigned>(heads);
  p.T = static_cast<unsigned>(tokens);
  p.layout = 0;
  p.hd = p.out_hd = 128;
  p.norm = 1;
  p.eps = eps;
  cudaError_t e = launch_qk_rmsnorm_rope(p, static_cast<cudaStream_t>(stream));
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
