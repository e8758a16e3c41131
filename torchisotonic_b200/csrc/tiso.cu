// The C ABI of include/tiso.h: argument checks, the choice of kernel configuration, launches.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <utility>

#include "../../include/tiso.h"
#include "fit_kernels.cuh"
#include "grad_kernels.cuh"
#include "grad_rows.cuh"
#include "short_rows.cuh"

namespace tiso {
namespace {
thread_local std::string g_error;
}  // namespace

// Records the calling thread's error message (for tiso_last_error) and returns code; also used
// by the calibration entry points (calib.cu).
int report_error(int code, const std::string& msg) {
  g_error = msg;
  return code;
}

namespace {

int fail(int code, const std::string& msg) { return report_error(code, msg); }

int cuda_fail(cudaError_t e, const char* what) {
  return fail(TISO_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

size_t align256(size_t x) { return (x + 255) & ~size_t{255}; }

int ilog2(int x) {
  int r = 0;
  while ((1 << r) < x) ++r;
  return r;
}

// Allows a kernel more than 48 KB of dynamic shared memory: once per (kernel, device).
std::mutex g_smem_mu;
std::set<std::pair<const void*, int>> g_smem_done;

template <typename F>
cudaError_t allow_smem(F* kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  std::lock_guard<std::mutex> lock(g_smem_mu);
  if (g_smem_done.count(key)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes));
  if (e == cudaSuccess) g_smem_done.insert(key);
  return e;
}

// ---------------------------------------------------------------------------------------------
// Forward

struct FitPlan {
  bool whole;      // rows fit one segment: one launch
  bool climb;      // long rows: the tree of tile merges climbed by climb_kernel (few rows)
  int log2g;
  int threads;     // long rows: threads per tile CTA
  int32_t tile;    // long rows: elements per tile
  int64_t tiles;   // per row (long rows)
  int64_t words;
  int64_t grid;
};

int64_t levels_of(int64_t tiles) {
  int64_t l = 0;
  while ((int64_t{1} << l) < tiles) ++l;
  return l;
}

FitPlan plan_fit(int64_t batch, int64_t n) {
  FitPlan p{};
  if (n <= kTile) {
    p.whole = true;
    const int g = static_cast<int>((n + kK - 1) / kK);
    p.log2g = ilog2(g < 1 ? 1 : g);
    const int64_t per_cta = kThreads >> p.log2g;
    p.tiles = 1;
    p.grid = (batch + per_cta - 1) / per_cta;
    return p;
  }
  // The tree of tile merges: for fewer than 512 rows a thread per pair of tiles climbing it
  // (climb_kernel), else a warp per row taking the levels in turn (merge_rows_kernel). Tiles:
  // one warp and 512 elements, except for many rows of few tiles each (shallow trees in all),
  // where four-warp tiles of 2048 (a quarter of the merges) win. Measured on B200.
  const int64_t tiles512 = (n + kTile - 1) / kTile;
  p.whole = false;
  p.climb = batch < 512;
  const bool few = levels_of(tiles512) >= 12 || batch * tiles512 <= 65536;
  p.threads = (few && !p.climb) ? kLongThreads : kThreads;
  p.tile = kK * p.threads;
  p.log2g = ilog2(p.threads);
  p.tiles = (n + p.tile - 1) / p.tile;
  p.words = (p.tiles + 31) / 32;
  p.grid = batch * p.tiles;
  return p;
}

struct FitLayout {
  size_t start, w, t, lo, hi, nan, ct, cw, nz, cnt, total;
  int64_t cnt_per_row;
};

// Nodes of a row's tree of tiles (levels whose half-span is below the tile count).
int64_t tree_nodes(int64_t tiles) {
  int64_t total = 0;
  for (int64_t span = 2; span / 2 < tiles; span *= 2) total += (tiles + span - 1) / span;
  return total;
}

FitLayout fit_layout(const FitPlan& p, int64_t batch, size_t s_bytes) {
  FitLayout l{};
  const size_t tiles = static_cast<size_t>(batch * p.tiles);
  const size_t slots = tiles * static_cast<size_t>(p.tile);
  size_t o = 0;
  l.start = o; o = align256(o + slots * 4);
  l.w = o;     o = align256(o + slots * s_bytes);
  l.t = o;     o = align256(o + slots * s_bytes);
  l.lo = o;    o = align256(o + tiles * 4);
  l.hi = o;    o = align256(o + tiles * 4);
  l.nan = o;   o = align256(o + tiles * 4);
  l.ct = o;    o = align256(o + tiles * s_bytes);
  l.cw = o;    o = align256(o + tiles * s_bytes);
  l.nz = o;    o = align256(o + static_cast<size_t>(batch * p.words) * 4);
  l.cnt_per_row = tree_nodes(p.tiles);
  l.cnt = o;   o = align256(o + static_cast<size_t>(batch * l.cnt_per_row) * 4);
  l.total = o;
  return l;
}

bool dtype_ok(int d) { return d == TISO_F16 || d == TISO_BF16 || d == TISO_F32 || d == TISO_F64; }

size_t sum_bytes(int dtype, unsigned flags) {
  return (dtype == TISO_F64 || (flags & TISO_EXACT)) ? 8 : 4;
}

template <typename In, typename S, bool kW, bool kInc, int N, int THREADS>
int launch_short(FitArgs a, cudaStream_t st) {
  const size_t smem = ShortLayout<S, kW, N, THREADS>::kBytes;
  auto* k = short_rows_kernel<In, S, kW, kInc, N, THREADS>;
  cudaError_t e = allow_smem(k, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(short)");
  const int64_t grid = (a.batch + THREADS - 1) / THREADS;
  k<<<static_cast<unsigned>(grid), THREADS, smem, st>>>(a);
  e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cuda_fail(e, "short_rows_kernel launch");
}

// Persistent CTAs of short_rows_u_kernel: as many as fit the GPU at once (at most one group of
// 32 rows per warp). The count per SM is looked up once per (kernel, device).
std::mutex g_occ_mu;
std::map<std::pair<const void*, int>, int> g_occ;

template <typename F>
cudaError_t resident_ctas(F* kernel, int threads, size_t smem, int* ctas) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  std::lock_guard<std::mutex> lock(g_occ_mu);
  auto it = g_occ.find(key);
  if (it == g_occ.end()) {
    int per_sm = 0, sms = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    it = g_occ.emplace(key, (per_sm > 0 ? per_sm : 1) * (sms > 0 ? sms : 1)).first;
  }
  *ctas = it->second;
  return cudaSuccess;
}

template <typename In, typename S, bool kInc, int N>
int launch_short_u(FitArgs a, cudaStream_t st) {
  const size_t smem = ShortULayout<S, N>::kBytes;
  const bool plain = !a.clip_lo && !a.clip_hi && !a.starts;
  auto* k = a.n == N ? (plain ? short_rows_u_kernel<In, S, kInc, N, true, true>
                              : short_rows_u_kernel<In, S, kInc, N, true, false>)
                     : short_rows_u_kernel<In, S, kInc, N, false>;
  cudaError_t e = allow_smem(k, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(short_u)");
  int ctas = 0;
  e = resident_ctas(k, 32 * kShortUWarps, smem, &ctas);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  const int64_t groups = (a.batch + 31) / 32;
  const int64_t need = (groups + kShortUWarps - 1) / kShortUWarps;
  const int64_t grid = need < ctas ? need : ctas;
  k<<<static_cast<unsigned>(grid), 32 * kShortUWarps, smem, st>>>(a);
  e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cuda_fail(e, "short_rows_u_kernel launch");
}

template <typename In, typename S, bool kW, int N, int THREADS>
int launch_short_dir(FitArgs a, cudaStream_t st) {
  if constexpr (!kW && !std::is_same_v<In, double>) {  // unweighted float32/16/bf16 rows
    return a.increasing ? launch_short_u<In, S, true, N>(a, st)
                        : launch_short_u<In, S, false, N>(a, st);
  }
  return a.increasing ? launch_short<In, S, kW, true, N, THREADS>(a, st)
                      : launch_short<In, S, kW, false, N, THREADS>(a, st);
}

template <typename In, typename S, bool kW>
int launch_fit(FitArgs a, const FitPlan& p, cudaStream_t st) {
  if (a.n <= 16) return launch_short_dir<In, S, kW, 16, 128>(a, st);
  if (a.n <= 32) return launch_short_dir<In, S, kW, 32, 128>(a, st);
  cudaError_t e;
  if (p.whole) {
    using Sm = TileSmem<S, kW, kK, kThreads>;
    auto* tk = fit_tile_kernel<In, S, kW, kK, kThreads>;
    e = allow_smem(tk, sizeof(Sm));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tile)");
    tk<<<static_cast<unsigned>(p.grid), kThreads, sizeof(Sm), st>>>(a);
    e = cudaGetLastError();
    return e == cudaSuccess ? TISO_OK : cuda_fail(e, "fit_tile_kernel launch");
  }
  if (p.threads == kLongThreads) {
    using Sm = TileSmem<S, kW, kK, kLongThreads>;
    auto* tk = fit_tile_kernel<In, S, kW, kK, kLongThreads>;
    e = allow_smem(tk, sizeof(Sm));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tile)");
    tk<<<static_cast<unsigned>(p.grid), kLongThreads, sizeof(Sm), st>>>(a);
  } else {
    using Sm = TileSmem<S, kW, kK, kThreads>;
    auto* tk = fit_tile_kernel<In, S, kW, kK, kThreads>;
    e = allow_smem(tk, sizeof(Sm));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tile)");
    tk<<<static_cast<unsigned>(p.grid), kThreads, sizeof(Sm), st>>>(a);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fit_tile_kernel launch");
  if (p.tiles > 1) {
    if (p.climb) {
      const int64_t pairs = (p.tiles + 1) / 2;
      const int64_t blocks = (a.batch * pairs + 127) / 128;
      climb_kernel<S><<<static_cast<unsigned>(blocks), 128, 0, st>>>(a, pairs);
    } else {
      const int64_t blocks = (a.batch + 3) / 4;  // a warp per row
      merge_rows_kernel<S><<<static_cast<unsigned>(blocks), 128, 0, st>>>(a);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "tile merge kernel launch");
  }
  if (p.threads == kLongThreads) {
    auto* ek = expand_kernel<In, S, kK, kLongThreads>;
    const size_t esm = sizeof(ExpandSmem<In, S, kK, kLongThreads>);
    e = allow_smem(ek, esm);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(expand)");
    ek<<<static_cast<unsigned>(p.grid), kLongThreads, esm, st>>>(a);
  } else {
    auto* ek = expand_kernel<In, S, kK, kThreads>;
    constexpr int tp = kExpandTilesPerCta<kThreads>;
    const size_t esm = tp * sizeof(ExpandSmem<In, S, kK, kThreads>);
    e = allow_smem(ek, esm);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(expand)");
    ek<<<static_cast<unsigned>((p.grid + tp - 1) / tp), kThreads * tp, esm, st>>>(a);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "expand_kernel launch");
  return TISO_OK;
}

template <typename In>
int dispatch_fit(FitArgs a, const FitPlan& p, bool weighted, bool exact, cudaStream_t st) {
  if constexpr (std::is_same_v<In, double>) {
    return weighted ? launch_fit<In, double, true>(a, p, st) : launch_fit<In, double, false>(a, p, st);
  } else {
    if (exact) {
      return weighted ? launch_fit<In, double, true>(a, p, st)
                      : launch_fit<In, double, false>(a, p, st);
    }
    return weighted ? launch_fit<In, float, true>(a, p, st) : launch_fit<In, float, false>(a, p, st);
  }
}

int check_shape(int dtype, int64_t batch, int64_t n) {
  if (!dtype_ok(dtype)) return fail(TISO_ERR_ARGUMENT, "dtype must be TISO_F16/BF16/F32/F64");
  if (batch < 0 || n < 1) return fail(TISO_ERR_ARGUMENT, "need batch >= 0 and n >= 1");
  if (n >= (int64_t{1} << 31) - 1)
    return fail(TISO_ERR_ARGUMENT, "rows must have fewer than 2^31 - 1 elements");
  if (batch * n >= (int64_t{1} << 62)) return fail(TISO_ERR_ARGUMENT, "batch * n too large");
  return TISO_OK;
}


// ---------------------------------------------------------------------------------------------
// Backward

struct GradPlan {
  bool whole;
  int log2g;
  int64_t tiles;
  int64_t grid;
};

GradPlan plan_grad(int64_t batch, int64_t n) {
  GradPlan p{};
  if (n <= kGTile) {
    p.whole = true;
    const int g = static_cast<int>((n + kGK - 1) / kGK);
    p.log2g = ilog2(g < 1 ? 1 : g);
    const int64_t per_cta = kGThreads >> p.log2g;
    p.tiles = 1;
    p.grid = (batch + per_cta - 1) / per_cta;
  } else {
    p.whole = false;
    p.log2g = ilog2(kGThreads);
    p.tiles = (n + kGTile - 1) / kGTile;
    p.grid = batch * p.tiles;
  }
  return p;
}

constexpr int kRowScanThreads = 256;

// Rows of more tiles than this are scanned in chunks of kRowScanThreads tiles by many CTAs
// (three launches); shorter ones by one CTA each.
constexpr int64_t kRowScanOneCta = 4 * kRowScanThreads;

int64_t grad_chunks(const GradPlan& p) {
  return p.tiles > kRowScanOneCta ? (p.tiles + kRowScanThreads - 1) / kRowScanThreads : 0;
}

struct GradLayout {
  size_t has, sums, carry, c_tot, c_carry, total;
};

GradLayout grad_layout(const GradPlan& p, int64_t batch) {
  GradLayout l{};
  const size_t tiles = static_cast<size_t>(batch * p.tiles);
  const size_t chunks = static_cast<size_t>(batch * grad_chunks(p));
  size_t o = 0;
  l.has = o;     o = align256(o + tiles * 4);
  l.sums = o;    o = align256(o + tiles * 9 * 8);
  l.carry = o;   o = align256(o + tiles * 6 * 8);
  l.c_tot = o;   o = align256(o + chunks * 8 * 8);
  l.c_carry = o; o = align256(o + chunks * 6 * 8);
  l.total = o;
  return l;
}

void set_grad_layout(GradArgs& a, const GradPlan& p, const GradLayout& l, char* ws) {
  a.t_has = reinterpret_cast<int32_t*>(ws + l.has);
  a.t_sums = reinterpret_cast<double*>(ws + l.sums);
  a.t_carry = reinterpret_cast<double*>(ws + l.carry);
  a.c_tot = reinterpret_cast<double*>(ws + l.c_tot);
  a.c_carry = reinterpret_cast<double*>(ws + l.c_carry);
  a.chunks = static_cast<int32_t>(grad_chunks(p));
}

template <typename In, bool kW, bool kY>
int launch_grad(GradArgs a, const GradPlan& p, cudaStream_t st) {
  cudaError_t e;
  if (p.whole && a.n <= kGRowsN && !a.has_y0 && !a.cont && !a.ext) {
    // rows of at most 64 elements: 8 elements a lane, 1, 2, 4 or 8 lanes a row
    const int lanes = a.n <= 8 ? 1 : a.n <= 16 ? 2 : a.n <= 32 ? 4 : 8;
    const unsigned grid = static_cast<unsigned>((a.batch * lanes + 127) / 128);
    switch (lanes) {
      case 1: grad_rows_kernel<In, kW, kY, 1><<<grid, 128, 0, st>>>(a); break;
      case 2: grad_rows_kernel<In, kW, kY, 2><<<grid, 128, 0, st>>>(a); break;
      case 4: grad_rows_kernel<In, kW, kY, 4><<<grid, 128, 0, st>>>(a); break;
      default: grad_rows_kernel<In, kW, kY, 8><<<grid, 128, 0, st>>>(a); break;
    }
    e = cudaGetLastError();
    return e == cudaSuccess ? TISO_OK : cuda_fail(e, "grad_rows_kernel launch");
  }
  if (p.whole) {
    using Sm = GradSmem<double, kGK, kGThreads, true>;
    auto* k = grad_tile_kernel<In, kW, kY>;
    e = allow_smem(k, sizeof(Sm));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(grad)");
    a.mode = 0;
    k<<<static_cast<unsigned>(p.grid), kGThreads, sizeof(Sm), st>>>(a);
    e = cudaGetLastError();
    return e == cudaSuccess ? TISO_OK : cuda_fail(e, "grad_tile_kernel launch");
  }
  if (!a.ext) {  // a segment of a split row ran its first pass already
    a.mode = 1;
    grad_tile_sums_kernel<In, kW, kY><<<static_cast<unsigned>(p.grid), kGThreads, 0, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "grad_tile_sums_kernel launch");
  }
  if (a.chunks > 0) {
    const unsigned chunk_grid = static_cast<unsigned>(a.batch * a.chunks);
    grad_chunk_total_kernel<kRowScanThreads><<<chunk_grid, kRowScanThreads, 0, st>>>(a);
    grad_chunk_carry_kernel<kRowScanThreads><<<static_cast<unsigned>(a.batch), kRowScanThreads, 0,
                                               st>>>(a);
    grad_row_scan_kernel<kRowScanThreads><<<chunk_grid, kRowScanThreads, 0, st>>>(a);
  } else {
    grad_row_scan_kernel<kRowScanThreads><<<static_cast<unsigned>(a.batch), kRowScanThreads, 0,
                                            st>>>(a);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "row scan kernels launch");
  a.mode = 2;
  grad_fill_kernel<In, kW, kY><<<static_cast<unsigned>(p.grid), kFillThreads, 0, st>>>(a);
  e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cuda_fail(e, "grad_fill_kernel launch");
}

template <typename In>
int dispatch_grad(GradArgs a, const GradPlan& p, bool weighted, bool need_y, cudaStream_t st) {
  if (weighted) {
    return need_y ? launch_grad<In, true, true>(a, p, st) : launch_grad<In, true, false>(a, p, st);
  }
  return need_y ? launch_grad<In, false, true>(a, p, st) : launch_grad<In, false, false>(a, p, st);
}

// ---------------------------------------------------------------------------------------------
// Ragged rows (tiso_fit_varlen, tiso_grad_varlen): whole rows of at most kVarMaxLen elements,
// each CTA's rows staged from their own offsets.

constexpr int64_t kVarMaxLen = kTile;  // 512: a row fits one segment of a one-warp CTA

template <typename In, typename S, bool kW>
int launch_fit_var(FitArgs a, cudaStream_t st) {
  using Sm = TileSmem<S, kW, kK, kThreads, true>;
  auto* tk = fit_tile_kernel<In, S, kW, kK, kThreads, true>;
  cudaError_t e = allow_smem(tk, sizeof(Sm));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tile, ragged)");
  const int64_t per_cta = kThreads >> a.log2g;
  const int64_t grid = (a.batch + per_cta - 1) / per_cta;
  tk<<<static_cast<unsigned>(grid), kThreads, sizeof(Sm), st>>>(a);
  e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cuda_fail(e, "fit_tile_kernel(ragged) launch");
}

template <typename In>
int dispatch_fit_var(FitArgs a, bool weighted, bool exact, cudaStream_t st) {
  if constexpr (std::is_same_v<In, double>) {
    return weighted ? launch_fit_var<In, double, true>(a, st) : launch_fit_var<In, double, false>(a, st);
  } else {
    if (exact) {
      return weighted ? launch_fit_var<In, double, true>(a, st)
                      : launch_fit_var<In, double, false>(a, st);
    }
    return weighted ? launch_fit_var<In, float, true>(a, st) : launch_fit_var<In, float, false>(a, st);
  }
}

template <typename In, bool kW, bool kY>
int launch_grad_var(GradArgs a, cudaStream_t st) {
  if (a.n <= kGRowsN) {  // rows of at most 64 elements: 8 elements a lane, 1, 2, 4 or 8 lanes a row
    const int lanes = a.n <= 8 ? 1 : a.n <= 16 ? 2 : a.n <= 32 ? 4 : 8;
    const unsigned grid = static_cast<unsigned>((a.batch * lanes + 127) / 128);
    switch (lanes) {
      case 1: grad_rows_kernel<In, kW, kY, 1, true><<<grid, 128, 0, st>>>(a); break;
      case 2: grad_rows_kernel<In, kW, kY, 2, true><<<grid, 128, 0, st>>>(a); break;
      case 4: grad_rows_kernel<In, kW, kY, 4, true><<<grid, 128, 0, st>>>(a); break;
      default: grad_rows_kernel<In, kW, kY, 8, true><<<grid, 128, 0, st>>>(a); break;
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TISO_OK : cuda_fail(e, "grad_rows_kernel(ragged) launch");
  }
  using Sm = GradSmem<double, kGK, kGThreads, true, true>;
  auto* k = grad_tile_kernel<In, kW, kY, true>;
  cudaError_t e = allow_smem(k, sizeof(Sm));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(grad, ragged)");
  const int64_t per_cta = kGThreads >> a.log2g;
  const int64_t grid = (a.batch + per_cta - 1) / per_cta;
  a.mode = 0;
  k<<<static_cast<unsigned>(grid), kGThreads, sizeof(Sm), st>>>(a);
  e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cuda_fail(e, "grad_tile_kernel(ragged) launch");
}

template <typename In>
int dispatch_grad_var(GradArgs a, bool weighted, bool need_y, cudaStream_t st) {
  if (weighted) {
    return need_y ? launch_grad_var<In, true, true>(a, st) : launch_grad_var<In, true, false>(a, st);
  }
  return need_y ? launch_grad_var<In, false, true>(a, st) : launch_grad_var<In, false, false>(a, st);
}

int check_var(int dtype, int64_t batch, int64_t max_len, const int64_t* offsets) {
  if (!dtype_ok(dtype)) return fail(TISO_ERR_ARGUMENT, "dtype must be TISO_F16/BF16/F32/F64");
  if (batch < 0 || max_len < 0) return fail(TISO_ERR_ARGUMENT, "need batch >= 0 and max_len >= 0");
  if (max_len > kVarMaxLen)
    return fail(TISO_ERR_ARGUMENT,
                "ragged rows of more than 512 elements are not supported: pad them into a "
                "[batch, n] batch for tiso_fit");
  if (batch > 0 && !offsets) return fail(TISO_ERR_ARGUMENT, "offsets must not be NULL");
  return TISO_OK;
}

// ---------------------------------------------------------------------------------------------
// tiso_check_weights: one pass over the weights, a flag set if any is not > 0 (NaN included).

template <typename T>
__global__ void __launch_bounds__(256) check_weights_kernel(const T* __restrict__ w, int64_t n,
                                                            int32_t* flag) {
  constexpr int V = 16 / sizeof(T);
  bool bad = false;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nvec = (reinterpret_cast<uintptr_t>(w) & 15) == 0 ? n / V : 0;
  for (int64_t v = t0; v < nvec; v += stride) {
    const uint4 r = __ldcs(reinterpret_cast<const uint4*>(w) + v);
    const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < V; ++i) bad |= !(e[i] > T(0));
  }
  for (int64_t i = nvec * V + t0; i < n; i += stride) bad |= !(w[i] > T(0));
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(flag, 1);
}

}  // namespace
}  // namespace tiso

using namespace tiso;

extern "C" {

int tiso_abi_version(void) { return TISO_ABI_VERSION; }

const char* tiso_last_error(void) { return g_error.c_str(); }

int tiso_fit_workspace_size(int dtype, int weighted, int64_t batch, int64_t n, unsigned flags,
                            size_t* bytes) {
  (void)weighted;
  if (!bytes) return fail(TISO_ERR_ARGUMENT, "bytes is NULL");
  *bytes = 0;
  const int rc = check_shape(dtype, batch, n);
  if (rc) return rc;
  const FitPlan p = plan_fit(batch, n);
  if (!p.whole && batch > 0) *bytes = fit_layout(p, batch, sum_bytes(dtype, flags)).total;
  return TISO_OK;
}

int tiso_fit(int dtype, const void* y, const void* w, void* out, uint8_t* starts, int64_t batch,
             int64_t n, unsigned flags, double y_min, double y_max, int32_t* bad_weight,
             void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_shape(dtype, batch, n);
  if (rc) return rc;
  if (!y || !out) return fail(TISO_ERR_ARGUMENT, "y and out must not be NULL");
  if (batch == 0) return TISO_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const FitPlan p = plan_fit(batch, n);
  FitArgs a{};
  a.y = y;
  a.w = w;
  a.out = out;
  a.starts = starts;
  a.batch = batch;
  a.n = static_cast<int32_t>(n);
  a.log2g = p.log2g;
  a.seg_len = p.whole ? static_cast<int32_t>(n) : p.tile;
  a.whole = p.whole ? 1 : 0;
  a.tiles = static_cast<int32_t>(p.tiles);
  a.words = static_cast<int32_t>(p.words);
  a.div_n = make_fastdiv(static_cast<uint32_t>(n));
  a.increasing = (flags & TISO_INCREASING) ? 1 : 0;
  a.clip_lo = (flags & TISO_CLIP_LO) ? 1 : 0;
  a.clip_hi = (flags & TISO_CLIP_HI) ? 1 : 0;
  a.lo = y_min;
  a.hi = y_max;
  a.bad_weight = w ? bad_weight : nullptr;
  if (!p.whole) {
    const FitLayout l = fit_layout(p, batch, sum_bytes(dtype, flags));
    if (!workspace || workspace_bytes < l.total)
      return fail(TISO_ERR_WORKSPACE, "workspace smaller than tiso_fit_workspace_size");
    char* ws = static_cast<char*>(workspace);
    if (reinterpret_cast<uintptr_t>(ws) & 255)
      return fail(TISO_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    a.l_start = reinterpret_cast<int32_t*>(ws + l.start);
    a.l_w = ws + l.w;
    a.l_t = ws + l.t;
    a.l_lo = reinterpret_cast<int32_t*>(ws + l.lo);
    a.l_hi = reinterpret_cast<int32_t*>(ws + l.hi);
    a.l_nan = reinterpret_cast<int32_t*>(ws + l.nan);
    a.l_nz = reinterpret_cast<uint32_t*>(ws + l.nz);
    a.l_cnt = reinterpret_cast<int32_t*>(ws + l.cnt);
    a.cnt_per_row = static_cast<int32_t>(l.cnt_per_row);
    if (!p.climb) {  // merge_rows_kernel leaves each tile's carry for the expand
      a.l_ct = ws + l.ct;
      a.l_cw = ws + l.cw;
    }
    // every tile starts with an alive block; no tree node has an arrival yet
    cudaError_t e = cudaMemsetAsync(ws + l.nz, 0xff, l.cnt - l.nz, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ws + l.cnt, 0, l.total - l.cnt, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
  }
  if (a.bad_weight) {
    const cudaError_t e = cudaMemsetAsync(a.bad_weight, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(bad_weight)");
  }
  const bool weighted = w != nullptr;
  const bool exact = (flags & TISO_EXACT) != 0;
  switch (dtype) {
    case TISO_F16: return dispatch_fit<__half>(a, p, weighted, exact, st);
    case TISO_BF16: return dispatch_fit<__nv_bfloat16>(a, p, weighted, exact, st);
    case TISO_F32: return dispatch_fit<float>(a, p, weighted, exact, st);
    default: return dispatch_fit<double>(a, p, weighted, exact, st);
  }
}

int tiso_grad_workspace_size(int dtype, int weighted, int64_t batch, int64_t n, unsigned flags,
                             size_t* bytes) {
  (void)weighted;
  (void)flags;
  if (!bytes) return fail(TISO_ERR_ARGUMENT, "bytes is NULL");
  *bytes = 0;
  const int rc = check_shape(dtype, batch, n);
  if (rc) return rc;
  const GradPlan p = plan_grad(batch, n);
  if (!p.whole && batch > 0) *bytes = grad_layout(p, batch).total;
  return TISO_OK;
}

int tiso_grad(int dtype, const void* y, const void* w, const uint8_t* starts, const void* g,
              void* grad_y, void* grad_w, int64_t batch, int64_t n, unsigned flags, double y_min,
              double y_max, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_shape(dtype, batch, n);
  if (rc) return rc;
  if (!starts || !g) return fail(TISO_ERR_ARGUMENT, "starts and g must not be NULL");
  const bool want_gw = (flags & TISO_WANT_GRAD_W) != 0;
  const bool clip = (flags & (TISO_CLIP_LO | TISO_CLIP_HI)) != 0;
  if (want_gw && (!w || !y || !grad_w))
    return fail(TISO_ERR_ARGUMENT, "the weights' gradient needs w, y and grad_w");
  if (clip && !y) return fail(TISO_ERR_ARGUMENT, "a clipped fit's gradient needs y");
  if (!grad_y && !want_gw) return TISO_OK;
  if (batch == 0) return TISO_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const GradPlan p = plan_grad(batch, n);
  GradArgs a{};
  a.y = y;
  a.w = w;
  a.starts = starts;
  a.g = g;
  a.grad_y = grad_y;
  a.grad_w = want_gw ? grad_w : nullptr;
  a.batch = batch;
  a.n = static_cast<int32_t>(n);
  a.log2g = p.log2g;
  a.seg_len = p.whole ? static_cast<int32_t>(n) : kGTile;
  a.tiles = static_cast<int32_t>(p.tiles);
  a.div_n = make_fastdiv(static_cast<uint32_t>(n));
  a.clip_lo = (flags & TISO_CLIP_LO) ? 1 : 0;
  a.clip_hi = (flags & TISO_CLIP_HI) ? 1 : 0;
  a.lo = y_min;
  a.hi = y_max;
  if (!p.whole) {
    const GradLayout l = grad_layout(p, batch);
    if (!workspace || workspace_bytes < l.total)
      return fail(TISO_ERR_WORKSPACE, "workspace smaller than tiso_grad_workspace_size");
    char* ws = static_cast<char*>(workspace);
    if (reinterpret_cast<uintptr_t>(ws) & 255)
      return fail(TISO_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    set_grad_layout(a, p, l, ws);
  }
  const bool need_y = want_gw || clip;
  const bool weighted = w != nullptr;
  switch (dtype) {
    case TISO_F16: return dispatch_grad<__half>(a, p, weighted, need_y, st);
    case TISO_BF16: return dispatch_grad<__nv_bfloat16>(a, p, weighted, need_y, st);
    case TISO_F32: return dispatch_grad<float>(a, p, weighted, need_y, st);
    default: return dispatch_grad<double>(a, p, weighted, need_y, st);
  }
}


int tiso_fit_varlen(int dtype, const void* y, const void* w, void* out, uint8_t* starts,
                    const int64_t* offsets, int64_t batch, int64_t max_len, unsigned flags,
                    double y_min, double y_max, int32_t* bad_weight, void* stream) {
  int rc = check_var(dtype, batch, max_len, offsets);
  if (rc) return rc;
  if (batch == 0 || max_len == 0) {
    if (bad_weight && w) {
      const cudaError_t e = cudaMemsetAsync(bad_weight, 0, sizeof(int32_t),
                                            static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(bad_weight)");
    }
    return TISO_OK;
  }
  if (!y || !out) return fail(TISO_ERR_ARGUMENT, "y and out must not be NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  FitArgs a{};
  a.y = y;
  a.w = w;
  a.out = out;
  a.starts = starts;
  a.batch = batch;
  a.n = static_cast<int32_t>(max_len);
  const int g = static_cast<int>((max_len + kK - 1) / kK);
  a.log2g = ilog2(g < 1 ? 1 : g);
  a.seg_len = a.n;
  a.whole = 1;
  a.tiles = 1;
  a.div_n = make_fastdiv(static_cast<uint32_t>(max_len));
  a.increasing = (flags & TISO_INCREASING) ? 1 : 0;
  a.clip_lo = (flags & TISO_CLIP_LO) ? 1 : 0;
  a.clip_hi = (flags & TISO_CLIP_HI) ? 1 : 0;
  a.lo = y_min;
  a.hi = y_max;
  a.bad_weight = w ? bad_weight : nullptr;
  a.offsets = offsets;
  if (a.bad_weight) {
    const cudaError_t e = cudaMemsetAsync(a.bad_weight, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(bad_weight)");
  }
  const bool weighted = w != nullptr;
  const bool exact = (flags & TISO_EXACT) != 0;
  switch (dtype) {
    case TISO_F16: return dispatch_fit_var<__half>(a, weighted, exact, st);
    case TISO_BF16: return dispatch_fit_var<__nv_bfloat16>(a, weighted, exact, st);
    case TISO_F32: return dispatch_fit_var<float>(a, weighted, exact, st);
    default: return dispatch_fit_var<double>(a, weighted, exact, st);
  }
}

int tiso_check_weights(int dtype, const void* w, int64_t numel, int32_t* flag, void* stream) {
  if (dtype != TISO_F32 && dtype != TISO_F64)
    return fail(TISO_ERR_ARGUMENT, "weights must be TISO_F32 or TISO_F64");
  if (!flag || numel < 0 || (numel > 0 && !w))
    return fail(TISO_ERR_ARGUMENT, "need a flag, numel >= 0 and the weights");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(flag)");
  if (numel == 0) return TISO_OK;
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  const int64_t per = 256 * 4 * (dtype == TISO_F32 ? 4 : 2);  // a few vectors a thread
  int64_t grid = (numel + per - 1) / per;
  const int64_t most = static_cast<int64_t>(sms > 0 ? sms : 1) * 8;
  grid = grid < most ? grid : most;
  if (dtype == TISO_F32) {
    check_weights_kernel<float><<<static_cast<unsigned>(grid), 256, 0, st>>>(
        static_cast<const float*>(w), numel, flag);
  } else {
    check_weights_kernel<double><<<static_cast<unsigned>(grid), 256, 0, st>>>(
        static_cast<const double*>(w), numel, flag);
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cuda_fail(e, "check_weights_kernel launch");
}

int tiso_grad_varlen(int dtype, const void* y, const void* w, const uint8_t* starts,
                     const void* g, void* grad_y, void* grad_w, const int64_t* offsets,
                     int64_t batch, int64_t max_len, unsigned flags, double y_min, double y_max,
                     void* stream) {
  int rc = check_var(dtype, batch, max_len, offsets);
  if (rc) return rc;
  const bool want_gw = (flags & TISO_WANT_GRAD_W) != 0;
  const bool clip = (flags & (TISO_CLIP_LO | TISO_CLIP_HI)) != 0;
  if (batch == 0 || max_len == 0) return TISO_OK;
  if (!starts || !g) return fail(TISO_ERR_ARGUMENT, "starts and g must not be NULL");
  if (want_gw && (!w || !y || !grad_w))
    return fail(TISO_ERR_ARGUMENT, "the weights' gradient needs w, y and grad_w");
  if (clip && !y) return fail(TISO_ERR_ARGUMENT, "a clipped fit's gradient needs y");
  if (!grad_y && !want_gw) return TISO_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GradArgs a{};
  a.y = y;
  a.w = w;
  a.starts = starts;
  a.g = g;
  a.grad_y = grad_y;
  a.grad_w = want_gw ? grad_w : nullptr;
  a.batch = batch;
  a.n = static_cast<int32_t>(max_len);
  const int gg = static_cast<int>((max_len + kGK - 1) / kGK);
  a.log2g = ilog2(gg < 1 ? 1 : gg);
  a.seg_len = a.n;
  a.tiles = 1;
  a.div_n = make_fastdiv(static_cast<uint32_t>(max_len));
  a.clip_lo = (flags & TISO_CLIP_LO) ? 1 : 0;
  a.clip_hi = (flags & TISO_CLIP_HI) ? 1 : 0;
  a.lo = y_min;
  a.hi = y_max;
  a.offsets = offsets;
  const bool need_y = want_gw || clip;
  const bool weighted = w != nullptr;
  switch (dtype) {
    case TISO_F16: return dispatch_grad_var<__half>(a, weighted, need_y, st);
    case TISO_BF16: return dispatch_grad_var<__nv_bfloat16>(a, weighted, need_y, st);
    case TISO_F32: return dispatch_grad_var<float>(a, weighted, need_y, st);
    default: return dispatch_grad_var<double>(a, weighted, need_y, st);
  }
}
}  // extern "C"

// ---------------------------------------------------------------------------------------------
// tiso_grad_noalloc: the backward with its scratch in a fixed device array instead of a
// caller-provided workspace, for callers that cannot allocate device memory.
//
// The array is a file-scope __device__ variable: every GPU that loads this library holds it
// until the process exits. In host code its name is only a host-side stand-in for the device
// variable, not a device address, so it must never be handed to a kernel as is. Its device
// address is looked up once per device (cudaGetSymbolAddress, with that device current) on the
// first call made on that device, and the pointer is what the kernels get.

namespace tiso {
namespace {

// Long rows of the backward need, per 1024-element tile, one int and 15 doubles of scratch.
constexpr int64_t kNoAllocMaxTiles = 32768;
// 32768 tiles (4 + 9 * 8 + 6 * 8 bytes each), plus room for the chunk arrays of rows scanned in
// chunks (at most 32768 / 256 + 32 chunks of 14 * 8 bytes) and alignment.
constexpr size_t kNoAllocScratchBytes = 32768 * 4 + 32768 * 9 * 8 + 32768 * 6 * 8 + 65536;

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};
void* g_noalloc_ctx[64] = {nullptr};  // the context each address was looked up in

}  // namespace
}  // namespace tiso

static __device__ __align__(256) unsigned char tiso_grad_scratch[tiso::kNoAllocScratchBytes];

namespace tiso {
namespace {

// The calling thread's current CUDA context (the driver's cuCtxGetCurrent, reached through the
// runtime's entry-point query so that the library links only the runtime); NULL if unknown.
void* current_context() {
  using CtxGetCurrent = int (*)(void**);
  static CtxGetCurrent fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      return static_cast<CtxGetCurrent>(nullptr);
    }
    return reinterpret_cast<CtxGetCurrent>(f);
  }();
  void* ctx = nullptr;
  if (!fn || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// The device address of tiso_grad_scratch on the current device, looked up (with that device
// current) on the first call there and again whenever the current context is not the one of
// the last lookup (another context made current on that device).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(TISO_ERR_ARGUMENT, "device index out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  void* ctx = g_noalloc_ptr[dev] ? current_context() : nullptr;
  if (!g_noalloc_ptr[dev] || ctx != g_noalloc_ctx[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, tiso_grad_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(tiso_grad_scratch)");
    g_noalloc_ptr[dev] = ptr;
    g_noalloc_ctx[dev] = current_context();  // after the lookup, which made the context current
  }
  *out = g_noalloc_ptr[dev];
  return TISO_OK;
}

}  // namespace
}  // namespace tiso

extern "C" int tiso_grad_noalloc(int dtype, const void* y, const void* w, const uint8_t* starts,
                                 const void* g, void* grad_y, void* grad_w, int64_t batch,
                                 int64_t n, unsigned flags, double y_min, double y_max,
                                 void* stream) {
  using namespace tiso;
  int rc = check_shape(dtype, batch, n);
  if (rc) return rc;
  if (!starts || !g) return fail(TISO_ERR_ARGUMENT, "starts and g must not be NULL");
  const bool want_gw = (flags & TISO_WANT_GRAD_W) != 0;
  const bool clip = (flags & (TISO_CLIP_LO | TISO_CLIP_HI)) != 0;
  if (want_gw && (!w || !y || !grad_w))
    return fail(TISO_ERR_ARGUMENT, "the weights' gradient needs w, y and grad_w");
  if (clip && !y) return fail(TISO_ERR_ARGUMENT, "a clipped fit's gradient needs y");
  const GradPlan p = plan_grad(batch, n);
  if (!p.whole && batch * p.tiles > kNoAllocMaxTiles) {
    return fail(TISO_ERR_WORKSPACE,
                "tiso_grad_noalloc: rows longer than 1024 elements need batch * ceil(n / 1024) "
                "<= 32768 (its fixed scratch); use tiso_grad with a workspace instead");
  }
  if (!grad_y && !want_gw) return TISO_OK;
  if (batch == 0) return TISO_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GradArgs a{};
  a.y = y;
  a.w = w;
  a.starts = starts;
  a.g = g;
  a.grad_y = grad_y;
  a.grad_w = want_gw ? grad_w : nullptr;
  a.batch = batch;
  a.n = static_cast<int32_t>(n);
  a.log2g = p.log2g;
  a.seg_len = p.whole ? static_cast<int32_t>(n) : kGTile;
  a.tiles = static_cast<int32_t>(p.tiles);
  a.div_n = make_fastdiv(static_cast<uint32_t>(n));
  a.clip_lo = (flags & TISO_CLIP_LO) ? 1 : 0;
  a.clip_hi = (flags & TISO_CLIP_HI) ? 1 : 0;
  a.lo = y_min;
  a.hi = y_max;
  if (!p.whole) {
    // Every scratch slot a call reads is written earlier in the same call (per-tile sums by the
    // first pass, carries by the row scan), so nothing needs clearing between calls.
    void* base = nullptr;
    rc = noalloc_scratch(&base);
    if (rc) return rc;
    char* ws = static_cast<char*>(base);
    const GradLayout l = grad_layout(p, batch);
    if (l.total > kNoAllocScratchBytes) {
      return fail(TISO_ERR_WORKSPACE, "tiso_grad_noalloc: the problem exceeds its fixed scratch");
    }
    set_grad_layout(a, p, l, ws);
  }
  const bool need_y = want_gw || clip;
  const bool weighted = w != nullptr;
  switch (dtype) {
    case TISO_F16: return dispatch_grad<__half>(a, p, weighted, need_y, st);
    case TISO_BF16: return dispatch_grad<__nv_bfloat16>(a, p, weighted, need_y, st);
    case TISO_F32: return dispatch_grad<float>(a, p, weighted, need_y, st);
    default: return dispatch_grad<double>(a, p, weighted, need_y, st);
  }
}

// ---------------------------------------------------------------------------------------------
// One long row split into segments across devices (include/tiso.h: tiso_segment_*).

namespace tiso {
namespace {

FitPlan plan_segment(int64_t seg_n) {
  FitPlan p{};
  p.whole = false;
  p.climb = true;
  p.threads = kThreads;
  p.tile = kTile;
  p.log2g = ilog2(kThreads);
  p.tiles = (seg_n + kTile - 1) / kTile;
  p.words = (p.tiles + 31) / 32;
  p.grid = p.tiles;
  return p;
}

constexpr int kSegScanThreads = 1024;

struct SegLayout {
  FitLayout fit;
  size_t counts, offs, chunk, total;
};

SegLayout seg_layout(int64_t seg_n) {
  SegLayout l{};
  const FitPlan p = plan_segment(seg_n);
  l.fit = fit_layout(p, 1, 8);
  const size_t chunks = static_cast<size_t>((p.tiles + kSegScanThreads - 1) / kSegScanThreads);
  size_t o = l.fit.total;
  l.counts = o; o = align256(o + static_cast<size_t>(p.tiles) * 4);
  l.offs = o;   o = align256(o + static_cast<size_t>(p.tiles + 1) * 8);
  l.chunk = o;  o = align256(o + chunks * 8);
  l.total = o;
  return l;
}

constexpr int kMaxParts = 32;

template <typename In, bool kW>
int launch_segment_tiles(FitArgs a, const FitPlan& p, cudaStream_t st) {
  using Sm = TileSmem<double, kW, kK, kThreads>;
  auto* tk = fit_tile_kernel<In, double, kW, kK, kThreads>;
  cudaError_t e = allow_smem(tk, sizeof(Sm));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tile)");
  tk<<<static_cast<unsigned>(p.grid), kThreads, sizeof(Sm), st>>>(a);
  if (p.tiles > 1) {
    const int64_t pairs = (p.tiles + 1) / 2;
    climb_kernel<double><<<static_cast<unsigned>((pairs + 127) / 128), 128, 0, st>>>(a, pairs);
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cuda_fail(e, "segment tile kernels launch");
}

}  // namespace
}  // namespace tiso

extern "C" {

int tiso_segment_blocks_workspace_size(int dtype, int weighted, int64_t seg_n, unsigned flags,
                                       size_t* bytes) {
  (void)weighted;
  (void)flags;
  if (!bytes) return fail(TISO_ERR_ARGUMENT, "bytes is NULL");
  *bytes = 0;
  const int rc = check_shape(dtype, 1, seg_n);
  if (rc) return rc;
  *bytes = seg_layout(seg_n).total;
  return TISO_OK;
}

int tiso_segment_tile_count(int64_t seg_n, int64_t* tiles) {
  if (!tiles) return fail(TISO_ERR_ARGUMENT, "tiles is NULL");
  if (seg_n < 0) return fail(TISO_ERR_ARGUMENT, "seg_n must be >= 0");
  *tiles = (seg_n + kTile - 1) / kTile;
  return TISO_OK;
}

int tiso_segment_blocks(int dtype, const void* y, const void* w, int64_t seg_n, int64_t seg_start,
                        unsigned flags, double y0, int64_t* blk_start, double* blk_t,
                        double* blk_w, int32_t* count, int32_t* nan_flag, int32_t* bad_weight,
                        int64_t* tile_offs, void* workspace, size_t workspace_bytes,
                        void* stream) {
  int rc = check_shape(dtype, 1, seg_n);
  if (rc) return rc;
  if (!y || !blk_start || !blk_t || !blk_w || !count || !nan_flag)
    return fail(TISO_ERR_ARGUMENT, "y, the block arrays, count and nan_flag must not be NULL");
  if (!(flags & TISO_EXACT) && dtype != TISO_F64)
    return fail(TISO_ERR_ARGUMENT, "segments of a split row are fitted with exact=True only");
  if (seg_start < 0) return fail(TISO_ERR_ARGUMENT, "seg_start must be >= 0");
  const SegLayout l = seg_layout(seg_n);
  if (!workspace || workspace_bytes < l.total)
    return fail(TISO_ERR_WORKSPACE, "workspace smaller than tiso_segment_blocks_workspace_size");
  char* ws = static_cast<char*>(workspace);
  if (reinterpret_cast<uintptr_t>(ws) & 255)
    return fail(TISO_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const FitPlan p = plan_segment(seg_n);
  FitArgs a{};
  a.y = y;
  a.w = w;
  a.batch = 1;
  a.n = static_cast<int32_t>(seg_n);
  a.log2g = p.log2g;
  a.seg_len = kTile;
  a.tiles = static_cast<int32_t>(p.tiles);
  a.words = static_cast<int32_t>(p.words);
  a.div_n = make_fastdiv(static_cast<uint32_t>(seg_n));
  a.increasing = (flags & TISO_INCREASING) ? 1 : 0;
  a.bad_weight = w ? bad_weight : nullptr;
  a.l_start = reinterpret_cast<int32_t*>(ws + l.fit.start);
  a.l_w = ws + l.fit.w;
  a.l_t = ws + l.fit.t;
  a.l_lo = reinterpret_cast<int32_t*>(ws + l.fit.lo);
  a.l_hi = reinterpret_cast<int32_t*>(ws + l.fit.hi);
  a.l_nan = reinterpret_cast<int32_t*>(ws + l.fit.nan);
  a.l_nz = reinterpret_cast<uint32_t*>(ws + l.fit.nz);
  a.l_cnt = reinterpret_cast<int32_t*>(ws + l.fit.cnt);
  a.cnt_per_row = static_cast<int32_t>(l.fit.cnt_per_row);
  a.has_y0 = 1;
  a.y0 = y0;
  cudaError_t e = cudaMemsetAsync(ws + l.fit.nz, 0xff, l.fit.cnt - l.fit.nz, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(ws + l.fit.cnt, 0, l.fit.total - l.fit.cnt, st);
  if (e == cudaSuccess && a.bad_weight) e = cudaMemsetAsync(a.bad_weight, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
  const bool weighted = w != nullptr;
  switch (dtype) {
    case TISO_F16: rc = weighted ? launch_segment_tiles<__half, true>(a, p, st) : launch_segment_tiles<__half, false>(a, p, st); break;
    case TISO_BF16: rc = weighted ? launch_segment_tiles<__nv_bfloat16, true>(a, p, st) : launch_segment_tiles<__nv_bfloat16, false>(a, p, st); break;
    case TISO_F32: rc = weighted ? launch_segment_tiles<float, true>(a, p, st) : launch_segment_tiles<float, false>(a, p, st); break;
    default: rc = weighted ? launch_segment_tiles<double, true>(a, p, st) : launch_segment_tiles<double, false>(a, p, st); break;
  }
  if (rc) return rc;
  int32_t* counts = reinterpret_cast<int32_t*>(ws + l.counts);
  // each tile's first block in the compacted list (the caller's array when it wants them)
  int64_t* offs = tile_offs ? tile_offs : reinterpret_cast<int64_t*>(ws + l.offs);
  seg_count_kernel<<<static_cast<unsigned>((p.tiles + 255) / 256), 256, 0, st>>>(a, counts);
  const int m = static_cast<int>(p.tiles);
  const int chunks = (m + kSegScanThreads - 1) / kSegScanThreads;
  int64_t* chunk = reinterpret_cast<int64_t*>(ws + l.chunk);
  seg_chunk_total_kernel<kSegScanThreads><<<chunks, kSegScanThreads, 0, st>>>(counts, chunk, m);
  seg_chunk_scan_kernel<kSegScanThreads><<<1, kSegScanThreads, 0, st>>>(chunk, chunks, offs, m);
  seg_chunk_fill_kernel<kSegScanThreads><<<chunks, kSegScanThreads, 0, st>>>(counts, chunk, offs, m);
  seg_gather_kernel<double><<<static_cast<unsigned>(p.tiles), 128, 0, st>>>(
      a, offs, seg_start, blk_start, blk_t, blk_w, count, nan_flag);
  e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cuda_fail(e, "segment list kernels launch");
}

int tiso_segment_expand_workspace_size(int parts, size_t* bytes) {
  if (!bytes) return fail(TISO_ERR_ARGUMENT, "bytes is NULL");
  if (parts < 1 || parts > kMaxParts) return fail(TISO_ERR_ARGUMENT, "parts must be 1..32");
  *bytes = 4 * 256;
  return TISO_OK;
}

int tiso_segment_expand(int dtype, int parts, int me, int64_t cap, int64_t* blk_start,
                        double* blk_t, double* blk_w, const int32_t* counts, const int32_t* nans,
                        int64_t seg_n, int64_t seg_start, unsigned flags, double y0, double y_min,
                        double y_max, void* out, uint8_t* starts, const int64_t* tile_offs,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!dtype_ok(dtype)) return fail(TISO_ERR_ARGUMENT, "dtype must be TISO_F16/BF16/F32/F64");
  if (parts < 1 || parts > kMaxParts || me < 0 || me >= parts)
    return fail(TISO_ERR_ARGUMENT, "need 1 <= parts <= 32 and 0 <= me < parts");
  if (cap < 1 || cap >= (int64_t{1} << 31)) return fail(TISO_ERR_ARGUMENT, "bad list capacity");
  if (seg_n < 0 || !out || !blk_start || !blk_t || !blk_w || !counts || !nans)
    return fail(TISO_ERR_ARGUMENT, "bad segment arguments");
  if (!workspace || workspace_bytes < 4 * 256)
    return fail(TISO_ERR_WORKSPACE, "workspace smaller than tiso_segment_expand_workspace_size");
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  FitArgs a{};
  a.out = out;
  a.starts = starts;
  a.batch = 1;
  a.tiles = parts;
  a.seg_len = static_cast<int32_t>(cap);
  a.words = 1;
  a.increasing = (flags & TISO_INCREASING) ? 1 : 0;
  a.clip_lo = (flags & TISO_CLIP_LO) ? 1 : 0;
  a.clip_hi = (flags & TISO_CLIP_HI) ? 1 : 0;
  a.lo = y_min;
  a.hi = y_max;
  a.has_y0 = 1;
  a.y0 = y0;
  a.l_w = blk_w;
  a.l_t = blk_t;
  a.l_lo = reinterpret_cast<int32_t*>(ws);
  a.l_hi = reinterpret_cast<int32_t*>(ws + 256);
  a.l_nan = reinterpret_cast<int32_t*>(ws + 512);
  a.l_nz = reinterpret_cast<uint32_t*>(ws + 768);
  seg_init_kernel<<<1, 32, 0, st>>>(parts, counts, nans, a.l_lo, a.l_hi, a.l_nan, a.l_nz);
  // the lists as one row of `parts` tiles: the tree of merges taken by a warp, level by level
  merge_rows_kernel<double><<<1, 32, 0, st>>>(a);
  if (seg_n > 0 && tile_offs) {  // a CTA per tile, its blocks found from the tile offsets
    const unsigned blocks = static_cast<unsigned>((seg_n + kTile - 1) / kTile);
    switch (dtype) {
      case TISO_F16: seg_expand_tiles_kernel<__half><<<blocks, 128, 0, st>>>(a, me, blk_start, tile_offs, seg_n, seg_start); break;
      case TISO_BF16: seg_expand_tiles_kernel<__nv_bfloat16><<<blocks, 128, 0, st>>>(a, me, blk_start, tile_offs, seg_n, seg_start); break;
      case TISO_F32: seg_expand_tiles_kernel<float><<<blocks, 128, 0, st>>>(a, me, blk_start, tile_offs, seg_n, seg_start); break;
      default: seg_expand_tiles_kernel<double><<<blocks, 128, 0, st>>>(a, me, blk_start, tile_offs, seg_n, seg_start); break;
    }
  } else if (seg_n > 0) {
    const int64_t threads = (seg_n + 15) / 16;
    const unsigned blocks = static_cast<unsigned>((threads + 127) / 128);
    switch (dtype) {
      case TISO_F16: seg_expand_kernel<__half><<<blocks, 128, 0, st>>>(a, me, blk_start, seg_n, seg_start); break;
      case TISO_BF16: seg_expand_kernel<__nv_bfloat16><<<blocks, 128, 0, st>>>(a, me, blk_start, seg_n, seg_start); break;
      case TISO_F32: seg_expand_kernel<float><<<blocks, 128, 0, st>>>(a, me, blk_start, seg_n, seg_start); break;
      default: seg_expand_kernel<double><<<blocks, 128, 0, st>>>(a, me, blk_start, seg_n, seg_start); break;
    }
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cuda_fail(e, "segment expand kernels launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// The backward of one long row split into segments across devices (include/tiso.h:
// tiso_segment_grad_*). The segment is fitted as a row of its own in 1024-element tiles; its
// first element continues the block from the segment before unless starts marks it, and the
// open sums flowing in from the other segments come from their gathered runs.

namespace tiso {
namespace {

GradPlan plan_segment_grad(int64_t seg_n) {
  GradPlan p{};
  p.whole = false;
  p.log2g = ilog2(kGThreads);
  p.tiles = (seg_n + kGTile - 1) / kGTile;
  p.grid = p.tiles;
  return p;
}

struct SegGradLayout {
  GradLayout g;
  size_t ext, total;
};

SegGradLayout seg_grad_layout(int64_t seg_n) {
  SegGradLayout l{};
  l.g = grad_layout(plan_segment_grad(seg_n), 1);
  l.ext = l.g.total;
  l.total = align256(l.ext + 6 * 8);
  return l;
}

int seg_grad_args(GradArgs& a, int dtype, const void* y, const void* w, const uint8_t* starts,
                  const void* g, int64_t seg_n, int64_t seg_start, unsigned flags, double y0,
                  void* workspace, size_t workspace_bytes, GradPlan& p, SegGradLayout& l) {
  int rc = check_shape(dtype, 1, seg_n);
  if (rc) return rc;
  if (!starts || !g) return fail(TISO_ERR_ARGUMENT, "starts and g must not be NULL");
  if (seg_start < 0) return fail(TISO_ERR_ARGUMENT, "seg_start must be >= 0");
  const bool want_gw = (flags & TISO_WANT_GRAD_W) != 0;
  const bool clip = (flags & (TISO_CLIP_LO | TISO_CLIP_HI)) != 0;
  if (want_gw && (!w || !y)) return fail(TISO_ERR_ARGUMENT, "the weights' gradient needs w and y");
  if (clip && !y) return fail(TISO_ERR_ARGUMENT, "a clipped fit's gradient needs y");
  p = plan_segment_grad(seg_n);
  l = seg_grad_layout(seg_n);
  if (!workspace || workspace_bytes < l.total)
    return fail(TISO_ERR_WORKSPACE, "workspace smaller than tiso_segment_grad_workspace_size");
  char* ws = static_cast<char*>(workspace);
  if (reinterpret_cast<uintptr_t>(ws) & 255)
    return fail(TISO_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  a = GradArgs{};
  a.y = y;
  a.w = w;
  a.starts = starts;
  a.g = g;
  a.batch = 1;
  a.n = static_cast<int32_t>(seg_n);
  a.log2g = p.log2g;
  a.seg_len = kGTile;
  a.tiles = static_cast<int32_t>(p.tiles);
  a.div_n = make_fastdiv(static_cast<uint32_t>(seg_n));
  a.cont = seg_start > 0 ? 1 : 0;
  a.has_y0 = 1;
  a.y0 = y0;
  set_grad_layout(a, p, l.g, ws);
  return TISO_OK;
}

}  // namespace
}  // namespace tiso

extern "C" {

int tiso_segment_grad_workspace_size(int dtype, int weighted, int64_t seg_n, unsigned flags,
                                     size_t* bytes) {
  (void)weighted;
  (void)flags;
  if (!bytes) return fail(TISO_ERR_ARGUMENT, "bytes is NULL");
  *bytes = 0;
  const int rc = check_shape(dtype, 1, seg_n);
  if (rc) return rc;
  *bytes = seg_grad_layout(seg_n).total;
  return TISO_OK;
}

int tiso_segment_grad_sums(int dtype, const void* y, const void* w, const uint8_t* starts,
                           const void* g, int64_t seg_n, int64_t seg_start, unsigned flags,
                           double y0, double* run, void* workspace, size_t workspace_bytes,
                           void* stream) {
  GradArgs a;
  GradPlan p;
  SegGradLayout l;
  int rc = seg_grad_args(a, dtype, y, w, starts, g, seg_n, seg_start, flags, y0, workspace,
                         workspace_bytes, p, l);
  if (rc) return rc;
  if (!run) return fail(TISO_ERR_ARGUMENT, "run must not be NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool weighted = w != nullptr;
  const bool need_y = (flags & (TISO_WANT_GRAD_W | TISO_CLIP_LO | TISO_CLIP_HI)) != 0;
  a.mode = 1;
  const unsigned grid = static_cast<unsigned>(p.grid);
  auto go = [&](auto in_tag) {
    using In = decltype(in_tag);
    if (weighted) {
      if (need_y) grad_tile_sums_kernel<In, true, true><<<grid, kGThreads, 0, st>>>(a);
      else grad_tile_sums_kernel<In, true, false><<<grid, kGThreads, 0, st>>>(a);
    } else {
      if (need_y) grad_tile_sums_kernel<In, false, true><<<grid, kGThreads, 0, st>>>(a);
      else grad_tile_sums_kernel<In, false, false><<<grid, kGThreads, 0, st>>>(a);
    }
  };
  switch (dtype) {
    case TISO_F16: go(__half{}); break;
    case TISO_BF16: go(__nv_bfloat16{}); break;
    case TISO_F32: go(float{}); break;
    default: go(double{}); break;
  }
  grad_join_tiles_kernel<kRowScanThreads><<<1, kRowScanThreads, 0, st>>>(a, run);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cuda_fail(e, "segment backward first pass launch");
}

int tiso_segment_grad(int dtype, int parts, int me, const double* runs, const void* y,
                      const void* w, const uint8_t* starts, const void* g, void* grad_y,
                      void* grad_w, int64_t seg_n, int64_t seg_start, unsigned flags, double y0,
                      double y_min, double y_max, void* workspace, size_t workspace_bytes,
                      void* stream) {
  GradArgs a;
  GradPlan p;
  SegGradLayout l;
  int rc = seg_grad_args(a, dtype, y, w, starts, g, seg_n, seg_start, flags, y0, workspace,
                         workspace_bytes, p, l);
  if (rc) return rc;
  if (parts < 1 || me < 0 || me >= parts || !runs)
    return fail(TISO_ERR_ARGUMENT, "need runs and 0 <= me < parts");
  const bool want_gw = (flags & TISO_WANT_GRAD_W) != 0;
  if (want_gw && !grad_w) return fail(TISO_ERR_ARGUMENT, "the weights' gradient needs grad_w");
  if (!grad_y && !want_gw) return TISO_OK;
  a.grad_y = grad_y;
  a.grad_w = want_gw ? grad_w : nullptr;
  a.clip_lo = (flags & TISO_CLIP_LO) ? 1 : 0;
  a.clip_hi = (flags & TISO_CLIP_HI) ? 1 : 0;
  a.lo = y_min;
  a.hi = y_max;
  double* ext = reinterpret_cast<double*>(static_cast<char*>(workspace) + l.ext);
  a.ext = ext;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  seg_grad_carry_kernel<<<1, 1, 0, st>>>(parts, me, runs, ext);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "seg_grad_carry_kernel launch");
  const bool need_y = want_gw || a.clip_lo || a.clip_hi;
  const bool weighted = w != nullptr;
  switch (dtype) {
    case TISO_F16: return dispatch_grad<__half>(a, p, weighted, need_y, st);
    case TISO_BF16: return dispatch_grad<__nv_bfloat16>(a, p, weighted, need_y, st);
    case TISO_F32: return dispatch_grad<float>(a, p, weighted, need_y, st);
    default: return dispatch_grad<double>(a, p, weighted, need_y, st);
  }
}

}  // extern "C"
