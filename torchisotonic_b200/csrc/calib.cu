// Calibration around the fit (include/tiso.h: tiso_calib_*): the pre-step that turns raw
// (score, label) pairs into the weighted row the fit takes, and the interpolation of new scores
// on the fitted curve. The reference gives both as plain torch code next to its fit
// (README.md:43-56, examples/ctr_calibration/calibrate.py:163-186): sort, unique_consecutive,
// index_add_, sums / counts, then isotonic(means, counts); searchsorted and a lerp.
//
// tiso_calib_groups is one radix sort of the pairs (CUB's, keys and labels together: no index
// array, no gather; skipped for pairs that come sorted) and three passes of our own over the
// sorted pairs, in tiles of kTile:
//   1. group_tile_kernel: per tile, how many groups (runs of equal scores) start in it and the
//      sum and count of the labels after its last start (its whole content if none starts);
//   2. group_scan_kernel (a CTA per 4096 tiles) and group_chunk_kernel (one CTA over the
//      chunks): the exclusive scan of those over the tiles - each tile's first group index and
//      the partial group that reaches into it from the left;
//   3. group_write_kernel: per tile, every group that ends in it gets its mean label and count
//      (the partial sum from the left added to the first), every group that starts in it its
//      score. Sums are double, in a fixed order: the result does not depend on the launch.
// The passes read 2 (key + label) elements per pair and write three arrays per group: the
// minimum traffic of the pre-step after the sort, where unique_consecutive and index_add_
// take several passes and atomics.
#include <cuda_runtime.h>

#include <cub/device/device_radix_sort.cuh>
#include <string>

#include "../../include/tiso.h"

namespace tiso {

int report_error(int code, const std::string& msg);

namespace {

constexpr int kCalThreads = 256;
constexpr int kCalItems = 8;
constexpr int kTile = kCalThreads * kCalItems;  // pairs per tile
constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;
constexpr int kChunk = kScanThreads * kScanItems;  // tiles per scan CTA

int cal_fail(cudaError_t e, const char* what) {
  return report_error(TISO_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

size_t align256(size_t x) { return (x + 255) & ~size_t{255}; }

// A run of pairs seen as part of the segmented sum over groups: how many groups start in it,
// and the sum and count of the labels after the last start (of all of it when none starts).
// combine(a, b) is the run a followed by b: associative, not commutative.
template <typename C>
struct Run {
  C heads;
  double s;
  C c;
};

template <typename C>
__device__ __forceinline__ Run<C> combine(const Run<C>& a, const Run<C>& b) {
  Run<C> r;
  r.heads = a.heads + b.heads;
  r.s = b.heads ? b.s : a.s + b.s;
  r.c = b.heads ? b.c : a.c + b.c;
  return r;
}

template <typename C>
__device__ __forceinline__ Run<C> shfl_up_run(const Run<C>& v, int d) {
  Run<C> r;
  r.heads = __shfl_up_sync(0xffffffffu, v.heads, d);
  r.s = __shfl_up_sync(0xffffffffu, v.s, d);
  r.c = __shfl_up_sync(0xffffffffu, v.c, d);
  return r;
}

// Exclusive scan of one Run per thread over the CTA (THREADS threads, whole warps), in thread
// order; also returns the CTA's total. warp_runs: THREADS / 32 entries of shared memory.
template <typename C, int THREADS>
__device__ Run<C> block_exclusive(Run<C> v, Run<C>* warp_runs, Run<C>& total) {
  constexpr int kWarps = THREADS / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  Run<C> inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const Run<C> o = shfl_up_run(inc, d);
    if (lane >= d) inc = combine(o, inc);
  }
  if (lane == 31) warp_runs[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    Run<C> x = lane < kWarps ? warp_runs[lane] : Run<C>{0, 0.0, 0};
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const Run<C> o = shfl_up_run(x, d);
      if (lane >= d) x = combine(o, x);
    }
    if (lane < kWarps) warp_runs[lane] = x;  // inclusive over warps
  }
  __syncthreads();
  total = warp_runs[kWarps - 1];
  Run<C> ex = shfl_up_run(inc, 1);
  if (lane == 0) ex = Run<C>{0, 0.0, 0};
  if (warp > 0) ex = lane == 0 ? warp_runs[warp - 1] : combine(warp_runs[warp - 1], ex);
  __syncthreads();  // warp_runs may be reused
  return ex;
}

// A thread's kCalItems consecutive pairs from `first`: 16-byte vector loads when all are in
// range (the tile and thread offsets keep them aligned), else element by element.
template <typename T>
__device__ __forceinline__ void load_items(const T* p, int64_t first, int64_t n,
                                           T (&v)[kCalItems]) {
  static_assert((kCalItems * sizeof(T)) % 16 == 0, "whole 16-byte vectors");
  if (first + kCalItems <= n) {
    const uint4* q = reinterpret_cast<const uint4*>(p + first);
    uint4 raw[kCalItems * sizeof(T) / 16];
#pragma unroll
    for (int k = 0; k < static_cast<int>(kCalItems * sizeof(T) / 16); ++k) raw[k] = __ldg(q + k);
    memcpy(v, raw, sizeof(v));
  } else {
#pragma unroll
    for (int j = 0; j < kCalItems; ++j) v[j] = first + j < n ? p[first + j] : T(0);
  }
}

// The thread's pairs as a Run, and (through `head`) which of them start a group: the first
// pair, and every pair whose score differs from the one before (NaN differs from everything,
// as in unique_consecutive).
template <typename K, typename L>
__device__ __forceinline__ Run<int> thread_run(const K (&k)[kCalItems], const L (&l)[kCalItems],
                                               K before, int64_t first, int64_t n,
                                               uint32_t& head, bool& nan) {
  Run<int> r{0, 0.0, 0};
  head = 0;
  K prev = before;
#pragma unroll
  for (int j = 0; j < kCalItems; ++j) {
    if (first + j < n) {
      const bool h = first + j == 0 || k[j] != prev;
      nan |= k[j] != k[j];
      head |= static_cast<uint32_t>(h) << j;
      r.heads += h;
      r.s = h ? static_cast<double>(l[j]) : r.s + static_cast<double>(l[j]);
      r.c = h ? 1 : r.c + 1;
      prev = k[j];
    }
  }
  return r;
}

template <typename K, typename L>
__global__ void __launch_bounds__(kCalThreads)
    group_tile_kernel(const K* __restrict__ keys, const L* __restrict__ labels, int64_t n,
                      int* __restrict__ t_heads, double* __restrict__ t_s, int* __restrict__ t_c,
                      int64_t* __restrict__ groups) {
  __shared__ Run<int> warp_runs[kCalThreads / 32];
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kTile +
                        static_cast<int64_t>(threadIdx.x) * kCalItems;
  K k[kCalItems];
  L l[kCalItems];
  load_items(keys, first, n, k);
  load_items(labels, first, n, l);
  const K before = first > 0 && first < n ? keys[first - 1] : K(0);
  uint32_t head;
  bool nan = false;
  const Run<int> r = thread_run(k, l, before, first, n, head, nan);
  if (nan) groups[1] = 1;
  Run<int> total;
  block_exclusive<int, kCalThreads>(r, warp_runs, total);
  if (threadIdx.x == 0) {
    t_heads[blockIdx.x] = total.heads;
    t_s[blockIdx.x] = total.s;
    t_c[blockIdx.x] = total.c;
  }
}

// Per chunk of kChunk tiles (one CTA each): for every tile of the chunk the groups that start
// before it within the chunk and the group reaching into it from the left within the chunk;
// the chunk's total in c_*.
__global__ void __launch_bounds__(kScanThreads)
    group_scan_kernel(int64_t tiles, const int* __restrict__ t_heads,
                      const double* __restrict__ t_s, const int* __restrict__ t_c,
                      int64_t* __restrict__ t_goff, double* __restrict__ t_cs,
                      int64_t* __restrict__ t_cc, int64_t* __restrict__ c_heads,
                      double* __restrict__ c_s, int64_t* __restrict__ c_c) {
  __shared__ Run<int64_t> warp_runs[kScanThreads / 32];
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kChunk +
                     static_cast<int64_t>(threadIdx.x) * kScanItems;
  auto item = [&](int j) {
    return t0 + j < tiles ? Run<int64_t>{t_heads[t0 + j], t_s[t0 + j], t_c[t0 + j]}
                          : Run<int64_t>{0, 0.0, 0};
  };
  Run<int64_t> mine{0, 0.0, 0};
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) mine = combine(mine, item(j));
  Run<int64_t> total;
  Run<int64_t> ex = block_exclusive<int64_t, kScanThreads>(mine, warp_runs, total);
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) {  // the items again (cached): fewer registers
    if (t0 + j < tiles) {
      t_goff[t0 + j] = ex.heads;
      t_cs[t0 + j] = ex.s;
      t_cc[t0 + j] = ex.c;
    }
    ex = combine(ex, item(j));
  }
  if (threadIdx.x == 0) {
    c_heads[blockIdx.x] = total.heads;
    c_s[blockIdx.x] = total.s;
    c_c[blockIdx.x] = total.c;
  }
}

// One CTA: the exclusive scan of the chunks' totals, in place; the number of groups.
__global__ void __launch_bounds__(kScanThreads)
    group_chunk_kernel(int64_t chunks, int64_t* __restrict__ c_heads, double* __restrict__ c_s,
                       int64_t* __restrict__ c_c, int64_t* __restrict__ groups) {
  __shared__ Run<int64_t> warp_runs[kScanThreads / 32];
  Run<int64_t> carry{0, 0.0, 0};
  for (int64_t base = 0; base < chunks; base += kScanThreads) {
    const int64_t i = base + threadIdx.x;
    const Run<int64_t> v = i < chunks ? Run<int64_t>{c_heads[i], c_s[i], c_c[i]}
                                      : Run<int64_t>{0, 0.0, 0};
    Run<int64_t> total;
    const Run<int64_t> ex = combine(carry, block_exclusive<int64_t, kScanThreads>(v, warp_runs,
                                                                                 total));
    if (i < chunks) {
      c_heads[i] = ex.heads;
      c_s[i] = ex.s;
      c_c[i] = ex.c;
    }
    carry = combine(carry, total);
  }
  if (threadIdx.x == 0) groups[0] = carry.heads;
}

// Per tile: the groups ending in it take consecutive output slots, as do the groups starting in
// it, so each thread puts its groups' values in shared memory first and the CTA then writes
// each range with coalesced stores (written straight from the threads, 8 consecutive pairs
// apart, the stores of a warp touched a sector each and the kernel ran at a fifth of the speed).
template <typename K, typename L>
__global__ void __launch_bounds__(kCalThreads)
    group_write_kernel(const K* __restrict__ keys, const L* __restrict__ labels, int64_t n,
                       const int64_t* __restrict__ t_goff, const double* __restrict__ t_cs,
                       const int64_t* __restrict__ t_cc, const int64_t* __restrict__ c_heads,
                       const double* __restrict__ c_s, const int64_t* __restrict__ c_c,
                       K* __restrict__ xs, double* __restrict__ y, double* __restrict__ w) {
  __shared__ Run<int> warp_runs[kCalThreads / 32];
  __shared__ double s_y[kTile + 1];  // slot = group index - (first group index - 1)
  __shared__ uint32_t s_c[kTile + 1];
  __shared__ K s_x[kTile];           // slot = group index - first group index
  __shared__ int s_ends[2];          // the tile's first pair starts a group; its last ends one
  const int64_t tile0 = static_cast<int64_t>(blockIdx.x) * kTile;
  const int64_t first = tile0 + static_cast<int64_t>(threadIdx.x) * kCalItems;
  K k[kCalItems];
  L l[kCalItems];
  load_items(keys, first, n, k);
  load_items(labels, first, n, l);
  const K before = first > 0 && first < n ? keys[first - 1] : K(0);
  const K after = first + kCalItems < n ? keys[first + kCalItems] : K(0);
  uint32_t head;
  bool nan = false;
  const Run<int> r = thread_run(k, l, before, first, n, head, nan);
  Run<int> total;
  const Run<int> ex = block_exclusive<int, kCalThreads>(r, warp_runs, total);
  // everything before the tile: the chunks before its chunk, then the tiles before it in it
  const int64_t ch = blockIdx.x / kChunk;
  const Run<int64_t> before_tile =
      combine(Run<int64_t>{c_heads[ch], c_s[ch], c_c[ch]},
              Run<int64_t>{t_goff[blockIdx.x], t_cs[blockIdx.x], t_cc[blockIdx.x]});
  const int64_t goff = before_tile.heads;
  // the group open before the thread's first pair: its slot and its sum and count so far
  int slot = ex.heads;  // = group index - (goff - 1)
  double sum = ex.heads ? ex.s : before_tile.s + ex.s;
  int64_t c = ex.heads ? static_cast<int64_t>(ex.c) : before_tile.c + ex.c;
#pragma unroll
  for (int j = 0; j < kCalItems; ++j) {
    const int64_t i = first + j;
    if (i < n) {
      const bool h = (head >> j) & 1u;
      slot += h;
      sum = h ? static_cast<double>(l[j]) : sum + static_cast<double>(l[j]);
      c = h ? 1 : c + 1;
      if (h) s_x[slot - 1] = k[j];
      const K next = j + 1 < kCalItems ? k[j + 1 < kCalItems ? j + 1 : j] : after;
      const bool end = i + 1 == n || next != k[j];
      if (end) {
        s_y[slot] = sum / static_cast<double>(c);
        s_c[slot] = static_cast<uint32_t>(c);
      }
      if (i == tile0) s_ends[0] = h;
      if (i + 1 == n || i + 1 == tile0 + kTile) s_ends[1] = end;
    }
  }
  __syncthreads();
  const int heads = total.heads;
  const int lo = s_ends[0], hi = heads + s_ends[1];  // slots of the groups ending here
  for (int e = lo + static_cast<int>(threadIdx.x); e < hi; e += kCalThreads) {
    y[goff - 1 + e] = s_y[e];
    w[goff - 1 + e] = static_cast<double>(s_c[e]);
  }
  for (int e = static_cast<int>(threadIdx.x); e < heads; e += kCalThreads) xs[goff + e] = s_x[e];
}

// ---------------------------------------------------------------------------------------------
// Interpolation: torch.searchsorted (left), the clamps and the lerp of the reference's
// `calibrate`, each step rounded as torch rounds it (no contraction into fma).

template <typename K>
__device__ __forceinline__ K sub_rn(K a, K b);
template <>
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
template <>
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
template <typename K>
__device__ __forceinline__ K div_rn(K a, K b);
template <>
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
template <>
__device__ __forceinline__ double div_rn(double a, double b) { return __ddiv_rn(a, b); }

template <typename K>
__global__ void __launch_bounds__(256)
    interp_kernel(const K* __restrict__ x, int64_t m, const K* __restrict__ xs,
                  const double* __restrict__ fit, int64_t g, double* __restrict__ out) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < m;
       e += stride) {
    const K v = x[e];
    // first i with v <= xs[i]; NaN goes past every point, as in torch.searchsorted
    int64_t lo = 0, hi = g;
    while (lo < hi) {
      const int64_t mid = lo + ((hi - lo) >> 1);
      if (!(v <= __ldg(xs + mid))) {
        lo = mid + 1;
      } else {
        hi = mid;
      }
    }
    int64_t i = lo < 1 ? 1 : lo;  // clamp(1, g - 1): the upper bound wins when g = 1
    i = i > g - 1 ? g - 1 : i;
    const int64_t im1 = i == 0 ? g - 1 : i - 1;  // index -1 is the last point
    const K x0 = __ldg(xs + im1), x1 = __ldg(xs + i);
    K t = div_rn(sub_rn(v, x0), sub_rn(x1, x0));
    t = t < K(0) ? K(0) : t;  // clamp(0, 1); NaN stays NaN
    t = t > K(1) ? K(1) : t;
    const double f0 = __ldg(fit + im1), f1 = __ldg(fit + i);
    out[e] = __dadd_rn(f0, __dmul_rn(static_cast<double>(t), __dsub_rn(f1, f0)));
  }
}

// ---------------------------------------------------------------------------------------------
// Host side

struct GroupLayout {
  size_t keys, labels, heads, s, c, goff, cs, cc, ch, chs, chc, sort, total;
  size_t sort_bytes;
};

// presorted: the pairs come sorted (no sort, no copies of them).
template <typename K, typename L>
int group_layout(int64_t n, bool presorted, GroupLayout& l) {
  const int64_t tiles = (n + kTile - 1) / kTile;
  size_t sort_bytes = 0;
  if (!presorted) {
    const cudaError_t e = cub::DeviceRadixSort::SortPairs(
        nullptr, sort_bytes, static_cast<const K*>(nullptr), static_cast<K*>(nullptr),
        static_cast<const L*>(nullptr), static_cast<L*>(nullptr), n);
    if (e != cudaSuccess) return cal_fail(e, "cub::DeviceRadixSort::SortPairs (size)");
  }
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align256(o + bytes);
    return at;
  };
  l.keys = take(presorted ? 0 : sizeof(K) * n);
  l.labels = take(presorted ? 0 : sizeof(L) * n);
  l.heads = take(sizeof(int) * tiles);
  l.s = take(sizeof(double) * tiles);
  l.c = take(sizeof(int) * tiles);
  l.goff = take(sizeof(int64_t) * tiles);
  l.cs = take(sizeof(double) * tiles);
  l.cc = take(sizeof(int64_t) * tiles);
  const int64_t chunks = (tiles + kChunk - 1) / kChunk;
  l.ch = take(sizeof(int64_t) * chunks);
  l.chs = take(sizeof(double) * chunks);
  l.chc = take(sizeof(int64_t) * chunks);
  l.sort = take(sort_bytes);
  l.sort_bytes = sort_bytes;
  l.total = o;
  return TISO_OK;
}

template <typename K, typename L>
int run_groups(const void* scores, const void* labels, int64_t n, bool presorted, void* xs,
               double* y, double* w, int64_t* groups, void* workspace, size_t workspace_bytes,
               cudaStream_t st) {
  GroupLayout l{};
  int rc = group_layout<K, L>(n, presorted, l);
  if (rc) return rc;
  if (!workspace || workspace_bytes < l.total)
    return report_error(TISO_ERR_WORKSPACE,
                        "workspace smaller than tiso_calib_groups_workspace_size");
  char* ws = static_cast<char*>(workspace);
  if (reinterpret_cast<uintptr_t>(ws) & 255)
    return report_error(TISO_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  const K* keys = static_cast<const K*>(scores);
  const L* labs = static_cast<const L*>(labels);
  cudaError_t e = cudaMemsetAsync(groups, 0, 2 * sizeof(int64_t), st);
  if (e != cudaSuccess) return cal_fail(e, "cudaMemsetAsync(groups)");
  if (!presorted) {
    K* sk = reinterpret_cast<K*>(ws + l.keys);
    L* sl = reinterpret_cast<L*>(ws + l.labels);
    size_t sort_bytes = l.sort_bytes;
    e = cub::DeviceRadixSort::SortPairs(ws + l.sort, sort_bytes, keys, sk, labs, sl, n, 0,
                                        static_cast<int>(sizeof(K) * 8), st);
    if (e != cudaSuccess) return cal_fail(e, "cub::DeviceRadixSort::SortPairs");
    keys = sk;
    labs = sl;
  }
  const int64_t tiles = (n + kTile - 1) / kTile;
  int* t_heads = reinterpret_cast<int*>(ws + l.heads);
  double* t_s = reinterpret_cast<double*>(ws + l.s);
  int* t_c = reinterpret_cast<int*>(ws + l.c);
  int64_t* t_goff = reinterpret_cast<int64_t*>(ws + l.goff);
  double* t_cs = reinterpret_cast<double*>(ws + l.cs);
  int64_t* t_cc = reinterpret_cast<int64_t*>(ws + l.cc);
  group_tile_kernel<K, L><<<static_cast<unsigned>(tiles), kCalThreads, 0, st>>>(
      keys, labs, n, t_heads, t_s, t_c, groups);
  const int64_t chunks = (tiles + kChunk - 1) / kChunk;
  int64_t* c_heads = reinterpret_cast<int64_t*>(ws + l.ch);
  double* c_s = reinterpret_cast<double*>(ws + l.chs);
  int64_t* c_c = reinterpret_cast<int64_t*>(ws + l.chc);
  group_scan_kernel<<<static_cast<unsigned>(chunks), kScanThreads, 0, st>>>(
      tiles, t_heads, t_s, t_c, t_goff, t_cs, t_cc, c_heads, c_s, c_c);
  group_chunk_kernel<<<1, kScanThreads, 0, st>>>(chunks, c_heads, c_s, c_c, groups);
  group_write_kernel<K, L><<<static_cast<unsigned>(tiles), kCalThreads, 0, st>>>(
      keys, labs, n, t_goff, t_cs, t_cc, c_heads, c_s, c_c, static_cast<K*>(xs), y, w);
  e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cal_fail(e, "calibration group kernels launch");
}

int check_calib(int key_dtype, int label_dtype, int64_t n) {
  if (key_dtype != TISO_F32 && key_dtype != TISO_F64)
    return report_error(TISO_ERR_ARGUMENT, "key_dtype must be TISO_F32 or TISO_F64");
  if (label_dtype != TISO_F32 && label_dtype != TISO_F64)
    return report_error(TISO_ERR_ARGUMENT, "label_dtype must be TISO_F32 or TISO_F64");
  // counts are staged as 32-bit words
  if (n < 1 || n > int64_t{2147483647})
    return report_error(TISO_ERR_ARGUMENT, "n must be in [1, 2^31 - 1]");
  return TISO_OK;
}

}  // namespace
}  // namespace tiso

using namespace tiso;

extern "C" {

int tiso_calib_groups_workspace_size(int key_dtype, int label_dtype, int64_t n, int presorted,
                                     size_t* bytes) {
  if (!bytes) return report_error(TISO_ERR_ARGUMENT, "bytes is NULL");
  *bytes = 0;
  const int rc = check_calib(key_dtype, label_dtype, n);
  if (rc) return rc;
  GroupLayout l{};
  const bool ps = presorted != 0;
  int r;
  if (key_dtype == TISO_F32) {
    r = label_dtype == TISO_F32 ? group_layout<float, float>(n, ps, l)
                                : group_layout<float, double>(n, ps, l);
  } else {
    r = label_dtype == TISO_F32 ? group_layout<double, float>(n, ps, l)
                                : group_layout<double, double>(n, ps, l);
  }
  if (r) return r;
  *bytes = l.total;
  return TISO_OK;
}

int tiso_calib_groups(int key_dtype, const void* scores, int label_dtype, const void* labels,
                      int64_t n, int presorted, void* xs, double* y, double* w, int64_t* groups,
                      void* workspace, size_t workspace_bytes, void* stream) {
  const int rc = check_calib(key_dtype, label_dtype, n);
  if (rc) return rc;
  if (!scores || !labels || !xs || !y || !w || !groups)
    return report_error(TISO_ERR_ARGUMENT, "scores, labels, xs, y, w and groups must not be NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool ps = presorted != 0;
  if (key_dtype == TISO_F32) {
    return label_dtype == TISO_F32
               ? run_groups<float, float>(scores, labels, n, ps, xs, y, w, groups, workspace,
                                          workspace_bytes, st)
               : run_groups<float, double>(scores, labels, n, ps, xs, y, w, groups, workspace,
                                           workspace_bytes, st);
  }
  return label_dtype == TISO_F32
             ? run_groups<double, float>(scores, labels, n, ps, xs, y, w, groups, workspace,
                                         workspace_bytes, st)
             : run_groups<double, double>(scores, labels, n, ps, xs, y, w, groups, workspace,
                                          workspace_bytes, st);
}

int tiso_calib_interp(int key_dtype, const void* x, int64_t m, const void* xs, const double* fit,
                      int64_t g, double* out, void* stream) {
  if (key_dtype != TISO_F32 && key_dtype != TISO_F64)
    return report_error(TISO_ERR_ARGUMENT, "key_dtype must be TISO_F32 or TISO_F64");
  if (m < 0 || g < 1) return report_error(TISO_ERR_ARGUMENT, "need m >= 0 and g >= 1");
  if (m == 0) return TISO_OK;
  if (!x || !xs || !fit || !out)
    return report_error(TISO_ERR_ARGUMENT, "x, xs, fit and out must not be NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (m + 255) / 256;
  const unsigned grid = static_cast<unsigned>(want < int64_t{sms} * 8 ? want : int64_t{sms} * 8);
  if (key_dtype == TISO_F32) {
    interp_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), m,
                                               static_cast<const float*>(xs), fit, g, out);
  } else {
    interp_kernel<double><<<grid, 256, 0, st>>>(static_cast<const double*>(x), m,
                                                static_cast<const double*>(xs), fit, g, out);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TISO_OK : cal_fail(e, "interp_kernel launch");
}

}  // extern "C"
