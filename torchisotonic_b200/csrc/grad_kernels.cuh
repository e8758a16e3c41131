// Backward kernels: the gradient of the fit in y and w from the fit's block starts.
//
// With g the gradient with respect to the (clipped) output, and G, W, T the sums over an
// element's block of g, w and w y:
//   fit = T / W (the block mean; its sign needs no care: a decreasing fit's blocks are those
//         of -y and its value the mean of y);
//   G is zeroed for a block whose fit lies outside [y_min, y_max] (the clamp's backward: bounds
//   inclusive, a NaN fit masked; src/torchisotonic/_api.py:68-69 under autograd);
//   d/dy = w G / W,  d/dw = (y - fit) G / W   (src/torchisotonic/_api.py:92-97).
//
// Here: whole rows of 65..1024 elements (grad_tile_kernel: a CTA of 128 threads, 8 elements
// each, in segments of 2^log2g threads, the rows staged in shared memory; per thread, one pass
// over its elements gives the sums before its first block start (H), from its last start (L), of
// all of it (A), and the results of the blocks strictly inside it; segmented scans across the
// segment's threads give each thread the sums of the blocks that reach into it from either side;
// a second pass writes the gradients), and the first two passes of long rows in tiles of 1024:
// each tile's run (grad_tile_sums_kernel) and the scans of the runs along a row, which give each
// tile its carries. The third pass of long rows (grad_fill_kernel) and rows of at most 64
// (grad_rows_kernel) are in grad_rows.cuh.
#pragma once

#include "common.cuh"
#include "fit_kernels.cuh"

namespace tiso {

constexpr int kGK = 8;          // elements per thread
constexpr int kGThreads = 128;  // threads per CTA
constexpr int kGTile = kGK * kGThreads;

template <typename S>
struct Sum3 {
  S g, w, t;
};

template <typename S>
TISO_DEV Sum3<S> add3(Sum3<S> a, Sum3<S> b) {
  return {a.g + b.g, a.w + b.w, a.t + b.t};
}

struct GradArgs {
  const void* y;
  const void* w;
  const uint8_t* starts;
  const void* g;
  void* grad_y;
  void* grad_w;
  int64_t batch;
  int32_t n;
  int32_t log2g;
  int32_t seg_len;
  int32_t tiles;
  FastDiv div_n;
  int32_t clip_lo, clip_hi;
  double lo, hi;
  // long rows: per tile (has, H, L, A) from the first pass, then (pre, post) from the row scan
  int32_t* t_has;
  double* t_sums;  // [tiles][3 (H, L, A)][3 (g, w, t)]
  double* t_carry; // [tiles][2 (pre, post)][3]
  // rows of many tiles, scanned in chunks of tiles: per chunk its totals and the carries into it
  double* c_tot;    // [chunks][2 (forward, backward)][4 (flag, g, w, t)]
  double* c_carry;  // [chunks][2 (from before, from after)][3]
  int32_t chunks;   // chunks per row; 0: one CTA scans each row
  // one segment of a row split across devices: its first element continues a block from the
  // segment before unless starts says otherwise (cont); the row's offset y0 given (has_y0); the
  // open sums flowing in from the segments before and after it (ext: [2][3], or NULL)
  int32_t cont;
  int32_t has_y0;
  double y0;
  const double* ext;
  int32_t mode;    // 0: whole rows; 1: the sums pass of long rows; 2: their fill pass
  // ragged rows (else NULL), whole rows only: row r is elements [offsets[r], offsets[r + 1])
  // of the packed arrays, of at most n elements (longer rows are cut to n)
  const int64_t* offsets;
};

template <typename S, int K, int THREADS, bool kFit, bool kVar = false>
struct GradSmem {
  static constexpr int kSlots = THREADS * (K + 1);
  S g[kSlots];     // g (whole rows: at an interior block's start, its masked G / W), then d/dy
  S w[kSlots];     // w
  S y[kSlots];     // y, then d/dw
  S res_fit[kFit ? kSlots : 1];  // whole rows: at an interior block's start, its fit
  uint8_t st[kSlots];
  uint8_t cnt[THREADS];
  uint8_t flag[THREADS];
  Sum3<S> incl[THREADS];
  uint8_t iflag[THREADS];
  VarGeom<THREADS, kVar> vg;  // ragged rows only
};

// The block's results from its sums: masked G / W and the fit.
// t sums w (y - y0), y0 the row's first element, as in the forward (the same offset keeps the
// recomputed fit equal to the forward's).
template <typename Acc, typename S, bool kY>
TISO_DEV void block_result(const Sum3<S>& s, S y0, const GradArgs& a, S& mg, S& fit) {
  mg = s.g / s.w;
  fit = 0;
  if (kY) {
    const Acc f = static_cast<Acc>(y0 + s.t / s.w);
    fit = static_cast<S>(f);
    if ((a.clip_lo && !(f >= static_cast<Acc>(a.lo))) ||
        (a.clip_hi && !(f <= static_cast<Acc>(a.hi)))) {
      mg = 0;
    }
  }
}

// Segmented inclusive scan across the threads of each segment of 2^log2g threads, forward
// (REV false: element u combines with those before it) or backward. Combine: a flagged element
// (a block starts in that thread) stops the accumulation from further away. Two levels: a scan
// within each warp by shuffles, then, for segments wider than a warp, each thread adds the
// totals of the other warps of its segment, nearest first, up to the first flagged one.
template <typename S, int THREADS, bool REV>
TISO_DEV void seg_scan(bool& f, Sum3<S>& v, int log2g, Sum3<S>* sm, uint8_t* fm) {
  const int u = threadIdx.x;
  const int G = 1 << log2g;
  const int r = REV ? (G - 1 - (u & (G - 1))) : (u & (G - 1));
  // distance to the warp's edge in the scan's direction: a shuffle from beyond it returns the
  // caller's own value, which must not be combined
  const int lane = REV ? (31 - (u & 31)) : (u & 31);
  for (int d = 1; d < 32 && d < G; d <<= 1) {
    const int f2 = REV ? __shfl_down_sync(0xffffffffu, static_cast<int>(f), d)
                       : __shfl_up_sync(0xffffffffu, static_cast<int>(f), d);
    Sum3<S> v2;
    v2.g = REV ? __shfl_down_sync(0xffffffffu, v.g, d) : __shfl_up_sync(0xffffffffu, v.g, d);
    v2.w = REV ? __shfl_down_sync(0xffffffffu, v.w, d) : __shfl_up_sync(0xffffffffu, v.w, d);
    v2.t = REV ? __shfl_down_sync(0xffffffffu, v.t, d) : __shfl_up_sync(0xffffffffu, v.t, d);
    if (r >= d && lane >= d) {
      if (!f) v = add3(v, v2);
      f = f || f2;
    }
  }
  if (G > 32) {
    const int wid = u >> 5;
    if (lane == 31) {  // the warp's last thread in the scan's direction holds the warp's total
      sm[wid] = v;
      fm[wid] = f;
    }
    __syncthreads();
    if (!f) {
      const int w0 = (u & ~(G - 1)) >> 5, w1 = w0 + (G >> 5);  // the segment's warps
      Sum3<S> acc{0, 0, 0};
      if (REV) {
        for (int k = wid + 1; k < w1; ++k) {
          acc = add3(acc, sm[k]);
          if (fm[k]) {
            f = true;
            break;
          }
        }
      } else {
        for (int k = wid - 1; k >= w0; --k) {
          acc = add3(acc, sm[k]);
          if (fm[k]) {
            f = true;
            break;
          }
        }
      }
      v = add3(v, acc);
    }
    __syncthreads();
  }
}

// Whole rows of 65..1024 elements (segments of 2^log2g threads, 128 / 2^log2g rows per CTA):
// each block's results kept at its first element and written in the unrolled pass 2.
// kVar: ragged rows (a.offsets); each row staged in and out on its own.
template <typename In, bool kW, bool kY, bool kVar = false>
__global__ void __launch_bounds__(kGThreads) grad_tile_kernel(const GradArgs a) {
  using S = double;
  using Acc = acc_of<In>;
  constexpr int K = kGK, THREADS = kGThreads;
  using Sm = GradSmem<S, K, THREADS, true, kVar>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Sm& s = *reinterpret_cast<Sm*>(smem_raw);
  const int tid = threadIdx.x;
  const int log2g = a.log2g;
  const int G = 1 << log2g;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * (THREADS >> log2g);
  const int64_t left = a.batch - row0;
  const int nseg = static_cast<int>(left < (THREADS >> log2g) ? left : (THREADS >> log2g));
  const int seglen = a.n;
  const int64_t gbase = row0 * a.n;
  const int span = nseg * a.n;
  const int q = tid >> log2g;
  if constexpr (kVar) {
    load_var_geom(s.vg, a.offsets, row0, nseg, K << log2g);
    __syncthreads();
  }
  {
    const int r = tid & (G - 1);
    int c = 0;
    if (q < nseg) {
      int sl = seglen;
      if constexpr (kVar) sl = s.vg.len[q];
      c = sl - r * K;
      c = c < 0 ? 0 : (c > K ? K : c);
    }
    s.cnt[tid] = static_cast<uint8_t>(c);
  }
  // staging
  const SpanMap m{seglen, log2g, a.div_n, true, seglen == (K << log2g), 0};
  if constexpr (kVar) {
    // each row on its own, coalesced along it
    for (int q2 = 0; q2 < nseg; ++q2) {
      const int64_t o = s.vg.ofs[q2];
      const int len = s.vg.len[q2];
      for (int e = tid; e < len; e += THREADS) {
        const int sl = slot_of((q2 << log2g) + e / K, e % K, K);
        s.g[sl] = to_s<S>(static_cast<const In*>(a.g)[o + e]);
        if constexpr (kW) s.w[sl] = static_cast<S>(static_cast<const Acc*>(a.w)[o + e]);
        if constexpr (kY) s.y[sl] = to_s<S>(static_cast<const In*>(a.y)[o + e]);
        s.st[sl] = a.starts[o + e];
      }
    }
  } else {
    stage_in_<K, THREADS, 4, false>(static_cast<const In*>(a.g) + gbase, span, s.g, m,
                            [](In v) { return to_s<S>(v); });
    if (kW) {
      stage_in_<K, THREADS, 4, false>(static_cast<const Acc*>(a.w) + gbase, span, s.w, m,
                              [](Acc v) { return static_cast<S>(v); });
    }
    if (kY) {
      stage_in_<K, THREADS, 4, false>(static_cast<const In*>(a.y) + gbase, span, s.y, m,
                              [](In v) { return to_s<S>(v); });
    }
    stage_in_<K, THREADS, 2, false>(a.starts + gbase, span, s.st, m, [](uint8_t v) { return v; });
  }
  __syncthreads();
  // a block starts at every row's first element
  if (tid < nseg) s.st[slot_of(tid << log2g, 0, K)] = 1;
  __syncthreads();

  S y0 = S(0);
  if (kY) {
    y0 = offset_of(s.y[slot_of(q << log2g, 0, K)]);
  }

  // pass 1
  const int c = s.cnt[tid];
  const int b = slot_of(tid, 0, K);
  bool has = false;
  int first = K, last = -1;
  Sum3<S> run{0, 0, 0}, H{0, 0, 0}, A{0, 0, 0};
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (j < c) {
      if (s.st[b + j]) {
        if (!has) {
          H = run;
          has = true;
          first = j;
        } else {
          S mg, fit;
          block_result<Acc, S, kY>(run, y0, a, mg, fit);
          s.g[b + last] = mg;  // g of that element has been summed already
          if (kY) s.res_fit[b + last] = fit;
        }
        run = Sum3<S>{0, 0, 0};
        last = j;
      }
      const S wv = kW ? s.w[b + j] : S(1);
      const Sum3<S> e{s.g[b + j], wv, kY ? wv * (s.y[b + j] - y0) : S(0)};
      run = add3(run, e);
      A = add3(A, e);
    }
  }
  const Sum3<S> L = has ? run : A;
  if (!has) H = A;

  // forward scan: the open block's sums up to the end of each thread
  bool f = has;
  Sum3<S> v = has ? L : A;
  seg_scan<S, THREADS, false>(f, v, log2g, s.incl, s.iflag);
  __syncthreads();
  s.incl[tid] = v;
  s.iflag[tid] = f;
  __syncthreads();
  const int r = tid & (G - 1);
  Sum3<S> pre{0, 0, 0};
  if (r > 0) pre = s.incl[tid - 1];
  __syncthreads();
  // backward scan: the sums from the start of each thread to the end of the block open there
  f = has;
  v = has ? H : A;
  seg_scan<S, THREADS, true>(f, v, log2g, s.incl, s.iflag);
  __syncthreads();
  s.incl[tid] = v;
  s.iflag[tid] = f;
  __syncthreads();
  Sum3<S> post{0, 0, 0};
  if (r < G - 1) post = s.incl[tid + 1];

  // totals of the block reaching into the thread from the left, and of its last block
  const Sum3<S> first_tot = add3(pre, has ? H : add3(A, post));
  const Sum3<S> last_tot = add3(L, post);
  S mg_first, fit_first, mg_last, fit_last;
  block_result<Acc, S, kY>(first_tot, y0, a, mg_first, fit_first);
  block_result<Acc, S, kY>(last_tot, y0, a, mg_last, fit_last);

  // pass 2
  S mg = mg_first, fit = fit_first;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (j < c) {
      if (has && j >= first && s.st[b + j]) {
        if (j == last) {
          mg = mg_last;
          fit = fit_last;
        } else {
          mg = s.g[b + j];
          if (kY) fit = s.res_fit[b + j];
        }
      }
      const S wv = kW ? s.w[b + j] : S(1);
      s.g[b + j] = wv * mg;
      if (kY) s.y[b + j] = (s.y[b + j] - fit) * mg;
    }
  }
  __syncthreads();
  if constexpr (kVar) {
    for (int q2 = 0; q2 < nseg; ++q2) {
      const int64_t o = s.vg.ofs[q2];
      const int len = s.vg.len[q2];
      for (int e = tid; e < len; e += THREADS) {
        const int sl = slot_of((q2 << log2g) + e / K, e % K, K);
        if (a.grad_y) static_cast<In*>(a.grad_y)[o + e] = from_acc<In>(static_cast<Acc>(s.g[sl]));
        if (kY && a.grad_w) static_cast<Acc*>(a.grad_w)[o + e] = static_cast<Acc>(s.y[sl]);
      }
    }
    return;
  }
  if (a.grad_y) {
    stage_out_<K, THREADS, false>(static_cast<In*>(a.grad_y) + gbase, span, m,
                          [&](const auto& it) {
                            return from_acc<In>(static_cast<Acc>(s.g[it.slot(m)]));
                          });
  }
  if (kY && a.grad_w) {
    stage_out_<K, THREADS, false>(static_cast<Acc*>(a.grad_w) + gbase, span, m,
                          [&](const auto& it) { return static_cast<Acc>(s.y[it.slot(m)]); });
  }
}

// K consecutive elements from p (16-byte vector loads when p is 16-byte aligned), streamed.
template <int K, typename T>
TISO_DEV void load_run(const T* p, int valid, T (&v)[K]) {
  constexpr int V = 16 / sizeof(T);
  if (valid == K && K % V == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
    for (int k = 0; k < K / V; ++k) {
      const uint4 r = __ldcs(reinterpret_cast<const uint4*>(p) + k);
#pragma unroll
      for (int i = 0; i < V; ++i) v[k * V + i] = reinterpret_cast<const T*>(&r)[i];
    }
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) v[k] = k < valid ? p[k] : T(0);
  }
}

// A run of elements as the first pass of the backward sees it: whether a block starts in it,
// the sums before its first start (H), from its last start on (L), and of all of it (A).
struct RunSums {
  bool has;
  Sum3<double> h, l, all;
};

// The run of x followed by the run of y.
TISO_DEV RunSums join_runs(const RunSums& x, const RunSums& y) {
  RunSums r;
  r.has = x.has || y.has;
  r.h = x.has ? x.h : add3(x.all, y.h);
  r.l = y.has ? y.l : add3(x.l, y.all);
  r.all = add3(x.all, y.all);
  return r;
}

TISO_DEV RunSums shfl_down_runs(const RunSums& x, int d) {
  RunSums r;
  r.has = __shfl_down_sync(0xffffffffu, static_cast<int>(x.has), d) != 0;
  r.h = {__shfl_down_sync(0xffffffffu, x.h.g, d), __shfl_down_sync(0xffffffffu, x.h.w, d),
         __shfl_down_sync(0xffffffffu, x.h.t, d)};
  r.l = {__shfl_down_sync(0xffffffffu, x.l.g, d), __shfl_down_sync(0xffffffffu, x.l.w, d),
         __shfl_down_sync(0xffffffffu, x.l.t, d)};
  r.all = {__shfl_down_sync(0xffffffffu, x.all.g, d), __shfl_down_sync(0xffffffffu, x.all.w, d),
           __shfl_down_sync(0xffffffffu, x.all.t, d)};
  return r;
}

// Long rows, first pass of the backward: per tile (has a start, H, L, A), read straight from
// global memory - every thread folds its K consecutive elements, then the runs of the CTA's
// threads are joined in order (shuffles within warps, then the warps' runs). Nothing is
// staged; the pass streams starts, g, w and y once.
template <typename In, bool kW, bool kY>
__global__ void __launch_bounds__(kGThreads) grad_tile_sums_kernel(const GradArgs a) {
  using S = double;
  using Acc = acc_of<In>;
  constexpr int K = kGK, THREADS = kGThreads;
  __shared__ RunSums warp_runs[THREADS / 32];
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t row = blockIdx.x / a.tiles;
  const int tile = static_cast<int>(blockIdx.x - row * a.tiles);
  const int64_t t0 = static_cast<int64_t>(tile) * a.seg_len;
  const int seglen = static_cast<int>(a.n - t0 < a.seg_len ? a.n - t0 : a.seg_len);
  const int64_t gbase = row * a.n + t0;
  const int e0 = tid * K;
  const int valid = seglen - e0 < 0 ? 0 : (seglen - e0 > K ? K : seglen - e0);
  S y0 = S(0);
  if (kY) {
    y0 = a.has_y0 ? static_cast<S>(a.y0)
                  : offset_of(to_s<S>(static_cast<const In*>(a.y)[row * a.n]));
  }
  RunSums run{false, {0, 0, 0}, {0, 0, 0}, {0, 0, 0}};
  if (valid > 0) {
    In gv[K];
    uint8_t sv[K];
    load_run<K>(static_cast<const In*>(a.g) + gbase + e0, valid, gv);
    if constexpr (K == 8) {
      if (valid == K && ((reinterpret_cast<uintptr_t>(a.starts + gbase + e0) & 7) == 0)) {
        const uint2 r = __ldcs(reinterpret_cast<const uint2*>(a.starts + gbase + e0));
#pragma unroll
        for (int k = 0; k < K; ++k) sv[k] = reinterpret_cast<const uint8_t*>(&r)[k];
      } else {
#pragma unroll
        for (int k = 0; k < K; ++k) sv[k] = k < valid ? a.starts[gbase + e0 + k] : 0;
      }
    } else {
#pragma unroll
      for (int k = 0; k < K; ++k) sv[k] = k < valid ? a.starts[gbase + e0 + k] : 0;
    }
    Acc wv[K];
    In yv[K];
    if (kW) load_run<K>(static_cast<const Acc*>(a.w) + gbase + e0, valid, wv);
    if (kY) load_run<K>(static_cast<const In*>(a.y) + gbase + e0, valid, yv);
    Sum3<S> cur{0, 0, 0};
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (k < valid) {
        if (sv[k] || (t0 + e0 + k == 0 && !a.cont)) {
          if (!run.has) run.h = cur;
          run.has = true;
          cur = Sum3<S>{0, 0, 0};
        }
        const S w = kW ? static_cast<S>(wv[k]) : S(1);
        const Sum3<S> e{to_s<S>(gv[k]), w, kY ? w * (to_s<S>(yv[k]) - y0) : S(0)};
        cur = add3(cur, e);
        run.all = add3(run.all, e);
      }
    }
    run.l = run.has ? cur : run.all;
    if (!run.has) run.h = run.all;
  }
  // join the runs in order: lane l takes lane l + d's run as its right neighbour
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const RunSums other = shfl_down_runs(run, d);
    if ((lane & (2 * d - 1)) == 0) run = join_runs(run, other);
  }
  if (lane == 0) warp_runs[tid >> 5] = run;
  __syncthreads();
  if (tid == 0) {
    RunSums t = warp_runs[0];
#pragma unroll
    for (int w = 1; w < THREADS / 32; ++w) t = join_runs(t, warp_runs[w]);
    const int64_t id = row * a.tiles + tile;
    a.t_has[id] = t.has;
    double* tp = a.t_sums + id * 9;
    tp[0] = t.h.g; tp[1] = t.h.w; tp[2] = t.h.t;
    tp[3] = t.l.g; tp[4] = t.l.w; tp[5] = t.l.t;
    tp[6] = t.all.g; tp[7] = t.all.w; tp[8] = t.all.t;
  }
}

// The segmented scans of a row's items [0, m) - tiles, or chunks of tiles - in both directions,
// in pieces of THREADS (one CTA). An item carries, per direction, whether a block starts in it
// and its open sums: forward, those after its last block start (all of it if none); backward,
// those before its first start. pre(i): the open sums reaching item i from the items before it
// (back to the last that starts a block; cin_f flows in before item 0); post(i): the sums from
// the items after i up to the first that starts a block (cin_b flows in after item m - 1).
template <int THREADS, typename ItemF, typename ItemB, typename PutPre, typename PutPost>
TISO_DEV void scan_row_items(int m, Sum3<double> cin_f, Sum3<double> cin_b, ItemF item_f,
                             ItemB item_b, PutPre put_pre, PutPost put_post) {
  using S = double;
  __shared__ Sum3<S> sm[THREADS];
  __shared__ uint8_t fm[THREADS];
  __shared__ Sum3<S> carry_v;
  const int tid = threadIdx.x;
  constexpr int log2t = THREADS == 1024 ? 10 : THREADS == 512 ? 9 : THREADS == 256 ? 8 : 7;
  static_assert((1 << log2t) == THREADS, "THREADS: 128 to 1024, a power of two");
  // forward
  if (tid == 0) carry_v = cin_f;
  __syncthreads();
  for (int c0 = 0; c0 < m; c0 += THREADS) {
    const int c = c0 + tid;
    bool f = false;
    Sum3<S> v{0, 0, 0};
    if (c < m) item_f(c, f, v);
    seg_scan<S, THREADS, false>(f, v, log2t, sm, fm);
    __syncthreads();
    sm[tid] = v;
    fm[tid] = f;
    __syncthreads();
    Sum3<S> pre = carry_v;
    if (tid > 0) {
      pre = sm[tid - 1];
      if (!fm[tid - 1]) pre = add3(pre, carry_v);
    }
    if (c < m) put_pre(c, pre);
    __syncthreads();
    if (tid == THREADS - 1) carry_v = fm[tid] ? sm[tid] : add3(sm[tid], carry_v);
    __syncthreads();
  }
  // backward
  if (tid == 0) carry_v = cin_b;
  __syncthreads();
  const int pieces = (m + THREADS - 1) / THREADS;
  for (int k = pieces - 1; k >= 0; --k) {
    const int c = k * THREADS + tid;
    bool f = false;
    Sum3<S> v{0, 0, 0};
    if (c < m) item_b(c, f, v);
    seg_scan<S, THREADS, true>(f, v, log2t, sm, fm);
    __syncthreads();
    sm[tid] = v;
    fm[tid] = f;
    __syncthreads();
    Sum3<S> post = carry_v;
    if (tid < THREADS - 1) {
      post = sm[tid + 1];
      if (!fm[tid + 1]) post = add3(post, carry_v);
    }
    if (c < m) put_post(c, post);
    __syncthreads();
    if (tid == 0) carry_v = fm[0] ? sm[0] : add3(sm[0], carry_v);
    __syncthreads();
  }
}

// A tile of a long row as an item of the scans: forward (has a start, L or A), backward
// (has a start, H or A); t_sums holds [H, L, A] x [g, w, t].
TISO_DEV void tile_item_f(const GradArgs& a, int64_t id, bool& f, Sum3<double>& v) {
  f = a.t_has[id] != 0;
  const double* tp = a.t_sums + id * 9;
  v = f ? Sum3<double>{tp[3], tp[4], tp[5]} : Sum3<double>{tp[6], tp[7], tp[8]};
}
TISO_DEV void tile_item_b(const GradArgs& a, int64_t id, bool& f, Sum3<double>& v) {
  f = a.t_has[id] != 0;
  const double* tp = a.t_sums + id * 9;
  v = f ? Sum3<double>{tp[0], tp[1], tp[2]} : Sum3<double>{tp[6], tp[7], tp[8]};
}

// pre and post of every tile. a.chunks == 0: one CTA per row scans all its tiles. Else one CTA
// per chunk of THREADS tiles, with the carries into the chunk from grad_chunk_carry_kernel.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) grad_row_scan_kernel(const GradArgs a) {
  int64_t row = blockIdx.x;
  int first = 0, m = a.tiles;
  Sum3<double> cin_f{0, 0, 0}, cin_b{0, 0, 0};
  if (a.ext) {
    cin_f = Sum3<double>{a.ext[0], a.ext[1], a.ext[2]};
    cin_b = Sum3<double>{a.ext[3], a.ext[4], a.ext[5]};
  }
  if (a.chunks > 0) {
    row = blockIdx.x / a.chunks;
    const int ch = static_cast<int>(blockIdx.x - row * a.chunks);
    first = ch * THREADS;
    m = a.tiles - first < THREADS ? a.tiles - first : THREADS;
    const double* cc = a.c_carry + (row * a.chunks + ch) * 6;
    cin_f = Sum3<double>{cc[0], cc[1], cc[2]};
    cin_b = Sum3<double>{cc[3], cc[4], cc[5]};
  }
  const int64_t base = row * a.tiles + first;
  scan_row_items<THREADS>(
      m, cin_f, cin_b,
      [&](int c, bool& f, Sum3<double>& v) { tile_item_f(a, base + c, f, v); },
      [&](int c, bool& f, Sum3<double>& v) { tile_item_b(a, base + c, f, v); },
      [&](int c, const Sum3<double>& pre) {
        double* cp = a.t_carry + (base + c) * 6;
        cp[0] = pre.g; cp[1] = pre.w; cp[2] = pre.t;
      },
      [&](int c, const Sum3<double>& post) {
        double* cp = a.t_carry + (base + c) * 6;
        cp[3] = post.g; cp[4] = post.w; cp[5] = post.t;
      });
}

// Rows of many tiles, step 1: per chunk of THREADS tiles, its totals as an item - forward,
// whether a block starts in it and the open sums at its end; backward, the same and the sums
// before its first start. c_tot: [chunk][2 (forward, backward)][4 (flag, g, w, t)].
template <int THREADS>
__global__ void __launch_bounds__(THREADS) grad_chunk_total_kernel(const GradArgs a) {
  using S = double;
  __shared__ Sum3<S> sm[THREADS];
  __shared__ uint8_t fm[THREADS];
  constexpr int log2t = THREADS == 1024 ? 10 : THREADS == 512 ? 9 : THREADS == 256 ? 8 : 7;
  const int64_t row = blockIdx.x / a.chunks;
  const int ch = static_cast<int>(blockIdx.x - row * a.chunks);
  const int c = ch * THREADS + threadIdx.x;
  const int64_t id = row * a.tiles + c;
  double* out = a.c_tot + (row * a.chunks + ch) * 8;
  bool f = false;
  Sum3<S> v{0, 0, 0};
  if (c < a.tiles) tile_item_f(a, id, f, v);
  seg_scan<S, THREADS, false>(f, v, log2t, sm, fm);
  if (threadIdx.x == THREADS - 1) {
    out[0] = f ? 1.0 : 0.0; out[1] = v.g; out[2] = v.w; out[3] = v.t;
  }
  __syncthreads();
  f = false;
  v = Sum3<S>{0, 0, 0};
  if (c < a.tiles) tile_item_b(a, id, f, v);
  seg_scan<S, THREADS, true>(f, v, log2t, sm, fm);
  if (threadIdx.x == 0) {
    out[4] = f ? 1.0 : 0.0; out[5] = v.g; out[6] = v.w; out[7] = v.t;
  }
}

// Step 2: per row (one CTA), the scans over its chunks: the carries into each chunk from the
// chunks before it and after it. c_carry: [chunk][2 (from before, from after)][3].
template <int THREADS>
__global__ void __launch_bounds__(THREADS) grad_chunk_carry_kernel(const GradArgs a) {
  const int64_t row = blockIdx.x;
  const double* tot = a.c_tot + row * a.chunks * 8;
  double* car = a.c_carry + row * a.chunks * 6;
  Sum3<double> cin_f{0, 0, 0}, cin_b{0, 0, 0};
  if (a.ext) {
    cin_f = Sum3<double>{a.ext[0], a.ext[1], a.ext[2]};
    cin_b = Sum3<double>{a.ext[3], a.ext[4], a.ext[5]};
  }
  scan_row_items<THREADS>(
      a.chunks, cin_f, cin_b,
      [&](int c, bool& f, Sum3<double>& v) {
        const double* t = tot + c * 8;
        f = t[0] != 0.0;
        v = Sum3<double>{t[1], t[2], t[3]};
      },
      [&](int c, bool& f, Sum3<double>& v) {
        const double* t = tot + c * 8 + 4;
        f = t[0] != 0.0;
        v = Sum3<double>{t[1], t[2], t[3]};
      },
      [&](int c, const Sum3<double>& pre) {
        double* cp = car + c * 6;
        cp[0] = pre.g; cp[1] = pre.w; cp[2] = pre.t;
      },
      [&](int c, const Sum3<double>& post) {
        double* cp = car + c * 6;
        cp[3] = post.g; cp[4] = post.w; cp[5] = post.t;
      });
}

// One segment of a row split across devices, after the first pass: the run of the whole
// segment (its tiles' runs joined in order) as 10 doubles: has a start, H, L, A.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) grad_join_tiles_kernel(const GradArgs a, double* out) {
  __shared__ RunSums warp_runs[THREADS / 32];
  __shared__ RunSums acc;
  const int tid = threadIdx.x, lane = tid & 31;
  const RunSums none{false, {0, 0, 0}, {0, 0, 0}, {0, 0, 0}};
  if (tid == 0) acc = none;
  __syncthreads();
  for (int c0 = 0; c0 < a.tiles; c0 += THREADS) {
    const int c = c0 + tid;
    RunSums run = none;
    if (c < a.tiles) {
      const double* tp = a.t_sums + static_cast<int64_t>(c) * 9;
      run.has = a.t_has[c] != 0;
      run.h = {tp[0], tp[1], tp[2]};
      run.l = {tp[3], tp[4], tp[5]};
      run.all = {tp[6], tp[7], tp[8]};
    }
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const RunSums other = shfl_down_runs(run, d);
      if ((lane & (2 * d - 1)) == 0) run = join_runs(run, other);
    }
    if (lane == 0) warp_runs[tid >> 5] = run;
    __syncthreads();
    if (tid == 0) {
      RunSums t = acc;
      for (int w = 0; w < THREADS / 32; ++w) t = join_runs(t, warp_runs[w]);
      acc = t;
    }
    __syncthreads();
  }
  if (tid == 0) {
    out[0] = acc.has ? 1.0 : 0.0;
    out[1] = acc.h.g; out[2] = acc.h.w; out[3] = acc.h.t;
    out[4] = acc.l.g; out[5] = acc.l.w; out[6] = acc.l.t;
    out[7] = acc.all.g; out[8] = acc.all.w; out[9] = acc.all.t;
  }
}

// The open sums flowing into segment `me` of `parts` from the segments before it (the end of
// their joined run) and after it (the start of theirs), from the gathered runs ([parts][10]).
__global__ void seg_grad_carry_kernel(int parts, int me, const double* runs, double* ext) {
  auto load = [&](int k) {
    const double* r = runs + k * 10;
    return RunSums{r[0] != 0.0, {r[1], r[2], r[3]}, {r[4], r[5], r[6]}, {r[7], r[8], r[9]}};
  };
  const RunSums none{false, {0, 0, 0}, {0, 0, 0}, {0, 0, 0}};
  RunSums before = none, after = none;
  for (int k = 0; k < me; ++k) before = join_runs(before, load(k));
  for (int k = parts - 1; k > me; --k) after = join_runs(load(k), after);
  const Sum3<double> f = before.has ? before.l : before.all;
  const Sum3<double> b = after.has ? after.h : after.all;
  ext[0] = f.g; ext[1] = f.w; ext[2] = f.t;
  ext[3] = b.g; ext[4] = b.w; ext[5] = b.t;
}

}  // namespace tiso
