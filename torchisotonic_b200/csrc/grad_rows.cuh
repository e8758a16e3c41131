// Backward kernels in registers, a lane per 8 elements: rows of at most 64 elements, of one
// length or ragged (grad_rows_kernel: G = 1, 2, 4 or 8 lanes per row, 32 / G rows per warp) and
// the fill pass of long rows (grad_fill_kernel: a tile of 1024 elements per CTA of 128 lanes).
//
// The gradients of the fit from its block starts (the reference's backward,
// src/torchisotonic/_api.py:86-115): with G, W, T an element's block sums of g, w and
// w (y - y0), d/dy = w G / W and d/dw = (y - fit) G / W, fit = y0 + T / W, G zeroed for a block
// whose fit lies outside [y_min, y_max] (bounds inclusive, a NaN fit masked) - the arithmetic of
// grad_tile_kernel's whole rows (block_result), in double.
//
// A lane's 8 elements are consecutive (16-byte loads where the row allows, so a warp's loads
// cover its rows' contiguous bytes). Per lane, one pass gives the sums before its first block
// start (H), from its last start (L) and of all of it (A); segmented shuffle scans across the
// row's lanes give the sums of the block arriving from the left (over L, or A where no block
// starts) and of the block continuing to the right (over H). A pass from the lane's last element
// down to its first closes each block at its start, a position known at compile time, so each
// block's masked G / W and fit land in registers indexed statically; a forward pass writes the
// gradients.
#pragma once

#include "common.cuh"
#include "grad_kernels.cuh"

namespace tiso {

constexpr int kGRowsN = 64;  // longest row
constexpr int kGRowsK = 8;   // elements per lane

// elements [base, base + 8) of a row of n (those below n): 16-byte loads (one to four) when vec
template <typename In, typename X>
TISO_DEV void load8(const In* p, int base, int n, bool vec, X (&x)[kGRowsK]) {
  constexpr int V = 16 / sizeof(In);
  if (vec) {
#pragma unroll
    for (int v = 0; v < (kGRowsK + V - 1) / V; ++v) {
      const uint4 r = __ldg(reinterpret_cast<const uint4*>(p + base) + v);
#pragma unroll
      for (int i = 0; i < V && v * V + i < kGRowsK; ++i) {
        if constexpr (std::is_same_v<In, X>) {
          x[v * V + i] = reinterpret_cast<const In*>(&r)[i];
        } else {
          x[v * V + i] = to_s<X>(reinterpret_cast<const In*>(&r)[i]);
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < kGRowsK; ++j) {
      if (base + j < n) {
        if constexpr (std::is_same_v<In, X>) {
          x[j] = p[base + j];
        } else {
          x[j] = to_s<X>(p[base + j]);
        }
      }
    }
  }
}

template <typename S>
TISO_DEV Sum3<S> shfl3_up(Sum3<S> v, int d, int width) {
  return {__shfl_up_sync(0xffffffffu, v.g, d, width), __shfl_up_sync(0xffffffffu, v.w, d, width),
          __shfl_up_sync(0xffffffffu, v.t, d, width)};
}

template <typename S>
TISO_DEV Sum3<S> shfl3_down(Sum3<S> v, int d, int width) {
  return {__shfl_down_sync(0xffffffffu, v.g, d, width),
          __shfl_down_sync(0xffffffffu, v.w, d, width),
          __shfl_down_sync(0xffffffffu, v.t, d, width)};
}

// A lane's part of the backward once the sums around it are known: in_l, the block arriving
// from the left; in_r, the block continuing to the right; e, st its elements' (g, w, w (y - y0))
// and block starts (valid of them in range), xy their y. From the lane's last element down, each
// block is closed at its start (a position known at compile time) and its masked G / W and fit
// written over that element's g and t, read already (w stays: d/dy needs it); then d/dy (to gy)
// and d/dw (to gw) of the elements, either pointer NULL when not wanted, by 16-byte stores when
// all K are in range and aligned.
template <typename In, bool kW, bool kY, int K>
TISO_DEV void lane_gradients(Sum3<double> (&e)[K], const bool (&st)[K], const double (&xy)[K],
                             Sum3<double> in_l, Sum3<double> in_r, bool has, double y0,
                             const GradArgs& a, In* gy, acc_of<In>* gw, int valid) {
  using Acc = acc_of<In>;
  using S = double;
  Sum3<S> acc{0, 0, 0};
  bool later = false;  // a start after this position within the lane
#pragma unroll
  for (int j = K - 1; j >= 0; --j) {
    acc = add3(acc, e[j]);
    if (st[j]) {
      const Sum3<S> tot = later ? acc : add3(acc, in_r);
      S mg, fit;
      block_result<Acc, S, kY>(tot, y0, a, mg, fit);
      e[j].g = mg;
      e[j].t = fit;
      acc = Sum3<S>{0, 0, 0};
      later = true;
    }
  }
  // the block the lane starts in: from the left, the lane's head, and (no start) the right
  S mg = S(0), fit = S(0);
  {
    Sum3<S> tot = add3(in_l, acc);
    if (!has) tot = add3(tot, in_r);
    if (!st[0]) block_result<Acc, S, kY>(tot, y0, a, mg, fit);
  }
  if (valid <= 0) return;
  constexpr int UY = (K * sizeof(In)) / 16, UW = (K * sizeof(Acc)) / 16;
  union {
    uint4 u[UY > 0 ? UY : 1];
    In e[K];
  } py;
  union {
    uint4 u[UW > 0 ? UW : 1];
    Acc e[K];
  } pw;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (st[j]) {
      mg = e[j].g;
      fit = e[j].t;
    }
    py.e[j] = from_acc<In>(static_cast<Acc>(e[j].w * mg));
    if constexpr (kY) pw.e[j] = static_cast<Acc>((xy[j] - fit) * mg);
  }
  if (gy) {
    if (UY > 0 && valid == K && (reinterpret_cast<uintptr_t>(gy) & 15) == 0) {
#pragma unroll
      for (int v = 0; v < UY; ++v) {
        __stcs(reinterpret_cast<uint4*>(gy) + v, py.u[v]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        if (j < valid) gy[j] = py.e[j];
      }
    }
  }
  if constexpr (kY) {
    if (gw) {
      if (UW > 0 && valid == K && (reinterpret_cast<uintptr_t>(gw) & 15) == 0) {
#pragma unroll
        for (int v = 0; v < UW; ++v) {
          __stcs(reinterpret_cast<uint4*>(gw) + v, pw.u[v]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < K; ++j) {
          if (j < valid) gw[j] = pw.e[j];
        }
      }
    }
  }
}

// kVar: ragged rows (a.offsets; row r is elements [offsets[r], offsets[r + 1]) of the packed
// arrays, its length clamped to 8 G, the capacity of its lanes, as the staged ragged kernels do).
template <typename In, bool kW, bool kY, int G, bool kVar = false>
__global__ void __launch_bounds__(128) grad_rows_kernel(const GradArgs a) {
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "lanes per row");
  using Acc = acc_of<In>;
  using S = double;
  constexpr int K = kGRowsK;
  const int lane = threadIdx.x & 31;
  const int u = lane % G;  // the lane's place in its row
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / G;
  // lanes past the last row stay for the shuffles with nothing to read or write
  const bool live = row < a.batch;
  const int base = u * K;
  // the row's first element in the arrays and its length
  int64_t rb = 0;
  int n = 0;
  if (live) {
    if constexpr (kVar) {
      rb = a.offsets[row];
      const int64_t len = a.offsets[row + 1] - rb;
      n = static_cast<int>(len < 0 ? 0 : (len > K * G ? K * G : len));
    } else {
      rb = row * a.n;
      n = a.n;
    }
  }
  const In* gr = static_cast<const In*>(a.g) + rb;
  const In* yr = kY ? static_cast<const In*>(a.y) + rb : nullptr;
  const Acc* wr = kW ? static_cast<const Acc*>(a.w) + rb : nullptr;
  const uint8_t* sr = a.starts + rb;
  const int valid = n - base < 0 ? 0 : (n - base > K ? K : n - base);
  auto vec = [&](const void* p, int bytes) {  // the lane's 8 elements as whole 16-byte units
    return valid == K && ((K * bytes) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(static_cast<const char*>(p) + base * bytes) & 15) == 0;
  };
  const bool mine = valid > 0;

  S xg[K], xw[K], xy[K];
  bool st[K];
  {
    uint8_t xs[K];
    Acc ag[K], aw[K], ay[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
      xs[j] = 0;
      ag[j] = aw[j] = ay[j] = Acc(0);
    }
    if (mine) {
      // starts: 8 bytes, one 8-byte load when aligned
      if (valid == K && (reinterpret_cast<uintptr_t>(sr + base) & 7) == 0) {
        const uint2 v = *reinterpret_cast<const uint2*>(sr + base);
#pragma unroll
        for (int j = 0; j < K; ++j) xs[j] = static_cast<uint8_t>((j < 4 ? v.x : v.y) >> (8 * (j & 3)));
      } else {
#pragma unroll
        for (int j = 0; j < K; ++j) xs[j] = j < valid ? sr[base + j] : 0;
      }
      load8<In>(gr, base, n, vec(gr, sizeof(In)), ag);
      if constexpr (kW) load8<Acc>(wr, base, n, vec(wr, sizeof(Acc)), aw);
      if constexpr (kY) load8<In>(yr, base, n, vec(yr, sizeof(In)), ay);
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const bool in = j < valid;
      // a block starts at every row's first element; positions past n start nothing
      st[j] = in && (base + j == 0 || xs[j] != 0);
      xg[j] = in ? static_cast<S>(ag[j]) : S(0);
      xw[j] = in ? (kW ? static_cast<S>(aw[j]) : S(1)) : S(0);
      xy[j] = static_cast<S>(ay[j]);
    }
  }
  // the row's offset (its first element, from lane 0 of the row)
  S y0 = S(0);
  if constexpr (kY) y0 = __shfl_sync(0xffffffffu, offset_of(xy[0]), 0, G);

  // per element: (g, w, w (y - y0)); per lane H, L, A and whether a block starts in it
  Sum3<S> e[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    e[j] = {xg[j], xw[j], kY ? xw[j] * (xy[j] - y0) : S(0)};
  }
  bool has = false;
  Sum3<S> H{0, 0, 0}, L{0, 0, 0};
#pragma unroll
  for (int j = 0; j < K; ++j) {
    L = st[j] ? e[j] : add3(L, e[j]);
    if (!has) H = st[j] ? H : add3(H, e[j]);
    has |= st[j];
  }
  // without a start, L summed the whole lane: A

  // the block arriving from the left: exclusive forward scan of (has ? L : A) that stops at a
  // lane with a start; the block continuing to the right: exclusive backward scan of H
  Sum3<S> in_l{0, 0, 0}, in_r{0, 0, 0};
  if constexpr (G > 1) {
    Sum3<S> v = L;
    bool f = has;
#pragma unroll
    for (int d = 1; d < G; d <<= 1) {
      const Sum3<S> o = shfl3_up(v, d, G);
      const bool of = __shfl_up_sync(0xffffffffu, f, d, G);
      if (u >= d && !f) v = add3(o, v);
      if (u >= d) f |= of;
    }
    // exclusive: the inclusive value of the lane before
    const Sum3<S> ex = shfl3_up(v, 1, G);
    if (u > 0) in_l = ex;
    Sum3<S> b = H;
    bool fb = has;
#pragma unroll
    for (int d = 1; d < G; d <<= 1) {
      const Sum3<S> o = shfl3_down(b, d, G);
      const bool of = __shfl_down_sync(0xffffffffu, fb, d, G);
      if (u + d < G && !fb) b = add3(b, o);
      if (u + d < G) fb |= of;
    }
    const Sum3<S> exb = shfl3_down(b, 1, G);
    if (u + 1 < G) in_r = exb;
  }

  In* gy = (mine && a.grad_y) ? static_cast<In*>(a.grad_y) + rb + base : nullptr;
  Acc* gw = (mine && kY && a.grad_w) ? static_cast<Acc*>(a.grad_w) + rb + base : nullptr;
  lane_gradients<In, kW, kY, K>(e, st, xy, in_l, in_r, has, y0, a, gy, gw, valid);
}

// The fill pass of long rows (mode 2: tiles of kGTile = 128 lanes x 8 elements, each tile's
// carries from the row scan in t_carry, the tiles' sums from grad_tile_sums_kernel before it):
// the lane work of lane_gradients, the lanes joined by warp scans (as in grad_rows_kernel, 32
// lanes wide) and the four warps by one exchange of their totals through shared memory - no
// staging of the tile, one barrier. (Four elements a lane, 256 lanes a tile, gave more resident
// warps but fewer bytes in flight each, and took 13-29% longer.)
constexpr int kFillK = 8;                      // elements per lane
constexpr int kFillThreads = kGTile / kFillK;  // lanes per tile (the sums pass's tiles)

template <typename In, bool kW, bool kY>
__global__ void __launch_bounds__(kFillThreads) grad_fill_kernel(const GradArgs a) {
  using Acc = acc_of<In>;
  using S = double;
  constexpr int K = kFillK, NW = kFillThreads / 32;
  __shared__ Sum3<S> fwd_v[NW], bwd_v[NW];
  __shared__ int fwd_f[NW], bwd_f[NW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x / a.tiles;
  const int tile = static_cast<int>(blockIdx.x - row * a.tiles);
  const int64_t t0 = static_cast<int64_t>(tile) * a.seg_len;
  const int seglen = static_cast<int>(a.n - t0 < a.seg_len ? a.n - t0 : a.seg_len);
  const int64_t gbase = row * a.n + t0;
  const int e0 = tid * K;
  const int valid = seglen - e0 < 0 ? 0 : (seglen - e0 > K ? K : seglen - e0);
  S y0 = S(0);
  if constexpr (kY) {
    y0 = a.has_y0 ? static_cast<S>(a.y0)
                  : offset_of(to_s<S>(static_cast<const In*>(a.y)[row * a.n]));
  }

  In gv[K], yv[K];
  Acc wv[K];
  uint8_t sv[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    gv[k] = yv[k] = In(0.0f);
    wv[k] = Acc(0);
    sv[k] = 0;
  }
  if (valid > 0) {
    load_run<K>(static_cast<const In*>(a.g) + gbase + e0, valid, gv);
    const uint8_t* sp = a.starts + gbase + e0;
    static_assert(K == 8, "the starts of a lane as one 8-byte word");
    if (valid == K && (reinterpret_cast<uintptr_t>(sp) & 7) == 0) {
      const uint2 r = __ldcs(reinterpret_cast<const uint2*>(sp));
#pragma unroll
      for (int k = 0; k < K; ++k) sv[k] = reinterpret_cast<const uint8_t*>(&r)[k];
    } else {
#pragma unroll
      for (int k = 0; k < K; ++k) sv[k] = k < valid ? sp[k] : 0;
    }
    if constexpr (kW) load_run<K>(static_cast<const Acc*>(a.w) + gbase + e0, valid, wv);
    if constexpr (kY) load_run<K>(static_cast<const In*>(a.y) + gbase + e0, valid, yv);
  }
  bool st[K];
  S xw[K], xy[K];
  Sum3<S> e[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const bool in = k < valid;
    // the row's first element starts a block (unless the segment continues one from before)
    st[k] = in && (sv[k] != 0 || (t0 + e0 + k == 0 && !a.cont));
    xw[k] = in ? (kW ? static_cast<S>(wv[k]) : S(1)) : S(0);
    xy[k] = in ? to_s<S>(yv[k]) : S(0);
    e[k] = in ? Sum3<S>{to_s<S>(gv[k]), xw[k], kY ? xw[k] * (xy[k] - y0) : S(0)}
              : Sum3<S>{0, 0, 0};
  }
  bool has = false;
  Sum3<S> H{0, 0, 0}, L{0, 0, 0};
#pragma unroll
  for (int k = 0; k < K; ++k) {
    L = st[k] ? e[k] : add3(L, e[k]);
    if (!has) H = st[k] ? H : add3(H, e[k]);
    has |= st[k];
  }

  // inclusive segmented scans over the warp: forward over L (A where no start), backward over H
  Sum3<S> v = L, b = H;
  bool f = has, fb = has;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const Sum3<S> o = shfl3_up(v, d, 32);
    const bool of = __shfl_up_sync(0xffffffffu, f, d);
    if (lane >= d && !f) v = add3(o, v);
    if (lane >= d) f |= of;
    const Sum3<S> ob = shfl3_down(b, d, 32);
    const bool obf = __shfl_down_sync(0xffffffffu, fb, d);
    if (lane + d < 32 && !fb) b = add3(b, ob);
    if (lane + d < 32) fb |= obf;
  }
  if (lane == 31) {
    fwd_v[warp] = v;
    fwd_f[warp] = f;
  }
  if (lane == 0) {
    bwd_v[warp] = b;
    bwd_f[warp] = fb;
  }
  // exclusive within the warp: the lane before (after) this one
  Sum3<S> ex = shfl3_up(v, 1, 32), exb = shfl3_down(b, 1, 32);
  bool exf = __shfl_up_sync(0xffffffffu, f, 1), exfb = __shfl_down_sync(0xffffffffu, fb, 1);
  if (lane == 0) {
    ex = Sum3<S>{0, 0, 0};
    exf = false;
  }
  if (lane == 31) {
    exb = Sum3<S>{0, 0, 0};
    exfb = false;
  }
  __syncthreads();
  // the warps before (after) this one, nearest first, up to one with a start; past the tile's
  // first (last) warp, the row scan's carry into the tile
  const double* cp = a.t_carry + (row * a.tiles + tile) * 6;
  Sum3<S> cl{0, 0, 0}, cr{0, 0, 0};
  bool fl = false, fr = false;
#pragma unroll
  for (int i = 1; i < NW; ++i) {
    const int wl = warp - i, wr = warp + i;
    if (wl >= 0 && !fl) {
      cl = add3(fwd_v[wl], cl);
      fl = fwd_f[wl] != 0;
    }
    if (wr < NW && !fr) {
      cr = add3(cr, bwd_v[wr]);
      fr = bwd_f[wr] != 0;
    }
  }
  if (!fl) cl = add3(Sum3<S>{cp[0], cp[1], cp[2]}, cl);
  if (!fr) cr = add3(cr, Sum3<S>{cp[3], cp[4], cp[5]});
  const Sum3<S> in_l = exf ? ex : add3(cl, ex);
  const Sum3<S> in_r = exfb ? exb : add3(exb, cr);

  In* gy = a.grad_y ? static_cast<In*>(a.grad_y) + gbase + e0 : nullptr;
  Acc* gw = (kY && a.grad_w) ? static_cast<Acc*>(a.grad_w) + gbase + e0 : nullptr;
  lane_gradients<In, kW, kY, K>(e, st, xy, in_l, in_r, has, y0, a, gy, gw, valid);
}

}  // namespace tiso
