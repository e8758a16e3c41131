// Backward for rows of at most 64 elements: a lane per 8 elements, G = 1, 2, 4 or 8 lanes per
// row (32 / G rows per warp), everything in registers.
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

// elements [base, base + 8) of a row of n (those below n): one or two 16-byte loads when vec
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

template <typename In, bool kW, bool kY, int G>
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
  const int n = a.n;
  const int base = u * K;
  const int64_t r = live ? row : 0;
  const In* gr = static_cast<const In*>(a.g) + r * n;
  const In* yr = kY ? static_cast<const In*>(a.y) + r * n : nullptr;
  const Acc* wr = kW ? static_cast<const Acc*>(a.w) + r * n : nullptr;
  const uint8_t* sr = a.starts + r * n;
  auto vec = [&](const void* p, int bytes) {  // the lane's 8 elements as whole 16-byte units
    return (n % K) == 0 && ((K * bytes) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(p) & 15) == 0;
  };
  const bool mine = live && base < n;

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
      if ((n % K) == 0 && (reinterpret_cast<uintptr_t>(sr) & 7) == 0) {
        const uint2 v = *reinterpret_cast<const uint2*>(sr + base);
#pragma unroll
        for (int j = 0; j < K; ++j) xs[j] = static_cast<uint8_t>((j < 4 ? v.x : v.y) >> (8 * (j & 3)));
      } else {
#pragma unroll
        for (int j = 0; j < K; ++j) xs[j] = base + j < n ? sr[base + j] : 0;
      }
      load8<In>(gr, base, n, vec(gr, sizeof(In)), ag);
      if constexpr (kW) load8<Acc>(wr, base, n, vec(wr, sizeof(Acc)), aw);
      if constexpr (kY) load8<In>(yr, base, n, vec(yr, sizeof(In)), ay);
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const bool in = mine && base + j < n;
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

  // each block's masked G / W and fit at its start, from the lane's last element down
  S rmg[K], rfit[K];
  Sum3<S> acc{0, 0, 0};
  bool later = false;  // a start after this position within the lane
#pragma unroll
  for (int j = K - 1; j >= 0; --j) {
    acc = add3(acc, e[j]);
    rmg[j] = S(0);
    rfit[j] = S(0);
    if (st[j]) {
      const Sum3<S> tot = later ? acc : add3(acc, in_r);
      block_result<Acc, S, kY>(tot, y0, a, rmg[j], rfit[j]);
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

  // the gradients
  if (!mine) return;
  union {
    uint4 u[K * sizeof(In) / 16];
    In e[K];
  } py;
  union {
    uint4 u[K * sizeof(Acc) / 16];
    Acc e[K];
  } pw;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (st[j]) {
      mg = rmg[j];
      fit = rfit[j];
    }
    py.e[j] = from_acc<In>(static_cast<Acc>(xw[j] * mg));
    if constexpr (kY) pw.e[j] = static_cast<Acc>((xy[j] - fit) * mg);
  }
  if (a.grad_y) {
    In* o = static_cast<In*>(a.grad_y) + r * n + base;
    if ((n % K) == 0 && ((K * sizeof(In)) % 16) == 0 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
      for (int v = 0; v < static_cast<int>(K * sizeof(In) / 16); ++v) {
        __stcs(reinterpret_cast<uint4*>(o) + v, py.u[v]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        if (base + j < n) o[j] = py.e[j];
      }
    }
  }
  if constexpr (kY) {
    if (a.grad_w) {
      Acc* o = static_cast<Acc*>(a.grad_w) + r * n + base;
      if ((n % K) == 0 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
        for (int v = 0; v < static_cast<int>(K * sizeof(Acc) / 16); ++v) {
          __stcs(reinterpret_cast<uint4*>(o) + v, pw.u[v]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < K; ++j) {
          if (base + j < n) o[j] = pw.e[j];
        }
      }
    }
  }
}

}  // namespace tiso
